"""ctypes bindings of libpinfer.so (the B200 build).

Mirrors the reference's python/pinfer/_lib.py: the same struct mirrors (Params, SpecParams,
SpecStats, GenOpts), the same required-function table (_lib.py:88-100) and optional,
feature-detected functions (:137-170), and the same library search order with the PINFER_LIB
environment variable first (:187-205). On top, the B200 extensions and the kernel-level ABI of
include/nb_b200.h.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path
from typing import Any

_PKG_DIR = Path(__file__).resolve().parent
_LIB_NAME = "libpinfer.so"
_lock = threading.Lock()
_cache: dict[str, "Lib"] = {}

_c_int32_p = ctypes.POINTER(ctypes.c_int32)
_c_int_p = ctypes.POINTER(ctypes.c_int)
_c_float_p = ctypes.POINTER(ctypes.c_float)

PINFER_OK, PINFER_E_IO, PINFER_E_FORMAT, PINFER_E_NOMEM, PINFER_E_ARG, PINFER_E_CTX_FULL = 0, -1, -2, -3, -4, -5


class LibraryNotFoundError(OSError):
    """libpinfer.so could not be loaded."""


class Params(ctypes.Structure):
    """Mirror of ``pinfer_params``."""
    _fields_ = [("n_threads", ctypes.c_int), ("max_ctx", ctypes.c_int),
                ("kv_dtype", ctypes.c_int), ("gpu_split", ctypes.c_float)]


class SpecParams(ctypes.Structure):
    """Mirror of ``pinfer_spec_params``."""
    _fields_ = [("k", ctypes.c_int), ("draft_vocab", ctypes.c_int),
                ("adaptive", ctypes.c_int), ("ngram", ctypes.c_int)]


class SpecStats(ctypes.Structure):
    """Mirror of ``pinfer_spec_stats``."""
    _fields_ = [("rounds", ctypes.c_int64), ("drafted", ctypes.c_int64),
                ("accepted", ctypes.c_int64), ("ngram_rounds", ctypes.c_int64),
                ("ngram_drafted", ctypes.c_int64), ("ngram_accepted", ctypes.c_int64)]


ON_TOKEN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_int32, ctypes.c_void_p)


class GenOpts(ctypes.Structure):
    """Mirror of ``pinfer_gen_opts``."""
    _fields_ = [("stop_ids", _c_int32_p), ("n_stop", ctypes.c_int),
                ("on_token", ON_TOKEN), ("user", ctypes.c_void_p)]


_REQUIRED = {
    "pinfer_default_params": (Params, []),
    "pinfer_load": (ctypes.c_void_p, [ctypes.c_char_p, ctypes.POINTER(Params), _c_int_p]),
    "pinfer_free": (None, [ctypes.c_void_p]),
    "pinfer_reset": (None, [ctypes.c_void_p]),
    "pinfer_eval": (ctypes.c_int, [ctypes.c_void_p, _c_int32_p, ctypes.c_int, _c_float_p]),
    "pinfer_n_vocab": (ctypes.c_int, [ctypes.c_void_p]),
    "pinfer_n_past": (ctypes.c_int, [ctypes.c_void_p]),
    "pinfer_eos_id": (ctypes.c_int, [ctypes.c_void_p]),
    "pinfer_argmax": (ctypes.c_int, [_c_float_p, ctypes.c_int]),
    "pinfer_version": (ctypes.c_char_p, []),
}

_GEN_EX = [ctypes.c_void_p, _c_int32_p, ctypes.c_int, _c_int32_p, ctypes.c_int,
           ctypes.POINTER(SpecParams), ctypes.POINTER(GenOpts), ctypes.POINTER(SpecStats), _c_int_p]

_OPTIONAL = {
    "pinfer_has_mtp": (ctypes.c_int, [ctypes.c_void_p]),
    "pinfer_default_spec_params": (SpecParams, []),
    "pinfer_generate_greedy": (ctypes.c_int, [ctypes.c_void_p, _c_int32_p, ctypes.c_int, _c_int32_p,
                                              ctypes.c_int, ctypes.POINTER(SpecParams),
                                              ctypes.POINTER(SpecStats)]),
    "pinfer_generate_greedy_ex": (ctypes.c_int, _GEN_EX),
    "pinfer_generate_greedy_cont": (ctypes.c_int, _GEN_EX),
    "pinfer_state_size": (ctypes.c_size_t, [ctypes.c_void_p]),
    "pinfer_state_save": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]),
    "pinfer_state_load": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]),
    "pinfer_eval_select": (ctypes.c_int, [ctypes.c_void_p, _c_int32_p, ctypes.c_int, _c_int32_p,
                                          ctypes.c_int, _c_float_p]),
    "pinfer_checkpoint": (ctypes.c_int, [ctypes.c_void_p]),
    "pinfer_rewind": (ctypes.c_int, [ctypes.c_void_p]),
    "pinfer_checkpoint_clear": (None, [ctypes.c_void_p]),
    "pinfer_checkpoint_n_past": (ctypes.c_int, [ctypes.c_void_p]),
    # B200 extensions (include/nb_b200.h)
    "pinfer_b200_last_error": (ctypes.c_char_p, []),
    "pinfer_b200_generate_synthetic": (ctypes.c_int, [
        ctypes.c_void_p, _c_int32_p, ctypes.c_int, _c_int32_p, ctypes.c_int, ctypes.c_int,
        _c_int32_p, ctypes.c_uint64, ctypes.c_float, ctypes.POINTER(SpecStats), _c_int_p]),
    "pinfer_b200_generate_synthetic_ex": (ctypes.c_int, [
        ctypes.c_void_p, _c_int32_p, ctypes.c_int, _c_int32_p, ctypes.c_int, ctypes.c_int,
        _c_int32_p, ctypes.c_uint64, ctypes.c_float, ctypes.c_int, ctypes.POINTER(SpecStats), _c_int_p,
        ctypes.POINTER(ctypes.c_float)]),
    "pinfer_b200_round_kernels": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "pinfer_b200_forward_all": (ctypes.c_int, [ctypes.c_void_p, _c_int32_p, ctypes.c_int, _c_float_p]),
    "pinfer_b200_stream": (ctypes.c_void_p, [ctypes.c_void_p]),
    "pinfer_b200_clone": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_int, _c_int_p]),
    "pinfer_b200_batch_create": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                   _c_int_p]),
    "pinfer_b200_batch_free": (None, [ctypes.c_void_p]),
    "pinfer_b200_batch_stream": (ctypes.c_void_p, [ctypes.c_void_p]),
    "pinfer_b200_batch_rounds": (ctypes.c_int, [ctypes.c_void_p]),
    "pinfer_b200_batch_generate_synthetic": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int, _c_int32_p, _c_int32_p, ctypes.c_int, ctypes.c_int, _c_int32_p,
        ctypes.POINTER(ctypes.c_uint64), ctypes.c_float, _c_int32_p, _c_int32_p, _c_int32_p,
        ctypes.POINTER(SpecStats), _c_float_p]),
    "pinfer_b200_nccl_id": (ctypes.c_int, [ctypes.c_void_p]),
    "pinfer_b200_shard_head": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "nb_q4k_panel_bytes": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    "nb_q4k_repack": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "nb_mv_create": (ctypes.c_void_p, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "nb_mv_destroy": (None, [ctypes.c_void_p]),
    "nb_mv_set_n": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "nb_mv_quant": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "nb_mv_matmul": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "nb_mv_matmul_repeat": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                           ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "nb_mv_head_repeat": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                         ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_void_p]),
    "nb_mv_run": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                 ctypes.c_void_p]),
    "nb_mv_get_act": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                     ctypes.c_void_p, ctypes.c_void_p]),
    "nb_mv_prepare": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "nb_mv_gemm": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_void_p]),
    "nb_mv_status": (ctypes.c_int, [ctypes.c_void_p]),
    "nb_mv_run_static": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "nb_argmax_key": (ctypes.c_ulonglong, [ctypes.c_float, ctypes.c_int]),
    "nb_test_bounded_wait": (ctypes.c_int, [ctypes.c_uint, ctypes.POINTER(ctypes.c_int)]),
    "nb_libm_selftest": (ctypes.c_int, [ctypes.c_int, ctypes.c_longlong, ctypes.POINTER(ctypes.c_longlong)]),
    "nb_libm_eval_host": (ctypes.c_int, [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong]),
    "nb_libm_eval_device": (ctypes.c_int, [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong,
                                           ctypes.c_void_p]),
}


class Lib:
    """A loaded ``libpinfer.so`` with typed entry points."""

    def __init__(self, path: str, cdll: ctypes.CDLL) -> None:
        self.path = path
        self.cdll = cdll
        for name, (restype, argtypes) in _REQUIRED.items():
            try:
                fn = getattr(cdll, name)
            except AttributeError as e:
                raise LibraryNotFoundError(f"{path}: missing symbol {name}; "
                                           "library too old or not pinfer") from e
            fn.restype = restype
            fn.argtypes = argtypes
            setattr(self, name, fn)
        self.version: str = self.pinfer_version().decode()
        for name, (restype, argtypes) in _OPTIONAL.items():
            setattr(self, name, self.optional(name, restype, argtypes))

    def has(self, name: str) -> bool:
        return hasattr(self.cdll, name)

    def optional(self, name: str, restype: Any, argtypes: list[Any]) -> Any | None:
        if not self.has(name):
            return None
        fn = getattr(self.cdll, name)
        fn.restype = restype
        fn.argtypes = argtypes
        return fn

    def last_error(self) -> str:
        return self.pinfer_b200_last_error().decode() if self.pinfer_b200_last_error else ""


def candidate_paths(path: str | os.PathLike[str] | None = None) -> list[str]:
    out: list[str] = []
    if path:
        out.append(os.fspath(path))
    env = os.environ.get("PINFER_LIB")
    if env:
        out.append(env)
    out.append(str(_PKG_DIR / "lib" / _LIB_NAME))
    return out


def load_library(path: str | os.PathLike[str] | None = None) -> Lib:
    """Load libpinfer.so (cached per resolved path). Raises LibraryNotFoundError."""
    candidates = [os.fspath(path)] if path else candidate_paths()
    errors: list[str] = []
    with _lock:
        for cand in candidates:
            if not os.path.exists(cand):
                errors.append(f"{cand}: not found")
                continue
            key = os.path.realpath(cand)
            if key in _cache:
                return _cache[key]
            try:
                cdll = ctypes.CDLL(cand)
            except OSError as e:
                errors.append(f"{cand}: {e}")
                continue
            lib = Lib(cand, cdll)
            _cache[key] = lib
            return lib
    raise LibraryNotFoundError("cannot load libpinfer.so (run python -m nibblemac_b200.build); "
                               "tried:\n  " + "\n  ".join(errors))
