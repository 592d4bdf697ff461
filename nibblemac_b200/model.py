"""Python view of a loaded model (the calls of the reference's pinfer.Model that touch the
verify path, python/pinfer/model.py:33-120), over the ctypes table in _lib.py."""
from __future__ import annotations

import ctypes
import os

import numpy as np

from ._lib import (GenOpts, Lib, PINFER_OK, SpecParams, SpecStats, load_library,
                   _c_float_p, _c_int32_p)


class PinferError(RuntimeError):
    def __init__(self, code: int, what: str, detail: str = "") -> None:
        super().__init__(f"{what} failed with {code}" + (f": {detail}" if detail else ""))
        self.code = code


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


class Model:
    """A context on the B200: ``Model(path).generate(prompt, 128)``."""

    def __init__(self, path: str | os.PathLike, max_ctx: int = 4096, lib: Lib | None = None,
                 kv_dtype: int = 0) -> None:
        self.lib = lib or load_library()
        p = self.lib.pinfer_default_params()
        p.max_ctx = max_ctx
        p.kv_dtype = kv_dtype   # PINFER_KV_F32 / F16 / I8
        err = ctypes.c_int(0)
        self.ctx = self.lib.pinfer_load(os.fspath(path).encode(), ctypes.byref(p), ctypes.byref(err))
        if not self.ctx:
            raise PinferError(err.value, "pinfer_load", self.lib.last_error())
        self.n_vocab = self.lib.pinfer_n_vocab(self.ctx)
        self.eos_id = self.lib.pinfer_eos_id(self.ctx)

    def clone(self, max_ctx: int = 0) -> "Model":
        """Another context on the same weights (pinfer_b200_clone): own states, KV cache,
        stream and graphs, for running independent request streams concurrently."""
        err = ctypes.c_int(0)
        ctx = self.lib.pinfer_b200_clone(self.ctx, max_ctx, ctypes.byref(err))
        if not ctx:
            raise PinferError(err.value, "pinfer_b200_clone", self.lib.last_error())
        m = Model.__new__(Model)
        m.lib, m.ctx, m.n_vocab, m.eos_id = self.lib, ctx, self.n_vocab, self.eos_id
        return m

    def close(self) -> None:
        if self.ctx:
            self.lib.pinfer_free(self.ctx)
            self.ctx = None

    def __enter__(self) -> "Model":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    @property
    def n_past(self) -> int:
        return self.lib.pinfer_n_past(self.ctx)

    def reset(self) -> None:
        self.lib.pinfer_reset(self.ctx)

    def eval(self, tokens, logits: bool = True) -> np.ndarray | None:
        t = _i32(tokens)
        out = np.empty(self.n_vocab, np.float32) if logits else None
        rc = self.lib.pinfer_eval(self.ctx, t.ctypes.data_as(_c_int32_p), len(t),
                                  out.ctypes.data_as(_c_float_p) if logits else None)
        if rc != PINFER_OK:
            raise PinferError(rc, "pinfer_eval", self.lib.last_error())
        return out

    def forward_all(self, tokens) -> np.ndarray:
        t = _i32(tokens)
        out = np.empty((len(t), self.n_vocab), np.float32)
        rc = self.lib.pinfer_b200_forward_all(self.ctx, t.ctypes.data_as(_c_int32_p), len(t),
                                              out.ctypes.data_as(_c_float_p))
        if rc != PINFER_OK:
            raise PinferError(rc, "pinfer_b200_forward_all", self.lib.last_error())
        return out

    def generate(self, prompt, n_max: int, k: int = 0, stop_ids=None, on_token=None,
                 draft_vocab: int = 0, stats: SpecStats | None = None, append: bool = False,
                 ngram: int = 0) -> tuple[list[int], int]:
        """pinfer_generate_greedy_ex (append: _cont): (tokens, status). k > 0 drafts with the
        MTP head over the first draft_vocab ids (0: all), ngram > 0 with prompt lookup;
        statistics accumulate into stats."""
        t = _i32(prompt)
        out = np.zeros(n_max, np.int32)
        sp = SpecParams(k, draft_vocab, 0, ngram)
        st = stats if stats is not None else SpecStats()
        status = ctypes.c_int(0)
        opts = None
        keep = []
        if stop_ids is not None or on_token is not None:
            ids = _i32(stop_ids or [])
            keep.append(ids)
            cb = ctypes.cast(None, type(GenOpts().on_token)) if on_token is None else \
                type(GenOpts().on_token)(lambda tok, user: int(bool(on_token(int(tok)))))
            keep.append(cb)
            opts = GenOpts(ids.ctypes.data_as(_c_int32_p) if len(ids) else None, len(ids), cb, None)
        fn = self.lib.pinfer_generate_greedy_cont if append else self.lib.pinfer_generate_greedy_ex
        n = fn(self.ctx, t.ctypes.data_as(_c_int32_p), len(t), out.ctypes.data_as(_c_int32_p), n_max,
               ctypes.byref(sp), ctypes.byref(opts) if opts else None, ctypes.byref(st), ctypes.byref(status))
        if n < 0:
            raise PinferError(n, "pinfer_generate_greedy_ex", self.lib.last_error())
        return out[:n].tolist(), status.value

    def generate_synthetic(self, prompt, n_max: int, k: int, greedy, seed: int, p: float
                           ) -> tuple[list[int], SpecStats, int]:
        """Speculative decoding with the synthetic drafter (pinfer_b200_generate_synthetic)."""
        t = _i32(prompt)
        g = _i32(greedy)
        if len(g) < n_max:
            raise ValueError("greedy stream shorter than n_max")
        out = np.zeros(n_max, np.int32)
        st = SpecStats()
        status = ctypes.c_int(0)
        n = self.lib.pinfer_b200_generate_synthetic(
            self.ctx, t.ctypes.data_as(_c_int32_p), len(t), out.ctypes.data_as(_c_int32_p), n_max,
            k, g.ctypes.data_as(_c_int32_p), seed, p, ctypes.byref(st), ctypes.byref(status))
        if n < 0:
            raise PinferError(n, "pinfer_b200_generate_synthetic", self.lib.last_error())
        return out[:n].tolist(), st, status.value

    def generate_synthetic_ex(self, prompt, n_max: int, k: int, greedy, seed: int, p: float,
                              append: bool = False):
        """(tokens, stats, status, decode_ms) with the device-timed decode loop."""
        t = _i32(prompt)
        g = _i32(greedy)
        if len(g) < n_max:
            raise ValueError("greedy stream shorter than n_max")
        out = np.zeros(n_max, np.int32)
        st = SpecStats()
        status = ctypes.c_int(0)
        ms = ctypes.c_float(0.0)
        n = self.lib.pinfer_b200_generate_synthetic_ex(
            self.ctx, t.ctypes.data_as(_c_int32_p), len(t), out.ctypes.data_as(_c_int32_p), n_max,
            k, g.ctypes.data_as(_c_int32_p), seed, p, int(append), ctypes.byref(st),
            ctypes.byref(status), ctypes.byref(ms))
        if n < 0:
            raise PinferError(n, "pinfer_b200_generate_synthetic_ex", self.lib.last_error())
        return out[:n].tolist(), st, status.value, ms.value

    def save_state(self) -> bytes:
        """The conversation state blob (pinfer_state_save; the reference's format)."""
        n = self.lib.pinfer_state_size(self.ctx)
        buf = ctypes.create_string_buffer(n)
        rc = self.lib.pinfer_state_save(self.ctx, buf, n)
        if rc != PINFER_OK:
            raise PinferError(rc, "pinfer_state_save", self.lib.last_error())
        return buf.raw

    def load_state(self, data: bytes) -> None:
        rc = self.lib.pinfer_state_load(self.ctx, data, len(data))
        if rc != PINFER_OK:
            raise PinferError(rc, "pinfer_state_load", self.lib.last_error())

    def checkpoint(self) -> None:
        rc = self.lib.pinfer_checkpoint(self.ctx)
        if rc != PINFER_OK:
            raise PinferError(rc, "pinfer_checkpoint", self.lib.last_error())

    def rewind(self) -> None:
        rc = self.lib.pinfer_rewind(self.ctx)
        if rc != PINFER_OK:
            raise PinferError(rc, "pinfer_rewind", self.lib.last_error())

    def nccl_id(self) -> bytes:
        """A fresh NCCL unique id (128 bytes) for shard_head, to be sent to every rank."""
        buf = ctypes.create_string_buffer(128)
        rc = self.lib.pinfer_b200_nccl_id(buf)
        if rc != PINFER_OK:
            raise PinferError(rc, "pinfer_b200_nccl_id", self.lib.last_error())
        return buf.raw

    def shard_head(self, rank: int, world: int, nccl_id: bytes | None) -> None:
        """Vocab-shard the LM head over `world` GPUs (collective: every rank calls it)."""
        rc = self.lib.pinfer_b200_shard_head(self.ctx, rank, world, nccl_id)
        if rc != PINFER_OK:
            raise PinferError(rc, "pinfer_b200_shard_head", self.lib.last_error())

    def batch(self, slots: int, max_ctx: int, max_k: int = 3) -> "Batch":
        """A multi-sequence batch on this context's weights (pinfer_b200_batch_create)."""
        return Batch(self, slots, max_ctx, max_k)

    def round_kernels(self, k: int) -> int:
        return self.lib.pinfer_b200_round_kernels(self.ctx, k)

    def stream(self) -> int:
        return self.lib.pinfer_b200_stream(self.ctx) or 0


class Batch:
    """Independent sequences generated together in merged passes (pinfer_b200_batch_*): each
    sequence's tokens equal what Model.generate_synthetic gives for it alone."""

    def __init__(self, model: Model, slots: int, max_ctx: int, max_k: int = 3) -> None:
        self.lib, self.model = model.lib, model
        err = ctypes.c_int(0)
        self.h = self.lib.pinfer_b200_batch_create(model.ctx, slots, max_ctx, max_k, ctypes.byref(err))
        if not self.h:
            raise PinferError(err.value, "pinfer_b200_batch_create", self.lib.last_error())
        self.slots = slots

    def close(self) -> None:
        if self.h:
            self.lib.pinfer_b200_batch_free(self.h)
            self.h = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def stream(self) -> int:
        return self.lib.pinfer_b200_batch_stream(self.h) or 0

    def rounds(self) -> int:
        """Verify rounds the last generation ran (passes over all sequences)."""
        return self.lib.pinfer_b200_batch_rounds(self.h)

    def generate_synthetic(self, prompts, n_max: int, k: int = 0, greedy=None, seeds=None, p: float = 0.0):
        """(list of token lists, SpecStats, statuses, decode_ms) for the prompts (a list of
        token arrays); k > 0 drafts with the synthetic drafter from greedy[i] (n_max tokens
        each) and seeds[i]."""
        n = len(prompts)
        lens = _i32([len(x) for x in prompts])
        flat = _i32(np.concatenate([np.asarray(x, np.int32) for x in prompts]))
        out = np.zeros((n, n_max), np.int32)
        counts = np.zeros(n, np.int32)
        status = np.zeros(n, np.int32)
        st = SpecStats()
        ms = ctypes.c_float(0.0)
        g = sd = None
        if k > 0:
            g = np.zeros((n, n_max), np.int32)
            for i, row in enumerate(greedy):
                r = np.asarray(row, np.int32)[:n_max]
                g[i, :len(r)] = r
            sd = np.ascontiguousarray(np.asarray(seeds, np.uint64))
        rc = self.lib.pinfer_b200_batch_generate_synthetic(
            self.h, n, flat.ctypes.data_as(_c_int32_p), lens.ctypes.data_as(_c_int32_p), n_max, k,
            g.ctypes.data_as(_c_int32_p) if g is not None else None,
            sd.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)) if sd is not None else None, p,
            out.ctypes.data_as(_c_int32_p), counts.ctypes.data_as(_c_int32_p),
            status.ctypes.data_as(_c_int32_p), ctypes.byref(st), ctypes.byref(ms))
        if rc != PINFER_OK:
            raise PinferError(rc, "pinfer_b200_batch_generate_synthetic", self.lib.last_error())
        return [out[i, :counts[i]].tolist() for i in range(n)], st, status.tolist(), ms.value
