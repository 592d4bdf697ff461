"""Python access to the CPU oracle: TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm, never
by the product. Two libraries:
  liboracle.so           the Q4K x A8 restatement (q4k_a8.c), pinned by the reference's
                         recorded kbench hashes;
  _ref/libpinfer_ref.so  the reference engine compiled from its own sources (scalar build) with
                         ref_shim.c (Q4K) and ref_spec.c (synthetic-drafter speculation).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_P = ctypes.c_void_p


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_P)


class Q4KOracle:
    """The restated Q4K x A8 arithmetic (liboracle.so)."""

    def __init__(self, path: Path | None = None) -> None:
        self.lib = ctypes.CDLL(str(path or HERE / "liboracle.so"))
        L = self.lib
        L.or_fnv1a.restype = ctypes.c_uint64
        L.or_fnv1a.argtypes = [_P, ctypes.c_size_t]
        L.or_kb_fill_vec.argtypes = [_P, ctypes.c_size_t, ctypes.c_uint64]
        L.or_kb_fill_q4k.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_uint64, _P]
        L.or_q4k_matmul.argtypes = [_P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, _P]
        L.or_quant_act.argtypes = [_P, ctypes.c_int, ctypes.c_int, _P, _P, _P]
        L.or_q4k_isums.argtypes = [_P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, _P]
        L.or_q4k_get_row.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P]

    def kb_matrix(self, rows: int, cols: int, seed: int = 42) -> np.ndarray:
        w = np.zeros(rows // 4 * (cols // 256) * 576, np.uint8)
        self.lib.or_kb_fill_q4k(rows, cols, seed, _ptr(w))
        return w

    def kb_vec(self, n: int, seed: int = 7) -> np.ndarray:
        x = np.zeros(n, np.float32)
        self.lib.or_kb_fill_vec(_ptr(x), x.size, seed)
        return x

    def matmul(self, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
        y = np.zeros((x.shape[0], rows), np.float32)
        self.lib.or_q4k_matmul(_ptr(w), rows, cols, _ptr(x), x.shape[0], _ptr(y))
        return y

    def quant_act(self, x: np.ndarray, cols: int):
        """Returns (q [n][cols] int8, d [n][cols/32], fsum [n][cols/32]) in vector-major order."""
        x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
        n, nb = x.shape[0], cols // 32
        q = np.zeros(n * cols, np.int8)
        d = np.zeros(n * nb, np.float32)
        fs = np.zeros(n * nb, np.float32)
        self.lib.or_quant_act(_ptr(x), n, cols, _ptr(q), _ptr(d), _ptr(fs))
        # oracle output is block-major [nb][n][32]; return vector-major
        q = q.reshape(nb, n, 32).transpose(1, 0, 2).reshape(n, cols)
        return q, d.reshape(nb, n).T.copy(), fs.reshape(nb, n).T.copy()

    def get_row(self, w: np.ndarray, rows: int, cols: int, row: int) -> np.ndarray:
        out = np.zeros(cols, np.float32)
        self.lib.or_q4k_get_row(_ptr(w), rows, cols, row, _ptr(out))
        return out

    def fnv1a(self, a: np.ndarray) -> int:
        return int(self.lib.or_fnv1a(_ptr(a), a.nbytes))


class _Params(ctypes.Structure):
    _fields_ = [("n_threads", ctypes.c_int), ("max_ctx", ctypes.c_int),
                ("kv_dtype", ctypes.c_int), ("gpu_split", ctypes.c_float)]


class _SpecParams(ctypes.Structure):
    _fields_ = [("k", ctypes.c_int), ("draft_vocab", ctypes.c_int), ("adaptive", ctypes.c_int),
                ("ngram", ctypes.c_int)]


class _SpecStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in ("rounds", "drafted", "accepted", "ngram_rounds",
                                              "ngram_drafted", "ngram_accepted")]


class RefEngine:
    """The reference engine (scalar build + Q4K restatement) on one model file."""

    def __init__(self, model_path, max_ctx: int = 4096, lib_path: Path | None = None,
                 kv_dtype: int = 0) -> None:
        path = lib_path or HERE / "_ref" / "libpinfer_ref.so"
        if not Path(path).exists():
            raise FileNotFoundError(f"{path} missing: build it with `make -C oracle ref`")
        self.lib = L = ctypes.CDLL(str(path))
        L.pinfer_default_params.restype = _Params
        L.pinfer_load.restype = ctypes.c_void_p
        L.pinfer_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(_Params), ctypes.POINTER(ctypes.c_int)]
        L.pinfer_free.argtypes = [_P]
        L.pinfer_reset.argtypes = [_P]
        L.pinfer_eval.argtypes = [_P, _P, ctypes.c_int, _P]
        L.pinfer_generate_greedy.argtypes = [_P, _P, ctypes.c_int, _P, ctypes.c_int, _P, _P]
        L.pinfer_n_vocab.argtypes = [_P]
        L.ref_spec_generate.argtypes = [_P, _P, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int, _P,
                                        ctypes.c_uint64, ctypes.c_uint32, _P]
        L.ref_spec_generate_cont.argtypes = L.ref_spec_generate.argtypes
        L.ref_forward_all.argtypes = [_P, _P, ctypes.c_int, _P]
        L.pinfer_generate_greedy_ex.argtypes = [_P, _P, ctypes.c_int, _P, ctypes.c_int, _P, _P, _P, _P]
        L.pinfer_generate_greedy_cont.argtypes = [_P, _P, ctypes.c_int, _P, ctypes.c_int, _P, _P, _P, _P]
        L.pinfer_state_size.restype = ctypes.c_size_t
        L.pinfer_state_size.argtypes = [_P]
        L.pinfer_state_save.argtypes = [_P, _P, ctypes.c_size_t]
        L.pinfer_state_load.argtypes = [_P, _P, ctypes.c_size_t]
        L.pinfer_checkpoint.argtypes = [_P]
        L.pinfer_rewind.argtypes = [_P]
        L.pinfer_n_past.argtypes = [_P]
        L.nb_synth_draft.restype = ctypes.c_int32
        L.nb_synth_draft.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_uint32, ctypes.c_int32,
                                     ctypes.c_int32]
        p = L.pinfer_default_params()
        p.max_ctx = max_ctx
        p.n_threads = 1
        p.kv_dtype = kv_dtype
        err = ctypes.c_int(0)
        self.ctx = L.pinfer_load(str(model_path).encode(), ctypes.byref(p), ctypes.byref(err))
        if not self.ctx:
            raise RuntimeError(f"reference pinfer_load failed: {err.value}")
        self.n_vocab = L.pinfer_n_vocab(self.ctx)

    def close(self) -> None:
        if self.ctx:
            self.lib.pinfer_free(self.ctx)
            self.ctx = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def reset(self) -> None:
        self.lib.pinfer_reset(self.ctx)

    def eval(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(self.n_vocab, np.float32)
        rc = self.lib.pinfer_eval(self.ctx, _ptr(t), len(t), _ptr(out))
        if rc:
            raise RuntimeError(f"reference pinfer_eval: {rc}")
        return out

    def save_state(self) -> bytes:
        n = self.lib.pinfer_state_size(self.ctx)
        buf = ctypes.create_string_buffer(n)
        rc = self.lib.pinfer_state_save(self.ctx, buf, n)
        if rc:
            raise RuntimeError(f"reference pinfer_state_save: {rc}")
        return buf.raw

    def load_state(self, data: bytes) -> int:
        return self.lib.pinfer_state_load(self.ctx, data, len(data))

    def checkpoint(self) -> None:
        rc = self.lib.pinfer_checkpoint(self.ctx)
        if rc:
            raise RuntimeError(f"reference pinfer_checkpoint: {rc}")

    def rewind(self) -> None:
        rc = self.lib.pinfer_rewind(self.ctx)
        if rc:
            raise RuntimeError(f"reference pinfer_rewind: {rc}")

    @property
    def n_past(self) -> int:
        return self.lib.pinfer_n_past(self.ctx)

    def forward_all(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros((len(t), self.n_vocab), np.float32)
        rc = self.lib.ref_forward_all(self.ctx, _ptr(t), len(t), _ptr(out))
        if rc:
            raise RuntimeError(f"reference forward: {rc}")
        return out

    def generate(self, prompt, n_max: int) -> list[int]:
        t = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_max, np.int32)
        n = self.lib.pinfer_generate_greedy(self.ctx, _ptr(t), len(t), _ptr(out), n_max, None, None)
        if n < 0:
            raise RuntimeError(f"reference generate: {n}")
        return out[:n].tolist()

    def generate_mtp(self, prompt, n_max: int, k: int, draft_vocab: int = 0, append: bool = False,
                     ngram: int = 0, all_stats: bool = False):
        """The reference's own speculative decoding (pinfer_generate_greedy_ex / _cont): MTP
        drafts at a fixed k, prompt-lookup drafts of up to `ngram` tokens, no adaptive policy:
        (tokens, [rounds, drafted, accepted] (+ the three n-gram counts with all_stats),
        status)."""
        t = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_max, np.int32)
        sp = _SpecParams(k, draft_vocab, 0, ngram)
        st = _SpecStats()
        status = ctypes.c_int(0)
        fn = self.lib.pinfer_generate_greedy_cont if append else self.lib.pinfer_generate_greedy_ex
        n = fn(self.ctx, _ptr(t), len(t), _ptr(out), n_max, ctypes.byref(sp), None, ctypes.byref(st),
               ctypes.byref(status))
        if n < 0:
            raise RuntimeError(f"reference generate: {n}")
        stats = [st.rounds, st.drafted, st.accepted]
        if all_stats:
            stats += [st.ngram_rounds, st.ngram_drafted, st.ngram_accepted]
        return out[:n].tolist(), stats, status.value

    def spec_generate(self, prompt, n_max: int, k: int, greedy, seed: int, p: float,
                      append: bool = False):
        """Synthetic-drafter speculation on the reference's verify/accept/commit steps;
        append keeps the context and feeds the prompt on top of it."""
        t = np.ascontiguousarray(prompt, np.int32)
        g = np.ascontiguousarray(greedy, np.int32)
        out = np.zeros(n_max, np.int32)
        st = np.zeros(4, np.int64)
        p24 = min(1 << 24, int(np.floor(p * (1 << 24) + 0.5)))
        fn = self.lib.ref_spec_generate_cont if append else self.lib.ref_spec_generate
        n = fn(self.ctx, _ptr(t), len(t), _ptr(out), n_max, k, _ptr(g), seed, p24, _ptr(st))
        if n < 0:
            raise RuntimeError(f"reference spec generate: {n}")
        self.last_decode_s = st[3] * 1e-9
        return out[:n].tolist(), st[:3].tolist()
