""".pq model files: the on-disk format, a writer, and the synthetic Qwen3.5 models used by the
tests and the benchmark.

The format is the reference engine's `.pq` v1 (engine/FORMAT.md; structs in
engine/src/pq_format.h:32-58): a 4096-byte header, a directory of 128-byte entries, then
64-byte-aligned tensor data from a 4096-aligned offset. The writer follows the reference
converter tools/convert.py (main, :126-179): tensors in sorted Hugging Face name order, norms
stored as their effective multiplier, conv weights as [C, K] F32, every 2-D matrix quantised
to Q4K_G32 (:82-102). Q4K packing is the C restatement of tools/quant.py in csrc/pq_quant.c.

Synthetic models (random init, no checkpoint is available offline): every 2-D matrix and
conv1d / A_log / dt_bias ~ N(0, std^2) (std 0.02), all norm multipliers 1.0. Each tensor draws
from its own generator seeded by (seed, crc32(name)), so the bytes do not depend on the order in
which tensors are built.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import struct
import zlib
from dataclasses import dataclass, asdict
from pathlib import Path

import numpy as np

MAGIC = b"PINFERQ\0"
VERSION = 1
HEADER_BYTES = 4096
ALIGN = 64
F32, BF16, Q4K = 0, 1, 4
HEADER_FMT = "<8sIIQQ" + "I" * 18 + "ff"   # pq_header, engine/src/pq_format.h:32-52
ENTRY_FMT = "<80sII4IQQ8x"                 # pq_tensor_entry (128 bytes), pq_format.h:54-62
TEXT_PREFIX = "model.language_model."

_LIB_DIR = Path(__file__).resolve().parent / "lib"


@dataclass(frozen=True)
class Dims:
    """Model dimensions as the .pq header stores them (engine/FORMAT.md "Header")."""
    hidden: int
    ffn: int
    n_layers: int
    vocab: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    rot_dim: int
    lin_k_heads: int
    lin_v_heads: int
    lin_k_dim: int
    lin_v_dim: int
    conv_k: int = 4
    full_every: int = 4           # layer i is full attention when i % full_every == full_every-1
    eos_id: int = 248044
    rms_eps: float = 1e-6
    rope_theta: float = 1e7
    has_mtp: bool = True

    @property
    def full_mask(self) -> int:
        return sum(1 << i for i in range(self.n_layers) if i % self.full_every == self.full_every - 1)


# Qwen3.5-0.8B shape (engine/FORMAT.md header table) and the 2B shape of the benchmark config
# (16 query heads, hidden 2048, ffn 6144).
QWEN35_08B = Dims(hidden=1024, ffn=3584, n_layers=24, vocab=248320, n_heads=8, n_kv_heads=2,
                  head_dim=256, rot_dim=64, lin_k_heads=16, lin_v_heads=16, lin_k_dim=128,
                  lin_v_dim=128)
QWEN35_2B = Dims(hidden=2048, ffn=6144, n_layers=24, vocab=248320, n_heads=16, n_kv_heads=2,
                 head_dim=256, rot_dim=64, lin_k_heads=16, lin_v_heads=16, lin_k_dim=128,
                 lin_v_dim=128)
# Small shapes for parity tests (all matrices obey the Q4K shape rule: rows % 4, cols % 256).
TINY = Dims(hidden=256, ffn=512, n_layers=4, vocab=2048, n_heads=1, n_kv_heads=1, head_dim=256,
            rot_dim=64, lin_k_heads=1, lin_v_heads=4, lin_k_dim=128, lin_v_dim=128, eos_id=2047)
SMALL = Dims(hidden=512, ffn=1024, n_layers=8, vocab=8192, n_heads=4, n_kv_heads=2,
             head_dim=256, rot_dim=64, lin_k_heads=4, lin_v_heads=4, lin_k_dim=128,
             lin_v_dim=128, eos_id=8191)
# The two configured shapes at reduced depth (one 3:1 group: 3 DeltaNet layers, then full
# attention) with every width and the full vocabulary kept: what the reference engine, run on
# the host, can check bit for bit within a test's time.
QWEN35_08B_4L = Dims(**{**asdict(QWEN35_08B), "n_layers": 4})
QWEN35_2B_4L = Dims(**{**asdict(QWEN35_2B), "n_layers": 4})
PRESETS = {"0.8b": QWEN35_08B, "2b": QWEN35_2B, "tiny": TINY, "small": SMALL,
           "0.8b-4l": QWEN35_08B_4L, "2b-4l": QWEN35_2B_4L}


def _quant_lib() -> ctypes.CDLL:
    path = _LIB_DIR / "libnbpq.so"
    if not path.exists():
        raise RuntimeError(f"{path} is missing: run `python -m nibblemac_b200.build` first")
    lib = ctypes.CDLL(str(path))
    lib.nb_q4k_quantize_pack.restype = ctypes.c_int
    lib.nb_q4k_quantize_pack.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_void_p, ctypes.c_int]
    return lib


def q4k_nbytes(rows: int, cols: int) -> int:
    return rows // 4 * (cols // 256) * 576


def quantize_q4k(w: np.ndarray, threads: int | None = None) -> bytes:
    """Quantise + pack one float32 matrix to Q4K_G32 (same bytes as tools/quant.py
    quantize_pack(4, w)[0])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    if rows % 4 or cols % 256:
        raise ValueError(f"Q4K needs rows % 4 == 0 and cols % 256 == 0, got {rows}x{cols}")
    out = np.empty(q4k_nbytes(rows, cols), np.uint8)
    nt = threads or max(1, os.cpu_count() or 1)
    rc = _quant_lib().nb_q4k_quantize_pack(w.ctypes.data, rows, cols, out.ctypes.data, nt)
    if rc != 0:
        raise ValueError("quantisation failed")
    return out.tobytes()


_F = np.float32


def _clip(v: np.ndarray, hi: float) -> np.ndarray:
    """np.clip(v, 0, hi) in float32 (NaN passes through)."""
    return np.clip(v, _F(0.0), _F(hi))


def _posmax(v: np.ndarray) -> np.ndarray:
    """max(v, 0) with NaN passed through, float32."""
    return np.maximum(v, _F(0.0))


def _fit(x: np.ndarray, q: np.ndarray, d: np.ndarray, m: np.ndarray, sign: float):
    """One least-squares refit of (scale, offset) over groups of 32 (last axis) from codes q:
    n = 32; den = n sqq - sq^2; d' = (n sqx - sq sx) / den; m' = sign (sx - d' sq) / n where
    den > 0, else the old (d, m). Group sums are numpy float32 sums over a contiguous axis of 32,
    the summation order of the reference quantiser."""
    n = _F(32.0)
    sq, sx = q.sum(-1), x.sum(-1)
    sqq, sqx = (q * q).sum(-1), (q * x).sum(-1)
    den = n * sqq - sq * sq
    ok = den > _F(0.0)
    with np.errstate(divide="ignore", invalid="ignore"):
        dn = np.where(ok, (n * sqx - sq * sx) / np.where(ok, den, _F(1.0)), d)
        mn = np.where(ok, (sx - dn * sq) / n, m)
    return dn.astype(_F), (mn if sign > 0 else np.where(ok, -mn, m)).astype(_F)


def _q4k_rows_numpy(w: np.ndarray) -> bytes:
    """Q4K_G32 of whole 4-row tiles, vectorised over every group: the same float32 steps as the
    C quantiser (csrc/pq_quant.c, which restates tools/quant.py quant_asym4 :78-105, quant_q4k
    :108-141, _pack6 :210-217 and pack_q4k :220-244)."""
    rows, cols = w.shape
    nsb = cols // 256
    x = w.reshape(rows, nsb, 8, 32)
    f16 = lambda v: v.astype(np.float16).astype(_F)
    # asym4 per group of 32: 4 refits of (d, m) with codes against the fp16-rounded fit
    lo, hi = x.min(-1), x.max(-1)
    d, m = ((hi - lo) / _F(15.0)).astype(_F), lo
    with np.errstate(divide="ignore", invalid="ignore"):
        for it in range(5):
            d16, m16 = f16(d), f16(m)
            safe = np.where(d16 == _F(0.0), _F(1.0), d16)
            q = _clip(np.rint((x - m16[..., None]) / safe[..., None]), 15.0)
            if it == 4:
                break
            d, m = _fit(x, q, d, m, 1.0)
        dg, mn = d16, _posmax(-m16)
        # superblock scales: 6-bit multiples of fp16 D = max d / 63 and M = max m / 63
        D, M = f16(dg.max(-1) / _F(63.0)), f16(mn.max(-1) / _F(63.0))
        Ds = np.where(D == _F(0.0), _F(1.0), D)[..., None]
        Ms = np.where(M == _F(0.0), _F(1.0), M)[..., None]
        sq, mq = _clip(np.rint(dg / Ds), 63.0), _clip(np.rint(mn / Ms), 63.0)
        for it in range(3):
            d_eff, m_eff = D[..., None] * sq, M[..., None] * mq
            safe = np.where(d_eff == _F(0.0), _F(1.0), d_eff)
            q = _clip(np.rint((x + m_eff[..., None]) / safe[..., None]), 15.0)
            if it == 2:
                break
            dn, mm = _fit(x, q, d_eff, m_eff, -1.0)
            sq, mq = _clip(np.rint(dn / Ds), 63.0), _clip(np.rint(_posmax(mm) / Ms), 63.0)
    # pack: per (tile, superblock) D[4] | M[4] fp16, 6-bit s and m of [group][row], then codes
    t = rows // 4
    out = np.empty((t, nsb, 576), np.uint8)
    Dt = D.astype(np.float16).view(np.uint16).reshape(t, 4, nsb).transpose(0, 2, 1)
    Mt = M.astype(np.float16).view(np.uint16).reshape(t, 4, nsb).transpose(0, 2, 1)
    out[:, :, 0:8] = np.ascontiguousarray(Dt).view(np.uint8).reshape(t, nsb, 8)
    out[:, :, 8:16] = np.ascontiguousarray(Mt).view(np.uint8).reshape(t, nsb, 8)
    for off, v in ((16, sq), (40, mq)):
        s6 = v.astype(np.uint8).reshape(t, 4, nsb, 8).transpose(0, 2, 3, 1).reshape(t, nsb, 32)
        out[:, :, off:off + 16] = (s6[..., :16] & 15) | ((s6[..., 16:] & 15) << 4)
        out[:, :, off + 16:off + 24] = ((s6[..., 0:8] >> 4) | ((s6[..., 8:16] >> 4) << 2) |
                                        ((s6[..., 16:24] >> 4) << 4) | ((s6[..., 24:32] >> 4) << 6))
    c = q.astype(np.uint8).reshape(t, 4, nsb, 8, 32).transpose(0, 2, 3, 1, 4)   # [t][sb][g][row][32]
    out[:, :, 64:] = (c[..., :16] | (c[..., 16:] << 4)).reshape(t, nsb, 512)
    return out.tobytes()


def quantize_q4k_numpy(w: np.ndarray, chunk_rows: int = 2048) -> bytes:
    """quantize_q4k without native code: numpy float32 arithmetic only, the same bytes (tested
    against the C quantiser and the reference's fixtures). Used where a process must not load
    this package's libraries (the benchmark's reference arm)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    if rows % 4 or cols % 256:
        raise ValueError(f"Q4K needs rows % 4 == 0 and cols % 256 == 0, got {rows}x{cols}")
    step = max(4, chunk_rows // 4 * 4)
    return b"".join(_q4k_rows_numpy(w[r:r + step]) for r in range(0, rows, step))


def header_bytes(d: Dims, n_tensors: int, dir_off: int, data_off: int) -> bytes:
    fields = (MAGIC, VERSION, n_tensors, dir_off, data_off, 1, d.hidden, d.n_layers, d.vocab,
              d.ffn, d.n_heads, d.n_kv_heads, d.head_dim, d.rot_dim, d.lin_k_heads,
              d.lin_v_heads, d.lin_k_dim, d.lin_v_dim, d.conv_k, d.full_mask, d.eos_id, 1,
              int(d.has_mtp), d.rms_eps, d.rope_theta)
    return struct.pack(HEADER_FMT, *fields).ljust(HEADER_BYTES, b"\0")


def write_pq(path: str | os.PathLike, d: Dims, tensors: list[tuple[str, int, list[int], bytes]]
             ) -> None:
    """Write (name, dtype, shape, data) entries in the given order (tools/convert.py:158-177)."""
    dir_off = HEADER_BYTES
    data_off = -(-(dir_off + 128 * len(tensors)) // 4096) * 4096
    entries, off = [], data_off
    for name, dt, shape, data in tensors:
        if len(name.encode()) >= 80:
            raise ValueError(f"name too long: {name}")
        entries.append(off)
        off = -(-(off + len(data)) // ALIGN) * ALIGN
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    with tmp.open("wb") as f:
        f.write(header_bytes(d, len(tensors), dir_off, data_off))
        for (name, dt, shape, data), o in zip(tensors, entries):
            dims = list(shape) + [0] * (4 - len(shape))
            f.write(struct.pack(ENTRY_FMT, name.encode(), dt, len(shape), *dims, o, len(data)))
        for (_, _, _, data), o in zip(tensors, entries):
            f.write(b"\0" * (o - f.tell()))
            f.write(data)
    os.replace(tmp, path)


# ---------------------------------------------------------------- synthetic Qwen3.5 models

def tensor_specs(d: Dims) -> list[tuple[str, str, list[int]]]:
    """(pq name, kind, shape) of every tensor the engine maps (engine/src/model.c:156-205 and
    the MTP head, engine/src/mtp.c:8-32). kind: 'mat' (Q4K), 'vec' (random F32), 'one'
    (F32 norm multiplier 1.0), 'conv' (random F32 [C, K])."""
    H, ffn, hd = d.hidden, d.ffn, d.head_dim
    kd, vd = d.lin_k_heads * d.lin_k_dim, d.lin_v_heads * d.lin_v_dim
    out: list[tuple[str, str, list[int]]] = []

    def attn(p: str) -> None:
        out.extend([(p + "self_attn.q_proj.weight", "mat", [d.n_heads * hd * 2, H]),
                    (p + "self_attn.k_proj.weight", "mat", [d.n_kv_heads * hd, H]),
                    (p + "self_attn.v_proj.weight", "mat", [d.n_kv_heads * hd, H]),
                    (p + "self_attn.o_proj.weight", "mat", [H, d.n_heads * hd]),
                    (p + "self_attn.q_norm.weight", "one", [hd]),
                    (p + "self_attn.k_norm.weight", "one", [hd])])

    def block(p: str, full: bool) -> None:
        out.extend([(p + "input_layernorm.weight", "one", [H]),
                    (p + "post_attention_layernorm.weight", "one", [H]),
                    (p + "mlp.gate_proj.weight", "mat", [ffn, H]),
                    (p + "mlp.up_proj.weight", "mat", [ffn, H]),
                    (p + "mlp.down_proj.weight", "mat", [H, ffn])])
        if full:
            attn(p)
            return
        out.extend([(p + "linear_attn.in_proj_qkv.weight", "mat", [2 * kd + vd, H]),
                    (p + "linear_attn.in_proj_z.weight", "mat", [vd, H]),
                    (p + "linear_attn.in_proj_b.weight", "mat", [d.lin_v_heads, H]),
                    (p + "linear_attn.in_proj_a.weight", "mat", [d.lin_v_heads, H]),
                    (p + "linear_attn.out_proj.weight", "mat", [H, vd]),
                    (p + "linear_attn.conv1d.weight", "conv", [2 * kd + vd, d.conv_k]),
                    (p + "linear_attn.A_log", "vec", [d.lin_v_heads]),
                    (p + "linear_attn.dt_bias", "vec", [d.lin_v_heads]),
                    (p + "linear_attn.norm.weight", "one", [d.lin_v_dim])])

    out.append(("embed_tokens.weight", "mat", [d.vocab, H]))
    out.append(("norm.weight", "one", [H]))
    for i in range(d.n_layers):
        block(f"layers.{i}.", (d.full_mask >> i) & 1 == 1)
    if d.has_mtp:
        out.append(("mtp.fc.weight", "mat", [H, 2 * H]))
        for n in ("pre_fc_norm_embedding", "pre_fc_norm_hidden", "norm"):
            out.append((f"mtp.{n}.weight", "one", [H]))
        block("mtp.layers.0.", True)
    return out


def hf_name(name: str) -> str:
    return name if name.startswith("mtp.") else TEXT_PREFIX + name


def tensor_values(name: str, kind: str, shape: list[int], seed: int, std: float) -> np.ndarray:
    """float32 values of one synthetic tensor."""
    if kind == "one":
        return np.ones(shape, np.float32)
    rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


OUT_PROJ_NAMES = ("o_proj.weight", "out_proj.weight", "down_proj.weight")


def _tensor_bytes(args) -> tuple[str, int, list[int], bytes]:
    """One synthetic tensor as (name, dtype, shape, bytes); native=False quantises with numpy
    only (a worker of make_synthetic's process pool)."""
    name, kind, shape, seed, sd, native = args
    v = tensor_values(name, kind, shape, seed, sd)
    if kind == "mat":
        return name, Q4K, shape, quantize_q4k(v) if native else quantize_q4k_numpy(v)
    return name, F32, shape, v.astype("<f4").tobytes()


def _synth_args(d: Dims, seed: int, std: float, out_scale: float, native: bool):
    specs = sorted(tensor_specs(d), key=lambda s: hf_name(s[0]))
    return [(name, kind, shape, seed, std * out_scale if name.endswith(OUT_PROJ_NAMES) else std, native)
            for name, kind, shape in specs]


def synth_tensors(d: Dims, seed: int, std: float = 0.02, out_scale: float = 1.0):
    """Yield (name, dtype, shape, bytes) in the converter's order (sorted HF names).
    out_scale multiplies the std of the projections that write into the residual stream
    (o_proj, out_proj, down_proj): small values give a model whose next token depends mostly
    on the current one, so greedy decoding falls into cycles (test models for prompt lookup)."""
    for a in _synth_args(d, seed, std, out_scale, True):
        yield _tensor_bytes(a)


def make_synthetic(path: str | os.PathLike, d: Dims, seed: int = 0, std: float = 0.02,
                   out_scale: float = 1.0, native: bool = True) -> Path:
    """Write a random-init, Q4K-quantised Qwen3.5-shaped model to `path`. native=False loads no
    native library: the matrices are quantised with numpy in a pool of spawned processes (the
    same bytes)."""
    args = _synth_args(d, seed, std, out_scale, native)
    if native:
        tensors = [_tensor_bytes(a) for a in args]
    else:
        import concurrent.futures as cf
        import multiprocessing as mp
        workers = max(1, min(16, os.cpu_count() or 1))
        with cf.ProcessPoolExecutor(workers, mp_context=mp.get_context("spawn")) as ex:
            tensors = list(ex.map(_tensor_bytes, args))
    write_pq(path, d, tensors)
    return Path(path)


def sha256_file(path: str | os.PathLike) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 22), b""):
            h.update(chunk)
    return h.hexdigest()


def cached_synthetic(name: str, d: Dims, seed: int = 0, cache_dir: str | os.PathLike | None = None
                     ) -> Path:
    """Path of a synthetic model, generated on first use under cache_dir (default:
    $NB_MODEL_CACHE or <repo>/_models)."""
    root = Path(cache_dir or os.environ.get("NB_MODEL_CACHE")
                or Path(__file__).resolve().parent.parent / "_models")
    key = hashlib.sha1(repr((asdict(d), seed)).encode()).hexdigest()[:10]
    path = root / f"{name}-s{seed}-{key}.pq"
    if not path.exists():
        make_synthetic(path, d, seed)
    return path
