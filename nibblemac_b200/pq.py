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
PRESETS = {"0.8b": QWEN35_08B, "2b": QWEN35_2B, "tiny": TINY, "small": SMALL}


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


def synth_tensors(d: Dims, seed: int, std: float = 0.02, out_scale: float = 1.0):
    """Yield (name, dtype, shape, bytes) in the converter's order (sorted HF names).
    out_scale multiplies the std of the projections that write into the residual stream
    (o_proj, out_proj, down_proj): small values give a model whose next token depends mostly
    on the current one, so greedy decoding falls into cycles (test models for prompt lookup)."""
    specs = sorted(tensor_specs(d), key=lambda s: hf_name(s[0]))
    for name, kind, shape in specs:
        sd = std * out_scale if name.endswith(OUT_PROJ_NAMES) else std
        v = tensor_values(name, kind, shape, seed, sd)
        if kind == "mat":
            yield name, Q4K, shape, quantize_q4k(v)
        else:
            yield name, F32, shape, v.astype("<f4").tobytes()


def make_synthetic(path: str | os.PathLike, d: Dims, seed: int = 0, std: float = 0.02,
                   out_scale: float = 1.0) -> Path:
    """Write a random-init, Q4K-quantised Qwen3.5-shaped model to `path`."""
    write_pq(path, d, list(synth_tensors(d, seed, std, out_scale)))
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
