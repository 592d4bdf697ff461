"""libpinfer.so on the host, no GPU needed: exports, error codes of pinfer_load on malformed
files (the reference's tests/test_malformed.py pattern: patched headers and directories must
fail with PINFER_E_FORMAT, never crash), host-side helpers, and the glibc tables."""
import ctypes
import os
import re
import shutil
import struct
from pathlib import Path

import numpy as np
import pytest

from conftest import has_gpu
from nibblemac_b200._lib import PINFER_E_ARG, PINFER_E_FORMAT, PINFER_E_IO, PINFER_E_NOMEM

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b((?:pinfer|nb)_\w+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_exports_every_declared_function(lib):
    exported = {n for n in declared_functions() if lib.has(n)}
    missing = declared_functions() - exported
    assert not missing, f"declared in include/*.h but not exported: {sorted(missing)}"
    assert "pinfer_load" in exported and "nb_mv_matmul" in exported


def test_internal_symbols_hidden(lib):
    assert not lib.has("_ZN2nb11repack_q4kEPKhiiPh")


def test_version_and_defaults(lib):
    assert lib.version == "0.3.0"
    p = lib.pinfer_default_params()
    assert (p.n_threads, p.max_ctx, p.kv_dtype, p.gpu_split) == (4, 4096, 0, 0.0)
    sp = lib.pinfer_default_spec_params()
    assert (sp.k, sp.draft_vocab, sp.adaptive, sp.ngram) == (4, 32768, 1, 7)


def test_argmax_first_maximum(lib):
    f = lambda a: lib.pinfer_argmax(np.asarray(a, np.float32).ctypes.data_as(ctypes.POINTER(ctypes.c_float)), len(a))
    assert f([1, 3, 3, 2]) == 1
    assert f([np.nan, 5, 1]) == 0          # NaN in element 0: the reference returns 0
    assert f([1, np.nan, 5, 5]) == 2
    assert lib.pinfer_argmax(None, 3) == -1


def load(lib, path, **kw):
    p = lib.pinfer_default_params()
    for k, v in kw.items():
        setattr(p, k, v)
    err = ctypes.c_int(123)
    ctx = lib.pinfer_load(str(path).encode(), ctypes.byref(p), ctypes.byref(err))
    if ctx:
        lib.pinfer_free(ctx)
    return ctx, err.value


def test_missing_file(lib, tmp_path):
    ctx, err = load(lib, tmp_path / "nope.pq")
    assert not ctx and err == PINFER_E_IO


def test_bad_params(lib, tiny_model):
    assert load(lib, tiny_model, gpu_split=2.0)[1] == PINFER_E_ARG
    assert load(lib, tiny_model, kv_dtype=7)[1] == PINFER_E_ARG
    assert load(lib, tiny_model, kv_dtype=-1)[1] == PINFER_E_ARG
    for dt in (1, 2):   # fp16 / int8 KV storage are accepted (this host then lacks the device)
        assert load(lib, tiny_model, kv_dtype=dt)[1] != PINFER_E_ARG


HEADER_PATCHES = {
    "magic": (0, b"PINFERX\0"),
    "version": (8, struct.pack("<I", 2)),
    "arch": (32, struct.pack("<I", 9)),
    "hidden0": (36, struct.pack("<I", 0)),
    "layers_big": (40, struct.pack("<I", 33)),
    "vocab_big": (44, struct.pack("<I", 1 << 22)),
    "heads_mod": (56, struct.pack("<I", 3)),
    "rot_odd": (64, struct.pack("<I", 63)),
    "conv_k0": (84, struct.pack("<I", 0)),
    "eos": (92, struct.pack("<I", 1 << 20)),
    "tied": (96, struct.pack("<I", 2)),
    "eps_nan": (104, struct.pack("<f", float("nan"))),
    "theta_neg": (108, struct.pack("<f", -1.0)),
    "dir_off": (16, struct.pack("<Q", 1 << 40)),
    "dir_misaligned": (16, struct.pack("<Q", 4097)),
    "data_off": (24, struct.pack("<Q", 1 << 40)),
}


@pytest.mark.parametrize("name", sorted(HEADER_PATCHES))
def test_malformed_header(lib, tiny_model, tmp_path, name):
    off, data = HEADER_PATCHES[name]
    p = tmp_path / "bad.pq"
    shutil.copy(tiny_model, p)
    with p.open("r+b") as f:
        f.seek(off)
        f.write(data)
    ctx, err = load(lib, p)
    assert not ctx and err == PINFER_E_FORMAT


def _entry_offset(path: Path, name: str) -> int:
    raw = path.read_bytes()
    n, dir_off = struct.unpack_from("<IQ", raw, 12)[0], struct.unpack_from("<Q", raw, 16)[0]
    for i in range(n):
        e = dir_off + 128 * i
        if raw[e:e + 80].split(b"\0")[0].decode() == name:
            return e
    raise KeyError(name)


ENTRY_PATCHES = {
    "nbytes": (112, struct.pack("<Q", 64)),
    "offset_misaligned": (104, None),
    "offset_oob": (104, struct.pack("<Q", 1 << 42)),
    "dtype_unknown": (80, struct.pack("<I", 77)),
    "dtype_q8": (80, struct.pack("<I", 2)),          # valid Q8 size? no: nbytes differs
    "ndim0": (84, struct.pack("<I", 0)),
    "rename": (0, b"layers.0.mlp.gate_projX"),
    "unterminated": (0, b"x" * 80),
}


@pytest.mark.parametrize("name", sorted(ENTRY_PATCHES))
def test_malformed_directory(lib, tiny_model, tmp_path, name):
    p = tmp_path / "bad.pq"
    shutil.copy(tiny_model, p)
    e = _entry_offset(p, "layers.0.mlp.gate_proj.weight")
    off, data = ENTRY_PATCHES[name]
    if data is None:
        cur = struct.unpack_from("<Q", p.read_bytes(), e + 104)[0]
        data = struct.pack("<Q", cur + 4)
    with p.open("r+b") as f:
        f.seek(e + off)
        f.write(data)
    ctx, err = load(lib, p)
    assert not ctx and err == PINFER_E_FORMAT


def test_truncated_file(lib, tiny_model, tmp_path):
    p = tmp_path / "bad.pq"
    raw = tiny_model.read_bytes()
    p.write_bytes(raw[: len(raw) // 2])
    assert load(lib, p)[1] == PINFER_E_FORMAT
    p.write_bytes(raw[:100])
    assert load(lib, p)[1] == PINFER_E_FORMAT


@pytest.mark.skipif(has_gpu(), reason="checks the no-device path")
def test_valid_model_without_device_fails_loudly(lib, tiny_model):
    ctx, err = load(lib, tiny_model)
    assert not ctx and err == PINFER_E_NOMEM
    assert "no CUDA device" in lib.last_error()


def test_glibc_restatement_matches_c_library(lib):
    """The restated glibc expf / log1pf of the DeltaNet gates, compiled for the host from the
    source the device uses, equal the C library's on every 4099th 32-bit input (about a million
    per function, every sign and exponent); NB_LIBM_EXHAUSTIVE=1 checks all 2^32."""
    mism = ctypes.c_longlong(-1)
    stride = 1 if os.environ.get("NB_LIBM_EXHAUSTIVE") == "1" else 4099
    assert lib.nb_libm_selftest(max(1, os.cpu_count() or 1), stride, ctypes.byref(mism)) == 0
    assert mism.value == 0


def test_repack_roundtrip(lib, q4k_oracle):
    """The panel layout keeps every code and scale: dequantising a row from it (host mirror
    of the device embedding read) equals the oracle's row dequantisation."""
    rows, cols = 100, 512
    w = q4k_oracle.kb_matrix(rows, cols, 5)
    nbytes = lib.nb_q4k_panel_bytes(rows, cols)
    assert nbytes == 4 * (cols // 256) * 4608
    out = np.zeros(nbytes, np.uint8)
    assert lib.nb_q4k_repack(w.ctypes.data, rows, cols, out.ctypes.data) == 0
    assert lib.nb_q4k_repack(w.ctypes.data, 6, cols, out.ctypes.data) == PINFER_E_ARG
    units = out.reshape(-1, cols // 256, 9, 32, 16)
    for r in (0, 1, 37, 99):
        p, lane = divmod(r, 32)
        row = []
        for sb in range(cols // 256):
            ent = units[p, sb, 0, lane]
            A, B = (int.from_bytes(ent[:8].tobytes(), "little"), int.from_bytes(ent[8:].tobytes(), "little"))
            D = np.frombuffer(struct.pack("<H", A >> 48), np.float16)[0].astype(np.float32)
            M = np.frombuffer(struct.pack("<H", B >> 48), np.float16)[0].astype(np.float32)
            for k in range(8):
                dd = np.float32(D * np.float32((A >> (6 * k)) & 63))
                mm = np.float32(M * np.float32((B >> (6 * k)) & 63))
                codes = units[p, sb, 1 + k, lane]
                u = np.concatenate([codes & 15, codes >> 4]).astype(np.float32)
                row.append((dd * u).astype(np.float32) - mm)
        assert np.array_equal(np.concatenate(row), q4k_oracle.get_row(w, rows, cols, r))
