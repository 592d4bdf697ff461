"""The state blob's narrow K / V rows on the host (pinfer_params.kv_dtype, the reference's format:
engine/src/state.c:64-83, rows stored by pf_kv_store, engine/src/forward_kv.c:83-123). The device
holds the rows widened to fp32; the blob carries binary16 bits or int8 codes with their row
scales. Exhaustive over the 65,536 binary16 patterns; int8 rows quantised as the reference does."""
import ctypes

import numpy as np
import pytest

from conftest import ROOT


@pytest.fixture(scope="module")
def hooks():
    lib = ctypes.CDLL(str(ROOT / "nibblemac_b200" / "lib" / "libpinfer.so"))
    lib.nb_test_kv_f16.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong]
    lib.nb_test_kv_f16.restype = ctypes.c_int
    lib.nb_test_kv_i8.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    lib.nb_test_kv_i8.restype = ctypes.c_int
    return lib


def test_f16_bits_and_values_exhaustive(hooks):
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    # binary16 -> float: exact widening (NaN: quiet bits kept, payload shifted into place)
    vals = np.zeros(bits.size, np.float32)
    assert hooks.nb_test_kv_f16(1, bits.ctypes.data, vals.ctypes.data, bits.size) == 0
    h = bits.astype(np.uint32)
    nan = ((h >> 10) & 0x1f) == 0x1f
    nan &= (h & 0x3ff) != 0
    want = bits.view(np.float16).astype(np.float32)
    assert np.array_equal(vals[~nan].view(np.uint32), want[~nan].view(np.uint32))
    want_nan = ((h & 0x8000) << 16) | 0x7f800000 | ((h & 0x3ff) << 13)
    assert np.array_equal(vals[nan].view(np.uint32), want_nan[nan])
    # float (binary16-representable) -> bits: the inverse, and the reference's NaN rule
    back = np.zeros(bits.size, np.uint16)
    assert hooks.nb_test_kv_f16(0, vals.ctypes.data, back.ctypes.data, vals.size) == 0
    u = vals.view(np.uint32)
    want_nan_bits = (((u >> 16) & 0x8000) | 0x7c00 | 0x200 | ((u & 0x7fffff) >> 13)).astype(np.uint16)
    assert np.array_equal(back[~nan], bits[~nan])
    assert np.array_equal(back[nan], want_nan_bits[nan])


def _quantise_rows(x: np.ndarray):
    """pf_kv_store's int8 rows in float32 arithmetic: absmax, 127 / amax, rint, clamp; the
    widened value q * (amax / 127) as pf_kv_widen reads it."""
    f = np.float32
    amax = np.max(np.abs(x), axis=1).astype(f)
    tiny = f(127.0) / np.finfo(f).max
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        inv = np.where(amax > tiny, f(127.0) / amax, f(0.0)).astype(f)
        scale = (amax / f(127.0)).astype(f)
        y = np.rint((x * inv[:, None]).astype(f))
    q = np.where(np.isnan(y), 0, np.clip(y, -127, 127)).astype(np.int8)
    with np.errstate(invalid="ignore"):
        v = (q.astype(f) * scale[:, None]).astype(f)
    return q, scale, v


def test_i8_codes_from_widened_rows(hooks):
    rng = np.random.default_rng(11)
    hd = 256
    x = (rng.standard_normal((64, hd)) * rng.choice([1e-3, 1.0, 40.0], (64, 1))).astype(np.float32)
    x[3] = 0.0                                   # a zero row: scale 0, codes 0
    x[5, 7] = np.inf                             # an infinity: scale inf, widened NaN, codes 0
    x[6, 1:4] = np.float32(1e-41)                # subnormals next to normal values
    q, scale, v = _quantise_rows(x)
    out = np.zeros_like(q)
    assert hooks.nb_test_kv_i8(v.ctypes.data, scale.ctypes.data, x.shape[0], hd, out.ctypes.data) == 0
    assert np.array_equal(out, q)
    assert not out[3].any() and not out[5].any()


def test_bad_arguments(hooks):
    buf = np.zeros(4, np.float32)
    assert hooks.nb_test_kv_f16(2, buf.ctypes.data, buf.ctypes.data, 4) == -4
    assert hooks.nb_test_kv_i8(None, buf.ctypes.data, 1, 4, buf.ctypes.data) == -4
