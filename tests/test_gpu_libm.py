"""The device's glibc expf / log1pf (the DeltaNet gate functions) against the C library.

The reference evaluates its gates with the host C library's expf and log1pf
(engine/src/forward_lin.c:19,290-293); the device evaluates glibc's published algorithms
restated in nb_math.cuh. Every 257th 32-bit pattern (about 16.7 million inputs, all signs and
exponents) plus the special values must give identical bits (NaN as NaN).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch
    assert torch.cuda.is_available()
    return torch


def _inputs() -> np.ndarray:
    bits = np.arange(0, 1 << 32, 257, dtype=np.uint64).astype(np.uint32)
    special = np.array([0x00000000, 0x80000000, 0x7f800000, 0xff800000, 0x7fc00000, 0x3f800000,
                        0xbf800000, 0x42b17217, 0x42b17218, 0xc2cff1b4, 0xc2cff1b5, 0xc2d00000,
                        0x00000001, 0x80000001, 0x3ed413d7, 0xbe95f61f, 0x5a000000, 0x31000000,
                        0x24800000], np.uint32)
    return np.concatenate([bits, special]).view(np.float32)


@pytest.mark.parametrize("fn", [0, 1], ids=["expf", "log1pf"])
def test_device_libm_equals_c_library(lib, torch, fn):
    x = _inputs()
    want = np.empty_like(x)
    assert lib.nb_libm_eval_host(fn, x.ctypes.data, want.ctypes.data, x.size) == 0
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty_like(dx)
    s = torch.cuda.current_stream().cuda_stream
    assert lib.nb_libm_eval_device(fn, dx.data_ptr(), dy.data_ptr(), x.size, s) == 0
    torch.cuda.synchronize()
    got = dy.cpu().numpy()
    nan = np.isnan(want) & np.isnan(got)
    bad = np.flatnonzero((got.view(np.uint32) != want.view(np.uint32)) & ~nan)
    assert bad.size == 0, [(hex(int(x.view(np.uint32)[i])), float(want[i]), float(got[i])) for i in bad[:5]]
