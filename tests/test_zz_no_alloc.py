"""nb_mv_run_static, the allocation-free matmul entry point, through the C ABI.

Collected last (file name) so that it also runs after every other test has used the device.
Each case makes two calls in a row with different inputs and vector counts and compares both
with the handle-based entry point (nb_mv_create / nb_mv_set_n / nb_mv_run) bit for bit, and
with the CPU oracle.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

E_ARG = -4


@pytest.fixture(scope="module")
def torch():
    import torch
    assert torch.cuda.is_available()
    return torch


def _bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("rows,cols,ns", [(3584, 1024, (4, 1)), (256, 8192, (16, 3)),
                                         (1024, 2048, (1, 7))])
def test_static_matches_handle_api(lib, torch, q4k_oracle, rows, cols, ns):
    w = q4k_oracle.kb_matrix(rows, cols, 42 + cols)
    panels = np.zeros(lib.nb_q4k_panel_bytes(rows, cols), np.uint8)
    assert lib.nb_q4k_repack(w.ctypes.data, rows, cols, panels.ctypes.data) == 0
    dW = torch.from_numpy(panels).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    h = lib.nb_mv_create(rows, cols, 16)
    assert h, lib.last_error()
    rng = np.random.default_rng(rows + cols)
    try:
        for call, n in enumerate(ns):
            x = rng.standard_normal((n, cols)).astype(np.float32)
            x[0, :32] = 0.0                          # an all-zero A8 block (amax == 0)
            dX = torch.from_numpy(x).cuda()
            y_handle = torch.full((n, rows), float("nan"), dtype=torch.float32, device="cuda")
            y_static = torch.full((n, rows), float("nan"), dtype=torch.float32, device="cuda")
            assert lib.nb_mv_set_n(h, n, stream) == 0
            assert lib.nb_mv_run(h, dW.data_ptr(), dX.data_ptr(), y_handle.data_ptr(), stream) == 0
            rc = lib.nb_mv_run_static(dW.data_ptr(), rows, cols, dX.data_ptr(), n, y_static.data_ptr(),
                                      stream)
            assert rc == 0, lib.last_error()
            torch.cuda.synchronize()
            a, b = y_handle.cpu().numpy(), y_static.cpu().numpy()
            assert np.array_equal(_bits(a), _bits(b)), f"call {call}: static != handle entry point"
            assert np.array_equal(_bits(b), _bits(q4k_oracle.matmul(w, rows, cols, x))), \
                f"call {call}: static != oracle"
    finally:
        lib.nb_mv_destroy(h)


def test_static_allocates_nothing(lib, torch, q4k_oracle):
    """After a first call (which does the per-device setup), further calls at different sizes
    change neither the device's free memory nor what torch's allocator has reserved."""
    rows, cols = 1024, 2048
    w = q4k_oracle.kb_matrix(rows, cols, 5)
    panels = np.zeros(lib.nb_q4k_panel_bytes(rows, cols), np.uint8)
    assert lib.nb_q4k_repack(w.ctypes.data, rows, cols, panels.ctypes.data) == 0
    dW = torch.from_numpy(panels).cuda()
    dX = torch.from_numpy(np.random.default_rng(1).standard_normal((16, cols)).astype(np.float32)).cuda()
    dY = torch.zeros((16, rows), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.nb_mv_run_static(dW.data_ptr(), rows, cols, dX.data_ptr(), 1, dY.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    free0, reserved0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_reserved()
    for n in (16, 3, 8, 1):
        rc = lib.nb_mv_run_static(dW.data_ptr(), rows, cols, dX.data_ptr(), n, dY.data_ptr(), stream)
        assert rc == 0, lib.last_error()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_reserved() == reserved0
    want = q4k_oracle.matmul(w, rows, cols, dX[:1].cpu().numpy())
    assert np.array_equal(_bits(dY[:1].cpu().numpy()), _bits(want))


def test_static_rejects_sizes_beyond_scratch(lib, torch):
    buf = torch.zeros(16, dtype=torch.float32, device="cuda")
    p = buf.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.nb_mv_run_static(p, 256, 8192 + 256, p, 1, p, stream) == E_ARG
    assert "static scratch" in lib.last_error()
    assert lib.nb_mv_run_static(p, 256, 1024, p, 17, p, stream) == E_ARG
    assert "static scratch" in lib.last_error()
    assert lib.nb_mv_run_static(p, 256, 1000, p, 1, p, stream) == E_ARG
    assert lib.nb_mv_run_static(None, 256, 1024, p, 1, p, stream) == E_ARG
