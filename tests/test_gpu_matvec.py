"""Q4K x A8 matmul on the B200 through the kernel-level C ABI, bit-exact against the oracle.

The oracle is pinned by the reference's recorded kbench hashes (test_oracle_golden.py), so a
hash match here proves the device kernel bit-identical to the reference's NEON kernel on the
same inputs: A8 quantisation, int32 block dots and the ordered fused block FMAs.
"""
import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLD = json.loads((Path(__file__).parent / "golden" / "kbench_yhash.json").read_text())


@pytest.fixture(scope="module")
def torch():
    import torch
    assert torch.cuda.is_available()
    return torch


class Dev:
    def __init__(self, lib, torch, rows, cols, nmax=16):
        self.lib, self.t, self.rows, self.cols = lib, torch, rows, cols
        self.h = lib.nb_mv_create(rows, cols, nmax)
        assert self.h, lib.last_error()
        self.stream = torch.cuda.current_stream().cuda_stream

    def upload(self, w_pq: np.ndarray):
        panels = np.zeros(self.lib.nb_q4k_panel_bytes(self.rows, self.cols), np.uint8)
        assert self.lib.nb_q4k_repack(w_pq.ctypes.data, self.rows, self.cols, panels.ctypes.data) == 0
        return self.t.from_numpy(panels).cuda()

    def run(self, dW, x: np.ndarray) -> np.ndarray:
        n = x.shape[0]
        dX = self.t.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
        dY = self.t.zeros((n, self.rows), dtype=self.t.float32, device="cuda")
        assert self.lib.nb_mv_set_n(self.h, n, self.stream) == 0
        assert self.lib.nb_mv_run(self.h, dW.data_ptr(), dX.data_ptr(), dY.data_ptr(), self.stream) == 0
        self.t.cuda.synchronize()
        return dY.cpu().numpy()

    def act(self, n):
        q = self.t.zeros((n, self.cols), dtype=self.t.int8, device="cuda")
        d = self.t.zeros((n, self.cols // 32), dtype=self.t.float32, device="cuda")
        f = self.t.zeros((n, self.cols // 32), dtype=self.t.float32, device="cuda")
        assert self.lib.nb_mv_get_act(self.h, q.data_ptr(), d.data_ptr(), f.data_ptr(), self.stream) == 0
        self.t.cuda.synchronize()
        return q.cpu().numpy(), d.cpu().numpy(), f.cpu().numpy()

    def close(self):
        self.lib.nb_mv_destroy(self.h)


SHAPES = sorted({(c["shape"], c["rows"], c["cols"]) for c in GOLD["cases"]})


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: s[0])
def test_kbench_yhash_on_device(lib, torch, q4k_oracle, shape):
    name, rows, cols = shape
    cases = [c for c in GOLD["cases"] if c["shape"] == name and c["n"] <= 16]
    dev = Dev(lib, torch, rows, cols)
    try:
        dW = dev.upload(q4k_oracle.kb_matrix(rows, cols, GOLD["matrix_seed"]))
        nmax = max(c["n"] for c in cases)
        x = q4k_oracle.kb_vec(nmax * cols, GOLD["vec_seed"]).reshape(nmax, cols)
        for c in cases:
            y = dev.run(dW, x[: c["n"]])
            assert f"{q4k_oracle.fnv1a(y):016x}" == c["yhash"], f"{name} n={c['n']}"
    finally:
        dev.close()


@pytest.mark.parametrize("rows,cols,n", [(3584, 1024, 1), (3584, 1024, 2), (3584, 1024, 4),
                                         (1024, 3584, 4), (8224, 1024, 3), (36, 256, 5),
                                         (4, 2048, 16), (100, 768, 7)])
def test_random_matrices_bit_exact(lib, torch, q4k_oracle, rows, cols, n):
    from nibblemac_b200 import pq
    rng = np.random.default_rng(rows * 7 + cols + n)
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
    wq = np.frombuffer(pq.quantize_q4k(w), np.uint8)
    x = rng.standard_normal((n, cols), dtype=np.float32)
    x[0, :32] = 0.0                                 # an all-zero activation block
    dev = Dev(lib, torch, rows, cols)
    try:
        y = dev.run(dev.upload(wq), x)
        ref = q4k_oracle.matmul(wq, rows, cols, x)
        assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))
        q, d, f = dev.act(n)
        rq, rd, rf = q4k_oracle.quant_act(x, cols)
        assert np.array_equal(q, rq) and np.array_equal(d.view(np.uint32), rd.view(np.uint32))
        assert np.array_equal(f.view(np.uint32), rf.view(np.uint32))
    finally:
        dev.close()


def test_rows_independent_of_batch(lib, torch, q4k_oracle):
    """kbench.c:216-219 on the device: row v of an n-vector call == the 1-vector call."""
    rows, cols = 3584, 1024
    dev = Dev(lib, torch, rows, cols)
    try:
        dW = dev.upload(q4k_oracle.kb_matrix(rows, cols, 42))
        x = q4k_oracle.kb_vec(9 * cols, 3).reshape(9, cols)
        yb = dev.run(dW, x)
        for v in range(9):
            assert np.array_equal(yb[v].view(np.uint32), dev.run(dW, x[v:v + 1])[0].view(np.uint32))
    finally:
        dev.close()


@pytest.mark.parametrize("rows,cols", [(4100, 1024), (2048, 2048)])
@pytest.mark.parametrize("n", [1, 2, 3, 4])
def test_head_kernel_bit_exact_and_argmax(lib, torch, q4k_oracle, rows, cols, n):
    """The LM-head kernel (per-panel argmax keys, optional logits) through the kernel ABI:
    logits bit-identical to the oracle, and the argmax from the keys equal to the first maximum
    of the oracle's logits (pf_argmax); rows 4100 leaves a partial last panel."""
    w = q4k_oracle.kb_matrix(rows, cols, 5)
    dev = Dev(lib, torch, rows, cols, nmax=4)
    try:
        dW = dev.upload(w)
        x = np.random.default_rng(rows + n).standard_normal((n, cols)).astype(np.float32)
        dX = torch.from_numpy(x).cuda()
        npan = (rows + 31) // 32
        y = torch.zeros((n, rows), dtype=torch.float32, device="cuda")
        part = torch.zeros((n, npan), dtype=torch.int64, device="cuda")
        nan0 = torch.zeros(16, dtype=torch.int32, device="cuda")
        s = dev.stream
        assert lib.nb_mv_set_n(dev.h, n, s) == 0 and lib.nb_mv_quant(dev.h, dX.data_ptr(), s) == 0
        assert lib.nb_mv_head_repeat(dev.h, dW.data_ptr(), 0, 1, y.data_ptr(), 1, part.data_ptr(),
                                     nan0.data_ptr(), s) == 0
        torch.cuda.synchronize()
        want = q4k_oracle.matmul(w, rows, cols, x)
        got = y.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        keys = part.cpu().numpy().view(np.uint64)
        for v in range(n):
            best = int(keys[v].max())
            assert 0xFFFFFFFF - (best & 0xFFFFFFFF) == int(np.argmax(want[v]))
        assert not nan0.cpu().numpy()[:n].any()
    finally:
        dev.close()


def test_bounded_wait_gives_up_and_reports(lib, torch):
    """A device wait whose data never comes (an mbarrier expecting bytes no copy brings, with a
    short poll limit) ends with status -90 instead of hanging, and the context stays usable."""
    import ctypes
    for limit in (64, 1024):
        st = ctypes.c_int(0)
        assert lib.nb_test_bounded_wait(limit, ctypes.byref(st)) == 0
        assert st.value == -90
    x = torch.ones(1024, device="cuda")
    assert float((x * 2).sum().item()) == 2048.0     # the context still works
    assert lib.nb_test_bounded_wait(0, ctypes.byref(ctypes.c_int())) == -4
