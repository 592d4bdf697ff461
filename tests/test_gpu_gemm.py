"""The tcgen05 tensor-core Q4K x A8 GEMM (passes of more than 16 activation rows) through the
kernel-level C ABI, bit-exact against the oracle and the reference's recorded kbench hashes.

The reference's pf_matmul takes up to 64 rows per call (engine/src/ops.h:49-52, PF_MAX_BATCH)
and its kbench recorded y-hashes at n = 17, 33 and 64 (engine/bench/kbench.c:164-219); a hash
match proves the tensor-core path bit-identical to the reference's NEON kernel on those inputs.
Larger n (prefill chunks, the multi-sequence verify batch) is checked against the oracle.
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


class Gemm:
    def __init__(self, lib, torch, rows, cols, nmax):
        self.lib, self.t, self.rows, self.cols = lib, torch, rows, cols
        self.h = lib.nb_mv_create(rows, cols, nmax)
        assert self.h, lib.last_error()
        self.s = torch.cuda.current_stream().cuda_stream

    def upload(self, w_pq):
        panels = np.zeros(self.lib.nb_q4k_panel_bytes(self.rows, self.cols), np.uint8)
        assert self.lib.nb_q4k_repack(w_pq.ctypes.data, self.rows, self.cols, panels.ctypes.data) == 0
        return self.t.from_numpy(panels).cuda()

    def quant(self, x):
        n = x.shape[0]
        self.dX = self.t.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
        assert self.lib.nb_mv_set_n(self.h, n, self.s) == 0
        assert self.lib.nb_mv_quant(self.h, self.dX.data_ptr(), self.s) == 0

    def matmul(self, dW, n, y0=None, epi=0):
        y = (self.t.zeros((n, self.rows), dtype=self.t.float32, device="cuda") if y0 is None
             else self.t.from_numpy(np.ascontiguousarray(y0, np.float32)).cuda())
        if epi == 0:
            assert self.lib.nb_mv_matmul(self.h, dW.data_ptr(), y.data_ptr(), self.s) == 0
        else:
            assert self.lib.nb_mv_prepare(self.h, dW.data_ptr(), None, self.s) == 0
            assert self.lib.nb_mv_gemm(self.h, epi, y.data_ptr(), None, None, None, None, None, self.s) == 0
        self.t.cuda.synchronize()
        assert self.lib.nb_mv_status(self.h) == 0
        return y.cpu().numpy()

    def close(self):
        self.lib.nb_mv_destroy(self.h)


def _rand_q4k(rng, rows, cols):
    from nibblemac_b200 import pq
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
    return np.frombuffer(pq.quantize_q4k(w), np.uint8)


SHAPES = sorted({(c["shape"], c["rows"], c["cols"]) for c in GOLD["cases"] if c["n"] > 16})


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: s[0])
def test_kbench_yhash_tensor_cores(lib, torch, q4k_oracle, shape):
    name, rows, cols = shape
    cases = [c for c in GOLD["cases"] if c["shape"] == name and c["n"] > 16]
    nmax = max(c["n"] for c in cases)
    g = Gemm(lib, torch, rows, cols, nmax)
    try:
        dW = g.upload(q4k_oracle.kb_matrix(rows, cols, GOLD["matrix_seed"]))
        x = q4k_oracle.kb_vec(nmax * cols, GOLD["vec_seed"]).reshape(nmax, cols)
        for c in cases:
            g.quant(x[: c["n"]])
            y = g.matmul(dW, c["n"])
            assert f"{q4k_oracle.fnv1a(y):016x}" == c["yhash"], f"{name} n={c['n']}"
    finally:
        g.close()


@pytest.mark.parametrize("rows,cols,n", [(3584, 1024, 17), (3584, 1024, 64), (3584, 1024, 100),
                                         (3584, 1024, 257), (1024, 3584, 65), (8224, 1024, 130),
                                         (36, 256, 40), (100, 768, 1000), (512, 2048, 4096)])
def test_random_matrices_bit_exact(lib, torch, q4k_oracle, rows, cols, n):
    """Partial weight tiles (8224 = 64.25 tiles, 36 and 100 rows: partial panels), partial
    activation tiles, and large n."""
    rng = np.random.default_rng(rows * 13 + cols + n)
    wq = _rand_q4k(rng, rows, cols)
    x = rng.standard_normal((n, cols), dtype=np.float32)
    x[0, :32] = 0.0                                 # an all-zero activation block
    x[n - 1, 64:96] *= 1e6                          # a block of large values
    g = Gemm(lib, torch, rows, cols, n)
    try:
        g.quant(x)
        y = g.matmul(g.upload(wq), n)
        ref = q4k_oracle.matmul(wq, rows, cols, x)
        assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))
    finally:
        g.close()


def test_rows_match_the_matvec_kernels(lib, torch, q4k_oracle):
    """kbench.c:216-219 across the two paths: row v of a 70-row tensor-core pass equals the
    1-row CUDA-core pass over the same vector, bit for bit."""
    rows, cols, n = 3584, 1024, 70
    g = Gemm(lib, torch, rows, cols, n)
    try:
        dW = g.upload(q4k_oracle.kb_matrix(rows, cols, 42))
        x = q4k_oracle.kb_vec(n * cols, 3).reshape(n, cols)
        g.quant(x)
        yb = g.matmul(dW, n)
        for v in (0, 1, 31, 32, 63, 64, 69):
            g.quant(x[v:v + 1])
            y1 = g.matmul(dW, 1)
            assert np.array_equal(yb[v].view(np.uint32), y1[0].view(np.uint32)), v
    finally:
        g.close()


def test_residual_epilogue(lib, torch, q4k_oracle):
    """Epilogue 1: y += W x with one fp32 rounding (pf_add_rows, engine/src/forward.c:68-72)."""
    rows, cols, n = 1024, 2048, 96
    rng = np.random.default_rng(11)
    wq = _rand_q4k(rng, rows, cols)
    x = rng.standard_normal((n, cols), dtype=np.float32)
    y0 = rng.standard_normal((n, rows), dtype=np.float32)
    g = Gemm(lib, torch, rows, cols, n)
    try:
        g.quant(x)
        y = g.matmul(g.upload(wq), n, y0=y0, epi=1)
        want = (y0 + q4k_oracle.matmul(wq, rows, cols, x)).astype(np.float32)
        assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
    finally:
        g.close()


# pf_expf / pf_silu of the reference (engine/src/forward_ops.c:41-59), restated in float32
# numpy for this check: every operation rounds to float32, no fused multiply-add.
def _pf_expf(x):
    f = np.float32
    x = np.clip(x.astype(f), f(-87.0), f(88.0))
    fx = np.rint(x * f(1.44269504088896341)).astype(f)
    r = (x - fx * f(0.693145751953125)).astype(f)
    r = (r - fx * f(1.428606765330187e-06)).astype(f)
    p = np.full_like(r, f(1.9875691500e-4))
    for c in (1.3981999507e-3, 8.3334519073e-3, 4.1665795894e-2, 1.6666665459e-1, 5.0000001201e-1):
        p = (p * r + f(c)).astype(f)
    y = (p * (r * r) + r).astype(f)
    y = (y + f(1.0)).astype(f)
    s = ((fx.astype(np.int32) + 127) << 23).astype(np.uint32).view(f)
    return (y * s).astype(f)


def _pf_silu(x):
    return (x / (np.float32(1.0) + _pf_expf(-x))).astype(np.float32)


def test_swiglu_epilogue(lib, torch, q4k_oracle):
    """Gate / up prepared as one concatenated tile image, then A8 of silu(gate x) * (up x)
    (pf_mlp / pf_silu_mul, engine/src/forward.c:49-58, then kern_quant_act): the input of
    down_proj."""
    ffn, cols, n = 3584, 1024, 80
    rng = np.random.default_rng(12)
    gq, uq = _rand_q4k(rng, ffn, cols), _rand_q4k(rng, ffn, cols)
    x = rng.standard_normal((n, cols), dtype=np.float32)
    g = Gemm(lib, torch, ffn, cols, n)
    try:
        dG, dU = g.upload(gq), g.upload(uq)
        g.quant(x)
        q = torch.zeros((n, ffn), dtype=torch.int8, device="cuda")
        d = torch.zeros((n, ffn // 32), dtype=torch.float32, device="cuda")
        f = torch.zeros((n, ffn // 32), dtype=torch.float32, device="cuda")
        assert lib.nb_mv_prepare(g.h, dG.data_ptr(), dU.data_ptr(), g.s) == 0
        assert lib.nb_mv_gemm(g.h, 3, None, q.data_ptr(), d.data_ptr(), f.data_ptr(), None, None, g.s) == 0
        torch.cuda.synchronize()
        assert lib.nb_mv_status(g.h) == 0
        gate = q4k_oracle.matmul(gq, ffn, cols, x)
        up = q4k_oracle.matmul(uq, ffn, cols, x)
        h = (_pf_silu(gate) * up).astype(np.float32)
        rq, rd, rf = q4k_oracle.quant_act(h, ffn)
        assert np.array_equal(q.cpu().numpy(), rq)
        assert np.array_equal(d.cpu().numpy().view(np.uint32), rd.view(np.uint32))
        assert np.array_equal(f.cpu().numpy().view(np.uint32), rf.view(np.uint32))
    finally:
        g.close()


@pytest.mark.parametrize("rows,cols,n", [(4100, 1024, 70), (2048, 2048, 33)])
def test_head_epilogue_logits_and_argmax(lib, torch, q4k_oracle, rows, cols, n):
    """Epilogue 4 (the LM head): logits bit-identical to the oracle, and the argmax from the
    per-panel keys equal to the first maximum of the oracle's logits (pf_argmax,
    engine/src/forward_ops.c:387-409); 4100 rows leave a partial tile and panel."""
    w = q4k_oracle.kb_matrix(rows, cols, 5)
    g = Gemm(lib, torch, rows, cols, n)
    try:
        dW = g.upload(w)
        x = np.random.default_rng(rows + n).standard_normal((n, cols)).astype(np.float32)
        g.quant(x)
        npan = (rows + 31) // 32
        y = torch.zeros((n, rows), dtype=torch.float32, device="cuda")
        part = torch.zeros((n, npan), dtype=torch.int64, device="cuda")
        nan0 = torch.ones(n, dtype=torch.int32, device="cuda")
        assert lib.nb_mv_prepare(g.h, dW.data_ptr(), None, g.s) == 0
        assert lib.nb_mv_gemm(g.h, 4, y.data_ptr(), None, None, None, part.data_ptr(), nan0.data_ptr(), g.s) == 0
        torch.cuda.synchronize()
        assert lib.nb_mv_status(g.h) == 0
        want = q4k_oracle.matmul(w, rows, cols, x)
        assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
        keys = part.cpu().numpy().view(np.uint64)
        for v in range(n):
            best = int(keys[v].max())
            assert 0xFFFFFFFF - (best & 0xFFFFFFFF) == int(np.argmax(want[v]))
        assert not nan0.cpu().numpy().any()
    finally:
        g.close()
