"""The CPU oracle against the reference's own recorded results.

The Q4K x A8 restatement (oracle/q4k_a8.c) with kbench's seeded inputs must reproduce every
yhash the reference recorded on the Pi (engine/bench/kbench.c:212-214, fixture made by
tests/golden/make_kbench_yhash.py). A hash match of 4*n*rows fp32 outputs pins the activation
quantisation, the integer block dots and the exact order of the fused block FMAs.
"""
import json
from pathlib import Path

import numpy as np
import pytest

GOLD = json.loads((Path(__file__).parent / "golden" / "kbench_yhash.json").read_text())


def _cases(max_work: float):
    out = []
    for c in GOLD["cases"]:
        work = c["rows"] * c["cols"] * c["n"]
        if work <= max_work:
            out.append(c)
    return out


@pytest.mark.parametrize("case", _cases(5e8), ids=lambda c: f"{c['shape']}-n{c['n']}")
def test_kbench_yhash(q4k_oracle, case):
    rows, cols, n = case["rows"], case["cols"], case["n"]
    w = q4k_oracle.kb_matrix(rows, cols, GOLD["matrix_seed"])
    x = q4k_oracle.kb_vec(n * cols, GOLD["vec_seed"]).reshape(n, cols)
    y = q4k_oracle.matmul(w, rows, cols, x)
    assert f"{q4k_oracle.fnv1a(y):016x}" == case["yhash"]


def test_fixture_covers_the_config1_shape():
    """Config 1 of the benchmark is the 3584 x 1024 shape at n = 1, 2, 4."""
    got = {(c["rows"], c["cols"], c["n"]) for c in GOLD["cases"]}
    for n in (1, 2, 4):
        assert (3584, 1024, n) in got


def test_batched_rows_equal_single_rows(q4k_oracle):
    """kbench.c:216-219: row v of a batched call equals the single-vector call bit for bit."""
    rows, cols = 512, 1024
    w = q4k_oracle.kb_matrix(rows, cols, 3)
    x = q4k_oracle.kb_vec(5 * cols, 11).reshape(5, cols)
    yb = q4k_oracle.matmul(w, rows, cols, x)
    for v in range(5):
        assert np.array_equal(yb[v].view(np.uint32), q4k_oracle.matmul(w, rows, cols, x[v]).view(np.uint32)[0])


def test_quant_act_edge_cases(q4k_oracle):
    """kern_act.c:14-41: zero blocks give zeros and d = 0; values hit +-127 at the extremes."""
    x = np.zeros((2, 64), np.float32)
    x[0, 32:] = np.linspace(-3, 3, 32)
    x[1, :32] = 1e-30
    q, d, fs = q4k_oracle.quant_act(x, 64)
    assert (q[0, :32] == 0).all() and d[0, 0] == 0 and fs[0, 0] == 0
    assert q[0, 32] == -127 and q[0, 63] == 127
    assert np.isclose(d[0, 1], 3 / 127)
