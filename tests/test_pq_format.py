"""The .pq writer and Q4K quantiser against fixtures made by the reference's own tools.

tests/golden/make_pq_fixtures.py ran tools/quant.py (quantize_pack) and tools/convert.py on
the same values; nibblemac_b200.pq must produce byte-identical output without them.
"""
import hashlib
import json
import struct
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "golden"))
from make_pq_fixtures import quant_matrix  # noqa: E402

from nibblemac_b200 import pq  # noqa: E402

FX = json.loads((ROOT / "tests" / "golden" / "pq_fixtures.json").read_text())


@pytest.mark.parametrize("case", FX["quant"], ids=lambda c: f"{c['rows']}x{c['cols']}-s{c['seed']}")
def test_quantiser_matches_reference(case):
    w = quant_matrix(case["rows"], case["cols"], case["seed"], case["std"], case["outliers"])
    assert hashlib.sha256(pq.quantize_q4k(w)).hexdigest() == case["sha256"]


@pytest.mark.parametrize("case", FX["quant"], ids=lambda c: f"{c['rows']}x{c['cols']}-s{c['seed']}")
def test_numpy_quantiser_matches_reference(case):
    """The native-code-free quantiser (the benchmark's reference arm writes its model with it)
    gives the reference's bytes too."""
    w = quant_matrix(case["rows"], case["cols"], case["seed"], case["std"], case["outliers"])
    assert hashlib.sha256(pq.quantize_q4k_numpy(w, chunk_rows=64)).hexdigest() == case["sha256"]


@pytest.mark.parametrize("case", FX["models"], ids=lambda c: c["preset"])
@pytest.mark.parametrize("native", [True, False], ids=["native", "numpy"])
def test_writer_matches_reference_converter(tmp_path, case, native):
    path = pq.make_synthetic(tmp_path / "m.pq", pq.PRESETS[case["preset"]], case["seed"], native=native)
    assert pq.sha256_file(path) == case["sha256"]


def test_numpy_quantiser_equals_native_on_edge_values():
    """Zero groups, a group of one repeated value, tiny and large outliers, negative-only rows."""
    rng = np.random.default_rng(11)
    w = rng.standard_normal((32, 512), dtype=np.float32) * np.float32(0.02)
    w[0, :32] = 0.0
    w[1, 32:64] = 0.25
    w[2, 5] = 40.0
    w[3, 100:140] = -1e-9
    w[4] = -np.abs(w[4]) - np.float32(0.5)
    w[5, 256:] = np.float32(1e-30)
    assert pq.quantize_q4k_numpy(w, chunk_rows=8) == pq.quantize_q4k(w)


def test_struct_sizes():
    assert struct.calcsize(pq.HEADER_FMT) == 8 + 4 + 4 + 8 + 8 + 18 * 4 + 8
    assert struct.calcsize(pq.ENTRY_FMT) == 128


def test_quantiser_rejects_bad_shapes():
    with pytest.raises(ValueError):
        pq.quantize_q4k(np.zeros((6, 256), np.float32))
    with pytest.raises(ValueError):
        pq.quantize_q4k(np.zeros((4, 200), np.float32))


def test_quantiser_thread_count_invariant():
    w = np.random.default_rng(3).standard_normal((64, 512), dtype=np.float32)
    assert pq.quantize_q4k(w, threads=1) == pq.quantize_q4k(w, threads=7)
