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


@pytest.mark.parametrize("case", FX["models"], ids=lambda c: c["preset"])
def test_writer_matches_reference_converter(tmp_path, case):
    path = pq.make_synthetic(tmp_path / "m.pq", pq.PRESETS[case["preset"]], case["seed"])
    assert pq.sha256_file(path) == case["sha256"]


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
