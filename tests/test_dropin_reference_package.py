"""The reference's own Python package (python/pinfer) on this library, on the host: it finds the
library through PINFER_LIB (python/pinfer/_lib.py:187-205), binds its required table (:88-100)
and every feature-detected function (:137-170) to real exports, passes structs of the same
layout, and turns a load on a host without a CUDA device into its ModelLoadError with this
library's code. Runs where a reference checkout is available ($NB_REFERENCE or `reference`
beside this repository); the device half of the drop-in is tests/test_gpu_dropin.py."""
import ctypes
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

from conftest import has_gpu

ROOT = Path(__file__).resolve().parents[1]
REF = Path(os.environ.get("NB_REFERENCE", ROOT.parent / "reference"))
PKG = REF / "python" / "pinfer" / "_lib.py"
LIB = ROOT / "nibblemac_b200" / "lib" / "libpinfer.so"

pytestmark = pytest.mark.skipif(not PKG.exists(), reason="no reference checkout with python/pinfer")

PROBE = r"""
import ctypes, json, sys
sys.path.insert(0, sys.argv[1])
import pinfer
from pinfer import _lib
L = _lib.load_library()
opt = ["pinfer_has_mtp", "pinfer_default_spec_params", "pinfer_generate_greedy", "pinfer_generate_greedy_ex",
       "pinfer_generate_greedy_cont", "pinfer_state_size", "pinfer_state_save", "pinfer_state_load",
       "pinfer_eval_select", "pinfer_checkpoint", "pinfer_rewind", "pinfer_checkpoint_clear",
       "pinfer_checkpoint_n_past"]
res = {"path": L.path, "version": L.version, "optional_missing": [n for n in opt if getattr(L, n) is None],
       "sizes": [ctypes.sizeof(c) for c in (_lib.Params, _lib.SpecParams, _lib.SpecStats, _lib.GenOpts)]}
sp = L.pinfer_default_spec_params()
res["spec_defaults"] = [sp.k, sp.draft_vocab, sp.adaptive, sp.ngram]
if len(sys.argv) > 2:
    try:
        pinfer.Model.load(sys.argv[2], tokenizer=None)
        res["load"] = "ok"
    except pinfer.ModelLoadError as e:
        res["load"] = ["ModelLoadError", e.code]
print(json.dumps(res))
"""


def _probe(model=None):
    env = dict(os.environ, PINFER_LIB=str(LIB))
    cmd = [sys.executable, "-c", PROBE, str(REF / "python")] + ([str(model)] if model else [])
    out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=120, cwd=str(ROOT.parent))
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


def test_reference_package_binds_this_library():
    from nibblemac_b200 import _lib as ours
    r = _probe()
    assert Path(r["path"]).resolve() == LIB.resolve()
    assert r["version"] == "0.3.0"
    assert r["optional_missing"] == [], "optional API the package detects but this library lacks"
    assert r["sizes"] == [ctypes.sizeof(c) for c in (ours.Params, ours.SpecParams, ours.SpecStats, ours.GenOpts)]
    assert r["spec_defaults"] == [4, 32768, 1, 7]


def test_binding_fixture_is_current():
    """The table the device test binds with is the package's own (regenerate the fixture with
    tests/golden/make_pinfer_py_bindings.py when the package changes)."""
    fixture = ROOT / "tests" / "golden" / "pinfer_py_bindings.json"
    before = fixture.read_text()
    env = dict(os.environ, NB_REFERENCE=str(REF))
    try:
        subprocess.run([sys.executable, str(ROOT / "tests" / "golden" / "make_pinfer_py_bindings.py")], env=env,
                       check=True, capture_output=True, timeout=120)
        assert json.loads(fixture.read_text()) == json.loads(before)
    finally:
        fixture.write_text(before)


@pytest.mark.skipif(has_gpu(), reason="checks the no-device error path")
def test_reference_package_load_without_device(tiny_model):
    r = _probe(tiny_model)
    assert r["load"] == ["ModelLoadError", -3]
