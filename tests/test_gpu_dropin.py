"""Drop-in check on the device: this library bound with the reference Python package's own
ctypes table (tests/golden/pinfer_py_bindings.json, recorded from python/pinfer/_lib.py by
tests/golden/make_pinfer_py_bindings.py), driven through the calls that package's Model makes
(python/pinfer/model.py: load, eval, eval_select, generate with speculation, the continuation,
state save / load, checkpoint / rewind), and compared with the reference engine (oracle/_ref)
on the same model: logits bit for bit, tokens and statistics equal."""
import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

from conftest import ref_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_available(), reason="oracle/_ref not built")]

BIND = json.loads((Path(__file__).parent / "golden" / "pinfer_py_bindings.json").read_text())
ROOT = Path(__file__).resolve().parents[1]


def _structs():
    out = {}

    def ctype(name):
        if name is None:
            return None
        if name.startswith("POINTER("):
            return ctypes.POINTER(ctype(name[8:-1]))
        if name.startswith("CFUNC("):
            return ctypes.CFUNCTYPE(*[ctype(p) for p in name[6:-1].split(",")])
        if name in out:
            return out[name]
        return getattr(ctypes, name)

    for sname in ("Params", "SpecParams", "SpecStats", "GenOpts"):
        spec = BIND["structs"][sname]
        cls = type(sname, (ctypes.Structure,), {"_fields_": [(f, ctype(t)) for f, t, _ in spec["fields"]]})
        assert ctypes.sizeof(cls) == spec["size"]
        assert [getattr(cls, f).offset for f, _, _ in spec["fields"]] == [o for _, _, o in spec["fields"]]
        out[sname] = cls
    return out, ctype


@pytest.fixture(scope="module")
def bound():
    """This library with every function typed exactly as the reference package types it."""
    structs, ctype = _structs()
    cdll = ctypes.CDLL(str(ROOT / "nibblemac_b200" / "lib" / "libpinfer.so"))
    fns = {}
    for name, sig in BIND["functions"].items():
        fn = getattr(cdll, name)   # every required and optional function is exported
        fn.restype = ctype(sig["restype"])
        fn.argtypes = [ctype(a) for a in sig["argtypes"]]
        fns[name] = fn
    return fns, structs


def _i32(a):
    a = np.ascontiguousarray(a, np.int32)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))


def _f32p(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def test_reference_package_calls_match_reference_engine(bound, small_model):
    from oracle import RefEngine
    fn, S = bound
    assert fn["pinfer_version"]().decode() == "0.3.0"
    # Model.load: default params, max_ctx, pinfer_load with an error out-parameter
    p = fn["pinfer_default_params"]()
    p.max_ctx = 512
    err = ctypes.c_int(0)
    ctx = fn["pinfer_load"](str(small_model).encode(), ctypes.byref(p), ctypes.byref(err))
    assert ctx and err.value == 0
    ref = RefEngine(small_model, max_ctx=512)
    try:
        V = fn["pinfer_n_vocab"](ctx)
        assert V == ref.n_vocab and fn["pinfer_has_mtp"](ctx) == 1
        rng = np.random.default_rng(4)
        prompt = rng.integers(0, V, 33).astype(np.int32)
        # eval: logits of the last token
        t, tp = _i32(prompt)
        out = np.zeros(V, np.float32)
        assert fn["pinfer_eval"](ctx, tp, len(t), _f32p(out)) == 0
        ref.reset()
        assert np.array_equal(out.view(np.uint32), ref.eval(prompt).view(np.uint32))
        assert fn["pinfer_n_past"](ctx) == 33
        # eval_select: logits of chosen ids only, equal to the same entries of a full eval
        nxt = rng.integers(0, V, 2).astype(np.int32)
        ids = np.array([5, 17, V - 1], np.int32)
        blob = ctypes.create_string_buffer(fn["pinfer_state_size"](ctx))
        assert fn["pinfer_state_save"](ctx, blob, len(blob)) == 0
        sel = np.zeros(len(ids), np.float32)
        tn, tnp = _i32(nxt)
        ti, tip = _i32(ids)
        assert fn["pinfer_eval_select"](ctx, tnp, len(tn), tip, len(ti), _f32p(sel)) == 0
        assert fn["pinfer_state_load"](ctx, blob, len(blob)) == 0
        full = np.zeros(V, np.float32)
        assert fn["pinfer_eval"](ctx, tnp, len(tn), _f32p(full)) == 0
        assert np.array_equal(sel.view(np.uint32), full[ids].view(np.uint32))
        # generate with MTP speculation (k = 3), a per-token callback, statistics
        got = []
        on_token = S["GenOpts"]._fields_[2][1](lambda tok, user: got.append(tok) or 0)
        opts = S["GenOpts"](None, 0, on_token, None)
        sp = fn["pinfer_default_spec_params"]()
        sp.k, sp.adaptive, sp.ngram = 3, 0, 0
        st = S["SpecStats"]()
        status = ctypes.c_int(0)
        buf = np.zeros(40, np.int32)
        n = fn["pinfer_generate_greedy_ex"](ctx, tp, len(t), buf.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), 40,
                                             ctypes.byref(sp), ctypes.byref(opts), ctypes.byref(st),
                                             ctypes.byref(status))
        toks = buf[:n].tolist()
        rtoks, rst, _ = ref.generate_mtp(prompt, 40, 3, sp.draft_vocab)
        assert status.value == 0 and toks == rtoks and got == toks
        assert [st.rounds, st.drafted, st.accepted] == rst
        # checkpoint / rewind around a continuation
        assert fn["pinfer_checkpoint"](ctx) == 0
        cp = fn["pinfer_checkpoint_n_past"](ctx)
        assert cp == fn["pinfer_n_past"](ctx)
        more, mp = _i32(rng.integers(0, V, 3))
        buf2 = np.zeros(12, np.int32)
        st2 = S["SpecStats"]()
        n2 = fn["pinfer_generate_greedy_cont"](ctx, mp, len(more), buf2.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                                                12, ctypes.byref(sp), None, ctypes.byref(st2), ctypes.byref(status))
        first = buf2[:n2].tolist()
        assert fn["pinfer_rewind"](ctx) == 0 and fn["pinfer_n_past"](ctx) == cp
        n3 = fn["pinfer_generate_greedy_cont"](ctx, mp, len(more), buf2.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                                                12, ctypes.byref(sp), None, ctypes.byref(st2), ctypes.byref(status))
        assert buf2[:n3].tolist() == first
        fn["pinfer_checkpoint_clear"](ctx)
        assert fn["pinfer_checkpoint_n_past"](ctx) == -1
        # the argmax helper, and an invalid token (state unchanged, PINFER_E_ARG)
        fa = np.array([1, 3, 3, 2], np.float32)
        assert fn["pinfer_argmax"](_f32p(fa), 4) == 1
        before = fn["pinfer_n_past"](ctx)
        bad, bp = _i32([V])
        assert fn["pinfer_eval"](ctx, bp, 1, None) == -4 and fn["pinfer_n_past"](ctx) == before
    finally:
        fn["pinfer_free"](ctx)
        ref.close()
