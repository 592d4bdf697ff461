"""The whole verify path on the B200 against the reference engine (oracle/_ref, the reference's
own C sources run on the host CPU): logits bit for bit, greedy tokens identical, and
speculative decoding with the synthetic drafter identical to plain decoding with the same
acceptance counts as the reference's own speculative loop."""
import ctypes

import numpy as np
import pytest

from conftest import ref_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_available(), reason="oracle/_ref not built")]


@pytest.fixture(scope="module", params=["tiny", "small"])
def pair(request, tiny_model, small_model):
    from nibblemac_b200.model import Model
    from oracle import RefEngine
    path = tiny_model if request.param == "tiny" else small_model
    dev = Model(path, max_ctx=512)
    ref = RefEngine(path, max_ctx=512)
    yield request.param, dev, ref
    dev.close()
    ref.close()


def prompt(vocab, n, seed):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("n", [40, 64, 130])
def test_logits_all_rows_bit_exact(pair, n):
    """The logits of every row of a prompt. `small` runs it as tensor-core prefill chunks of up
    to 64 rows (40: one chunk of three 16-row sub-passes; 130: 64 + 64 + 2), `tiny` (a DeltaNet
    shape without the chunk kernels) as 16-row CUDA-core passes."""
    name, dev, ref = pair
    toks = prompt(dev.n_vocab, n, 1)
    dev.reset()
    ref.reset()
    got = dev.forward_all(toks)
    want = ref.forward_all(toks)
    bad = np.nonzero((bits(got) != bits(want)).any(axis=1))[0]
    assert len(bad) == 0, f"{name}: rows {bad[:8]} differ; max |d| {np.abs(got - want).max()}"


@pytest.mark.parametrize("lens", [(64,), (130, 70), (17, 200)])
def test_long_prompts_continue_exactly(pair, lens):
    """Evals of long prompts in a row: the rows before the last pass go through the prefill
    chunks (positions continuing across chunks and calls), the last-token logits and the whole
    state blob after each equal the reference's."""
    name, dev, ref = pair
    dev.reset()
    ref.reset()
    for i, n in enumerate(lens):
        toks = prompt(dev.n_vocab, n, 40 + i)
        assert np.array_equal(bits(dev.eval(toks)), bits(ref.eval(toks))), f"{name}: eval {i} ({n} rows)"
        assert dev.save_state() == ref.save_state(), f"{name}: state after eval {i} ({n} rows)"
    assert dev.n_past == sum(lens)


def test_eval_continues_exactly(pair):
    """Two evals in a row (positions continue) and the last-token logits of each."""
    name, dev, ref = pair
    a, b = prompt(dev.n_vocab, 21, 2), prompt(dev.n_vocab, 5, 3)
    dev.reset()
    ref.reset()
    assert np.array_equal(bits(dev.eval(a)), bits(ref.eval(a)))
    assert np.array_equal(bits(dev.eval(b)), bits(ref.eval(b)))
    assert dev.n_past == 26


def test_plain_greedy_tokens_identical(pair):
    name, dev, ref = pair
    p = prompt(dev.n_vocab, 64, 4)
    got, status = dev.generate(p, 48)
    assert status == 0
    assert got == ref.generate(p, 48)


@pytest.mark.parametrize("p_acc", [0.0, 0.5, 0.8, 1.0])
def test_synthetic_speculation_matches_plain_and_reference(pair, p_acc):
    name, dev, ref = pair
    p = prompt(dev.n_vocab, 64, 5)
    n = 40
    greedy, _ = dev.generate(p, n)
    got, st, status = dev.generate_synthetic(p, n, 3, greedy, seed=11, p=p_acc)
    assert status == 0 and got == greedy
    ref_toks, ref_st = ref.spec_generate(p, n, 3, greedy, 11, p_acc)
    assert ref_toks == greedy
    assert [st.rounds, st.drafted, st.accepted] == ref_st
    if p_acc == 1.0:
        assert st.accepted == st.drafted


def test_state_after_speculation_equals_plain(pair):
    """After a speculative generation (deferred commits flushed) the next eval gives the same
    logits as after a plain one: the rollback / replay left exact states."""
    name, dev, ref = pair
    p = prompt(dev.n_vocab, 30, 6)
    greedy, _ = dev.generate(p, 20)
    nxt = np.array([greedy[-1], 7, 9], np.int32)
    plain_logits = dev.eval(nxt)
    dev.generate_synthetic(p, 20, 3, greedy, seed=5, p=0.5)
    assert np.array_equal(bits(dev.eval(nxt)), bits(plain_logits))


def test_invalid_token_leaves_state(pair):
    from nibblemac_b200.model import PinferError
    name, dev, ref = pair
    dev.reset()
    dev.eval([1, 2, 3])
    with pytest.raises(PinferError) as e:
        dev.eval([1, dev.n_vocab])
    assert e.value.code == -4 and dev.n_past == 3


def test_context_full(pair):
    from nibblemac_b200.model import PinferError
    name, dev, ref = pair
    dev.reset()
    with pytest.raises(PinferError) as e:
        dev.eval(np.zeros(513, np.int32))
    assert e.value.code == -5 and dev.n_past == 0


def test_state_blob_equals_reference_and_round_trips(pair):
    """pinfer_state_save after the same prompt gives the reference engine's blob byte for byte
    (header with the model fingerprint, conv and recurrent states, K/V rows); loading either
    blob and continuing gives the reference's logits; bad blobs are refused like the reference
    (engine/src/state.c:120-160)."""
    from nibblemac_b200._lib import PINFER_E_ARG, PINFER_E_FORMAT
    from nibblemac_b200.model import PinferError
    name, dev, ref = pair
    a, b = prompt(dev.n_vocab, 37, 21), prompt(dev.n_vocab, 6, 22)
    dev.reset()
    ref.reset()
    dev.eval(a)
    ref.eval(a)
    blob, rblob = dev.save_state(), ref.save_state()
    assert len(blob) == len(rblob) == dev.lib.pinfer_state_size(dev.ctx)
    assert blob == rblob, f"{name}: state blob differs from the reference's"
    want = ref.eval(b)
    assert np.array_equal(bits(dev.eval(b)), bits(want))
    dev.eval(prompt(dev.n_vocab, 9, 23))          # move on, then come back
    dev.load_state(rblob)
    assert dev.n_past == len(a)
    assert np.array_equal(bits(dev.eval(b)), bits(want))
    dev.reset()
    dev.load_state(blob)
    assert np.array_equal(bits(dev.eval(b)), bits(want))
    bad = bytearray(blob)
    bad[0] ^= 1
    for data, code in ((bytes(bad), PINFER_E_FORMAT), (blob[:len(blob) - 4], PINFER_E_FORMAT),
                       (blob[:40], PINFER_E_ARG)):
        with pytest.raises(PinferError) as e:
            dev.load_state(data)
        assert e.value.code == code
    small = ctypes.create_string_buffer(16)
    assert dev.lib.pinfer_state_save(dev.ctx, small, 16) == PINFER_E_ARG


def test_long_context_attention_bit_exact(small_model):
    """Attention over ~1300 positions (the V stream wraps its 512-row ring of the cluster kernel
    more than twice): last-token logits after a long prompt and after a speculative generation
    continuing it, against the reference engine."""
    from nibblemac_b200.model import Model
    from oracle import RefEngine
    dev = Model(small_model, max_ctx=2048)
    ref = RefEngine(small_model, max_ctx=2048)
    try:
        p = prompt(dev.n_vocab, 1300, 31)
        assert np.array_equal(bits(dev.eval(p)), bits(ref.eval(p)))
        q = prompt(dev.n_vocab, 7, 32)
        assert np.array_equal(bits(dev.eval(q)), bits(ref.eval(q)))
        dev.reset()
        ref.reset()
        greedy = ref.generate(p, 24)
        toks, st, status = dev.generate_synthetic(p, 24, 3, greedy, seed=5, p=0.8)
        assert status == 0 and toks == greedy
    finally:
        dev.close()
        ref.close()


def test_clones_share_weights_and_run_concurrently(small_model):
    """pinfer_b200_clone: contexts on the source's weights with their own states, freed in
    either order; four of them generating at once from four host threads give the same tokens
    and statistics as one context alone."""
    import threading
    from nibblemac_b200.model import Model
    src = Model(small_model, max_ctx=512)
    clones = [src.clone(256) for _ in range(4)]
    try:
        prompts = [prompt(src.n_vocab, 20 + 7 * i, 40 + i) for i in range(4)]
        want = []
        for p in prompts:
            g, _ = src.generate(p, 32)
            t, st, _ = src.generate_synthetic(p, 32, 3, g, seed=3, p=0.6)
            assert t == g
            want.append((g, (st.rounds, st.drafted, st.accepted)))
        got = [None] * 4

        def run(i):
            m, p = clones[i], prompts[i]
            g, _ = m.generate(p, 32)
            t, st, _ = m.generate_synthetic(p, 32, 3, g, seed=3, p=0.6)
            got[i] = (t, (st.rounds, st.drafted, st.accepted))

        ths = [threading.Thread(target=run, args=(i,)) for i in range(4)]
        for th in ths:
            th.start()
        for th in ths:
            th.join(120)
        assert got == want
        src.close()                          # the weights live on with the clones
        g, _ = clones[0].generate(prompts[0], 32)
        assert g == want[0][0]
    finally:
        src.close()
        for m in clones:
            m.close()


@pytest.mark.parametrize("k,nv", [(1, 0), (2, 0), (3, 0), (4, 0), (3, 1000)])
def test_mtp_speculation_matches_reference(pair, k, nv):
    """pinfer_generate_greedy_ex with k > 0: drafts from the MTP head (draft chain, verify,
    pass over the committed rows, all on the device) give the plain greedy tokens and exactly the
    reference's rounds / drafted / accepted counts (its MTP drafts are bit-identical), and the
    state after it, MTP KV rows included, equals the reference's byte for byte."""
    from nibblemac_b200._lib import SpecStats
    name, dev, ref = pair
    p = prompt(dev.n_vocab, 29, 50 + k)
    dev.reset()
    plain, _ = dev.generate(p, 40)
    st = SpecStats()
    toks, status = dev.generate(p, 40, k=k, draft_vocab=nv, stats=st)
    rtoks, rst, rstatus = ref.generate_mtp(p, 40, k, nv)
    assert status == rstatus == 0
    assert toks == plain == rtoks
    assert [st.rounds, st.drafted, st.accepted] == rst, f"{name} k={k}: stats {st.rounds, st.drafted, st.accepted} vs {rst}"
    assert dev.save_state() == ref.save_state()
    # a continuation keeps drafting from the MTP rows of the first call
    q = prompt(dev.n_vocab, 3, 60 + k)
    st2 = SpecStats()
    toks2, _ = dev.generate(q, 24, k=k, draft_vocab=nv, stats=st2, append=True)
    rtoks2, rst2, _ = ref.generate_mtp(q, 24, k, nv, append=True)
    assert toks2 == rtoks2 and [st2.rounds, st2.drafted, st2.accepted] == rst2


@pytest.mark.parametrize("k", [1, 3])
def test_mtp_long_prompts_match_reference(pair, k):
    """Prompts long enough for the tensor-core prefill chunks with the MTP head's pass over each
    chunk (150 rows: chunks of 64, 64 and 16, then a 6-row pass; a 70-row continuation: one
    64-row chunk after the first call's rows): tokens and statistics as the reference's, and the
    state, MTP KV rows included, byte for byte."""
    from nibblemac_b200._lib import SpecStats
    name, dev, ref = pair
    p = prompt(dev.n_vocab, 150, 70 + k)
    dev.reset()
    st = SpecStats()
    toks, status = dev.generate(p, 32, k=k, stats=st)
    rtoks, rst, rstatus = ref.generate_mtp(p, 32, k, 0)
    assert status == rstatus == 0 and toks == rtoks
    assert [st.rounds, st.drafted, st.accepted] == rst
    assert dev.save_state() == ref.save_state(), f"{name} k={k}: state after a 150-token prompt"
    q = prompt(dev.n_vocab, 70, 80 + k)
    st2 = SpecStats()
    toks2, _ = dev.generate(q, 24, k=k, stats=st2, append=True)
    rtoks2, rst2, _ = ref.generate_mtp(q, 24, k, 0, append=True)
    assert toks2 == rtoks2 and [st2.rounds, st2.drafted, st2.accepted] == rst2
    assert dev.save_state() == ref.save_state(), f"{name} k={k}: state after the continuation"


@pytest.fixture(scope="module")
def looping_pair(looping_model):
    from nibblemac_b200.model import Model
    from oracle import RefEngine
    dev = Model(looping_model, max_ctx=512)
    ref = RefEngine(looping_model, max_ctx=512)
    yield dev, ref
    dev.close()
    ref.close()


@pytest.mark.parametrize("k,ngram", [(0, 3), (0, 7), (3, 4), (2, 7)])
def test_ngram_drafts_match_reference(looping_pair, k, ngram):
    """Prompt-lookup drafts (spec.c ngram_pick with ngram.c's index, alone at k = 0 or beside
    the MTP head) on a model whose greedy output repeats itself: the plain greedy tokens and
    exactly the reference's six statistics (n-gram rounds among them), then a continuation
    (the history drops its last token and appends the new prompt)."""
    from nibblemac_b200._lib import SpecStats
    dev, ref = looping_pair
    p = prompt(dev.n_vocab, 30, 90 + k + ngram)
    dev.reset()
    plain, _ = dev.generate(p, 48)
    st = SpecStats()
    toks, status = dev.generate(p, 48, k=k, stats=st, ngram=ngram)
    rtoks, rst, rstatus = ref.generate_mtp(p, 48, k, ngram=ngram, all_stats=True)
    assert status == rstatus == 0
    assert toks == plain == rtoks
    got = [st.rounds, st.drafted, st.accepted, st.ngram_rounds, st.ngram_drafted, st.ngram_accepted]
    assert got == rst, f"k={k} ngram={ngram}: {got} vs {rst}"
    assert rst[3] > 0, "the looping model should give n-gram rounds"
    q = np.concatenate([[toks[-1]], p[5:20]]).astype(np.int32)
    st2 = SpecStats()
    toks2, _ = dev.generate(q, 40, k=k, stats=st2, append=True, ngram=ngram)
    rtoks2, rst2, _ = ref.generate_mtp(q, 40, k, append=True, ngram=ngram, all_stats=True)
    got2 = [st2.rounds, st2.drafted, st2.accepted, st2.ngram_rounds, st2.ngram_drafted, st2.ngram_accepted]
    assert toks2 == rtoks2 and got2 == rst2, f"continuation: {got2} vs {rst2}"


@pytest.mark.parametrize("k,ngram", [(2, 0), (4, 0), (4, 5)])
def test_adaptive_speculation_keeps_tokens(pair, k, ngram):
    """pinfer_spec_params.adaptive (spec_adapt.c): k becomes an upper bound, the MTP chain runs
    on only while the newest draft's top-1 probability is >= 0.6, and plain steps replace
    speculation while it measures slower. The tokens stay the plain greedy ones (and the
    reference's); on a random model the drafts' confidence is far below 0.6, so the chain stops
    after the first draft: fewer than k drafts per speculative round. (The statistics depend on
    measured times on both sides and are not compared.)"""
    from nibblemac_b200._lib import SpecStats, SpecParams
    import ctypes
    name, dev, ref = pair
    p = prompt(dev.n_vocab, 33, 70 + k)
    dev.reset()
    plain, _ = dev.generate(p, 40)
    st = SpecStats()
    t = np.ascontiguousarray(p, np.int32)
    out = np.zeros(40, np.int32)
    sp = SpecParams(k, 0, 1, ngram)
    status = ctypes.c_int(0)
    n = dev.lib.pinfer_generate_greedy_ex(dev.ctx, t.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(t),
                                          out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), 40,
                                          ctypes.byref(sp), None, ctypes.byref(st), ctypes.byref(status))
    assert n == len(plain) and status.value == 0
    assert out[:n].tolist() == plain
    rtoks, _, _ = ref.generate_mtp(p, 40, k, ngram=ngram)
    assert rtoks == plain
    assert st.rounds > 0 and st.drafted < k * st.rounds, (st.rounds, st.drafted)


@pytest.mark.parametrize("kv_dtype", [1, 2])
def test_narrow_kv_storage_matches_reference(small_model, kv_dtype):
    """pinfer_params.kv_dtype fp16 (1) and int8 (2): K / V rows rounded as pf_kv_store stores
    them (forward_kv.c:83-123) and read widened (pf_kv_widen): the logits of a 130-row prompt
    (prefill chunks, then a 16-row pass) and of its continuation, the state blob (rows at the
    storage precision, int8 scales after each group's rows) byte for byte, MTP speculation
    tokens and counts, and a blob loaded into a fresh context continuing exactly."""
    from nibblemac_b200._lib import SpecStats
    from nibblemac_b200.model import Model
    from oracle import RefEngine
    dev = Model(small_model, max_ctx=512, kv_dtype=kv_dtype)
    ref = RefEngine(small_model, max_ctx=512, kv_dtype=kv_dtype)
    try:
        a, b = prompt(dev.n_vocab, 130, 90 + kv_dtype), prompt(dev.n_vocab, 7, 95)
        assert np.array_equal(bits(dev.eval(a)), bits(ref.eval(a)))
        assert np.array_equal(bits(dev.eval(b)), bits(ref.eval(b)))
        blob = dev.save_state()
        assert blob == ref.save_state()
        st = SpecStats()
        toks, status = dev.generate(prompt(dev.n_vocab, 40, 97), 24, k=3, stats=st, append=True)
        rtoks, rst, _ = ref.generate_mtp(prompt(dev.n_vocab, 40, 97), 24, 3, 0, append=True)
        assert status == 0 and toks == rtoks and [st.rounds, st.drafted, st.accepted] == rst
        assert dev.save_state() == ref.save_state()
        fresh = Model(small_model, max_ctx=512, kv_dtype=kv_dtype)
        try:
            fresh.load_state(blob)
            dev.load_state(blob)
            nxt = prompt(dev.n_vocab, 5, 99)
            assert np.array_equal(bits(fresh.eval(nxt)), bits(dev.eval(nxt)))
        finally:
            fresh.close()
    finally:
        dev.close()
        ref.close()
