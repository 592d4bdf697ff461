"""The verify path at the configured model widths against the reference engine (oracle/_ref,
the reference's own C sources on the host CPU), bit for bit.

Presets `0.8b-4l` and `2b-4l` (nibblemac_b200.pq) keep every width of the two configured
Qwen3.5 shapes and the full 248,320-row vocabulary, with one 3:1 group of layers (three Gated
DeltaNet layers, then gated full attention) so the scalar reference finishes in about a minute:
  0.8B: H 1024, ffn 3584, 16 DeltaNet heads x 128, attention 8 Q / 2 KV heads x 256 (a query
        group of 4), rot 64;
  2B:   H 2048, ffn 6144, the same DeltaNet, attention 16 Q / 2 KV heads (a query group of 8).
Weights are the configured random init (std 0.02, norms 1). Each preset fills a context of
`CTX` uniform-random tokens, then checks the logits of every row of the context's last 130
positions, the state blob after the context, plain greedy tokens continuing it, and synthetic
k = 3 speculation continuing it (tokens, and rounds / drafted / accepted equal to the
reference's own verify / accept / commit loop, engine/src/spec.c:323-351)."""
import numpy as np
import pytest

from conftest import _model, ref_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_available(), reason="oracle/_ref not built")]

CTX = {"0.8b-4l": 512, "2b-4l": 320}
TAIL = 130         # rows of the context's end compared with the logits of every row
GEN = 32           # tokens generated after the context
SPEC_P = {"0.8b-4l": (0.0, 0.8), "2b-4l": (0.8,)}


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.fixture(scope="module", params=["0.8b-4l", "2b-4l"])
def shaped(request):
    """(preset, device model, reference engine, context tokens, state blob after the context,
    greedy continuation): the context is filled once on each side; later tests start from its
    blob."""
    from nibblemac_b200.model import Model
    from oracle import RefEngine
    name = request.param
    path = _model(name, 7, 0.02)
    n_ctx = CTX[name]
    dev = Model(path, max_ctx=n_ctx + GEN + 8)
    ref = RefEngine(path, max_ctx=n_ctx + GEN + 8)
    toks = np.random.default_rng(17).integers(0, dev.n_vocab, n_ctx + 1).astype(np.int32)
    ctx, nxt = toks[:n_ctx], toks[n_ctx:]
    dev.reset()
    ref.reset()
    head = n_ctx - TAIL
    dlast = dev.eval(ctx[:head])
    rlast = ref.eval(ctx[:head])
    tail_dev = dev.forward_all(ctx[head:])
    tail_ref = ref.forward_all(ctx[head:])
    blob_dev, blob_ref = dev.save_state(), ref.save_state()
    ref.load_state(blob_ref)
    greedy_ref, _, _ = ref.generate_mtp(nxt, GEN, 0, append=True)
    yield dict(name=name, dev=dev, ref=ref, nxt=nxt, blob=blob_ref, blob_dev=blob_dev,
               dlast=dlast, rlast=rlast, tail_dev=tail_dev, tail_ref=tail_ref, greedy=greedy_ref)
    dev.close()
    ref.close()


def test_context_logits_every_row_bit_exact(shaped):
    """The last-token logits after the first part of the context (tensor-core prefill chunks of
    64 rows, then one 16-row pass with the head), then the logits of every row of its last 130
    positions (prefill chunks of 64, 64 and 2 rows with the head's logits), over all 248,320
    vocabulary rows."""
    s = shaped
    assert np.array_equal(bits(s["dlast"]), bits(s["rlast"])), f"{s['name']}: prefill logits differ"
    bad = np.nonzero((bits(s["tail_dev"]) != bits(s["tail_ref"])).any(axis=1))[0]
    assert len(bad) == 0, (f"{s['name']}: rows {bad[:8]} of the context tail differ; "
                           f"max |d| {np.abs(s['tail_dev'] - s['tail_ref']).max()}")


def test_state_blob_after_context_equals_reference(shaped):
    """DeltaNet recurrent and conv states of 16 heads per layer and the K/V rows of every
    position, byte for byte (the reference's blob format, engine/src/state.c)."""
    s = shaped
    assert s["blob_dev"] == s["blob"], f"{s['name']}: state blob after the context differs"


def test_plain_greedy_continuation_identical(shaped):
    s = shaped
    s["dev"].load_state(s["blob"])
    got, status = s["dev"].generate(s["nxt"], GEN, append=True)
    assert status == 0
    assert got == s["greedy"], f"{s['name']}: greedy tokens differ"


@pytest.mark.parametrize("p_acc", [0.0, 0.8])
def test_speculation_k3_matches_reference(shaped, p_acc):
    """k = 3 synthetic drafts continuing the context: the plain greedy tokens, and exactly the
    reference's rounds / drafted / accepted (rejected drafts roll the DeltaNet states back and
    truncate the KV rows on both sides)."""
    s = shaped
    if p_acc not in SPEC_P[s["name"]]:
        pytest.skip(f"{s['name']}: p = {p_acc} covered at the other width")
    dev, ref = s["dev"], s["ref"]
    dev.load_state(s["blob"])
    toks, st, status, _ = dev.generate_synthetic_ex(s["nxt"], GEN, 3, s["greedy"], seed=23, p=p_acc,
                                                    append=True)
    assert status == 0 and toks == s["greedy"], f"{s['name']} p={p_acc}: tokens differ from greedy"
    ref.load_state(s["blob"])
    rtoks, rst = ref.spec_generate(s["nxt"], GEN, 3, s["greedy"], 23, p_acc, append=True)
    assert rtoks == s["greedy"]
    assert [st.rounds, st.drafted, st.accepted] == rst, \
        f"{s['name']} p={p_acc}: {[st.rounds, st.drafted, st.accepted]} vs reference {rst}"
    # after the flush the state equals the reference's after the same tokens
    assert dev.save_state() == ref.save_state(), f"{s['name']} p={p_acc}: state after speculation differs"
