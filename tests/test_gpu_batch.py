"""Multi-sequence batches (pinfer_b200_batch_*): many sequences in merged passes, every
projection a tcgen05 GEMM over all their rows. Each sequence's tokens and speculation counts
must equal a generation of that sequence alone on a context, which the model tests pin to the
reference engine (greedy tokens, synthetic-drafter counts of spec.c)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def prompts_of(vocab, lens, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, int(n)).astype(np.int32) for n in lens]


@pytest.fixture(scope="module")
def small(small_model):
    from nibblemac_b200.model import Model
    m = Model(small_model, max_ctx=512)
    yield m
    m.close()


@pytest.mark.parametrize("k,p", [(0, 0.0), (3, 0.8), (3, 0.0), (3, 1.0), (2, 0.5)])
def test_batch_equals_single_sequences(small, k, p):
    """Ragged prompts (1 .. 70 tokens: prefill chunks of 16 with sequences dropping out),
    speculation with acceptance from none to all."""
    lens = [1, 5, 16, 17, 33, 70, 2, 40]
    ps = prompts_of(small.n_vocab, lens, 100 + k)
    n_max = 30
    want, greedy, stats = [], [], []
    for i, pr in enumerate(ps):
        g, st = small.generate(pr, n_max)
        assert st == 0
        greedy.append(g)
        if k > 0:
            t, s, status = small.generate_synthetic(pr, n_max, k, g + [0] * (n_max - len(g)), seed=70 + i, p=p)
            assert status == 0 and t == g
            stats.append((s.rounds, s.drafted, s.accepted))
        want.append(g)
    b = small.batch(len(ps), 256, max_k=3)
    try:
        got, st, status, _ = b.generate_synthetic(ps, n_max, k, greedy=[g + [0] * (n_max - len(g)) for g in greedy],
                                                  seeds=[70 + i for i in range(len(ps))], p=p)
        assert status == [0] * len(ps)
        for i in range(len(ps)):
            assert got[i] == want[i], f"sequence {i} (prompt {lens[i]})"
        if k > 0:
            tot = [sum(x[j] for x in stats) for j in range(3)]
            assert [st.rounds, st.drafted, st.accepted] == tot
    finally:
        b.close()


@pytest.mark.parametrize("k,p", [(12, 1.0), (15, 1.0), (15, 0.7)])
def test_batch_deep_drafts(small, k, p):
    """Draft depths beyond a context's PINFER_SPEC_MAX_K (the batch takes up to 15): 16-row
    passes whose commits of up to 16 tokens the next pass's DeltaNet replays from the update
    log. Tokens equal plain greedy; at p = 1 every draft is accepted."""
    lens = [3, 20, 47]
    ps = prompts_of(small.n_vocab, lens, 300 + k)
    n_max = 50
    greedy = [small.generate(pr, n_max)[0] for pr in ps]
    b = small.batch(len(ps), 256, max_k=k)
    try:
        got, st, status, _ = b.generate_synthetic(ps, n_max, k, greedy=[g + [0] * (n_max - len(g)) for g in greedy],
                                                  seeds=[5 + i for i in range(len(ps))], p=p)
        assert status == [0] * len(ps)
        assert got == greedy
        assert st.drafted > 0
        if p == 1.0:
            assert st.accepted == st.drafted
    finally:
        b.close()


def test_batch_reuse_and_partial_slots(small):
    """A batch object runs several generations (fresh states each time), with fewer sequences
    than slots, and the same sequence gives the same tokens at any slot."""
    ps = prompts_of(small.n_vocab, [12, 9, 25], 7)
    want = [small.generate(pr, 20)[0] for pr in ps]
    b = small.batch(6, 128, max_k=3)
    try:
        got, _, status, _ = b.generate_synthetic(ps, 20)
        assert got == want and status == [0, 0, 0]
        got, _, _, _ = b.generate_synthetic(ps[::-1] + ps, 20)
        assert got == want[::-1] + want
    finally:
        b.close()


def test_batch_many_sequences_0p8b(model_08b):
    """The 0.8B shape at 64 sequences x 4 rows = 256-row verify passes (the GEMM's multi-tile
    path), against single-context generation of a few of them."""
    from nibblemac_b200.model import Model
    m = Model(model_08b, max_ctx=320)
    try:
        rng = np.random.default_rng(5)
        lens = rng.integers(8, 200, 64)
        ps = prompts_of(m.n_vocab, lens, 8)
        n_max = 24
        greedy = [m.generate(pr, n_max)[0] for pr in ps]
        pad = [g + [0] * (n_max - len(g)) for g in greedy]
        b = m.batch(64, 256, max_k=3)
        try:
            got, st, status, _ = b.generate_synthetic(ps, n_max, 3, greedy=pad, seeds=list(range(64)), p=0.8)
            assert status == [0] * 64
            assert got == greedy
            tot = [0, 0, 0]
            for i in range(64):
                t, s1, _ = m.generate_synthetic(ps[i], n_max, 3, pad[i], seed=i, p=0.8)
                assert t == greedy[i]
                tot = [tot[0] + s1.rounds, tot[1] + s1.drafted, tot[2] + s1.accepted]
            assert [st.rounds, st.drafted, st.accepted] == tot
        finally:
            b.close()
    finally:
        m.close()
