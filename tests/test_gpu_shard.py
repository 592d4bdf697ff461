"""Vocab-sharded LM head over 2 GPUs (pinfer_b200_shard_head): one process per GPU, NCCL
all-reduce of the argmax keys. Each rank checks its sharded results against its own unsharded
run of the same model and inputs: last-token logits after an eval (all-gathered shards) bit for
bit, greedy tokens, and speculative tokens and statistics. Needs two GPUs; skipped otherwise.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _worker(rank: int, world: int, path: str, nccl_id: bytes, q) -> None:
    import torch
    torch.cuda.set_device(rank)
    from nibblemac_b200.model import Model
    try:
        with Model(path, max_ctx=512) as m:
            rng = np.random.default_rng(3)
            p = rng.integers(0, m.n_vocab, 40).astype(np.int32)
            q2 = rng.integers(0, m.n_vocab, 5).astype(np.int32)
            m.reset()
            m.eval(p)
            plain_logits = m.eval(q2)
            m.reset()
            greedy, _ = m.generate(p, 24)
            spec, st, _ = m.generate_synthetic(p, 24, 3, greedy, seed=9, p=0.7)
            plain_stats = (st.rounds, st.drafted, st.accepted)
            m.shard_head(rank, world, nccl_id)
            m.reset()
            m.eval(p)
            sh_logits = m.eval(q2)
            m.reset()
            sh_greedy, _ = m.generate(p, 24)
            sh_spec, st2, _ = m.generate_synthetic(p, 24, 3, greedy, seed=9, p=0.7)
            ok = (np.array_equal(plain_logits.view(np.uint32), sh_logits.view(np.uint32))
                  and sh_greedy == greedy and sh_spec == spec == greedy
                  and (st2.rounds, st2.drafted, st2.accepted) == plain_stats)
            q.put((rank, ok, ""))
    except Exception as e:   # reported to the parent, which fails the test
        q.put((rank, False, repr(e)))


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_sharded_head_two_gpus(small_model):
    import torch.multiprocessing as mp
    from nibblemac_b200._lib import load_library
    lib = load_library()
    import ctypes
    buf = ctypes.create_string_buffer(128)
    assert lib.pinfer_b200_nccl_id(buf) == 0, lib.last_error()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, str(small_model), buf.raw, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = [q.get(timeout=10) for _ in procs]
    assert all(ok for _, ok, _ in res), res


def _batch_worker(rank: int, world: int, path: str, nccl_id: bytes, q) -> None:
    import torch
    torch.cuda.set_device(rank)
    from nibblemac_b200.model import Model
    try:
        with Model(path, max_ctx=512) as m:
            rng = np.random.default_rng(4)
            ps = [rng.integers(0, m.n_vocab, int(n)).astype(np.int32) for n in (7, 33, 19, 50)]
            b = m.batch(4, 256, max_k=3)
            greedy, _, _, _ = b.generate_synthetic(ps, 24)
            pad = [g + [0] * (24 - len(g)) for g in greedy]
            spec, st, _, _ = b.generate_synthetic(ps, 24, 3, pad, [1, 2, 3, 4], 0.7)
            b.close()
            m.shard_head(rank, world, nccl_id)
            b = m.batch(4, 256, max_k=3)
            sh_greedy, _, _, _ = b.generate_synthetic(ps, 24)
            sh_spec, st2, _, _ = b.generate_synthetic(ps, 24, 3, pad, [1, 2, 3, 4], 0.7)
            b.close()
            ok = (sh_greedy == greedy and sh_spec == spec == greedy
                  and (st2.rounds, st2.drafted, st2.accepted) == (st.rounds, st.drafted, st.accepted))
            q.put((rank, ok, ""))
    except Exception as e:   # reported to the parent, which fails the test
        q.put((rank, False, repr(e)))


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_sharded_head_batch_two_gpus(small_model):
    """The multi-sequence batch on a vocab-sharded context: per-row argmax keys of each shard
    merged by one NCCL all-reduce per pass; tokens and statistics equal the unsharded batch's."""
    import torch.multiprocessing as mp
    from nibblemac_b200._lib import load_library
    lib = load_library()
    import ctypes
    buf = ctypes.create_string_buffer(128)
    assert lib.pinfer_b200_nccl_id(buf) == 0, lib.last_error()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_batch_worker, args=(r, 2, str(small_model), buf.raw, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = [q.get(timeout=10) for _ in procs]
    assert all(ok for _, ok, _ in res), res
