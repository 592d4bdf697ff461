"""The vocab-sharded LM head's argmax merge, on CPU with two gloo ranks.

Each rank takes its shard of the vocabulary rows [rank * V / 2, (rank + 1) * V / 2), reduces it
to one key per verify row with the library's own key function (nb_argmax_key, the device's), and
the ranks combine the keys with an all-reduce (max), as the device path does with NCCL. The
merged key must decode to pf_argmax of the whole row: the first maximum, ties across the shard
boundary resolved to the lower index, -0 == +0, NaN never chosen, and 0 when logit 0 is NaN
(engine/src/forward_ops.c:387-409, restated in the check below).
"""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

V, ROWS = 4096, 6


def pf_argmax(x: np.ndarray) -> int:
    """The reference's scalar argmax: best = x[0], replaced only by a strictly larger value."""
    best, bi = x[0], 0
    for i in range(1, len(x)):
        if x[i] > best:
            best, bi = x[i], i
    return bi


def logits() -> np.ndarray:
    rng = np.random.default_rng(5)
    x = rng.standard_normal((ROWS, V)).astype(np.float32)
    x[1, [100, V // 2 + 7]] = 9.0           # tie across the shard boundary: lower index wins
    x[2, [V // 2, V // 2 + 1]] = 9.0        # tie at the first row of shard 1
    x[3, :] = -0.0
    x[3, V - 1] = 0.0                       # all zeros of either sign: index 0
    x[4, 0] = np.nan                        # NaN at row 0: pf_argmax returns 0
    x[5, 17] = np.nan                       # NaN elsewhere is skipped
    x[5, V - 3] = 50.0
    return x


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nibblemac_b200._lib import load_library
        lib = load_library()
        x = logits()
        s = V // world
        keys = np.zeros(ROWS, np.uint64)
        nan0 = np.zeros(ROWS, np.int64)
        for v in range(ROWS):
            keys[v] = max(int(lib.nb_argmax_key(float(x[v, r]), r)) for r in range(rank * s, (rank + 1) * s))
            nan0[v] = int(rank == 0 and np.isnan(x[v, 0]))
        # unsigned maximum through a signed all-reduce: flip the top bit on the way in and out
        t = torch.from_numpy((keys ^ np.uint64(1 << 63)).view(np.int64).copy())
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        f = torch.from_numpy(nan0)
        dist.all_reduce(f, op=dist.ReduceOp.MAX)
        merged = t.numpy().view(np.uint64) ^ np.uint64(1 << 63)
        got = [0 if f[v] else int(0xFFFFFFFF - (int(merged[v]) & 0xFFFFFFFF)) for v in range(ROWS)]
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_sharded_argmax_merge_two_gloo_ranks():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict(q.get(timeout=10) for _ in procs)
    want = [pf_argmax(row) for row in logits()]
    assert want[1] == 100 and want[2] == V // 2 and want[3] == 0 and want[4] == 0 and want[5] == V - 3
    assert res[0] == res[1] == want
