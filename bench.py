"""Benchmark of the speculative verify path (metric: greedy spec-decode tok/s/GPU at k = 3, and
Q4K matvec HBM GB/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N ...

Workload: the Qwen3.5-0.8B-shaped model, random init (std 0.02,
norms 1), Q4K-quantised; a 512-token uniform-random context; 128 greedy tokens with draft
depth k = 3 and the synthetic drafter at acceptance p = 0.8 (the sweep p in {0, 0.5, 0.8, 1}
is reported beside it). A step is one generation of 128 tokens continuing the prefilled
context (restored with pinfer_rewind before every step, outside the timed region).
  value  tokens / device time of the verify / accept loop (CUDA events on the engine's stream;
         weights, states and context already in HBM)
  e2e    tokens / wall time of the public API call (pinfer_b200_generate_synthetic_ex: prompt
         and greedy stream copied in, 1-token prefill, decode, tokens copied out)
  prefill  pinfer_eval of the 511 context tokens from an empty state (tensor-core chunks of up
         to 64 rows), and at N=1 of configs[4]'s 4095 tokens on the 2B shape: device and wall ms
  config4 / config5  configs[3] (256 requests per GPU, one batch) and, at N=1, configs[4] on one
         GPU (batch of 8 contexts of 4096 tokens, head unsharded; --config5 shards it over ranks)
Multi-GPU: one independent replica per GPU (replicas only, no collective on the data path),
weak scaling; value = all tokens / max over ranks of the device time.
--impl reference: the reference engine's own CPU path (oracle/_ref, scalar C) on the host
cores, same metric, a bounded sample per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

K_DRAFT = 3
N_GEN = 128
CTX = 512
P_MAIN = 0.8
P_SWEEP = (0.0, 0.5, 0.8, 1.0)
SEED_MODEL = 0
METRIC = "greedy spec-decode tok/s/GPU (k=3) and Q4K matvec HBM GB/s vs ~8 TB/s peak"
UNIT = "tok/s"


def peaks() -> tuple[float, str]:
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons during the timed region."""

    def __init__(self, gpu: int) -> None:
        self.gpu, self.rows, self.proc = gpu, [], None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[0]))
                mx = max(mx, float(r[1]))
                for n, v in zip(names, r[3:7]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def model_path(rank: int, dist, preset: str = "0.8b", native: bool = True) -> Path:
    """The synthetic model of `preset`, written once by rank 0 (to a temporary name, then
    renamed, so no rank opens a partial file). native=False writes it with numpy only (the
    same bytes), for a process that must not load this package's libraries."""
    from nibblemac_b200 import pq
    path = ROOT / "_models" / f"bench-{preset}-s{SEED_MODEL}.pq"
    if rank == 0 and not path.exists():
        tmp = path.with_suffix(".tmp")
        pq.make_synthetic(tmp, pq.PRESETS[preset], SEED_MODEL, std=0.02, native=native)
        os.replace(tmp, path)
    if dist is not None:
        dist.barrier()
    while not path.exists():
        time.sleep(0.5)
    return path


def context_tokens(rank: int, vocab: int) -> np.ndarray:
    return np.random.default_rng(1234 + rank).integers(0, vocab, CTX).astype(np.int32)


def measure_prefill(m, torch, tokens: np.ndarray, reps: int = 3) -> dict:
    """pinfer_eval of a context's tokens from an empty state (tensor-core prefill chunks of up
    to 64 rows): device time from CUDA events on the context's stream, and the call's wall time
    (tokens copied in, launches, the final synchronisation). One untimed call first; leaves
    the context filled with the tokens."""
    stream = torch.cuda.ExternalStream(m.stream())
    dev, wall = [], []
    for i in range(reps + 1):
        m.reset()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        t0 = time.perf_counter()
        m.eval(tokens, logits=False)
        t1 = time.perf_counter()
        e1.record(stream)
        e1.synchronize()
        if i:
            dev.append(e0.elapsed_time(e1))
            wall.append((t1 - t0) * 1000.0)
    d = statistics.median(dev)
    return {"tokens": int(len(tokens)), "device_ms": round(d, 3), "wall_ms": round(statistics.median(wall), 3),
            "tok_s": round(len(tokens) / (d / 1000.0), 1)}


def measure_config5(torch, rank: int, local: int) -> tuple[dict, dict]:
    """configs[4] on one GPU (the head unsharded): the 2B-shaped model's 4095-token context
    prefilled on one context (pinfer_eval), then one step of the configured batch of 8 such
    contexts at k = 3, p = 0.8 (as `--config5`: tokens / device time of the verify rounds, the
    prompts' prefill outside). Returns (prefill record, decode record)."""
    from nibblemac_b200.model import Model
    path = model_path(rank, None, "2b")
    max_ctx = CTX5 + N_GEN + 16
    m = Model(path, max_ctx=max_ctx)
    try:
        rng = np.random.default_rng(4321)
        ctx = rng.integers(0, m.n_vocab, CTX5).astype(np.int32)
        prefill = {"model": "2b", **measure_prefill(m, torch, ctx[:-1], reps=2)}
        nseq = 8
        b = m.batch(nseq, max_ctx, max_k=K_DRAFT)
        try:
            prompts = [ctx] + [rng.integers(0, m.n_vocab, CTX5).astype(np.int32) for _ in range(nseq - 1)]
            greedy, _, status, _ = b.generate_synthetic(prompts, N_GEN)
            assert status == [0] * nseq
            pad = [g + [0] * (N_GEN - len(g)) for g in greedy]
            seeds = [600 + j for j in range(nseq)]
            b.generate_synthetic(prompts, N_GEN, K_DRAFT, pad, seeds, P_MAIN)   # warm-up
            with Clocks(local) as clk:
                toks, st, status, ms = b.generate_synthetic(prompts, N_GEN, K_DRAFT, pad, seeds, P_MAIN)
            assert status == [0] * nseq and toks == greedy, "speculative output differs from plain greedy"
            tokens = sum(len(g) - 1 for g in greedy)
            decode = {"metric": "greedy spec-decode tok/s (k=3), 2B shape", "value": round(tokens / (ms / 1000.0), 1),
                      "unit": UNIT, "n_gpus": 1, "ms": round(ms, 1), "verify_rounds": b.rounds(),
                      "workload": f"configs[4] on one GPU: Qwen3.5-2B-shaped Q4K, k=3, p={P_MAIN}, "
                                  f"{CTX5}-token contexts, {N_GEN} generated each, batch {nseq}; the LM "
                                  "head unsharded (one GPU); verify rounds timed, prefill outside",
                      "clocks": clk.summary()}
        finally:
            b.close()
        return prefill, decode
    finally:
        m.close()


def matvec_roofline(torch, lib, peak_gbs: float) -> dict:
    """The dominant kernel, the Q4K x A8 matvec, timed alone with CUDA events on the stream it
    runs on: the LM-head shape (248320 x 1024, n = 4 verify rows, 143 MB of weights, the
    largest matrix of a round) over two weight copies (286 MB > L2, so every launch streams
    from HBM), and the config-1 shape (3584 x 1024, n = 1, 2, 4) over a rotating arena of
    copies larger than 2x L2."""
    from oracle import Q4KOracle
    orc = Q4KOracle()
    s = torch.cuda.current_stream()
    out = {}

    def run(rows, cols, n, copies, iters, head=False):
        w = orc.kb_matrix(rows, cols, 42)
        nbytes = lib.nb_q4k_panel_bytes(rows, cols)
        panels = np.zeros(nbytes, np.uint8)
        lib.nb_q4k_repack(w.ctypes.data, rows, cols, panels.ctypes.data)
        stride = (nbytes + 255) // 256 * 256
        arena = torch.empty(stride * copies, dtype=torch.uint8, device="cuda")
        one = torch.from_numpy(panels).cuda()
        for c in range(copies):
            arena[c * stride:c * stride + nbytes].copy_(one)
        x = torch.from_numpy(orc.kb_vec(n * cols, 7).reshape(n, cols)).cuda()
        y = torch.empty((n, rows), dtype=torch.float32, device="cuda")
        part = torch.empty((n, (rows + 31) // 32), dtype=torch.int64, device="cuda")
        nan0 = torch.empty(16, dtype=torch.int32, device="cuda")
        h = lib.nb_mv_create(rows, cols, max(4, n))
        lib.nb_mv_set_n(h, n, s.cuda_stream)
        lib.nb_mv_quant(h, x.data_ptr(), s.cuda_stream)

        def launch(k):
            if head:
                return lib.nb_mv_head_repeat(h, arena.data_ptr(), stride, copies, y.data_ptr(), k,
                                             part.data_ptr(), nan0.data_ptr(), s.cuda_stream)
            return lib.nb_mv_matmul_repeat(h, arena.data_ptr(), stride, copies, y.data_ptr(), k, s.cuda_stream)

        assert launch(max(copies, 3)) == 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(s)
        assert launch(iters) == 0
        e1.record(s)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / iters
        ref = orc.matmul(w, rows, cols, x.cpu().numpy())
        exact = bool(np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32)))
        lib.nb_mv_destroy(h)
        wbytes = rows // 4 * (cols // 256) * 576
        alg = wbytes + n * cols * 4 + n * rows * 4     # W + X (fp32 in) + Y (fp32 out)
        del arena, one
        torch.cuda.empty_cache()
        return us, alg, exact

    us, alg, exact = run(248320, 1024, 4, 2, 20, head=True)
    out["head"] = {"rows": 248320, "cols": 1024, "n": 4, "us": round(us, 2),
                   "bytes": alg, "gbs": round(alg / (us * 1e-6) / 1e9, 1), "bit_exact": exact}
    # the dominant kernel of a verify round: the 8-row slice matvec of the out / o / down
    # projections (1024 rows x 2048 / 3584 columns, the pass's 4 rows)
    sl, tb, tt = {}, 0, 0.0
    for rows, cols in ((1024, 2048), (1024, 3584)):
        us1, alg1, ex1 = run(rows, cols, 4, 256, 512)
        sl[f"{rows}x{cols}"] = {"us": round(us1, 2), "bytes": alg1, "gbs": round(alg1 / (us1 * 1e-6) / 1e9, 1),
                                "bit_exact": ex1}
        tb += alg1
        tt += us1
    out["slice_out_down"] = sl
    achieved = tb / (tt * 1e-6) / 1e9
    cfg1 = {}
    for n in (1, 2, 4):
        us1, alg1, ex1 = run(3584, 1024, n, 128, 256)
        cfg1[str(n)] = {"us": round(us1, 2), "gbs": round(alg1 / (us1 * 1e-6) / 1e9, 1), "bit_exact": ex1}
    out["config1_3584x1024"] = cfg1
    out["_achieved"] = achieved
    out["_peak"] = peak_gbs
    return out


def round_bytes(path: Path, ctx_avg: int, k: int) -> int:
    """Algorithmic bytes of one verify round of the model at `path`: every tensor of the forward
    (the layers, the tied head and the norms; not the MTP head) read once, the DeltaNet
    recurrent states read and written, the conv states read and written, the K/V rows of
    ctx_avg positions read, and the k rows of the update log written."""
    import struct
    from nibblemac_b200 import pq
    with open(path, "rb") as f:
        hdr = f.read(pq.HEADER_BYTES)
        fields = struct.unpack_from(pq.HEADER_FMT, hdr)
        n_tensors, dir_off = fields[2], fields[3]
        f.seek(dir_off)
        d = f.read(128 * n_tensors)
    wbytes = 0
    for i in range(n_tensors):
        name, dt, nd, s0, s1, s2, s3, off, nb = struct.unpack_from(pq.ENTRY_FMT, d, 128 * i)
        if not name.split(b"\0", 1)[0].startswith(b"mtp."):
            wbytes += nb
    (_, _, _, _, _, _, H, L, V, ffn, nq, nkv, hd, rot, lkh, lvh, lkd, lvd, K, mask, *_rest) = fields
    n_full = bin(mask).count("1")
    n_lin = L - n_full
    C = 2 * lkh * lkd + lvh * lvd
    state = 2 * n_lin * lvh * lkd * lvd * 4
    conv = 2 * n_lin * (K - 1) * C * 4
    kv = n_full * 2 * nkv * hd * 4 * ctx_avg
    log = k * n_lin * lvh * (lkd + lvd + 1) * 4
    return int(wbytes + state + conv + kv + log)


def traffic_from_profiles(name: str = "q4k_slice_out_down_n4.md") -> float | None:
    """dram bytes per launch of the dominant kernel from its committed ncu summary."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


REF_TOKENS = 16   # tokens per step of the reference CPU path: a bounded sample of the N_GEN


class RefContext:
    """The reference engine (oracle/_ref: its own scalar C sources, one thread) holding the
    benchmark context, prefilled once and checkpointed; each step rewinds to it
    (pinfer_checkpoint / pinfer_rewind, engine/include/pinfer.h:170-175) and runs the
    synthetic-drafter verify loop for REF_TOKENS tokens at k = 3 continuing the context, the
    same workload as the device's steps cut to a bounded sample."""

    def __init__(self, path: Path) -> None:
        from oracle import RefEngine
        self.ref = RefEngine(path, max_ctx=CTX + N_GEN + 16)
        self.ctx = context_tokens(0, self.ref.n_vocab)
        t0 = time.perf_counter()
        self.ref.reset()
        self.ref.eval(self.ctx[:-1])
        self.prefill_s = time.perf_counter() - t0
        self.blob = self.ref.save_state()
        self.ref.checkpoint()
        self.greedy, _, st = self.ref.generate_mtp(self.ctx[-1:], REF_TOKENS, 0, append=True)
        assert st == 0 and len(self.greedy) == REF_TOKENS

    def step(self, seed: int, p: float = P_MAIN) -> tuple[int, float]:
        """(decode-loop tokens, decode-loop seconds) of one sample."""
        self.ref.rewind()
        toks, _ = self.ref.spec_generate(self.ctx[-1:], REF_TOKENS, K_DRAFT, self.greedy, seed, p,
                                         append=True)
        assert toks == self.greedy, "reference speculative tokens differ from its greedy tokens"
        return len(toks) - 1, self.ref.last_decode_s   # the first token comes from the prefill

    def close(self) -> None:
        self.ref.close()


def ref_sample_text(steps: int) -> str:
    return (f"reference engine (scalar C, oracle/_ref, 1 thread) on the same 0.8B-shaped model: "
            f"the {CTX}-token context prefilled once and restored by pinfer_rewind before each "
            f"step, then {REF_TOKENS} of the {N_GEN} generated tokens at k={K_DRAFT} p={P_MAIN} "
            f"per step, {steps} steps, decode loop timed")


def cpu_baseline_sample(path: Path, dev_blob: bytes, dev_greedy: list[int]) -> dict:
    """The reference's CPU path on a bounded sample of the bench workload (RefContext), after
    two checks against the device run on the same context: the reference's state blob after
    the context equals the device's byte for byte, and its greedy tokens continuing it equal
    the device's first REF_TOKENS tokens."""
    rc = RefContext(path)
    try:
        assert rc.blob == dev_blob, "reference state after the bench context differs from the device's"
        assert rc.greedy == dev_greedy[:REF_TOKENS], "reference greedy tokens differ from the device's"
        steps = 2
        toks = secs = 0.0
        for i in range(steps):
            n, t = rc.step(1000 + i)
            toks += n
            secs += t
    finally:
        rc.close()
    return {"value": round(toks / secs, 3), "unit": UNIT, "cores": 1, "kind": "reference",
            "sample": ref_sample_text(steps), "tokens_match_device": True, "state_matches_device": True}


def bench_config(world: int) -> dict:
    return {"workload": "configs[2]: Qwen3.5-0.8B-shaped Q4K, k=3 speculation, "
                        f"p={P_MAIN}, {CTX}-token context, {N_GEN} generated",
            "k": K_DRAFT, "p": P_MAIN, "context": CTX, "generated": N_GEN,
            "parallelism": f"replicas x{world}" if world > 1 else "single replica",
            "l2": "inputs larger than L2 (425 MB of weights streamed per round)"}


def run_reference(args, rank: int, world: int) -> None:
    """--impl reference: the reference's own CPU implementation of the path (oracle/_ref,
    built from its sources; scalar C, whose thread pool is a stub, so one host thread) on this
    arm's workload. Each step is a bounded sample (RefContext). Loads no library of this
    package: the model file, if missing, is written by the numpy-only writer."""
    if rank != 0:
        return
    path = model_path(0, None, native=False)
    rc = RefContext(path)
    secs, toks = [], 0
    for i in range(args.warmup + args.steps):
        n, t = rc.step(11 + i)
        if i >= args.warmup:
            secs.append(t)
            toks += n
    rc.close()
    total = sum(secs)
    value = toks / total
    cfg = bench_config(1)
    if world > 1:
        cfg["parallelism"] = f"single process (rank 0 of {world})"
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total * 1000 / args.steps, 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4k x int8 -> fp32",
            "data": "synthetic (random-init 0.8B-shaped weights, uniform-random context, "
                    "synthetic drafter)",
            "config": cfg,
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": 1, "kind": "reference",
                             "sample": ref_sample_text(args.steps),
                             "prefill_s": round(rc.prefill_s, 1)},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


CTX5 = 4096
N_SEQ4, GEN4 = 256, 256


def measure_config4(m, rank: int, world: int, local: int, dist, dev_tensors: bool) -> dict | None:
    """256 independent requests per GPU (uniform-random prompts of length
    U[32, 1024], 256 generated tokens each, k = 3 at p = 0.8) on the 0.8B-shaped model `m`, all
    in one multi-sequence batch (pinfer_b200_batch on m's weights): the prompts' prefill and every
    verify round run the 256 sequences in merged passes, so each projection is one tcgen05
    tensor-core GEMM over up to 4096 prefill rows or 1024 verify rows; one replica per GPU (weak
    scaling). The greedy streams the drafter needs come from an untimed plain (k = 0) batch run,
    whose tokens equal single-sequence greedy decoding. value = generated tokens of all ranks /
    max over ranks of the device time of the whole batched generation (prefill included; CUDA
    events on the batch's stream); e2e = the same over the host wall time of the API call
    (prompts in, tokens out). Returns the record on rank 0."""
    import torch
    max_ctx = 1024 + GEN4 + 16
    batch = m.batch(N_SEQ4, max_ctx, max_k=K_DRAFT)
    rng = np.random.default_rng(777 + rank)
    lens = rng.integers(32, 1025, N_SEQ4)
    prompts = [rng.integers(0, m.n_vocab, int(n)).astype(np.int32) for n in lens]
    seeds = [9000 + j for j in range(N_SEQ4)]
    # untimed: the greedy streams (shorter where the random model emits EOS), then a short run
    # that captures the k = 3 round graph
    greedy, _, status, _ = batch.generate_synthetic(prompts, GEN4)
    assert status == [0] * N_SEQ4 and all(0 < len(g) <= GEN4 for g in greedy)
    padded = [g + [0] * (GEN4 - len(g)) for g in greedy]
    batch.generate_synthetic(prompts, 8, K_DRAFT, [x[:8] for x in padded], seeds, P_MAIN)
    stream = torch.cuda.ExternalStream(batch.stream())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    with Clocks(local) as clk:
        ev0.record(stream)
        w0 = time.perf_counter()
        toks, st, status, decode_ms = batch.generate_synthetic(prompts, GEN4, K_DRAFT, padded, seeds, P_MAIN)
        w1 = time.perf_counter()
        ev1.record(stream)
        torch.cuda.synchronize()
    assert status == [0] * N_SEQ4 and toks == greedy, "speculative output differs from plain greedy"
    batch_rounds = batch.rounds()
    t = ev0.elapsed_time(ev1) / 1000.0
    wall = w1 - w0
    if dist is not None:
        tt = torch.tensor([t, wall], dtype=torch.float64, device="cuda" if dev_tensors else "cpu")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t, wall = tt.tolist()
    batch.close()
    if rank != 0:
        return None
    tokens = sum(len(g) for g in greedy) * world
    h2d = int(lens.sum()) * 4 + N_SEQ4 * GEN4 * 4 + N_SEQ4 * 12
    return {
        "metric": "greedy spec-decode tok/s (k=3), multi-stream, whole job", "value": round(tokens / t, 1),
        "unit": UNIT, "n_gpus": world, "ms": round(t * 1000.0, 1), "scaling": "weak",
        "workload": f"configs[3]: {N_SEQ4} requests per GPU, prompts U[32,1024], {GEN4} generated "
                    f"each, k=3, p={P_MAIN}; prefill inside the timed span",
        "batching": f"{N_SEQ4} sequences in merged passes (verify rows {N_SEQ4 * (K_DRAFT + 1)})",
        "parallelism": f"replicas x{world}" if world > 1 else "single replica",
        "batch_rounds": batch_rounds, "rounds_per_gpu": int(st.rounds), "accepted_per_gpu": int(st.accepted),
        "decode_ms": round(decode_ms, 1), "prefill_and_setup_ms": round(t * 1000.0 - decode_ms, 1),
        "mean_prompt": float(lens.mean()), "l2": "inputs larger than L2 (weights 425 MB, states 4.8 GB)",
        "e2e": {"value": round(tokens / wall, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": N_SEQ4 * GEN4 * 4 + N_SEQ4 * 8},
        "clocks": clk.summary()}


def run_config4(args, rank: int, world: int, local: int) -> None:
    """--config4: the configs[3] record (measure_config4) as its own JSON line."""
    import datetime
    import torch
    sys.path.insert(0, str(ROOT / "oracle"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=1800))
    from nibblemac_b200.model import Model
    path = model_path(rank, dist)
    base = Model(path, max_ctx=1024 + GEN4 + 16)
    rec = measure_config4(base, rank, world, local, dist, False)
    base.close()
    if rank == 0:
        line = {k: rec[k] for k in ("metric", "value", "unit", "n_gpus")}
        line.update({"steps": 1, "warmup": 1, "ms_per_step": rec["ms"], "higher_is_better": True,
                     "scaling": "weak", "vs_baseline": None, "dtype": "q4k x int8 -> fp32",
                     "data": "synthetic (random-init 0.8B-shaped weights, uniform-random prompts, "
                             "synthetic drafter)",
                     "config": {k: rec[k] for k in ("workload", "batching", "parallelism", "batch_rounds",
                                                    "rounds_per_gpu", "accepted_per_gpu", "decode_ms",
                                                    "prefill_and_setup_ms", "mean_prompt", "l2")},
                     "e2e": rec["e2e"], "clocks": rec["clocks"]})
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_profile_gemm(n: int) -> None:
    """The tensor-core GEMM through the kernel ABI on the config-1 matrix shape, for ncu."""
    import torch
    from nibblemac_b200._lib import load_library
    lib = load_library()
    rows, cols = 3584, 1024
    h = lib.nb_mv_create(rows, cols, n)
    assert h, lib.last_error()
    g = torch.Generator(device="cpu").manual_seed(1)
    w = torch.randint(0, 255, (lib.nb_q4k_panel_bytes(rows, cols),), dtype=torch.uint8, generator=g).cuda()
    x = torch.randn(n, cols, generator=g).cuda()
    y = torch.zeros(n, rows, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.nb_mv_set_n(h, n, s) == 0 and lib.nb_mv_quant(h, x.data_ptr(), s) == 0
    assert lib.nb_mv_prepare(h, w.data_ptr(), None, s) == 0
    for _ in range(5):
        assert lib.nb_mv_gemm(h, 0, y.data_ptr(), None, None, None, None, None, s) == 0
    torch.cuda.synchronize()
    assert lib.nb_mv_status(h) == 0
    lib.nb_mv_destroy(h)


def run_profile_matvec(rows: int, cols: int, n: int) -> None:
    """The Q4K x A8 matmul through the kernel ABI (nb_mv_matmul: the slice kernel for 2048 or more
    columns and 2-4 vectors, else the panel kernel), 4 launches on the kbench-seeded matrix,
    checked bit for bit against the oracle; for ncu -k."""
    import torch
    sys.path.insert(0, str(ROOT / "oracle"))
    from nibblemac_b200._lib import load_library
    from oracle import Q4KOracle
    lib, orc = load_library(), Q4KOracle()
    s = torch.cuda.current_stream().cuda_stream
    w = orc.kb_matrix(rows, cols, 42)
    panels = np.zeros(lib.nb_q4k_panel_bytes(rows, cols), np.uint8)
    assert lib.nb_q4k_repack(w.ctypes.data, rows, cols, panels.ctypes.data) == 0
    dW = torch.from_numpy(panels).cuda()
    x = torch.from_numpy(orc.kb_vec(n * cols, 7).reshape(n, cols)).cuda()
    y = torch.empty((n, rows), dtype=torch.float32, device="cuda")
    h = lib.nb_mv_create(rows, cols, max(n, 4))
    assert h, lib.last_error()
    assert lib.nb_mv_set_n(h, n, s) == 0 and lib.nb_mv_quant(h, x.data_ptr(), s) == 0
    for _ in range(4):
        assert lib.nb_mv_matmul(h, dW.data_ptr(), y.data_ptr(), s) == 0
    torch.cuda.synchronize()
    lib.nb_mv_destroy(h)
    ref = orc.matmul(w, rows, cols, x.cpu().numpy())
    assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32)), "matvec != oracle"


def run_profile_prefill(preset: str, ntok: int) -> None:
    """One untimed pinfer_eval of ntok uniform-random tokens on the bench model of `preset`,
    then the same prefill inside cudaProfilerStart/Stop (for ncu --profile-from-start off)."""
    import torch
    from nibblemac_b200.model import Model
    path = model_path(0, None, preset)
    m = Model(path, max_ctx=ntok + 16)
    toks = np.random.default_rng(4321).integers(0, m.n_vocab, ntok).astype(np.int32)
    m.eval(toks, logits=False)
    m.reset()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    m.eval(toks, logits=False)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    m.close()


def run_profile_batch(nseq: int, ntok: int) -> None:
    """Config-4 style batch generation for ncu: plain and warm-up runs, then one k = 3 run
    inside cudaProfilerStart/Stop."""
    import torch
    from nibblemac_b200.model import Model
    path = model_path(0, None)
    max_ctx = 1024 + GEN4 + 16
    base = Model(path, max_ctx=max_ctx)
    b = base.batch(nseq, max_ctx, max_k=K_DRAFT)
    rng = np.random.default_rng(777)
    lens = rng.integers(32, 1025, nseq)
    prompts = [rng.integers(0, base.n_vocab, int(n)).astype(np.int32) for n in lens]
    greedy, _, _, _ = b.generate_synthetic(prompts, ntok)
    pad = [g + [0] * (ntok - len(g)) for g in greedy]
    args = (prompts, ntok, K_DRAFT, pad, list(range(nseq)), P_MAIN)
    b.generate_synthetic(*args)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    toks, _, status, _ = b.generate_synthetic(*args)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    assert status == [0] * nseq and toks == greedy
    b.close()
    base.close()


def run_config5(args, rank: int, world: int, local: int) -> None:
    """the 2B-shaped model, k = 3 at p = 0.8 on a 4096-token context, the
    LM head vocab-sharded over the `world` GPUs with the argmax merged by one NCCL all-reduce
    per verify pass (pinfer_b200_shard_head). Every rank runs the same single stream (batch 1;
    the configured batch of 8 sequences needs multi-stream batching, not built), so the total
    work is fixed: strong scaling. value = the stream's tokens / max over ranks of the device
    time of the verify loop."""
    import datetime
    import torch
    sys.path.insert(0, str(ROOT / "oracle"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=900))
    from nibblemac_b200.model import Model
    path = model_path(rank, dist, "2b")
    m = Model(path, max_ctx=CTX5 + N_GEN + 16)
    if world > 1:
        obj = [m.nccl_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        m.shard_head(rank, world, obj[0])
    ctx = np.random.default_rng(4321).integers(0, m.n_vocab, CTX5).astype(np.int32)   # same on every rank
    m.reset()
    m.eval(ctx[:-1], logits=False)
    m.checkpoint()
    greedy, _, st0, _ = m.generate_synthetic_ex(ctx[-1:], N_GEN, 0, np.zeros(N_GEN, np.int32), 0, 0.0,
                                                append=True)
    assert st0 == 0 and len(greedy) == N_GEN

    def step(seed: int):
        m.rewind()
        toks, st, status, ms = m.generate_synthetic_ex(ctx[-1:], N_GEN, K_DRAFT, greedy, seed, P_MAIN,
                                                       append=True)
        assert status == 0 and toks == greedy, "speculative output differs from plain greedy"
        return ms, st

    for i in range(args.warmup):
        step(500 + i)
    if dist is not None:
        dist.barrier()
    ms_all, rounds = [], 0
    for i in range(args.steps):
        ms, st = step(600 + i)
        ms_all.append(ms)
        rounds += st.rounds
    t_dev = sum(ms_all) / 1000.0
    if dist is not None:
        t = torch.tensor([t_dev], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_dev = float(t.item())
    m.close()
    if rank == 0:
        print(json.dumps({
            "metric": "greedy spec-decode tok/s (k=3), 2B shape, LM head vocab-sharded",
            "value": round((N_GEN - 1) * args.steps / t_dev, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_dev * 1000.0 / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "q4k x int8 -> fp32",
            "data": "synthetic (random-init 2B-shaped weights, uniform-random context, synthetic drafter)",
            "config": {"workload": f"configs[4]: Qwen3.5-2B-shaped Q4K, k=3, p={P_MAIN}, {CTX5}-token "
                                   f"context, {N_GEN} generated, batch 1 (of the configured 8)",
                       "head_rows_per_gpu": 248320 // world, "collective": "ncclAllReduce max, 32 x u64 per verify pass" if world > 1 else None,
                       "rounds": rounds}}), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_config5_batch(args, rank: int, world: int, local: int) -> None:
    """configs[4] as configured: the 2B-shaped model, k = 3 at p = 0.8, 8 sequences of
    a 4096-token context each in one multi-sequence batch (pinfer_b200_batch), the LM head
    vocab-sharded over the `world` GPUs: every verify round of the 8 x 4 rows ends with one
    NCCL all-reduce (max) of the per-row argmax keys. The same batch on every rank (the layers
    are replicated), so the total work is fixed: strong scaling. A step is one batch generation
    of N_GEN tokens per sequence; value = 8 x (N_GEN - 1) tokens / the device time of its verify
    rounds (the prompts' prefill is outside it), max over ranks."""
    import datetime
    import torch
    sys.path.insert(0, str(ROOT / "oracle"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=1800))
    from nibblemac_b200.model import Model
    path = model_path(rank, dist, "2b")
    max_ctx = CTX5 + N_GEN + 16
    m = Model(path, max_ctx=max_ctx)
    if world > 1:
        obj = [m.nccl_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        m.shard_head(rank, world, obj[0])
    nseq = args.batch5
    b = m.batch(nseq, max_ctx, max_k=K_DRAFT)
    rng = np.random.default_rng(4321)   # the same contexts on every rank
    prompts = [rng.integers(0, m.n_vocab, CTX5).astype(np.int32) for _ in range(nseq)]
    greedy, _, status, _ = b.generate_synthetic(prompts, N_GEN)
    assert status == [0] * nseq
    pad = [g + [0] * (N_GEN - len(g)) for g in greedy]
    tokens_per_step = sum(len(g) - 1 for g in greedy)

    def step(i: int):
        toks, st, status, ms = b.generate_synthetic(prompts, N_GEN, K_DRAFT, pad,
                                                    [600 + 97 * i + j for j in range(nseq)], P_MAIN)
        assert status == [0] * nseq and toks == greedy, "speculative output differs from plain greedy"
        return ms, st

    for i in range(args.warmup):
        step(i)
    if dist is not None:
        dist.barrier()
    ms_all, rounds = [], 0
    with Clocks(local) as clk:
        for i in range(args.steps):
            ms, st = step(100 + i)
            ms_all.append(ms)
            rounds += b.rounds()
    t_dev = sum(ms_all) / 1000.0
    if dist is not None:
        t = torch.tensor([t_dev], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_dev = float(t.item())
    b.close()
    m.close()
    if rank == 0:
        print(json.dumps({
            "metric": "greedy spec-decode tok/s (k=3), 2B shape, LM head vocab-sharded",
            "value": round(tokens_per_step * args.steps / t_dev, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_dev * 1000.0 / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "q4k x int8 -> fp32",
            "data": "synthetic (random-init 2B-shaped weights, uniform-random contexts, synthetic drafter)",
            "config": {"workload": f"configs[4]: Qwen3.5-2B-shaped Q4K, k=3, p={P_MAIN}, {CTX5}-token "
                                   f"contexts, {N_GEN} generated each, batch {nseq} (multi-sequence batch)",
                       "head_rows_per_gpu": 248320 // world,
                       "collective": (f"ncclAllReduce max of the per-row argmax keys per verify round"
                                      if world > 1 else None),
                       "verify_rounds_per_step": rounds // max(args.steps, 1)},
            "clocks": clk.summary()}), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config4", action="store_true",
                    help="leave the configs[3] multi-stream record out of the default line")
    ap.add_argument("--no-prefill5", action="store_true",
                    help="leave the configs[4] (2B, 4095-token contexts) prefill time and one-GPU batch "
                         "record out of the default line")
    ap.add_argument("--config4", action="store_true",
                    help="configs[3]: 256 requests per GPU in one multi-sequence batch "
                         "(one JSON line)")
    ap.add_argument("--batch5", type=int, default=8,
                    help="sequences of the --config5 batch (1: one context, the earlier form)")
    ap.add_argument("--config5", action="store_true",
                    help="configs[4]: 2B shape, 4096-token context, LM head vocab-sharded "
                         "over the torchrun ranks (one JSON line, strong scaling)")
    ap.add_argument("--profile", action="store_true",
                    help="setup, then exactly one generation inside cudaProfilerStart/Stop (for "
                         "ncu --profile-from-start off); prints nothing else")
    ap.add_argument("--profile-gemm", type=int, default=0, metavar="N",
                    help="the tensor-core GEMM on the config-1 matrix (3584 x 1024) over N activation "
                         "rows through the kernel ABI: prepare once, then 5 launches (for ncu -k)")
    ap.add_argument("--profile-matvec", type=int, nargs=3, default=None, metavar=("ROWS", "COLS", "N"),
                    help="the Q4K x A8 matmul through the kernel ABI on the kbench matrix: 4 launches, "
                         "checked against the oracle (for ncu -k)")
    ap.add_argument("--profile-batch", type=int, nargs=2, default=None, metavar=("SEQS", "TOKENS"),
                    help="config-4 prompts (bench seed) for SEQS sequences: one plain and one warm-up "
                         "batch generation of TOKENS tokens at k = 3, then one inside "
                         "cudaProfilerStart/Stop")
    ap.add_argument("--profile-prefill", nargs=2, default=None, metavar=("PRESET", "TOKENS"),
                    help="one untimed prefill of TOKENS tokens on the PRESET bench model (0.8b, 2b), "
                         "then one inside cudaProfilerStart/Stop")
    args = ap.parse_args()
    if args.profile_prefill:
        run_profile_prefill(args.profile_prefill[0], int(args.profile_prefill[1]))
        return
    if args.profile_gemm:
        run_profile_gemm(args.profile_gemm)
        return
    if args.profile_batch:
        run_profile_batch(*args.profile_batch)
        return
    if args.profile_matvec:
        run_profile_matvec(*args.profile_matvec)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        sys.path.insert(0, str(ROOT / "oracle"))
        run_reference(args, rank, world)
        return
    if args.config5:
        if args.batch5 > 1:
            run_config5_batch(args, rank, world, local)
        else:
            run_config5(args, rank, world, local)
        return
    if args.config4:
        run_config4(args, rank, world, local)
        return

    import torch
    sys.path.insert(0, str(ROOT / "oracle"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    from nibblemac_b200._lib import load_library
    from nibblemac_b200.model import Model
    lib = load_library()
    path = model_path(rank, dist)
    # a batch's contexts cannot be longer than the context whose weights it shares
    m = Model(path, max_ctx=max(CTX + N_GEN + 16, 1024 + GEN4 + 16))
    ctx = context_tokens(rank, m.n_vocab)
    prefill = {"config3": measure_prefill(m, torch, ctx[:-1])}   # leaves the context filled
    dev_blob = m.save_state() if rank == 0 else b""
    m.checkpoint()
    greedy, _, st0, _ = m.generate_synthetic_ex(ctx[-1:], N_GEN, 0, np.zeros(N_GEN, np.int32), 0, 0.0,
                                                append=True)
    assert st0 == 0 and len(greedy) == N_GEN
    kernels_per_round = m.round_kernels(K_DRAFT)

    def step(p: float, seed: int):
        m.rewind()
        t0 = time.perf_counter()
        toks, st, status, ms = m.generate_synthetic_ex(ctx[-1:], N_GEN, K_DRAFT, greedy, seed, p,
                                                       append=True)
        wall = time.perf_counter() - t0
        assert status == 0 and toks == greedy, "speculative output differs from plain greedy"
        return ms, wall, st

    if args.profile:
        step(P_MAIN, 99)
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        ms, wall, st = step(P_MAIN, 100)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"profile_step_ms": ms, "rounds": st.rounds,
                          "kernels_per_round": kernels_per_round}), flush=True)
        m.close()
        return
    for i in range(args.warmup):
        step(P_MAIN, 100 + i)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    dev_ms, walls, rounds = [], [], 0
    with Clocks(local) as clk:
        for i in range(args.steps):
            ms, wall, st = step(P_MAIN, 1000 + i)
            dev_ms.append(ms)
            walls.append(wall)
            rounds += st.rounds
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    t_dev = sum(dev_ms) / 1000.0
    t_wall = sum(walls)
    if dist is not None:
        tt = torch.tensor([t_dev, t_wall], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_dev, t_wall = tt.tolist()
    # the device-timed loop emits N_GEN - 1 tokens (the first comes from the one-token prefill);
    # the end-to-end call produces all N_GEN
    value = (N_GEN - 1) * args.steps * world / t_dev
    e2e = N_GEN * args.steps * world / t_wall

    sweep = {}
    for p in P_SWEEP:
        ms, _, st = step(p, 77)
        sweep[str(p)] = {"tok_s": round((N_GEN - 1) / (ms / 1000.0), 1),
                         "tokens_per_round": round((N_GEN - 1) / st.rounds, 3)}

    # plain greedy decode (no speculation, batch 1) of a 64-token uniform-random
    # prompt, 128 tokens; decode steps timed on the device like the reference's pinfer_run
    # (prefill excluded, N - 1 decode steps)
    p64 = context_tokens(rank + 7, m.n_vocab)[:64]
    c2 = []
    for _ in range(3):
        m.reset()
        _, _, st2, ms2 = m.generate_synthetic_ex(p64, N_GEN, 0, np.zeros(N_GEN, np.int32), 0, 0.0)
        assert st2 == 0
        c2.append(ms2)
    config2 = {"tok_s": round((N_GEN - 1) / (statistics.median(c2) / 1000.0), 1), "prompt": 64,
               "generated": N_GEN, "k": 0, "ms": round(statistics.median(c2), 3)}

    config4 = None if args.no_config4 else measure_config4(m, rank, world, local, dist, True)

    roof = None
    extra = {}
    if rank == 0:
        peak, kind = peaks()
        mv = matvec_roofline(torch, lib, peak)
        rb = round_bytes(path, CTX + N_GEN // 2, K_DRAFT)
        round_s = t_dev / max(rounds, 1)
        roof = {"bound": "hbm", "achieved": round(mv["_achieved"], 1), "peak": peak, "unit": "GB/s",
                "frac": round(mv["_achieved"] / peak, 4), "traffic": traffic_from_profiles(),
                "peak_kind": kind,
                "kernel": "k_mv_slice: q4k x a8 matvec of the out / o / down projections (1024 x 2048 and "
                          "1024 x 3584, n=4 verify rows), timed alone over a rotating arena of weight copies; "
                          "the largest share of a verify round (profiles/verify_round_launches_config3.md)",
                "round": {"bytes": rb, "us": round(round_s * 1e6, 1),
                          "gbs": round(rb / round_s / 1e9, 1), "frac": round(rb / round_s / 1e9 / peak, 4),
                          "what": "algorithmic bytes of one verify round (weights, DeltaNet and conv "
                                  "states read and written, K/V rows read, logs written) / device time "
                                  "per round"}}
        extra["matvec"] = {k: v for k, v in mv.items() if not k.startswith("_")}
    m.close()
    config5 = None
    if rank == 0 and world == 1 and not args.no_prefill5:
        prefill["config5"], config5 = measure_config5(torch, rank, local)
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(t_dev * 1000.0 / args.steps, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "q4k x int8 -> fp32",
                "data": "synthetic (random-init 0.8B-shaped weights, uniform-random context, "
                        "synthetic drafter)",
                "config": bench_config(world),
                "e2e": {"value": round(e2e, 2), "unit": UNIT,
                        "h2d_bytes_per_step": 4 * (1 + N_GEN), "d2h_bytes_per_step": 4 * N_GEN},
                "gpu_launches": int(rounds * kernels_per_round * world),
                "kernels_per_round": kernels_per_round, "rounds": rounds,
                "sweep": sweep, "config2_plain": config2, "roofline": roof, "clocks": clk.summary(),
                "config4": config4, "config5": config5, "prefill": prefill}
        line.update(extra)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample(path, dev_blob, greedy)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
