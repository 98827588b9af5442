"""Benchmark of the decision hot path (BASELINE.json metric: decide requests/s
and prefill tok/s at 1/2/4/8 GPUs, decode GEMV HBM GB/s against peak).

Workload: Llama-16L decoder (d 2048, 32/8 heads, FFN 8192,
V 32000) with Q8_0 weights written from seed; ONE batch of 64 decide
requests of 512 uniform-random token ids sharing one "choose" question over
4 single-token options, sharded by request across the N ranks (contiguous
ranges, balanced by tokens, as laya_decide_batch shards across devices).
One step = one laya_decide_batch call per rank over its share.  Scaling is
strong: value = 64 requests / the slowest rank's time.  At N > 1 the line
also carries the weak figure (64 requests on every rank).  The line's
`decode` object is configs[4] on the same decoder: context 4096, greedy
tokens at batch 1 and 8 per GPU, timed apart from the decide steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Timing: W warm-up steps, then K timed steps between a barrier and a device
synchronize; `value` uses the library's CUDA-event time on its own stream
(inputs already in HBM), `e2e` the wall time of the public call (ids copied
from pinned host memory, answers read back).  The step's working set
(1 GB of weights, 0.5 GB activations per layer) exceeds the 126 MB L2.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from laya_goish_b200 import synth  # noqa: E402

REQUESTS, TOKENS, OPTIONS = 64, 512, 4
CFG = synth.CONFIGS["cfg1"]
WORKLOAD = ("cfg1: Llama-16L (d 2048, 32/8 heads, FFN 8192, V 32000) Q8_0 from seed; one batch of "
            f"{REQUESTS} requests x {TOKENS} tokens sharded across the GPUs, one choose question over {OPTIONS} "
            "single-token options")


# DRAM bytes (read + write) per GEMM launch at the benchmark size: in one ncu
# capture of the 16-request case the layer's four GEMM launches moved
# 1091 MB; every term grows with the token rows, so x4 for 64 requests,
# averaged over the four launches.
GEMM_TRAFFIC_BYTES = 1091e6 * 4 / 4


def gemm_flops_per_token(cfg) -> float:
    """Algorithmic GEMM FLOPs per prompt token: 2 x the layer matrix parameters."""
    return 2.0 * cfg.matrix_params()


def attention_flops(cfg, n) -> float:
    """Causal attention FLOPs of one n-token sequence: 4 * sum_i (i+1) * H * hd * L."""
    return 4.0 * (n * (n + 1) / 2) * cfg.heads * cfg.hd * cfg.layers


def inputs(rank: int, requests: int = REQUESTS):
    rng = np.random.default_rng(1000 + rank)
    prompts = [synth.token_ids(rng, CFG.vocab, TOKENS) for _ in range(requests)]
    cand = synth.candidates(np.random.default_rng(1), CFG.vocab, OPTIONS)
    return prompts, cand


def shard(lengths, world: int, rank: int):
    """Contiguous request range [a, b) of `rank`: cuts placed where the
    running token count crosses rank/world of the total (the split
    laya_decide_batch makes across its devices)."""
    total = float(sum(lengths))
    csum = np.concatenate([[0], np.cumsum(lengths)])

    def cut(r):
        if r <= 0:
            return 0
        if r >= world:
            return len(lengths)
        return int(np.searchsorted(csum, total * r / world, side="left"))

    return cut(rank), cut(rank + 1)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class Clocks:
    """Samples nvidia-smi clocks and throttle reasons every 100 ms.  Started
    before the warm-up; summary() keeps the samples whose timestamps fall in
    the timed window [begin(), end()]."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.p = None
        self.t0 = self.t1 = None
        self.lines = []

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100", "-i", str(self.device)], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        return self

    def begin(self):
        self.t0 = time.time()

    def end(self):
        self.t1 = time.time()

    def stop(self):
        if self.p:
            time.sleep(0.25)
            self.p.terminate()
            try:
                out, _ = self.p.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
                out, _ = self.p.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        import datetime

        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                if self.t0 is not None and not (self.t0 - 0.1 <= ts <= (self.t1 or ts) + 0.1):
                    continue
                sm.append(float(f[2]))
                mx = max(mx, float(f[3]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def reduce_max(values, dist, device):
    """Element-wise max of per-rank timings over all ranks (identity without a process group)."""
    import torch

    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.cpu()]


def throughput(units_per_rank: int, world: int, steps: int, max_ms: float) -> float:
    """Whole-job units per second: every rank's units over the slowest rank's time."""
    return units_per_rank * world * steps / (max_ms / 1000.0)


def cpu_baseline(path: str, prompts, cand, sample_requests: int = 1) -> dict:
    """The oracle (C restatement of the reference CPU engine) on a bounded
    sample of the same workload: `sample_requests` requests, all host threads."""
    import oracle

    threads = os.cpu_count() or 1
    o = oracle.Model(open(path, "rb").read(), threads=threads)
    t0 = time.perf_counter()
    for p in prompts[:sample_requests]:
        o.decide(p, 0, cand.reshape(-1, 1))
    dt = time.perf_counter() - t0
    o.close()
    return {"value": sample_requests / dt, "unit": "req/s", "cores": threads, "kind": "port",
            "sample": f"{sample_requests} of the {REQUESTS} {TOKENS}-token requests, {dt:.1f} s"}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args):
    world, rank, _ = dist_setup(args)
    if rank != 0:
        return  # under torchrun only rank 0 runs the CPU reference
    path = synth.model_path("cfg1")
    prompts, cand = inputs(0)
    import oracle

    threads = os.cpu_count() or 1
    o = oracle.Model(open(path, "rb").read(), threads=threads)
    times = []
    for s in range(args.warmup + args.steps):
        p = prompts[s % len(prompts)]
        t0 = time.perf_counter()
        o.decide(p, 0, cand.reshape(-1, 1))
        if s >= args.warmup:
            times.append(time.perf_counter() - t0)
    o.close()
    total = sum(times)
    value = len(times) / total
    line = {"impl": "reference", "metric": "decide requests/s", "value": value, "unit": "req/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000 * total / len(times), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "step": f"one {TOKENS}-token request (bounded sample of the batch)"},
            "cpu_baseline": {"value": value, "unit": "req/s", "cores": threads, "kind": "port",
                             "sample": f"{len(times)} requests of {TOKENS} tokens, one per step"},
            "e2e": {"value": value, "unit": "req/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def timed_steps(e, prompts, qs, steps, dist):
    """K decide steps between barriers: (device ms, wall ms, launches, h2d, d2h) summed."""
    import torch

    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    dev_ms, wall, launches, h2d, d2h = 0.0, 0.0, 0, 0, 0
    for _ in range(steps):
        t0 = time.perf_counter()
        e.decide_batch(prompts, qs)
        wall += (time.perf_counter() - t0) * 1000.0
        t = e.timing()
        dev_ms += t["device_ms"]
        launches += t["launches"]
        h2d += t["h2d_bytes"]
        d2h += t["d2h_bytes"]
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    return dev_ms, wall, launches, h2d, d2h


def decode_bytes(batch: int, ctx: int, gen: int):
    """Algorithmic HBM bytes of one decode step: the Q8_0 weights incl. the
    lm_head once, plus every sequence's K and V read once (mean context)."""
    qd, kd = CFG.heads * CFG.hd, CFG.kv * CFG.hd
    per_layer = CFG.d * (qd + 2 * kd) + qd * CFG.d + 3 * CFG.d * CFG.ffn
    wbytes = (per_layer * CFG.layers + CFG.vocab * CFG.d) * 34 / 32
    kv_bytes = batch * CFG.layers * 2 * (ctx + gen / 2) * kd * 2
    return wbytes, kv_bytes


def decode_point(e, batch: int, ctx: int, gen: int, dist, device):
    """One decode run: `batch` sequences of `ctx` seeded ids,
    `gen` greedy tokens; device time of steps 1..gen-1 (CUDA events of the
    library), max over ranks."""
    rng = np.random.default_rng(4)
    ctxs = [synth.token_ids(rng, CFG.vocab, ctx) for _ in range(batch)]
    e.decode(ctxs, 4)  # warm-up: packed GEMV images, graph capture, first launches
    if dist:
        dist.barrier()
    _, st = e.decode(ctxs, gen)
    t = e.timing()
    ms, = reduce_max([t["device_ms"] / (gen - 1)], dist, device)
    wbytes, kv_bytes = decode_bytes(batch, ctx, gen)
    pk, pk_kind = peaks()
    gbs = (wbytes + kv_bytes) / (ms / 1000) / 1e9
    return {"batch_per_gpu": batch, "ms_per_token": ms, "tokens_per_s_per_gpu": batch / (ms / 1000),
            "step_gbs": gbs, "step_frac": gbs / pk["hbm_gbs"], "weight_bytes": wbytes, "kv_bytes": kv_bytes,
            "launches_per_step": t["launches"] / (gen - 1)}


def decode_cpu_baseline(path: str, ctx: int, steps: int = 3) -> dict:
    """The oracle on configs[4] at batch 1: a greedy decode step (the
    reference's Matrix::apply with one token row, its single-threaded
    attention over the cached keys, the full-vocabulary head) at context
    `ctx`, all host threads for the matrices.  Bounded sample: the cache is
    filled with arbitrary K/V for the timing (the work per step does not
    depend on the values), then `steps` steps are timed."""
    import oracle

    threads = os.cpu_count() or 1
    o = oracle.Model(open(path, "rb").read(), threads=threads)
    c = o.cache(ctx + steps)
    c.fill_for_timing(ctx)
    tok = 5
    t0 = time.perf_counter()
    for _ in range(steps):
        h = c.forward([tok], [0])
        tok = int(np.argmax(o.head(h)[0]))
    dt = (time.perf_counter() - t0) / steps
    c.close()
    o.close()
    return {"value": 1000 * dt, "unit": "ms/token", "cores": threads, "kind": "port",
            "sample": f"{steps} greedy steps at context {ctx}, batch 1 (cache filled for timing)"}


def run_ours(args):
    world, rank, local = dist_setup(args)
    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    if rank == 0:
        path = synth.model_path("cfg1")
    if dist:
        dist.barrier()
    path = synth.model_path("cfg1")
    from laya_goish_b200 import engine
    from laya_goish_b200.engine import Question

    # one 64-request batch, this rank's contiguous share
    batch, cand = inputs(0, args.requests)
    a, b = shard([len(p) for p in batch], world, rank)
    prompts = batch[a:b]
    qs = [Question("choice", cand)]
    e = engine.Engine(path, devices=[local])
    clk = Clocks(local).start()
    for _ in range(args.warmup):
        e.decide_batch(prompts, qs)
    clk.begin()
    dev_ms, wall, launches, h2d, d2h = timed_steps(e, prompts, qs, args.steps, dist)
    clk.end()
    # Per-kernel CUDA events (roofline, shares) from separate untimed steps:
    # an event between two kernels stops the second from starting early
    # (programmatic dependent launch), so the timed steps run without them.
    psteps = max(1, min(args.steps, 3))
    e.profile(True)
    e.profile_read()
    timed_steps(e, prompts, qs, psteps, dist)
    prof = e.profile_read()
    e.profile(False)
    dev_ms, wall = reduce_max([dev_ms, wall], dist, "cuda")
    value = throughput(args.requests, 1, args.steps, dev_ms)
    e2e = throughput(args.requests, 1, args.steps, wall)
    # roofline of the dominant kernel class on this rank: the tcgen05 GEMMs
    mine = b - a
    gemm_ms = sum(v[1] for k, v in prof.items() if k.startswith("gemm_"))
    gemm_launches = sum(v[0] for k, v in prof.items() if k.startswith("gemm_")) // psteps * args.steps
    gemm_flops = gemm_flops_per_token(CFG) * mine * TOKENS * psteps
    achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms else None
    pk, pk_kind = peaks()
    peak = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
    step_ms = dev_ms / args.steps
    rank_ms = sum(v[1] for v in prof.values())
    shares = {k: round(v[1] / rank_ms, 4) for k, v in sorted(prof.items())} if rank_ms else {}
    line = {
        "metric": "decide requests/s", "value": value, "unit": "req/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": args.requests, "requests_per_gpu": mine,
                   "prompt_tokens": TOKENS, "weights": "Q8_0 (RTN from seeded F16 N(0,0.02))",
                   "compute": "F16 operands, F32 accumulation",
                   "l2": "working set > L2 (weights 1.03 GB, activations 0.5 GB/layer at 64 requests); no flush",
                   "parallelism": f"request sharding x{world} (contiguous ranges balanced by tokens), full replica "
                                  "per GPU, no collective"},
        "prefill_tok_s": value * TOKENS,
        "roofline": {"bound": "tensor", "kernel": "gemm_pair_kernel + gemm_tc_kernel (tcgen05, all prefill GEMMs)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": (achieved / peak) if achieved else None, "traffic": GEMM_TRAFFIC_BYTES,
                     "traffic_unit": "bytes per GEMM launch (ncu DRAM read+write, 16-request capture x 4)",
                     "peak_kind": f"{pk_kind} bf16 dense sustained", "launches": gemm_launches,
                     "share_of_step": round(gemm_ms / rank_ms, 4) if rank_ms else None,
                     "flops_per_step": gemm_flops / psteps, "rank": rank,
                     "timing": f"per-GEMM CUDA events over {psteps} separate profiled steps"},
        "kernel_shares": shares,
        "e2e": {"value": e2e, "unit": "req/s", "h2d_bytes_per_step": h2d // args.steps,
                "d2h_bytes_per_step": d2h // args.steps},
        "gpu_launches": launches,
    }
    if world > 1:
        # weak scaling figure: every rank runs a whole 64-request batch
        own, _ = inputs(1000 + rank, args.requests)
        e.decide_batch(own, qs)
        wsteps = max(1, min(args.steps, 3))
        wms, _, _, _, _ = timed_steps(e, own, qs, wsteps, dist)
        wms, = reduce_max([wms], dist, "cuda")
        line["weak"] = {"value": throughput(args.requests, world, wsteps, wms), "unit": "req/s",
                        "requests_per_gpu": args.requests, "steps": wsteps, "ms_per_step": wms / wsteps}
    clk.stop()
    line["clocks"] = clk.summary()
    if not args.no_decode:
        dec = {"workload": f"configs[4]: the same Q8_0 decoder, context {args.ctx}, {args.gen} greedy tokens, "
                           "one CUDA graph per step; device time of the steps (CUDA events), max over ranks",
               "points": [decode_point(e, bsz, args.ctx, args.gen, dist, "cuda") for bsz in (1, 8)],
               "peak_gbs": pk["hbm_gbs"], "peak_kind": pk_kind}
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            dec["cpu_baseline"] = decode_cpu_baseline(path, args.ctx)
        line["decode"] = dec
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(path, prompts, cand)
    e.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


AUX = {
    # name: (config, requests per GPU, prompt tokens, question builder, description)
    "cfg0": ("cfg0", 1, 256, "check over 2 candidate ids",
             "cfg0: Llama-16L F16 from seed, one 256-token request, one check question over 2 candidates"),
    "cfg0q8": ("cfg1", 1, 256, "check over 2 candidate ids",
               "cfg0's request (one 256-token check over 2 candidates) on the cfg1 Llama-16L Q8_0 decoder: the "
               "layer GEMMs decode the Q8_0 blocks in their shared-memory staging"),
    "cfg2": ("cfg2", 128, 768, "score over 5 criteria x 3-token continuations (full-vocabulary log-softmax)",
             "cfg2: Llama-16L Q4_K_M (attn_v/ffn_down Q6_K) from seed, 128 requests x 768-token shared prefix, "
             "one score question over 5 criteria of 3-token continuations"),
    "cfg3": ("cfg3", 128, 1024, "3 check questions, each a 16-id suffix and 2 candidates",
             "cfg3: Qwen2-28L F16 from seed (d 3584, 28/4 heads, FFN 18944, V 152064, QKV bias), 128 requests "
             "per GPU (1024 over 8 GPUs) x 1024 tokens, 3 check questions with 16-id suffixes"),
}


def aux_questions(name, vocab):
    from laya_goish_b200.engine import Question

    rng = np.random.default_rng(7)
    if name in ("cfg0", "cfg0q8"):
        return [Question("noul", synth.candidates(rng, vocab, 2))], 0
    if name == "cfg2":
        return [Question("score", synth.token_ids(rng, vocab, 15).reshape(5, 3))], 15
    return [Question("noul", synth.candidates(rng, vocab, 2), suffix=synth.token_ids(rng, vocab, 16))
            for _ in range(3)], 48


def aux_cpu_baseline(name, path, prompts, qs) -> dict:
    """The oracle on a bounded sample of an auxiliary configuration, all host
    threads for the matrices and the reference's single-threaded attention.
    cfg0 / cfg2: one whole request (cfg2's 5 continuations branch off its
    768-token prefix, computed once).  cfg3: a 14 TFLOP request is hours of
    CPU work, so one 128-token prefix is timed and scaled to the request's
    1024 + 3 x 16 tokens by its matrix FLOPs (attention grows faster than
    that, so the extrapolated CPU time is a lower bound)."""
    import oracle

    threads = os.cpu_count() or 1
    o = oracle.Model(open(path, "rb").read(), threads=threads)
    t0 = time.perf_counter()
    if name == "cfg3":
        n = 128
        o.forward(prompts[0][:n], [n - 1])
        dt = (time.perf_counter() - t0) * (len(prompts[0]) + 3 * 16) / n
        sample = f"one {n}-token prefix of a cfg3 request, extrapolated by matrix FLOPs to 1024 + 3 x 16 tokens"
    else:
        for q in qs:
            kind, opts, suf = q.arrays()
            o.decide(prompts[0], kind, opts, suf)
        dt = time.perf_counter() - t0
        sample = f"1 request of {len(prompts[0])} tokens, {dt:.1f} s"
    o.close()
    return {"value": 1.0 / dt, "unit": "req/s", "cores": threads, "kind": "port", "sample": sample,
            "extrapolated": name == "cfg3"}


def run_aux(args):
    """The other BASELINE configs on one GPU (auxiliary lines; the contract
    line is the default cfg1 run).  Same timing as run_ours: W warm-up
    steps, K timed steps, CUDA-event device time of the library's stream."""
    import torch

    _, _, local = dist_setup(args)
    torch.cuda.set_device(local)
    from laya_goish_b200 import engine

    cname, requests, tokens, qdesc, desc = AUX[args.workload]
    if args.tokens:
        tokens = args.tokens
        desc += f" (prompt cut to {tokens} tokens)"
    cfg = synth.CONFIGS[cname]
    path = synth.model_path(cname)
    rng = np.random.default_rng(1000)
    prompts = [synth.token_ids(rng, cfg.vocab, tokens) for _ in range(requests)]
    qs, branch_tokens = aux_questions(args.workload, cfg.vocab)
    e = engine.Engine(path, devices=[local])
    clk = Clocks(local).start()
    for _ in range(args.warmup):
        e.decide_batch(prompts, qs)
    torch.cuda.synchronize()
    dev_ms, wall = 0.0, 0.0
    clk.begin()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        e.decide_batch(prompts, qs)
        wall += (time.perf_counter() - t0) * 1000.0
        dev_ms += e.timing()["device_ms"]
    torch.cuda.synchronize()
    clk.end()
    clk.stop()
    # per-kernel events from separate untimed steps (they would stop the
    # timed kernels from starting early behind their predecessors)
    psteps = max(1, min(args.steps, 3))
    e.profile(True)
    e.profile_read()
    prof_ms = 0.0
    for _ in range(psteps):
        e.decide_batch(prompts, qs)
        prof_ms += e.timing()["device_ms"]
    prof = e.profile_read()
    e.close()
    gemm_ms = sum(v[1] for k, v in prof.items() if k.startswith("gemm_") and k != "gemm_head")
    tok = requests * (tokens + branch_tokens)
    gemm_flops = gemm_flops_per_token(cfg) * tok * psteps  # over the profiled steps
    pk, pk_kind = peaks()
    step_ms = dev_ms / args.steps
    wbytes = os.path.getsize(path)  # every weight byte is read at least once per step
    line = {
        "metric": "decide requests/s", "value": requests * args.steps / (dev_ms / 1000.0), "unit": "req/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
        "higher_is_better": True, "dtype": "f16", "data": "synthetic",
        "config": {"workload": desc, "requests": requests, "prompt_tokens": tokens, "questions": qdesc},
        "prefill_tok_s": tok / (step_ms / 1000.0),
        "gemm_tflops": gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms else None,
        "gemm_frac": (gemm_flops / (gemm_ms / 1000.0) / 1e12) / pk["bf16_tflops_sustained"] if gemm_ms else None,
        "weight_stream_frac": (wbytes / (step_ms / 1000.0) / 1e9) / pk["hbm_gbs"],
        "weight_bytes": wbytes,
        "peak_kind": pk_kind,
        "e2e_req_s": requests * args.steps / (wall / 1000.0),
        "kernel_shares": {k: round(v[1] / prof_ms, 4) for k, v in sorted(prof.items())} if prof_ms else {},
        "profiled_ms_per_step": prof_ms / psteps,
        "clocks": clk.summary(),
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = aux_cpu_baseline(args.workload, path, prompts, qs)
    print(json.dumps(line), flush=True)


def run_decode(args):
    """cfg4: KV-cached greedy decode on the cfg1 Q8_0 decoder.  Context of
    `--ctx` seeded ids per sequence, `--gen` generated tokens, `--batch`
    sequences per GPU.  Reports ms per decode step and the HBM GB/s of the
    GEMV launches (Q8_0 weight bytes incl. lm_head per step / GEMV time) and of
    the whole step (weights + KV bytes / step time).  Not the contract line:
    the default invocation measures configs[1]."""
    import torch

    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    from laya_goish_b200 import engine

    path = synth.model_path("cfg1")
    rng = np.random.default_rng(4)
    ctxs = [synth.token_ids(rng, CFG.vocab, args.ctx) for _ in range(args.batch)]
    e = engine.Engine(path, devices=[local])
    e.decode(ctxs[:1], 4)  # warm-up
    clk = Clocks(local).start()
    clk.begin()
    toks, st = e.decode(ctxs, args.gen)
    clk.end()
    clk.stop()
    t = e.timing()
    # per-kernel CUDA events of one step from a separate short decode (events
    # between kernels would stop the timed ones from starting early)
    e.profile(True)
    e.profile_read()
    e.decode(ctxs, 2)
    prof = e.profile_read()
    e.close()
    steps = args.gen - 1
    ms = t["device_ms"] / steps
    qd, kd = CFG.heads * CFG.hd, CFG.kv * CFG.hd
    per_layer = CFG.d * (qd + 2 * kd) + qd * CFG.d + 3 * CFG.d * CFG.ffn
    wbytes = (per_layer * CFG.layers + CFG.vocab * CFG.d) * 34 / 32
    kv_bytes = args.batch * CFG.layers * 2 * (args.ctx + args.gen / 2) * kd * 2
    pk, pk_kind = peaks()
    # the per-kernel profile covers decode step 1 (run outside the graph); later
    # steps replay the same launches as one CUDA graph
    gemv_ms = prof.get("gemv", (0, 0.0))[1]
    out = {"workload": f"cfg4 decode: Llama-16L Q8_0, batch {args.batch}, ctx {args.ctx}, {args.gen} greedy tokens",
           "ms_per_token": ms, "tokens_per_s": args.batch / (ms / 1000),
           "step_gbs": (wbytes + kv_bytes) / (ms / 1000) / 1e9,
           "gemv_gbs": (wbytes / (gemv_ms / 1000) / 1e9) if gemv_ms else None,
           "peak_gbs": pk["hbm_gbs"], "peak_kind": pk_kind,
           "weight_bytes_per_step": wbytes, "kv_bytes_per_step": kv_bytes,
           "prefill_ms": st["prefill_ms"], "kernel_ms_step1": {k: v[1] for k, v in sorted(prof.items()) if not k.startswith("prefill:")},
           "launches_per_step": t["launches"] / steps, "clocks": clk.summary()}
    if out["gemv_gbs"]:
        out["gemv_frac"] = out["gemv_gbs"] / pk["hbm_gbs"]
    out["step_frac"] = out["step_gbs"] / pk["hbm_gbs"]
    if not args.no_cpu_baseline and args.batch == 1:
        out["cpu_baseline"] = decode_cpu_baseline(path, args.ctx)
    print(json.dumps(out), flush=True)


def run_inproc(args):
    """configs[1] through the product's own multi-device sharding: ONE
    process opens the model on GPUs 0..N-1 (the first replica read from the
    file, the others copied over NVLink) and each step is one
    laya_decide_batch over the 64-request batch, which the library splits
    into contiguous token-balanced ranges, one host thread per device.
    value = 64 requests / the step's device time (CUDA events, max over
    devices); e2e = the same over the wall time of the call.  Not the
    contract line (that one runs one process per GPU under torchrun)."""
    import torch

    from laya_goish_b200 import engine
    from laya_goish_b200.engine import Question

    n = max(1, args.gpus)
    if torch.cuda.device_count() < n:
        raise SystemExit(f"--workload inproc needs {n} visible GPUs")
    path = synth.model_path("cfg1")
    batch, cand = inputs(0, args.requests)
    qs = [Question("choice", cand)]
    t0 = time.perf_counter()
    e = engine.Engine(path, devices=list(range(n)))
    open_s = time.perf_counter() - t0
    for _ in range(args.warmup):
        e.decide_batch(batch, qs)
    dev_ms, wall = 0.0, 0.0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        e.decide_batch(batch, qs)
        wall += (time.perf_counter() - t0) * 1000.0
        dev_ms += e.timing()["device_ms"]
    e.close()
    out = {"workload": f"inproc: {WORKLOAD}; one process, Engine(devices=0..{n - 1})", "n_gpus": n,
           "value": args.requests * args.steps / (dev_ms / 1000.0), "unit": "req/s",
           "ms_per_step": dev_ms / args.steps, "e2e_req_s": args.requests * args.steps / (wall / 1000.0),
           "open_s": open_s, "steps": args.steps, "warmup": args.warmup}
    print(json.dumps(out), flush=True)


def run_load(args):
    """Start-up cost: one laya_open of a synthetic GGUF onto GPUs 0..N-1 from
    one process (the C ABI's multi-device model).  The file is opened once
    untimed first, so the page cache holds it and the timed open measures the
    upload path, not the disk.  Not the contract line."""
    import torch

    from laya_goish_b200 import engine

    n = max(1, args.gpus)
    if torch.cuda.device_count() < n:
        raise SystemExit(f"--workload load needs {n} visible GPUs")
    path = synth.model_path(args.load_cfg)
    file_gb = os.path.getsize(path) / 1e9
    engine.Engine(path, devices=[0]).close()  # page cache warm-up
    t0 = time.perf_counter()
    e = engine.Engine(path, devices=list(range(n)))
    dt = time.perf_counter() - t0
    info = e.info
    e.close()
    rep_gb = info["device_bytes"] / 1e9
    out = {"workload": f"load {args.load_cfg} onto {n} GPU(s)", "open_s": dt, "file_gb": file_gb,
           "replica_gb": rep_gb, "replicas_gb_per_s": n * rep_gb / dt,
           "peer_copies": n > 1 and os.environ.get("LAYA_LOAD_PEER", "1") != "0"}
    print(json.dumps(out), flush=True)


def openthai_cpu_baseline(path: str, tokens: int) -> dict:
    """The oracle's OpenThai forward (C mixers and Matrix::apply in the
    reference's loop order, all host threads) on a bounded sample: one pass of
    `tokens` tokens through the same model, timed once after reading the
    weights."""
    import oracle
    from laya_goish_b200 import openthai

    threads = os.cpu_count() or 1
    w = openthai.load_weights(path, strict=False)
    ids = np.random.default_rng(2).integers(0, 4096, tokens)
    t0 = time.perf_counter()
    oracle.ot_forward(w, ids, [tokens - 1], threads=threads)
    dt = time.perf_counter() - t0
    return {"value": tokens / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"one {tokens}-token pass, {dt:.1f} s"}


def run_openthai(args):
    """OpenThai forward on one GPU at the reference's widths (d 1024, FFN
    3584, 24 layers: 18 gated DeltaNet layers of 16 x 128 heads and 6 gated
    attention layers of 8/2 x 256 heads, one in four, a synthetic F16 model
    from seed; vocabulary cut to 4096 rows, which only sizes the embedding
    table).  One step = one `--ot-tokens`-token pass through the host API
    (ids up, three answer rows of slot logits down), so the time includes
    the copies.  Not the contract line."""
    import tempfile

    import torch

    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    from laya_goish_b200 import openthai

    d, ffn, H, KV, hd, nh, hk, L = 1024, 3584, 8, 2, 256, 16, 128, 24
    types = tuple((["linear_attention"] * 3 + ["full_attention"]) * (L // 4))
    s = args.ot_tokens
    with tempfile.TemporaryDirectory() as tmp:
        path = synth.write_openthai(os.path.join(tmp, "openthai.gguf"), d=d, ffn=ffn, vocab=4096, heads=H, kv=KV,
                                    hd=hd, lin_heads=nh, lin_dim=hk, layer_types=types, seed=1, width_scaled=True)
        t0 = time.perf_counter()
        m = openthai.Model(path, device=local, strict=False)
        open_s = time.perf_counter() - t0
        cpu = None if args.no_cpu_baseline else openthai_cpu_baseline(path, args.ot_cpu_tokens)
    ids = np.random.default_rng(2).integers(0, 4096, s)
    pos = [s - 201, s - 101, s - 1] if s > 201 else [s - 1]
    for _ in range(args.warmup):
        m.forward(ids, pos)
    clk = Clocks(local).start()
    clk.begin()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = m.forward(ids, pos)
    ms = (time.perf_counter() - t0) * 1000 / args.steps
    # three permutation passes (an order-invariant choice question) in one
    # forward: the passes' cyclic option orders give sequences of nearly the
    # same length; here three seeded sequences of s tokens
    trio = [(np.random.default_rng(10 + k).integers(0, 4096, s), pos) for k in range(3)]
    for _ in range(args.warmup):
        m.forward_batch(trio)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.forward_batch(trio)
    ms3 = (time.perf_counter() - t0) * 1000 / args.steps
    clk.end()
    clk.stop()
    m.close()
    w = nh * hk
    per_delta = d * (3 * w + w + 2 * nh) + w * d
    per_full = d * (2 * H * hd + 2 * KV * hd) + H * hd * d
    mlp = 3 * d * ffn
    gemm_flops = 2.0 * s * (L * mlp + (3 * L // 4) * per_delta + (L // 4) * per_full) + 2.0 * len(pos) * 256 * d
    out_line = {"workload": f"OpenThai forward: d {d}, FFN {ffn}, {L} layers ({3 * L // 4} DeltaNet {nh}x{hk}, "
                            f"{L // 4} gated attention {H}/{KV}x{hd}), synthetic F16, {s}-token pass, "
                            f"{len(pos)} answer rows",
                "ms_per_pass": ms, "tokens_per_s": s / (ms / 1000), "passes_per_s": 1000 / ms,
                "three_passes_in_one_forward": {"ms": ms3, "ms_per_pass": ms3 / 3,
                                                "note": "laya_openthai_forward_batch of three seeded passes"},
                "gemm_tflops_incl_all_kernels": gemm_flops / (ms / 1000) / 1e12, "open_s": open_s,
                "finite": bool(np.isfinite(out).all()), "timing": "host wall clock around the API call",
                "cpu_baseline": cpu, "clocks": clk.summary()}
    print(json.dumps(out_line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="cfg1", choices=["cfg1", "decode", "cfg0", "cfg0q8", "cfg2", "cfg3", "load", "openthai", "inproc"])
    ap.add_argument("--load-cfg", default="cfg3", help="load: synthetic model to open")
    ap.add_argument("--batch", type=int, default=1, help="decode: sequences per GPU")
    ap.add_argument("--tokens", type=int, default=0, help="cfg0/cfg0q8/cfg2/cfg3: prompt tokens instead of the configured length")
    ap.add_argument("--ctx", type=int, default=4096, help="decode: context tokens")
    ap.add_argument("--gen", type=int, default=128, help="decode: generated tokens")
    ap.add_argument("--ot-tokens", type=int, default=1024, help="openthai: tokens per pass")
    ap.add_argument("--ot-cpu-tokens", type=int, default=128, help="openthai: tokens of the CPU baseline pass")
    ap.add_argument("--requests", type=int, default=REQUESTS,
                    help="requests of the batch (64 is the benchmark; smaller only for profiler captures)")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode object of the cfg1 line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "decode":
        run_decode(args)
    elif args.workload == "load":
        run_load(args)
    elif args.workload == "inproc":
        run_inproc(args)
    elif args.workload == "openthai":
        run_openthai(args)
    elif args.workload in AUX:
        run_aux(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
