"""Benchmark: Llama-3.2-1B-shape Q4_0 decode tok/s and Q4 matvec HBM GB/s on B200.

Workload (the headline configuration): Llama-3.2-1B-shaped model (dim 2048,
16 layers, 32/8 heads, FFN 8192, vocab 128256, tied Q4_0 embedding), random
init N(0, 0.02) from a fixed seed, a 128-token seeded prompt prefilled
untimed, then greedy batch-1 decode with the KV cache growing from position
128 (wrapping back to 128 at position 640, the config's maximum).  A step is
one decode token.  Every step streams all 695 MB of weights, far more than
the 126 MB L2, so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference algorithm on the host cores: the C
restatement in oracle/ (the JavaScript reference cannot run: no JS engine in
this image), on a bounded number of decode tokens.
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

CFG = dict(kind=0, emb_type=2, dim=2048, hidden_dim=8192, n_layers=16, n_heads=32, n_kv_heads=8, head_dim=64,
           vocab=128256, seq_len=2048, rope_theta=500000.0, eps=1e-5)
SEED = 20261201
PROMPT = 128
MAX_POS = 640
METRIC = "Llama-3.2-1B-shape Q4 decode tok/s; Q4 matvec HBM GB/s vs B200 peak"
WORKLOAD = "llama3.2-1B-shape Q4_0 batch-1 greedy decode (configs[3])"


# DRAM bytes over algorithmic bytes of the Q4_0 matvec, from one ncu capture of
# the gate-up launch (dram__bytes_read.sum + dram__bytes_write.sum)
MV_DRAM_OVER_ALG = 18948864 / 18948096


def load_flop_peak():
    """Dense bf16 tensor peak (TFLOP/s): the measured burst figure, else the pool's fallback."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"])
    return 1590.0


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region.
    A reader thread stamps each sample on arrival; entering the block waits
    for the first sample (nvidia-smi takes a while to start), and only the
    samples that arrive between entering and leaving the block are kept."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index, interval_ms=50, cmd=None):
        self.index = index
        self.interval = interval_ms / 1000.0
        self.cmd = cmd or ["nvidia-smi", f"--id={index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                           "-lms", str(interval_ms)]
        self.p = None
        self.stamped = []
        self.lines = []

    def _read(self):
        for line in self.p.stdout:
            if line.strip():
                self.stamped.append((time.monotonic(), line))

    def __enter__(self):
        import threading
        try:
            self.p = subprocess.Popen(self.cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
            return self
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()
        deadline = time.monotonic() + 5.0
        while not self.stamped and time.monotonic() < deadline and self.p.poll() is None:
            time.sleep(0.01)
        self.t0 = time.monotonic()
        return self

    def __exit__(self, *a):
        self.lines = []
        if not self.p:
            return
        t1 = time.monotonic()
        time.sleep(self.interval)  # the sample that covers the end of the region
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
            self.p.wait()
        self.reader.join(timeout=5)
        inside = [l for t, l in self.stamped if self.t0 <= t <= t1 + self.interval]
        self.lines = inside or [l for t, l in self.stamped if t >= self.t0][:1]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def build_model(ctx):
    from purebee_b200.runtime import LlamaConfig, StreamingLlamaRuntime
    c = CFG
    lc = LlamaConfig(dim=c["dim"], hiddenDim=c["hidden_dim"], nLayers=c["n_layers"], nHeads=c["n_heads"],
                     nKvHeads=c["n_kv_heads"], vocabSize=c["vocab"], seqLen=c["seq_len"], headDim=c["head_dim"],
                     ropeTheta=c["rope_theta"], rmsNormEps=c["eps"])
    rt = StreamingLlamaRuntime(lc, ctx=ctx, emb_type=c["emb_type"])
    rt.loadSynthetic(SEED)
    return rt


def prompt_tokens():
    from purebee_b200 import _native as N
    import ctypes
    out = np.zeros(PROMPT, np.int32)
    rc = N.lib().pb_synth_tokens(N.ptr(out), PROMPT, SEED, 1, CFG["vocab"])
    assert rc == 0
    return out.tolist()


def graph_time_us(ctx, torch, stream, launch, reps):
    """Mean device time of one launch: `reps` launches recorded back to back
    in one graph (pb_capture_begin / pb_capture_end), replayed once warm and
    once timed with events on the launching stream (host launch cost
    excluded)."""
    ctx.sync()
    g = ctx.capture(lambda: [launch(i) for i in range(reps)])
    g.launch()  # warm
    ctx.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.launch()
    e1.record(stream)
    e1.synchronize()
    ctx.sync()
    us = e0.elapsed_time(e1) * 1e3 / reps
    g.free()
    return us


def matvec_roofline(ctx, torch, stream, peak, reps=200):
    """Per-launch device time of the Q4_0 matvec kernel on the decode shapes
    and the config-2 shapes: `reps` launches back to back in one CUDA graph,
    each on a different weight copy, the copies together > 4x L2 so HBM is
    measured rather than L2."""
    from purebee_b200 import _native as N
    L = N.lib()
    shapes = {"qkv 3072x2048": (3072, 2048), "o 2048x2048": (2048, 2048), "gate|up 16384x2048": (16384, 2048),
              "down 2048x8192": (2048, 8192), "kv 512x2048": (512, 2048), "ffn 8192x2048": (8192, 2048),
              "vocab 128256x2048": (128256, 2048)}
    per_token_launches = {"qkv 3072x2048": 16, "o 2048x2048": 16, "gate|up 16384x2048": 16, "down 2048x8192": 16}
    rng = np.random.default_rng(7)
    res = {}
    tot_b, tot_t = 0.0, 0.0
    for name, (n, k) in shapes.items():
        nbytes = n * k // 32 * 18
        copies = max(2, int(np.ceil(4 * 126e6 / nbytes)))
        r = min(reps, max(20, copies * 2)) if n > 100000 else reps
        raw = rng.integers(0, 256, n * (k // 32) * 18, dtype=np.uint8)
        raw.reshape(-1, 18)[:, :2] = (rng.standard_normal(n * (k // 32)) * 0.01).astype(np.float16).view(
            np.uint8).reshape(-1, 2)
        mats = [N.QMat(ctx, N.TYPE_Q4_0, raw, n, k) for _ in range(copies)]
        x = ctx.to_device(rng.standard_normal(k).astype(np.float32))
        y = ctx.alloc(n * 4)
        us = graph_time_us(ctx, torch, stream,
                           lambda i: ctx._check(L.pb_qmat_matvec(ctx.h, mats[i % copies].h, x.ptr, y.ptr, 0, 0)), r)
        alg = nbytes + k * 4 + n * 4
        gbs = alg / (us * 1e-6) / 1e9
        res[name] = {"us": round(us, 3), "GBps": round(gbs, 1), "frac": round(gbs / peak, 3), "bytes": alg,
                     "copies": copies}
        if name in per_token_launches:
            tot_b += alg * per_token_launches[name]
            tot_t += us * 1e-6 * per_token_launches[name]
        for m in mats:
            m.free()
    return res, tot_b / tot_t / 1e9, tot_b / sum(per_token_launches.values())


def row_split_vocab(ctx, torch, dist, world, peak, reps=40):
    """Config 2's vocab-head matvec (128256 x 2048 Q4_0) split by rows over the
    ranks (thread-pool.js's row split, one GPU per worker) with the library's
    NCCL all-gather of the y slices (pb_comm_allgather).  Each rank rotates
    over weight copies larger than 4x L2 in total.  Times are device event
    times on the library stream, max over ranks."""
    from purebee_b200 import _native as N
    from purebee_b200.thread_pool import NcclComm, RowSplitMatvec, rows_per_rank
    n, k = 128256, 2048
    rng = np.random.default_rng(11)
    raw = rng.integers(0, 256, n * (k // 32) * 18, dtype=np.uint8)
    raw.reshape(-1, 18)[:, :2] = (rng.standard_normal(n * (k // 32)) * 0.01).astype(np.float16).view(
        np.uint8).reshape(-1, 2)
    per = rows_per_rank(n, world)
    slice_bytes = per * (k // 32) * 18
    copies = max(2, int(np.ceil(4 * 126e6 / slice_bytes)))
    comm = NcclComm.from_torch(ctx)
    mats = [RowSplitMatvec(ctx, raw, N.TYPE_Q4_0, n, k, comm) for _ in range(copies)]
    dev = torch.device("cuda", ctx.device)
    x = ctx.to_device(rng.standard_normal(k).astype(np.float32))
    stream = torch.cuda.ExternalStream(N.lib().pb_stream(ctx.h), device=dev)

    def timed(fn):
        for i in range(3):
            fn(i)
        ctx.sync()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(reps):
            fn(i)
        e1.record(stream)
        e1.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / reps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    local_us = timed(lambda i: mats[i % copies].local(x.ptr))
    full_us = timed(lambda i: mats[i % copies].matvec(x.ptr))
    ctx.sync()
    for m in mats:
        m.free()
    comm.free()
    alg = n * k // 32 * 18 + 4 * k + 4 * n
    return {"shape": "128256x2048 Q4_0 (vocab head)", "gpus": world, "rows_per_gpu": per, "copies_per_gpu": copies,
            "local_us": round(local_us, 3),
            "local_GBps_per_gpu": round((slice_bytes + 4 * k + 4 * per) / (local_us * 1e-6) / 1e9, 1),
            "aggregate_GBps_local": round(alg / (local_us * 1e-6) / 1e9, 1),
            "with_allgather_us": round(full_us, 3),
            "aggregate_GBps_with_allgather": round(alg / (full_us * 1e-6) / 1e9, 1),
            "frac_local_of_measured_peak_per_gpu": round((slice_bytes + 4 * k + 4 * per) / (local_us * 1e-6) / 1e9 / peak, 3),
            "allgather": "pb_comm_allgather (NCCL, library stream)"}


def run_batched(ctx, torch, stream, rt, peak, flop_peak, n_seqs=64, n_prompt=512, steps=256, dist=None, warm=2,
                clk=None, e2e=False):
    """n_seqs seeded prompts of n_prompt tokens prefilled as one
    batch (tensor-core GEMMs), then `steps` greedy decode steps of every
    sequence (one replayed graph per step).  With N ranks the model is row
    split over the N GPUs (pb_batch_create_split: each GPU holds 1/N of every
    projection, of the head and of the KV cache; NCCL all-gathers inside the
    step), so the work is fixed and the time falls with N (strong scaling).
    Device event times, max over ranks; the linear-layer FLOPs of the prefill
    give its tensor roofline against N GPUs' peak."""
    from purebee_b200.runtime import BatchedLlamaRuntime
    from purebee_b200.thread_pool import NcclComm
    c = CFG
    world = dist.get_world_size() if dist else 1
    rng = np.random.default_rng(SEED + 5)
    prompts = rng.integers(1, c["vocab"], (n_seqs, n_prompt)).astype(np.int32)
    comm = NcclComm.from_torch(ctx) if world > 1 else None
    comm_p2p = bool(comm is not None and comm.peer_access)
    bt = BatchedLlamaRuntime(rt, n_seqs, comm=comm)
    dev = torch.device("cuda", ctx.device) if hasattr(ctx, "device") else torch.device("cuda")

    def max_over_ranks(ms):
        if not dist:
            return ms
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    bt.prefill(prompts)  # warm, at full size: activation buffers, GEMM scratch, kernels
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    ctx.sync()
    if dist:
        dist.barrier()
    e0.record(stream)
    bt.prefill(prompts)
    e1.record(stream)
    e1.synchronize()
    prefill_ms = max_over_ranks(e0.elapsed_time(e1))
    l0 = ctx.launches
    bt.decode(1)  # records the decode graph (its launches are counted once, here)
    launches_per_step = ctx.launches - l0
    if warm > 1:
        bt.decode(warm - 1)
    ctx.sync()
    if dist:
        dist.barrier()
    from contextlib import nullcontext
    with clk if clk is not None else nullcontext():
        e1.record(stream)
        toks = bt.decode(steps)
        e2.record(stream)
        e2.synchronize()
    decode_ms = max_over_ranks(e1.elapsed_time(e2))
    e2e_line = None
    if e2e:
        # through the public calls with host buffers: the seeded prompts in,
        # `steps` greedy steps with every step's tokens copied out
        ctx.sync()
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        bt.prefill(prompts)
        bt.decode(steps)
        wall = time.perf_counter() - t0
        if dist:
            t = torch.tensor([wall], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            wall = float(t.item())
        e2e_line = {"value": round(n_seqs * steps / wall, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": int(prompts.nbytes // steps), "d2h_bytes_per_step": 4 * n_seqs,
                    "api": "BatchedLlamaRuntime.prefill (host prompts) + decode (tokens to the host every step), "
                           "wall clock, generated tokens / s"}
    bt.free()  # before the communicator: the decode graph holds its NCCL work
    if comm is not None:
        comm.free()
    d, F, L, V, kv = c["dim"], c["hidden_dim"], c["n_layers"], c["vocab"], c["n_kv_heads"] * c["head_dim"]
    lin_params = L * ((d + 2 * kv) * d + d * d + 2 * F * d + d * F)
    tokens = n_seqs * n_prompt
    lin_flops = 2.0 * lin_params * tokens + 2.0 * V * d * n_seqs
    # decode step bytes: weights once + every sequence's K and V rows at the mean position
    mid = n_prompt + 2 + steps // 2
    step_bytes = lin_params * 18 / 32 + V * d * 18 / 32 + 2.0 * L * n_seqs * mid * kv * 4
    dec_s = decode_ms / 1e3 / steps
    hd_bytes = n_seqs * d * 4
    gathered = c["n_layers"] * (3 * hd_bytes + n_seqs * F * 4) + n_seqs * 8  # per step, whole buffers
    return {"workload": f"configs[4]: {n_seqs} seqs x {n_prompt}-token seeded prompts, then {steps} greedy steps",
            "n_gpus": world, "scaling": "strong",
            "parallelism": (f"rowsplit{world}: " + (
                f"{2 * c['n_layers'] + 1} exchange kernels per decode step over NVLink peer memory (low-latency "
                f"exchange) and {2 * c['n_layers']} residual exchanges fused into the add epilogues and the next "
                f"norms" if comm_p2p else f"{4 * c['n_layers'] + 1} NCCL all-gathers per decode step"))
            if world > 1 else "single-gpu",
            "prefill_ms": round(prefill_ms, 2), "prefill_tok_s": round(tokens / (prefill_ms / 1e3), 1),
            "prefill_linear_TFLOPs": round(lin_flops / (prefill_ms / 1e3) / 1e12, 1),
            "prefill_frac_of_bf16_peak": round(lin_flops / (prefill_ms / 1e3) / 1e12 / (world * flop_peak), 3),
            # the three-term products issue three f16 MMAs per algorithmic one
            "prefill_tensor_TFLOPs_issued": round(3 * lin_flops / (prefill_ms / 1e3) / 1e12, 1),
            "prefill_issued_frac_of_bf16_peak": round(3 * lin_flops / (prefill_ms / 1e3) / 1e12 / (world * flop_peak),
                                                      3),
            "decode_ms_per_step": round(decode_ms / steps, 3),
            "decode_tok_s": round(n_seqs / dec_s, 1),
            "decode_step_bytes": int(step_bytes),
            "decode_frac_of_hbm": round(step_bytes / dec_s / 1e9 / (world * peak), 3),
            "decode_allgather_bytes_per_step": int(gathered) if world > 1 else 0,
            "tokens_sample": toks[-1][:4].tolist(),
            "decode_launches_per_step": int(launches_per_step),
            "e2e": e2e_line,
            "arithmetic": "three-term: every operand as an f16 hi/lo pair, hi*hi + hi*lo + lo*hi with f32 "
                          "accumulation -- projections and head on tcgen05, prefill attention on mma.sync; logits "
                          "within 1e-4 of the one-sequence path at this shape"}


def run_split(args, rank, world, torch, dist):
    """N > 1: the batched configuration row-split over the N GPUs
    (north_star: batch-1 decode is a one-GPU figure, the batched config is the
    one reported at 1/2/4/8 GPUs).  A step is one batched decode step of all
    64 sequences; W warm-up and K timed steps after the 512-token prefill,
    device event time, max over ranks; the work is fixed, so the scaling is
    strong.  Rank 0 first times the same workload on its GPU alone, the
    one-GPU reference the speed-up is read against.  Config 2's vocab-head
    row split is reported alongside."""
    from purebee_b200 import _native as N
    dev = int(os.environ.get("LOCAL_RANK", 0))
    ctx = N.Context(dev)
    ctx.set_timeout_ms(120000)
    torch.cuda.set_device(dev)
    stream = torch.cuda.ExternalStream(N.lib().pb_stream(ctx.h), device=dev)
    peak, peak_kind = load_peaks()
    flop_peak = load_flop_peak()
    rt = build_model(ctx)
    one = None
    if rank == 0:
        one = run_batched(ctx, torch, stream, rt, peak, flop_peak, steps=args.steps, warm=args.warmup, dist=None)
    dist.barrier()
    clk = ClockSampler(dev)
    sp = run_batched(ctx, torch, stream, rt, peak, flop_peak, steps=args.steps, warm=args.warmup, dist=dist, clk=clk,
                     e2e=True)
    split = row_split_vocab(ctx, torch, dist, world, peak)
    result = None
    if rank == 0:
        n_seqs = 64
        result = {
            "metric": METRIC,
            "value": sp["decode_tok_s"],
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": sp["decode_ms_per_step"],
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "u4 weights; f16 tensor-core operands, f32 accumulation",
            "data": "synthetic (seeded N(0,0.02) weights, seeded prompt tokens)",
            "config": {"workload": "llama3.2-1B-shape Q4_0 batched serving, 64 seqs x 512-token prompts, greedy "
                                   "decode steps (configs[4])", "model": "llama3.2-1B-shape", "global_batch": n_seqs,
                       "seq_len": 2048, "prompt": 512, "parallelism": f"rowsplit{world}",
                       "rope_scaling": "off (the reference applies none)",
                       "l2": "a decode step reads the weights once plus every sequence's KV (> 126 MB L2)"},
            "one_gpu_same_workload": {"decode_tok_s": one["decode_tok_s"], "decode_ms_per_step":
                                      one["decode_ms_per_step"], "prefill_ms": one["prefill_ms"]},
            "batched": sp,
            "roofline": {"bound": "hbm", "kernel": "the batched decode step (every kernel; weights / N and the "
                                                  "rank's KV per GPU)",
                         "achieved": round(sp["decode_step_bytes"] / (sp["decode_ms_per_step"] / 1e3) / 1e9 / world, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": sp["decode_frac_of_hbm"],
                         "traffic": None},
            "row_split": split,
            "gpu_launches": sp["decode_launches_per_step"] * args.steps,
            "clocks": clk.summary(),
            "e2e": sp["e2e"],
        }
    rt.shutdown()
    ctx.close()
    return result


def run_ours(args, rank, world, torch, dist):
    from purebee_b200 import _native as N
    dev = int(os.environ.get("LOCAL_RANK", 0))
    ctx = N.Context(dev)
    ctx.set_timeout_ms(120000)
    torch.cuda.set_device(dev)
    stream = torch.cuda.ExternalStream(N.lib().pb_stream(ctx.h), device=dev)
    peak, peak_kind = load_peaks()
    rt = build_model(ctx)
    m = rt.model
    prompt = prompt_tokens()
    # prefill (untimed), leaves the first greedy token on the device
    rt.forward(prompt, 0)

    def device_steps(pos, n):
        """n graph replays starting at pos; wraps at MAX_POS."""
        while n > 0:
            room = MAX_POS - pos
            if room <= 0:
                pos = PROMPT
                room = MAX_POS - pos
            k = min(n, room)
            ctx._check(N.lib().pb_model_decode_loop(m.h, pos, k, None))
            pos += k
            n -= k
        return pos

    pos = device_steps(PROMPT, args.warmup)
    ctx.sync()
    launches_per_step = int(N.lib().pb_model_decode_launches(m.h))
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ctx.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        e0.record(stream)
        pos_end = device_steps(pos, args.steps)
        e1.record(stream)
        e1.synchronize()
    ctx.sync()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device=f"cuda:{dev}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    clocks = clk.summary()
    # the whole configs[3] decode window (positions 128 -> 640, one pass) and
    # the step time around three positions of it
    def window_ms(p0, n):
        ctx.sync()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        ctx._check(N.lib().pb_model_decode_loop(m.h, p0, n, None))
        b.record(stream)
        b.synchronize()
        return a.elapsed_time(b)
    full_ms = window_ms(PROMPT, MAX_POS - PROMPT)
    by_pos = {str(p): round(window_ms(p, 8) / 8, 4) for p in (PROMPT, 384, MAX_POS - 8)}
    # algorithmic bytes per token at the mean position of the timed steps
    mid = min(pos + args.steps // 2, MAX_POS - 1)
    step_bytes = int(N.lib().pb_model_decode_bytes(m.h, mid))

    # ---- e2e through the public API: H2D token+pos, graph, D2H next token ----
    e2e_steps = min(args.steps, 64)
    rt.resetCache()
    rt.forward(prompt, 0)
    nxt, _ = m.decode(1, PROMPT)  # warm the host path
    p = PROMPT + 1
    tok = nxt
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        if p >= MAX_POS:
            p = PROMPT
        tok, _ = m.decode(tok, p)
        p += 1
    e2e_s = time.perf_counter() - t0
    e2e_tps = e2e_steps / e2e_s
    if dist:
        t = torch.tensor([e2e_s], device=f"cuda:{dev}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_tps = e2e_steps / float(t.item())

    split = row_split_vocab(ctx, torch, dist, world, peak) if dist else None
    batched = None
    if not args.no_batched:
        rt.resetCache()
        batched = run_batched(ctx, torch, stream, rt, peak, load_flop_peak(), dist=dist)

    result = None
    if rank == 0:
        mv, mv_agg, mv_bytes_avg = matvec_roofline(ctx, torch, stream, peak)
        total_tokens = args.steps * world
        value = total_tokens / (ms / 1e3)
        step_gbs = step_bytes / (ms / 1e3 / args.steps) / 1e9
        result = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "u4 weights, f32 math (f64 for the reference's double ops)",
            "data": "synthetic (seeded N(0,0.02) weights, seeded prompt tokens)",
            "config": config_line(world),
            "decode_step": {"bytes": step_bytes, "GBps": round(step_gbs, 1), "frac_of_hbm": round(step_gbs / peak, 3),
                            "launches": launches_per_step, "ms_by_position": by_pos,
                            "full_window": {"positions": f"{PROMPT}-{MAX_POS - 1}", "steps": MAX_POS - PROMPT,
                                            "ms": round(full_ms, 3),
                                            "tok_s": round((MAX_POS - PROMPT) / (full_ms / 1e3), 2)}},
            "roofline": {"bound": "hbm", "kernel": "k_mvf (Q4_0, fast decode matvec)",
                         "achieved": round(mv_agg, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(mv_agg / peak, 3),
                         "traffic": int(round(mv_bytes_avg * MV_DRAM_OVER_ALG)),
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one gate-up launch "
                                           f"(16384x2048), as a ratio to its algorithmic bytes ({MV_DRAM_OVER_ALG:.6f}) "
                                           "times the bytes per launch",
                         "bytes_per_launch": int(mv_bytes_avg), "per_shape": mv},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "e2e": {"value": round(e2e_tps * world, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": 4, "steps": e2e_steps,
                    "api": "StreamingLlamaRuntime model.decode (pb_model_decode)"},
        }
        if split:
            result["row_split"] = split
        if batched:
            result["batched"] = batched
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline(rt, prompt)
    rt.shutdown()
    ctx.close()
    return result


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    return O


def oracle_prompt(O):
    """The same seeded prompt as prompt_tokens() (one shared generator, pb_synth.h)."""
    return O.synth_tokens(PROMPT, SEED, 1, CFG["vocab"]).tolist()


def config_line(world):
    return {"workload": WORKLOAD, "model": "llama3.2-1B-shape", "global_batch": world, "seq_len": MAX_POS,
            "prompt": PROMPT, "parallelism": f"replicas{world}" if world > 1 else "single-gpu",
            "rope_scaling": "off (the reference applies none)",
            "l2": "weights 695 MB per step > 126 MB L2 (no flush needed)"}


def cpu_baseline(rt, prompt, sample_tokens=32):
    """The oracle (C restatement of the reference's decode, thread-pool.js row
    split over every host thread) on the same model and the same workload
    position: the device prefills the prompt, its weights and KV cache are
    copied into the oracle, and `sample_tokens` greedy decode tokens from
    position PROMPT are timed."""
    O = _oracle()
    rt.resetCache()
    tok = O.argmax(rt.forward(prompt, 0)["logits"])
    om = O.Model(O.Config(**CFG))
    for w in range(8):
        for l in (range(CFG["n_layers"]) if w else [0]):
            om.tensor(l, w)[:] = rt.getTensor(l, w)
    om.refresh()
    for l in range(CFG["n_layers"]):
        for v in (0, 1):
            om.kv(l, v)[:PROMPT] = rt.model.kv(l, v)[:PROMPT]
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    t0 = time.perf_counter()
    pos = PROMPT
    for _ in range(sample_tokens):
        tok = O.argmax(om.forward([tok], pos))
        pos += 1
    dt = time.perf_counter() - t0
    return {"value": round(sample_tokens / dt, 4), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{sample_tokens} greedy decode tokens at positions {PROMPT}-{PROMPT + sample_tokens - 1} after "
                      f"the same {PROMPT}-token prompt, same weights (oracle/pb_oracle.c: WASM-order Q4 matvecs, "
                      f"batch_dot head, double attention; {threads} threads row split as thread-pool.js)"}


def run_reference(args):
    """The reference algorithm on the host cores, on the same workload as the
    GPU arm: the oracle (C restatement; the JavaScript reference has no engine
    in this image) builds the same seeded weights with its own generator
    (bit-identical to the device's), prefills the same 128-token prompt
    (untimed), then decodes W warm-up and K timed greedy tokens from position
    128, wrapping at 640 like the GPU arm.  Nothing of the product is loaded."""
    O = _oracle()
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    om = O.Model(O.Config(**CFG))
    om.init_synthetic(SEED)
    prompt = oracle_prompt(O)
    tok = O.argmax(om.forward(prompt, 0))
    pos = PROMPT

    def step(tok, pos):
        if pos >= MAX_POS:
            pos = PROMPT
        return O.argmax(om.forward([tok], pos)), pos + 1

    for _ in range(args.warmup):
        tok, pos = step(tok, pos)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok, pos = step(tok, pos)
    dt = time.perf_counter() - t0
    v = args.steps / dt
    return {"metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": 0, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (reference lane order), f64 reductions",
            "data": "synthetic (seeded N(0,0.02) weights, seeded prompt tokens)", "impl": "reference",
            "config": config_line(1),
            "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} greedy decode tokens from position {PROMPT} after the same "
                                       f"{PROMPT}-token prompt (oracle/pb_oracle.c, {threads} threads; the "
                                       f"JavaScript reference has no engine in this image)"},
            "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_exchange_case(args):
    """`--case exchange:BYTES` under torchrun: the row split's exchange step
    alone, an in-place all-gather of BYTES per rank over a registered buffer
    (pb_comm_allgather_inplace: the peer-memory kernel when the ranks have
    peer access, else NCCL).  W untimed calls, then K back to back on the
    context stream, timed with CUDA events; rank 0 prints the max over ranks
    in microseconds per exchange."""
    import ctypes
    import torch
    import torch.distributed as td
    from datetime import timedelta
    from purebee_b200 import _native as N
    from purebee_b200.thread_pool import NcclComm
    nbytes = int(args.case.split(":", 1)[1])
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    td.init_process_group("gloo", timeout=timedelta(seconds=120))
    ctx = N.Context(local)
    stream = torch.cuda.ExternalStream(N.lib().pb_stream(ctx.h), device=local)
    comm = NcclComm.from_torch(ctx)
    buf = ctx.alloc(nbytes * world)
    pb = ctypes.c_void_p()
    ctx._check(N.lib().pb_comm_register(comm.h, buf.ptr, ctypes.byref(pb)))
    call = lambda: ctx._check(N.lib().pb_comm_allgather_inplace(comm.h, pb.value, nbytes))
    for _ in range(args.warmup):
        call()
    ctx.sync()
    td.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        call()
    b.record(stream)
    b.synchronize()
    us = torch.tensor([a.elapsed_time(b) * 1e3 / args.steps])
    td.all_reduce(us, op=td.ReduceOp.MAX)
    if rank == 0:
        print(json.dumps({"case": args.case, "n_gpus": world, "us_per_exchange": round(float(us[0]), 3),
                          "bytes_per_rank": nbytes, "transport": "peer memory" if comm.peer_access else "NCCL",
                          "steps": args.steps}), flush=True)
    ctx._check(N.lib().pb_comm_deregister(comm.h, pb.value))
    comm.free()
    td.barrier()
    td.destroy_process_group()
    ctx.close()


def run_case(args):
    """One kernel on a small case, for profiler captures: `--case matvec:NxK`
    runs the Q4_0 matvec on one seeded N x K matrix (W plain launches, then K
    launches in one CUDA graph, replayed twice); `--case head:VxD` the Q4_0 LM
    head with argmax.  Prints the mean device time per launch."""
    import torch
    from purebee_b200 import _native as N
    L = N.lib()
    kind, shape = args.case.split(":", 1)
    if kind == "exchange":
        run_exchange_case(args)
        return
    if kind == "batched":  # batched:BxP -> one batched prefill of B x P seeded tokens, 3 decode steps
        from purebee_b200 import _native as N
        from purebee_b200.runtime import BatchedLlamaRuntime
        nb_, np_ = (int(v) for v in shape.lower().split("x"))
        ctx = N.Context(0)
        rt = build_model(ctx)
        bt = BatchedLlamaRuntime(rt, nb_)
        bt.prefill(np.random.default_rng(1).integers(1, CFG["vocab"], (nb_, np_)).astype(np.int32))
        bt.decode(3)
        ctx.sync()
        print(json.dumps({"case": args.case, "ok": True}), flush=True)
        bt.free()
        rt.shutdown()
        ctx.close()
        return
    if kind == "decode":  # decode:N[@POS] -> N decode steps of the headline model from POS (default 128)
        import torch
        from purebee_b200 import _native as N
        steps, _, pos0 = shape.partition("@")
        steps, pos0 = int(steps), int(pos0 or PROMPT)
        ctx = N.Context(0)
        torch.cuda.set_device(0)
        stream = torch.cuda.ExternalStream(N.lib().pb_stream(ctx.h), device=0)
        rt = build_model(ctx)
        rt.forward(prompt_tokens(), 0)
        ctx._check(N.lib().pb_model_decode_loop(rt.model.h, PROMPT, args.warmup, None))
        ctx.sync()
        torch.cuda.profiler.start()  # ncu --profile-from-start off captures these steps only
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        ctx._check(N.lib().pb_model_decode_loop(rt.model.h, pos0, steps, None))
        b.record(stream)
        b.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"case": args.case, "ms_per_step": round(a.elapsed_time(b) / steps, 4),
                          "launches_per_step": int(N.lib().pb_model_decode_launches(rt.model.h))}), flush=True)
        rt.shutdown()
        ctx.close()
        return
    mtok = 1
    if kind in ("gemm", "gemm3", "gemmhl"):  # gemm / gemm3:MxNxK (f32 activations, one / three terms), gemmhl:MxNxK
        mtok, n, k = (int(v) for v in shape.lower().split("x"))
    else:
        n, k = (int(v) for v in shape.lower().split("x"))
    ctx = N.Context(0)
    torch.cuda.set_device(0)
    stream = torch.cuda.ExternalStream(L.pb_stream(ctx.h), device=0)
    rng = np.random.default_rng(7)
    raw = rng.integers(0, 256, n * (k // 32) * 18, dtype=np.uint8)
    raw.reshape(-1, 18)[:, :2] = (rng.standard_normal(n * (k // 32)) * 0.01).astype(np.float16).view(
        np.uint8).reshape(-1, 2)
    m = N.QMat(ctx, N.TYPE_Q4_0 | (N.QMAT_TABLE if kind == "head" else 0), raw, n, k)
    x = ctx.to_device(rng.standard_normal(k).astype(np.float32))
    y = ctx.alloc(n * 4)
    idx = ctx.alloc(16)
    if kind == "gemm":
        X = ctx.to_device(rng.standard_normal((mtok, k)).astype(np.float32))
        Cb = ctx.alloc(mtok * n * 4)
        call = lambda: ctx._check(L.pb_q4_gemm(ctx.h, m.h, X.ptr, mtok, k, Cb.ptr, n))
    elif kind == "gemm3":  # the three-term product (M >= 512: hi/lo copies and the persistent TMA kernel)
        X = ctx.to_device(rng.standard_normal((mtok, k)).astype(np.float32))
        Cb = ctx.alloc(mtok * n * 4)
        call = lambda: ctx._check(L.pb_q4_gemm_ex(ctx.h, m.h, X.ptr, mtok, k, Cb.ptr, n, 3))
    elif kind == "gemmhl":  # the batched decode GEMM's three-term form (M <= 64: the warp-specialised kernel)
        Xf = rng.standard_normal((mtok, k)).astype(np.float32)
        hi = Xf.astype(np.float16)
        lo = (Xf - hi.astype(np.float32)).astype(np.float16)
        Xhl = np.stack([hi.reshape(mtok, k // 64, 64), lo.reshape(mtok, k // 64, 64)], axis=2).reshape(mtok, 2 * k)
        X = ctx.to_device(np.ascontiguousarray(Xhl))
        Cb = ctx.alloc(mtok * n * 4)
        call = lambda: ctx._check(L.pb_q4_gemm_hl(ctx.h, m.h, X.ptr, mtok, Cb.ptr, n))
    elif kind == "matvec":
        call = lambda: ctx._check(L.pb_qmat_matvec(ctx.h, m.h, x.ptr, y.ptr, 0, 0))
    elif kind == "head":
        call = lambda: ctx._check(L.pb_qmat_head(ctx.h, m.h, x.ptr, y.ptr, idx.ptr))
    else:
        raise SystemExit(f"unknown case {kind}")
    for _ in range(args.warmup):
        call()
    us = graph_time_us(ctx, torch, stream, lambda i: call(), args.steps)
    line = {"case": args.case, "us_per_launch": round(us, 3), "bytes": int(raw.nbytes)}
    if kind in ("gemm", "gemm3", "gemmhl"):
        line["TFLOPs"] = round(2.0 * mtok * n * k / (us * 1e-6) / 1e12, 1)
    print(json.dumps(line), flush=True)
    m.free()
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="skip the batched configuration (configs[4])")
    ap.add_argument("--case", default=None, help="profile one kernel: matvec:NxK, head:VxD, gemm:MxNxK, gemm3:MxNxK, gemmhl:MxNxK, batched:BxP "
                                                 "(batched prefill + 3 steps), decode:N[@POS] (N decode steps), or exchange:BYTES "
                                                 "(under torchrun: in-place all-gathers of BYTES per rank)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.case:
        run_case(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return
    import torch
    dist = None
    if world > 1:
        import torch.distributed as td
        from datetime import timedelta
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        td.init_process_group("nccl", timeout=timedelta(seconds=180),
                              device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))))
        dist = td
    res = run_split(args, rank, world, torch, dist) if world > 1 else run_ours(args, rank, world, torch, dist)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
