"""Benchmark: MX-int4 7B-MLP linear pair (up 4096->11008, down 11008->4096),
the reference's MX qlinear hot path, on B200.

One step = one token batch through quantise(x) -> up GEMV -> requantise ->
down GEMV (fp32 in, fp32 out).  The headline is batch 1 (decode); batches 8,
64 and 512 (GEMV -> tensor-core GEMM crossover) are reported under "sweep".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun each rank runs an independent replica on its own GPU (weights
replicated, its own token stream; no collective on the data path), so
`value` is the whole-job tokens/s over all ranks and scaling is weak.

Weights: int4 uniform in [-8, 7], E8M0 exponents uniform in [-8, -3];
activations fp32 N(0, 1) (seeded synthetic data, see cpu_model_b200.synth).
Eight distinct copies of the weight pair (8 x 47.9 MB = 383 MB, > 3x the
126 MB L2) are rotated step by step, so every step streams its weights from
HBM.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

UP = (11008, 4096)     # (N, K)
DOWN = (4096, 11008)
EMIN, EMAX = -8, -3
COPIES = 8
# DRAM bytes of one batch-1 up-projection launch on MX input, measured with
# ncu (dram__bytes_read.sum 24,021,760 + dram__bytes_write.sum 0) against the
# 24,001,664 algorithmic bytes: every weight byte crosses DRAM once
ROOFLINE_TRAFFIC_B1 = 24021760
SWEEP = [8, 64, 512]
# the roofline leg times this many launches of the dominant kernel whatever
# --steps is, so its per-launch figure does not depend on the run length
ROOFLINE_LAUNCHES = 200
# int8 dense tensor peak of the B200 (spec; MEASURED_PEAKS.json holds no int8
# figure): north_star's denominator for the tensor-core GEMM
INT8_SPEC_TOPS = 4500.0
# single MX-int8 linear GEMV: 4096 x 4096, exponents [-10, -4], batch 1,
# seed 0; distinct weight copies rotated so the timed launches stream from
# HBM (32 x 17.3 MB = 554 MB > 4 x the 126 MB L2)
CFG1 = {"n": 4096, "k": 4096, "emin": -10, "emax": -4, "copies": 32}
# block-sparse MoE layer: 4096 tokens, d 4096, 8 experts, top-2, SwiGLU FFN
# 14336, MX-int4 expert matrices with 25 % of their 64x64 blocks present
MOE = {"tokens": 4096, "d": 4096, "ffn": 14336, "experts": 8, "top_k": 2, "density": 0.25}


def pair_bytes(b):
    """Algorithmic bytes of one pair step: packed int4 weights + E8M0 scales
    + MX activations in (u8 + scale) + fp32 outputs, for both linears."""
    tot = 0
    for n, k in (UP, DOWN):
        tot += n * k // 2 + n * k // 32 + b * (k + k // 32) + b * n * 4
    return tot


def gemv_bytes(n, k, b):
    return n * k // 2 + n * k // 32 + b * (k + k // 32) + b * n * 4


def int8_gemv_bytes(n, k, b):
    """Algorithmic bytes of one MX-int8 linear: int8 weights + E8M0 scales +
    MX activations + fp32 outputs (17,322,112 at 4096 x 4096, batch 1)."""
    return n * k + n * k // 32 + b * (k + k // 32) + b * n * 4


def pair_flops(b):
    return 2 * b * (UP[0] * UP[1] + DOWN[0] * DOWN[1])


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                f = [v.strip() for v in line.split(",")]
                if len(f) < 7:
                    continue
                try:
                    sm.append(float(f[0]))
                    mx.append(float(f[1]))
                except ValueError:
                    continue
                for nm, v in zip(names, f[3:7]):
                    if v.lower() == "active":
                        reasons.add(nm)
            os.remove(self.path)
        except OSError:
            pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# --------------------------------------------------------------- CPU ---
def cpu_pair_sample(seconds=10.0, batch=1, threads=0):
    """The multi-threaded dpbusd restatement of the removed reference VNNI
    kernel (oracle/mx_cpu_baseline.c), timed on the host over whole pair
    steps for about `seconds`."""
    from oracle import oracle
    from cpu_model_b200 import synth
    wu, su = synth.weights(4, UP[0], UP[1], EMIN, EMAX, 101)
    wd, sd = synth.weights(4, DOWN[0], DOWN[1], EMIN, EMAX, 102)
    swu = oracle.weight_sums(4, wu, *UP)
    swd = oracle.weight_sums(4, wd, *DOWN)
    x = synth.normal((batch, UP[1]), 103)
    steps = 0
    used = False
    t0 = time.perf_counter()
    while True:
        xq, xs = oracle.quantize_x(x)
        y1, used = oracle.baseline_gemv(4, xq, xs, wu, su, swu, UP[0], UP[1], threads)
        hq, hs = oracle.quantize_x(y1)
        oracle.baseline_gemv(4, hq, hs, wd, sd, swd, DOWN[0], DOWN[1], threads)
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    cores = threads if threads > 0 else oracle.max_threads()
    return {"value": batch * steps / el, "unit": "tokens/s", "cores": cores, "kind": "port",
            "bytes_per_s": steps * pair_bytes(batch) / el,
            "sample": "%d pair steps at batch %d (%.1f s), %s" % (
                steps, batch, el, "AVX-512 VNNI _mm512_dpbusd_epi32" if used else "portable int loop")}


def cpu_int8_sample(seconds=5.0, threads=0):
    """The single MX-int8 4096 x 4096 linear at batch 1 on the host cores
    (the dpbusd restatement), quantisation included."""
    from oracle import oracle
    from cpu_model_b200 import synth
    n, k = CFG1["n"], CFG1["k"]
    w, ws = synth.weights(8, n, k, CFG1["emin"], CFG1["emax"], 0)
    sums = oracle.weight_sums(8, w, n, k)
    x = synth.normal((1, k), 0)
    steps = 0
    t0 = time.perf_counter()
    while True:
        xq, xs = oracle.quantize_x(x)
        _, used = oracle.baseline_gemv(8, xq, xs, w, ws, sums, n, k, threads)
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    cores = threads if threads > 0 else oracle.max_threads()
    return {"value": steps / el, "unit": "tokens/s", "cores": cores, "kind": "port",
            "bytes_per_s": steps * int8_gemv_bytes(n, k, 1) / el,
            "sample": "%d linears at batch 1 (%.1f s), %s" % (
                steps, el, "AVX-512 VNNI _mm512_dpbusd_epi32" if used else "portable int loop")}


def moe_weights(ctx, dev, seed=7, experts_range=None):
    """Per expert (gate [F][D], up [F][D], down [D][F]) block-sparse MX-int4
    weights generated on the device (uniform int4 nibbles, exponents
    [EMIN, EMAX]) with uniform-random 64x64 block masks; returns the weight
    handles, the masks and the raw device data (for the CPU sample).  Each
    expert has its own seed, so any subset (expert parallelism) holds the
    same bytes as the full set."""
    import torch
    from cpu_model_b200 import mx, synth
    g = torch.Generator(device=dev)
    d, f = MOE["d"], MOE["ffn"]
    experts = []
    lo, hi = experts_range or (0, MOE["experts"])
    for e in range(lo, hi):
        g.manual_seed(seed * 1000 + e)
        mats = []
        for j, (n, k) in enumerate(((f, d), (f, d), (d, f))):
            data = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=dev, generator=g)
            sc = torch.randint(127 + EMIN, 127 + EMAX + 1, (n, k // 32), dtype=torch.uint8, device=dev, generator=g)
            mask = synth.block_mask(n, k, MOE["density"], seed * 1000 + e * 10 + j)
            mats.append((mx.MXWeight(data, sc, 4, n, k, ctx, block_mask=mask), mask, data, sc))
        experts.append(mats)
    return experts


def cpu_moe_sample(experts, x, logits, tokens=16, threads=0):
    """The same layer on the host for a few tokens: routing and requantisation
    from the oracle, each expert linear by the multi-threaded dpbusd
    restatement (oracle/mx_cpu_baseline.c) on the masked dense weights."""
    from oracle import oracle
    from cpu_model_b200 import synth
    d, f, k = MOE["d"], MOE["ffn"], MOE["top_k"]
    host = []
    for mats in experts:
        hm = []
        for (W, mask, data, sc) in mats:
            w = synth.apply_block_mask(4, data.cpu().numpy(), mask)
            s_ = sc.cpu().numpy()
            hm.append((w, s_, oracle.weight_sums(4, w, W.n, W.k)))
        host.append(hm)
    xs_h = x[:tokens].cpu().numpy()
    idx, gate = oracle.route_topk(logits[:tokens].cpu().numpy(), k)
    used = False
    t0 = time.perf_counter()
    for t in range(tokens):
        xq, xs = oracle.quantize_x(xs_h[t:t + 1])
        acc = np.zeros(d, np.float64)
        for j in range(k):
            (wg, sg, zg), (wu, su, zu), (wd, sd, zd) = host[idx[t, j]]
            gv, used = oracle.baseline_gemv(4, xq, xs, wg, sg, zg, f, d, threads)
            uv, _ = oracle.baseline_gemv(4, xq, xs, wu, su, zu, f, d, threads)
            hq, hs = oracle.swiglu_quantize(gv, uv)
            out, _ = oracle.baseline_gemv(4, hq, hs, wd, sd, zd, d, f, threads)
            acc += np.float64(gate[t, j]) * out[0]
    el = time.perf_counter() - t0
    cores = threads if threads > 0 else oracle.max_threads()
    return {"value": tokens / el, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": "%d tokens x top-%d experts, dense masked weights (%.1f s), %s" % (
                tokens, k, el, "AVX-512 VNNI dpbusd" if used else "portable int loop")}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count()))
    from oracle import oracle
    oracle.build()
    per_step = []
    for i in range(args.warmup + args.steps):
        s = cpu_pair_sample(seconds=1.0, batch=1)
        if i >= args.warmup:
            per_step.append(s)
    value = statistics.mean(p["value"] for p in per_step)
    line = {
        "impl": "reference", "metric": "MX-int4 qlinear tokens/s (7B MLP up+down pair)",
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 / value, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "mx-int4 (int4 w, int8 a, int32 dot, fp32 sum)",
        "data": "synthetic", "config": workload_config(1),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": per_step[0]["cores"], "kind": "port",
                         "sample": "each step ~1 s of whole pair steps at batch 1 (CPU restatement of the "
                                   "reference's removed AVX-512 VNNI MX kernel; the reference's own MX code is "
                                   "absent from its snapshot)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def time_cfg1(ctx, dev, args, world, max_over_ranks, barrier, peaks, rank, capture):
    """The single MX-int8 4096 x 4096 linear (fp32 x quantised inside the
    GEMV, fp32 y) at batch 1: ROOFLINE_LAUNCHES mxq_linear calls rotating
    CFG1["copies"] weight copies (copy 0 is the seed-0 matrix), replayed as
    one CUDA graph and timed with CUDA events on the launching stream."""
    import torch
    from cpu_model_b200 import mx, synth
    n, k = CFG1["n"], CFG1["k"]
    ws_ = []
    for c in range(CFG1["copies"]):
        w, s_ = synth.weights(8, n, k, CFG1["emin"], CFG1["emax"], c)
        ws_.append(mx.MXWeight(torch.from_numpy(w), torch.from_numpy(s_), 8, n, k, ctx))
    x = torch.from_numpy(synth.normal((1, k), 0)).to(dev)
    y = torch.empty((1, n), dtype=torch.float32, device=dev)
    lib = ctx.lib
    ctx._bind()

    def one(i):
        mx.check(lib.mxq_linear(ctx.h, ws_[i % len(ws_)].h, mx._ptr(x), 1, mx._ptr(y)), ctx.h)

    for i in range(max(3, len(ws_))):
        one(i)
    ctx.synchronize()
    l0 = ctx.launch_count()
    g = capture(lambda: [one(i) for i in range(ROOFLINE_LAUNCHES)])
    launches = ctx.launch_count() - l0
    g.replay()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / ROOFLINE_LAUNCHES)
    ctx.synchronize()
    del g
    nbytes = int8_gemv_bytes(n, k, 1)
    gbs = nbytes / (ms / 1e3) / 1e9
    out = {"metric": "MX-int8 qlinear tokens/s (4096x4096, batch 1)", "tokens_per_s": world / (ms / 1e3),
           "ms_per_token": ms, "launches": ROOFLINE_LAUNCHES, "kernel_launches_per_call": launches // ROOFLINE_LAUNCHES,
           "config": {"workload": "mx_int8_linear_4096", "weights": "int8 [-127,127], E8M0 exp [-10,-4], seed 0",
                      "activations": "fp32 N(0,1) -> MX-int8 per 32-block, seed 0",
                      "l2": "rotating %d weight copies (%.0f MB) vs 126 MB L2" % (CFG1["copies"], CFG1["copies"] * nbytes / 1e6)},
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": gbs / peaks["hbm_gbs"], "algorithmic_bytes_per_launch": nbytes,
                        "peak_src": peaks["src"] + " hbm_gbs (burst copy)",
                        "kernel": "cogemv_kernel<int8, fp32 in> (batch-1 GEMV, two launches resident per SM)"},
           "api": "mxq_linear"}
    if rank == 0 and world == 1 and not args.no_cpu:
        out["cpu_baseline"] = cpu_int8_sample(seconds=min(5.0, args.cpu_seconds))
    for w in ws_:
        w.close()
    return out


# 7B dense decoder: 32 layers, d 4096, 32 heads x 128, SwiGLU 11008, vocab
# 32000, MX-int4 weights; 2048-token prompts of uniform ids, then 256 decode
# steps, batch 1 / 8 / 32
DEC7B = {"n_layers": 32, "d_model": 4096, "n_heads": 32, "ffn": 11008, "vocab": 32000, "prompt": 2048,
         "decode": 256, "batches": [1, 8, 32]}
# 1B rollout policy: 16 layers, d 2048, 16 heads, FFN 5632, vocab 32000,
# MX-int8, value head; 256 rollouts x 512 tokens, GAE gamma 0.99 lambda 0.95
PPO1B = {"n_layers": 16, "d_model": 2048, "n_heads": 16, "ffn": 5632, "vocab": 32000, "rollouts": 256,
         "tokens": 512}


def decoder_weight_bytes(cfg, fmt):
    """MX bytes of every linear of the decoder (data + E8M0 scales)."""
    d, F, L, V = cfg["d_model"], cfg["ffn"], cfg["n_layers"], cfg["vocab"]
    per = 1.0 / (2 if fmt == 4 else 1) + 1.0 / 32
    return (L * (3 * d * d + d * d + 2 * F * d + d * F) + V * d) * per


def time_decoder_7b(ctx, dev, args, world, max_over_ranks, barrier, peaks, rank):
    """The 7B decoder: per batch size, the prompt (chunked prefill) timed as
    one call, then 256 one-token steps (each a replayed CUDA graph) timed
    with CUDA events around the loop.  Decode tokens are uniform ids drawn
    ahead of time (no sampling step).  Roofline: the weights (3.6 GB MX-int4)
    plus the bf16 K/V read by every step, against the HBM peak."""
    import torch
    from cpu_model_b200 import mx
    c = DEC7B
    D = mx.Decoder(c["n_layers"], c["d_model"], c["n_heads"], c["ffn"], c["vocab"], fmt=4,
                   max_batch=max(c["batches"]), max_ctx=c["prompt"] + c["decode"], max_rows=8192, seed=3, ctx=ctx)
    g = torch.Generator(device=dev)
    out = {"config": dict({k: v for k, v in c.items() if k != "batches"}, weights="mx-int4, E8M0 exp [-8,-3]",
                          kv_cache="bf16", data="uniform-random token ids"), "api": "mxq_decoder_prefill/decode",
           "batches": {}}
    wbytes = decoder_weight_bytes(c, 4)
    for b in c["batches"]:
        g.manual_seed(100 + b)
        prompt = torch.randint(0, c["vocab"], (b, c["prompt"]), dtype=torch.int32, device=dev, generator=g)
        steps = torch.randint(0, c["vocab"], (c["decode"], b), dtype=torch.int32, device=dev, generator=g)
        D.reset()
        D.prefill(prompt)                                  # warm-up (workspaces, graphs)
        for i in range(3):
            D.decode(steps[i].contiguous())
        torch.cuda.synchronize()
        D.reset()
        barrier()
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        D.prefill(prompt)
        e1.record()
        for i in range(c["decode"]):
            D.decode(steps[i])
        e2.record()
        torch.cuda.synchronize()
        pre_ms = max_over_ranks(e0.elapsed_time(e1))
        dec_ms = max_over_ranks(e1.elapsed_time(e2))
        step_ms = dec_ms / c["decode"]
        avg_ctx = c["prompt"] + (c["decode"] + 1) / 2.0
        kv = b * c["n_layers"] * 2 * avg_ctx * c["d_model"] * 2
        gbs = (wbytes + kv) / (step_ms / 1e3) / 1e9
        out["batches"][str(b)] = {
            "decode_tokens_per_s": world * b * c["decode"] / (dec_ms / 1e3), "decode_ms_per_step": step_ms,
            "prefill_tokens_per_s": world * b * c["prompt"] / (pre_ms / 1e3), "prefill_ms": pre_ms,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "bytes_per_step": wbytes + kv,
                         "bytes": "MX weights %.2f GB + bf16 K/V %.2f GB (mean context %.0f)" % (
                             wbytes / 1e9, kv / 1e9, avg_ctx)}}
    D.close()
    return out


def time_decoder_7b_tp(ctx, dev, args, world, max_over_ranks, barrier, peaks, rank):
    """N > 1: the same 7B decoder tensor-parallel over the N GPUs
    (mxq_decoder_create_sharded): each rank holds 32/N heads and 11008/N FFN
    units (their QKV and gate/up rows, their O and down columns); two peer
    exchanges of partial sums a layer.  Every rank serves the same
    sequences, so tokens/s counts them once.  Roofline: each rank's share of
    the weights and K/V (the head is replicated) against one GPU's HBM peak."""
    import torch
    import torch.distributed as dist
    from cpu_model_b200 import mx
    c = DEC7B
    D = mx.Decoder(c["n_layers"], c["d_model"], c["n_heads"], c["ffn"], c["vocab"], fmt=4,
                   max_batch=max(c["batches"]), max_ctx=c["prompt"] + c["decode"], max_rows=8192, seed=3, ctx=ctx,
                   rank=rank, world=world)
    handles = [None] * world
    dist.all_gather_object(handles, D.handle())
    D.connect(handles)
    barrier()
    g = torch.Generator(device=dev)
    out = {"config": dict({k: v for k, v in c.items() if k != "batches"}, weights="mx-int4, E8M0 exp [-8,-3]",
                          kv_cache="bf16", data="uniform-random token ids", parallelism="tp%d" % world,
                          exchange="peer exchange of O / down partial sums over NVLink, 2 per layer"),
           "api": "mxq_decoder_create_sharded + prefill/decode", "batches": {}}
    head = c["vocab"] * c["d_model"] * (0.5 + 1.0 / 32)
    wbytes = (decoder_weight_bytes(c, 4) - head) / world + head
    for b in c["batches"]:
        g.manual_seed(100 + b)                             # the same tokens on every rank
        prompt = torch.randint(0, c["vocab"], (b, c["prompt"]), dtype=torch.int32, device=dev, generator=g)
        steps = torch.randint(0, c["vocab"], (c["decode"], b), dtype=torch.int32, device=dev, generator=g)
        D.reset()
        D.prefill(prompt)
        for i in range(3):
            D.decode(steps[i].contiguous())
        torch.cuda.synchronize()
        D.reset()
        barrier()
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        D.prefill(prompt)
        e1.record()
        for i in range(c["decode"]):
            D.decode(steps[i])
        e2.record()
        torch.cuda.synchronize()
        pre_ms = max_over_ranks(e0.elapsed_time(e1))
        dec_ms = max_over_ranks(e1.elapsed_time(e2))
        step_ms = dec_ms / c["decode"]
        avg_ctx = c["prompt"] + (c["decode"] + 1) / 2.0
        kv = b * c["n_layers"] * 2 * avg_ctx * c["d_model"] * 2 / world
        gbs = (wbytes + kv) / (step_ms / 1e3) / 1e9
        out["batches"][str(b)] = {
            "decode_tokens_per_s": b * c["decode"] / (dec_ms / 1e3), "decode_ms_per_step": step_ms,
            "prefill_tokens_per_s": b * c["prompt"] / (pre_ms / 1e3), "prefill_ms": pre_ms,
            "roofline": {"bound": "hbm", "achieved_per_gpu": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "bytes_per_step_per_gpu": wbytes + kv}}
    torch.cuda.synchronize()
    barrier()
    D.close()
    return out


def time_ppo_1b(ctx, dev, args, world, max_over_ranks, barrier, peaks, rank):
    """The 1B MX-int8 rollout policy: 256 rollouts x 512 tokens scored
    (per-token log-probs of the next token, a value per token), then GAE over
    the [512][256] trajectory with rewards ~ N(0, 1) at each rollout's last
    token (done there); data parallel (each rank its own batch)."""
    import torch
    from cpu_model_b200 import mx
    c = PPO1B
    D = mx.Decoder(c["n_layers"], c["d_model"], c["n_heads"], c["ffn"], c["vocab"], fmt=8, max_batch=16,
                   max_ctx=c["tokens"], max_rows=8192, value_head=True, seed=4, ctx=ctx)
    g = torch.Generator(device=dev)
    g.manual_seed(500 + rank)
    R, T = c["rollouts"], c["tokens"]
    tok = torch.randint(0, c["vocab"], (R, T), dtype=torch.int32, device=dev, generator=g)
    rewards = torch.zeros((T, R), device=dev)
    rewards[-1] = torch.randn(R, generator=g, device=dev)
    dones = torch.zeros((T, R), dtype=torch.uint8, device=dev)
    dones[-1] = 1
    nv = torch.zeros(R, device=dev)

    def step():
        logp, values = D.score(tok)
        return mx.fused_compute_gae(rewards, values.t().contiguous(), dones, nv, 0.99, 0.95, ctx)

    step()
    torch.cuda.synchronize()
    barrier()
    n = 2
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / n)
    d, F, L, V = c["d_model"], c["ffn"], c["n_layers"], c["vocab"]
    lin_flops = 2.0 * R * T * (L * (4 * d * d + 3 * d * F) + (V + 1) * d)
    att_flops = 4.0 * R * L * d * T * T / 2
    tf = (lin_flops + att_flops) / (ms / 1e3) / 1e12
    D.close()
    return {"tokens_per_s": world * R * T / (ms / 1e3), "ms_per_batch": ms, "batches": n,
            "tflops": tf, "linear_tflop_per_batch": lin_flops / 1e12, "attention_tflop_per_batch": att_flops / 1e12,
            "roofline": {"bound": "tensor", "achieved": tf, "unit": "TFLOP/s", "peak": peaks["bf16_tflops_sustained"],
                         "frac": tf / peaks["bf16_tflops_sustained"], "frac_of_int8_spec": tf / INT8_SPEC_TOPS,
                         "peak_src": peaks["src"] + " bf16_tflops_sustained"},
            "config": dict(c, weights="mx-int8, E8M0 exp [-10,-4]", value_head=True, gae="gamma 0.99, lambda 0.95",
                           data="uniform-random token ids, rewards N(0,1) at rollout ends"),
            "api": "mxq_decoder_score + mxq_gae"}


def time_moe(ctx, dev, args, world, max_over_ranks, barrier, peaks, rank):
    """The block-sparse MoE layer (mxq_moe_swiglu) at its full size: whole
    layer calls timed with CUDA events (each call reads the per-expert token
    counts back once to size its launches, so the loop is not captured)."""
    import torch
    from cpu_model_b200 import mx, synth
    experts = moe_weights(ctx, dev)
    gate_w = [m[0][0] for m in experts]
    up_w = [m[1][0] for m in experts]
    down_w = [m[2][0] for m in experts]
    t, d, e, k = MOE["tokens"], MOE["d"], MOE["experts"], MOE["top_k"]
    x = torch.from_numpy(synth.normal((t, d), 201)).to(dev)
    logits = torch.from_numpy(synth.normal((t, e), 202)).to(dev)
    for _ in range(2):
        mx.moe_swiglu(x, logits, gate_w, up_w, down_w, k, ctx)
    ctx.synchronize()
    steps = max(3, args.steps // 20)
    barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        mx.moe_swiglu(x, logits, gate_w, up_w, down_w, k, ctx)
    e1.record(stream)
    torch.cuda.synchronize()
    ctx.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    # algorithmic (nonzero-block) work: 2 flops per stored nonzero weight per
    # route, over the experts the routing actually chose
    idx, _ = mx.route_topk(logits, k, ctx)
    counts = np.bincount(idx.cpu().numpy().ravel(), minlength=e)
    nnz = [sum(int(m[1].sum()) * 64 * 64 for m in mats) for mats in experts]
    flops = 2.0 * float(sum(int(counts[j]) * nnz[j] for j in range(e)))
    tf = flops / (ms / 1e3) / 1e12
    out = {"tokens_per_s": world * t / (ms / 1e3), "ms_per_step": ms, "steps": steps,
           "nonzero_tflops": tf,
           "frac_of_bf16_peak": tf / peaks["bf16_tflops"],
           "roofline": {"bound": "tensor", "achieved": tf, "unit": "TFLOP/s",
                        "peak": peaks["bf16_tflops_sustained"], "frac": tf / peaks["bf16_tflops_sustained"],
                        "peak_src": peaks["src"] + " bf16_tflops_sustained (a ms-long layer call)",
                        "frac_of_int8_spec": tf / INT8_SPEC_TOPS,
                        "int8_spec_tops": INT8_SPEC_TOPS,
                        "ops": "2 per stored nonzero weight per route (nonzero 64x64 blocks only)",
                        "kernel": "whole layer: gemm_tc_kernel<int4> on block-sparse tiles (kind::f16, "
                                  "bf16 operands) + router/quantiser/combine kernels"},
           "nonzero_gop_per_step": flops / 1e9,
           "config": dict(MOE, weights="mx-int4 block-sparse 64x64", routing="softmax top-2 over N(0,1) logits"),
           "api": "mxq_moe_swiglu"}
    if rank == 0 and world == 1 and not args.no_cpu:
        out["cpu_baseline"] = cpu_moe_sample(experts, x, logits)
    for mats in experts:
        for m in mats:
            m[0].close()
    return out


# the reference's PPO rollout forward (training/ppo_trainer.cpp:57-66, :77):
# states 1616 -> latent 2048 -> 80 logits + value, MX-int8 weights; 256
# rollouts x 512 steps per batch, then GAE (gamma 0.99, lambda 0.95)
PPO = {"rollouts": 256, "steps": 512, "state": 1616, "state_padded": 1632, "latent": 2048, "actions": 80}


def time_ppo(ctx, dev, args, world, max_over_ranks, barrier, peaks, rank):
    """One rollout batch through the MX policy forward and GAE (data
    parallel: every rank its own batch)."""
    import torch
    from cpu_model_b200 import mx, synth
    p = PPO
    rows = p["rollouts"] * p["steps"]
    wp, sp = synth.weights(8, p["latent"], p["state_padded"], -9, -5, 401)
    wpi, spi = synth.weights(8, p["actions"], p["latent"], -9, -5, 402)
    wv, sv = synth.weights(8, 1, p["latent"], -9, -5, 403)
    Wp = mx.MXWeight(torch.from_numpy(wp), torch.from_numpy(sp), 8, p["latent"], p["state_padded"], ctx)
    Wpi = mx.MXWeight(torch.from_numpy(wpi), torch.from_numpy(spi), 8, p["actions"], p["latent"], ctx)
    Wv = mx.MXWeight(torch.from_numpy(wv), torch.from_numpy(sv), 8, 1, p["latent"], ctx)
    # policy and value rows as one head weight: the latent is quantised once
    Wh = mx.MXWeight(torch.from_numpy(np.concatenate([wpi, wv])), torch.from_numpy(np.concatenate([spi, sv])), 8,
                     p["actions"] + 1, p["latent"], ctx)
    g = torch.Generator(device=dev)
    g.manual_seed(404)
    states = torch.randn((rows, p["state_padded"]), generator=g, device=dev)
    states[:, p["state"]:] = 0.0
    actions = torch.nn.functional.one_hot(torch.randint(0, p["actions"], (rows,), generator=g, device=dev),
                                          p["actions"]).float()
    rewards = torch.randn((p["steps"], p["rollouts"]), generator=g, device=dev)
    dones = torch.zeros((p["steps"], p["rollouts"]), dtype=torch.uint8, device=dev)
    dones[-1] = 1
    nv = torch.zeros(p["rollouts"], device=dev)

    def step():
        lp, alp, ent, val = mx.ppo_rollout_forward(states, actions, Wp, Wh, None, ctx)
        return mx.fused_compute_gae(rewards, val.reshape(p["steps"], p["rollouts"]), dones, nv, 0.99, 0.95, ctx)

    for _ in range(2):
        step()
    ctx.synchronize()
    n = max(3, args.steps // 40)
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / n)
    flops = 2.0 * rows * p["latent"] * (p["state_padded"] + p["actions"] + 1)
    Wpi.close()
    Wv.close()
    out = {"rows_per_s": world * rows / (ms / 1e3), "ms_per_batch": ms, "batches": n,
           "tflops": flops / (ms / 1e3) / 1e12, "frac_of_bf16_peak": flops / (ms / 1e3) / 1e12 / peaks["bf16_tflops"],
           "config": dict(p, weights="mx-int8", gae="gamma 0.99, lambda 0.95"),
           "api": "mx.ppo_rollout_forward (mxq_linear projection + one combined policy/value head linear + mxq_policy_head) + mxq_gae"}
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import oracle
        sample = 64
        st = states[:sample].cpu().numpy()
        zp, zpi, zv = (oracle.weight_sums(8, w, n_, k_) for w, n_, k_ in
                       ((wp, p["latent"], p["state_padded"]), (wpi, p["actions"], p["latent"]), (wv, 1, p["latent"])))
        t0 = time.perf_counter()
        reps = 0
        while True:
            q, s_ = oracle.quantize_x(st)
            lat, used = oracle.baseline_gemv(8, q, s_, wp, sp, zp, p["latent"], p["state_padded"])
            lq, ls = oracle.quantize_x(lat)
            lg, _ = oracle.baseline_gemv(8, lq, ls, wpi, spi, zpi, p["actions"], p["latent"])
            oracle.baseline_gemv(8, lq, ls, wv, sv, zv, 1, p["latent"])
            oracle.policy_head(lg, np.zeros_like(lg))
            reps += 1
            el = time.perf_counter() - t0
            if el >= 3.0:
                break
        out["cpu_baseline"] = {"value": reps * sample / el, "unit": "rows/s", "cores": oracle.max_threads(),
                               "kind": "port", "sample": "%d x %d rows through the three MX linears + head (%.1f s), %s"
                               % (reps, sample, el, "AVX-512 VNNI dpbusd" if used else "portable int loop")}
    for w in (Wp, Wh):
        w.close()
    return out


def time_sharded_peer(ctx, dev, args, world, rank, max_over_ranks, barrier, up_full, dn_full):
    """N > 1: the batch-1 pair column-sharded through mxq_linear_pair_sharded
    (no NCCL on the data path: each linear's rows go straight into every
    rank's mailbox over NVLink).  Each rank holds 1/N of both matrices;
    enough distinct shard copies rotate that a step's weights come from HBM,
    not L2; CUDA graph of the steps, CUDA events, max over ranks."""
    import torch
    import torch.distributed as dist
    from cpu_model_b200 import mx, synth
    n1, n2 = UP[0], DOWN[0]
    n1s, n2s = n1 // world, n2 // world
    shard_bytes = pair_bytes(1) / world
    copies = max(2, int(math.ceil(4 * 126e6 / shard_bytes)))
    (wu, su), (wd, sd) = up_full, dn_full
    w1 = (np.ascontiguousarray(wu[rank * n1s:(rank + 1) * n1s]), np.ascontiguousarray(su[rank * n1s:(rank + 1) * n1s]))
    w2 = (np.ascontiguousarray(wd[rank * n2s:(rank + 1) * n2s]), np.ascontiguousarray(sd[rank * n2s:(rank + 1) * n2s]))
    shards = [(mx.MXWeight(torch.from_numpy(w1[0]), torch.from_numpy(w1[1]), 4, n1s, UP[1], ctx),
               mx.MXWeight(torch.from_numpy(w2[0]), torch.from_numpy(w2[1]), 4, n2s, DOWN[1], ctx))
              for _ in range(copies)]
    P = mx.PeerGroup(rank, world, n1, n2, ctx)
    handles = [None] * world
    dist.all_gather_object(handles, P.handle())
    P.connect(handles)
    barrier()
    x = torch.from_numpy(synth.normal((1, UP[1]), 303)).to(dev)
    y = torch.empty((1, n2), dtype=torch.float32, device=dev)
    for i in range(max(3, args.warmup)):
        P.linear_pair(x, *shards[i % copies], out=y)
    ctx.synchronize()
    steps = max(20, args.steps)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(steps):
                P.linear_pair(x, *shards[i % copies], out=y)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):          # replay and events on the same stream
        g.replay()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    del g
    ctx.synchronize()
    barrier()
    P.close()
    for a, b in shards:
        a.close()
        b.close()
    return {"1": {"ms_per_step": ms, "tokens_per_s": 1.0 / (ms / 1e3)}, "scaling": "strong",
            "weight_copies": copies, "api": "mxq_linear_pair_sharded",
            "collective": "none: rows stored into every rank's mailbox over NVLink by the GEMV epilogues, "
                          "bounded flag waits"}


def time_sharded(ctx, dev, args, world, rank, max_over_ranks, barrier):
    """N > 1 only: the multi-GPU forms of the path, over NCCL.
    pair -- the MLP pair column-sharded (each rank owns F/N rows of up and
    D/N rows of down, full K), one all-gather after each linear; one token
    stream of `batch`, so tokens/s does not multiply with N (strong scaling).
    moe -- the MoE layer with the 8 experts partitioned over the ranks and
    the 4096 tokens split over them, routes dispatched and returned with
    all_to_all_single."""
    import torch
    from cpu_model_b200 import mx, shard, synth
    out = {}
    up_full = synth.weights(4, UP[0], UP[1], EMIN, EMAX, 301)
    dn_full = synth.weights(4, DOWN[0], DOWN[1], EMIN, EMAX, 302)

    def slice_weight(full, n, k):
        def fn(lo, hi):
            w, s_ = full
            return mx.MXWeight(torch.from_numpy(np.ascontiguousarray(w[lo:hi])),
                               torch.from_numpy(np.ascontiguousarray(s_[lo:hi])), 4, hi - lo, k, ctx)
        return fn

    lin = lambda x, w: mx.mx_linear(x, w, ctx)
    up = shard.ColumnShardedLinear(UP[0], slice_weight(up_full, *UP), lin)
    down = shard.ColumnShardedLinear(DOWN[0], slice_weight(dn_full, *DOWN), lin)
    pair = {}
    for b in (1, 64):
        x = torch.from_numpy(synth.normal((b, UP[1]), 303)).to(dev)
        for _ in range(args.warmup):
            shard.sharded_pair(x, up, down)
        steps = max(10, args.steps // 4)
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            shard.sharded_pair(x, up, down)
        e1.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1) / steps)
        pair[str(b)] = {"ms_per_step": ms, "tokens_per_s": b / (ms / 1e3)}
    up.w.close()
    down.w.close()
    out["pair_column_sharded"] = dict(pair, scaling="strong", collective="all_gather (NCCL) after each linear")
    out["pair_column_sharded_peer"] = time_sharded_peer(ctx, dev, args, world, rank, max_over_ranks, barrier,
                                                        up_full, dn_full)

    e_lo, e_hi = shard.row_shards(MOE["experts"], world)[rank]
    experts = moe_weights(ctx, dev, experts_range=(e_lo, e_hi))
    local = {e_lo + i: (m[0][0], m[1][0], m[2][0]) for i, m in enumerate(experts)}
    t_local = MOE["tokens"] // world
    x = torch.from_numpy(synth.normal((MOE["tokens"], MOE["d"]), 201)).to(dev)[rank * t_local:(rank + 1) * t_local]
    logits = torch.from_numpy(synth.normal((MOE["tokens"], MOE["experts"]), 202)).to(dev)[rank * t_local:(rank + 1) * t_local]

    def expert_mlp(e, rows):
        g, u, d_ = local[e]
        return mx.gated_mlp_step(rows, g, u, d_, ctx)

    def layer():
        idx, gate = mx.route_topk(logits.contiguous(), MOE["top_k"], ctx)
        return shard.moe_expert_parallel(x.contiguous(), idx, gate, MOE["experts"], expert_mlp)

    for _ in range(2):
        layer()
    steps = max(3, args.steps // 20)
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        layer()
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    out["moe_expert_parallel"] = {"ms_per_step": ms, "tokens_per_s": MOE["tokens"] / (ms / 1e3),
                                  "experts_per_rank": e_hi - e_lo, "tokens_per_rank": t_local,
                                  "collective": "all_to_all_single (NCCL) dispatch + return"}
    if MOE["experts"] % world == 0:
        # the same layer in libmxq (mxq_moe_swiglu_sharded): every rank holds
        # all 4096 tokens, runs its experts, and the expert outputs cross
        # NVLink once, into every rank's mailbox; the full y on every rank
        import torch.distributed as dist
        G = mx.MoEGroup(rank, world, MOE["tokens"], MOE["top_k"], MOE["d"], ctx)
        handles = [None] * world
        dist.all_gather_object(handles, G.handle())
        G.connect(handles)
        xf = torch.from_numpy(synth.normal((MOE["tokens"], MOE["d"]), 201)).to(dev)
        lf = torch.from_numpy(synth.normal((MOE["tokens"], MOE["experts"]), 202)).to(dev)
        yb = torch.empty_like(xf)
        gw, uw, dw = ([m[i][0] for m in experts] for i in range(3))

        def layer_peer():
            G.moe_swiglu(xf, lf, gw, uw, dw, MOE["top_k"], out=yb)

        for _ in range(2):
            layer_peer()
        barrier()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            layer_peer()
        e1.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1) / steps)
        out["moe_expert_parallel_peer"] = {
            "ms_per_step": ms, "tokens_per_s": MOE["tokens"] / (ms / 1e3), "experts_per_rank": e_hi - e_lo,
            "tokens_per_rank": MOE["tokens"], "api": "mxq_moe_swiglu_sharded",
            "exchange": "expert-output rows over NVLink peer stores, one exchange a layer"}
        torch.cuda.synchronize()
        barrier()
        G.close()
    for mats in experts:
        for m in mats:
            m[0].close()
    return out


def workload_config(batch, copies=COPIES):
    return {"workload": "mx_int4_mlp_pair_7b", "up": "4096->11008", "down": "11008->4096",
            "batch": batch, "weights": "int4 [-8,7], E8M0 exp [-8,-3]", "activations": "fp32 N(0,1) -> MX-int8",
            "l2": "rotating %d weight copies (%.0f MB) vs 126 MB L2" % (copies, copies * pair_bytes(0) / 1e6),
            "parallelism": "replicas"}


# --------------------------------------------------------------- GPU ---
def run_ours(args):
    import torch
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    from cpu_model_b200 import mx, synth

    ctx = mx.MXContext(local)
    peaks = load_peaks()
    stream = torch.cuda.current_stream(dev)

    # weights: COPIES distinct pairs (seeded per copy), uploaded once
    pairs = []
    for c in range(args.copies):
        wu, su = synth.weights(4, UP[0], UP[1], EMIN, EMAX, 1000 + 2 * c)
        wd, sd = synth.weights(4, DOWN[0], DOWN[1], EMIN, EMAX, 1001 + 2 * c)
        pairs.append((mx.MXWeight(torch.from_numpy(wu), torch.from_numpy(su), 4, UP[0], UP[1], ctx),
                      mx.MXWeight(torch.from_numpy(wd), torch.from_numpy(sd), 4, DOWN[0], DOWN[1], ctx)))
    ctx.reserve(max(SWEEP + [args.batch]), DOWN[1])

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        import torch.distributed as dist
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def capture(fn):
        """Record fn() (a sequence of library calls on the current stream) into
        a CUDA graph; the library's launches become graph nodes, with their
        programmatic (PDL) dependencies kept as graph edges."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ctx._bind()
            fn()
        ctx._bind()
        return g

    def time_pairs(batch, steps, warmup):
        """K pair steps, rotating the weight copies, replayed as one CUDA graph
        (a decode loop launches its step graph once per token); timed with
        CUDA events around the replay."""
        x = torch.from_numpy(synth.normal((batch, UP[1]), 7 + rank)).to(dev)
        y = torch.empty((batch, DOWN[0]), dtype=torch.float32, device=dev)
        ctx._bind()
        lib = ctx.lib

        def step(i):
            wu, wd = pairs[i % len(pairs)]
            mx.check(lib.mxq_linear_pair(ctx.h, wu.h, wd.h, mx._ptr(x), batch, mx._ptr(y)), ctx.h)

        for i in range(warmup):
            step(i)
        ctx.synchronize()
        l0 = ctx.launch_count()
        g = capture(lambda: [step(i) for i in range(steps)])
        launches = ctx.launch_count() - l0
        g.replay()                      # untimed graph warm-up
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1))
        ctx.synchronize()
        del g
        return ms / steps, launches

    def time_gemv(batch, steps):
        """The dominant kernel alone: the up-projection linear kernel (GEMV or
        tensor-core GEMM by batch) on pre-quantised activations, rotating
        weight copies, as one CUDA graph; CUDA events on the launching
        stream."""
        x = torch.from_numpy(synth.normal((batch, UP[1]), 9)).to(dev)
        a = mx.mx_quantize_x(x, ctx)
        y = torch.empty((batch, UP[0]), dtype=torch.float32, device=dev)
        lib = ctx.lib
        ctx._bind()

        def one(i):
            mx.check(lib.mxq_gemv(ctx.h, pairs[i % len(pairs)][0].h, mx._ptr(a.q), mx._ptr(a.s), batch,
                                  mx._ptr(y)), ctx.h)

        for i in range(3):
            one(i)
        ctx.synchronize()
        g = capture(lambda: [one(i) for i in range(steps)])
        g.replay()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ctx.synchronize()
        del g
        return e0.elapsed_time(e1) / steps

    def time_e2e(batch, steps):
        """Through the public host-buffer entry (mxq_linear_pair_host):
        pinned x in, y out, copies inside the timed region.  Warm-up covers
        every weight pair twice (the first call of a pair sizes the buffers,
        the second records its launch graph), as a serving loop would."""
        xh = torch.from_numpy(synth.normal((batch, UP[1]), 11)).pin_memory()
        yh = torch.empty((batch, DOWN[0]), dtype=torch.float32).pin_memory()
        lib = ctx.lib
        ctx._bind()
        for i in range(max(3, 2 * len(pairs))):
            wu, wd = pairs[i % len(pairs)]
            mx.check(lib.mxq_linear_pair_host(ctx.h, wu.h, wd.h, mx._ptr(xh), batch, mx._ptr(yh)), ctx.h)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            wu, wd = pairs[i % len(pairs)]
            mx.check(lib.mxq_linear_pair_host(ctx.h, wu.h, wd.h, mx._ptr(xh), batch, mx._ptr(yh)), ctx.h)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1)) / steps
        return ms, batch * UP[1] * 4, batch * DOWN[0] * 4

    b = args.batch
    with Clocks(local) as clk:
        ms, launches = time_pairs(b, args.steps, args.warmup)
    clocks = clk.summary()
    value = world * b / (ms / 1e3)
    gemv_ms = time_gemv(b, ROOFLINE_LAUNCHES)
    gbytes = gemv_bytes(UP[0], UP[1], b)
    achieved = gbytes / (gemv_ms / 1e3) / 1e9
    e2e_ms, h2d, d2h = time_e2e(b, max(10, args.steps // 4))

    sweep = {}
    for sb in ([] if args.no_sweep else SWEEP):
        sms, _ = time_pairs(sb, max(10, args.steps // 4), 3)
        kms = time_gemv(sb, ROOFLINE_LAUNCHES if sb <= 64 else 40)
        fl = 2 * sb * UP[0] * UP[1]
        entry = {"tokens_per_s": world * sb / (sms / 1e3), "ms_per_step": sms,
                 "up_kernel_ms": kms,
                 "up_kernel_hbm_gbs": gemv_bytes(UP[0], UP[1], sb) / (kms / 1e3) / 1e9,
                 "up_kernel_tflops": fl / (kms / 1e3) / 1e12}
        if sb > 16:
            # the tensor-core GEMM against north_star's int8 denominator and
            # against the bf16 rate its kind::f16 MMAs run at (their ceiling)
            entry["up_kernel_frac_of_int8_spec"] = fl / (kms / 1e3) / 1e12 / INT8_SPEC_TOPS
            entry["up_kernel_frac_of_bf16_burst"] = fl / (kms / 1e3) / 1e12 / peaks["bf16_tflops"]
        entry["path"] = ("gemv-resident-dp4a" if sb == 1 else "gemv-ring-dp4a" if sb == 2 else
                         "gemv-mma-s8" if sb <= 16 else "tcgen05-bf16")
        sweep[str(sb)] = entry

    cfg1 = None
    if not args.no_cfg1:
        cfg1 = time_cfg1(ctx, dev, args, world, max_over_ranks, barrier, peaks, rank, capture)
    moe = None
    if not args.no_moe:
        moe = time_moe(ctx, dev, args, world, max_over_ranks, barrier, peaks, rank)
    ppo = None
    if not args.no_ppo:
        ppo = time_ppo(ctx, dev, args, world, max_over_ranks, barrier, peaks, rank)
    dec7b = None
    if not args.no_decoder:
        dec7b = time_decoder_7b(ctx, dev, args, world, max_over_ranks, barrier, peaks, rank)
    ppo1b = None
    if not args.no_ppo:
        ppo1b = time_ppo_1b(ctx, dev, args, world, max_over_ranks, barrier, peaks, rank)
    sharded = None
    if world > 1 and not args.no_shard:
        sharded = time_sharded(ctx, dev, args, world, rank, max_over_ranks, barrier)
        if not args.no_decoder:
            sharded["decoder_7b_tensor_parallel"] = time_decoder_7b_tp(ctx, dev, args, world, max_over_ranks,
                                                                       barrier, peaks, rank)

    if rank == 0:
        line = {
            "metric": "MX-int4 qlinear tokens/s (7B MLP up+down pair)",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "mx-int4 (int4 w, int8 a, int32 dot, fp32 sum)",
            "data": "synthetic", "config": workload_config(b, args.copies),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"],
                         "traffic": ROOFLINE_TRAFFIC_B1 if b == 1 else None,
                         "traffic_src": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                         "cogemv_kernel<int4, MX in> launch (up 4096->11008)")
                                        if b == 1 else None,
                         "kernel": ("cogemv_kernel<int4, MX in> (up 4096->11008, two launches resident per SM)" if b == 1 else
                                    "rgemv_kernel<int4> (up 4096->11008)" if b <= 4 else "gemm_tc_kernel<int4> (up 4096->11008)"),
                         "algorithmic_bytes_per_launch": gbytes, "launch_ms": gemv_ms,
                         "peak_src": peaks["src"] + " hbm_gbs (burst copy)"},
            "pair_hbm_gbs": pair_bytes(b) / (ms / 1e3) / 1e9,
            "e2e": {"value": world * b / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "api": "mxq_linear_pair_host"},
            "gpu_launches": launches,
            "clocks": clocks,
            "sweep": sweep,
        }
        if cfg1 is not None:
            line["int8_linear_4096"] = cfg1
        if moe is not None:
            line["moe"] = moe
        if ppo is not None:
            line["ppo_rollout"] = ppo
        if dec7b is not None:
            line["decoder_7b"] = dec7b
        if ppo1b is not None:
            line["ppo_policy_1b"] = ppo1b
        if sharded is not None:
            line["sharded"] = sharded
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_pair_sample(seconds=args.cpu_seconds, batch=b)
        print(json.dumps(line), flush=True)

    for p in pairs:
        p[0].close()
        p[1].close()
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_case(args):
    """Small single-workload runs for profiling (ncu) on one GPU: a few
    launches of one kernel family, nothing timed.
      gemm512   3 up-projection linears at batch 512 (tcgen05 GEMM)
      gemv1     3 up-projection GEMVs at batch 1 on MX input (co-resident GEMV)
      pair1     8 batch-1 MLP pair steps (mxq_linear_pair)
      moe       one full-size block-sparse MoE layer
      decode7b  the 7B decoder: a 2048-token prompt, then 3 decode steps"""
    import torch
    from cpu_model_b200 import mx, synth
    ctx = mx.MXContext(0)
    if args.case in ("gemm512", "gemv1"):
        b = 512 if args.case == "gemm512" else 1
        wu, su = synth.weights(4, UP[0], UP[1], EMIN, EMAX, 1000)
        W = mx.MXWeight(torch.from_numpy(wu), torch.from_numpy(su), 4, UP[0], UP[1], ctx)
        x = torch.from_numpy(synth.normal((b, UP[1]), 9)).cuda()
        if b == 1:
            # the roofline leg's kernel: the batch-1 GEMV on MX input
            a = mx.mx_quantize_x(x, ctx)
            for _ in range(3):
                mx.mx_gemv(a, W, ctx)
        else:
            for _ in range(3):
                mx.mx_linear(x, W, ctx)
        W.close()
    elif args.case == "pair1":
        wu, su = synth.weights(4, UP[0], UP[1], EMIN, EMAX, 1000)
        wd, sd = synth.weights(4, DOWN[0], DOWN[1], EMIN, EMAX, 1001)
        Wu = mx.MXWeight(torch.from_numpy(wu), torch.from_numpy(su), 4, UP[0], UP[1], ctx)
        Wd = mx.MXWeight(torch.from_numpy(wd), torch.from_numpy(sd), 4, DOWN[0], DOWN[1], ctx)
        x = torch.from_numpy(synth.normal((1, UP[1]), 9)).cuda()
        for _ in range(8):
            mx.mx_linear_pair(x, Wu, Wd, ctx)
        Wu.close()
        Wd.close()
    elif args.case == "moe":
        experts = moe_weights(ctx, torch.device("cuda", 0))
        x = torch.from_numpy(synth.normal((MOE["tokens"], MOE["d"]), 201)).cuda()
        logits = torch.from_numpy(synth.normal((MOE["tokens"], MOE["experts"]), 202)).cuda()
        mx.moe_swiglu(x, logits, [m[0][0] for m in experts], [m[1][0] for m in experts],
                      [m[2][0] for m in experts], MOE["top_k"], ctx)
    elif args.case == "decode7b":
        c = DEC7B
        D = mx.Decoder(c["n_layers"], c["d_model"], c["n_heads"], c["ffn"], c["vocab"], fmt=4, max_batch=1,
                       max_ctx=c["prompt"] + 8, max_rows=8192, seed=3, ctx=ctx)
        D.prefill(torch.randint(0, c["vocab"], (1, c["prompt"]), dtype=torch.int32, device="cuda"))
        for i in range(3):
            D.decode(torch.full((1,), i, dtype=torch.int32, device="cuda"))
        D.close()
    ctx.synchronize()
    print(json.dumps({"case": args.case, "ok": True}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-moe", action="store_true")
    ap.add_argument("--no-decoder", action="store_true", help="skip the 7B decoder line")
    ap.add_argument("--no-cfg1", action="store_true", help="skip the single MX-int8 4096x4096 linear line")
    ap.add_argument("--no-ppo", action="store_true")
    ap.add_argument("--no-shard", action="store_true", help="N > 1: skip the column-sharded / expert-parallel forms")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--copies", type=int, default=COPIES,
                    help="distinct weight-pair copies rotated per step (default 8 = 383 MB)")
    ap.add_argument("--case", choices=["gemm512", "gemv1", "pair1", "moe", "decode7b"],
                    help="profiling: run one small workload (nothing timed) and exit")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.case:
        run_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
