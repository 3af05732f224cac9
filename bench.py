#!/usr/bin/env python
"""bench.py -- Qwen2.5-7B-shape Q4_K decode on B200 through liblalb.so.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl lalb|reference]

A step is one decode token of the matmul set: 28 layers x (qkv 4608x3584,
o 3584x3584, gate/up 37888x3584 with fused SwiGLU, down 3584x18944), all
Q4_K, plus the 152064x3584 int8 LM head with argmax -- 4.22 GB of weights
streamed from HBM per token (inputs larger than L2, so no flush is needed).
Weights are seeded N(0, 0.02) drawn and quantized on the GPU by the library;
the hidden state is seeded N(0, 1).  Attention is outside the measured path
(the q projection stands in for the attention output).

One JSON line on rank 0.  Under torchrun (N > 1) the ranks decode the SAME
token tensor-parallel (strong scaling): every rank holds a row shard of the
gate/up, down and LM-head matrices (qkv and o whole), and the persistent
kernels exchange rows over NVLink.  After the timed region the sharded token
is checked against a one-GPU decoder built on rank 0 from the same seeds
(`tp_check`); a mismatch fails the run.
`--impl reference` times the CPU kernels (AVX2 + OpenMP port of the
reference's absent lal_q4k_kernel.h / lal_q8_kernel.h) on the host cores,
with the OpenMP team set to the host's core count.
"""
import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(n_layer=28, hidden=3584, q_rows=3584, kv_rows=512, ffn=18944, vocab=152064)
METRIC = "Q4_K GEMV HBM GB/s (% of peak); 7B-shape decode tok/s at 1/2/4/8 B200"
WORKLOAD = ("qwen2.5-7b-shape decode matmul set: 28 layers x (qkv 4608x3584, o 3584x3584, "
            "gate/up 37888x3584 + fused SwiGLU, down 3584x18944) Q4_K + 152064x3584 int8 "
            "LM head + argmax, batch 1")
FALLBACK_HBM_GBS = 6650.0


def q4k_bytes(rows, K):
    return rows * (K // 256) * 144


def layer_mats(c):
    """(rows, K) of the four Q4_K matrices of one layer."""
    return [(c["q_rows"] + 2 * c["kv_rows"], c["hidden"]), (c["hidden"], c["q_rows"]),
            (2 * c["ffn"], c["hidden"]), (c["hidden"], c["ffn"])]


def algorithmic_bytes(c):
    """Bytes that must cross HBM per token: weights + activations in/out."""
    per_layer = [q4k_bytes(rows, K) + 4 * K + 4 * rows for rows, K in layer_mats(c)]
    head = c["vocab"] * c["hidden"] + 4 * c["vocab"] + 4 * c["hidden"] + 4
    return per_layer, head


def decode_config(c, world, persistent=True):
    """The decode line's `config`, shared by both arms so that they describe
    the same workload at the same N."""
    per_layer_b, head_b = algorithmic_bytes(c)
    tok_bytes = c["n_layer"] * sum(per_layer_b) + head_b
    return {"workload": WORKLOAD, "n_layer": c["n_layer"], "global_batch": 1, "seq_len": 1,
            "parallelism": "tp%d (row shards, in-kernel NVLink exchange)" % world
                           if world > 1 else "single",
            "path": "persistent" if persistent else "kernels",
            "l2": "inputs larger than L2: %.2f GB of weights streamed per step" % (tok_bytes / 1e9),
            "bytes_per_step": tok_bytes}


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(name, key):
    """A dram-bytes figure (`key: value` line) from a committed ncu summary."""
    p = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(p):
            if line.startswith(key + ":"):
                return float(line.split(":")[1])
    except (OSError, ValueError):
        pass
    return None


# --------------------------------------------------------------------------
# clocks during the timed region
# --------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id):
        self.bus_id = bus_id.lower()
        self.proc = None

    def start(self):
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + self.QUERY, "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.tmp.seek(0)
        rows = [r.split(", ") for r in self.tmp.read().strip().splitlines()]
        os.unlink(self.tmp.name)
        mine = [r for r in rows if len(r) >= 10 and r[1].lower().endswith(self.bus_id[-12:])]
        if not mine:
            return None

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None

        sm = [v for v in (num(r[2]) for r in mine) if v is not None]
        power = [v for v in (num(r[4]) for r in mine) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in mine for n, v in zip(names, r[6:10]) if v.strip() == "Active"})
        busy = sorted(sm)[len(sm) // 4:] if sm else []
        return {"sm_mhz": statistics.median(busy) if busy else None,
                "sm_max_mhz": num(mine[0][3]), "power_w_max": max(power) if power else None,
                "reasons": reasons, "samples": len(sm)}


# --------------------------------------------------------------------------
# the GPU arm
# --------------------------------------------------------------------------
def build_decoder(ctx, lb, torch, c, seed, n_rank=1, rank=0):
    """Seeded N(0,0.02) weights drawn and quantized on the GPU.  With
    n_rank > 1 every rank draws the same full matrices and keeps (quantizes)
    only its row shard."""
    big = max(max(r * k for r, k in layer_mats(c)), c["vocab"] * c["hidden"])
    tmp = torch.empty(big, dtype=torch.float32, device="cuda")
    layers = []
    for l in range(c["n_layer"]):
        mats = []
        for j, (rows, K) in enumerate(layer_mats(c)):
            w = tmp[: rows * K].view(rows, K)
            ctx.fill_normal(w, seed=seed + 16 * l + j, sigma=0.02)
            r0, r1 = lb.tp_range(c, j, n_rank, rank)
            mats.append(ctx.q4k_quantize(w[r0:r1]))
        layers.append(mats)
    w = tmp[: c["vocab"] * c["hidden"]].view(c["vocab"], c["hidden"])
    ctx.fill_normal(w, seed=seed + 9999, sigma=0.02)
    r0, r1 = lb.tp_range(c, 4, n_rank, rank)
    lm_q, lm_s = ctx.q8_quantize_rows(w[r0:r1])
    torch.cuda.synchronize()
    del tmp, w
    torch.cuda.empty_cache()   # the fp32 staging buffer is not needed any more
    dec = lb.Decoder(ctx, **c, n_rank=n_rank, rank=rank)
    for l, m in enumerate(layers):
        dec.set_layer_shard(rank, l, *m)
    dec.set_lm_head_shard(rank, lm_q, lm_s)
    return dec, layers, (lm_q, lm_s)


def gemv_standalone(ctx, torch, stream, reps=200, ncopies=8):
    """The single 18944x3584 Q4_K GEMV with the fused quantizer; weight
    copies (8 x 38 MB = 305 MB, > 2x L2) rotated so every launch streams
    from HBM."""
    rows, K = 18944, 3584
    copies = []
    w = torch.empty(rows * K, dtype=torch.float32, device="cuda")
    for i in range(ncopies):
        ctx.fill_normal(w, seed=500 + i, sigma=0.02)
        copies.append(ctx.q4k_quantize(w.view(rows, K)))
    del w
    x = torch.empty(K, dtype=torch.float32, device="cuda")
    ctx.fill_normal(x, seed=600, sigma=1.0)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    with torch.cuda.stream(stream):
        for i in range(16):
            ctx.matmul_q4_k(copies[i % ncopies], x, rows, K, out=y)
    torch.cuda.synchronize()
    # the timed launches are replayed from a CUDA graph: no host overhead
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(reps):
            ctx.matmul_q4_k(copies[i % ncopies], x, rows, K, out=y)
    with torch.cuda.stream(stream):
        g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / reps
    nbytes = q4k_bytes(rows, K) + 4 * K + 4 * rows
    return {"shape": [rows, K], "us_per_launch": round(us, 3), "bytes": nbytes,
            "gbs": round(nbytes / us / 1e3, 1)}


STE = dict(n_layer=8, d=448, ffn=1792, vocab=32768, rows=1024)


def run_ste_case(args, ctx=None):
    """The seed STE model's forward matmuls (8 layers, d=448, FFN 1792, vocab
    32768) on X 1024 x 448 fp32: per-element CORE/BINARY/PRUNE weights drawn
    10/50/40, packed as int8 codes with a per-row scale; every matmul on the
    tcgen05 GEMM that decodes the codes on chip (exact fp16) against the
    activations as two fp16 parts.  Five weight sets (larger than L2 together)
    are used in turn.  Returns its own JSON line (`--case ste`; the decode line
    carries it as "ste")."""
    import torch

    import lalmodel_b200 as lb

    c = STE
    own_ctx = ctx is None
    ctx = ctx or lb.Context(0)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(55)
    M, d, f = c["rows"], c["d"], c["ffn"]
    shapes = [(3 * d, d), (d, d), (f, d), (d, f)] * c["n_layer"] + [(c["vocab"], d)]
    nsets = 5   # 34 MB of codes each: 170 MB in rotation, more than L2
    sets = []
    for ws in range(nsets):
        layers = []
        for i, (rows, K) in enumerate(shapes):
            W = torch.empty((rows, K), dtype=torch.float32, device="cuda")
            ctx.fill_normal(W, seed=900 + 97 * ws + i, sigma=0.02)
            u = torch.rand((rows, K), generator=gen, device="cuda")
            state = torch.where(u < 0.10, 0, torch.where(u < 0.60, 1, 2)).to(torch.uint8)
            codes, srow = lb.LogicLayer.pack(ctx, W, state)
            bias = torch.zeros(rows, dtype=torch.float32, device="cuda")
            layers.append(lb.LogicLayer(ctx, codes, srow, bias, max_rows=M))
            del W, u, state
        sets.append(layers)
    X = torch.empty((M, d), dtype=torch.float32, device="cuda")
    X2 = torch.empty((M, f), dtype=torch.float32, device="cuda")
    ctx.fill_normal(X, seed=7, sigma=1.0)
    ctx.fill_normal(X2, seed=8, sigma=1.0)
    outs = [torch.empty((M, rows), dtype=torch.float32, device="cuda") for rows, _ in shapes]
    flops = sum(2.0 * M * rows * K for rows, K in shapes)
    weight_bytes = sum(rows * K + rows * 8 for rows, K in shapes)   # int8 codes + scale, bias
    stream = torch.cuda.Stream()

    def step(layers):
        for L, (rows, K), Y in zip(layers, shapes, outs):
            L.forward(X if K == d else X2, Y)

    with torch.cuda.stream(stream):
        for layers in sets:
            step(layers)   # first calls set kernel attributes outside the capture
    torch.cuda.synchronize()
    graphs = []
    for layers in sets:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step(layers)
        graphs.append(g)
    props = torch.cuda.get_device_properties(0)
    sampler = ClockSampler("%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id,
                                                 props.pci_device_id))
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            graphs[i % nsets].replay()
    torch.cuda.synchronize()
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(args.steps):
            graphs[i % nsets].replay()
        e1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    tflops = flops / (ms * 1e-3) / 1e12

    # end to end through the public entry point: the step's activations copied
    # in from pinned host memory, the first row of the LM-head output copied back
    hx, hx2 = X.cpu().pin_memory(), X2.cpu().pin_memory()
    hy = torch.empty(c["vocab"], dtype=torch.float32).pin_memory()
    n_e2e = max(5, min(args.steps, 50))
    with torch.cuda.stream(stream):
        for i in range(2):
            graphs[i % nsets].replay()
        stream.synchronize()
        t0 = time.perf_counter()
        for i in range(n_e2e):
            X.copy_(hx, non_blocking=True)
            X2.copy_(hx2, non_blocking=True)
            graphs[i % nsets].replay()
            hy.copy_(outs[-1][0], non_blocking=True)
            stream.synchronize()
        e2e_s = (time.perf_counter() - t0) / n_e2e
    e2e = {"value": round(flops / e2e_s / 1e12, 2), "unit": "TFLOP/s",
           "h2d_bytes_per_step": int(hx.numel() * 4 + hx2.numel() * 4),
           "d2h_bytes_per_step": int(hy.numel() * 4)}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            bf16 = float(json.load(fh)["bf16_tflops"])
        kind = "measured bf16 burst (cuBLAS; fp16 runs at the bf16 rate)"
    except Exception:
        bf16, kind = 1590.0, "fallback bf16"
    with torch.cuda.stream(stream):
        f16_mma = ctx.measure_mma_peak(lb.MMA_F16)
    # launches per step: per matmul the token preparation and the GEMM, plus
    # the split-sum where K is split over CTAs (the library's cost model:
    # fewer 128 x 128 tiles than 148 SMs, waves x (K-blocks per CTA + 6) + 10
    # for the split-sum launch)
    def splits(rows, K):
        tiles, nkb = -(-rows // 128) * -(-M // 128), -(-K // 64)
        best, cost = 1, nkb + 6
        if tiles < 148:
            for sp in range(2, min(nkb, 16) + 1):
                per = -(-nkb // sp)
                se = -(-nkb // per)
                cc = -(-tiles * se // 148) * (per + 6) + 10
                if cc < cost:
                    best, cost = se, cc
        return best
    launches = sum(2 + (splits(rows, K) > 1) for rows, K in shapes)
    # the CPU port (the oracle's OpenMP restatement of the per-element forward)
    # on a bounded sample: the first layer's qkv over 64 rows, repeated for
    # ~cpu_seconds, scaled to the step's flops
    cpu = None
    if not args.no_cpu:
        O = _cpu_lib()
        codes, srow, bias = (t.cpu().numpy() for t in sets[0][0]._keep)
        xs = X[:64].cpu().numpy()
        rows, K = shapes[0]
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < args.cpu_seconds:
            O.logic_forward(codes, srow, bias, xs)
            n += 1
        dt = (time.perf_counter() - t0) / n
        cpu_tflops = 2.0 * 64 * rows * K / dt / 1e12
        cpu = {"value": round(cpu_tflops, 4), "unit": "TFLOP/s", "cores": O.lib().lalb_cpu_threads(),
               "kind": "port",
               "sample": "%d x layer-0 qkv (%dx%d codes) over 64 rows, %.2f ms each; step time "
                         "at this rate %.1f ms" % (n, rows, K, dt * 1e3, flops / (cpu_tflops * 1e12) * 1e3)}
    line = {"case": "seed-ste-forward", "metric": "seed STE forward matmuls TFLOPS",
            "value": round(tflops, 2), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 codes decoded to exact fp16 x activations as fp16 hi+lo parts under a per-row "
                     "power of two, fp32 accumulate",
            "data": "synthetic: seeded N(0,0.02) weights, per-element states 10/50/40, X N(0,1)",
            "config": {"workload": "seed STE forward: 8 x (qkv 1344x448, o 448x448, fc 1792x448, "
                                   "down 448x1792) + LM head 32768x448 on X 1024x448",
                       "flops_per_step": flops, "gemm_calls_per_step": len(shapes),
                       "l2": "inputs larger than L2: %d weight sets of %.0f MB used in turn"
                             % (nsets, weight_bytes / 1e6)},
            "roofline": {"kernel": "logic_gemm_kernel", "bound": "tensor", "achieved": round(tflops, 2),
                         "tensor_work": round(2 * tflops, 2), "peak": bf16,
                         "peak_kind": kind, "unit": "TFLOP/s",
                         "frac": round(2 * tflops / bf16, 4),
                         "f16_mma_peak": round(f16_mma, 1),
                         "frac_of_f16_mma_peak": round(2 * tflops / f16_mma, 4),
                         "note": "tensor_work = 2 x useful: the B_hi and B_lo products",
                         "traffic": None},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches * args.steps,
            "clocks": clocks}
    for layers in sets:
        for L in layers:
            L.close()
    if own_ctx:
        ctx.close()
    return line


PREFILL_T = 512


def run_prefill_case(args, ctx=None, rank=0, world=1, dist=None):
    """Qwen2.5-7B-shape prefill: T = 512 tokens through every Q4_K matrix of
    the 28 layers (qkv 4608x3584, o 3584x3584, gate/up 37888x3584, down
    3584x18944) on the tcgen05 prefill kernel.  One step = the 112 matmuls;
    the metric is int8-equivalent ops (2 T rows K) per second.  Returns its own
    JSON line (`--case prefill`; the decode line carries it as "prefill").

    At N GPUs (one process each, `dist` initialised) the layer is split the
    tensor-parallel way, so that each attention and MLP block needs one
    exchange: qkv by rows (rows / N), o along K, gate/up by rows in pairs (the
    gate and up rows of the rank's FFN slice, so SwiGLU stays on the rank),
    down along K (the same FFN slice); after o and after down an NCCL
    all-reduce sums the [T][hidden] partial outputs.  K splits follow
    super-block boundaries (o: 14 super-blocks, down: 74, as even as they go).
    value = the whole model's ops over the slowest rank's step time.  A check
    on rank 0 compares its gate/up shard with those rows of the whole matrix
    (bit-identical) and the all-reduced down output with the whole down matrix
    on one GPU (the partial sums are added in another order: within 1e-5)."""
    import torch

    import lalmodel_b200 as lb

    c = CFG
    T = PREFILL_T
    own_ctx = ctx is None
    ctx = ctx or lb.Context(torch.cuda.current_device())
    mats = layer_mats(c)
    hid, ffn = c["hidden"], c["ffn"]

    def part(n):
        """[lo, hi) of this rank's share of n items, as even as it goes."""
        return n * rank // world, n * (rank + 1) // world

    q0, q1 = part(mats[0][0])                    # qkv rows
    o0, o1 = (256 * v for v in part(hid // 256))  # o: K columns
    f0, f1 = (256 * v for v in part(ffn // 256))  # FFN slice: gate/up rows, down K columns
    big = max(r * k for r, k in mats)
    tmp = torch.empty(big, dtype=torch.float32, device="cuda")
    wq, q4k_o, w_check = [], None, {}

    def shard(q, j, rows, K):
        """This rank's part of the whole Q4_K matrix q (rows x K), as its own
        contiguous Q4_K matrix: (bytes, rows, K)."""
        b = q.view(rows, K // 256, 144)
        if j == 0:
            return b[q0:q1].reshape(-1).clone(), q1 - q0, K
        if j == 2:
            half = rows // 2
            return (torch.cat((b[f0:f1], b[half + f0:half + f1])).reshape(-1).clone(),
                    2 * (f1 - f0), K)
        k0, k1 = (o0, o1) if j == 1 else (f0, f1)
        return b[:, k0 // 256:k1 // 256].reshape(-1).clone(), rows, k1 - k0

    for l in range(c["n_layer"]):
        for j, (rows, K) in enumerate(mats):
            w = tmp[: rows * K].view(rows, K)
            ctx.fill_normal(w, seed=1234 + 16 * l + j, sigma=0.02)
            q = ctx.q4k_quantize(w)   # the whole matrix, the same bytes on every rank
            if l == 0 and j == 1:
                q4k_o = q.cpu().numpy()   # the CPU sample's matrix
            if world > 1:
                if l == 0 and j in (2, 3) and rank == 0:
                    w_check[j] = q        # layer 0's gate/up and down, whole, for the check
                wq.append(shard(q, j, rows, K))
            else:
                wq.append((q, rows, K))
            del q
    torch.cuda.synchronize()
    del tmp, w
    torch.cuda.empty_cache()
    X = {K: torch.empty((T, K), dtype=torch.float32, device="cuda") for K in {k for _, k in mats}}
    for i, K in enumerate(sorted(X)):
        ctx.fill_normal(X[K], seed=70 + i, sigma=1.0)
    # the inputs of the K-split matrices: this rank's columns of the attention
    # output (o) and of the SwiGLU output (down), which the rank computes itself
    Xo = X[hid][:, o0:o1].contiguous() if world > 1 else X[hid]
    Xd = X[ffn][:, f0:f1].contiguous() if world > 1 else X[ffn]
    x_in = [X[hid], Xo, X[hid], Xd]
    ws = torch.empty(max(lb.prefill_ws_bytes(r, k, T) for _, r, k in wq), dtype=torch.uint8, device="cuda")
    # outputs: qkv and gate/up shards; o and down [T][hidden] partial sums, all-reduced
    Y = [torch.empty((T, wq[j][1]), dtype=torch.float32, device="cuda") for j in range(4)]
    calls = [(wq[4 * l + j][0], wq[4 * l + j][1], wq[4 * l + j][2], x_in[j], Y[j], world > 1 and j in (1, 3))
             for l in range(c["n_layer"]) for j in range(4)]
    ops = sum(2.0 * T * rows * K for _ in range(c["n_layer"]) for rows, K in mats)
    stream = torch.cuda.Stream()

    def step():
        for P, rows, K, x, y, reduce in calls:
            ctx.matmul_q4_k_prefill(P, rows, K, x, ws=ws, out=y)
            if reduce:
                dist.all_reduce(y)

    with torch.cuda.stream(stream):
        step()   # first calls set kernel attributes outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step()
    props = torch.cuda.get_device_properties(0)
    sampler = ClockSampler("%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id,
                                                 props.pci_device_id))
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = max_over_ranks(torch, dist, world, e0.elapsed_time(e1) / args.steps)
    tops = ops / (ms * 1e-3) / 1e12

    tp_check = None
    if world > 1:
        # layer 0's gate/up shard and all-reduced down against the whole matrices on rank 0
        with torch.cuda.stream(stream):
            for j in (2, 3):
                P, rows, K, x, y, reduce = calls[j]
                ctx.matmul_q4_k_prefill(P, rows, K, x, ws=ws, out=y)
                if reduce:
                    dist.all_reduce(y)
        torch.cuda.synchronize()
        bad = torch.zeros(1, dtype=torch.int32, device="cuda")
        if rank == 0:
            (gr, gk), (dr, dk) = mats[2], mats[3]
            gu = ctx.matmul_q4_k_prefill(w_check[2], gr, gk, X[hid])
            dn = ctx.matmul_q4_k_prefill(w_check[3], dr, dk, X[ffn])
            torch.cuda.synchronize()
            half = gr // 2
            gu_mine = torch.cat((gu[:, f0:f1], gu[:, half + f0:half + f1]), dim=1)
            same = bool(torch.equal(gu_mine, Y[2]))
            rel = float(((Y[3].double() - dn.double()).norm() / dn.double().norm()).item())
            tp_check = {"gate_up_shard": "rank 0's %d of %d rows, T=%d" % (Y[2].shape[1], gr, T),
                        "gate_up_bit_identical": same,
                        "down_allreduced_normwise_rel_err": rel, "tolerance": 1e-5}
            bad.fill_(0 if same and rel < 1e-5 else 1)
            del gu, dn, gu_mine, w_check
        dist.all_reduce(bad, op=dist.ReduceOp.MAX)
        if int(bad.item()):
            if rank == 0:
                print(json.dumps({"case": "prefill-7b", "n_gpus": world, "tp_check": tp_check}), flush=True)
            raise SystemExit(3)

    # the tensor-core kernel alone: one gate/up launch, by events around it
    P, rows, K, x, y, _ = calls[2]
    with torch.cuda.stream(stream):
        ctx.matmul_q4_k_prefill(P, rows, K, x, ws=ws, out=y)   # tokens prepared
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_k = 20
        gk = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gk, stream=stream):
        for _ in range(n_k):
            ctx.matmul_q4_k_prefill(P, rows, K, x, ws=ws, out=y)
    with torch.cuda.stream(stream):
        gk.replay()
        k0.record(stream)
        gk.replay()
        k1.record(stream)
    torch.cuda.synchronize()
    gu_us = k0.elapsed_time(k1) * 1e3 / n_k

    # end to end through the public entry point: the step's token activations
    # copied in from pinned host memory, the last output copied back
    hx = {K: v.cpu().pin_memory() for K, v in X.items()}
    hy = torch.empty(Y[3].shape, dtype=torch.float32).pin_memory()
    n_e2e = max(5, min(args.steps, 30))
    if world > 1:
        dist.barrier()
    with torch.cuda.stream(stream):
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(n_e2e):
            for K, v in hx.items():
                X[K].copy_(v, non_blocking=True)
            g.replay()
            hy.copy_(Y[3], non_blocking=True)
        f1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(torch, dist, world, f0.elapsed_time(f1))
    e2e_tops = ops * n_e2e / (e2e_ms * 1e-3) / 1e12

    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            bf16 = float(json.load(fh)["bf16_tflops"])
        kind = "measured bf16 burst (cuBLAS)"
    except Exception:
        bf16, kind = 1590.0, "fallback bf16"
    # tensor work actually issued: per 64 weights 8 fp16 MMAs (two B parts)
    # + 1 bf16 min-term MMA of the same width = 2.25 x the int8-equivalent ops
    work = 2.25 * tops
    # the tensor pipe's own peaks, measured here: back-to-back M=128 N=256 MMAs
    # on every SM (kind::i8 is the int8 rate the metric's ops are counted in)
    with torch.cuda.stream(stream):
        peak_i8 = ctx.measure_mma_peak(lb.MMA_I8)
        peak_f16 = ctx.measure_mma_peak(lb.MMA_F16)

    cpu = None
    if not args.no_cpu and world == 1:
        O = _cpu_lib()
        L = O.lib()
        rows, K = mats[1]
        xs = X[K][:64].cpu().numpy()
        xq = np.empty(K, np.int8)
        sx = np.empty(K // 32, np.float32)
        sq = np.empty(K // 32, np.int32)
        y = np.empty(rows, np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < args.cpu_seconds:
            L.lalb_cpu_quantize_act(O._p(np.ascontiguousarray(xs[n % 64])), 1, K, O._p(xq), O._p(sx),
                                    O._p(sq))
            L.lalb_cpu_q4k_gemv(O._p(q4k_o), rows, K, O._p(xq), O._p(sx), O._p(sq), O._p(y))
            n += 1
        dt = (time.perf_counter() - t0) / n
        cpu_tops = 2.0 * rows * K / dt / 1e12
        cpu = {"value": round(cpu_tops, 5), "unit": "TOPS", "cores": L.lalb_cpu_threads(),
               "kind": "port",
               "sample": "%d tokens x the layer-0 o matrix (%dx%d Q4_K), one AVX2 GEMV per token "
                         "(the reference has no batched kernel), %.2f ms each; step time at this "
                         "rate %.1f s" % (n, rows, K, dt * 1e3, ops / (cpu_tops * 1e12))}
    in_bytes = sum(v.numel() * 4 for v in hx.values())
    line = {"case": "prefill-7b", "metric": "Qwen2.5-7B-shape prefill int8 TOPS (M=512)",
            "value": round(tops, 2), "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "int8 x uint4 semantics; tensor cores: fp16 sc*q (exact) x xq*sx in two fp16 "
                     "parts, min terms in three bf16 parts, fp32 accumulate",
            "data": "synthetic: seeded N(0,0.02) weights quantized to Q4_K on the GPU, seeded "
                    "N(0,1) activations",
            "config": {"workload": "qwen2.5-7b-shape prefill: %d tokens x %d layers x (qkv 4608x3584, "
                                   "o 3584x3584, gate/up 37888x3584, down 3584x18944) Q4_K"
                                   % (T, c["n_layer"]),
                       "tokens": T, "matmuls_per_step": len(calls), "ops_per_step": ops,
                       "parallelism": ("tp%d: qkv and gate/up by rows, o and down along K, an "
                                       "NCCL all-reduce of [T][hidden] after o and after down"
                                       % world) if world > 1 else "single",
                       "l2": "inputs larger than L2: %.2f GB of Q4_K weights per step, read as "
                             "they are (0.5625 B/weight)"
                             % (sum(r * k // 256 * 144 for _, r, k, _, _, _ in calls) / 1e9)},
            "roofline": {"kernel": "prefill_q4k_kernel", "bound": "tensor",
                         "achieved": round(work, 1), "peak": bf16, "peak_kind": kind,
                         "unit": "TFLOP/s", "frac": round(work / bf16, 4),
                         "note": "achieved = issued fp16/bf16 tensor work (2.25 x the int8-"
                                 "equivalent ops) over the whole step",
                         "mma_peaks": {"i8_tops": round(peak_i8, 1), "f16_tflops": round(peak_f16, 1),
                                       "how": "lalb_measure_mma_peak: back-to-back tcgen05.mma "
                                              "M=128 N=256 on every SM, this run"},
                         "frac_of_i8_mma_peak": round(tops / peak_i8, 4),
                         "frac_of_f16_mma_peak": round(work / peak_f16, 4),
                         "gate_up_launch_us": round(gu_us, 2),
                         "gate_up_tensor_tflops": round(2.25 * 2 * T * calls[2][1] * calls[2][2]
                                                        / (gu_us * 1e-6) / 1e12, 1),
                         "traffic": None},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_tops, 2), "unit": "TOPS", "h2d_bytes_per_step": in_bytes,
                    "d2h_bytes_per_step": hy.numel() * 4},
            "gpu_launches": args.steps * 2 * len(calls),
            "clocks": clocks}
    if tp_check is not None:
        line["tp_check"] = tp_check
    del g, gk
    del wq, X, Xo, Xd, x_in, Y, ws, calls
    torch.cuda.empty_cache()
    if own_ctx:
        ctx.close()
    return line


def run_prefill_standalone(args, rank, world, local_rank):
    """`--case prefill`: one GPU, or N under torchrun with row-sharded weights."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                timeout=datetime.timedelta(seconds=300))
    line = run_prefill_case(args, None, rank, world, dist if world > 1 else None)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def full_token_case(ctx, lb, torch, c, layers, lm, stream, h_in, am, warmup, peak,
                    start=512, steps=200):
    """The whole decode token as a GPU step: the same weights with decode
    attention over F32 KV caches (GQA, head_dim 128, 28 q heads over 4 KV
    heads at the 7B shape), positions start .. start + steps, the earlier
    positions' keys and values seeded at random.  A sub-measurement of the
    decode line (its headline is the matmul set, config 3)."""
    max_ctx = start + warmup + steps + 8
    dec = lb.Decoder(ctx, **c, head_dim=128, max_ctx=max_ctx, rope_theta=1e6)
    for l, m in enumerate(layers):
        dec.set_layer_shard(0, l, *m)
    dec.set_lm_head_shard(0, *lm)
    kv = []
    for l in range(c["n_layer"]):
        k = torch.empty((max_ctx, c["kv_rows"]), dtype=torch.float32, device="cuda")
        v = torch.empty_like(k)
        ctx.fill_normal(k, seed=3000 + 2 * l, sigma=1.0)
        ctx.fill_normal(v, seed=3001 + 2 * l, sigma=1.0)
        dec.set_kv_cache(l, k, v)
        kv.append((k, v))
    with torch.cuda.stream(stream):
        dec.set_position(start - warmup)
        for _ in range(warmup):
            dec.step(h_in, None, None, am)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            dec.step(h_in, None, None, am)
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    status = ctx.device_status()
    per_layer_b, head_b = algorithmic_bytes(c)
    kv_b = c["n_layer"] * 2 * c["kv_rows"] * 4 * (start + steps / 2.0)   # keys and values read, mean position
    tok_b = c["n_layer"] * sum(per_layer_b) + head_b + kv_b
    dec.close()
    del kv
    return {"tok_s": round(1000.0 / ms, 2), "ms_per_step": round(ms, 5),
            "context": "positions %d..%d (F32 KV caches, RoPE theta 1e6)" % (start, start + steps),
            "bytes_per_token": int(tok_b), "gbs": round(tok_b / (ms * 1e-3) / 1e9, 1),
            "frac": round(tok_b / (ms * 1e-3) / 1e9 / peak, 4), "steps": steps,
            "status": status}


def max_over_ranks(torch, dist, world, v):
    """The largest of every rank's v (a float), on every rank."""
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_gemv_case(args):
    """Only the single-GEMV workload (4 rotating copies, 153 MB > L2): a small
    case for profiler captures, not a bench line."""
    import torch

    import lalmodel_b200 as lb

    ctx = lb.Context(0)
    r = gemv_standalone(ctx, torch, torch.cuda.Stream(), reps=args.steps, ncopies=4)
    print(json.dumps({"case": "gemv", **r}), flush=True)
    ctx.close()


def run_trace_case(args, rank, world, local_rank):
    """Phase timeline of the persistent decode (one process per GPU under
    torchrun, tensor-parallel when N > 1): one traced token after 30 untimed
    ones; rank 0 prints, per phase kind, the median over layers of the grid
    barrier after the phase, the next phase's prologue and its work (us).
    A profiling aid, not a bench line."""
    import torch
    import torch.distributed as dist

    import lalmodel_b200 as lb

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                timeout=datetime.timedelta(seconds=300))
    c = CFG
    ctx = lb.Context(local_rank)
    dec, _, _ = build_decoder(ctx, lb, torch, c, seed=1234, n_rank=world, rank=rank)
    if world > 1:
        dec.connect(lb.exchange_handles(dec.ipc_handle()))
        dist.barrier()
    h = torch.empty(c["hidden"], dtype=torch.float32, device="cuda")
    ctx.fill_normal(h, seed=77, sigma=1.0)
    am = torch.empty(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(30):
            dec.step(h, None, None, am)
        tr = dec.trace_step(h)
    s.synchronize()
    if rank == 0:
        n_p = tr.shape[1]
        t0 = tr[:, 0, 0].min()
        work_end = tr[:, :, 0].max(0) - t0
        bar_left = np.median(tr[:, :, 1], 0) - t0
        pro = np.median(tr[:, :, 2], 0) - t0
        kinds = ["qkv", "o", "gate/up", "down"]
        rows = {k: [] for k in kinds}
        for p in range(n_p - 1):
            rows[kinds[p % 4]].append(((bar_left[p] - work_end[p]) / 1e3,
                                       (pro[p + 1] - bar_left[p]) / 1e3,
                                       (work_end[p + 1] - pro[p + 1]) / 1e3))
        # consumer warp 0 of every CTA: time spent waiting on its ring slots
        # against time spent on the math, and the producers' last copy issued
        # relative to the phase's prologue end (median CTA, median layer)
        cons = {k: [] for k in kinds}
        for p in range(n_p - 1):
            cons[kinds[p % 4]].append((np.median(tr[:, p, 3]) / 1e3, np.median(tr[:, p, 4]) / 1e3,
                                       np.median(tr[:, p, 5] - tr[:, p, 2]) / 1e3))
        out = {"case": "trace", "n_gpus": world,
               "token_us": round(float(tr[:, n_p - 1, 0].max() - t0) / 1e3, 1),
               "after_phase_us": {k: dict(zip(("barrier", "next_prologue", "next_work"),
                                              (round(float(v), 2)
                                               for v in np.median(np.array(rows[k]), 0))))
                                  for k in kinds},
               "consumer0_us": {k: dict(zip(("ring_wait", "math", "last_copy_after_prologue"),
                                            (round(float(v), 2)
                                             for v in np.median(np.array(cons[k]), 0))))
                                for k in kinds}}
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
    dec.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def shard_bytes(lb, c, n_rank, rank):
    """Weight and activation bytes that rank `rank` of `n_rank` streams per token."""
    total = 0
    for j, (rows, K) in enumerate(layer_mats(c)):
        r0, r1 = lb.tp_range(c, j, n_rank, rank)
        total += c["n_layer"] * (q4k_bytes(r1 - r0, K) + 4 * K + 4 * (r1 - r0))
    r0, r1 = lb.tp_range(c, 4, n_rank, rank)
    return total + (r1 - r0) * (c["hidden"] + 8) + 4 * c["hidden"] + 4


def phase_chain(dec, lb, torch, stream, h_in, am, args, c, per_layer_b, head_b, q4k_launches,
                q4k_bytes_tok):
    """The per-phase kernel chain (one launch per matvec) on the same weights:
    its step rate, and each kernel's duration from events between kernels."""
    dec.set_path(lb.Decoder.KERNELS)
    n_chain = max(20, min(args.steps, 300))
    with torch.cuda.stream(stream):
        for _ in range(3):
            dec.step(h_in, None, None, am)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(n_chain):
            dec.step(h_in, None, None, am)
        g1.record(stream)
        prof = np.median(np.array([dec.profile_step(h_in) for _ in range(5)]), axis=0)
    torch.cuda.synchronize()
    chain_ms = g0.elapsed_time(g1) / n_chain
    dec.set_path({"auto": lb.Decoder.AUTO, "kernels": lb.Decoder.KERNELS,
                  "persistent": lb.Decoder.PERSISTENT}[args.path])
    q4k_us = float(sum(prof[:q4k_launches]))
    head_us = float(prof[-1])
    kinds = ["qkv", "o", "gate_up", "down"]
    per_kind = {k: round(float(np.mean(prof[i:q4k_launches:4])), 2) for i, k in enumerate(kinds)}
    per_kind_gbs = {k: round(per_layer_b[i] / (per_kind[k] * 1e-6) / 1e9, 1)
                    for i, k in enumerate(kinds)}
    return {"tok_s": round(1000.0 / chain_ms, 2), "ms_per_step": round(chain_ms, 5),
            "launches_per_step": q4k_launches + 1, "q4k_us": q4k_us,
            "q4k_gbs": round(q4k_bytes_tok / (q4k_us * 1e-6) / 1e9, 1),
            "us_by_kind": per_kind, "gbs_by_kind": per_kind_gbs,
            "lm_head_us": round(head_us, 2),
            "lm_head_gbs": round(head_b / (head_us * 1e-6) / 1e9, 1)}


def run_gpu(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import lalmodel_b200 as lb

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                timeout=datetime.timedelta(seconds=300))
    c = CFG
    ctx = lb.Context(local_rank)
    # tensor parallel over the ranks: each GPU holds a row shard of every
    # matrix and all of them decode the same token
    tp = world > 1
    dec, layers, lm = build_decoder(ctx, lb, torch, c, seed=1234, n_rank=world, rank=rank)
    if tp:
        dec.connect(lb.exchange_handles(dec.ipc_handle()))
        dist.barrier()
    h_in = torch.empty(c["hidden"], dtype=torch.float32, device="cuda")
    ctx.fill_normal(h_in, seed=77, sigma=1.0)
    am = torch.empty(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.Stream()
    dec.set_path({"auto": lb.Decoder.AUTO, "kernels": lb.Decoder.KERNELS,
                  "persistent": lb.Decoder.PERSISTENT}[args.path])
    persistent = dec.path() == lb.Decoder.PERSISTENT
    launches = dec.launches_per_step()

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            dec.step(h_in, None, None, am)
    torch.cuda.synchronize()

    props = torch.cuda.get_device_properties(local_rank)
    bus = "%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
    sampler = ClockSampler(bus)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            dec.step(h_in, None, None, am)
        e1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    if world > 1:
        dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_per_step = ms_max / args.steps
    value = args.steps / (ms_max / 1000.0)   # tokens: every rank works on the same one

    per_layer_b, head_b = algorithmic_bytes(c)
    q4k_launches = 4 * c["n_layer"]
    q4k_bytes_tok = c["n_layer"] * sum(per_layer_b)
    tok_bytes = q4k_bytes_tok + head_b
    rank_bytes = shard_bytes(lb, c, world, rank)   # what this GPU streams per token
    peak, peak_kind = measured_peak()

    chain = None
    if not tp:
        chain = phase_chain(dec, lb, torch, stream, h_in, am, args, c, per_layer_b, head_b,
                            q4k_launches, q4k_bytes_tok)
    if persistent:
        # one launch per token: its duration is the step time measured above
        achieved = rank_bytes / (ms_per_step * 1e-3) / 1e9
        roofline = {"kernel": "decode_persistent_kernel (the whole token, one launch per GPU)",
                    "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                    "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                    "traffic": profile_traffic("decode_persistent_qwen7b_ncu.md",
                                               "traffic_bytes_per_launch") if not tp else None,
                    "bytes_per_launch": rank_bytes, "us_per_launch": round(ms_per_step * 1e3, 2)}
    else:
        q4k_us = chain["q4k_us"]
        achieved = q4k_bytes_tok / (q4k_us * 1e-6) / 1e9
        roofline = {"kernel": "q4k_gemv (the %d Q4_K matvec launches of a token)" % q4k_launches,
                    "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                    "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                    # measured DRAM/algorithmic ratio of the GEMV (ncu) x this average launch
                    "traffic": (lambda r: r and round(r * q4k_bytes_tok / q4k_launches))(
                        profile_traffic("q4k_gemv_decode7b_ncu.md", "traffic_ratio")),
                    "bytes_per_launch_avg": q4k_bytes_tok / q4k_launches,
                    "us_per_launch_avg": round(q4k_us / q4k_launches, 3)}
    roofline["step_gbs"] = round(rank_bytes / (ms_per_step * 1e-3) / 1e9, 1)

    # end to end through the host-buffer entry point (H2D input, D2H argmax)
    pinned = h_in.cpu().pin_memory()
    n_e2e = max(20, min(args.steps, 400))
    with torch.cuda.stream(stream):
        for _ in range(3):
            dec.step_host(pinned)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(n_e2e):
            dec.step_host(pinned)
        f1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([f0.elapsed_time(f1)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = n_e2e / (float(t.item()) / 1000.0)

    tp_check = check_tp_against_one_gpu(ctx, lb, torch, dist, dec, c, rank, world, stream) \
        if tp else None

    gemv = gemv_standalone(ctx, torch, stream) if rank == 0 else None

    # configs 4 and 5 on one GPU, each a compact sub-line of this one
    subs = {}
    if world == 1 and not args.no_sub:
        subs["full_token"] = full_token_case(ctx, lb, torch, c, layers, lm, stream, h_in, am,
                                             args.warmup, peak)
        sub_args = argparse.Namespace(**vars(args))
        sub_args.steps, sub_args.warmup = 20, 3
        sub_args.cpu_seconds = min(args.cpu_seconds, 5.0)
        del dec
        torch.cuda.empty_cache()
        dec = None
        for name, fn in (("prefill", run_prefill_case), ("ste", run_ste_case)):
            sub = fn(sub_args, ctx)
            subs[name] = {k: sub[k] for k in ("metric", "value", "unit", "ms_per_step", "steps",
                                              "dtype", "config", "roofline", "e2e",
                                              "cpu_baseline", "gpu_launches", "clocks")}
    elif world > 1 and not args.no_sub:
        # config 4 at N GPUs: the prefill with row-sharded weights (every rank)
        sub_args = argparse.Namespace(**vars(args))
        sub_args.steps, sub_args.warmup, sub_args.no_cpu = 20, 3, True
        dist.barrier()
        sub = run_prefill_case(sub_args, ctx, rank, world, dist)
        subs["prefill"] = {k: sub[k] for k in ("metric", "value", "unit", "ms_per_step", "steps",
                                               "dtype", "config", "roofline", "e2e", "gpu_launches",
                                               "clocks", "tp_check") if k in sub}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_sample(layers, lm, c, budget_s=args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8 (q4 x i8 dp4a -> int32 per 32-block, fp32 terms, f64 row sum)",
            "data": "synthetic: seeded N(0,0.02) weights quantized on the GPU (Q4_K min-max, "
                    "int8 per-row LM head); seeded N(0,1) hidden state",
            "config": decode_config(c, world, persistent),
            "roofline": roofline,
            "phase_chain": chain,
            "gemv": gemv and {**gemv, "frac": round(gemv["gbs"] / peak, 4)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": 4 * c["hidden"], "d2h_bytes_per_step": 4},
            "gpu_launches": args.steps * launches,
            "clocks": clocks,
        }
        if tp_check is not None:
            line["tp_check"] = tp_check
        line.update(subs)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()   # no rank unmaps its exchange buffer while a peer may still use it
    if dec is not None:
        dec.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    if tp_check is not None and not tp_check["ok"]:
        sys.exit(3)


TP_CHECK_TOL = 1e-4   # normwise, after the rows of every shard are joined


def check_tp_against_one_gpu(ctx, lb, torch, dist, dec, c, rank, world, stream, tokens=3):
    """Runs `tokens` tokens through the tensor-parallel decoder (every rank)
    and through a one-GPU decoder that rank 0 builds from the same seeds, and
    compares the final residual stream, the joined logits and the argmax
    (first maximum over the whole vocabulary).  Every rank takes the same
    collective steps."""
    r0, r1 = lb.tp_range(c, 4, world, rank)
    shard = max(lb.tp_range(c, 4, world, j)[1] - lb.tp_range(c, 4, world, j)[0]
                for j in range(world))
    h_out = torch.empty(c["hidden"], dtype=torch.float32, device="cuda")
    logits = torch.zeros(c["vocab"], dtype=torch.float32, device="cuda")
    am = torch.empty(1, dtype=torch.int32, device="cuda")
    h_in = torch.empty(c["hidden"], dtype=torch.float32, device="cuda")
    outs = []
    for t in range(tokens):
        ctx.fill_normal(h_in, seed=4100 + t, sigma=1.0)
        with torch.cuda.stream(stream):
            dec.step(h_in, h_out, logits, am)
        stream.synchronize()
        part = torch.zeros(shard, dtype=torch.float32, device="cuda")
        part[: r1 - r0] = logits[r0:r1]
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        outs.append((h_out.clone(), parts, int(am.item())))
    dist.barrier()
    result = None
    if rank == 0:
        one, _, _ = build_decoder(ctx, lb, torch, c, seed=1234, n_rank=1, rank=0)
        ref_h = torch.empty_like(h_out)
        ref_l = torch.empty_like(logits)
        ref_am = torch.empty_like(am)
        err_h, err_l, same_am, exact = 0.0, 0.0, True, []
        for t, (h_tp, parts, am_tp) in enumerate(outs):
            ctx.fill_normal(h_in, seed=4100 + t, sigma=1.0)
            with torch.cuda.stream(stream):
                one.step(h_in, ref_h, ref_l, ref_am)
            stream.synchronize()
            joined = torch.cat([p[: lb.tp_range(c, 4, world, j)[1] - lb.tp_range(c, 4, world, j)[0]]
                                for j, p in enumerate(parts)])

            def nerr(a, b):
                return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))

            err_h = max(err_h, nerr(h_tp, ref_h))
            err_l = max(err_l, nerr(joined, ref_l))
            same_am = same_am and am_tp == int(ref_am.item())
            exact.append(float((joined == ref_l).float().mean()))
        one.close()
        result = {"tokens": tokens, "max_rel_err_h": err_h, "max_rel_err_logits": err_l,
                  "argmax_equal": same_am, "logits_bit_identical_frac": min(exact),
                  "tol": TP_CHECK_TOL, "against": "one-GPU decoder, same seeds, on rank 0",
                  "ok": bool(same_am and err_h <= TP_CHECK_TOL and err_l <= TP_CHECK_TOL)}
    flag = torch.tensor([0 if rank != 0 else (1 if result["ok"] else 2)], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MAX)
    if rank != 0:
        result = {"ok": int(flag.item()) == 1}
    return result


# --------------------------------------------------------------------------
# CPU: the oracle's AVX2 + OpenMP kernels (port of the reference's absent
# CPU kernels) timed on the host cores
# --------------------------------------------------------------------------
def host_cores():
    """Host cores this process may run on (torchrun's OMP_NUM_THREADS=1 is
    not a statement about the machine)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def _cpu_lib():
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import _oracle as O  # builds oracle/liblalb_oracle.so if needed

    O.lib().lalb_cpu_set_threads(host_cores())
    return O


def cpu_layer_and_head(O, L, mats, lmq, lms, c, h):
    """One decoder layer of the matmul chain + the LM head on the CPU.
    Returns (seconds for the layer, seconds for the head)."""
    p = O._p
    hid, qr, kv, ffn = c["hidden"], c["q_rows"], c["kv_rows"], c["ffn"]
    xq = np.empty(max(hid, ffn), np.int8)
    sx = np.empty(max(hid, ffn) // 32, np.float32)
    sq = np.empty(max(hid, ffn) // 32, np.int32)
    t0 = time.perf_counter()
    qkv = np.empty(qr + 2 * kv, np.float32)
    L.lalb_cpu_quantize_act(p(O.rms_normalise(h)), 1, hid, p(xq), p(sx), p(sq))
    L.lalb_cpu_q4k_gemv(p(mats[0]), qr + 2 * kv, hid, p(xq), p(sx), p(sq), p(qkv))
    L.lalb_cpu_quantize_act(p(np.ascontiguousarray(qkv[:qr])), 1, qr, p(xq), p(sx), p(sq))
    o = np.empty(hid, np.float32)
    L.lalb_cpu_q4k_gemv(p(mats[1]), hid, qr, p(xq), p(sx), p(sq), p(o))
    h = (h + o).astype(np.float32)
    L.lalb_cpu_quantize_act(p(O.rms_normalise(h)), 1, hid, p(xq), p(sx), p(sq))
    gu = np.empty(2 * ffn, np.float32)
    L.lalb_cpu_q4k_gemv(p(mats[2]), 2 * ffn, hid, p(xq), p(sx), p(sq), p(gu))
    gu = gu.reshape(-1, 2, 32)
    act = O.swiglu(gu[:, 0].reshape(-1), gu[:, 1].reshape(-1))
    L.lalb_cpu_quantize_act(p(act), 1, ffn, p(xq), p(sx), p(sq))
    d = np.empty(hid, np.float32)
    L.lalb_cpu_q4k_gemv(p(mats[3]), hid, ffn, p(xq), p(sx), p(sq), p(d))
    h = (h + d).astype(np.float32)
    t1 = time.perf_counter()
    L.lalb_cpu_quantize_act(p(O.rms_normalise(h)), 1, hid, p(xq), p(sx), p(sq))
    logits = np.empty(lmq.shape[0], np.float32)
    L.lalb_cpu_q8_lmhead(p(lmq), p(lms), lmq.shape[0], hid, p(xq), p(sx), p(logits))
    t2 = time.perf_counter()
    return t1 - t0, t2 - t1


def cpu_timed(O, mats, lmq, lms, c, warmup, max_steps, budget_s):
    L = O.lib()
    h = O.normal(c["hidden"], seed=77)
    for _ in range(max(1, warmup)):
        cpu_layer_and_head(O, L, mats, lmq, lms, c, h)
    tl, th = [], []
    t_start = time.perf_counter()
    while len(tl) < max_steps and (not tl or time.perf_counter() - t_start < budget_s):
        a, b = cpu_layer_and_head(O, L, mats, lmq, lms, c, h)
        tl.append(a)
        th.append(b)
    t_layer, t_head = statistics.median(tl), statistics.median(th)
    tok_s = 1.0 / (c["n_layer"] * t_layer + t_head)
    sample = ("%d x (1 decoder layer %.2f ms + LM head %.2f ms) on the same weights; "
              "token time = %d layers + head" % (len(tl), 1e3 * t_layer, 1e3 * t_head, c["n_layer"]))
    return tok_s, len(tl), L.lalb_cpu_threads(), sample


def cpu_baseline_sample(layers, lm, c, budget_s):
    """Layer 0's weights and the LM head copied from the GPU; the host cores
    run one layer + the head repeatedly for ~budget_s seconds."""
    O = _cpu_lib()
    mats = [m.cpu().numpy().reshape(-1) for m in layers[0]]
    lmq, lms = lm[0].cpu().numpy(), lm[1].cpu().numpy()
    tok_s, n, cores, sample = cpu_timed(O, mats, lmq, lms, c, 2, 10 ** 6, budget_s)
    return {"value": round(tok_s, 3), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": sample}


def run_reference(args, rank, world):
    """The CPU arm: the same metric and workload on the host cores."""
    if rank != 0:
        return
    O = _cpu_lib()
    c = CFG
    mats = []
    for j, (rows, K) in enumerate(layer_mats(c)):
        w = O.normal(rows * K, seed=1234 + j, sigma=0.02).reshape(rows, K)
        mats.append(O.q4k_quantize(w).reshape(-1))
        del w
    w = O.normal(c["vocab"] * c["hidden"], seed=1234 + 9999, sigma=0.02).reshape(c["vocab"], c["hidden"])
    lmq, lms = O.q8_quantize_rows(w)
    del w
    tok_s, n, cores, sample = cpu_timed(O, mats, lmq, lms, c, args.warmup, args.steps,
                                        args.cpu_seconds * 4)
    line = {"impl": "reference", "metric": METRIC, "value": round(tok_s, 3), "unit": "tok/s",
            "n_gpus": world, "steps": n, "warmup": args.warmup,
            "ms_per_step": round(1e3 / tok_s, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8 (AVX2 maddubs -> int32, fp32 combine)",
            "data": "synthetic: seeded N(0,0.02) weights quantized on the CPU, N(0,1) hidden state",
            "config": decode_config(c, world),
            "host": "the whole token on rank 0's host cores (OpenMP, %d threads)" % cores,
            "cpu_baseline": {"value": round(tok_s, 3), "unit": "tok/s", "cores": cores,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(tok_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="lalb", choices=["lalb", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-sub", action="store_true",
                    help="skip the prefill and seed-STE sub-measurements of the decode line")
    ap.add_argument("--n-layer", type=int, default=CFG["n_layer"],
                    help="fewer layers: only for profiling captures, not a bench line")
    ap.add_argument("--vocab", type=int, default=CFG["vocab"],
                    help="smaller LM head: only for profiling captures, not a bench line")
    ap.add_argument("--path", default="auto", choices=["auto", "kernels", "persistent"],
                    help="decoder path: one persistent kernel per token, or one kernel per matvec")
    ap.add_argument("--case", default="decode", choices=["decode", "gemv", "ste", "prefill", "trace"],
                    help="gemv: only the single 18944x3584 GEMV, for profiler captures; "
                         "ste: the seed STE model's forward matmuls (its own line); "
                         "prefill: the 7B-shape prefill of 512 tokens (its own line); "
                         "trace: the persistent decode's phase timeline (profiling aid)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    CFG["n_layer"] = args.n_layer
    CFG["vocab"] = args.vocab
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
    elif args.case == "gemv":
        run_gemv_case(args)
    elif args.case == "ste":
        print(json.dumps(run_ste_case(args)), flush=True)
    elif args.case == "trace":
        run_trace_case(args, rank, world, local_rank)
    elif args.case == "prefill":
        run_prefill_standalone(args, rank, world, local_rank)
    else:
        run_gpu(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
