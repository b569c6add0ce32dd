"""Benchmark: rel-pos MHA encoder frames/s on B200.

One step = one RelPositionMultiHeadAttention forward (fused Q|K|V GEMM,
linear_pos GEMM, fused rel-pos attention, linear_out GEMM) over a batch of
16 utterances of T=750 frames (d_model 1024, 8 heads of 128, bf16), lengths
uniform in [375, 750] with the key padding mask.  Frames counted are valid
frames (sum of lengths).  Multi-GPU: one process per GPU, each with its own
16-utterance batch (weak scaling, no collective on the data path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the CPU restatement of the reference algorithm
(oracle/, ORC_REFERENCE_ALGO mode: query blocks, materialised (q+v)P^T,
rel_shift by pad/reshape, masked softmax) on the host cores; the reference
itself (Rust over MLX/Metal, macOS only) cannot run on this machine.
"""
from __future__ import annotations

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

METRIC = "rel-pos MHA encoder frames/s at 1/2/4/8 B200; % of tensor/HBM roofline"
B, T, D, H = 16, 750, 1024, 8
LEN_LO, LEN_HI = 375, 750
WORKLOAD = ("BASELINE config 1: offline batched full-context rel-pos MHA layer, bf16, "
            "B=16 T=750 d_model=1024 8x128 heads, lengths U[375,750] with key padding mask")
L2_FLUSH_BYTES = 256 << 20
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of each
# of the forward's four launches, from one ncu capture of this workload's
# bench command; None = not captured.
TRAFFIC_BYTES = {"linear_pos": 5.23e6, "qkv_gemm": 26.14e6 + 13.66e6,
                 "attention": 62.49e6 + 1.28e6, "linear_out": 21.94e6}
# config 4's attention launch on one GPU: DRAM read + write of one ncu capture
LONG_ATTN_TRAFFIC = 309.311e6 + 82.413e6
# The forward's launches in the order the host issues them (linear_pos on
# the context's second stream, beside the q|k|v GEMM)
FORWARD_LAUNCHES = (("linear_pos", "gemm_bf16"), ("qkv_gemm", "gemm_bf16"),
                    ("attention", "attn_sm100"), ("linear_out", "gemm_bf16"))


def workload(seed: int):
    rng = np.random.default_rng(seed)
    f = lambda *s: (rng.standard_normal(s) * 0.02).astype(np.float32)
    w = {"wq": f(D, D), "bq": f(D), "wk": f(D, D), "bk": f(D), "wv": f(D, D), "bv": f(D),
         "wo": f(D, D), "bo": f(D), "wp": f(D, D), "pos_bias_u": f(H, D // H),
         "pos_bias_v": f(H, D // H)}
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    lengths = rng.integers(LEN_LO, LEN_HI + 1, B).astype(np.int32)
    return w, x, lengths


def algorithmic_flops(lengths):
    """Per forward, counting useful work only: projections 2*K*N per valid
    frame (Q,K,V,out), linear_pos over the 2T-1 positions, attention
    3 products (ac, bd, PV) x 2*dh per visible (query, key) pair of valid
    queries."""
    dh = D // H
    valid = int(np.sum(lengths))
    proj = 4 * 2 * valid * D * D
    pos = 2 * (2 * T - 1) * D * D
    attn = 3 * 2 * dh * H * int(np.sum(lengths.astype(np.int64) ** 2))
    return proj, pos, attn


# long-form windowed attention, sequence split across ranks
LONG_B, LONG_T, LONG_WINDOW = 4, 12500, (128, 128)
LONG_WORKLOAD = ("BASELINE config 4: long-form rel-pos local attention, window [128,128], bf16, "
                 "B=4 T=12500 d_model=1024 8x128 heads; the sequence is split across the ranks "
                 "with a 128-frame K/V halo exchanged over NCCL")


def long_flops():
    """Per forward (all frames valid): projections Q,K,V,out 2*K*N per
    frame, linear_pos over the 2*128+1 positions the window reaches,
    attention 3 products x 2*dh per visible (query, key) pair."""
    dh = D // H
    left, right = LONG_WINDOW
    i = np.arange(LONG_T)
    pairs = int(np.sum(np.minimum(LONG_T - 1, i + right) - np.maximum(0, i - left) + 1))
    proj = 4 * 2 * LONG_B * LONG_T * D * D
    pos = 2 * (left + right + 1) * D * D
    attn = 3 * 2 * dh * H * LONG_B * pairs
    return proj, pos, attn


def run_pipelined(steps, h2d, compute, d2h):
    """End-to-end steps as a serving loop runs them: step k's host->device
    copy, its compute and its device->host read each on their own stream,
    two buffer slots, so the copy engines move step k+1's input and step
    k-1's result while step k computes.  Every step still copies its own
    input in and reads its own result back.  h2d(slot), compute(slot) and
    d2h(slot) issue their work on the current stream.  Returns the elapsed
    ms from the first copy-in to the last copy-out (CUDA events)."""
    import torch
    s_in, s_cmp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    in_done = [torch.cuda.Event() for _ in range(steps)]
    cmp_done = [torch.cuda.Event() for _ in range(steps)]
    out_done = [torch.cuda.Event() for _ in range(steps)]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(s_in)
    for k in range(steps):
        slot = k & 1
        with torch.cuda.stream(s_in):
            if k >= 2:
                s_in.wait_event(cmp_done[k - 2])  # the slot's input buffer is free
            h2d(slot)
            in_done[k].record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(in_done[k])
            if k >= 2:
                s_cmp.wait_event(out_done[k - 2])  # the slot's output buffer is free
            compute(slot)
            cmp_done[k].record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(cmp_done[k])
            d2h(slot)
            out_done[k].record(s_out)
    end.record(s_out)
    torch.cuda.synchronize()
    return start.elapsed_time(end)


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def oracle_sample(w, x, lengths, n_utts, threads):
    """Time the CPU restatement on the first n_utts utterances; returns
    (valid frames, seconds)."""
    from oracle import oracle as orc
    orc.set_threads(threads)
    pe = orc.get_encoding(D, 5000, T)
    xs, ls = x[:n_utts], lengths[:n_utts]
    t0 = time.perf_counter()
    orc.mha_forward(xs, w, pe, H, lengths=ls, mode=orc.ORC_REFERENCE_ALGO, bf16=True)
    return int(ls.sum()), time.perf_counter() - t0


class ClockSampler:
    """nvidia-smi clocks during the timed region (one GPU)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        # raw samples (the JSON line carries their summary)
        self.path = os.path.join(os.environ.get("NRP_CLOCKS_DIR", tempfile.gettempdir()),
                                 f"nrp_clocks_gpu{gpu_index}_{os.getpid()}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return self
        # nvidia-smi takes ~0.1-1 s to print its first line: wait for it
        # (bounded), so a short timed region still sees the sampler running
        t_end = time.time() + 5.0
        while time.time() < t_end and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.02)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            p = [s.strip() for s in line.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                smax = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "samples": len(sm), "reasons": sorted(reasons)}


def run_reference(args):
    """The reference arm: CPU restatement of the reference algorithm."""
    rank = env_int("RANK", 0)
    if rank != 0:
        return 0
    w, x, lengths = workload(1234)
    threads = os.cpu_count() or 1
    n_utts = B
    for _ in range(args.warmup):
        oracle_sample(w, x, lengths, n_utts, threads)
    # each step is the whole batch; the run stops early once 90 s of CPU
    # time have been measured, so the arm ends within a few minutes
    times, frames = [], 0
    for _ in range(args.steps):
        fr, dt = oracle_sample(w, x, lengths, n_utts, threads)
        times.append(dt)
        frames = fr
        if sum(times) > 90.0:
            break
    total = sum(times)
    value = frames * len(times) / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "frames/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / len(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (f32 math, bf16 rounding)",
        "data": "synthetic", "config": {"workload": WORKLOAD, "sample_utterances": n_utts,
                                        "steps_measured": len(times)},
        "cpu_baseline": {"value": value, "unit": "frames/s", "cores": threads, "kind": "port",
                         "sample": f"all {n_utts} utterances per step (valid frames "
                                   f"{frames}), CPU restatement of the reference algorithm "
                                   f"(ORC_REFERENCE_ALGO), host CPU: {cpu_model()}"},
        "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference (Rust + MLX Metal/Accelerate, macOS only) cannot be built or "
                "run here; this arm times its algorithm restated in C (oracle/)",
    }
    print(json.dumps(line), flush=True)
    return 0


def _max_ranks(v, world, dev):
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def host_link(world, dev, h2d_bytes, d2h_bytes, barrier, reps=20):
    """Pinned host <-> device copy time of one step's bytes on this rank
    while every rank copies at the same time: host to device alone, device
    to host alone, and both directions at once on two streams (as the e2e
    loop runs them).  Device-timed, max over ranks.  Together with the
    device step time this bounds the e2e rate."""
    import torch
    hi = torch.empty(h2d_bytes, dtype=torch.uint8).pin_memory()
    ho = torch.empty(d2h_bytes, dtype=torch.uint8).pin_memory()
    di = torch.empty(h2d_bytes, dtype=torch.uint8, device=dev)
    do = torch.empty(d2h_bytes, dtype=torch.uint8, device=dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    cur = torch.cuda.current_stream(dev)

    def run(do_in, do_out):
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        barrier()
        start.record(cur)
        s_in.wait_event(start)
        s_out.wait_event(start)
        for _ in range(reps):
            if do_in:
                with torch.cuda.stream(s_in):
                    di.copy_(hi, non_blocking=True)
            if do_out:
                with torch.cuda.stream(s_out):
                    ho.copy_(do, non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)
        stop.record(cur)
        torch.cuda.synchronize(dev)
        return _max_ranks(start.elapsed_time(stop) / reps, world, dev)

    run(True, True)  # warm-up
    t_in, t_out, t_both = run(True, False), run(False, True), run(True, True)
    return {"h2d_gbs": h2d_bytes / t_in / 1e6, "d2h_gbs": d2h_bytes / t_out / 1e6,
            "bidir_ms_per_step": t_both,
            "bidir_gbs": (h2d_bytes + d2h_bytes) / t_both / 1e6,
            "ranks_copying_at_once": world,
            "how": f"{reps} copies of one step's bytes each way from/to pinned host memory, "
                   f"every rank at once, CUDA events, slowest rank"}


def _timed_steps(step, n, dev, world, barrier, flush):
    """n steps timed with CUDA events (L2 flushed between them, outside the
    events), summed; max over ranks."""
    import torch
    stream = torch.cuda.current_stream(dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
    torch.cuda.synchronize(dev)
    barrier()
    for k in range(n):
        flush.zero_()
        starts[k].record(stream)
        step()
        ends[k].record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    return _max_ranks(sum(a.elapsed_time(b) for a, b in zip(starts, ends)), world, dev)


def strong_split_attention(nrp, ctx, attn, pos, w, x, lengths, world, rank, dev, barrier, args):
    """Config 1's one batch of 16 utterances split over the ranks by
    nrp_partition_utterances (longest first onto the least loaded rank);
    every rank runs the layer on its share; strong scaling: all 16
    utterances' valid frames / the slowest rank's step time."""
    import torch
    parts, cost = nrp.partition_utterances(lengths, world, D)
    idx = parts[rank]
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    if len(idx):
        xr = torch.from_numpy(np.ascontiguousarray(x[idx])).to(dev, torch.bfloat16)
        out = torch.empty_like(xr)
        mask = nrp.key_padding_mask(lengths[idx], T)

        def step():
            attn.forward(xr, pos, None, mask, out=out)
    else:
        def step():
            pass
    for _ in range(3):
        step()
    ctx.check()
    n = min(args.steps, 500)
    ms = _timed_steps(step, n, dev, world, barrier, flush)
    ctx.check()
    frames = int(lengths.sum())
    return {"value": frames * n / (ms / 1e3), "unit": "frames/s", "ms_per_step": ms / n,
            "n_gpus": world, "steps": n, "scaling": "strong",
            "utterances_per_rank": [int(len(p)) for p in parts],
            "cost_per_rank": [float(c) for c in cost],
            "workload": "config 1's one batch (16 utterances, B=16 T=750) split over the ranks "
                        "by nrp_partition_utterances; no collective"}


def _long_module(nrp, ctx, local):
    """Config 4's layer: seeded N(0, 0.02^2) weights, the (128, 128) window,
    the positional table for T = 12500, and the input sequence."""
    rng = np.random.default_rng(4321)
    f = lambda *sh: (rng.standard_normal(sh) * 0.02).astype(np.float32)
    w = {"wq": f(D, D), "bq": f(D), "wk": f(D, D), "bk": f(D), "wv": f(D, D), "bv": f(D),
         "wo": f(D, D), "bo": f(D), "wp": f(D, D), "pos_bias_u": f(H, D // H),
         "pos_bias_v": f(H, D // H)}
    attn = nrp.RelPositionMultiHeadAttention(D, H, True, ctx=ctx)
    for which, (wk, bk) in enumerate((("wq", "bq"), ("wk", "bk"), ("wv", "bv"), ("wo", "bo"),
                                      ("wp", None))):
        attn.set_linear(which, nrp.LinearLayer.standard(w[wk], w[bk] if bk else None))
    attn.set_pos_bias(w["pos_bias_u"], w["pos_bias_v"])
    attn.set_dtype(nrp.BF16)
    actx = nrp.AttentionContext.new(LONG_WINDOW, "regular")
    pe = nrp.RelPositionalEncoding(D, 5000, True, device=local)
    pe.set_dtype(nrp.BF16)
    pos = pe.get_encoding(LONG_T)
    # every rank draws the whole sequence (same seed) and keeps its segment
    x = np.random.default_rng(8765).standard_normal((LONG_B, LONG_T, D)).astype(np.float32)
    return w, attn, actx, pos, x


def seq_split_config4(nrp, ctx, world, rank, local, dev, barrier, args):
    """Config 4 ([4, 12500, 1024], window (128, 128)) with the sequence split
    over the ranks (nrp_attn_forward_seq_sharded: 128-frame K/V halo over
    NCCL); one GPU runs the plain windowed forward.  Strong scaling."""
    import torch
    _, attn, actx, pos, x = _long_module(nrp, ctx, local)
    halo = None
    if world > 1:
        halo = nrp.HaloComm.from_process_group(ctx=ctx, timeout_ms=120000)
        plan = halo.plan(LONG_T, actx)
        s0, n0 = plan.start, plan.len
    else:
        s0, n0 = 0, LONG_T
    xd = torch.from_numpy(np.ascontiguousarray(x[:, s0:s0 + n0])).to(dev, torch.bfloat16)
    out = torch.empty_like(xd)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def step():
        if halo is None:
            attn.forward(xd, pos, actx, None, out=out)
        else:
            attn.forward_seq_sharded(xd, pos, LONG_T, halo, actx, None, out=out)

    for _ in range(3):
        step()
    if halo is not None:
        halo.check()
    ctx.check()
    n = min(args.steps, 300)
    ms = _timed_steps(step, n, dev, world, barrier, flush)
    if halo is not None:
        halo.check()
        halo.close()
    ctx.check()
    return {"value": LONG_B * LONG_T * n / (ms / 1e3), "unit": "frames/s", "ms_per_step": ms / n,
            "n_gpus": world, "steps": n, "scaling": "strong", "frames_per_rank": LONG_B * n0,
            "workload": LONG_WORKLOAD if world > 1 else
            "BASELINE config 4 on one GPU (plain windowed forward)"}


def strong_split_encoder(nrp, ctx, world, rank, dev, barrier, args):
    """Config 3's one batch (32 utterances, 24 layers, 8-bit linears read as
    codes every forward: the weight cache is off) split over the ranks by
    nrp_partition_utterances.  Strong scaling."""
    import torch
    from oracle import oracle as orc  # quantiser of the synthetic checkpoint only
    rng = np.random.default_rng(5150)
    enc = nrp.ConformerEncoder(ENC_LAYERS, D, H, ENC_FF, ENC_K, ctx=ctx)
    _load_quant_layers(nrp, orc, enc, rng)
    enc.set_dtype(nrp.BF16)
    x = rng.standard_normal((ENC_B, ENC_T, D), dtype=np.float32)
    lengths = rng.integers(ENC_LEN_LO, ENC_LEN_HI + 1, ENC_B).astype(np.int32)
    parts, cost = nrp.partition_utterances(lengths, world, D)
    idx = parts[rank]
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    ctx.set_weight_cache(False)
    if len(idx):
        xr = torch.from_numpy(np.ascontiguousarray(x[idx])).to(dev, torch.bfloat16)
        out = torch.empty((len(idx), D, ENC_T), dtype=torch.bfloat16, device=dev)
        lr = lengths[idx]

        def step():
            enc.forward_from_embeddings(xr, lr, None, out=out)
    else:
        def step():
            pass
    for _ in range(2):
        step()
    ctx.check()
    n = min(args.steps, 20)
    ms = _timed_steps(step, n, dev, world, barrier, flush)
    ctx.check()
    ctx.set_weight_cache(True)
    frames = int(lengths.sum())
    del enc
    return {"value": frames * n / (ms / 1e3), "unit": "frames/s", "ms_per_step": ms / n,
            "n_gpus": world, "steps": n, "scaling": "strong",
            "utterances_per_rank": [int(len(p)) for p in parts],
            "cost_per_rank": [float(c) for c in cost],
            "workload": "config 3's one batch (B=32 T=500, 24 layers, MLX 8-bit linears read as "
                        "u8 codes each forward) split over the ranks by "
                        "nrp_partition_utterances; no collective"}


def ql_shapes():
    """Config 3's block linears (N, K): FF1 1024->4096->1024, the pointwise
    convs, FF2, then q, k, v, out, pos."""
    return [(ENC_FF, D), (D, ENC_FF), (2 * D, D), (D, D), (ENC_FF, D), (D, ENC_FF),
            (D, D), (D, D), (D, D), (D, D), (D, D)]


QL_WORKLOAD = ("config 3's MLX 8-bit linears (group 64, bf16 scales and biases): the 11 linears "
               "of each of 24 layers, one after another on one stream, at M rows (M = 14: one "
               "streaming session's 14-frame chunk; M = 128)")


def main_qlinear(args):
    """North-star kernel (3), LinearLayer::forward's quantised arm
    (quantization.rs:137-160) through nrp_qlinear: one step runs all 264
    linears of config 3's 24 layers on M rows, replayed as a CUDA graph (the
    launches are microseconds each).  Both row counts take the small-M
    8-bit kernel (codes staged in shared memory by bulk copies, dequantised
    in registers into bf16 MMA fragments); M = 128 runs two 64-row chunks.
    one_large_launch: a single linear over 64 MB of codes, the kernel's
    streaming rate with its launch latency amortised.  Algorithmic bytes per
    linear: N*K codes + 4*N*K/64 scale/bias + 2*M*K in + 2*M*N out; FLOP
    2*M*N*K."""
    import torch
    from __graft_entry__ import load_package
    world, rank, local = _dist_init(args)
    nrp = load_package()
    ctx = nrp.Context(local)
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    layers = []
    for _ in range(ENC_LAYERS):
        for n, k in ql_shapes():
            wq = torch.randint(-2**31, 2**31 - 1, (n, k // 4), dtype=torch.int32, device=dev,
                               generator=g)
            sc = (torch.rand((n, k // 64), device=dev, generator=g) * 4e-4 + 1e-4).bfloat16()
            zp = (torch.rand((n, k // 64), device=dev, generator=g) * -0.1).bfloat16()
            b = (torch.randn(n, device=dev, generator=g) * 0.02).bfloat16()
            layers.append((wq, sc, zp, b, n, k))
    stream = torch.cuda.Stream(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peaks = json.load(open(peaks_path)) if os.path.exists(peaks_path) else {}
    hbm_peak = peaks.get("hbm_gbs") or 6650.0
    burst, _, peak_src = _peaks()
    barrier = (lambda: torch.distributed.barrier()) if world > 1 else (lambda: None)

    def measure(M, n_steps):
        xs = {k: torch.randn((M, k), device=dev, generator=g).bfloat16()
              for k in {k for _, k in ql_shapes()}}
        ys = [torch.empty((M, n), dtype=torch.bfloat16, device=dev) for *_, n, _ in layers]

        def run():
            for (wq, sc, zp, b, n, k), y in zip(layers, ys):
                nrp.qlinear(xs[k], wq, sc, zp, b, ctx=ctx, out=y)

        with torch.cuda.stream(stream):
            run()  # warm-up outside capture
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            run()
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        ctx.check()
        ms = _timed_steps(graph.replay, n_steps, dev, world, barrier, flush)
        ctx.check()
        nbytes = sum(n * k + 4 * n * k // 64 + 2 * M * k + 2 * M * n + 2 * n
                     for *_, n, k in layers)
        flop = sum(2 * M * n * k for *_, n, k in layers)
        t = ms / n_steps / 1e3
        del graph
        return {"rows": M, "ms_per_step": ms / n_steps, "steps": n_steps,
                "linears_per_step": len(layers), "bytes_per_step": nbytes,
                "flop_per_step": flop, "gbs": nbytes / t / 1e9, "tflops": flop / t / 1e12,
                "hbm_frac": nbytes / t / 1e9 / hbm_peak, "tensor_frac": flop / t / 1e12 / burst}

    def one_launch(M, N, K, reps):
        """One linear over a large weight, eager, CUDA events around each
        launch (L2 flushed between): the kernel's streaming rate with its
        launch latency amortised."""
        wq = torch.randint(-2**31, 2**31 - 1, (N, K // 4), dtype=torch.int32, device=dev,
                           generator=g)
        sc = (torch.rand((N, K // 64), device=dev, generator=g) * 4e-4 + 1e-4).bfloat16()
        zp = (torch.rand((N, K // 64), device=dev, generator=g) * -0.1).bfloat16()
        x = torch.randn((M, K), device=dev, generator=g).bfloat16()
        y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            nrp.qlinear(x, wq, sc, zp, None, ctx=ctx, out=y)
        ts = []
        for _ in range(reps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            nrp.qlinear(x, wq, sc, zp, None, ctx=ctx, out=y)
            b.record()
            torch.cuda.synchronize(dev)
            ts.append(a.elapsed_time(b))
        ctx.check()
        ms = statistics.median(ts)
        nbytes = N * K + 4 * N * K // 64 + 2 * M * K + 2 * M * N
        return {"rows": M, "N": N, "K": K, "ms_per_launch": ms, "bytes_per_launch": nbytes,
                "gbs": nbytes / (ms / 1e3) / 1e9, "hbm_frac": nbytes / (ms / 1e3) / 1e9 / hbm_peak,
                "how": f"median of {reps} eager launches, CUDA events, L2 flushed between"}

    if args.qlinear_large_only:  # the large launch alone (an ncu capture's driver)
        large = one_launch(14, 16384, 4096, 5)
        if rank == 0:
            print(json.dumps({"one_large_launch": large}), flush=True)
        return 0
    n_steps = min(args.steps, 500)
    with ClockSampler(local) as clocks:
        small = measure(14, n_steps)
        big = measure(128, n_steps)
        large = one_launch(14, 16384, 4096, 50)
    # e2e through the public API: the 14 rows in from pinned host memory,
    # the last linear's output back, per step (eager launches)
    x_host = torch.randn((14, D)).bfloat16().pin_memory()
    y_host = torch.empty((14, D), dtype=torch.bfloat16).pin_memory()
    xd = torch.empty((14, D), dtype=torch.bfloat16, device=dev)
    xk = torch.empty((14, ENC_FF), dtype=torch.bfloat16, device=dev)
    ys = [torch.empty((14, n), dtype=torch.bfloat16, device=dev) for *_, n, _ in layers]

    def compute(slot):
        for (wq, sc, zp, b, n, k), y in zip(layers, ys):
            nrp.qlinear(xd if k == D else xk, wq, sc, zp, b, ctx=ctx, out=y)

    e2e_ms = run_pipelined(n_steps, lambda s: xd.copy_(x_host, non_blocking=True), compute,
                           lambda s: y_host.copy_(ys[-1], non_blocking=True))
    e2e_ms = _max_ranks(e2e_ms, world, dev)
    if rank == 0:
        line = {
            "metric": METRIC, "value": world * 14 * n_steps / (small["ms_per_step"] * n_steps / 1e3),
            "unit": "frames/s", "n_gpus": world, "steps": n_steps, "warmup": max(args.warmup, 3),
            "ms_per_step": small["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 activations, u8 weights", "data": "synthetic",
            "config": {"workload": QL_WORKLOAD, "rows": 14, "layers": ENC_LAYERS,
                       "l2": "flushed between timed steps (256 MiB write, outside the events); "
                             "the weights (643 MB) exceed L2 anyway"},
            "e2e": {"value": world * 14 * n_steps / (e2e_ms / 1e3), "unit": "frames/s",
                    "h2d_bytes_per_step": x_host.numel() * 2,
                    "d2h_bytes_per_step": y_host.numel() * 2},
            "gpu_launches": len(layers) * n_steps,
            "roofline": {"bound": "hbm", "kernel": "small-M 8-bit GEMM (M = 14)",
                         "achieved": small["gbs"],
                         "peak": hbm_peak, "unit": "GB/s", "frac": small["hbm_frac"],
                         "traffic": None, "peak_source": "measured (hbm_gbs, MEASURED_PEAKS.json)",
                         "algorithmic_bytes_per_step": small["bytes_per_step"]},
            "rows_14": small,
            "one_large_launch": large,
            "rows_128": dict(big, roofline={"bound": "tensor",
                                            "kernel": "small-M 8-bit GEMM (M = 128)",
                                            "achieved": big["tflops"], "peak": burst,
                                            "unit": "TFLOP/s", "frac": big["tensor_frac"],
                                            "peak_source": peak_src}),
            "clocks": clocks.summary(),
            "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--qlinear-large-only", action="store_true",
                    help="qlinear workload: only the one large launch (5 launches, for ncu)")
    ap.add_argument("--no-extras", action="store_true",
                    help="config 1 only: skip the strong-scaling and sequence-split keys")
    ap.add_argument("--workload", default="offline",
                    choices=["offline", "long", "encoder", "stream", "single", "subsampling",
                             "stream_encoder", "qlinear"],
                    help="offline: BASELINE config 1 (the headline line); long: config 4, "
                         "the sequence split across the ranks; encoder: config 3; stream: "
                         "config 2; single: config 0; subsampling: the pre_encode of "
                         "config 3's batch from mel frames; stream_encoder: the whole "
                         "streaming encoder step from mel chunks; qlinear: config 3's 8-bit "
                         "linears at 14 and 128 rows (the GEMV and the dequantising GEMM)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "long":
        return main_long(args)
    if args.workload == "encoder":
        return main_encoder(args)
    if args.workload == "stream":
        return main_stream(args)
    if args.workload == "single":
        return main_single(args)
    if args.workload == "subsampling":
        return main_subsampling(args)
    if args.workload == "stream_encoder":
        return main_stream_encoder(args)
    if args.workload == "qlinear":
        return main_qlinear(args)

    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    nrp = load_package()
    ctx = nrp.Context(local)
    w, x, lengths = workload(1234 + rank)
    attn = nrp.RelPositionMultiHeadAttention(D, H, True, ctx=ctx)
    attn.set_linear(nrp.LINEAR_Q, nrp.LinearLayer.standard(w["wq"], w["bq"]))
    attn.set_linear(nrp.LINEAR_K, nrp.LinearLayer.standard(w["wk"], w["bk"]))
    attn.set_linear(nrp.LINEAR_V, nrp.LinearLayer.standard(w["wv"], w["bv"]))
    attn.set_linear(nrp.LINEAR_OUT, nrp.LinearLayer.standard(w["wo"], w["bo"]))
    attn.set_linear(nrp.LINEAR_POS, nrp.LinearLayer.standard(w["wp"], None))
    attn.set_pos_bias(w["pos_bias_u"], w["pos_bias_v"])
    attn.set_dtype(nrp.BF16)
    pe = nrp.RelPositionalEncoding(D, 5000, True, device=local)
    pe.set_dtype(nrp.BF16)
    pos = pe.get_encoding(T)
    dev = torch.device("cuda", local)
    xd = torch.from_numpy(x).to(dev, torch.bfloat16)
    out = torch.empty_like(xd)
    mask = nrp.key_padding_mask(lengths, T)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()

    def step(o=out, xin=xd):
        attn.forward(xin, pos, None, mask, out=o)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(args.warmup, 3)):
        step()
    ctx.check()

    # ---- device-timed region: inputs resident in HBM, L2 flushed between steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for k in range(args.steps):
            flush.zero_()
            starts[k].record(stream)
            step()
            ends[k].record(stream)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ctx.check()
    total_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    frames = int(lengths.sum())
    value = world * frames * args.steps / (total_ms / 1e3)

    # ---- per-launch device times (CUDA events the library records around
    # each launch on its launching stream), same steps
    ctx.profile(True)
    ctx.profile_reset()
    for k in range(args.steps):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    log = ctx.profile_launches()
    ctx.profile(False)
    launches = len(log)
    nl = len(FORWARD_LAUNCHES)
    if launches != nl * args.steps or any(
            kind != FORWARD_LAUNCHES[i % nl][1] for i, (kind, _) in enumerate(log)):
        raise RuntimeError(f"unexpected launch sequence: {log[:2 * nl]}")
    per_launch = {name: [ms for i, (_, ms) in enumerate(log) if i % nl == j]
                  for j, (name, _) in enumerate(FORWARD_LAUNCHES)}

    # ---- end to end through the public API with host buffers: each step
    # moves its utterances' valid frames (packed back to back in pinned host
    # memory) in with one copy and reads the valid output frames back with
    # one copy (padded rows are unspecified, conformer.rs:1590-1593).  On the
    # device, unpack_frames scatters the packed rows (and the lengths) into
    # the [B, T, D] input and pack_frames gathers the output rows; both run
    # on the compute stream, so each copy stream carries nothing but its
    # copies.  run_pipelined overlaps the copies with the neighbouring steps'
    # compute.
    x_host = torch.cat([torch.from_numpy(x[b, :n]) for b, n in enumerate(lengths)]).to(
        torch.bfloat16).pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    xs = [torch.empty_like(xd) for _ in range(2)]
    outs = [torch.empty_like(xd) for _ in range(2)]
    masks = [nrp.key_padding_mask(lengths, T) for _ in range(2)]
    packed_in = [torch.empty_like(x_host, device=dev) for _ in range(2)]
    packed_out = [torch.empty_like(x_host, device=dev) for _ in range(2)]

    def h2d_fn(slot):
        packed_in[slot].copy_(x_host, non_blocking=True)

    def compute_fn(slot):
        nrp.unpack_frames(xs[slot], packed_in[slot], lengths, dev_lengths=masks[slot].lengths)
        attn.forward(xs[slot], pos, None, masks[slot], out=outs[slot])
        nrp.pack_frames(packed_out[slot], outs[slot], lengths)

    def d2h_fn(slot):
        out_host.copy_(packed_out[slot], non_blocking=True)

    run_pipelined(4, h2d_fn, compute_fn, d2h_fn)  # warm-up
    barrier()
    e2e_ms = run_pipelined(args.steps, h2d_fn, compute_fn, d2h_fn)
    barrier()
    t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    e2e_value = world * frames * args.steps / (e2e_ms / 1e3)
    h2d = frames * D * 2 + lengths.size * 4  # the lengths go in the scatter's parameters
    d2h = frames * D * 2
    link = host_link(world, dev, h2d, d2h, barrier)
    floor_ms = max(link["bidir_ms_per_step"], total_ms / args.steps)
    link["e2e_ceiling_frames_per_s"] = world * frames / (floor_ms / 1e3)
    link["e2e_frac_of_ceiling"] = e2e_value / link["e2e_ceiling_frames_per_s"]

    # ---- roofline of each launch; the dominant one is `roofline`
    burst, sustained, peak_src = _peaks()
    proj, pos_f, attn_f = algorithmic_flops(lengths)
    flop = {"linear_pos": pos_f, "qkv_gemm": proj * 3 // 4, "attention": attn_f,
            "linear_out": proj // 4}
    total_launch_ms = sum(sum(v) for v in per_launch.values())
    rk = {}
    for name, ms_list in per_launch.items():
        ms = sum(ms_list) / len(ms_list)
        a = flop[name] / (ms / 1e3) / 1e12
        rk[name] = {"launches": len(ms_list), "ms_per_launch": ms,
                    "share": sum(ms_list) / total_launch_ms,
                    "algorithmic_flop_per_launch": flop[name], "achieved": a,
                    "unit": "TFLOP/s", "frac": a / burst, "frac_of_sustained": a / sustained,
                    "traffic": TRAFFIC_BYTES.get(name)}
    dominant = max(rk, key=lambda n: rk[n]["share"])
    d = rk[dominant]
    roof = {"bound": "tensor", "kernel": dominant, "achieved": d["achieved"], "peak": burst,
            "unit": "TFLOP/s", "frac": d["frac"], "traffic": d["traffic"],
            "peak_source": peak_src + "; burst: each step is 0.2 ms, not a seconds-long loop",
            "algorithmic_flop_per_launch": d["algorithmic_flop_per_launch"]}
    whole = (proj + pos_f + attn_f) * args.steps / (total_ms / 1e3) / 1e12
    kern = {}
    for name, kind in FORWARD_LAUNCHES:
        k = kern.setdefault(kind, {"launches": 0, "ms_total": 0.0})
        k["launches"] += len(per_launch[name])
        k["ms_total"] += sum(per_launch[name])
    for k in kern.values():
        k["share"] = k["ms_total"] / total_launch_ms

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        oracle_sample(w, x, lengths, 2, threads)  # warm-up
        runs = [oracle_sample(w, x, lengths, B, threads) for _ in range(3)]
        fr = runs[0][0]
        med = statistics.median(r[1] for r in runs)
        cpu = {"value": fr / med, "unit": "frames/s", "cores": threads, "kind": "port",
               "sample": f"the whole batch ({B} utterances, {fr} valid frames), median of 3 "
                         f"after a warm-up; CPU restatement of the reference algorithm "
                         f"(ORC_REFERENCE_ALGO, bf16 rounding), host CPU: {cpu_model()}"}

    # ---- multi-GPU designs beside the weak-scaled replicas (every rank)
    extras = {}
    if not args.no_extras:
        extras["strong_scaling_config1"] = strong_split_attention(
            nrp, ctx, attn, pos, w, x, lengths, world, rank, dev, barrier, args)
        extras["seq_split_config4"] = seq_split_config4(nrp, ctx, world, rank, local, dev,
                                                        barrier, args)
        extras["strong_scaling_config3"] = strong_split_encoder(nrp, ctx, world, rank, dev,
                                                                barrier, args)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch_per_gpu": B, "seq_len": T, "d_model": D,
                       "heads": H, "valid_frames_per_gpu": frames,
                       "l2": "flushed between timed steps (256 MiB write, outside the events)",
                       "parallelism": f"utterance-parallel replicas x{world}"},
            "e2e": {"value": e2e_value, "unit": "frames/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "roofline": roof,
            "roofline_kernels": rk,
            "kernel_times_note": "per-launch CUDA events on each launch's stream; linear_pos "
                                 "runs on a second stream beside the q|k|v GEMM, so the "
                                 "launch times overlap and their sum exceeds ms_per_step",
            "whole_step_tflops": whole,
            "kernels": kern,
            "host_link": link,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


# the 24-layer encoder, all linears MLX 8-bit
ENC_LAYERS, ENC_B, ENC_T, ENC_FF, ENC_K = 24, 32, 500, 4096, 9
ENC_LEN_LO, ENC_LEN_HI = 250, 500
ENC_WORKLOAD = ("BASELINE config 3: 24-layer FastConformer encoder (forward_from_embeddings), "
                "macaron FF 1024->4096->1024 SiLU, rel-pos MHA 8x128, conv module (depthwise 9, "
                "GLU, BatchNorm affine), every linear MLX 8-bit g64 from N(0,0.02^2) masters, "
                "bf16 activations, B=32 T=500 lengths U[250,500]")
# streaming attention over 24 layers
STR_LAYERS, STR_SESS, STR_CHUNK, STR_CACHE, STR_CHUNKS = 24, 64, 14, 70, 50
STR_WORKLOAD = ("BASELINE config 2: cache-aware streaming rel-pos attention, 24 layers, "
                "64 sessions, chunk 14 (13 lookahead + 1), 70-frame left K/V cache, "
                "chunked_limited [70,13], bf16; a step is one chunk through the 24 layers, the "
                "caches restart empty every 50 chunks")
# The encoder's pre_encode on config 3's batch as mel input (feat_in 128, as
# the parakeet FastConformers): 500 encoder frames = 4000 mel frames
SUB_B, SUB_T, SUB_F, SUB_C, SUB_FACTOR = 32, 4000, 128, 256, 8
SUB_LEN_LO, SUB_LEN_HI = 2000, 4000
SUB_WORKLOAD = ("dw_striding subsampling (pre_encode): 8x, conv channels 256, feat_in 128, "
                "d_model 1024, non-causal, bf16; mel [B=32, 128, 4000] f32 with lengths "
                "U[2000,4000] masked (config 3's batch before subsampling)")
STRENC_WORKLOAD = ("cache-aware streaming encoder step (forward_streaming): 64 sessions, "
                   "112 mel frames per chunk (128 bins) -> causal 8x subsampling, 1 pre-encoded "
                   "frame dropped -> 14 frames through 24 streaming blocks (config 3's layer, "
                   "causal conv with its cache, 8-bit weights), attention cache 70, "
                   "chunked_limited [70,13]; caches restart every 50 chunks")
# one fp32 layer, batch 1, T=125
SGL_T = 125
SGL_WORKLOAD = ("BASELINE config 0: one rel-pos MHA layer, fp32, B=1 T=125 d_model=1024 "
                "8x128 heads, no mask")


def _harness(args, world, rank, local, ctx, step, frames, flops, kinds_bound, workload,
             config, scaling, e2e, dtype, cpu=None, hbm_bytes=None, reset=None,
             prof_step=None, long_step=False, extra=None):
    """Common timing for the secondary workloads: W warm-up steps, K steps
    timed with CUDA events (L2 flushed between steps, outside the events),
    max over ranks; per-kernel device time from the library's events over K
    more steps; e2e = (h2d(slot), compute(slot), d2h(slot), bytes in, bytes
    out) run for K steps by run_pipelined (host copies inside); one JSON
    line.  flops / hbm_bytes: per step, per kernel kind (algorithmic).
    prof_step: the same step run without CUDA graphs, for the pass that times
    each launch (a graph replay runs no host code to record its events)."""
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for k in range(max(args.warmup, 3)):
        step(k)
    ctx.check()
    if reset:
        reset()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for k in range(args.steps):
            flush.zero_()
            starts[k].record(stream)
            step(k)
            ends[k].record(stream)
        torch.cuda.synchronize()
    barrier()
    ctx.check()
    total_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in zip(starts, ends)))
    value = world * frames * args.steps / (total_ms / 1e3)
    if reset:
        reset()
    ctx.profile(True)
    ctx.profile_reset()
    for k in range(args.steps):
        flush.zero_()
        (prof_step or step)(k)
    torch.cuda.synchronize()
    prof = ctx.profile_read()
    ctx.profile(False)
    launches = sum(n for n, _ in prof.values())
    h2d_fn, compute_fn, d2h_fn, h2d, d2h = e2e
    if reset:
        reset()
    run_pipelined(2, h2d_fn, compute_fn, d2h_fn)  # warm-up
    barrier()
    e2e_ms = max_over_ranks(run_pipelined(args.steps, h2d_fn, compute_fn, d2h_fn))
    barrier()
    e2e_value = world * frames * args.steps / (e2e_ms / 1e3)

    tflops_peak, peak_src = _peak(long_step)
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peaks = json.load(open(peaks_path)) if os.path.exists(peaks_path) else {}
    hbm_peak = peaks.get("hbm_gbs") or 6650.0
    hbm_src = "measured (hbm_gbs, MEASURED_PEAKS.json)" if peaks.get("hbm_gbs") else \
        "fallback 6.65 TB/s"
    tot = max(sum(m for _, m in prof.values()), 1e-9)
    kern, rk = {}, {}
    for name, (n, ms) in prof.items():
        kern[name] = {"launches": n, "ms_total": ms, "share": ms / tot}
        if flops and name in flops:
            a = flops[name] * args.steps / (ms / 1e3) / 1e12
            rk[name] = {"achieved": a, "frac": a / tflops_peak, "unit": "TFLOP/s",
                        "algorithmic_flop_per_launch": flops[name] * args.steps / n}
        if hbm_bytes and name in hbm_bytes:
            g = hbm_bytes[name] * args.steps / (ms / 1e3) / 1e9
            rk[name] = {"achieved": g, "frac": g / hbm_peak, "unit": "GB/s",
                        "algorithmic_bytes_per_launch": hbm_bytes[name] * args.steps / n}
    if dtype == "f32":
        # f32 modules: the GEMM runs as three TF32 tensor-core products per
        # f32 product (frac above is against the bf16 peak), the attention on
        # the FFMA pipes; both also get their fraction of the nominal FFMA
        # peak (SMs x 128 FMA/clock x 2 FLOP x the maximum SM clock seen),
        # the rate of an f32 path without tensor cores
        import torch
        n_sm = torch.cuda.get_device_properties(local).multi_processor_count
        mhz = clocks.summary().get("sm_max_mhz") or 1965.0
        ffma_peak = n_sm * 128 * 2 * mhz * 1e6 / 1e12
        for r in rk.values():
            if r["unit"] == "TFLOP/s":
                r["ffma_peak"] = ffma_peak
                r["ffma_frac"] = r["achieved"] / ffma_peak
    dominant = max(prof.items(), key=lambda kv: kv[1][1])[0] if prof else None
    roof = None
    if dominant in rk:
        hbm = rk[dominant]["unit"] == "GB/s"
        roof = {"bound": "hbm" if hbm else "tensor", "kernel": dominant,
                "achieved": rk[dominant]["achieved"],
                "peak": hbm_peak if hbm else tflops_peak, "unit": rk[dominant]["unit"],
                "frac": rk[dominant]["frac"], "traffic": None,
                "peak_source": hbm_src if hbm else peak_src}
        if "ffma_frac" in rk[dominant]:
            roof["ffma_peak"] = rk[dominant]["ffma_peak"]
            roof["ffma_frac"] = rk[dominant]["ffma_frac"]
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": dtype, "data": "synthetic",
            "config": dict({"workload": workload,
                            "l2": "flushed between timed steps (256 MiB write, outside the "
                                  "events)"}, **config),
            "e2e": {"value": e2e_value, "unit": "frames/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "roofline": roof,
            "roofline_kernels": rk,
            "kernels": kern,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu() if (cpu and rank == 0 and world == 1 and
                                      not args.no_cpu_baseline) else None,
        }
        line.update(extra or {})
        print(json.dumps(line), flush=True)


def _dist_init(args):
    import torch
    import torch.distributed as dist
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def _load_quant_layers(nrp, orc, enc, rng):
    """Config 3's layer weights into every block of `enc`: all linears MLX
    8-bit g64 from N(0, 0.02^2) masters with fp16 scales and biases, norms
    1 + N(0, 0.02^2) / N(0, 0.02^2), BatchNorm affine, depthwise k = 9.
    Returns the first two layers' (prefix, weights) for the CPU sample."""
    f = lambda *sh: (rng.standard_normal(sh, dtype=np.float32) * 0.02)
    shapes = {"feed_forward1.linear1": (ENC_FF, D), "feed_forward1.linear2": (D, ENC_FF),
              "conv.pointwise_conv1": (2 * D, D), "conv.pointwise_conv2": (D, D),
              "feed_forward2.linear1": (ENC_FF, D), "feed_forward2.linear2": (D, ENC_FF),
              "self_attn.linear_q": (D, D), "self_attn.linear_k": (D, D),
              "self_attn.linear_v": (D, D), "self_attn.linear_out": (D, D),
              "self_attn.linear_pos": (D, D)}
    sample_layers = []
    for i, blk in enumerate(enc.layers):
        wd = {}
        p = f"encoder.layers.{i}"
        for name, (n, k) in shapes.items():
            wq, sc, zp = orc.quantize(f(n, k), 64, 8)
            wd[f"{p}.{name}.weight"] = wq
            wd[f"{p}.{name}.scales"] = sc.astype(np.float16).astype(np.float32)
            wd[f"{p}.{name}.biases"] = zp.astype(np.float16).astype(np.float32)
            if not name.endswith("linear_pos"):
                wd[f"{p}.{name}.bias"] = f(n)
        for nm in nrp.BLOCK_NORMS:
            wd[f"{p}.{nm}.weight"] = 1 + f(D)
            wd[f"{p}.{nm}.bias"] = f(D)
        wd[f"{p}.self_attn.pos_bias_u"] = f(H, D // H)
        wd[f"{p}.self_attn.pos_bias_v"] = f(H, D // H)
        wd[f"{p}.conv.depthwise_conv.weight"] = f(D, ENC_K, 1)
        wd[f"{p}.conv.depthwise_conv.bias"] = f(D)
        bn = f"{p}.conv.batch_norm"
        wd[f"{bn}.weight"], wd[f"{bn}.bias"] = 1 + f(D), f(D)
        wd[f"{bn}.running_mean"], wd[f"{bn}.running_var"] = f(D), 1 + np.abs(f(D))
        blk.load_weights(wd, p, nrp.QuantizationConfig(8, 64))
        if i < 2:
            sample_layers.append((p, wd))
    return sample_layers


def main_encoder(args):
    """Config 3: forward_from_embeddings over 24 quantised blocks; weak
    scaling (each rank its own 32-utterance batch).  The line measures the
    8-bit weights read as codes every forward; bf16_weight_copies gives the
    same forward over kept bf16 copies of the weights."""
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package
    from oracle import oracle as orc  # quantiser of the synthetic checkpoint only
    world, rank, local = _dist_init(args)
    nrp = load_package()
    ctx = nrp.Context(local)
    rng = np.random.default_rng(5150 + rank)
    enc = nrp.ConformerEncoder(ENC_LAYERS, D, H, ENC_FF, ENC_K, ctx=ctx)
    sample_layers = _load_quant_layers(nrp, orc, enc, rng)
    enc.set_dtype(nrp.BF16)
    dev = torch.device("cuda", local)
    x = rng.standard_normal((ENC_B, ENC_T, D), dtype=np.float32)
    lengths = rng.integers(ENC_LEN_LO, ENC_LEN_HI + 1, ENC_B).astype(np.int32)
    xd = torch.from_numpy(x).to(dev, torch.bfloat16)
    out = torch.empty((ENC_B, D, ENC_T), dtype=torch.bfloat16, device=dev)

    def step(k, xin=xd, o=out):
        enc.forward_from_embeddings(xin, lengths, None, out=o)

    x_host = torch.from_numpy(x).to(torch.bfloat16).pin_memory()
    out_host = torch.empty_like(out, device="cpu").pin_memory()
    xs = [torch.empty_like(xd) for _ in range(2)]
    outs = [torch.empty_like(out) for _ in range(2)]
    e2e = (lambda slot: xs[slot].copy_(x_host, non_blocking=True),
           lambda slot: step(0, xs[slot], outs[slot]),
           lambda slot: out_host.copy_(outs[slot], non_blocking=True),
           x_host.numel() * 2, out_host.numel() * 2)

    valid = int(lengths.sum())
    L2s = int(np.sum(lengths.astype(np.int64) ** 2))
    per_frame = 2 * 2 * (2 * D * ENC_FF) + 4 * 2 * D * D + 2 * D * 2 * D + 2 * D * D
    # the quantised linears run as dequantise-once + bf16 GEMM at these row
    # counts (M = 16000 > 1024 rows)
    flops = {"gemm_bf16": ENC_LAYERS * (per_frame * valid + 2 * (2 * ENC_T - 1) * D * D),
             "attn_sm100": ENC_LAYERS * 3 * 2 * (D // H) * H * L2s}
    w_params = 2 * 2 * D * ENC_FF + 2 * D * D + D * D + 5 * D * D  # per layer
    bytes_ = {"layernorm": ENC_LAYERS * 5 * 2 * ENC_B * ENC_T * D * 2,
              "dwconv": ENC_LAYERS * 2 * ENC_B * ENC_T * D * 2,
              "dequant": ENC_LAYERS * w_params * (1 + 2)}

    def cpu():
        """The oracle on utterance 0 through the first two layers, scaled to
        24 layers (the layers cost the same)."""
        threads = os.cpu_count() or 1
        orc.set_threads(threads)
        L0 = int(lengths[0])
        h = orc.bf16_round(orc.bf16_round(x[:1, :L0]) * np.float32(np.sqrt(D)))
        pe_h = orc.get_encoding(D, 5000, L0)
        deq = lambda wd, k: orc.dequantize(wd[k + ".weight"], orc.bf16_round(wd[k + ".scales"]),
                                           orc.bf16_round(wd[k + ".biases"]), 64, 8)
        blocks = []
        for p, wd in sample_layers:
            lin = lambda n: (deq(wd, f"{p}.{n}"), wd.get(f"{p}.{n}.bias"))
            bw = {"ff1_1": lin("feed_forward1.linear1"), "ff1_2": lin("feed_forward1.linear2"),
                  "pw1": lin("conv.pointwise_conv1"), "pw2": lin("conv.pointwise_conv2"),
                  "ff2_1": lin("feed_forward2.linear1"), "ff2_2": lin("feed_forward2.linear2"),
                  "dw": (wd[f"{p}.conv.depthwise_conv.weight"].reshape(D, ENC_K),
                         wd[f"{p}.conv.depthwise_conv.bias"]),
                  "conv_norm": tuple(wd[f"{p}.conv.batch_norm.{n}"] for n in
                                     ("weight", "bias", "running_mean", "running_var")),
                  "norms": {o: (wd[f"{p}.{n}.weight"], wd[f"{p}.{n}.bias"])
                            for o, n in zip(orc.BLOCK_NORMS, nrp.BLOCK_NORMS)},
                  "attn": {"wq": deq(wd, f"{p}.self_attn.linear_q"),
                           "bq": wd[f"{p}.self_attn.linear_q.bias"],
                           "wk": deq(wd, f"{p}.self_attn.linear_k"),
                           "bk": wd[f"{p}.self_attn.linear_k.bias"],
                           "wv": deq(wd, f"{p}.self_attn.linear_v"),
                           "bv": wd[f"{p}.self_attn.linear_v.bias"],
                           "wo": deq(wd, f"{p}.self_attn.linear_out"),
                           "bo": wd[f"{p}.self_attn.linear_out.bias"],
                           "wp": deq(wd, f"{p}.self_attn.linear_pos"),
                           "pos_bias_u": wd[f"{p}.self_attn.pos_bias_u"],
                           "pos_bias_v": wd[f"{p}.self_attn.pos_bias_v"]}}
            blocks.append(bw)
        t0 = time.perf_counter()
        for bw in blocks:
            h = orc.block_forward(h, bw, pe_h, H, ENC_FF, ENC_K, bf16=True)
        dt = (time.perf_counter() - t0) * ENC_LAYERS / len(blocks)
        return {"value": L0 / dt, "unit": "frames/s", "cores": threads, "kind": "port",
                "sample": f"utterance 0 ({L0} frames) through the first {len(blocks)} of the "
                          f"{ENC_LAYERS} layers, time scaled to {ENC_LAYERS} layers; CPU "
                          f"restatement (oracle block_forward, bf16 rounding), host CPU: "
                          f"{cpu_model()}"}
    # the variant with the weight cache on: each quantised weight's bf16 copy
    # is kept after its first use, so the timed steps read bf16 weights
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    barrier = (lambda: dist.barrier()) if world > 1 else (lambda: None)
    for k in range(3):
        step(k)
    n_kept = min(args.steps, 50)
    kept_ms = _timed_steps(lambda: step(0), n_kept, dev, world, barrier, flush)
    kept = {"value": world * valid * n_kept / (kept_ms / 1e3), "unit": "frames/s",
            "ms_per_step": kept_ms / n_kept, "steps": n_kept,
            "weights": "bf16 copies of the 8-bit weights, kept after their first use "
                       "(nrp_context_set_weight_cache on; 0.6 GB of device memory)"}
    # the measured line: every forward reads the u8 codes (weight cache off):
    # each layer's weights are dequantised once per forward, on a side stream
    # one layer ahead, into two bf16 slots
    ctx.set_weight_cache(False)
    _harness(args, world, rank, local, ctx, step, valid, flops, None, ENC_WORKLOAD,
             {"batch_per_gpu": ENC_B, "seq_len": ENC_T, "layers": ENC_LAYERS,
              "valid_frames_per_gpu": valid,
              "weights": "MLX 8-bit g64, fp16 scales; the u8 codes are read every forward "
                         "(weight cache off)",
              "parallelism": f"utterance-parallel replicas x{world}"},
             "weak", e2e, "bf16", cpu=cpu,
             hbm_bytes=bytes_, long_step=True, extra={"bf16_weight_copies": kept})
    if world > 1:
        dist.destroy_process_group()
    return 0


def main_subsampling(args):
    """Subsampling::forward_frames of config 3's batch from mel frames; one
    step = one forward; frames counted = encoder frames out (B * T')."""
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package
    world, rank, local = _dist_init(args)
    nrp = load_package()
    ctx = nrp.Context(local)
    rng = np.random.default_rng(77 + rank)
    sub = nrp.Subsampling(SUB_F, D, SUB_FACTOR, SUB_C, False, ctx=ctx)
    f = lambda sd, *sh: (rng.standard_normal(sh, dtype=np.float32) * sd)
    Fp, C = sub.feat_out, SUB_C
    wts = {"conv0": (f(0.3, C, 3, 3, 1), f(0.1, C)),
           "dw": [(f(0.3, C, 3, 3, 1), f(0.1, C)) for _ in range(2)],
           "pw": [(f(1 / 16, C, 1, 1, C), f(0.1, C)) for _ in range(2)],
           "out": (f(1 / math.sqrt(C * Fp), D, C * Fp), f(0.1, D))}
    sub.set_conv(0, *wts["conv0"])
    for i in range(2):
        sub.set_conv(2 + 3 * i, *wts["dw"][i])
        sub.set_conv(3 + 3 * i, *wts["pw"][i])
    sub.set_out(nrp.LinearLayer.standard(*wts["out"]))
    sub.set_dtype(nrp.BF16)
    dev = torch.device("cuda", local)
    x = rng.standard_normal((SUB_B, SUB_F, SUB_T), dtype=np.float32)
    lengths = rng.integers(SUB_LEN_LO, SUB_LEN_HI + 1, SUB_B).astype(np.int32)
    xd = torch.from_numpy(x).to(dev)
    ld = torch.from_numpy(lengths).to(dev)
    Tp = sub.output_length(SUB_T)
    out = torch.empty((SUB_B, Tp, D), dtype=torch.bfloat16, device=dev)

    def step(k, xin=xd, o=out):
        sub.forward(xin, ld, layout=nrp.FEATURES_BFT, out=o)

    x_host = torch.from_numpy(x).pin_memory()
    out_host = torch.empty_like(out, device="cpu").pin_memory()
    xs = [torch.empty_like(xd) for _ in range(2)]
    outs = [torch.empty_like(out) for _ in range(2)]
    e2e = (lambda slot: xs[slot].copy_(x_host, non_blocking=True),
           lambda slot: step(0, xs[slot], outs[slot]),
           lambda slot: out_host.copy_(outs[slot], non_blocking=True),
           x_host.numel() * 4, out_host.numel() * 2)
    T1, F1 = (SUB_T - 1) // 2 + 1, (SUB_F - 1) // 2 + 1
    T2, F2 = (T1 - 1) // 2 + 1, (F1 - 1) // 2 + 1
    T3, F3 = (T2 - 1) // 2 + 1, (F2 - 1) // 2 + 1
    frames = SUB_B * Tp
    # tensor work: the two pointwise convs and `out`; HBM work of the direct
    # convs: the mel read + the first depthwise output written, and the
    # second depthwise conv's input read + output written
    flops = {"gemm_bf16": 2 * SUB_B * (T2 * F2 + T3 * F3) * C * C + 2 * SUB_B * T3 * C * F3 * D}
    bytes_ = {"subsample": SUB_B * SUB_F * SUB_T * 4 + SUB_B * T2 * F2 * C * 2 * 2
              + SUB_B * T3 * F3 * C * 2}

    def cpu():
        """The oracle on utterance 0 (its masked mel), all host threads."""
        from oracle import oracle as orc
        threads = os.cpu_count() or 1
        orc.set_threads(threads)
        L0 = int(lengths[0])
        xu = np.ascontiguousarray(x[:1].transpose(0, 2, 1))
        xu[:, L0:] = 0.0
        t0 = time.perf_counter()
        orc.subsampling_forward(xu, wts, D, SUB_FACTOR, False, bf16=True)
        dt = time.perf_counter() - t0
        return {"value": Tp / dt, "unit": "frames/s", "cores": threads, "kind": "port",
                "sample": f"utterance 0 ({SUB_T} mel frames -> {Tp} encoder frames); CPU "
                          f"restatement (oracle subsampling_forward, bf16 rounding), host "
                          f"CPU: {cpu_model()}"}
    _harness(args, world, rank, local, ctx, step, frames, flops, None, SUB_WORKLOAD,
             {"batch_per_gpu": SUB_B, "mel_frames": SUB_T, "feat_in": SUB_F,
              "encoder_frames": Tp, "conv_channels": C, "d_model": D,
              "parallelism": f"utterance-parallel replicas x{world}"},
             "weak", e2e, "bf16", cpu=cpu, hbm_bytes=bytes_)
    if world > 1:
        dist.destroy_process_group()
    return 0


def main_stream_encoder(args):
    """The whole cache-aware streaming encoder step (forward_streaming): 64
    sessions, a chunk of 112 mel frames (14 encoder frames after causal 8x
    subsampling and the one pre-encoded frame dropped) through the
    subsampling and 24 streaming blocks (8-bit weights, conv caches, 70-frame
    attention caches, chunked_limited [70, 13]), each step replayed as a CUDA
    graph; the caches restart every 50 chunks; weak scaling (each rank its
    own sessions)."""
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package
    from oracle import oracle as orc  # quantiser of the synthetic checkpoint only
    world, rank, local = _dist_init(args)
    nrp = load_package()
    ctx = nrp.Context(local)
    rng = np.random.default_rng(4242 + rank)
    enc = nrp.ConformerEncoder(ENC_LAYERS, D, H, ENC_FF, ENC_K, causal_conv=True, ctx=ctx,
                               feat_in=SUB_F, subsampling_factor=8,
                               subsampling_conv_channels=SUB_C, causal_downsampling=True)
    sample_layers = _load_quant_layers(nrp, orc, enc, rng)
    f = lambda sd, *sh: (rng.standard_normal(sh, dtype=np.float32) * sd)
    sub = enc.subsampling
    Fp = sub.feat_out
    sub.set_conv(0, f(0.3, SUB_C, 3, 3, 1), f(0.1, SUB_C))
    for i in range(2):
        sub.set_conv(2 + 3 * i, f(0.3, SUB_C, 3, 3, 1), f(0.1, SUB_C))
        sub.set_conv(3 + 3 * i, f(1 / 16, SUB_C, 1, 1, SUB_C), f(0.1, SUB_C))
    sub.set_out(nrp.LinearLayer.standard(f(1 / math.sqrt(SUB_C * Fp), D, SUB_C * Fp), f(0.1, D)))
    enc.set_dtype(nrp.BF16)
    cache = enc.new_stream_cache(STR_SESS, STR_CACHE)
    actx = nrp.AttentionContext.new((STR_CACHE, STR_CHUNK - 1), "chunked_limited")
    dev = torch.device("cuda", local)
    mel_frames, drop = 8 * STR_CHUNK, 1
    mels = [torch.from_numpy(rng.standard_normal((STR_SESS, SUB_F, mel_frames), dtype=np.float32))
            .to(dev) for _ in range(4)]
    xin = [torch.empty_like(mels[0]) for _ in range(2)]
    outs = [torch.empty((STR_SESS, D, STR_CHUNK), dtype=torch.bfloat16, device=dev)
            for _ in range(2)]
    state = {"chunk": 0}

    def reset():
        cache.reset()
        state["chunk"] = 0

    def encoder_step(filled, slot):
        cache.filled = filled
        enc.forward_streaming(xin[slot], None, cache, drop, actx, out=outs[slot])

    # each chunk step replayed as a CUDA graph per (fill level, ring slots, slot)
    graphs = nrp.StreamingStepGraphs(encoder_step, cache.rings())

    def step(k, slot=None, eager=False):
        if state["chunk"] == STR_CHUNKS:
            reset()
        if slot is None:  # device-timed steps: the chunk comes from device memory
            slot = 0
            xin[0].copy_(mels[k % len(mels)], non_blocking=True)
        filled = min(state["chunk"] * STR_CHUNK, STR_CACHE)
        (encoder_step if eager else graphs)(filled, slot)
        state["chunk"] += 1
        return outs[slot]

    # capture every graph before anything is timed (each key's first step runs
    # eagerly, its second is captured)
    period = STR_CACHE // math.gcd(STR_CACHE, STR_CHUNK)
    for slot in (0, 1):
        for _ in range(2):
            reset()
            for k in range(STR_CACHE // STR_CHUNK + 1 + period):
                step(k, slot)
    torch.cuda.synchronize()
    reset()

    x_host = mels[0].cpu().pin_memory()
    out_host = torch.empty_like(outs[0], device="cpu").pin_memory()
    e2e = (lambda slot: xin[slot].copy_(x_host, non_blocking=True),
           lambda slot: step(0, slot),
           lambda slot: out_host.copy_(outs[slot], non_blocking=True),
           x_host.numel() * 4, out_host.numel() * 2)
    frames = STR_SESS * STR_CHUNK
    per_frame = 2 * 2 * (2 * D * ENC_FF) + 4 * 2 * D * D + 2 * D * 2 * D + 2 * D * D
    flops = {"gemm_bf16": ENC_LAYERS * per_frame * frames}

    def cpu():
        """The oracle on session 0: its subsampled chunk through the first two
        streaming layers, time scaled to 24 layers (the layers cost the same;
        the subsampling is timed once per chunk)."""
        threads = os.cpu_count() or 1
        orc.set_threads(threads)
        deq = lambda wd, k: orc.dequantize(wd[k + ".weight"], orc.bf16_round(wd[k + ".scales"]),
                                           orc.bf16_round(wd[k + ".biases"]), 64, 8)
        x = orc.bf16_round(rng.standard_normal((1, STR_CHUNK, D)).astype(np.float32))
        pe_h = orc.get_encoding(D, 5000, STR_CACHE + STR_CHUNK)
        t0 = time.perf_counter()
        for p, wd in sample_layers:
            lin = lambda n: (deq(wd, f"{p}.{n}"), wd.get(f"{p}.{n}.bias"))
            bw = {"ff1_1": lin("feed_forward1.linear1"), "ff1_2": lin("feed_forward1.linear2"),
                  "pw1": lin("conv.pointwise_conv1"), "pw2": lin("conv.pointwise_conv2"),
                  "ff2_1": lin("feed_forward2.linear1"), "ff2_2": lin("feed_forward2.linear2"),
                  "dw": (wd[f"{p}.conv.depthwise_conv.weight"].reshape(D, ENC_K),
                         wd[f"{p}.conv.depthwise_conv.bias"]),
                  "conv_norm": tuple(wd[f"{p}.conv.batch_norm.{n}"] for n in
                                     ("weight", "bias", "running_mean", "running_var")),
                  "norms": {o: (wd[f"{p}.{n}.weight"], wd[f"{p}.{n}.bias"])
                            for o, n in zip(orc.BLOCK_NORMS, nrp.BLOCK_NORMS)},
                  "attn": {"wq": deq(wd, f"{p}.self_attn.linear_q"),
                           "bq": wd[f"{p}.self_attn.linear_q.bias"],
                           "wk": deq(wd, f"{p}.self_attn.linear_k"),
                           "bk": wd[f"{p}.self_attn.linear_k.bias"],
                           "wv": deq(wd, f"{p}.self_attn.linear_v"),
                           "bv": wd[f"{p}.self_attn.linear_v.bias"],
                           "wo": deq(wd, f"{p}.self_attn.linear_out"),
                           "bo": wd[f"{p}.self_attn.linear_out.bias"],
                           "wp": deq(wd, f"{p}.self_attn.linear_pos"),
                           "pos_bias_u": wd[f"{p}.self_attn.pos_bias_u"],
                           "pos_bias_v": wd[f"{p}.self_attn.pos_bias_v"]}}
            hc = np.zeros((1, STR_CACHE, D), np.float32)
            cc = np.zeros((1, ENC_K - 1, D), np.float32)
            x, _ = orc.stream_block_step(x, bw, pe_h, H, ENC_FF, ENC_K, hc, cc, STR_CACHE,
                                         STR_CHUNK, STR_CACHE, STR_CHUNK - 1, True)
        dt = (time.perf_counter() - t0) * ENC_LAYERS / len(sample_layers)
        return {"value": STR_CHUNK / dt, "unit": "frames/s", "cores": threads, "kind": "port",
                "sample": f"one session's chunk ({STR_CHUNK} frames, full caches) through the "
                          f"first {len(sample_layers)} of {ENC_LAYERS} streaming layers, time "
                          f"scaled to {ENC_LAYERS} layers (subsampling not timed); CPU "
                          f"restatement (oracle stream_block_step, bf16 rounding), host CPU: "
                          f"{cpu_model()}"}
    _harness(args, world, rank, local, ctx, step, frames, flops, None, STRENC_WORKLOAD,
             {"sessions_per_gpu": STR_SESS, "chunk": STR_CHUNK, "cache": STR_CACHE,
              "layers": ENC_LAYERS, "mel_frames_per_chunk": mel_frames, "feat_in": SUB_F,
              "weights": "MLX 8-bit g64, fp16 scales",
              "parallelism": f"session-parallel replicas x{world}"},
             "weak", e2e, "bf16", cpu=cpu, reset=reset,
             prof_step=lambda k: step(k, eager=True))
    if world > 1:
        dist.destroy_process_group()
    return 0


def main_stream(args):
    """Config 2: one chunk of 14 frames for 64 sessions through 24 layers of
    forward_with_cache, each chunk step replayed as a CUDA graph (one per fill
    level and ring position); weak scaling (each rank its own 64 sessions)."""
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package
    world, rank, local = _dist_init(args)
    nrp = load_package()
    ctx = nrp.Context(local)
    rng = np.random.default_rng(777 + rank)
    dev = torch.device("cuda", local)
    f = lambda *sh: (rng.standard_normal(sh, dtype=np.float32) * 0.02)
    layers, caches = [], []
    for i in range(STR_LAYERS):
        a = nrp.RelPositionMultiHeadAttention(D, H, True, ctx=ctx)
        for which, bias in ((nrp.LINEAR_Q, True), (nrp.LINEAR_K, True), (nrp.LINEAR_V, True),
                            (nrp.LINEAR_OUT, True), (nrp.LINEAR_POS, False)):
            a.set_linear(which, nrp.LinearLayer.standard(f(D, D), f(D) if bias else None))
        a.set_pos_bias(f(H, D // H), f(H, D // H))
        a.set_dtype(nrp.BF16)
        layers.append(a)
        caches.append(nrp.AttentionCache(a, STR_SESS, STR_CACHE))
    actx = nrp.AttentionContext.new((STR_CACHE, STR_CHUNK - 1), "chunked_limited")
    pe = nrp.RelPositionalEncoding(D, 5000, True, device=local)
    pe.set_dtype(nrp.BF16)
    pos = pe.get_encoding(STR_CACHE + STR_CHUNK)
    xs = [torch.from_numpy(rng.standard_normal((STR_SESS, STR_CHUNK, D), dtype=np.float32))
          .to(dev, torch.bfloat16) for _ in range(4)]
    bufs = [torch.empty_like(xs[0]) for _ in range(2)]
    # fixed input/output buffers per slot: the chunk step runs as CUDA graphs
    # (StreamingStepGraphs), whose launches read and write fixed addresses
    xin = [torch.empty_like(xs[0]) for _ in range(2)]
    outs = [torch.empty_like(xs[0]) for _ in range(2)]
    state = {"chunk": 0}

    def reset():
        for c in caches:
            c.reset()
        state["chunk"] = 0

    def layers_step(filled, slot):
        h = xin[slot]
        for i, a in enumerate(layers):
            o = outs[slot] if i == len(layers) - 1 else bufs[i & 1]
            a.forward_with_cache(h, pos, caches[i], filled, STR_CHUNK, actx, out=o)
            h = o

    graphs = nrp.StreamingStepGraphs(layers_step, caches)

    def step(k, slot=None, eager=False):
        c = state["chunk"]
        if c == STR_CHUNKS:
            reset()
            c = 0
        if slot is None:  # device-timed steps: the chunk comes from device memory
            slot = 0
            xin[0].copy_(xs[k % len(xs)], non_blocking=True)
        (layers_step if eager else graphs)(min(c * STR_CHUNK, STR_CACHE), slot)
        state["chunk"] = c + 1
        return outs[slot]

    # capture every (fill level, ring position, slot) graph before anything is
    # timed: each key's first step runs eagerly, its second is captured
    period = STR_CACHE // math.gcd(STR_CACHE, STR_CHUNK)
    for slot in (0, 1):
        for _ in range(2):
            reset()
            for k in range(STR_CACHE // STR_CHUNK + 1 + period):
                step(k, slot)
    torch.cuda.synchronize()
    reset()

    x_host = torch.empty((STR_SESS, STR_CHUNK, D), dtype=torch.bfloat16).pin_memory()
    x_host.copy_(xs[0].cpu())
    out_host = torch.empty_like(x_host).pin_memory()
    e2e = (lambda slot: xin[slot].copy_(x_host, non_blocking=True),
           lambda slot: step(0, slot),
           lambda slot: out_host.copy_(outs[slot], non_blocking=True),
           x_host.numel() * 2, out_host.numel() * 2)

    frames = STR_SESS * STR_CHUNK
    M = frames
    # linear_pos runs once per positional length (attention.rs:749-761): not per step
    flops = {"gemm_bf16": STR_LAYERS * 4 * 2 * M * D * D}
    kv = STR_SESS * (STR_CACHE + STR_CHUNK) * D * 2 * 2
    qo = 2 * STR_SESS * STR_CHUNK * D * 2
    p_rows = (2 * (STR_CACHE + STR_CHUNK) - 1) * D * 2
    hbm = {"attn_stream": STR_LAYERS * (kv + qo + p_rows),
           "ring_append": STR_LAYERS * 3 * STR_SESS * STR_CHUNK * D * 2 * 2}
    _harness(args, world, rank, local, ctx, step, frames, flops, None, STR_WORKLOAD,
             {"sessions_per_gpu": STR_SESS, "chunk": STR_CHUNK, "cache": STR_CACHE,
              "layers": STR_LAYERS,
              "parallelism": f"session-parallel replicas x{world}"},
             "weak", e2e, "bf16", hbm_bytes=hbm,
             reset=reset, prof_step=lambda k: step(k, eager=True))
    if world > 1:
        dist.destroy_process_group()
    return 0


def main_single(args):
    """Config 0: one fp32 layer on [1, 125, 1024] (launch-bound)."""
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package
    world, rank, local = _dist_init(args)
    nrp = load_package()
    ctx = nrp.Context(local)
    rng = np.random.default_rng(99 + rank)
    f = lambda *sh: (rng.standard_normal(sh, dtype=np.float32) * 0.02)
    w = {"wq": f(D, D), "bq": f(D), "wk": f(D, D), "bk": f(D), "wv": f(D, D), "bv": f(D),
         "wo": f(D, D), "bo": f(D), "wp": f(D, D), "pos_bias_u": f(H, D // H),
         "pos_bias_v": f(H, D // H)}
    attn = nrp.RelPositionMultiHeadAttention(D, H, True, ctx=ctx)
    for which, (wk, bk) in enumerate((("wq", "bq"), ("wk", "bk"), ("wv", "bv"), ("wo", "bo"),
                                      ("wp", None))):
        attn.set_linear(which, nrp.LinearLayer.standard(w[wk], w[bk] if bk else None))
    attn.set_pos_bias(w["pos_bias_u"], w["pos_bias_v"])
    dev = torch.device("cuda", local)
    x = rng.standard_normal((1, SGL_T, D), dtype=np.float32)
    xd = torch.from_numpy(x).to(dev)
    out = torch.empty_like(xd)
    pe = nrp.RelPositionalEncoding(D, 5000, True, device=local)
    pos = pe.get_encoding(SGL_T)

    def step(k, xin=xd, o=out):
        attn.forward(xin, pos, None, None, out=o)

    x_host = torch.from_numpy(x).pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    xs = [torch.empty_like(xd) for _ in range(2)]
    outs = [torch.empty_like(xd) for _ in range(2)]
    e2e = (lambda slot: xs[slot].copy_(x_host, non_blocking=True),
           lambda slot: step(0, xs[slot], outs[slot]),
           lambda slot: out_host.copy_(outs[slot], non_blocking=True),
           x_host.numel() * 4, out_host.numel() * 4)

    def cpu():
        from oracle import oracle as orc
        threads = os.cpu_count() or 1
        orc.set_threads(threads)
        pe_h = orc.get_encoding(D, 5000, SGL_T)
        orc.mha_forward(x, w, pe_h, H)
        runs = []
        for _ in range(5):
            t0 = time.perf_counter()
            orc.mha_forward(x, w, pe_h, H, mode=orc.ORC_REFERENCE_ALGO)
            runs.append(time.perf_counter() - t0)
        med = statistics.median(runs)
        return {"value": SGL_T / med, "unit": "frames/s", "cores": threads, "kind": "port",
                "sample": f"the whole config-0 forward ({SGL_T} frames), median of 5; CPU "
                          f"restatement of the reference algorithm in f32, host CPU: "
                          f"{cpu_model()}"}
    flops = {"gemm_f32": 4 * 2 * SGL_T * D * D + 2 * (2 * SGL_T - 1) * D * D,
             "attn_simt": 3 * 2 * (D // H) * H * SGL_T * SGL_T}
    _harness(args, world, rank, local, ctx, step, SGL_T, flops, None, SGL_WORKLOAD,
             {"batch_per_gpu": 1, "seq_len": SGL_T, "d_model": D, "heads": H,
              "parallelism": f"replicas x{world}"},
             "weak", e2e, "f32", cpu=cpu)
    if world > 1:
        dist.destroy_process_group()
    return 0


def _peaks():
    """(burst, sustained) bf16 TFLOP/s and where they come from."""
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peaks = json.load(open(peaks_path)) if os.path.exists(peaks_path) else {}
    b, s_ = peaks.get("bf16_tflops"), peaks.get("bf16_tflops_sustained")
    if b and s_:
        return b, s_, "measured (bf16_tflops, MEASURED_PEAKS.json)"
    return 1590.0, 1400.0, "fallback 1.59 PFLOP/s burst"


def _peak(long_step=False):
    """The denominator of a workload's tensor roofline: the burst peak for
    steps of a few ms or less, the sustained one for steps long enough to
    settle under the power cap."""
    b, s_, src = _peaks()
    if long_step:
        return s_, src.replace("bf16_tflops,", "bf16_tflops_sustained,").replace(
            "1.59 PFLOP/s burst", "1.4 PFLOP/s sustained") + "; sustained: long steps"
    return b, src


def main_long(args):
    """Config 4: one step = the windowed forward over [4, 12500, 1024]; with
    N ranks each rank runs its segment of the sequence
    (nrp_attn_forward_seq_sharded: local projections, 128-frame K/V halo
    over NCCL, attention, linear_out).  Strong scaling: the total work is
    fixed; value = all frames / the slowest rank's time."""
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    nrp = load_package()
    ctx = nrp.Context(local)
    w, attn, actx, pos, x = _long_module(nrp, ctx, local)
    dev = torch.device("cuda", local)
    halo = None
    if world > 1:
        halo = nrp.HaloComm.from_process_group(ctx=ctx, timeout_ms=120000)
        plan = halo.plan(LONG_T, actx)
        s0, n0 = plan.start, plan.len
    else:
        s0, n0 = 0, LONG_T
    x_loc = np.ascontiguousarray(x[:, s0:s0 + n0])
    xd = torch.from_numpy(x_loc).to(dev, torch.bfloat16)
    out = torch.empty_like(xd)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()

    def step(o=out, xin=xd):
        if halo is None:
            attn.forward(xin, pos, actx, None, out=o)
        else:
            attn.forward_seq_sharded(xin, pos, LONG_T, halo, actx, None, out=o)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(args.warmup, 3)):
        step()
    if halo is not None:
        halo.check()
    ctx.check()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for k in range(args.steps):
            flush.zero_()
            starts[k].record(stream)
            step()
            ends[k].record(stream)
        if halo is not None:
            halo.check()
        torch.cuda.synchronize()
    barrier()
    ctx.check()
    total_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in zip(starts, ends)))
    frames = LONG_B * LONG_T
    value = frames * args.steps / (total_ms / 1e3)

    ctx.profile(True)
    ctx.profile_reset()
    for k in range(args.steps):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    prof = ctx.profile_read()
    ctx.profile(False)
    launches = sum(n for n, _ in prof.values())

    x_host = torch.from_numpy(x_loc).to(torch.bfloat16).pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    xs = [torch.empty_like(xd) for _ in range(2)]
    outs = [torch.empty_like(xd) for _ in range(2)]

    def h2d_fn(slot):
        xs[slot].copy_(x_host, non_blocking=True)

    def compute_fn(slot):
        step(outs[slot], xs[slot])

    def d2h_fn(slot):
        out_host.copy_(outs[slot], non_blocking=True)

    run_pipelined(4, h2d_fn, compute_fn, d2h_fn)  # warm-up
    barrier()
    e2e_ms = run_pipelined(args.steps, h2d_fn, compute_fn, d2h_fn)
    if halo is not None:
        halo.check()
    barrier()
    e2e_ms = max_over_ranks(e2e_ms)
    e2e_value = frames * args.steps / (e2e_ms / 1e3)

    tflops_peak, peak_src = _peak()
    proj, pos_f, attn_f = long_flops()
    share = {"gemm_bf16": (proj + pos_f) / world, "attn_sm100": attn_f / world}
    kern, rk = {}, {}
    tot = max(sum(m for _, m in prof.values()), 1e-9)
    for name, (n, ms) in prof.items():
        kern[name] = {"launches": n, "ms_total": ms, "share": ms / tot}
        if name in share:
            a = share[name] * args.steps / (ms / 1e3) / 1e12
            rk[name] = {"achieved": a, "frac": a / tflops_peak, "unit": "TFLOP/s",
                        "algorithmic_flop_per_launch": share[name] * args.steps / n}
    if world == 1 and "attn_sm100" in rk:
        rk["attn_sm100"]["traffic"] = LONG_ATTN_TRAFFIC
    dominant = max(prof.items(), key=lambda kv: kv[1][1])[0] if prof else None
    roof = None
    if dominant in rk:
        roof = {"bound": "tensor", "kernel": dominant, "achieved": rk[dominant]["achieved"],
                "peak": tflops_peak, "unit": "TFLOP/s", "frac": rk[dominant]["frac"],
                "traffic": None, "peak_source": peak_src,
                "algorithmic_flop_per_launch": rk[dominant]["algorithmic_flop_per_launch"]}
    whole = (proj + pos_f + attn_f) * args.steps / (total_ms / 1e3) / 1e12

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as orc
        threads = os.cpu_count() or 1
        orc.set_threads(threads)
        pe_h = orc.get_encoding(D, 5000, LONG_T)
        t0 = time.perf_counter()
        orc.mha_forward(x[:1], w, pe_h, H, context=(*LONG_WINDOW, False), bf16=True)
        dt = time.perf_counter() - t0
        cpu = {"value": LONG_T / dt, "unit": "frames/s", "cores": threads, "kind": "port",
               "sample": f"1 of the 4 utterances ({LONG_T} frames), one run; CPU restatement "
                         f"(ORC_DIRECT: window-skipping attention, every P row projected as "
                         f"the reference does), host CPU: {cpu_model()}"}

    if halo is not None:
        halo.close()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": LONG_WORKLOAD, "batch": LONG_B, "seq_len": LONG_T,
                       "d_model": D, "heads": H, "window": list(LONG_WINDOW),
                       "frames_per_rank": n0 * LONG_B,
                       "l2": "flushed between timed steps (256 MiB write, outside the events)",
                       "parallelism": f"sequence split x{world}, K/V halo over NCCL"
                                      if world > 1 else "one GPU"},
            "e2e": {"value": e2e_value, "unit": "frames/s",
                    "h2d_bytes_per_step": x_host.numel() * 2,
                    "d2h_bytes_per_step": out_host.numel() * 2},
            "gpu_launches": launches,
            "whole_step_tflops": whole,
            "roofline": roof,
            "roofline_kernels": rk,
            "kernels": kern,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
