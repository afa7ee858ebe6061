#!/usr/bin/env python
"""Weight-stream bandwidth of the GGUF decode GEMV / MoE hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--quick]

Headline (one JSON line on rank 0): BASELINE config 1 -- Q4Gemv iq2=3 (IQ2_XXS), R=1, K=4096,
N=14336 -- as weight-stream GB/s (algorithmic bytes = the weight tensor, 15,138,816 B per call).

* A step = one CUDA-graph replay of `rounds` passes over `copies` distinct weight copies
  (copies * 15.1 MB > 2 x L2, so every call streams from HBM); calls are launched with
  programmatic dependent launch.  value = weight bytes of all ranks / max-over-ranks time.
* e2e = the same metric through the public C ABI with host buffers: each step copies x from pinned
  host memory, runs one pass over the weight copies and reads every y back to pinned host memory
  (all inside the captured step).
* roofline = achieved GB/s of the GEMV kernel vs the measured HBM copy bandwidth in
  MEASURED_PEAKS.json; traffic (DRAM bytes per launch) comes from the committed ncu summary
  profiles/dram_traffic.json when present.
* cpu_baseline = the oracle port of the reference's CPU path (gguf-py dequantise + fp32 matmul)
  on a bounded row sample, all host threads.
* configs = every BASELINE config at 1 GPU (skipped with --quick or N > 1).

N > 1 (torchrun): the headline is the sharded config, BASELINE config 4 (the Q8_0 LM head, R=1,
N=131072) row-split over the N GPUs with the all-gather fused into the GEMV kernel (strong scaling,
value = whole-tensor bytes / max-over-ranks time per call; parity against the single-GPU op checked
in the same run).  The line also carries the same workload on one GPU, C4 at R=4/8/16, the GEMV +
NCCL all-gather baseline, the expert-parallel C3 MoE and config 1 as independent replicas.
``--impl reference`` times the reference's CPU path (oracle port) on the same metric.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
HEADLINE = dict(cfg="C1", op="iq2_xxs", R=1, N=14336, K=4096)
ROW_BYTES = {"q8_0": lambda K: K // 32 * 34, "iq2_xxs": lambda K: K // 256 * 66, "nvfp4": lambda K: K // 64 * 36}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--quick", action="store_true", help="headline only")
    ap.add_argument("--cpu-table", action="store_true",
                    help="print the reference CPU path's time per BASELINE config (host cores only) and exit")
    # --profile-case: run one op a few times with eager launches (the target of the ncu captures
    # whose summaries are in profiles/), then exit
    ap.add_argument("--profile-case", action="store_true", help="run one op --iters times (for ncu) and exit")
    ap.add_argument("--op", default="iq2_xxs",
                    choices=["q8_0", "iq2_xxs", "nvfp4", "moe", "route", "embed", "norm", "q4_split", "mamba"])
    ap.add_argument("--R", type=int, default=1)
    ap.add_argument("--N", type=int, default=14336)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--copies", type=int, default=3)
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--fast-mode", type=int, default=1, help="gguf_set_fast_paths value (0 = generic engine)")
    return ap.parse_args()


def profile_case(a):
    """One op, `a.iters` eager launches on cuda:0 (weights with the BASELINE distributions, a distinct
    weight copy per iteration when `a.copies` > 1 so that launches stream from HBM, not L2):

        python bench.py --profile-case --op iq2_xxs --R 1 --N 14336 --K 4096 --iters 3
        python bench.py --profile-case --op moe --R 1 --iters 3
        python bench.py --profile-case --op embed --R 4096 --N 131072 --K 4096
        python bench.py --profile-case --op norm --R 4096 --K 4096
        python bench.py --profile-case --op q4_split --R 1 --N 14336 --K 4096
        python bench.py --profile-case --op mamba --R 1
    """
    import torch

    from gguf_onnx_ops_b200 import ops

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    ops.set_pdl(not a.no_pdl)
    ops.set_fast_paths(a.fast_mode)
    if a.op == "embed":  # Q8Embed: R ids from a [N, K] Q8_0 table
        table = gen_weights("q8_0", a.N, a.K, seed=4, dev=dev)
        ids = torch.randint(0, a.N, (a.R,), device=dev)
        out = torch.empty(a.R, a.K, dtype=torch.bfloat16, device=dev)
        for _ in range(a.iters):
            ops.q8_0_embed_into(table, ids, out, a.N, a.K // 32 * 34, a.R)
    elif a.op == "norm":  # SkipRmsNorm [R, K] with the sum written
        xs = [torch.randn(a.R, a.K, device=dev).bfloat16() for _ in range(a.copies)]
        sk = torch.randn(a.R, a.K, device=dev).bfloat16()
        gamma = torch.rand(a.K, device=dev) + 0.5
        y, sm = torch.empty_like(sk), torch.empty_like(sk)
        for i in range(a.iters):
            ops.rms_norm_into(xs[i % a.copies], sk, gamma, y, sm, a.R, a.K, 1e-5)
    elif a.op == "q4_split":  # Q4Gemv iq2=0 (legacy split layout)
        from gguf_onnx_ops_b200 import _lib

        ws = [torch.randint(0, 256, (a.N, a.K // 2), device=dev, dtype=torch.uint8) for _ in range(a.copies)]
        sc = (torch.rand(a.N, a.K // 32, device=dev) * 0.02).bfloat16()
        x = torch.randn(a.R, a.K, device=dev).bfloat16()
        y = torch.empty(a.R, a.N, dtype=torch.bfloat16, device=dev)
        for i in range(a.iters):
            ops.gemv_legacy_into(_lib.GGUF_LAYOUT_Q4_SPLIT, x, ws[i % a.copies], sc, None, y, a.R, a.N, a.K)
    elif a.op == "mamba":  # MambaStep, heads 128, n_groups 8
        heads, ng = 128, 8
        di, cd = heads * 64, heads * 64 + 2 * ng * 128
        proj = torch.randn(a.R, di + cd + heads, device=dev).bfloat16()
        cs = torch.randn(1, cd, 3, device=dev).bfloat16()
        ss = [torch.randn(1, heads, 128, 64, device=dev) * 0.1 for _ in range(a.copies)]
        cw, cb = (torch.randn(cd, 4, device=dev) * 0.3).bfloat16(), (torch.randn(cd, device=dev) * 0.1).bfloat16()
        hv = [torch.randn(heads, device=dev) for _ in range(3)]
        nw = torch.rand(di, device=dev) + 0.5
        y = torch.empty(a.R, di, dtype=torch.bfloat16, device=dev)
        cso, sso = torch.empty_like(cs), torch.empty_like(ss[0])
        xbc = torch.empty(a.R, cd, dtype=torch.bfloat16, device=dev)
        ypre = torch.empty(a.R, di, device=dev)
        for i in range(a.iters):
            ops.mamba_step_into(proj, cs, ss[i % a.copies], cw, cb, hv[0], -hv[1].abs(), hv[2], nw, None, y, cso, sso,
                                xbc, ypre, R=a.R, state_rows=1, heads=heads, n_groups=ng, eps=1e-5, tmin=0.001)
    elif a.op in ("moe", "route"):
        E, H, I, topk = 128, 1024, 1792, 6
        w1 = gen_weights("iq2_xxs", E * I, H, seed=2, dev=dev).reshape(E, I, -1)
        w2 = gen_weights("iq2_xxs", E * H, I, seed=3, dev=dev).reshape(E, H, -1)
        gw = torch.randn(E, H, device=dev) * 0.02
        bias = torch.randn(E, device=dev) * 0.01
        x = torch.randn(a.R, H, device=dev).bfloat16()
        z = torch.randn(a.R, H, device=dev).bfloat16()
        for _ in range(a.iters):
            idx, wt, _ = ops.MoeRouteGGUF(x, gw, bias, topk, 1.0)
            if a.op == "moe":
                ops.MoeVerify(z, idx, wt, w1, None, w2, None, topk=topk)
    else:
        base = gen_weights(a.op, a.N, a.K, seed=1, dev=dev)
        ws = replicate(base, a.copies)
        x = torch.randn(a.R, a.K, device=dev).bfloat16()
        gs = torch.tensor([1.0 / 448.0], device=dev)
        y = torch.empty(a.R, a.N, dtype=torch.bfloat16, device=dev)
        for i in range(a.iters):
            gemv_call(a.op, x, ws[i % len(ws)], y, gs, a.R, a.N, a.K)
    torch.cuda.synchronize()
    print("ok")


def cpu_table():
    """The reference harness's CPU path per BASELINE config on this host: bounded row samples of
    dequantise + fp32 matmul and of the matmul alone, scaled to µs per full call; for C3 the oracle's
    per-(row, expert) MoE loop on 6 distinct experts per row."""
    import oracle as O
    from oracle import inputs as I

    out = {}
    for name, op, R, N, K in ([("C0", "q8_0", 1, 4096, 4096)] +
                              [("C1", "iq2_xxs", R, 14336, 4096) for R in (1, 4, 8)] +
                              [("C2", "nvfp4", R, 13824, 5120) for R in (1, 8, 16)] +
                              [("C4", "q8_0", R, 131072, 4096) for R in (1, 4, 8, 16)]):
        cb = cpu_baseline(op, R, N, K, budget_s=2.0)
        wbytes = N * ROW_BYTES[op](K)
        out[f"{name}_R{R}"] = {"cores": cb["cores"], "dequant_matmul_us": round(wbytes / (cb["value"] * 1e9) * 1e6, 1),
                               "matmul_only_us": round(wbytes / (cb["matmul_only_gbs"] * 1e9) * 1e6, 1),
                               "sample": cb["sample"]}
    for R in (1, 4, 8):
        g = I.rng(R)
        E, H, Idim, topk = 128, 1024, 1792, 6
        z = I.bf16_normal(g, (R, H))
        idx = np.stack([g.permutation(E)[:topk] for _ in range(R)]).astype(np.int32)
        w = g.random((R, topk)).astype(np.float32)
        used = sorted(set(idx.reshape(-1).tolist()))
        t0 = time.perf_counter()
        d1 = {e: O.dequant_iq2_xxs(I.iq2_xxs_weights(g, (Idim,), H)) for e in used}
        d2 = {e: O.dequant_iq2_xxs(I.iq2_xxs_weights(g, (H,), Idim)) for e in used}
        t1 = time.perf_counter()
        O.moe_ref(z, idx, w, d1, d2)
        t2 = time.perf_counter()
        out[f"C3_R{R}"] = {"cores": 1, "dequant_matmul_us": round((t2 - t0) * 1e6, 1),
                           "matmul_only_us": round((t2 - t1) * 1e6, 1),
                           "sample": f"{len(used)} experts: numpy dequantise + fp64 per-pair loop (1 thread)"}
    print(json.dumps(out), flush=True)


# ------------------------------------------------------------------------------------------------
# distributed plumbing
# ------------------------------------------------------------------------------------------------
def dist_setup(n):
    import torch

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------------------------
# clocks (NVML, sampled in a thread during the timed region)
# ------------------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index):
        self.samples, self.reasons, self.max = [], 0, None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 -- clocks are reported as unavailable
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv:
            self.t.join()

    def report(self):
        if not self.nv or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max, "reasons": ["unavailable"]}
        names = [n for b, n in self.REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max, "reasons": names,
                "samples": len(self.samples)}


# ------------------------------------------------------------------------------------------------
# synthetic weights on the device (BASELINE distributions)
# ------------------------------------------------------------------------------------------------
def gen_weights(op, N, K, seed, dev):
    """Raw GGUF bytes [N, row_bytes] with the BASELINE config distributions, built on the device."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    if op == "q8_0":  # Q8_0 of N(0, 0.02): d = amax/127, q = roundf(v / d) (ggml rounding), d as fp16
        w = torch.randn(N, K // 32, 32, generator=g, device=dev) * 0.02
        d = w.abs().amax(-1, keepdim=True) / 127
        inv = torch.where(d == 0, torch.zeros_like(d), 1.0 / d)
        v = w * inv
        q = (torch.sign(v) * torch.floor(v.abs() + 0.5)).to(torch.int8)
        blk = torch.cat([d.half().view(torch.uint8), q.view(torch.uint8)], -1)
        return blk.reshape(N, -1).contiguous()
    if op == "iq2_xxs":  # fp16 d = |N(0,1)| * 0.002, then 64 uniform bytes
        blk = torch.randint(0, 256, (N, K // 256, 66), generator=g, device=dev, dtype=torch.uint8)
        d = (torch.randn(N, K // 256, 1, generator=g, device=dev).abs() * 0.002).half()
        blk[..., :2] = d.view(torch.uint8)
        return blk.reshape(N, -1).contiguous()
    if op == "nvfp4":  # 4 UE4M3 scales uniform over the codes of [2^-4, 2^2], then 32 uniform bytes
        blk = torch.randint(0, 256, (N, K // 64, 36), generator=g, device=dev, dtype=torch.uint8)
        blk[..., :4] = torch.randint(0x18, 0x49, (N, K // 64, 4), generator=g, device=dev, dtype=torch.uint8)
        return blk.reshape(N, -1).contiguous()
    raise ValueError(op)


def replicate(t, copies):
    import torch

    out = [t]
    for _ in range(copies - 1):
        c = torch.empty_like(t)
        c.copy_(t)
        out.append(c)
    return out


def n_copies(bytes_per):
    return max(1, math.ceil(2.2 * L2_BYTES / bytes_per)) if bytes_per < 2.2 * L2_BYTES else 1


# ------------------------------------------------------------------------------------------------
# timing helpers
# ------------------------------------------------------------------------------------------------
def capture(fn):
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()  # warm-up outside capture (sets kernel attributes)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def time_graph(g, steps, warmup, world=1):
    import torch

    torch.cuda.synchronize()
    barrier(world)  # ranks start the warm-up together (sharded calls wait on their peers)
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    return e0.elapsed_time(e1)  # ms


def gemv_call(op, x, w, y, gs, R, N, K):
    from gguf_onnx_ops_b200 import ops

    if op == "q8_0":
        ops.q8_0_gemv_into(x, w, y, R, N, K)
    elif op == "iq2_xxs":
        ops.iq2_xxs_gemv_into(x, w, y, R, N, K)
    else:
        ops.nvfp4_gemv_into(x, w, gs, y, R, N, K)


def bench_gemv(op, R, N, K, steps, warmup, dev, target_step_ms=8.0, world=1, sampler=None):
    """Returns dict(us_per_call, gbs, calls, ...) for a dense GGUF GEMV config."""
    import torch

    wbytes = N * ROW_BYTES[op](K)
    copies = n_copies(wbytes)
    base = gen_weights(op, N, K, seed=1, dev=dev)
    ws = replicate(base, copies)
    del base
    x = (torch.randn(R, K, device=dev)).bfloat16()
    ys = [torch.empty(R, N, dtype=torch.bfloat16, device=dev) for _ in range(copies)]
    gs = torch.tensor([1.0 / 448.0], device=dev)

    def one_pass():
        for w, y in zip(ws, ys):
            gemv_call(op, x, w, y, gs, R, N, K)

    # calibrate rounds per step so one step lasts ~target_step_ms
    g1 = capture(one_pass)
    ms1 = time_graph(g1, 5, 2) / 5
    rounds = max(1, int(round(target_step_ms / max(ms1, 1e-3))))

    def step():
        for _ in range(rounds):
            one_pass()

    g = capture(step) if rounds > 1 else g1
    if sampler is not None:
        with sampler:
            ms = time_graph(g, steps, warmup, world)
    else:
        ms = time_graph(g, steps, warmup, world)
    ms = max_over_ranks(ms, world)
    calls = steps * rounds * copies
    us = ms * 1e3 / calls
    out = dict(us_per_call=us, gbs=wbytes / (us * 1e-6) / 1e9, weight_bytes=wbytes, copies=copies, rounds=rounds,
               calls=calls, ms_total=ms, ms_per_step=ms / steps, step_ms_graph_single_pass=ms1)
    del g, g1
    return out, (ws, x, ys, gs, wbytes, copies)


def seeded_bf16(shape, seed, dev):
    """bf16 N(0, 1) from a seeded device generator: the same tensor on every rank."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return torch.randn(*shape, generator=g, device=dev).bfloat16()


def bench_rowsplit(R, steps, warmup, dev, world, rank, nccl=False, e2e=False, sampler=None):
    """C4 LM head (Q8_0, N=131072, K=4096) row-split over the group: per call, each GPU streams its
    N/world rows and stores its y shard into every GPU's y inside the same kernel (NVLink peer
    stores + epoch flags).  Every rank builds the same full weight matrix and keeps its shard, so
    before timing the gathered y of one call is compared bit for bit with the single-GPU op on the
    full matrix (same kernel per row: equal bits expected), on every rank.  Optional baseline: the
    same per-GPU GEMV into a local shard followed by an NCCL all-gather (R = 1).  Optional e2e: x from
    pinned host memory, one pass of calls, every y back to pinned host memory on rank 0.  Times are
    the max over ranks."""
    import torch
    import torch.distributed as dist

    from gguf_onnx_ops_b200 import _lib, ops
    from gguf_onnx_ops_b200.sharded import RowSplitGemv, shard_rows

    N, K = 131072, 4096
    rb = ROW_BYTES["q8_0"](K)
    row0, rows = shard_rows(N, world, rank)
    _lib.device_status()  # clear: the status reported below is this entry's own
    full = gen_weights("q8_0", N, K, seed=1, dev=dev)  # the same on every rank
    base = full[row0:row0 + rows].contiguous()
    copies = n_copies(rows * rb)
    x = seeded_bf16((R, K), 100 + R, dev)
    op = RowSplitGemv(_lib.GGUF_TYPE_Q8_0, base, N, row0, K, r_max=R)
    # parity: the gathered y against the single-GPU op on the full matrix
    y = op(x, w=base)
    y_ref = torch.empty(R, N, dtype=torch.bfloat16, device=dev)
    ops.q8_0_gemv_into(x, full, y_ref, R, N, K)
    torch.cuda.synchronize()
    bad = torch.tensor([float((y.view(torch.int16) != y_ref.view(torch.int16)).sum().item())], device=dev)
    dist.all_reduce(bad, op=dist.ReduceOp.MAX)
    mismatches = int(bad.item())
    del full, y_ref, y
    ws = replicate(base, copies)
    del base
    torch.cuda.empty_cache()

    def fused_pass():
        for w in ws:
            op(x, w=w)

    # rounds of the pass per step so that a step lasts ~4 ms (the same count on every rank: every
    # rank must issue the same calls)
    g = capture(fused_pass)
    pass_ms = max_over_ranks(time_graph(g, 3, 1, world) / 3, world)
    rounds = max(1, int(math.ceil(4.0 / max(pass_ms, 1e-3))))
    if rounds > 1:
        del g

        def step():
            for _ in range(rounds):
                fused_pass()

        g = capture(step)
    if sampler is not None:
        with sampler:
            ms = max_over_ranks(time_graph(g, steps, warmup, world), world)
    else:
        ms = max_over_ranks(time_graph(g, steps, warmup, world), world)
    del g
    fused_us = ms * 1e3 / (steps * rounds * copies)
    total = N * rb
    out = dict(world=world, R=R, fused_us_per_call=fused_us, fused_gbs=total / (fused_us * 1e-6) / 1e9,
               rows_per_gpu=rows, copies=copies, rounds=rounds, calls=steps * rounds * copies, ms_total=ms,
               parity="ok" if mismatches == 0 else f"mismatch: {mismatches} of {R * N} values differ (max over ranks)",
               parity_check="gathered y of one call == single-GPU Q8Gemv on the full matrix, bit for bit, every rank")
    if e2e:
        # public API end to end: pinned host x -> device, one pass of row-split calls, y -> pinned host
        xh = torch.randn(R, K).bfloat16().pin_memory()
        yh = torch.empty(copies, R, N, dtype=torch.bfloat16).pin_memory()
        yd = [torch.empty(R, N, dtype=torch.bfloat16, device=dev) for _ in range(copies)]
        xd = torch.empty_like(x)
        copy_stream = torch.cuda.Stream()
        done = [torch.cuda.Event() for _ in range(copies)]

        def step():
            xd.copy_(xh, non_blocking=True)
            for i, w in enumerate(ws):
                yy = op(xd, w=w, out=yd[i])  # each call's y in its own buffer, read back while the next runs
                if rank == 0:
                    done[i].record()
                    with torch.cuda.stream(copy_stream):
                        copy_stream.wait_event(done[i])
                        yh[i].copy_(yy, non_blocking=True)
            if rank == 0:
                torch.cuda.current_stream().wait_stream(copy_stream)

        g2 = capture(step)
        ms2 = max_over_ranks(time_graph(g2, steps, warmup, world), world)
        del g2
        ms_step = ms2 / steps
        out["e2e"] = dict(value=total * copies / (ms_step * 1e-3) / 1e9, unit="GB/s", h2d_bytes_per_step=R * K * 2,
                          d2h_bytes_per_step=copies * R * N * 2, ms_per_step=ms_step,
                          note="x copied from pinned host memory on every rank; every y read back on rank 0")
    if nccl and R == 1 and N % world == 0:
        y_local = torch.empty(R, rows, dtype=torch.bfloat16, device=dev)
        y_all = torch.empty(world * R * rows, dtype=torch.bfloat16, device=dev)
        dist.all_gather_into_tensor(y_all, y_local.view(-1))  # warm the communicator outside capture
        torch.cuda.synchronize()

        def nccl_pass():
            for w in ws:
                ops.q8_0_gemv_into(x, w, y_local, R, rows, K)
                dist.all_gather_into_tensor(y_all, y_local.view(-1))

        try:
            g2 = capture(nccl_pass)
            ms2 = max_over_ranks(time_graph(g2, steps, warmup, world), world)
            del g2  # graphs holding NCCL calls are released before the process group
            out["nccl_us_per_call"] = ms2 * 1e3 / (steps * copies)
            out["nccl_gbs"] = total / (out["nccl_us_per_call"] * 1e-6) / 1e9
        except Exception as e:  # noqa: BLE001 -- the baseline is optional; report why it is missing
            out["nccl_error"] = f"{type(e).__name__}: {str(e)[:160]}"
    torch.cuda.synchronize()
    out["device_status"] = list(_lib.device_status())  # [status, site]: [0, 0] = every bounded wait ended in time
    op.close()
    del ws
    torch.cuda.empty_cache()
    return out


def bench_single_c4(R, steps, warmup, dev):
    """C4 R on this GPU alone (the 1-GPU point of the row-split curve, measured in the same run)."""
    r, st = bench_gemv("q8_0", R, 131072, 4096, steps, warmup, dev, target_step_ms=4.0)
    del st
    return r["us_per_call"]


def bench_moe_ep(R, steps, warmup, dev, world, rank):
    """C3 (MoeRouteGGUF -> MoeVerify iq2=3, E=128, I=1792, topk=6) with the experts split over the
    group: each call runs the router (replicated) and the expert-parallel MoeVerify (partial outputs
    summed through peer memory inside the finalize kernel).  Every rank builds the same 128 experts
    and keeps its share, rotated over distinct copies (> 2x L2 per GPU) so that every call streams its
    experts from HBM.  Before timing the output is compared with the single-GPU MoeVerify on all
    experts (rel-L2 <= 5e-3, max over ranks).  Time per call = max over ranks."""
    import torch
    import torch.distributed as dist

    from gguf_onnx_ops_b200 import _lib, ops
    from gguf_onnx_ops_b200.sharded import ExpertParallelMoE, shard_experts

    E, H, I, topk = 128, 1024, 1792, 6
    e0, el = shard_experts(E, world, rank)
    _lib.device_status()  # clear: the status reported below is this entry's own
    w1 = gen_weights("iq2_xxs", E * I, H, seed=2, dev=dev).reshape(E, I, -1)
    w2 = gen_weights("iq2_xxs", E * H, I, seed=3, dev=dev).reshape(E, H, -1)
    w1l, w2l = w1[e0:e0 + el].contiguous(), w2[e0:e0 + el].contiguous()
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    gw = torch.randn(E, H, generator=g, device=dev) * 0.02
    bias = torch.randn(E, generator=g, device=dev) * 0.01
    x, z = seeded_bf16((R, H), 200 + R, dev), seeded_bf16((R, H), 300 + R, dev)
    idx = torch.empty(R, topk, dtype=torch.int32, device=dev)
    wt = torch.empty(R, topk, dtype=torch.float32, device=dev)
    sc = torch.empty(R, E, dtype=torch.float32, device=dev)
    op = ExpertParallelMoE(w1l, w2l, e0, topk, r_max=8)
    out = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
    ops.moe_route_into(x, gw, bias, idx, wt, sc, R, H, E, topk, 1.0)
    op(z, idx, wt, out=out)
    ref = ops.MoeVerify(z, idx, wt, w1, None, w2, None, topk=topk)[0]
    torch.cuda.synchronize()
    err = torch.tensor([((out.float() - ref.float()).norm() / ref.float().norm()).item()], device=dev)
    dist.all_reduce(err, op=dist.ReduceOp.MAX)
    rel_err = float(err.item())
    U = len(torch.unique(idx))
    del w1, w2, ref
    copies = n_copies(w1l.numel() + w2l.numel())
    w1s, w2s = replicate(w1l, copies), replicate(w2l, copies)
    del w1l, w2l
    torch.cuda.empty_cache()

    def one_pass():
        for c in range(copies):
            ops.moe_route_into(x, gw, bias, idx, wt, sc, R, H, E, topk, 1.0)
            op(z, idx, wt, out=out, w1=w1s[c], w2=w2s[c])

    gr = capture(one_pass)
    ms = max_over_ranks(time_graph(gr, steps, warmup, world), world)
    del gr
    torch.cuda.synchronize()
    status = list(_lib.device_status())  # [status, site]: [0, 0] = every bounded wait ended in time
    op.close()
    del w1s, w2s
    torch.cuda.empty_cache()
    us = ms * 1e3 / (steps * copies)
    wbytes = E * H * 4 + E * 4 + U * (I * (H // 256) * 66 + H * (I // 256) * 66)
    return dict(world=world, R=R, us_per_call=us, gbs=wbytes / (us * 1e-6) / 1e9, unique_experts=U,
                experts_per_gpu=el, copies=copies, device_status=status,
                parity="ok" if rel_err <= 5e-3 else f"rel-L2 {rel_err:.2e} > 5e-3", rel_l2_vs_single_gpu=rel_err,
                note="router inside every call; expert copies rotated (> 2x L2 per GPU)")


def bench_embed(R, steps, warmup, dev, V=131072, K=4096):
    """Q8Embed gather of R token rows from a [V, K] Q8_0 table (C4's LM-head shape as the embedding).
    Algorithmic bytes per call: R x (row bytes read + bf16 row written + 8-byte id)."""
    import torch

    from gguf_onnx_ops_b200 import ops

    row_bytes = K // 32 * 34
    w = gen_weights("q8_0", V, K, seed=3, dev=dev)
    g = torch.Generator(device="cpu").manual_seed(R)
    copies = 8  # distinct id sets per pass so consecutive calls read different rows
    ids = [torch.randint(0, V, (R,), generator=g).to(dev) for _ in range(copies)]
    outs = [torch.empty(R, K, dtype=torch.bfloat16, device=dev) for _ in range(copies)]

    def one_pass():
        for i, o in zip(ids, outs):
            ops.q8_0_embed_into(w, i, o, V, row_bytes, R)

    gr = capture(one_pass)
    ms = time_graph(gr, steps, warmup)
    us = ms * 1e3 / (steps * copies)
    algo = R * (row_bytes + 2 * K + 8)
    del gr, w
    return {"us_per_call": round(us, 4), "gbs": round(algo / (us * 1e-6) / 1e9, 2), "algorithmic_bytes": algo,
            "table": f"[{V}, {row_bytes}] u8 (Q8_0, K={K})"}


def bench_norm(R, steps, warmup, dev, H=4096, skip=True):
    """SkipRmsNorm (sum written) or RmsNorm over [R, H] bf16; algorithmic bytes per call:
    R*H*2 x (x + skip + y + sum, or x + y) + 4H of gamma."""
    import torch

    from gguf_onnx_ops_b200 import ops

    copies = max(1, min(8, (256 << 20) // max(1, R * H * 2 * 4)))  # distinct buffers per pass
    xs = [torch.randn(R, H, device=dev).bfloat16() for _ in range(copies)]
    ss = [torch.randn(R, H, device=dev).bfloat16() for _ in range(copies)] if skip else [None] * copies
    ys = [torch.empty(R, H, dtype=torch.bfloat16, device=dev) for _ in range(copies)]
    sums = [torch.empty(R, H, dtype=torch.bfloat16, device=dev) for _ in range(copies)] if skip else [None] * copies
    gamma = torch.rand(H, device=dev) + 0.5

    def one_pass():
        for x, sk, y, su in zip(xs, ss, ys, sums):
            ops.rms_norm_into(x, sk, gamma, y, su, R, H, 1e-5)

    g = capture(one_pass)
    ms = time_graph(g, steps, warmup)
    us = ms * 1e3 / (steps * copies)
    algo = R * H * 2 * (4 if skip else 2) + 4 * H
    del g
    return {"us_per_call": round(us, 4), "gbs": round(algo / (us * 1e-6) / 1e9, 2), "algorithmic_bytes": algo,
            "op": "SkipRmsNorm (sum written)" if skip else "RmsNorm", "H": H}


def _time_rotating(make_call, copies, steps, warmup):
    """us per call of make_call(i) over `copies` distinct input sets, graph-replayed."""
    def one_pass():
        for i in range(copies):
            make_call(i)

    g = capture(one_pass)
    ms = time_graph(g, steps, warmup)
    del g
    return ms * 1e3 / (steps * copies)


def bench_legacy(layout, R, N, K, steps, warmup, dev):
    """Legacy split-layout GEMV (Q8Gemv gguf=0, Q4Gemv iq2=0/1/2, Nvfp4Gemv gguf=0); algorithmic bytes
    per call = weight bytes + scale bytes."""
    import torch

    from gguf_onnx_ops_b200 import _lib, ops

    wb = {_lib.GGUF_LAYOUT_Q8_SPLIT: K, _lib.GGUF_LAYOUT_IQ2_NATIVE: K // 4}.get(layout, K // 2)
    sb = {_lib.GGUF_LAYOUT_IQ2_NATIVE: K // 128, _lib.GGUF_LAYOUT_NVFP4_SPLIT: K // 16}.get(layout, K // 16)
    per = N * (wb + sb)
    copies = n_copies(per)
    gen = torch.Generator(device=dev)
    gen.manual_seed(layout)
    ws = [torch.randint(0, 256, (N, wb), generator=gen, device=dev, dtype=torch.uint8) for _ in range(copies)]
    if layout == _lib.GGUF_LAYOUT_NVFP4_SPLIT:
        ss = [torch.randint(0x30, 0x48, (N, sb), generator=gen, device=dev, dtype=torch.uint8) for _ in range(copies)]
    elif layout == _lib.GGUF_LAYOUT_IQ2_NATIVE:
        ss = [(torch.rand(N, sb // 2, generator=gen, device=dev) * 0.02 + 0.001).half().view(torch.uint8)
              for _ in range(copies)]
    else:
        ss = [(torch.rand(N, sb // 2, generator=gen, device=dev) * 0.02).bfloat16().view(torch.uint8)
              for _ in range(copies)]
    x = torch.randn(R, K, device=dev).bfloat16()
    y = torch.empty(R, N, dtype=torch.bfloat16, device=dev)
    gs = torch.tensor([0.37], device=dev)
    us = _time_rotating(lambda i: ops.gemv_legacy_into(layout, x, ws[i], ss[i], gs, y, R, N, K), copies, steps, warmup)
    return {"us_per_call": round(us, 3), "gbs": round(per / (us * 1e-6) / 1e9, 1), "algorithmic_bytes": per,
            "shape": f"R={R} N={N} K={K}"}


def bench_mamba(R, steps, warmup, dev, heads=128, ng=8, verify=False):
    """MambaStep (or MambaVerify over R tokens) at heads=128, n_groups=8 (di 8192, cd 10240); bytes per
    call = fp32 state read once + written once per output row + conv state, proj and outputs."""
    import torch

    from gguf_onnx_ops_b200 import ops

    di, cd = heads * 64, heads * 64 + 2 * ng * 128
    rows = R if verify else 1
    state = rows * heads * 128 * 64 * 4
    per = heads * 128 * 64 * 4 + state + R * (di + cd + heads) * 2 + 2 * rows * cd * 3 * 2 + R * (di * 2 + cd * 2 + di * 4)
    copies = n_copies(per)
    proj = torch.randn(R, di + cd + heads, device=dev).bfloat16()
    cs = [torch.randn(rows, cd, 3, device=dev).bfloat16() for _ in range(copies)]
    ss = [torch.randn(rows, heads, 128, 64, device=dev) * 0.1 for _ in range(copies)]
    cso = [torch.empty_like(c) for c in cs]
    sso = [torch.empty_like(t) for t in ss]
    cw = (torch.randn(cd, 4, device=dev) * 0.3).bfloat16()
    cb = (torch.randn(cd, device=dev) * 0.1).bfloat16()
    dtb, D = torch.randn(heads, device=dev) * 0.3, torch.randn(heads, device=dev)
    an = -torch.rand(heads, device=dev) * 4 - 0.1
    nw = torch.rand(di, device=dev) + 0.5
    y = torch.empty(R, di, dtype=torch.bfloat16, device=dev)
    xbc = torch.empty(R, cd, dtype=torch.bfloat16, device=dev)
    ypre = torch.empty(R, di, device=dev)
    row = torch.zeros(1, dtype=torch.int32, device=dev) if verify else None

    def call(i):
        ops.mamba_step_into(proj, cs[i], ss[i], cw, cb, dtb, an, D, nw, row, y, cso[i], sso[i], xbc, ypre, R=R,
                            state_rows=rows, heads=heads, n_groups=ng, eps=1e-5, tmin=0.001)

    us = _time_rotating(call, copies, steps, warmup)
    return {"us_per_call": round(us, 3), "gbs": round(per / (us * 1e-6) / 1e9, 1), "algorithmic_bytes": per,
            "op": "MambaVerify" if verify else "MambaStep"}


def bench_fused_norm_gemv(steps, warmup, dev, N=14336, K=4096):
    """Decode step of config 1 with its input norm: SkipRmsNorm then Q4Gemv iq2=3 (two launches, PDL
    chained) against the fused single launch; same rotating weight copies."""
    import torch

    from gguf_onnx_ops_b200 import ops

    wbytes = N * (K // 256) * 66
    copies = n_copies(wbytes)
    base = gen_weights("iq2_xxs", N, K, seed=1, dev=dev)
    ws = replicate(base, copies)
    del base
    x = torch.randn(1, K, device=dev).bfloat16()
    sk = torch.randn(1, K, device=dev).bfloat16()
    gamma = torch.rand(K, device=dev) + 0.5
    xn, sm = torch.empty_like(x), torch.empty_like(x)
    y = torch.empty(1, N, dtype=torch.bfloat16, device=dev)

    def chain(i):
        ops.rms_norm_into(x, sk, gamma, xn, sm, 1, K, 1e-5)
        ops.iq2_xxs_gemv_into(xn, ws[i], y, 1, N, K)

    def fused(i):
        ops.rms_norm_iq2_xxs_gemv_into(x, sk, gamma, 1e-5, ws[i], y, xn, sm, N, K)

    us_chain = _time_rotating(chain, copies, steps, warmup)
    us_fused = _time_rotating(fused, copies, steps, warmup)
    del ws
    return {"us_norm_then_gemv": round(us_chain, 3), "us_fused": round(us_fused, 3),
            "gbs_fused": round(wbytes / (us_fused * 1e-6) / 1e9, 1), "shape": f"R=1 N={N} K={K} (SkipRmsNorm + Q4Gemv iq2=3)"}


def bench_gguf_load(dev, rows=131072, K=4096, reps=3):
    """GGUF loader: a page-cache resident synthetic file holding one Q8_0 [rows, K] tensor (C4's LM
    head, 557 MB) copied into HBM by gguf_file_upload; GB/s = tensor bytes / wall time of the
    (host-synchronous) call, median of reps."""
    import tempfile

    import numpy as np
    import torch

    from gguf import GGMLQuantizationType as Q
    from gguf import GGUFWriter

    from gguf_onnx_ops_b200.gguf_file import GGUFFile

    row_bytes = K // 32 * 34
    tmpdir = "/dev/shm" if os.path.isdir("/dev/shm") else None
    with tempfile.TemporaryDirectory(dir=tmpdir) as d:
        path = os.path.join(d, "lm_head.gguf")
        data = np.random.default_rng(0).integers(0, 256, size=(rows, row_bytes), dtype=np.uint8)
        w = GGUFWriter(path, "bench")
        w.add_tensor("output.weight", data, raw_dtype=Q.Q8_0)
        w.write_header_to_file()
        w.write_kv_data_to_file()
        w.write_tensors_to_file()
        w.close()
        del data
        with GGUFFile(path) as f:
            out = torch.empty(rows, row_bytes, dtype=torch.uint8, device=dev)
            f.load("output.weight", out=out)  # warm-up: page cache, staging buffers
            times = []
            for _ in range(reps):
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                f.load("output.weight", out=out)
                times.append(time.perf_counter() - t0)
            nbytes = f["output.weight"].nbytes
            del out
    t = statistics.median(times)
    return {"gbs": round(nbytes / t / 1e9, 2), "ms": round(t * 1e3, 2), "bytes": nbytes,
            "source": "page-cache resident file (tmpfs when available)"}


def bench_e2e_gemv(op, R, N, K, steps, warmup, dev, state):
    """Public-API end to end: pinned host x -> device, one pass over the weight copies, every y -> pinned host
    (on a copy stream, overlapped with the next calls); the step ends when every y is on the host."""
    import torch

    ws, x, ys, gs, wbytes, copies = state
    xh = torch.randn(R, K).bfloat16().pin_memory()
    yh = torch.empty(copies, R, N, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty_like(x)
    # each call's y goes back to the host on a copy stream as soon as its GEMV ends, overlapping the
    # following GEMVs (the serving pattern: outputs stream out while the next op computes)
    copy_stream = torch.cuda.Stream()
    done = [torch.cuda.Event() for _ in range(copies)]

    def step():
        xd.copy_(xh, non_blocking=True)
        for i, (w, y) in enumerate(zip(ws, ys)):
            gemv_call(op, xd, w, y, gs, R, N, K)
            done[i].record()
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(done[i])
                yh[i].copy_(y, non_blocking=True)
        torch.cuda.current_stream().wait_stream(copy_stream)

    g = capture(step)
    ms = time_graph(g, steps, warmup)
    ms_step = ms / steps
    return dict(value=wbytes * copies / (ms_step * 1e-3) / 1e9, unit="GB/s", h2d_bytes_per_step=R * K * 2,
                d2h_bytes_per_step=copies * R * N * 2, ms_per_step=ms_step)


def bench_moe(R, steps, warmup, dev):
    """Config C3: MoeRouteGGUF -> MoeVerify iq2=3 (E=128, I=1792, topk=6) over distinct expert copies."""
    import torch

    from gguf_onnx_ops_b200 import ops

    E, H, I, topk = 128, 1024, 1792, 6
    w1 = gen_weights("iq2_xxs", E * I, H, seed=2, dev=dev).reshape(E, I, -1)
    w2 = gen_weights("iq2_xxs", E * H, I, seed=3, dev=dev).reshape(E, H, -1)
    per_copy = w1.numel() + w2.numel() + E * H * 4
    copies = n_copies(per_copy)
    w1s, w2s = replicate(w1, copies), replicate(w2, copies)
    gwt = (torch.randn(E, H, device=dev) * 0.02)
    gws = replicate(gwt, copies)
    bias = torch.randn(E, device=dev) * 0.01
    x = torch.randn(R, H, device=dev).bfloat16()
    z = torch.randn(R, H, device=dev).bfloat16()
    P = R * topk
    idx = [torch.empty(R, topk, dtype=torch.int32, device=dev) for _ in range(copies)]
    wt = [torch.empty(R, topk, dtype=torch.float32, device=dev) for _ in range(copies)]
    sc = torch.empty(R, E, dtype=torch.float32, device=dev)
    out = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
    h = torch.empty(P, I, dtype=torch.bfloat16, device=dev)
    part = torch.empty(P, H, dtype=torch.float32, device=dev)
    meta = torch.empty(1 + 9 * P, dtype=torch.int32, device=dev)

    def one_pass():
        for c in range(copies):
            ops.moe_route_into(x, gws[c], bias, idx[c], wt[c], sc, R, H, E, topk, 1.0)
            ops.moe_verify_into(z, idx[c], wt[c], w1s[c], w2s[c], out, h, part, meta, R, E, I, topk)

    g1 = capture(one_pass)
    ms1 = time_graph(g1, 5, 2) / 5
    rounds = max(1, int(round(8.0 / max(ms1, 1e-3))))

    def step():
        for _ in range(rounds):
            one_pass()

    g = capture(step) if rounds > 1 else g1
    ms = time_graph(g, steps, warmup)
    U = len(torch.unique(idx[0]))
    bytes_call = E * H * 4 + U * (I * (H // 256) * 66 + H * (I // 256) * 66)
    calls = steps * rounds * copies
    us = ms * 1e3 / calls
    return dict(us_per_call=us, gbs=bytes_call / (us * 1e-6) / 1e9, weight_bytes=bytes_call, unique_experts=U,
                copies=copies, rounds=rounds, kernels_per_call=4)


# ------------------------------------------------------------------------------------------------
# CPU baseline: the reference's CPU path (gguf-py dequantise + fp32 matmul), oracle port
# ------------------------------------------------------------------------------------------------
def cpu_baseline(op, R, N, K, budget_s=10.0):
    import concurrent.futures as cf

    import torch

    import oracle as O
    from oracle import inputs as I

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    deq = {"q8_0": O.dequant_q8_0, "iq2_xxs": O.dequant_iq2_xxs, "nvfp4": O.dequant_nvfp4}[op]
    g = I.rng(0)
    x = I.bf16_normal(g, (R, K))
    xf = torch.from_numpy((x.astype(np.uint32) << 16).view(np.float32))
    chunk = 256

    def make(rows):
        if op == "q8_0":
            return I.q8_0_weights(g, rows, K)
        if op == "iq2_xxs":
            return I.iq2_xxs_weights(g, (rows,), K)
        return I.nvfp4_weights(g, rows, K)

    pool = cf.ThreadPoolExecutor(max_workers=cores)

    def run(w):
        parts = list(pool.map(deq, [w[i:i + chunk] for i in range(0, w.shape[0], chunk)]))
        d = torch.from_numpy(np.concatenate(parts))
        return xf @ d.T

    w = make(chunk * cores)
    t0 = time.perf_counter()
    run(w)
    t1 = time.perf_counter() - t0
    rows = int(min(N, max(chunk, chunk * cores * budget_s / max(t1, 1e-3) / 4)))
    rows = max(chunk, rows // chunk * chunk)
    w = make(rows)
    t0 = time.perf_counter()
    run(w)
    dt = time.perf_counter() - t0
    # second figure: the matmul alone on the pre-dequantised fp32 weights
    d = torch.from_numpy(np.concatenate(list(pool.map(deq, [w[i:i + chunk] for i in range(0, rows, chunk)]))))
    t0 = time.perf_counter()
    _ = xf @ d.T
    dt_mm = time.perf_counter() - t0
    pool.shutdown()
    bytes_ = rows * ROW_BYTES[op](K)
    return dict(value=bytes_ / dt / 1e9, unit="GB/s", cores=cores, kind="port",
                sample=f"{rows} of {N} rows, R={R}, K={K}: numpy dequantise ({cores} threads) + torch fp32 matmul",
                seconds=dt, matmul_only_gbs=bytes_ / dt_mm / 1e9,
                matmul_only_note="torch fp32 x @ W^T on pre-dequantised W, GB/s of the GGUF bytes those rows hold")


# ------------------------------------------------------------------------------------------------
def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, "fallback"


def traffic_per_launch():
    try:
        with open(os.path.join(ROOT, "profiles", "dram_traffic.json")) as f:
            t = json.load(f)
        return t.get("C1_R1", {}).get("dram_bytes_per_launch")
    except Exception:  # noqa: BLE001
        return None


def main():
    args = parse_args()
    if args.cpu_table:
        cpu_table()
        return
    if args.profile_case:
        import gguf_onnx_ops_b200

        gguf_onnx_ops_b200.load()
        profile_case(args)
        return
    import torch

    hd = HEADLINE
    if args.impl == "reference":  # host CPU only; under torchrun rank 0 alone runs and prints
        rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", args.gpus))
    else:
        rank, world, local = dist_setup(args.gpus)
    metric = "weight-stream HBM GB/s per GEMV/MoE op call"
    config = {"workload": "BASELINE config 1: Q4Gemv iq2=3 (IQ2_XXS) R=1 K=4096 N=14336",
              "parallelism": "single", "global_batch": hd["R"],
              "l2": "distinct weight copies per pass, total > 2x L2 (126 MB)"}

    if args.impl == "reference":
        if rank != 0:
            return
        # the reference's CPU path on this arm's workload: config 1 at N = 1, config 4's LM head (the
        # sharded headline of the multi-GPU line) at N > 1
        op, R, N, K = (hd["op"], hd["R"], hd["N"], hd["K"]) if world == 1 else ("q8_0", 1, 131072, 4096)
        if world > 1:
            config = {"workload": "BASELINE config 4: Q8Gemv gguf=1 R=1 K=4096 N=131072 (LM head)",
                      "parallelism": "host CPU", "global_batch": 1}
        runs = []
        for i in range(args.warmup + args.steps):
            cb = cpu_baseline(op, R, N, K, budget_s=max(1.0, 120.0 / (args.warmup + args.steps)))
            if i >= args.warmup:
                runs.append(cb)
        v = statistics.median(r["value"] for r in runs)
        line = {"impl": "reference", "metric": metric, "value": v, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": statistics.median(r["seconds"] for r in runs) * 1e3,
                "higher_is_better": True, "scaling": "weak" if world == 1 else "strong", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic", "config": config,
                "cpu_baseline": {"value": v, "unit": "GB/s", "cores": runs[0]["cores"], "kind": "port",
                                 "sample": runs[0]["sample"]},
                "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    dev = torch.device("cuda", torch.cuda.current_device())
    import gguf_onnx_ops_b200

    gguf_onnx_ops_b200.load()
    if world > 1:
        sharded_main(args, rank, world, local, dev, metric)
        return
    sampler = ClockSampler(local)
    res, state = bench_gemv(hd["op"], hd["R"], hd["N"], hd["K"], args.steps, args.warmup, dev, world=world,
                            sampler=sampler)
    value = res["gbs"] * world
    peak, src = peaks()
    line = {"metric": metric, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": config,
            "us_per_call": res["us_per_call"],
            "roofline": {"bound": "hbm", "achieved": res["gbs"], "peak": peak, "unit": "GB/s",
                         "frac": res["gbs"] / peak, "traffic": traffic_per_launch(), "peak_source": src,
                         "algorithmic_bytes_per_launch": res["weight_bytes"]},
            "gpu_launches": res["calls"], "clocks": sampler.report()}
    line["e2e"] = bench_e2e_gemv(hd["op"], hd["R"], hd["N"], hd["K"], args.steps, args.warmup, dev, state)
    del state
    torch.cuda.empty_cache()
    line["cpu_baseline"] = cpu_baseline(hd["op"], hd["R"], hd["N"], hd["K"])
    if not args.quick:
        cfgs = {}
        for name, op, R, N, K in ([("C0", "q8_0", 1, 4096, 4096)] +
                                  [("C1", "iq2_xxs", R, 14336, 4096) for R in (1, 4, 8)] +
                                  [("C2", "nvfp4", R, 13824, 5120) for R in (1, 8, 16)] +
                                  [("C4", "q8_0", R, 131072, 4096) for R in (1, 4, 8, 16)]):
            r, st = bench_gemv(op, R, N, K, max(5, args.steps // 2), args.warmup, dev)
            del st
            torch.cuda.empty_cache()
            cfgs[f"{name}_R{R}"] = {k: round(v, 4) if isinstance(v, float) else v for k, v in r.items()
                                    if k in ("us_per_call", "gbs", "weight_bytes", "copies", "rounds")}
            cfgs[f"{name}_R{R}"]["frac_of_peak"] = round(r["gbs"] / peak, 4)
        for R in (1, 4, 8):
            r = bench_moe(R, max(5, args.steps // 2), args.warmup, dev)
            r["frac_of_peak"] = r["gbs"] / peak
            cfgs[f"C3_R{R}"] = {k: round(v, 4) if isinstance(v, float) else v for k, v in r.items()}
            torch.cuda.empty_cache()
        line["configs"] = cfgs
        line["next_rows"] = next_rows(args, dev)
    print(json.dumps(line), flush=True)


def next_rows(args, dev):
    """The ops either side of the GEMVs and the legacy layouts, one GPU."""
    import torch

    from gguf_onnx_ops_b200 import _lib as L

    st2 = max(5, args.steps // 2)
    out = {f"Q8Embed_R{R}": bench_embed(R, st2, args.warmup, dev) for R in (1, 8, 4096)}
    torch.cuda.empty_cache()
    for R in (1, 8, 4096):
        out[f"SkipRmsNorm_R{R}"] = bench_norm(R, st2, args.warmup, dev)
    out["RmsNorm_R1"] = bench_norm(1, st2, args.warmup, dev, skip=False)
    torch.cuda.empty_cache()
    out["GGUF_load_C4_lm_head"] = bench_gguf_load(dev)
    for name, layout, R, N, K in (("Q8Gemv_gguf0", L.GGUF_LAYOUT_Q8_SPLIT, 1, 4096, 4096),
                                  ("Q4Gemv_iq2_0", L.GGUF_LAYOUT_Q4_SPLIT, 1, 14336, 4096),
                                  ("Q4Gemv_iq2_1", L.GGUF_LAYOUT_IQ2_CODES, 8, 14336, 4096),
                                  ("Q4Gemv_iq2_2", L.GGUF_LAYOUT_IQ2_NATIVE, 1, 14336, 4096),
                                  ("Nvfp4Gemv_gguf0", L.GGUF_LAYOUT_NVFP4_SPLIT, 1, 13824, 5120)):
        out[f"{name}_R{R}"] = bench_legacy(layout, R, N, K, st2, args.warmup, dev)
        torch.cuda.empty_cache()
    out["SkipRmsNorm_Q4Gemv_C1_R1"] = bench_fused_norm_gemv(st2, args.warmup, dev)
    torch.cuda.empty_cache()
    out["MambaStep_R1"] = bench_mamba(1, st2, args.warmup, dev)
    out["MambaVerify_R8"] = bench_mamba(8, st2, args.warmup, dev, verify=True)
    torch.cuda.empty_cache()
    return out


def sharded_main(args, rank, world, local, dev, metric):
    """N > 1: the headline is the sharded config -- C4's LM head (Q8Gemv gguf=1, R = 1, K = 4096,
    N = 131072) row-split over the N GPUs with the all-gather fused into the GEMV.
    value = the whole weight tensor's bytes / the max-over-ranks time per call (strong scaling: the
    total work is fixed).  The line also carries the same workload on one GPU (measured in this run),
    C4 at R = 4, 8, 16, the GEMV + NCCL all-gather baseline, the expert-parallel C3 MoE, and config 1
    as independent replicas; every sharded entry carries its parity check against the single-GPU op."""
    import torch
    import torch.distributed as dist

    peak, src = peaks()
    st2 = max(5, args.steps // 2)
    sampler = ClockSampler(local)
    one_gpu_us = bench_single_c4(1, st2, args.warmup, dev)  # every rank on its own GPU; rank 0's figure
    torch.cuda.empty_cache()
    barrier(world)
    r1 = bench_rowsplit(1, args.steps, args.warmup, dev, world, rank, nccl=True, e2e=True, sampler=sampler)
    total = 131072 * ROW_BYTES["q8_0"](4096)
    sharded = {"C4_R1": {k: v for k, v in r1.items() if k != "e2e"}}
    for R in (4, 8, 16):
        sharded[f"C4_R{R}"] = bench_rowsplit(R, st2, args.warmup, dev, world, rank)
    for R in (1, 4, 8):
        sharded[f"C3_R{R}_expert_parallel"] = bench_moe_ep(R, st2, args.warmup, dev, world, rank)
    rep, st = bench_gemv(HEADLINE["op"], 1, HEADLINE["N"], HEADLINE["K"], st2, args.warmup, dev, world=world)
    del st
    torch.cuda.empty_cache()
    per_gpu_bytes = r1["rows_per_gpu"] * ROW_BYTES["q8_0"](4096)
    gbs_per_gpu = per_gpu_bytes / (r1["fused_us_per_call"] * 1e-6) / 1e9
    line = {"metric": metric, "value": r1["fused_gbs"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r1["ms_total"] / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE config 4: Q8Gemv gguf=1 R=1 K=4096 N=131072 (LM head), row-split "
                                   f"over {world} GPUs, all-gather of y fused into the GEMV (NVLink peer stores)",
                       "parallelism": f"rowsplit{world}", "global_batch": 1,
                       "l2": "distinct weight-shard copies per pass, > 2x L2 per GPU"},
            "us_per_call": r1["fused_us_per_call"],
            "one_gpu_same_workload": {"us_per_call": one_gpu_us, "gbs": total / (one_gpu_us * 1e-6) / 1e9,
                                      "note": "C4 R=1 on one GPU (rank 0's GPU), measured in this run"},
            "parity": r1["parity"],
            "roofline": {"bound": "hbm", "achieved": gbs_per_gpu, "peak": peak, "unit": "GB/s",
                         "frac": gbs_per_gpu / peak, "traffic": None, "peak_source": src,
                         "algorithmic_bytes_per_launch": per_gpu_bytes,
                         "note": "per GPU: its shard's bytes / the call time (peer stores and completion included)"},
            "gpu_launches": r1["calls"], "clocks": sampler.report(), "e2e": r1.get("e2e"),
            "sharded": sharded,
            "replicas_C1": {"value": rep["gbs"] * world, "unit": "GB/s", "us_per_call": rep["us_per_call"],
                            "note": "config 1 (does not shard) as independent replicas, aggregate, max over ranks"}}
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
