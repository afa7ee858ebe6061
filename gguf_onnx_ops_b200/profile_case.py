"""Run one hot-path op a few times on cuda:0 (eager launches) -- the target for Nsight Compute.

    python -m gguf_onnx_ops_b200.profile_case --op iq2_xxs --R 1 --N 14336 --K 4096 --iters 3
    python -m gguf_onnx_ops_b200.profile_case --op moe --R 1 --iters 3

Weights use the BASELINE distributions (device-generated); each iteration uses a distinct weight
copy when `--copies` > 1 so that repeated launches stream from HBM rather than L2.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="iq2_xxs", choices=["q8_0", "iq2_xxs", "nvfp4", "moe", "route"])
    ap.add_argument("--R", type=int, default=1)
    ap.add_argument("--N", type=int, default=14336)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--copies", type=int, default=3)
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--fast-mode", type=int, default=1, help="gguf_set_fast_paths value (0 = generic engine)")
    a = ap.parse_args()

    import bench  # device weight generators with the BASELINE distributions
    from gguf_onnx_ops_b200 import ops

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    ops.set_pdl(not a.no_pdl)
    ops.set_fast_paths(a.fast_mode)
    if a.op in ("moe", "route"):
        E, H, I, topk = 128, 1024, 1792, 6
        w1 = bench.gen_weights("iq2_xxs", E * I, H, seed=2, dev=dev).reshape(E, I, -1)
        w2 = bench.gen_weights("iq2_xxs", E * H, I, seed=3, dev=dev).reshape(E, H, -1)
        gw = torch.randn(E, H, device=dev) * 0.02
        bias = torch.randn(E, device=dev) * 0.01
        x = torch.randn(a.R, H, device=dev).bfloat16()
        z = torch.randn(a.R, H, device=dev).bfloat16()
        for _ in range(a.iters):
            idx, wt, _ = ops.MoeRouteGGUF(x, gw, bias, topk, 1.0)
            if a.op == "moe":
                ops.MoeVerify(z, idx, wt, w1, None, w2, None, topk=topk)
    else:
        base = bench.gen_weights(a.op, a.N, a.K, seed=1, dev=dev)
        ws = bench.replicate(base, a.copies)
        x = torch.randn(a.R, a.K, device=dev).bfloat16()
        gs = torch.tensor([1.0 / 448.0], device=dev)
        y = torch.empty(a.R, a.N, dtype=torch.bfloat16, device=dev)
        for i in range(a.iters):
            bench.gemv_call(a.op, x, ws[i % len(ws)], y, gs, a.R, a.N, a.K)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main()
