"""Run one hot-path op a few times on cuda:0 (eager launches) -- the target for Nsight Compute.

    python -m gguf_onnx_ops_b200.profile_case --op iq2_xxs --R 1 --N 14336 --K 4096 --iters 3
    python -m gguf_onnx_ops_b200.profile_case --op moe --R 1 --iters 3
    python -m gguf_onnx_ops_b200.profile_case --op embed --R 4096 --N 131072 --K 4096
    python -m gguf_onnx_ops_b200.profile_case --op norm --R 4096 --K 4096
    python -m gguf_onnx_ops_b200.profile_case --op q4_split --R 1 --N 14336 --K 4096
    python -m gguf_onnx_ops_b200.profile_case --op mamba --R 1

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
    ap.add_argument("--op", default="iq2_xxs",
                    choices=["q8_0", "iq2_xxs", "nvfp4", "moe", "route", "embed", "norm", "q4_split", "mamba"])
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
    if a.op == "embed":  # Q8Embed: R ids from a [N, K] Q8_0 table
        table = bench.gen_weights("q8_0", a.N, a.K, seed=4, dev=dev)
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
