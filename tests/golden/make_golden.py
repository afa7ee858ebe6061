"""Generate the committed golden fixtures in tests/golden/ (run in the build container only).

Every expected value here comes from the reference's own CPU path, not from the repo's oracle:

* dequantised weights: ``gguf.quants.dequantize`` of gguf-py 0.19.0, the call the reference's test
  harness makes (tests/test_bolt_ops.py:225-230);
* GEMV outputs: that dequantisation followed by a torch fp32 ``x.float() @ deq.T``
  (tests/test_bolt_ops.py:237-238);
* MoE outputs: the reference harness's per-(row, expert) loop (tests/test_bolt_ops.py:253-259) on
  gguf-py dequantised experts (kept in fp32: the repo's kernels consume the exact weights);
* router outputs: the harness's torch router (tests/test_bolt_ops.py:116-119) on bf16-rounded gate
  weights, as MoeRouteGGUF specifies (src/bolt_ops.cu:441-448);
* Q8Embed output: the harness's torch expression (tests/test_bolt_ops.py:310-311) with ids outside
  [0, vocab) replaced by row 0, the op's rule (src/bolt_ops.cu:1680);
* RmsNorm / SkipRmsNorm outputs: the harness's torch expressions (tests/test_bolt_ops.py:321-337);
* MambaStep outputs: the harness's torch reference loop (tests/test_bolt_ops.py:389-413) at heads=4;
* the IQ2_XXS codebook: parsed from the reference's src/iq2xxs_grid.h (kIq2xxsGrid, line 6, and
  kIq2xxsGridBf16, line 75).

Inputs use the reference test builders (iq2_native_blocks, the Q8 block builder, the NVFP4 block
builder of tests/test_bolt_ops.py:210-215, :290-294, :274-275) with numpy RNG, plus the BASELINE
config distributions at reduced sizes.

    python tests/golden/make_golden.py --reference <reference checkout> [--only embed|norm|mamba]
"""

from __future__ import annotations

import argparse
import hashlib
import os
import re
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import inputs as I  # noqa: E402  (input builders only; expected values come from gguf/torch)
from tests.golden.cases import (GEMV_CASES, embed_inputs, mamba_inputs, moe_inputs, norm_inputs,  # noqa: E402
                                route_inputs, sha)


def gguf_deq(raw: np.ndarray, qt) -> np.ndarray:
    from gguf import quants

    return np.asarray(quants.dequantize(np.ascontiguousarray(raw), qt), dtype=np.float32).reshape(raw.shape[0], -1)


def bf16_tensor(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)


def parse_reference_grid(ref: str):
    src = open(os.path.join(ref, "src", "iq2xxs_grid.h")).read()
    u64 = re.search(r"kIq2xxsGrid\[256\]\s*=\s*\{(.*?)\};", src, re.S).group(1)
    grid64 = np.array([int(v, 16) for v in re.findall(r"0x([0-9a-fA-F]+)", u64)], dtype=np.uint64)
    b16 = re.search(r"kIq2xxsGridBf16\[256\]\[4\]\s*=\s*\{(.*)\};", src, re.S).group(1)
    gridbf = np.array([int(v, 16) for v in re.findall(r"0x([0-9a-fA-F]+)u", b16)], dtype=np.uint32).reshape(256, 4)
    assert grid64.size == 256
    return grid64, gridbf


def make_embed():
    blk, ids = embed_inputs()
    V = blk.shape[0]
    nb = blk.shape[1] // 34
    t = torch.from_numpy(blk).reshape(V, nb, 34)
    d = t[:, :, :2].contiguous().view(torch.float16).reshape(V, nb)
    table = (d.float().unsqueeze(-1) * t[:, :, 2:].contiguous().view(torch.int8).float()).reshape(V, -1).bfloat16()
    tid = torch.from_numpy(ids)
    tid = torch.where((tid >= 0) & (tid < V), tid, torch.zeros_like(tid))
    out = table[tid]
    np.savez_compressed(os.path.join(HERE, "embed.npz"), out_bf16=out.view(torch.int16).numpy().view(np.uint16),
                        sha=np.array(sha(blk, ids)))


def make_norm():
    cases = {}
    for name in ("h4096", "h2048"):
        x, skip, gamma, eps = norm_inputs(name)
        xt, st, gt = bf16_tensor(x), bf16_tensor(skip), torch.from_numpy(gamma)
        rn = (xt.float() * torch.rsqrt(xt.float().pow(2).mean(-1, keepdim=True) + eps) * gt.bfloat16().float()).bfloat16()
        s = xt + st
        srn = (s.float() * torch.rsqrt(s.float().pow(2).mean(-1, keepdim=True) + eps) * gt.bfloat16().float()).bfloat16()
        cases.update({f"{name}_rms": rn.view(torch.int16).numpy().view(np.uint16),
                      f"{name}_skip_rms": srn.view(torch.int16).numpy().view(np.uint16),
                      f"{name}_sum": s.view(torch.int16).numpy().view(np.uint16),
                      f"{name}_sha": np.array(sha(x, skip, gamma))})
    np.savez_compressed(os.path.join(HERE, "norm.npz"), **cases)


def make_mamba():
    m = mamba_inputs()
    heads, ng, hd, ds = m["heads"], m["n_groups"], 64, 128
    di = heads * hd
    cd = di + 2 * ng * ds
    R = m["proj"].shape[0]
    proj = bf16_tensor(m["proj"])
    cst = bf16_tensor(m["cst"])
    sst = torch.from_numpy(m["sst"])
    cw = torch.from_numpy(m["cw"]).reshape(cd, 1, 4).bfloat16()
    cb = torch.from_numpy(m["cb"]).bfloat16()
    dtb, an, D, nw = (torch.from_numpy(m[k]) for k in ("dtb", "an", "D", "nw"))
    gate, xbc, dt = proj.split([di, cd, heads], -1)
    inp = torch.cat([cst[0].T.float(), xbc.float()], 0)
    conv = torch.zeros(R, cd)
    for r in range(R):
        win = inp[r:r + 4]
        conv[r] = torch.nn.functional.silu((win * cw[:, 0, :].T.float()).sum(0) + cb.float())
    conv = conv.bfloat16().float()
    xs, Bm, Cm = conv.split([di, ng * ds, ng * ds], -1)
    st = sst[0].clone()
    ys = []
    for r in range(R):
        dts = torch.clamp(torch.nn.functional.softplus(dt[r].float() + dtb), min=m["tmin"])
        dA = torch.exp(an * dts)
        xh = xs[r].reshape(heads, hd)
        Bh = Bm[r].reshape(ng, ds).repeat_interleave(heads // ng, 0)
        Ch = Cm[r].reshape(ng, ds).repeat_interleave(heads // ng, 0)
        st = st * dA[:, None, None] + (dts[:, None] * xh)[:, None, :] * Bh[:, :, None]
        ys.append((st * Ch[:, :, None]).sum(1) + D[:, None] * xh)
    yp = torch.stack(ys).reshape(R, di)
    g = (yp * torch.nn.functional.silu(gate.float())).reshape(R, ng, di // ng)
    g = g * torch.rsqrt(g.pow(2).mean(-1, keepdim=True) + m["eps"])
    y = g.reshape(R, di) * nw
    np.savez_compressed(os.path.join(HERE, "mamba.npz"), y=y.numpy(), ssm=st.numpy(),
                        conv=inp[-3:].T.contiguous().bfloat16().view(torch.int16).numpy().view(np.uint16),
                        sha=np.array(sha(*(m[k] for k in ("proj", "cst", "sst", "cw", "cb", "dtb", "an", "D", "nw")))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("GGUF_REFERENCE_DIR", ""),
                    help="checkout of the reference (its src/iq2xxs_grid.h is parsed for the codebook fixture)")
    ap.add_argument("--only", choices=["embed", "norm", "mamba"], default=None)
    args = ap.parse_args()
    if args.only:
        {"embed": make_embed, "norm": make_norm, "mamba": make_mamba}[args.only]()
        return
    from gguf import GGMLQuantizationType as Q

    # 1. IQ2_XXS codebook of the reference
    if not args.reference:
        ap.error("--reference (or GGUF_REFERENCE_DIR) must name the reference checkout")
    g64, gbf = parse_reference_grid(args.reference)
    np.savez_compressed(os.path.join(HERE, "iq2xxs_grid.npz"), grid_u64=g64, grid_bf16x2=gbf)

    # 2. dequantisation goldens (reference test builders)
    g = I.rng(1001)
    q8 = I.q8_test_blocks(g, 24, 1024)
    iq2 = I.iq2_test_blocks(g, (24,), 1024)
    fp4 = g.integers(0, 256, size=(24, 1024 // 64, 36), dtype=np.uint8)
    fp4[:, :, :4] = g.integers(0x30, 0x48, size=(24, 1024 // 64, 4), dtype=np.uint8)  # tests/test_bolt_ops.py:275
    fp4 = fp4.reshape(24, -1)
    fp4_all = np.zeros((4, 1024 // 64, 36), dtype=np.uint8)  # every scale byte 0..255, every nibble
    fp4_all[:, :, 4:] = g.integers(0, 256, size=(4, 1024 // 64, 32), dtype=np.uint8)
    fp4_all[:, :, :4] = np.arange(256, dtype=np.uint8).reshape(4, 16, 4)
    fp4_all = fp4_all.reshape(4, -1)
    np.savez_compressed(
        os.path.join(HERE, "dequant.npz"),
        q8_raw=q8, q8_deq=gguf_deq(q8, Q.Q8_0),
        iq2_raw=iq2, iq2_deq=gguf_deq(iq2, Q.IQ2_XXS),
        fp4_raw=fp4, fp4_deq=gguf_deq(fp4, Q.NVFP4),
        fp4all_raw=fp4_all, fp4all_deq=gguf_deq(fp4_all, Q.NVFP4),
    )

    # 3. GEMV goldens: x @ gguf_deq(W)^T in torch fp32 (the harness's CPU reference)
    cases = {}
    qts = {"q8_0": Q.Q8_0, "iq2_xxs": Q.IQ2_XXS, "nvfp4": Q.NVFP4}
    for name, (op, R, N, K, seed) in GEMV_CASES.items():
        x, w, extra = I.gemv_case(op, R, N, K, seed=seed)
        deq = torch.from_numpy(gguf_deq(w, qts[op]))
        y = (bf16_tensor(x).float() @ deq.T)
        if op == "nvfp4":
            y = y * float(extra["gscale"][0])
        cases[f"{name}_x"] = x
        cases[f"{name}_w"] = w
        cases[f"{name}_y"] = y.numpy()
    np.savez_compressed(os.path.join(HERE, "gemv.npz"), **cases)

    # 4. router goldens: config C3 shape, and the harness's E=240 topk=9 scale=5 (K reduced to 1024)
    rcases = {}
    for name in ("c3", "harness"):
        x, gw, b, topk, scale = route_inputs(name)
        sc = (bf16_tensor(x).float() @ torch.from_numpy(gw).bfloat16().float().T).sigmoid()
        ridx = torch.topk(sc + torch.from_numpy(b), topk, dim=-1)[1]
        rw = sc.gather(1, ridx)
        rw = rw / (rw.sum(-1, keepdim=True) + 1e-20) * scale
        rcases.update({f"{name}_idx": ridx.numpy().astype(np.int32), f"{name}_w": rw.numpy(),
                       f"{name}_scores": sc.numpy(), f"{name}_sha": np.array(sha(x, gw, b))})
    np.savez_compressed(os.path.join(HERE, "route.npz"), **rcases)

    # 5. MoE golden: the harness loop (tests/test_bolt_ops.py:253-259) on gguf-py dequantised experts
    z, idx, wts, b1, b2, (R, E, H, Idim, topk) = moe_inputs()
    d1 = torch.from_numpy(gguf_deq(b1.reshape(E * Idim, -1), Q.IQ2_XXS).reshape(E, Idim, H))
    d2 = torch.from_numpy(gguf_deq(b2.reshape(E * H, -1), Q.IQ2_XXS).reshape(E, H, Idim))
    zt = bf16_tensor(z)
    ref = torch.zeros(R, H)
    for t in range(R):
        for j in range(topk):
            e = int(idx[t, j])
            h = (zt[t].float() @ d1[e].T).bfloat16().float()
            h = (torch.relu(h) ** 2).bfloat16().float()
            ref[t] += float(wts[t, j]) * (h @ d2[e].T).bfloat16().float()
    np.savez_compressed(os.path.join(HERE, "moe.npz"), out=ref.numpy(), sha=np.array(sha(z, idx, wts, b1, b2)))
    make_embed()
    make_norm()
    make_mamba()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
