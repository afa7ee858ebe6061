"""Worker for tests/test_gpu_dist.py: one process per GPU (launched by torch.distributed.run).

Every rank builds the same seeded weights, keeps its row shard, and checks the row-split GEMV with
the fused peer-store all-gather against the single-GPU op on the full matrix, over several calls
(both output buffers): bit-identical where both run the same kernel (Q8_0), within 2e-3 rel-L2
where the single-GPU op has a specialised kernel the shard does not use."""

import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from gguf_onnx_ops_b200 import _lib, ops  # noqa: E402
from gguf_onnx_ops_b200.sharded import RowSplitGemv, shard_rows  # noqa: E402
from oracle import inputs as I  # noqa: E402

I_ = I

TYPES = {"q8_0": _lib.GGUF_TYPE_Q8_0, "iq2_xxs": _lib.GGUF_TYPE_IQ2_XXS, "nvfp4": _lib.GGUF_TYPE_NVFP4}


def single(op, x, w, gs):
    if op == "q8_0":
        return ops.Q8Gemv(x, w)
    if op == "iq2_xxs":
        return ops.Q4Gemv(x, w)
    return ops.Nvfp4Gemv(x, w, None, gs)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    dev = torch.device("cuda", rank)
    failures = []
    for op, N, K, Rs in (("q8_0", 8192, 4096, (1, 4, 16)), ("iq2_xxs", 4096, 4096, (1, 8)), ("nvfp4", 2048, 5120, (1, 3)),
                         ("q8_0", 1000, 1024, (2,))):
        _, w, extra = I.gemv_case(op, 1, N, K, seed=N + K)
        wt = torch.from_numpy(w).to(dev)
        gs = torch.from_numpy(extra.get("gscale", np.array([1.0 / 448.0], np.float32))).to(dev)
        row0, rows = shard_rows(N, world, rank)
        sharded = RowSplitGemv(TYPES[op], wt[row0:row0 + rows], N, row0, K, r_max=16, gscale=gs)
        for R in Rs:
            for it in range(3):
                x = torch.from_numpy(I.bf16_normal(I.rng(100 * R + it), (R, K)).view(np.int16)).view(torch.bfloat16).to(dev)
                y = sharded(x)
                ref = single(op, x, wt, gs)
                torch.cuda.synchronize()
                if op == "q8_0":  # the shard runs the single-GPU op's kernel on its rows: bit-identical
                    ok = torch.equal(y, ref)
                else:  # IQ2_XXS / NVFP4: the single-GPU op takes the integer or few-row kernels, the shard
                    # the bf16 slice kernel or the engine (same exact weights, another summation order)
                    err = ((y.float() - ref.float()).norm() / ref.float().norm()).item()
                    ok = err < 2e-3
                if not ok:
                    failures.append((op, N, K, R, it))
        sharded.close()
    # expert-parallel MoeVerify against the single-GPU op on all experts
    E, H, Iw, topk = 16, 1024, 512, 6
    from gguf_onnx_ops_b200.sharded import ExpertParallelMoE, shard_experts
    g = I_.rng(42)
    w1 = torch.from_numpy(I_.iq2_xxs_weights(g, (E, Iw), H)).to(dev)
    w2 = torch.from_numpy(I_.iq2_xxs_weights(g, (E, H), Iw)).to(dev)
    e0, el = shard_experts(E, world, rank)
    ep = ExpertParallelMoE(w1[e0:e0 + el].contiguous(), w2[e0:e0 + el].contiguous(), e0, topk, r_max=8)
    for R in (1, 3, 8, 1):
        for it in range(2):
            gg = I_.rng(1000 * R + it)
            z = torch.from_numpy(I_.bf16_normal(gg, (R, H)).view(np.int16)).view(torch.bfloat16).to(dev)
            idx = torch.from_numpy(np.stack([gg.choice(E, topk, replace=False) for _ in range(R)]).astype(np.int32)).to(dev)
            wt = torch.from_numpy(gg.random((R, topk)).astype(np.float32)).to(dev)
            out = ep(z, idx, wt)
            ref = ops.MoeVerify(z, idx, wt, w1, None, w2, None, topk=topk)[0]
            torch.cuda.synchronize()
            err = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
            if not err < 5e-3:
                failures.append(("moe_ep", R, it, err))
    ep.close()
    rc, site = _lib.device_status()
    if rc:
        failures.append(("device status", rc, site))
    dist.barrier()
    dist.destroy_process_group()
    if failures:
        print(f"rank {rank} FAILED {failures}", flush=True)
        sys.exit(1)
    print(f"rank {rank} ok", flush=True)


if __name__ == "__main__":
    main()
