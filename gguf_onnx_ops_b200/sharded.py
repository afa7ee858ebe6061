"""Multi-GPU sharding of the GGUF decode path (one process per GPU).

The reference runs on one GPU; the two sharded patterns here are the row-split GEMV of a large
output (the Q8 LM head) and -- through the same peer-memory machinery -- its building blocks.
torch.distributed is the plumbing only: it exchanges CUDA IPC handles once at set-up.  The data
path is a single kernel per call that computes this GPU's rows and stores them straight into a
staging buffer of every GPU of the group over NVLink (each value tagged with the call number), then
converts its own staging buffer into y as the tagged words arrive (bounded waits).

    shard = shard_rows(n_total, world, rank)          # (row0, rows) of this rank
    op = RowSplitGemv(GGUF_TYPE_Q8_0, w_full[row0:row0 + rows], n_total, row0, K, r_max=16)
    y = op(x)                                          # [R, n_total] bf16, complete on every GPU

Every rank must construct the op and call it the same number of times in the same order.  The
returned tensor is valid until the next call.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from ._lib import check, load
from .ops import IQ2_XXS_BYTES, NVFP4_BYTES, Q8_0_BYTES

MAX_PEERS = 8
_FMT = {_lib.GGUF_TYPE_Q8_0: (32, Q8_0_BYTES), _lib.GGUF_TYPE_IQ2_XXS: (256, IQ2_XXS_BYTES),
        _lib.GGUF_TYPE_NVFP4: (64, NVFP4_BYTES)}


def shard_rows(n_total: int, world: int, rank: int, align: int = 16) -> tuple[int, int]:
    """Contiguous, balanced split of n_total output rows; every boundary but the last is a multiple
    of `align` (the kernels' 16-row tiles)."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    units = -(-n_total // align)
    lo = (units * rank) // world * align
    hi = n_total if rank == world - 1 else (units * (rank + 1)) // world * align
    return min(lo, n_total), max(0, min(hi, n_total) - min(lo, n_total))


def exchange(payload, group=None) -> list:
    """all_gather_object of a picklable payload (the set-up step; works on gloo and NCCL groups)."""
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, payload, group=group)
    return out


def ipc_handle(t: torch.Tensor) -> tuple[bytes, int]:
    h = (ctypes.c_char * 64)()
    off = ctypes.c_int64(0)
    check(load().gguf_ipc_get_handle(ctypes.c_void_p(t.data_ptr()), h, ctypes.byref(off)))
    return bytes(h), off.value


def ipc_open(handle: bytes, offset: int) -> tuple[int, int]:
    """(pointer to use, base to close)."""
    p = ctypes.c_void_p(0)
    check(load().gguf_ipc_open(ctypes.c_char_p(handle), ctypes.byref(p)))
    return p.value + offset, p.value


class RowSplitGemv:
    """Row-split GEMV over raw GGUF rows with the all-gather fused into the kernel (see module doc)."""

    def __init__(self, gguf_type: int, w_shard: torch.Tensor, n_total: int, row0: int, K: int, r_max: int = 16,
                 gscale: torch.Tensor | None = None, group=None):
        if gguf_type not in _FMT:
            raise ValueError("unknown GGUF type")
        blk, nbytes = _FMT[gguf_type]
        self.type, self.K, self.n_total, self.row0 = gguf_type, K, n_total, row0
        self.rows = w_shard.shape[0]
        if w_shard.dtype != torch.uint8 or w_shard.numel() != self.rows * (K // blk) * nbytes:
            raise ValueError("w_shard must be raw GGUF rows [rows, (K/block)*type_size] (uint8)")
        self.w, self.gscale, self.group = w_shard.contiguous(), gscale, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > MAX_PEERS:
            raise ValueError("at most 8 GPUs per group")
        dev = w_shard.device
        self.r_max = r_max
        # this GPU's output, and per call parity a staging buffer that every GPU of the group writes
        # its shard into (32-bit words: bf16 value | call number << 16)
        self.y = torch.empty(r_max, n_total, dtype=torch.bfloat16, device=dev)
        self.stage = [torch.zeros(r_max, n_total, dtype=torch.int32, device=dev) for _ in range(2)]
        self.state = torch.zeros(1, dtype=torch.int64, device=dev)
        torch.cuda.synchronize(dev)
        # every GPU launches the same number of CTAs per call (the smallest SM count of the group): a
        # GPU numbers its calls by counting the CTAs it started
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        mine = [ipc_handle(self.stage[0]), ipc_handle(self.stage[1]), sms]
        allh = exchange(mine, group)
        self.ctas = min(h[2] for h in allh)
        self._opened = []
        self._po = _lib.GgufPeerOut()
        for p, hs in enumerate(allh):
            for c in range(2):
                if p == self.rank:
                    self._po.stage[c][p] = self.stage[c].data_ptr()
                else:
                    h, off = hs[c]
                    ptr, base = ipc_open(h, off)
                    self._opened.append(base)
                    self._po.stage[c][p] = ptr
        po = self._po
        po.y = self.y.data_ptr()
        po.state = self.state.data_ptr()
        po.world, po.rank = self.world, self.rank
        po.n_total, po.row0 = n_total, row0
        po.ctas, po.r_max = self.ctas, r_max

    def __call__(self, x: torch.Tensor, w: torch.Tensor | None = None, stream=None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        """y = x @ W^T over the whole group; `w` optionally replaces the shard (same shape and type).
        Returns `out` (bf16 [R, n_total], contiguous) or, without it, a view of this GPU's own output
        buffer that is valid until the next call."""
        R = x.shape[0]
        if x.dtype != torch.bfloat16 or x.shape[1] != self.K or not 1 <= R <= self.r_max:
            raise ValueError("x must be bf16 [R, K] with R <= r_max")
        w = self.w if w is None else w
        if w.shape != self.w.shape or w.dtype != torch.uint8 or not w.is_contiguous():
            raise ValueError("w must have the shard's shape")
        if out is not None and (out.dtype != torch.bfloat16 or out.shape != (R, self.n_total) or not out.is_contiguous()):
            raise ValueError("out must be contiguous bf16 [R, n_total]")
        y = self.y[:R] if out is None else out
        self._po.y = y.data_ptr()
        s = (stream or torch.cuda.current_stream()).cuda_stream
        gs = ctypes.c_void_p(self.gscale.data_ptr()) if self.gscale is not None else None
        check(load().gguf_gemv_rowsplit(self.type, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()), gs,
                                        ctypes.byref(self._po), R, self.rows, self.K, ctypes.c_void_p(s)))
        return y

    def close(self) -> None:
        for base in self._opened:
            load().gguf_ipc_close(ctypes.c_void_p(base))
        self._opened = []


def shard_experts(n_experts: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced split of the experts: (first expert, count) of this rank."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    lo, hi = (n_experts * rank) // world, (n_experts * (rank + 1)) // world
    return lo, hi - lo


class ExpertParallelMoE:
    """MoeVerify iq2=3 with the experts split across the group (one process per GPU).

    Every rank holds experts [offset, offset + E_local) and processes the pairs routed to them; the
    f32 partial outputs are summed across the group inside the finalize kernel through peer memory
    (see gguf_moe_verify_iq2_xxs_ep).  idx holds global expert ids (the router is replicated).
    """

    H = 1024

    def __init__(self, fc1_local: torch.Tensor, fc2_local: torch.Tensor, expert_offset: int, topk: int, r_max: int = 8,
                 group=None):
        self.E, self.I = fc1_local.shape[0], fc1_local.shape[1]
        if fc2_local.shape[0] != self.E or fc1_local.dtype != torch.uint8 or fc2_local.dtype != torch.uint8:
            raise ValueError("fc1 / fc2 must be raw IQ2_XXS expert tensors of the same experts")
        if not 1 <= r_max <= 8 or r_max * topk > 128:
            raise ValueError("r_max must be in [1, 8] with r_max * topk <= 128")
        self.w1, self.w2, self.offset, self.topk, self.r_max = fc1_local, fc2_local, expert_offset, topk, r_max
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        dev = fc1_local.device
        P = r_max * topk
        self.red = torch.zeros(2, self.world, r_max * self.H, dtype=torch.float32, device=dev)
        self.flags = torch.zeros(MAX_PEERS, dtype=torch.int32, device=dev)
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)
        self.h = torch.empty(P, self.I, dtype=torch.bfloat16, device=dev)
        self.part = torch.empty(P, self.H, dtype=torch.float32, device=dev)
        self.meta = torch.empty(1 + 9 * P, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        allh = exchange([ipc_handle(self.red), ipc_handle(self.flags)], group)
        self._opened = []
        self._pr = _lib.GgufPeerReduce()
        for p, ((hr, offr), (hf, offf)) in enumerate(allh):
            if p == self.rank:
                self._pr.slots[p], self._pr.flags[p] = self.red.data_ptr(), self.flags.data_ptr()
                continue
            pr_, br = ipc_open(hr, offr)
            pf, bf = ipc_open(hf, offf)
            self._opened += [br, bf]
            self._pr.slots[p], self._pr.flags[p] = pr_, pf
        self._pr.state = self.state.data_ptr()
        self._pr.world, self._pr.rank, self._pr.r_max = self.world, self.rank, r_max

    def __call__(self, z: torch.Tensor, idx: torch.Tensor, weights: torch.Tensor, out: torch.Tensor | None = None,
                 stream=None, w1: torch.Tensor | None = None, w2: torch.Tensor | None = None) -> torch.Tensor:
        """out = MoeVerify over the whole group; `w1` / `w2` optionally replace this rank's expert
        tensors (same shapes and type, e.g. another copy of the same experts)."""
        R = z.shape[0]
        w1 = self.w1 if w1 is None else w1
        w2 = self.w2 if w2 is None else w2
        if w1.shape != self.w1.shape or w2.shape != self.w2.shape or w1.dtype != torch.uint8 or w2.dtype != torch.uint8:
            raise ValueError("w1 / w2 must have the shapes of this rank's expert tensors")
        if z.dtype != torch.bfloat16 or z.shape[1] != self.H or not 1 <= R <= self.r_max:
            raise ValueError("z must be bf16 [R, 1024] with R <= r_max")
        if idx.dtype != torch.int32 or weights.dtype != torch.float32 or idx.shape != (R, self.topk):
            raise ValueError("idx int32 [R, topk] and weights f32 [R, topk] expected")
        out = torch.empty(R, self.H, dtype=torch.bfloat16, device=z.device) if out is None else out
        s = (stream or torch.cuda.current_stream()).cuda_stream
        p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        check(load().gguf_moe_verify_iq2_xxs_ep(p(z), p(idx), p(weights), p(w1), p(w2), p(out), p(self.h),
                                                p(self.part), p(self.meta), ctypes.byref(self._pr), R, self.E, self.offset,
                                                self.I, self.topk, ctypes.c_void_p(s)))
        return out

    def close(self) -> None:
        for base in self._opened:
            load().gguf_ipc_close(ctypes.c_void_p(base))
        self._opened = []
