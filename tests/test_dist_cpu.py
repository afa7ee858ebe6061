"""Host logic of the multi-GPU path on CPU: the row partition, the set-up exchange over a real
2-rank gloo group, and the sharded computation's semantics (every rank computes its rows with the
oracle; the gathered rows equal the single-device result bit for bit)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from gguf_onnx_ops_b200.sharded import exchange, shard_rows
from oracle import inputs as I


@pytest.mark.parametrize("n", [1, 15, 16, 17, 96, 4096, 131072, 14336, 13824])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_rows_partition(n, world):
    spans = [shard_rows(n, world, r) for r in range(world)]
    pos = 0
    for r, (row0, rows) in enumerate(spans):
        assert row0 == pos and rows >= 0
        if r < world - 1:
            assert (row0 + rows) % 16 == 0 or row0 + rows == n
        pos = row0 + rows
    assert pos == n
    sizes = [rows for _, rows in spans]
    assert max(sizes) - min(sizes) <= 16 * (1 + (n % 16 != 0))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # set-up exchange: every rank sees every payload, in rank order
        got = exchange({"rank": rank, "handle": bytes([rank]) * 64})
        assert [g["rank"] for g in got] == list(range(world))
        assert all(g["handle"] == bytes([i]) * 64 for i, g in enumerate(got))
        # sharded Q8 GEMV semantics with the oracle standing in for the kernel
        x, w, _ = I.gemv_case("q8_0", 3, 200, 256, seed=5)
        row0, rows = shard_rows(200, world, rank)
        y_shard = O.gemv_ref(x, O.dequant_q8_0(w[row0:row0 + rows])).astype(np.float32)
        parts = [None] * world
        dist.all_gather_object(parts, (row0, y_shard))
        y = np.zeros((3, 200), np.float32)
        for r0, ys in parts:
            y[:, r0:r0 + ys.shape[1]] = ys
        full = O.gemv_ref(x, O.dequant_q8_0(w)).astype(np.float32)
        q.put((rank, bool(np.array_equal(y, full))))
    finally:
        dist.destroy_process_group()


@pytest.mark.dist
def test_two_rank_gloo_exchange_and_sharded_semantics():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res == {0: True, 1: True}
