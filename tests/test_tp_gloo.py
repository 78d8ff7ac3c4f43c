"""KV-head tensor-parallel host logic on CPU ranks (gloo, world size 2).

Covers the two exchanges of the sharded path (tp.py): the all-gather of
per-head boundary scores that H2O global needs, and the attention-output
reduction of the row-parallel output projection; plus the head split.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cache_eviction_b200 import tp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g_local = 8 // world
        # per-head scores: value = 1000*global_head + 10*layer + row
        R, L, C = 3, 2, 5
        local = torch.zeros((R, L, g_local, C))
        for r in range(R):
            for l in range(L):
                for g in range(g_local):
                    local[r, l, g] = 1000 * (rank * g_local + g) + 10 * l + r
        full = tp.all_gather_heads(local, dist.group.WORLD)
        ok_gather = full.shape == (R, L, 8, C) and all(
            bool((full[r, l, h] == 1000 * h + 10 * l + r).all())
            for r in range(R) for l in range(L) for h in range(8))
        # output reduction: sum over ranks of attn_out[:, local heads] @ w[local rows]
        gen = torch.Generator().manual_seed(7)
        attn = torch.randn((4, 8, 64), generator=gen)
        w = torch.randn((8 * 64, 16), generator=gen)
        h0 = rank * g_local
        partial = tp.output_reduction(attn[:, h0:h0 + g_local].contiguous(),
                                      w[h0 * 64:(h0 + g_local) * 64], dist.group.WORLD)
        ok_reduce = torch.allclose(partial, attn.reshape(4, -1) @ w, rtol=1e-4, atol=1e-4)
        q.put((rank, ok_gather, ok_reduce))
    finally:
        dist.destroy_process_group()


def test_all_gather_heads_and_output_reduction_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_gather, ok_reduce in results:
        assert ok_gather, f"rank {rank}: gathered heads out of order"
        assert ok_reduce, f"rank {rank}: output reduction mismatch"


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_splits_heads(world):
    g, h, off = tp.shard(8, 64, world - 1, world)
    assert g == 8 // world and h == 64 // world and off == (world - 1) * g
    with pytest.raises(ValueError):
        tp.shard(8, 64, 0, 3)


def test_init_from_env_single_process_is_noop(monkeypatch):
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    assert tp.init_from_env("gloo") == (None, 0, 1)
