"""KV-head tensor parallelism over NCCL (one process per GPU).

KV heads shard naturally: rank r of tp owns KV heads [r*G/tp, (r+1)*G/tp) and
their query heads for every row, its own pools, scores, positions and tables.
Per-head selection and compaction need no communication, and every rank frees
the same units because targets depend only on the shared protected columns
and the budget.  Two exchanges remain:

  * the attention-output reduction of a layer: each rank multiplies its heads'
    outputs by its row slice of the output projection and the partial hidden
    states are summed with an NCCL all-reduce (row-parallel o_proj);
  * H2O global at a boundary: the per-head scores of the boundary rows are
    all-gathered so every rank ranks the same sum over all KV heads.
"""
from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def init_from_env(backend: str = "nccl", timeout_s: int = 120):
    """torchrun-style initialisation (RANK/WORLD_SIZE/LOCAL_RANK/MASTER_*)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return None, 0, 1
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    if backend == "nccl":
        torch.cuda.set_device(local)
    if not dist.is_initialized():
        kwargs = dict(backend=backend, timeout=timedelta(seconds=timeout_s))
        if backend == "nccl":
            kwargs["device_id"] = torch.device("cuda", local)
        dist.init_process_group(**kwargs)
    return dist.group.WORLD, rank, world


def shard(kv_heads: int, q_heads: int, rank: int, world: int):
    """(local kv heads, local q heads, head offset) of a rank."""
    if kv_heads % world:
        raise ValueError(f"{kv_heads} KV heads do not split over {world} ranks")
    g = kv_heads // world
    return g, q_heads // world, rank * g


def all_gather_heads(local: torch.Tensor, group) -> torch.Tensor:
    """[R, L, G_local, C] per rank -> [R, L, G_local*world, C], heads in rank order."""
    world = dist.get_world_size(group)
    R, L, G, C = local.shape
    # ranks concatenated along dim 0 (the layout every backend accepts)
    buf = torch.empty((world * R, L, G, C), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, local.contiguous(), group=group)
    return buf.view(world, R, L, G, C).permute(1, 2, 0, 3, 4).reshape(R, L, world * G, C).contiguous()


def output_reduction(attn_out: torch.Tensor, w_slice: torch.Tensor, group, out=None):
    """Row-parallel output projection + NCCL all-reduce of one layer.

    attn_out [B, H_local, D] bf16, w_slice [H_local*D, hidden] bf16.
    """
    partial = torch.matmul(attn_out.reshape(attn_out.shape[0], -1), w_slice, out=out)
    if group is not None and dist.get_world_size(group) > 1:
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial
