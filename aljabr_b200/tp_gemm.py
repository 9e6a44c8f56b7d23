"""Tensor-parallel batched linear layers (a Llama-3-70B
layer with its weights row-sharded over the GPUs of one node and the outputs
all-gathered over NVLink).

Every weight matrix is row-sharded (each rank holds a contiguous block of
rows, `decode.shard_rows`), each rank runs the batched NF4 GEMM on its block,
and the per-rank outputs y_r [M][rows_r] are joined in rank order into
[M][world * rows_r] on every rank.  The join is `torch.distributed.all_gather`
(NCCL over NVLink on GPUs, gloo on CPU).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def gather_token_rows(y_local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather a row-sharded batched output: y_local is this rank's
    [M][rows] block; returns [M][world * rows] with rank r's rows at
    [r * rows, (r + 1) * rows)."""
    if world == 1:
        return y_local
    y_local = y_local.contiguous()
    parts = [torch.empty_like(y_local) for _ in range(world)]
    dist.all_gather(parts, y_local, group=group)
    return torch.cat(parts, dim=1)


def shard_extent(n: int, world: int, rank: int) -> tuple:
    """(first row, rows) of rank's contiguous block of an n-row matrix."""
    if n % world:
        raise ValueError(f"{n} rows do not divide over {world} ranks")
    rows = n // world
    return rank * rows, rows
