"""Column (N) sharding of the W4A16 GEMM across the GPUs of one node.

Output columns of y = x . W are independent, so rank r of P owns columns
[r*N/P, (r+1)*N/P): its slice of qweight is qweight[:, r*N/(8P):(r+1)*N/(8P)]
(packed words never straddle shards because N/P is a multiple of 8, in fact
of 32 for the TMA pitch rule), and scales/zeros[:, r*N/P:(r+1)*N/P].  x is
replicated.  The one exchange step is an all-gather of the [M, N/P] output
slices over NCCL (NVLink/NVSwitch), gathered as [P, M, N/P] and laid out as
[M, N].  Nothing else is partitioned.

The reference has no multi-GPU path (every task is gpus = 1,
generate_tasks.py:149); this module is the benchmark's sharded configuration.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist
import torch.nn as nn


def shard_bounds(N: int, world: int, rank: int) -> tuple[int, int]:
    if N % world:
        raise ValueError(f"N={N} is not divisible by world size {world}")
    n = N // world
    if n % 32:
        raise ValueError(f"shard width {n} must be a multiple of 32 columns")
    return rank * n, (rank + 1) * n


def shard_weights(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, world: int,
                  rank: int):
    """This rank's column shard (contiguous copies) of the packed weight,
    scales and zero points."""
    N = qweight.shape[1] * 8
    lo, hi = shard_bounds(N, world, rank)
    return (qweight[:, lo // 8:hi // 8].contiguous(), scales[:, lo:hi].contiguous(),
            zeros[:, lo:hi].contiguous())


def gather_columns(y_local: torch.Tensor, world: int, group: Optional[dist.ProcessGroup] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All-gather [M, N/P] slices into y [M, N] (column block r from rank r)."""
    M, n = y_local.shape
    buf = torch.empty((world * M, n), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local.contiguous(), group=group)
    if out is None:
        out = torch.empty((M, world * n), dtype=y_local.dtype, device=y_local.device)
    out.view(M, world, n).copy_(buf.view(world, M, n).permute(1, 0, 2))
    return out


class ColumnShardedW4A16(nn.Module):
    """Tensor-parallel W4A16 linear: local dequant-GEMM on this rank's column
    shard, then all-gather of the output columns."""

    def __init__(self, group_size: int = 128, process_group: Optional[dist.ProcessGroup] = None,
                 local_gemm: Optional[Callable] = None):
        super().__init__()
        self.group_size = group_size
        self.pg = process_group
        if local_gemm is None:
            from . import ops
            local_gemm = ops.w4a16_gemm
        self.local_gemm = local_gemm

    def forward(self, x: torch.Tensor, qweight_shard: torch.Tensor, scales_shard: torch.Tensor,
                zeros_shard: torch.Tensor) -> torch.Tensor:
        world = dist.get_world_size(self.pg) if dist.is_initialized() else 1
        y_local = self.local_gemm(x, qweight_shard, scales_shard, zeros_shard, self.group_size)
        if world == 1:
            return y_local
        return gather_columns(y_local, world, self.pg)
