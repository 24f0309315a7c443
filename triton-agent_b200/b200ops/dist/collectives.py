"""Column-sharded INT8 GEMM with an all-gather of the output blocks.

Rank r holds W rows [n0_r, n1_r) (equal blocks, column_shard) and the whole
A; it computes C_r = A W_r^T, [M, n_r], then every rank receives every block.
NCCL all-gather needs equal contiguous chunks, so blocks are gathered as
[world, M, n_blk] and placed into the row-major [M, N] output with one
device copy; both steps are inside the timed region of the benchmark.
"""

from __future__ import annotations

import torch

from .sharding import column_shard


def allgather_columns(local: torch.Tensor, N: int, group=None) -> torch.Tensor:
    """local [M, n_blk] (n_blk the padded block width) -> full C [M, N]."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    M, n_blk = local.shape
    buf = torch.empty(world * M, n_blk, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, local.contiguous(), group=group)
    return buf.view(world, M, n_blk).permute(1, 0, 2).reshape(M, world * n_blk)[:, :N]


def sharded_int8_gemm(A, W_local, sA, sW_local, N: int, gemm, out_dtype=torch.float16, group=None):
    """C = gather_r(gemm(A, W_r)) for the column block of this rank.

    `gemm(A, W, sA, sW, out)` writes [M, n_r] into `out`; blocks narrower than
    the common width (last rank) are zero-padded before the gather.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n0, n1 = column_shard(N, world, rank)
    n_blk = column_shard(N, world, 0)[1]
    M = A.shape[0]
    local = torch.zeros(M, n_blk, dtype=out_dtype, device=A.device)
    if n1 > n0:
        gemm(A, W_local, sA, sW_local, local[:, : n1 - n0])
    return allgather_columns(local, N, group)
