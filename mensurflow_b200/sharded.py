"""Sharding of the GEMM path over ranks (one process per GPU, torch.distributed).

The path has no reduction across ranks: a 2-D GEMM splits by row blocks of A and C (B and the
bias replicated), a batched GEMM by the batch index, a gemv by rows of A. Each rank computes its
own slice in its own HBM with the single-GPU kernels; nothing crosses NVLink on the data path.
The one collective is optional: when the caller wants C on every rank (or on one), the row blocks
are all-gathered with NCCL (`all_gather_into_tensor`) into one contiguous [M, N] tensor — the
blocks are contiguous rows, so the gathered buffer needs no repacking.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist


def block_range(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [start, stop) of `rank`: equal blocks of ceil(total / world), the last one short."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    per = -(-total // world)
    start = min(total, rank * per)
    return start, min(total, start + per)


def local_rows(x: torch.Tensor, world: int, rank: int, dim: int = 0) -> torch.Tensor:
    """This rank's block of `x` along `dim` (a view, no copy)."""
    start, stop = block_range(x.shape[dim], world, rank)
    return x.narrow(dim, start, stop - start)


def gather_rows(local: torch.Tensor, total: int, group=None) -> torch.Tensor:
    """All-gathers every rank's row block (rows of block_range) into one [total, ...] tensor.
    Blocks are padded to the common block size for the collective and trimmed after it."""
    world = dist.get_world_size(group)
    per = -(-total // world)
    if local.shape[0] < per:
        pad = torch.zeros((per - local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                          device=local.device)
        send = torch.cat([local, pad], 0)
    else:
        send = local.contiguous()
    out = torch.empty((per * world,) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    dist.all_gather_into_tensor(out, send, group=group)
    return out[:total]


def sharded_gemm(a_local: torch.Tensor, b: torch.Tensor, m_total: int, alpha: float = 1.0,
                 c_local: Optional[torch.Tensor] = None, beta: float = 0.0,
                 transpose_b: bool = False, *, bias: Optional[torch.Tensor] = None,
                 activation: Optional[str] = None, gather: bool = False, group=None,
                 gemm_fn: Optional[Callable] = None) -> torch.Tensor:
    """C[rows of this rank] = act(alpha * A_local op(B) + beta * C_local + bias); with
    `gather=True` every rank receives the whole [m_total, N] C.

    `gemm_fn` defaults to the B200 kernel (mensurflow_b200.ops.gemm); it is a parameter so the
    host logic can be exercised with CPU ranks."""
    if gemm_fn is None:
        from .ops import gemm as gemm_fn
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    start, stop = block_range(m_total, world, rank)
    if a_local.shape[0] != stop - start:
        raise ValueError(f"sharded_gemm: rank {rank} holds {a_local.shape[0]} rows of A, its "
                         f"block is {stop - start}")
    c = gemm_fn(a_local, b, alpha, c_local, beta, False, transpose_b, bias=bias,
                activation=activation)
    if gather and world > 1:
        return gather_rows(c, m_total, group)
    return c


def sharded_gemm_batched(a_local: torch.Tensor, b_local: torch.Tensor, batch_total: int,
                         alpha: float = 1.0, transpose_b: bool = False, *, gather: bool = False,
                         group=None, gemm_fn: Optional[Callable] = None) -> torch.Tensor:
    """The batched GEMM split by the (flattened) batch index: each rank multiplies its matrices."""
    if gemm_fn is None:
        from .ops import gemm_strided_batched as gemm_fn
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    out = gemm_fn(a_local, b_local, alpha, None, 0.0, False, transpose_b)
    if gather and world > 1:
        return gather_rows(out, batch_total, group)
    return out
