"""The two cross-rank exchange steps of vocabulary-sharded CCE.

Kept free of any kernel call so the collective sequence can be exercised on
CPU ranks (gloo) as well as on GPUs (NCCL): every rank issues the same
collectives in the same order.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def gather_shard_stats(lse_local: torch.Tensor, tgt_local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather each rank's per-row (lse_r, tgt_r): returns [world, 2, N] fp32.

    One collective of 2 * N * 4 bytes per rank.
    """
    part = torch.stack([lse_local, tgt_local])                      # [2, N]
    world = dist.get_world_size(group)
    out = torch.empty((world * 2, part.shape[1]), dtype=part.dtype, device=part.device)
    dist.all_gather_into_tensor(out, part, group=group)             # rank-major concat
    return out.view(world, 2, part.shape[1])


def sum_grad_e(grad_e_partial: torch.Tensor, group=None) -> torch.Tensor:
    """In-place all-reduce(SUM) of the fp32 grad_e partials; returns the tensor."""
    dist.all_reduce(grad_e_partial, op=dist.ReduceOp.SUM, group=group)
    return grad_e_partial
