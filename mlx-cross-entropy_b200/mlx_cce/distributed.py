"""Vocabulary-sharded CCE across the GPUs of one node (one process per GPU).

Each rank holds the full hidden states ``e [N, D]`` and targets, and one
contiguous slice ``c[v0:v1]`` (and ``bias[v0:v1]``) of the classifier.  Rows
are independent and the per-row log-sum-exp over V decomposes exactly into
per-shard (lse_r, target-logit_r) pairs, so the path has two real exchange
steps, both through ``torch.distributed`` (NCCL over NVLink on B200):

* forward: one ``all_gather_into_tensor`` of the [2, N] fp32 (lse_r, tgt_r)
  rows, merged on every rank by the ``cce_lse_combine`` kernel, so every rank
  holds the identical loss;
* backward: grad_e is summed across the ranks inside the library's backward
  (``cce_backward_peer``): the last grad_e GEMM of each rank stores its fp32
  tiles into the exchange buffer of the rank that owns those rows over NVLink
  peer memory, owners reduce in rank order and every rank gathers the summed
  rows.  ``CCE_GRAD_E_EXCHANGE=nccl`` selects the unfused baseline instead
  (fp32 partials, one NCCL ``all_reduce``).  grad_c and grad_bias stay sharded.

The reference has no multi-device code; this is the build's own addition for
the multi-GPU rows of the benchmark.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import REDUCTIONS, FILTER_LOG_EPS
from ._autograd import CCEFunction, sanitize_targets


def vocab_shard(V: int, rank: int, world: int):
    """Even split of [0, V) into ``world`` contiguous ranges; returns (v0, v1)."""
    base, rem = divmod(V, world)
    v0 = rank * base + min(rank, rem)
    v1 = v0 + base + (1 if rank < rem else 0)
    return v0, v1


def linear_cross_entropy(e, c_shard, targets, bias_shard=None, reduction="mean",
                         ignore_index=-100, *, v_offset, group=None,
                         filter_log_eps=FILTER_LOG_EPS, return_lse=False, skip_stats=None):
    """Vocabulary-parallel ``linear_cross_entropy``.

    ``c_shard`` [V_r, D] holds global vocabulary rows [v_offset, v_offset + V_r);
    ``targets`` hold global ids.  Every rank must call with the same e,
    targets, reduction and ignore_index.  Returns the same loss on every rank.
    """
    if reduction not in REDUCTIONS:
        raise ValueError(f"Unknown reduction: {reduction}")
    orig_shape = targets.shape
    D = e.shape[-1]
    safe, valid = sanitize_targets(targets.reshape(-1), ignore_index)
    e2 = e.reshape(-1, D).contiguous()
    g = group if group is not None else dist.group.WORLD
    loss, lse = CCEFunction.apply(e2, c_shard.contiguous(),
                                  bias_shard.contiguous() if bias_shard is not None else None,
                                  safe, valid, reduction, filter_log_eps, g, int(v_offset),
                                  skip_stats)
    if reduction == "none":
        loss = loss.reshape(orig_shape)
    return (loss, lse) if return_lse else loss
