"""torch.autograd.Function around the C-ABI forward / backward.

This replaces the reference's ``mx.custom_function`` pair ``_cce_fused`` /
``_cce_fused_vjp`` (mlx_cce/__init__.py:21-51) and the C++ VJP
``CutCrossEntropy::vjp`` (csrc/cce/cce.cpp:395-452).  Differences that are
deliberate:

* gradients w.r.t. ``c`` and ``bias`` are real whenever those tensors require
  grad (the reference's shipped VJP returns zeros for them,
  mlx_cce/__init__.py:46-51; its compute_all_grads path,
  reference/_fused_backward.py:1618-1655, defines what they must be);
* with a process group, ``c``/``bias`` are this rank's vocabulary shard and
  the per-row LSE / target logit are merged across ranks (one all-gather), and
  grad_e is summed across ranks inside the library's backward over NVLink
  peer memory (``cce_backward_peer``; ``_peer`` holds the exchange buffers).
  ``CCE_GRAD_E_EXCHANGE=nccl`` in the environment selects the unfused
  baseline instead: an fp32 grad_e partial per rank and one NCCL all-reduce.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from . import _ext, _peer
from ._exchange import gather_shard_stats, sum_grad_e

REDUCTIONS = ("none", "sum", "mean")


def _peer_exchange() -> bool:
    return os.environ.get("CCE_GRAD_E_EXCHANGE", "peer") != "nccl"


class CCEFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, e, c, bias, targets, valid, reduction, filter_log_eps, group, v_offset,
                skip_stats):
        # e [N, D], c [V, D], targets int32 sanitised [N], valid bool [N]
        tile_max, lse_l, tgt_l = _ext.forward(e, c, targets, bias, v_offset=v_offset)
        world = dist.get_world_size(group) if group is not None else 1
        if world > 1:
            gathered = gather_shard_stats(lse_l, tgt_l, group)        # [world, 2, N]
            lse, _tgt, nll = _ext.lse_combine(gathered[:, 0, :], gathered[:, 1, :])
        else:
            lse, nll = lse_l, lse_l - tgt_l
        validf = valid.to(torch.float32)
        per = nll * validf
        if reduction == "none":
            out = per
            count = None
        elif reduction == "sum":
            out = per.sum()
            count = None
        else:
            count = validf.sum().clamp_min(1.0)
            out = per.sum() / count
        ctx.reduction = reduction
        ctx.filter_log_eps = filter_log_eps
        ctx.group = group
        ctx.world = world
        ctx.v_offset = v_offset
        ctx.skip_stats = skip_stats
        ctx.has_bias = bias is not None
        ctx.save_for_backward(e, c, bias, targets, validf, lse, tile_max, count)
        ctx.mark_non_differentiable(lse)
        return out, lse

    @staticmethod
    def backward(ctx, grad_out, _grad_lse):
        e, c, bias, targets, validf, lse, tile_max, count = ctx.saved_tensors
        need_e = ctx.needs_input_grad[0]
        need_c = ctx.needs_input_grad[1]
        need_b = ctx.has_bias and ctx.needs_input_grad[2]
        if grad_out is None or not (need_e or need_c or need_b):
            return (None,) * 10
        g = grad_out.to(torch.float32)
        if ctx.reduction == "none":
            d_nll = (g.reshape(-1) * validf).contiguous()
        elif ctx.reduction == "sum":
            d_nll = (validf * g).contiguous()
        else:
            d_nll = (validf * (g / count)).contiguous()
        sharded = ctx.world > 1
        peer = sharded and need_e and _peer_exchange()
        pg = _peer.group_for(ctx.group, e.device, e.shape[0], e.shape[1], e.dtype) if peer else None
        ge, gc, gb = _ext.backward(e, c, targets, lse, d_nll, tile_max, bias, v_offset=ctx.v_offset,
                                   need_e=need_e, need_c=need_c, need_bias=need_b,
                                   grad_e_f32=sharded and need_e and not peer,
                                   filter_log_eps=ctx.filter_log_eps,
                                   skip_stats=ctx.skip_stats, peer_group=pg)
        if sharded and need_e and not peer:
            ge = sum_grad_e(ge, ctx.group).to(e.dtype)
        if gb is not None:
            gb = gb.to(bias.dtype)
        return ge, gc, gb, None, None, None, None, None, None, None


def sanitize_targets(targets, ignore_index):
    """mlx_cce/__init__.py:59-64: valid mask and int32 targets with ignored rows set to 0."""
    t = targets.reshape(-1)
    if ignore_index is None:
        valid = torch.ones(t.shape, dtype=torch.bool, device=t.device)
        return t.to(torch.int32).contiguous(), valid
    valid = t != ignore_index
    safe = torch.where(valid, t, torch.zeros_like(t)).to(torch.int32).contiguous()
    return safe, valid
