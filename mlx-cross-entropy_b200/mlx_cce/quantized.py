"""Cut Cross-Entropy with an affine group-quantised classifier.

The reference's mlx-lm recipe (README.md:84-95) dequantises the whole [V, D]
head with ``mx.dequantize`` before every call, because its kernels take a
dense ``c``.  Here the quantised head stays quantised in HBM and the library
expands it one vocabulary chunk at a time (``cce_forward_q`` /
``cce_backward_q``): two chunk buffers in the workspace, the next chunk
expanded on a side stream while the current chunk's GEMMs run, so the
expansion (HBM-bound) hides behind the tensor-core work:

* forward: every chunk's fused forward writes its columns of the tile maxima
  and of the LSE partials; one fold gives lse for the whole vocabulary;
* backward: the dense chunk loop (filter mask, dlogits, grad_e accumulated in
  fp32 across chunks) on the expanded chunks; grad_bias when the bias
  requires grad.

The quantised weight is frozen (as in LoRA fine-tuning, the recipe's use):
no gradient flows to ``weight``, ``scales`` or ``biases``.  Layout (MLX's
affine format for bits in {2, 4, 8}): ``weight`` uint32 (or int32 storage)
[V, D * bits / 32], 32 / bits values per word with the low bits first;
``scales`` and ``biases`` [V, D / group_size]; w = scales * q + biases per group.
"""

from __future__ import annotations

from typing import NamedTuple

import torch

from . import _ext
from ._autograd import REDUCTIONS, sanitize_targets
from ._ext import FILTER_LOG_EPS

__all__ = ["QuantizedClassifier", "linear_cross_entropy_quantized", "quantize"]


class QuantizedClassifier(NamedTuple):
    """An affine group-quantised [V, D] classifier (MLX layout, see the module docstring)."""

    weight: torch.Tensor   # uint32 / int32 [V, D * bits / 32]
    scales: torch.Tensor   # [V, D / group_size]
    biases: torch.Tensor   # [V, D / group_size]
    group_size: int = 64
    bits: int = 4

    @property
    def shape(self):
        return (self.weight.shape[0], self.weight.shape[1] * 32 // self.bits)

    def dequantize(self, dtype, v0: int = 0, v1: int | None = None, out=None):
        """Rows [v0, v1) as a dense ``dtype`` tensor (on the device)."""
        v1 = self.weight.shape[0] if v1 is None else v1
        return _ext.dequantize(self.weight[v0:v1], self.scales[v0:v1], self.biases[v0:v1],
                               self.group_size, self.bits, dtype, out=out)


def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4) -> QuantizedClassifier:
    """Affine group quantisation of a [V, D] matrix, on w's device (mx.quantize's format).

    Per group of ``group_size`` values along D: bias = min, scale =
    (max - min) / (2^bits - 1) (1 for a constant group), q = round((w - bias) /
    scale) clipped to [0, 2^bits); q packed 32 / bits per uint32, low bits
    first.  scales / biases keep w's dtype (float32 for float32 input).
    """
    if bits not in (2, 4, 8) or group_size not in (32, 64, 128):
        raise ValueError(f"bits must be 2, 4 or 8 and group_size 32, 64 or 128, got {bits}, {group_size}")
    V, D = w.shape
    if D % group_size != 0:
        raise ValueError(f"D={D} is not a multiple of group_size={group_size}")
    g = w.float().reshape(V, D // group_size, group_size)
    lo = g.amin(dim=2)
    scale = (g.amax(dim=2) - lo) / float((1 << bits) - 1)
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    q = torch.clamp(torch.round((g - lo[..., None]) / scale[..., None]), 0, (1 << bits) - 1)
    per = 32 // bits
    q = q.to(torch.int64).reshape(V, D // per, per)
    shifts = torch.arange(per, device=w.device, dtype=torch.int64) * bits
    words = (q << shifts).sum(dim=2)                        # < 2^32
    words = torch.where(words >= (1 << 31), words - (1 << 32), words).to(torch.int32)
    sdt = w.dtype if w.dtype in (torch.float16, torch.bfloat16, torch.float32) else torch.float32
    return QuantizedClassifier(words.contiguous(), scale.to(sdt).contiguous(), lo.to(sdt).contiguous(),
                               group_size, bits)


class QuantizedCCEFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, e, weight, scales, biases, bias, targets, valid, reduction, filter_log_eps,
                group_size, bits):
        tile_max, lse, tgt = _ext.forward_q(e, weight, scales, biases, group_size, bits, targets, bias)
        nll = lse - tgt
        validf = valid.to(torch.float32)
        per = nll * validf
        count = None
        if reduction == "none":
            out = per
        elif reduction == "sum":
            out = per.sum()
        else:
            count = validf.sum().clamp_min(1.0)
            out = per.sum() / count
        ctx.reduction = reduction
        ctx.filter_log_eps = filter_log_eps
        ctx.quant = (group_size, bits)
        ctx.has_bias = bias is not None
        ctx.save_for_backward(e, weight, scales, biases, bias, targets, validf, lse, count, tile_max)
        ctx.mark_non_differentiable(lse)
        return out, lse

    @staticmethod
    def backward(ctx, grad_out, _grad_lse):
        e, weight, scales, biases, bias, targets, validf, lse, count, tile_max = ctx.saved_tensors
        need_e = ctx.needs_input_grad[0]
        need_b = ctx.has_bias and ctx.needs_input_grad[4]
        none = (None,) * 11
        if grad_out is None or not (need_e or need_b):
            return none
        g = grad_out.to(torch.float32)
        if ctx.reduction == "none":
            d_nll = (g.reshape(-1) * validf).contiguous()
        elif ctx.reduction == "sum":
            d_nll = (validf * g).contiguous()
        else:
            d_nll = (validf * (g / count)).contiguous()
        grad_e, grad_b = _ext.backward_q(e, weight, scales, biases, *ctx.quant, targets, lse, d_nll, tile_max,
                                         bias, need_e=need_e, need_bias=need_b,
                                         filter_log_eps=ctx.filter_log_eps)
        return (grad_e, None, None, None, grad_b.to(bias.dtype) if need_b else None, None, None, None, None,
                None, None)


def linear_cross_entropy_quantized(e, c: QuantizedClassifier, targets, bias=None, reduction="mean",
                                   ignore_index=-100, shift=0, return_lse=False, *,
                                   filter_log_eps=FILTER_LOG_EPS):
    """``linear_cross_entropy`` with a quantised classifier ``c`` (frozen).

    Same arguments and results as ``mlx_cce.linear_cross_entropy``; the
    library expands the head one vocabulary chunk at a time, in e's dtype, on
    a side stream while the previous chunk's GEMMs run, and never as a whole
    [V, D] tensor.
    """
    if reduction not in REDUCTIONS:
        raise ValueError(f"Unknown reduction: {reduction}")
    if not isinstance(c, QuantizedClassifier):
        raise ValueError("c must be a QuantizedClassifier")
    V, D = c.shape
    if e.shape[-1] != D:
        raise ValueError(f"e's last dimension ({e.shape[-1]}) must equal the classifier's D ({D})")
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != V):
        raise ValueError(f"bias must be [V={V}], got {tuple(bias.shape)}")
    if shift:
        e = e[..., :-shift, :]
        targets = targets[..., shift:]
    orig_shape = targets.shape
    safe, valid = sanitize_targets(targets.reshape(-1), ignore_index)
    e2 = e.reshape(-1, D).contiguous()
    loss, lse = QuantizedCCEFunction.apply(e2, c.weight.contiguous(), c.scales.contiguous(),
                                           c.biases.contiguous(),
                                           None if bias is None else bias.contiguous(), safe, valid,
                                           reduction, filter_log_eps, int(c.group_size), int(c.bits))
    if reduction == "none":
        loss = loss.reshape(orig_shape)
    return (loss, lse) if return_lse else loss
