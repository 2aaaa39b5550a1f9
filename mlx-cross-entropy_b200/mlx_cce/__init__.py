"""B200-native Cut Cross-Entropy with the reference's Python API.

    from mlx_cce import linear_cross_entropy
    loss = linear_cross_entropy(hidden_states, classifier_weight, targets)

Same entry points and argument meaning as the reference package
(mlx_cce/__init__.py:54-107 of sb1992/mlx-cross-entropy): ``linear_cross_entropy``,
the flat ``cce_loss`` and the one-call ``cut_cross_entropy``, with
``reduction`` in {"mean", "sum", "none"} and ``ignore_index`` (default -100,
``None`` = nothing ignored).  The operands are CUDA ``torch.Tensor`` objects
(float32, float16 or bfloat16) instead of MLX arrays; the loss is float32.
The [N, V] logits are never materialised.  The research package's extras
``shift`` and ``return_lse`` (reference/__init__.py:22-57) and the
``LinearCrossEntropy`` module (reference/__init__.py:88-118) are provided too,
and ``linear_cross_entropy_quantized`` for an affine group-quantised head
(the reference's mlx-lm recipe dequantises the whole head first, README.md:84-95).

Kernels: hand-written sm_100a CUDA in ``libcce_b200.so`` (tcgen05 / TMEM / TMA
for 16-bit inputs, CUDA-core FFMA for float32), called through its C ABI.
"""

from __future__ import annotations

__version__ = "0.1.0"

import torch

from . import _ext
from ._autograd import REDUCTIONS, CCEFunction, sanitize_targets
from ._ext import FILTER_LOG_EPS, cce_backward_raw, cce_forward_raw, cut_cross_entropy

__all__ = ["linear_cross_entropy", "cce_loss", "cut_cross_entropy", "LinearCrossEntropy",
           "cce_forward_raw", "cce_backward_raw", "FILTER_LOG_EPS", "QuantizedClassifier",
           "linear_cross_entropy_quantized"]


def _cce(e, c, targets, bias, reduction, ignore_index, filter_log_eps, group, v_offset,
         skip_stats):
    if reduction not in REDUCTIONS:
        raise ValueError(f"Unknown reduction: {reduction}")
    if e.dim() != 2:
        raise ValueError(f"e must be 2D [B, D], got {e.dim()}D")
    if c.dim() != 2:
        raise ValueError(f"c must be 2D [V, D], got {c.dim()}D")
    if targets.reshape(-1).shape[0] != e.shape[0]:
        raise ValueError(f"targets hold {targets.numel()} values for {e.shape[0]} rows of e")
    safe, valid = sanitize_targets(targets, ignore_index)
    e = e.contiguous()
    c = c.contiguous()
    if bias is not None:
        bias = bias.contiguous()
    return CCEFunction.apply(e, c, bias, safe, valid, reduction, filter_log_eps, group, v_offset,
                             skip_stats)


def cce_loss(e, c, targets, bias=None, reduction="mean", ignore_index=-100, *,
             return_lse=False, filter_log_eps=FILTER_LOG_EPS, skip_stats=None):
    """Flat-input CCE (reference mlx_cce/__init__.py:54-76).

    e [N, D], c [V, D], targets [N]; returns a float32 scalar, or [N] for
    ``reduction='none'``.  ``skip_stats`` (optional CUDA int64[2]) accumulates
    (skipped, total) 128-row x 32-column backward blocks.
    """
    loss, lse = _cce(e, c, targets, bias, reduction, ignore_index, filter_log_eps, None, 0,
                     skip_stats)
    return (loss, lse) if return_lse else loss


IMPLS = ("auto", "fused", "chunked", "reference")


def linear_cross_entropy(e, c, targets, bias=None, reduction="mean", ignore_index=-100,
                         shift=0, return_lse=False, impl="auto", compute_all_grads=False, *,
                         filter_log_eps=FILTER_LOG_EPS, skip_stats=None):
    """Memory-efficient cross-entropy that never materialises [N, V] logits.

    Args (reference mlx_cce/__init__.py:79-107, reference/__init__.py:22-57):
        e: hidden states [..., D]
        c: classifier weights [V, D]
        targets: target ids [...]
        bias: optional classifier bias [V]
        reduction: "mean", "sum" or "none"
        ignore_index: target value to mask (-100 default; None masks nothing)
        shift: drop the last ``shift`` positions of e and the first ``shift``
            of targets along the sequence axis (causal-LM alignment)
        return_lse: also return the per-row log-sum-exp (float32, flat [N])
        impl: accepted for signature compatibility with the research package
            (reference/__init__.py:22-85, which picks one of several MLX / Metal
            implementations); every value runs the one CUDA path here
        compute_all_grads: accepted for signature compatibility; gradients
            reach ``c`` and ``bias`` whenever those tensors require grad
    Returns:
        float32 loss scalar, or per-token loss shaped like ``targets`` for
        reduction="none"; ``(loss, lse)`` with ``return_lse``.
    """
    if reduction not in REDUCTIONS:
        raise ValueError(f"Unknown reduction: {reduction}")
    if impl not in IMPLS:
        raise ValueError(f"Unknown impl: {impl!r}; expected one of {IMPLS}")
    if shift:
        e = e[..., :-shift, :]
        targets = targets[..., shift:]
    orig_shape = targets.shape
    D = e.shape[-1]
    loss, lse = _cce(e.reshape(-1, D), c, targets.reshape(-1), bias, reduction, ignore_index,
                     filter_log_eps, None, 0, skip_stats)
    if reduction == "none":
        loss = loss.reshape(orig_shape)
    return (loss, lse) if return_lse else loss


class LinearCrossEntropy(torch.nn.Module):
    """Module form (reference/__init__.py:88-118).

    ``criterion = LinearCrossEntropy(reduction="mean")`` then
    ``loss = criterion(hidden_states, classifier_weight, targets, bias=None)``.
    """

    def __init__(self, reduction="mean", ignore_index=-100, shift=0, compute_all_grads=False):
        super().__init__()
        if reduction not in REDUCTIONS:
            raise ValueError(f"Unknown reduction: {reduction}")
        self.reduction = reduction
        self.ignore_index = ignore_index
        self.shift = shift
        self.compute_all_grads = compute_all_grads

    def forward(self, e, c, targets, bias=None):
        return linear_cross_entropy(e, c, targets, bias=bias, reduction=self.reduction,
                                    ignore_index=self.ignore_index, shift=self.shift)


from .quantized import QuantizedClassifier, linear_cross_entropy_quantized  # noqa: E402
