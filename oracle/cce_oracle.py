"""CPU oracle for the Cut Cross-Entropy hot path (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
(``cpu_baseline`` / ``--impl reference``) import it.  The CUDA path in
``mlx-cross-entropy_b200/`` never calls into it and fails loudly when its
extension is missing.

It restates, in numpy, the reference's pure-MLX implementation of the path:

* ``dense_forward``     -- reference/_reference.py:5-48
  (logits = e @ c.T [+ bias], per-row cross-entropy, ignore mask, reduction).
* ``chunked_forward``   -- reference/_chunked.py:4-71 and the chunked path of
  reference/_ops.py:80-110 (target-logit gather, online max / sum-exp over
  vocab chunks of 4096 starting from running_max = -1e38, fp32 statistics).
* ``backward_full``     -- reference/_metal_backward.py:245-261
  (dlogits = d_nll * (softmax - onehot); dE = dlogits @ c; dC = dlogits.T @ e;
  dBias = sum_rows dlogits).
* ``backward_filtered`` -- the same gradients with the block-skip rule of
  csrc/cce/cce.metal:143,190-204 (a block of rows x vocab columns is kept when
  any row has its target in it or ``tile_max - lse >= ln(2^-12)``).
* ``reduce``            -- mlx_cce/__init__.py:59-76 (sanitised targets,
  valid mask, none / sum / mean with the max(count, 1) denominator).
* ``quantize_affine`` / ``dequantize_affine`` -- the affine group
  quantisation the reference's mlx-lm recipe undoes before every call
  (README.md:84-95, ``mx.dequantize`` of a quantised head): per group of
  ``group_size`` values along D, w = scale * q + bias with q in
  [0, 2^bits); q packed 32 / bits per uint32, low bits first.  The format is
  MLX's (mlx.core.quantize, third-party, not vendored); this restates its
  published definition for bits in {2, 4, 8}.

PARITY UNPINNED: the reference's arithmetic lives in MLX (pinned only as
``mlx>=0.22.0``, pyproject.toml:5,18), which is not installed here and cannot
be installed (no network); the reference ships no golden vectors (its tests,
tests/test_correctness.py and tests/test_gradients.py, compare differentially
against MLX's own dense ``nn.losses.cross_entropy``).  This restatement is
therefore cross-checked against ``torch.nn.functional.cross_entropy`` and
torch autograd -- an independent implementation of the same definition the
reference's tests use as their oracle -- in tests/test_oracle.py.
"""

from __future__ import annotations

import math

import numpy as np

# ln(2^-12): the gradient-filter threshold of csrc/cce/cce.metal:143 and
# reference/_metal_backward.py:17.
FILTER_LOG_EPS = math.log(2.0 ** -12)
# Vocab chunk of the pure-MLX online-LSE path (reference/_chunked.py:12).
CHUNK = 4096
# Initial running max of reference/_chunked.py:31.
RUNNING_MAX_INIT = -1e38


def _f(x, dtype):
    return np.asarray(x, dtype=dtype)


def sanitize(targets, ignore_index=-100):
    """mlx_cce/__init__.py:59-64: valid mask and targets with ignored rows set to 0."""
    t = np.asarray(targets).reshape(-1).astype(np.int64)
    if ignore_index is None:
        valid = np.ones(t.shape, dtype=bool)
        return t, valid
    valid = t != ignore_index
    return np.where(valid, t, 0), valid


def reduce(nll, valid, reduction):
    """mlx_cce/__init__.py:67-76 and reference/_reference.py:33-44."""
    per = nll * valid.astype(nll.dtype)
    if reduction == "none":
        return per
    if reduction == "sum":
        return per.sum()
    if reduction == "mean":
        return per.sum() / max(int(valid.sum()), 1)
    raise ValueError(f"Unknown reduction: {reduction!r}")


def logits_f64(e, c, bias=None):
    """e @ c.T (+ bias) in float64 (reference/_reference.py:24-26)."""
    z = _f(e, np.float64) @ _f(c, np.float64).T
    if bias is not None:
        z = z + _f(bias, np.float64)[None, :]
    return z


def dense_forward(e, c, targets, bias=None, ignore_index=-100):
    """Per-row NLL, LSE and target logit in float64 (reference/_reference.py:24-31).

    Returns (nll[N], lse[N], tgt[N], valid[N]); ``nll`` is not yet masked.
    """
    t, valid = sanitize(targets, ignore_index)
    z = logits_f64(e, c, bias)
    m = z.max(axis=1)
    lse = m + np.log(np.exp(z - m[:, None]).sum(axis=1))
    tgt = z[np.arange(z.shape[0]), t]
    return lse - tgt, lse, tgt, valid


def chunked_forward(e, c, targets, bias=None, ignore_index=-100, chunk=CHUNK):
    """Online-LSE forward of reference/_chunked.py:26-54 in float32.

    Returns (nll[N], lse[N], tgt[N], valid[N]) as float32 (nll unmasked).
    """
    t, valid = sanitize(targets, ignore_index)
    e32 = _f(e, np.float32)
    c32 = _f(c, np.float32)
    b32 = None if bias is None else _f(bias, np.float32)
    n = e32.shape[0]
    V = c32.shape[0]
    tgt = (e32 * c32[t]).sum(axis=-1, dtype=np.float32)
    if b32 is not None:
        tgt = tgt + b32[t]
    run_max = np.full((n,), RUNNING_MAX_INIT, dtype=np.float32)
    run_sum = np.zeros((n,), dtype=np.float32)
    for v0 in range(0, V, chunk):
        v1 = min(v0 + chunk, V)
        z = e32 @ c32[v0:v1].T
        if b32 is not None:
            z = z + b32[None, v0:v1]
        new_max = np.maximum(run_max, z.max(axis=1))
        run_sum = run_sum * np.exp(run_max - new_max) + np.exp(z - new_max[:, None]).sum(axis=1)
        run_max = new_max
    lse = run_max + np.log(run_sum)
    return (lse - tgt).astype(np.float32), lse.astype(np.float32), tgt.astype(np.float32), valid


def d_nll_from_reduction(valid, reduction, grad_out=None):
    """Cotangent of the per-row NLL implied by the reduction (mlx_cce/__init__.py:67-76)."""
    v = valid.astype(np.float64)
    if reduction == "mean":
        g = 1.0 if grad_out is None else float(grad_out)
        return v * g / max(int(valid.sum()), 1)
    if reduction == "sum":
        g = 1.0 if grad_out is None else float(grad_out)
        return v * g
    if reduction == "none":
        return v * np.asarray(grad_out, dtype=np.float64).reshape(-1)
    raise ValueError(f"Unknown reduction: {reduction!r}")


def backward_full(e, c, lse, targets, d_nll, bias=None):
    """Analytic gradients of reference/_metal_backward.py:245-261 in float64.

    ``targets`` must already be sanitised (in [0, V)).  Returns (dE, dC, dBias).
    """
    t = np.asarray(targets).astype(np.int64)
    z = logits_f64(e, c, bias)
    p = np.exp(z - _f(lse, np.float64)[:, None])
    p[np.arange(z.shape[0]), t] -= 1.0
    dl = _f(d_nll, np.float64)[:, None] * p
    dE = dl @ _f(c, np.float64)
    dC = dl.T @ _f(e, np.float64)
    dB = dl.sum(axis=0) if bias is not None else None
    return dE, dC, dB


def block_keep_mask(z, lse, targets, block_rows, block_cols, log_eps=FILTER_LOG_EPS,
                    row_active=None):
    """Block-skip rule of csrc/cce/cce.metal:190-204 at a given block size.

    A (block_rows x block_cols) block is kept when some row in it has its
    target inside the block's columns, or when the block's maximum logit minus
    that row's LSE is >= ``log_eps``.  ``row_active`` (optional bool [N])
    restricts the decision to rows that carry gradient (rows with a zero
    cotangent contribute nothing either way).  Returns keep[n_row_blocks,
    n_col_blocks].
    """
    n, V = z.shape
    nb = -(-n // block_rows)
    vb = -(-V // block_cols)
    keep = np.zeros((nb, vb), dtype=bool)
    t = np.asarray(targets).astype(np.int64)
    act = np.ones(n, dtype=bool) if row_active is None else np.asarray(row_active, dtype=bool)
    for i in range(nb):
        r0, r1 = i * block_rows, min((i + 1) * block_rows, n)
        rows = np.arange(r0, r1)[act[r0:r1]]
        if rows.size == 0:
            continue
        zz = z[rows] - _f(lse, np.float64)[rows, None]
        for j in range(vb):
            c0, c1 = j * block_cols, min((j + 1) * block_cols, V)
            hit = np.any((t[rows] >= c0) & (t[rows] < c1))
            big = np.any(zz[:, c0:c1].max(axis=1) >= log_eps)
            keep[i, j] = hit or big
    return keep


def backward_filtered(e, c, lse, targets, d_nll, bias=None, block_rows=32, block_cols=32,
                      log_eps=FILTER_LOG_EPS, skip_zero_rows=False):
    """Gradients with skipped blocks dropped (cce.metal:190-204 + :276-304).

    ``skip_zero_rows`` leaves rows with d_nll == 0 out of the keep decision
    (the B200 kernels do; the reference's Metal kernel does not).
    Returns (dE, dC, dBias, skipped_fraction).
    """
    t = np.asarray(targets).astype(np.int64)
    z = logits_f64(e, c, bias)
    act = (np.asarray(d_nll) != 0) if skip_zero_rows else None
    keep = block_keep_mask(z, lse, t, block_rows, block_cols, log_eps, row_active=act)
    p = np.exp(z - _f(lse, np.float64)[:, None])
    p[np.arange(z.shape[0]), t] -= 1.0
    mask = np.repeat(np.repeat(keep, block_rows, axis=0), block_cols, axis=1)[: z.shape[0], : z.shape[1]]
    dl = _f(d_nll, np.float64)[:, None] * p * mask
    dE = dl @ _f(c, np.float64)
    dC = dl.T @ _f(e, np.float64)
    dB = dl.sum(axis=0) if bias is not None else None
    return dE, dC, dB, 1.0 - keep.mean()


def loss_and_grads(e, c, targets, bias=None, reduction="mean", ignore_index=-100, grad_out=None):
    """Full float64 oracle: (loss, lse, dE, dC, dBias) for small shapes."""
    nll, lse, _tgt, valid = dense_forward(e, c, targets, bias, ignore_index)
    loss = reduce(nll, valid, reduction)
    t, _ = sanitize(targets, ignore_index)
    d_nll = d_nll_from_reduction(valid, reduction, grad_out)
    dE, dC, dB = backward_full(e, c, lse, t, d_nll, bias)
    return loss, lse, dE, dC, dB


# ---------------------------------------------------------------------------
# Row / column sampled checks for shapes too large for a dense CPU pass.
# ---------------------------------------------------------------------------

def rows_lse_tgt(e, c, targets, rows, bias=None, chunk=16384):
    """float64 LSE and target logit for a subset of rows (chunked over V)."""
    er = _f(np.asarray(e)[rows], np.float64)
    t = np.asarray(targets).astype(np.int64)[rows]
    V = c.shape[0]
    m = np.full(len(rows), -np.inf)
    s = np.zeros(len(rows))
    for v0 in range(0, V, chunk):
        z = er @ _f(c[v0:v0 + chunk], np.float64).T
        if bias is not None:
            z = z + _f(bias[v0:v0 + chunk], np.float64)[None, :]
        mn = np.maximum(m, z.max(axis=1))
        s = s * np.exp(m - mn) + np.exp(z - mn[:, None]).sum(axis=1)
        m = mn
    lse = m + np.log(s)
    tgt = (er * _f(c[t], np.float64)).sum(axis=1)
    if bias is not None:
        tgt = tgt + _f(bias, np.float64)[t]
    return lse, tgt


def rows_grad_e(e, c, targets, lse_rows, d_nll_rows, rows, bias=None, chunk=16384):
    """dE for a subset of rows: d_nll * (softmax @ c - c[t]) (float64)."""
    er = _f(np.asarray(e)[rows], np.float64)
    t = np.asarray(targets).astype(np.int64)[rows]
    V, D = c.shape
    acc = np.zeros((len(rows), D))
    for v0 in range(0, V, chunk):
        cc = _f(c[v0:v0 + chunk], np.float64)
        z = er @ cc.T
        if bias is not None:
            z = z + _f(bias[v0:v0 + chunk], np.float64)[None, :]
        acc += np.exp(z - np.asarray(lse_rows, np.float64)[:, None]) @ cc
    acc -= _f(c[t], np.float64)
    return acc * np.asarray(d_nll_rows, np.float64)[:, None]


def cols_grad_c(e, c, targets, lse, d_nll, cols, bias=None, chunk=4096):
    """dC (and dBias) for a subset of vocab rows, given the full per-row LSE.

    dC[v] = sum_n d_nll[n] * (exp(z[n,v] - lse[n]) - [t_n == v]) * e[n].
    """
    t = np.asarray(targets).astype(np.int64)
    cc = _f(np.asarray(c)[cols], np.float64)
    n = np.asarray(e).shape[0]
    dC = np.zeros((len(cols), cc.shape[1]))
    dB = np.zeros(len(cols))
    cols = np.asarray(cols)
    for r0 in range(0, n, chunk):
        er = _f(np.asarray(e)[r0:r0 + chunk], np.float64)
        z = er @ cc.T
        if bias is not None:
            z = z + _f(np.asarray(bias)[cols], np.float64)[None, :]
        p = np.exp(z - _f(lse[r0:r0 + chunk], np.float64)[:, None])
        p -= (t[r0:r0 + chunk, None] == cols[None, :]).astype(np.float64)
        dl = p * _f(d_nll[r0:r0 + chunk], np.float64)[:, None]
        dC += dl.T @ er
        dB += dl.sum(axis=0)
    return dC, dB


def rel_max_abs(got, ref):
    """max |got - ref| / max |ref|: the gradient tolerance metric."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.abs(ref).max()
    return float(np.abs(got - ref).max() / (den if den > 0 else 1.0))


def cpu_fwd_bwd_step(e, c, targets, bias=None, reduction="mean", ignore_index=-100,
                     chunk=CHUNK):
    """One forward + backward of the pure-MLX path restated on the CPU in float32.

    Forward: reference/_chunked.py:26-54 (online LSE over vocab chunks of
    4096).  Backward: reference/_metal_backward.py:245-261 (dE, dC and dBias
    from dlogits = d_nll * (softmax - onehot)), evaluated chunk by chunk so
    memory stays O(N * chunk).  Used as the timed CPU baseline; numpy's BLAS
    runs it on all host threads.  Returns (loss, dE, dC, dBias).
    """
    nll, lse, _tgt, valid = chunked_forward(e, c, targets, bias, ignore_index, chunk)
    loss = reduce(nll.astype(np.float64), valid, reduction)
    t, _ = sanitize(targets, ignore_index)
    d = d_nll_from_reduction(valid, reduction).astype(np.float32)
    e32 = _f(e, np.float32)
    c32 = _f(c, np.float32)
    b32 = None if bias is None else _f(bias, np.float32)
    n, D = e32.shape
    V = c32.shape[0]
    dE = np.zeros((n, D), np.float32)
    dC = np.zeros((V, D), np.float32)
    dB = np.zeros((V,), np.float32) if bias is not None else None
    rows = np.arange(n)
    for v0 in range(0, V, chunk):
        v1 = min(v0 + chunk, V)
        z = e32 @ c32[v0:v1].T
        if b32 is not None:
            z += b32[None, v0:v1]
        p = np.exp(z - lse[:, None])
        hit = (t >= v0) & (t < v1)
        p[rows[hit], t[hit] - v0] -= 1.0
        p *= d[:, None]
        dE += p @ c32[v0:v1]
        dC[v0:v1] = p.T @ e32
        if dB is not None:
            dB[v0:v1] = p.sum(axis=0)
    return loss, dE, dC, dB


# ---------------------------------------------------------------------------
# Affine group quantisation of the classifier (see the module docstring).
# ---------------------------------------------------------------------------

def pack_words(q, bits):
    """q int [rows, D] in [0, 2^bits) -> uint32 [rows, D * bits / 32], low bits first."""
    q = np.asarray(q, dtype=np.uint64)
    per = 32 // bits
    rows, D = q.shape
    qq = q.reshape(rows, D // per, per)
    shifts = (np.arange(per, dtype=np.uint64) * bits)[None, None, :]
    return (qq << shifts).sum(axis=2).astype(np.uint32)


def unpack_words(wq, bits):
    """Inverse of pack_words: uint32 [rows, W] -> int64 [rows, W * 32 / bits]."""
    w = np.asarray(wq, dtype=np.uint64)
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint64) * bits)[None, None, :]
    q = (w[:, :, None] >> shifts) & np.uint64((1 << bits) - 1)
    return q.reshape(w.shape[0], -1).astype(np.int64)


def quantize_affine(w, group_size, bits):
    """w [rows, D] -> (wq uint32, scales, biases) with w ~ scales * q + biases per group
    (scale = (max - min) / (2^bits - 1), bias = min, q = round((w - bias) / scale))."""
    w = np.asarray(w, dtype=np.float64)
    rows, D = w.shape
    g = w.reshape(rows, D // group_size, group_size)
    lo, hi = g.min(axis=2), g.max(axis=2)
    scale = (hi - lo) / ((1 << bits) - 1)
    scale = np.where(scale == 0, 1.0, scale)
    q = np.clip(np.rint((g - lo[:, :, None]) / scale[:, :, None]), 0, (1 << bits) - 1).astype(np.int64)
    return pack_words(q.reshape(rows, D), bits), scale, lo


def dequantize_affine(wq, scales, biases, group_size, bits):
    """uint32 [rows, D * bits / 32] + per-group scales / biases -> float64 [rows, D]."""
    q = unpack_words(wq, bits).astype(np.float64)
    s = np.repeat(np.asarray(scales, np.float64), group_size, axis=1)
    b = np.repeat(np.asarray(biases, np.float64), group_size, axis=1)
    return s * q + b
