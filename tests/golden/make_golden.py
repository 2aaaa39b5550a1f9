"""Generate the golden fixtures under tests/golden/ from the CPU oracle.

    python tests/golden/make_golden.py

Inputs are NOT stored: every case is regenerated from a seed by
``mlx_cce.synthetic.make_inputs`` (BASELINE workloads) or by ``ref_inputs``
below (the reference's own test shapes, tests/test_correctness.py:25-30,
regenerated with torch's CPU generator because MLX's RNG is unavailable).
Outputs are the float64 oracle (oracle/cce_oracle.py); large arrays are
stored on a fixed random subset of rows / vocabulary ids.

The reference ships no golden vectors and MLX cannot run here, so these
fixtures pin the restated oracle, not the reference itself (parity unpinned).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "mlx-cross-entropy_b200"))

from oracle import cce_oracle as O  # noqa: E402
from mlx_cce import synthetic  # noqa: E402

N_SAMPLE = 64

# The reference's test shapes (B, D, V): tests/test_correctness.py:25-30 and
# tests/test_gradients.py:36-41; batched (4, 128, 256, 4096): :83.
REF_SHAPES = [(32, 64, 1024), (64, 128, 4096), (128, 256, 32000), (32, 2048, 128256)]


def ref_inputs(B, D, V, seed=42, dtype=torch.float32):
    """e, c ~ N(0, 1), targets ~ U[0, V) (tests/test_correctness.py:11-17)."""
    g = torch.Generator().manual_seed(seed)
    e = torch.randn(B, D, generator=g)
    c = torch.randn(V, D, generator=g)
    t = torch.randint(0, V, (B,), generator=g)
    return e.to(dtype), c.to(dtype), t


def sample_ids(n, k, seed):
    g = np.random.default_rng(seed)
    return np.sort(g.choice(n, size=min(k, n), replace=False))


def f64(t):
    return t.double().numpy() if isinstance(t, torch.Tensor) else np.asarray(t, np.float64)


def full_lse_tgt(e, c, t, bias):
    """float64 LSE and target logit of every row (torch CPU, chunked over V)."""
    e64 = torch.from_numpy(f64(e))
    N = e64.shape[0]
    V = c.shape[0]
    m = torch.full((N,), -float("inf"), dtype=torch.float64)
    s = torch.zeros(N, dtype=torch.float64)
    for v0 in range(0, V, 8192):
        cc = torch.from_numpy(f64(c[v0:v0 + 8192]))
        z = e64 @ cc.T
        if bias is not None:
            z = z + torch.from_numpy(f64(bias[v0:v0 + 8192]))[None, :]
        mn = torch.maximum(m, z.max(dim=1).values)
        s = s * torch.exp(m - mn) + torch.exp(z - mn[:, None]).sum(dim=1)
        m = mn
    lse = (m + torch.log(s)).numpy()
    tt = np.asarray(t)
    tgt = (f64(e) * f64(c[tt])).sum(axis=1)
    if bias is not None:
        tgt = tgt + f64(bias)[tt]
    return lse, tgt


def case(e, c, targets, bias, reduction, ignore_index=-100, grad_out=None, seed=0):
    e2 = e.reshape(-1, e.shape[-1])
    tflat = targets.reshape(-1).numpy()
    safe, valid = O.sanitize(tflat, ignore_index)
    lse, tgt = full_lse_tgt(e2, c, safe, bias)
    nll = lse - tgt
    loss = O.reduce(nll, valid, reduction)
    d_nll = O.d_nll_from_reduction(valid, reduction,
                                   None if grad_out is None else grad_out.reshape(-1).numpy())
    N, D = e2.shape
    V = c.shape[0]
    k = N_SAMPLE if D <= 1024 else 16
    rows = sample_ids(N, k, seed + 1)
    cols = sample_ids(V, k, seed + 2)
    # always include a few target ids among the sampled vocabulary rows
    tgt_cols = np.unique(safe[valid])[:8] if valid.any() else np.array([], dtype=np.int64)
    cols = np.unique(np.concatenate([cols, tgt_cols])).astype(np.int64)
    e64 = f64(e2)
    c64 = f64(c)
    b64 = None if bias is None else f64(bias)
    dE_rows = O.rows_grad_e(e64, c64, safe, lse[rows], d_nll[rows], rows, bias=b64)
    dC_cols, dB_cols = O.cols_grad_c(e64, c64, safe, lse, d_nll, cols, bias=b64)
    out = dict(loss=np.asarray(loss, np.float64), lse=lse, tgt=tgt, nll=nll * valid,
               rows=rows, cols=cols, dE_rows=dE_rows.astype(np.float32),
               dC_cols=dC_cols.astype(np.float32))
    if bias is not None:
        out["dB_cols"] = dB_cols
    return out


def main():
    torch.set_num_threads(max(1, torch.get_num_threads()))
    out_dir = HERE
    # reference test shapes, fp32 and bf16, mean reduction
    for (B, D, V) in REF_SHAPES:
        for name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
            e, c, t = ref_inputs(B, D, V, dtype=dt)
            res = case(e, c, t, None, "mean", seed=B + D + V)
            np.savez_compressed(out_dir / f"ref_{B}x{D}x{V}_{name}.npz", **res)
            print("ref", B, D, V, name, float(res["loss"]))
    # BASELINE workloads 1-4 (5 is checked through properties on the GPU)
    for cfg in (1, 2, 3, 4):
        e, c, t, bias, grad_out, w = synthetic.make_inputs(cfg)
        res = case(e, c, t, bias, w.reduction, grad_out=grad_out, seed=100 * cfg)
        np.savez_compressed(out_dir / f"cfg{cfg}.npz", **res)
        print("cfg", cfg, w.name, float(np.sum(res["loss"])))


if __name__ == "__main__":
    main()
