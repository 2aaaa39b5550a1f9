"""Seeded synthetic inputs for the five benchmark / parity workloads.

No public dataset is involved: these tensors stand in for a language-model
head's hidden states ``e [N, D]``, classifier ``c [V, D]``, optional bias
``[V]`` and targets ``[N]``.  Every tensor is drawn on the CPU from
``torch.Generator().manual_seed(1000 + cfg)`` so that the tests, the benchmark
and the fixture script see identical data on any machine running the same
torch build; callers move them to the GPU themselves.

Workloads (N = flattened tokens):

=== ====== ===== ======= ===== ===================================================
cfg N      D     V       dtype notes
=== ====== ===== ======= ===== ===================================================
1   512    512   32000   f32   e~N(0,1), c~N(0,1/512), 10% ignored, mean
2   1024   2048  128256  bf16  e~N(0,1), c~N(0,.02^2), uniform targets, mean
3   4096   4096  128256  bf16  peaked e = z + 12 c_t/|c_t|^2, Zipf(1.1), 5% ign.
4   2048   2304  256000  bf16  fp32 bias~N(0,.1^2), 25% ignored, 'none'
5   32768  8192  128256  bf16  peaked as 3, Zipf(1.1), 5% ignored, 'sum'
=== ====== ===== ======= ===== ===================================================
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

IGNORE_INDEX = -100


@dataclass(frozen=True)
class Workload:
    cfg: int
    name: str
    batch: tuple          # leading shape of e / targets, e.g. (4, 1024)
    D: int
    V: int
    dtype: torch.dtype
    c_std: float
    targets: str          # "uniform" | "zipf"
    peaked: bool
    ignore_frac: float
    bias_std: float | None
    reduction: str

    @property
    def N(self) -> int:
        n = 1
        for b in self.batch:
            n *= b
        return n

    @property
    def flops(self) -> float:
        """Nominal fwd+bwd work: 2*N*V*D forward plus three times that backward."""
        return 8.0 * self.N * self.V * self.D


WORKLOADS = {
    1: Workload(1, "small-fp32", (2, 256), 512, 32000, torch.float32, 512 ** -0.5,
                "uniform", False, 0.10, None, "mean"),
    2: Workload(2, "llama-3.2-1b-head-uniform", (1024,), 2048, 128256, torch.bfloat16, 0.02,
                "uniform", False, 0.0, None, "mean"),
    3: Workload(3, "llama-3.1-8b-head-peaked", (4, 1024), 4096, 128256, torch.bfloat16, 0.02,
                "zipf", True, 0.05, None, "mean"),
    4: Workload(4, "gemma-2-2b-head-bias-none", (4, 512), 2304, 256000, torch.bfloat16, 0.02,
                "uniform", False, 0.25, 0.1, "none"),
    5: Workload(5, "llama-3-70b-head-sharded", (8, 4096), 8192, 128256, torch.bfloat16, 0.02,
                "zipf", True, 0.05, None, "sum"),
}


def zipf_targets(n: int, V: int, s: float, gen: torch.Generator) -> torch.Tensor:
    """Truncated Zipf over [0, V): P(k) proportional to (k + 1)^-s."""
    w = (torch.arange(V, dtype=torch.float64) + 1.0).pow(-s)
    return torch.multinomial(w, n, replacement=True, generator=gen)


def make_inputs(cfg: int | Workload, *, N: int | None = None, V: int | None = None,
                D: int | None = None, seed: int | None = None):
    """Build (e, c, targets, bias, grad_out, workload) on the CPU.

    ``N``/``V``/``D`` override the workload's sizes (for scaled-down parity
    cases with the same value distributions).  ``grad_out`` is the upstream
    gradient for ``reduction='none'`` workloads (N(0,1) fp32), else None.
    """
    w = WORKLOADS[cfg] if isinstance(cfg, int) else cfg
    n = N if N is not None else w.N
    V_ = V if V is not None else w.V
    D_ = D if D is not None else w.D
    g = torch.Generator(device="cpu")
    g.manual_seed(1000 + w.cfg if seed is None else seed)

    c = torch.randn(V_, D_, generator=g, dtype=torch.float32) * w.c_std
    if w.targets == "zipf":
        t = zipf_targets(n, V_, 1.1, g)
    else:
        t = torch.randint(0, V_, (n,), generator=g, dtype=torch.int64)
    z = torch.randn(n, D_, generator=g, dtype=torch.float32)
    if w.peaked:
        ct = c[t]
        e = z + 12.0 * ct / (ct * ct).sum(dim=1, keepdim=True)
    else:
        e = z
    n_ign = int(round(w.ignore_frac * n))
    if n_ign:
        idx = torch.randperm(n, generator=g)[:n_ign]
        t[idx] = IGNORE_INDEX
    bias = None
    if w.bias_std is not None:
        bias = torch.randn(V_, generator=g, dtype=torch.float32) * w.bias_std
    grad_out = None
    if w.reduction == "none":
        grad_out = torch.randn(n, generator=g, dtype=torch.float32)

    e = e.to(w.dtype)
    c = c.to(w.dtype)
    if N is None and len(w.batch) > 1:
        e = e.reshape(*w.batch, D_)
        t = t.reshape(*w.batch)
        if grad_out is not None:
            grad_out = grad_out.reshape(*w.batch)
    return e, c, t, bias, grad_out, w
