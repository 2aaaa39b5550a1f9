"""Parity of the CTA-pair (cta_group::2) tensor-core engine, selected with
CCE_TC_PAIR=1.  The switch is read once per process, so the checks run in a
child process: forward + backward of bf16 / fp16 cases (with and without bias,
ragged sizes, K-block skipping) against the float64 oracle."""

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parent.parent

CHILD = r"""
import sys
sys.path.insert(0, "{repo}"); sys.path.insert(0, "{repo}/mlx-cross-entropy_b200"); sys.path.insert(0, "{repo}/tests")
import numpy as np, torch
import mlx_cce
from mlx_cce import _ext, synthetic
from oracle import cce_oracle as O
from test_parity_gpu import run, oracle, check, small
cases = [
    small(300, 256, 5000, torch.bfloat16, seed=1, bias=torch.float32, ignore=0.1),
    small(257, 128, 4097, torch.float16, seed=2, ignore=0.1),
    small(513, 64, 2000, torch.bfloat16, seed=3),
]
for e, c, t, b in cases:
    check(run(e, c, t, bias=b), oracle(e, c, t, bias=b), e.dtype)
e, c, t, _, _, _ = synthetic.make_inputs(3, N=512, V=8192, D=512)
check(run(e, c, t, filter_log_eps=-float("inf")), oracle(e, c, t), torch.bfloat16, grad_tol=1e-2)
torch.cuda.synchronize()
_ext.device_status()
print("PAIR_OK")
"""


def test_pair_engine_parity():
    env = dict(os.environ, CCE_TC_PAIR="1")
    res = subprocess.run([sys.executable, "-c", CHILD.format(repo=REPO)], env=env,
                         capture_output=True, text=True, timeout=600)
    assert res.returncode == 0 and "PAIR_OK" in res.stdout, res.stdout[-2000:] + res.stderr[-4000:]
