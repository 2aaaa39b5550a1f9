"""The quantised-classifier path on a B200: the dequantisation kernel against
the oracle's definition, and linear_cross_entropy_quantized against (a) the
dense path on the same dequantised head and (b) the float64 oracle."""

import numpy as np
import pytest
import torch

import mlx_cce
from mlx_cce import _ext
from oracle import cce_oracle as O

pytestmark = pytest.mark.gpu

GRAD_TOL = 2e-2


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def _quantized(V, D, group, bits, scale_dtype, seed=0):
    rng = np.random.default_rng(seed)
    w = rng.normal(scale=D ** -0.5, size=(V, D))
    wq, s, b = O.quantize_affine(w, group, bits)
    dev = _dev()
    q = mlx_cce.QuantizedClassifier(torch.from_numpy(wq.view(np.int32)).to(dev),
                                    torch.from_numpy(s).to(scale_dtype).to(dev),
                                    torch.from_numpy(b).to(scale_dtype).to(dev), group, bits)
    return q, wq


@pytest.mark.parametrize("bits,group", [(4, 64), (8, 32), (2, 128)])
@pytest.mark.parametrize("scale_dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_dequantize_kernel_matches_oracle(bits, group, scale_dtype, out_dtype):
    q, wq = _quantized(300, 256, group, bits, scale_dtype, seed=bits)
    got = q.dequantize(out_dtype).float().cpu().numpy()
    ref = O.dequantize_affine(wq, q.scales.float().cpu().numpy(), q.biases.float().cpu().numpy(),
                              group, bits)
    tol = {torch.float32: 1e-6, torch.bfloat16: 2 ** -8, torch.float16: 2 ** -11}[out_dtype]
    assert np.all(np.abs(got - ref) <= tol * np.abs(ref) + 1e-6)
    # a row range is the same rows of the whole
    part = q.dequantize(out_dtype, 100, 220).float().cpu().numpy()
    assert np.array_equal(part, got[100:220])


@pytest.mark.parametrize("reduction", ["mean", "none"])
def test_quantized_cce_matches_dense_and_oracle(reduction, monkeypatch):
    # backward chunks of 1024 rows: five, the last one ragged; the library
    # expands each into one of its two chunk buffers while the previous runs
    monkeypatch.setenv("CCE_BWD_CHUNK_ROWS", "1024")
    dev = _dev()
    N, D, V = 300, 256, 5000
    q, wq = _quantized(V, D, 64, 4, torch.bfloat16, seed=7)
    g = torch.Generator().manual_seed(8)
    e = torch.randn(N, D, generator=g).to(torch.bfloat16)
    bias = (torch.randn(V, generator=g) * 0.3)
    t = torch.randint(0, V, (N,), generator=g)
    t[::10] = -100
    go = torch.randn(N, generator=g) if reduction == "none" else None

    def run(fn, c):
        e_ = e.to(dev).requires_grad_(True)
        b_ = bias.to(dev).requires_grad_(True)
        loss = fn(e_, c, t.to(dev), bias=b_, reduction=reduction)
        loss.backward(go.to(dev) if go is not None else None)
        torch.cuda.synchronize()
        return (loss.detach().double().cpu().numpy(), e_.grad.double().cpu().numpy(),
                b_.grad.double().cpu().numpy())

    lq, eq, bq = run(mlx_cce.linear_cross_entropy_quantized, q)
    c_dense = q.dequantize(torch.bfloat16)
    ld, ed, bd = run(mlx_cce.linear_cross_entropy, c_dense)
    np.testing.assert_allclose(lq, ld, rtol=1e-5, atol=1e-6)
    assert O.rel_max_abs(eq, ed) < 1e-2
    assert O.rel_max_abs(bq, bd) < 1e-2
    # float64 oracle on the same (bf16-rounded) head
    loss, _lse, dE, _dC, dB = O.loss_and_grads(e.double().numpy(), c_dense.double().cpu().numpy(),
                                               t.numpy(), bias.double().numpy(), reduction=reduction,
                                               grad_out=None if go is None else go.double().numpy())
    np.testing.assert_allclose(lq.reshape(-1), np.asarray(loss).reshape(-1), rtol=1e-3, atol=1e-6)
    assert O.rel_max_abs(eq, dE) < GRAD_TOL
    assert O.rel_max_abs(bq, dB) < GRAD_TOL


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_quantized_head_several_forward_chunks(dtype, monkeypatch):
    """V = 40000 spans two 32768-row forward chunks (the last one ragged)
    and five 8192-row backward chunks; bf16 runs on the tensor cores, float32
    on the CUDA cores.  Against the dense path on the same dequantised head."""
    monkeypatch.setenv("CCE_BWD_CHUNK_ROWS", "8192")
    dev = _dev()
    N, D, V = 256, 128, 40000
    q, _wq = _quantized(V, D, 32, 8, torch.float16, seed=9)
    g = torch.Generator().manual_seed(10)
    e = torch.randn(N, D, generator=g).to(dtype)
    t = torch.randint(0, V, (N,), generator=g)
    t[::9] = -100
    t[1] = V - 1

    def run(fn, c):
        e_ = e.to(dev).requires_grad_(True)
        loss, lse = fn(e_, c, t.to(dev), reduction="sum", return_lse=True)
        loss.backward()
        torch.cuda.synchronize()
        return loss.item(), lse.double().cpu().numpy(), e_.grad.double().cpu().numpy()

    lq, lseq, eq = run(mlx_cce.linear_cross_entropy_quantized, q)
    ld, lsed, ed = run(mlx_cce.linear_cross_entropy, q.dequantize(dtype))
    np.testing.assert_allclose(lq, ld, rtol=1e-5)
    np.testing.assert_allclose(lseq, lsed, rtol=1e-5)
    assert O.rel_max_abs(eq, ed) < 1e-2
