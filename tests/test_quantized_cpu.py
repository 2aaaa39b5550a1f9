"""CPU tests of the quantised-classifier path: the oracle's packing, the C ABI's
argument checks (no kernel runs) and the Python API's validation."""

import numpy as np
import pytest
import torch

import mlx_cce
from mlx_cce import _ext
from oracle import cce_oracle as O


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_pack_unpack_roundtrip(bits):
    rng = np.random.default_rng(bits)
    q = rng.integers(0, 1 << bits, (6, 256))
    wq = O.pack_words(q, bits)
    assert wq.dtype == np.uint32 and wq.shape == (6, 256 * bits // 32)
    assert np.array_equal(O.unpack_words(wq, bits), q)
    # value j sits in bits [(j * bits) % 32, +bits) of word (j * bits) // 32
    j = 37
    assert (int(wq[0, j * bits // 32]) >> ((j * bits) % 32)) & ((1 << bits) - 1) == q[0, j]


@pytest.mark.parametrize("bits,group", [(4, 64), (8, 32), (2, 128)])
def test_quantize_dequantize_error_bound(bits, group):
    rng = np.random.default_rng(0)
    w = rng.normal(size=(9, 512))
    wq, s, b = O.quantize_affine(w, group, bits)
    r = O.dequantize_affine(wq, s, b, group, bits)
    assert np.all(np.abs(r - w) <= np.repeat(s, group, axis=1) / 2 + 1e-12)


def test_dequantize_abi_rejects_bad_arguments_without_gpu_work():
    lib = _ext.lib
    assert lib.cce_dequantize(None, None, None, 0, 4, 64, 64, 3, 2, None, None) == _ext.CCE_ERR_ARG
    assert b"bits" in lib.cce_last_error()
    assert lib.cce_dequantize(None, None, None, 0, 4, 64, 48, 4, 2, None, None) == _ext.CCE_ERR_ARG
    assert lib.cce_dequantize(None, None, None, 0, 4, 96, 64, 4, 2, None, None) == _ext.CCE_ERR_SHAPE
    assert lib.cce_dequantize(None, None, None, 9, 4, 64, 64, 4, 2, None, None) == _ext.CCE_ERR_DTYPE
    assert lib.cce_dequantize(None, None, None, 0, 0, 64, 64, 4, 2, None, None) == _ext.CCE_OK


def test_quantized_api_validation():
    wq = torch.zeros(10, 8, dtype=torch.int32)      # D = 8 * 32 / 4 = 64
    s = torch.ones(10, 1)
    q = mlx_cce.QuantizedClassifier(wq, s, s, 64, 4)
    assert q.shape == (10, 64)
    e = torch.randn(3, 64)
    t = torch.tensor([1, 2, 3])
    with pytest.raises(ValueError, match="Unknown reduction"):
        mlx_cce.linear_cross_entropy_quantized(e, q, t, reduction="avg")
    with pytest.raises(ValueError, match="QuantizedClassifier"):
        mlx_cce.linear_cross_entropy_quantized(e, torch.randn(10, 64), t)
    with pytest.raises(ValueError, match="must equal"):
        mlx_cce.linear_cross_entropy_quantized(torch.randn(3, 32), q, t)
    with pytest.raises(ValueError, match="CUDA tensor"):
        _ext.dequantize(wq, s, s, 64, 4, torch.bfloat16)


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("group_size", [32, 64, 128])
def test_torch_quantize_matches_the_oracle_format(bits, group_size):
    """mlx_cce.quantized.quantize (runs on any torch device) packs the same
    words, scales and biases as the oracle's restatement of MLX's affine format."""
    from mlx_cce.quantized import quantize
    w = torch.randn(48, 256, generator=torch.Generator().manual_seed(bits * group_size))
    w[3, :group_size] = 0.25   # a constant group: scale 1
    q = quantize(w, group_size, bits)
    wq, scales, biases = O.quantize_affine(w.numpy(), group_size, bits)
    assert q.weight.dtype == torch.int32
    np.testing.assert_array_equal(q.weight.numpy().view(np.uint32), wq)
    np.testing.assert_allclose(q.scales.numpy(), scales, rtol=1e-6)
    np.testing.assert_allclose(q.biases.numpy(), biases, rtol=1e-6)
