"""cce_forward_noalloc: the forward for callers that cannot allocate device memory.

Some hosts can hand the loss its inputs and outputs but have no device
allocator to offer for a workspace (a plugin or FFI slot with a fixed memory
contract, or a runtime that forbids allocation while it executes).  For them
cce_forward_noalloc keeps its scratch in a static 32 MiB array inside the
library.  These tests call it through the C ABI twice in a row -- the second
call smaller than the first, so the shared array still holds the first call's
partials -- and check each result against cce_forward with a caller-owned
workspace, within the tests' 16-bit loss tolerance: once on the tensor-core
path (bf16) and once on the CUDA-core path (float32) at nearly the array's
full capacity.  It also checks that a call
beyond the array's capacity is refused with a clear error.

The file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from mlx_cce import _ext

pytestmark = pytest.mark.gpu

RTOL = 1e-3  # the 16-bit loss tolerance used by tests/test_parity_gpu.py
CAPACITY = 8 << 20  # floats in the static array: 2 * ceil(V / 128) * N may not exceed it


def _inputs(N, D, V, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda", 0)
    e = torch.randn(N, D, generator=g).to(dtype).to(dev)
    c = (torch.randn(V, D, generator=g) * D ** -0.5).to(dtype).to(dev)
    t = torch.randint(0, V, (N,), generator=g, dtype=torch.int32).to(dev)
    return e, c, t


def _noalloc(e, c, t):
    N, D = e.shape
    V = c.shape[0]
    dev = e.device
    tile_max = torch.empty((_ext.num_stat_tiles(V), N), dtype=torch.float32, device=dev)
    lse = torch.empty(N, dtype=torch.float32, device=dev)
    tgt = torch.empty(N, dtype=torch.float32, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = _ext.lib.cce_forward_noalloc(
        ctypes.c_void_p(e.data_ptr()), ctypes.c_void_p(c.data_ptr()), None, 0,
        ctypes.c_void_p(t.data_ptr()), N, D, V, 0, _ext.dtype_code(e.dtype, "test"),
        ctypes.c_void_p(tile_max.data_ptr()), ctypes.c_void_p(lse.data_ptr()),
        ctypes.c_void_p(tgt.data_ptr()), stream)
    assert rc == _ext.CCE_OK, _ext.lib.cce_last_error().decode()
    return tile_max, lse, tgt


def _compare(N, D, V, seed, dtype):
    e, c, t = _inputs(N, D, V, seed, dtype)
    tm_a, lse_a, tgt_a = _noalloc(e, c, t)
    tm_b, lse_b, tgt_b = _ext.forward(e, c, t)
    torch.cuda.synchronize()
    np.testing.assert_allclose(lse_a.cpu().numpy(), lse_b.cpu().numpy(), rtol=RTOL)
    np.testing.assert_allclose(tgt_a.cpu().numpy(), tgt_b.cpu().numpy(), rtol=RTOL, atol=1e-4)
    np.testing.assert_allclose(tm_a.cpu().numpy(), tm_b.cpu().numpy(), rtol=RTOL, atol=1e-4)


def test_noalloc_forward_matches_workspace_forward_twice():
    # first a large call (fills most of the static array), then a smaller one
    for (N, D, V, seed) in ((4096, 512, 128256, 1), (200, 256, 5000, 2)):
        _compare(N, D, V, seed, torch.bfloat16)


def test_noalloc_float32_fills_the_whole_array_then_a_small_call():
    # float32 runs on the CUDA-core kernels, whose LSE partials are 128 columns
    # wide: 2 * ceil(32000 / 128) * 16000 = 8,000,000 of the 8,388,608 floats,
    # the layout the capacity is sized for.  Then a small call reuses the array.
    N, D, V = 16000, 64, 32000
    assert 2 * -(-V // 128) * N <= CAPACITY
    assert 2 * -(-V // 128) * N > 0.95 * CAPACITY
    _compare(N, D, V, 3, torch.float32)
    _compare(300, 64, 1000, 4, torch.float32)


def test_noalloc_rejects_calls_beyond_its_capacity():
    # 2 * ceil(V / 128) * N above 8388608 partials: refused before any GPU work
    rc = _ext.lib.cce_forward_noalloc(None, None, None, 0, None, 4186, 4096, 128256, 0,
                                      _ext.CCE_BF16, None, None, None, None)
    assert rc == _ext.CCE_ERR_WORKSPACE
    assert b"static scratch" in _ext.lib.cce_last_error()
