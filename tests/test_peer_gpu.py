"""The grad_e exchange of the vocabulary-sharded backward, on one GPU.

``cce_backward_peer`` sums grad_e over a group of ranks through their exchange
buffers: the last grad_e GEMM stores its tiles into the owning rank's buffer,
the owner reduces its rows and every rank copies the others' rows back.  The
2-GPU test (test_dist_gpu.py) runs it across real ranks; here one GPU covers
what one process can:

* a group of one rank: the push epilogue (tensor-core path, one and several
  vocabulary chunks, with the chunk accumulation added in), the push kernel of
  the CUDA-core path, the reduce and its dtype conversion, against the float64
  oracle and against the plain backward;
* a group of two ranks whose second rank never arrives: every wait on it runs
  out after the group's (short) limit, cce_device_status reports the exchange
  code, and the context keeps computing correctly afterwards.  No fault, trap
  or hang is involved: the waits are bounded.
"""

import ctypes
import os

import numpy as np
import pytest
import torch

import mlx_cce
from mlx_cce import _ext
from oracle import cce_oracle as O

pytestmark = pytest.mark.gpu

GRAD_TOL = 2e-2


class Buffer:
    """One exchange buffer from cce_peer_buffer_alloc, freed on close()."""

    def __init__(self, nbytes):
        ptr, fd = ctypes.c_void_p(), ctypes.c_int(-1)
        _ext._check(_ext.lib.cce_peer_buffer_alloc(nbytes, ctypes.byref(ptr), ctypes.byref(fd)), "alloc")
        os.close(fd.value)   # no other process maps it
        self.ptr, self.nbytes = ptr.value, nbytes

    def close(self):
        torch.cuda.synchronize()
        _ext._check(_ext.lib.cce_peer_buffer_free(self.ptr), "free")


def group(buf, world=1, rank=0, wait_ms=10_000):
    g = _ext.CcePeerGroup()
    g.rank, g.world = rank, world
    g.wait_limit_ns = int(wait_ms * 1e6)
    g.bytes = buf.nbytes
    for r in range(world):
        g.bases[r] = buf.ptr   # an emulated peer shares this rank's buffer
    return g


def inputs(N, D, V, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    e = torch.randn(N, D, generator=gen).to(dtype)
    c = (torch.randn(V, D, generator=gen) * D ** -0.5).to(dtype)
    t = torch.randint(0, V, (N,), generator=gen)
    t[::7] = -100
    return e, c, t


def raw_backward(e, c, t, peer_group=None, grad_e_f32=False):
    dev = torch.device("cuda", 0)
    ed, cd = e.to(dev), c.to(dev)
    safe, valid = mlx_cce._autograd.sanitize_targets(t.to(dev), -100)
    tm, lse, tgt = _ext.forward(ed, cd, safe)
    d_nll = (valid.float() / valid.sum()).contiguous()
    ge, gc, _ = _ext.backward(ed, cd, safe, lse, d_nll, tm, need_c=True, grad_e_f32=grad_e_f32,
                              peer_group=peer_group)
    torch.cuda.synchronize()
    return ge, gc


@pytest.mark.parametrize("N,D,V,dtype", [
    (640, 256, 5000, torch.bfloat16),      # tensor cores, one vocabulary chunk
    (8300, 64, 20000, torch.bfloat16),     # two chunks: the push adds chunk 0's slabs
    (300, 96, 3000, torch.float16),        # fp16 (scaled dlogits)
    (200, 100, 2000, torch.float32),       # CUDA-core path: push kernel
])
def test_group_of_one_matches_oracle_and_plain_backward(N, D, V, dtype, monkeypatch):
    monkeypatch.setenv("CCE_BWD_CHUNK_ROWS", "16384")   # N = 8300, V = 20000: two chunks
    e, c, t = inputs(N, D, V, dtype, seed=N + V)
    out_dtype = dtype
    buf = Buffer(_ext.lib.cce_peer_buffer_bytes(N, D, 1, _ext.dtype_code(out_dtype, "t")))
    try:
        g = group(buf)
        ge_p, gc_p = raw_backward(e, c, t, peer_group=g)
        ge_p2, _ = raw_backward(e, c, t, peer_group=g)   # a second exchange on the same buffer
        ge, gc = raw_backward(e, c, t)
        _ext.device_status()
    finally:
        buf.close()
    assert ge_p.dtype == dtype and ge_p.shape == (N, D)
    np.testing.assert_array_equal(ge_p.float().cpu().numpy(), ge_p2.float().cpu().numpy())
    ref = O.loss_and_grads(e.double().numpy(), c.double().numpy(), t.numpy(), None, "mean")
    assert O.rel_max_abs(ge_p.double().cpu().numpy(), ref[2]) < GRAD_TOL
    assert O.rel_max_abs(ge_p.double().cpu().numpy(), ge.double().cpu().numpy()) < 1e-2
    np.testing.assert_array_equal(gc_p.float().cpu().numpy(), gc.float().cpu().numpy())


def test_exchange_fp32_output():
    """CCE_DE_F32 with the exchange: the summed grad_e comes back in fp32."""
    e, c, t = inputs(384, 128, 4000, torch.bfloat16, seed=5)
    buf = Buffer(_ext.lib.cce_peer_buffer_bytes(384, 128, 1, _ext.CCE_F32))
    try:
        ge_p, _ = raw_backward(e, c, t, peer_group=group(buf), grad_e_f32=True)
    finally:
        buf.close()
    assert ge_p.dtype == torch.float32
    ref = O.loss_and_grads(e.double().numpy(), c.double().numpy(), t.numpy(), None, "mean")
    assert O.rel_max_abs(ge_p.double().cpu().numpy(), ref[2]) < GRAD_TOL


def test_buffer_too_small_is_refused():
    e, c, t = inputs(256, 64, 1000, torch.bfloat16, seed=6)
    need = _ext.lib.cce_peer_buffer_bytes(256, 64, 2, _ext.CCE_BF16)
    buf = Buffer(need // 2)
    try:
        with pytest.raises(RuntimeError, match="exchange buffers"):
            raw_backward(e, c, t, peer_group=group(buf, world=2))
    finally:
        buf.close()


def test_missing_rank_times_out_and_the_context_survives():
    N, D, V = 512, 128, 3000
    e, c, t = inputs(N, D, V, torch.bfloat16, seed=7)
    buf = Buffer(_ext.lib.cce_peer_buffer_bytes(N, D, 2, _ext.CCE_BF16))
    try:
        _ext.device_status(reset=True)
        raw_backward(e, c, t, peer_group=group(buf, world=2, rank=0, wait_ms=50))
        with pytest.raises(RuntimeError, match=f"code {_ext.CCE_PEER_WAIT_PUSH}"):
            _ext.device_status()
        with pytest.raises(RuntimeError, match=f"code {_ext.CCE_PEER_WAIT_PUSH}"):
            _ext.device_status(reset=True)   # reports, then clears
        _ext.device_status()
    finally:
        buf.close()
    ge, _ = raw_backward(e, c, t)
    ref = O.loss_and_grads(e.double().numpy(), c.double().numpy(), t.numpy(), None, "mean")
    assert O.rel_max_abs(ge.double().cpu().numpy(), ref[2]) < GRAD_TOL
