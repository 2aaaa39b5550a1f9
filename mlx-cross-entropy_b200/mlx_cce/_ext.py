"""ctypes binding of ``libcce_b200.so`` (the C ABI declared in include/cce_b200.h).

This module is the torch-facing replacement of the reference's nanobind module
``mlx_cce._ext`` (csrc/bindings.cpp:12-87).  It keeps that module's three entry
points with the same argument meaning -- ``cut_cross_entropy``,
``cce_forward_raw`` and ``cce_backward_raw`` -- and adds the lower-level calls
the autograd function and the vocabulary-sharded wrapper use.

There is no CPU or eager-PyTorch fallback: if the shared library is missing
the import fails, and every call demands CUDA tensors on an sm_100 device.
Library status codes become ``ValueError`` (shape / dtype / argument errors)
or ``RuntimeError`` (CUDA / architecture / workspace errors), as the
reference's C++ exceptions become Python exceptions through nanobind.
"""

from __future__ import annotations

import contextlib
import ctypes
import math
import os
from pathlib import Path

import torch

# CCE_LIB_PATH may point at another build of the same library (A/B timing).
_LIB_PATH = Path(os.environ.get("CCE_LIB_PATH") or Path(__file__).resolve().parent / "libcce_b200.so")

CCE_OK = 0
CCE_ERR_SHAPE = -1
CCE_ERR_DTYPE = -2
CCE_ERR_ALIGN = -3
CCE_ERR_CUDA = -4
CCE_ERR_ARCH = -5
CCE_ERR_WORKSPACE = -6
CCE_ERR_ARG = -7

CCE_F32, CCE_F16, CCE_BF16 = 0, 1, 2
CCE_STAT_TILE = 32

CCE_NEED_DE = 1
CCE_NEED_DC = 2
CCE_NEED_DBIAS = 4
CCE_DE_F32 = 8
CCE_NO_FILTER = 16

# ln(2^-12), csrc/cce/cce.metal:143 of the reference.
FILTER_LOG_EPS = math.log(2.0 ** -12)

CCE_PEER_MAX_WORLD = 16
CCE_PEER_WAIT_PUSH = 201
CCE_PEER_WAIT_REDUCE = 202

EXPORTED_SYMBOLS = (
    "cce_version", "cce_last_error", "cce_launch_count", "cce_device_status", "cce_num_stat_tiles",
    "cce_forward_workspace_bytes", "cce_forward", "cce_forward_noalloc", "cce_lse_combine",
    "cce_backward_workspace_bytes", "cce_backward", "cce_dequantize", "cce_selftest_wait_timeout",
    "cce_peer_buffer_bytes", "cce_peer_buffer_alloc", "cce_peer_buffer_open", "cce_peer_buffer_close",
    "cce_peer_buffer_free", "cce_backward_peer", "cce_mma_flops",
    "cce_forward_q_workspace_bytes", "cce_forward_q", "cce_backward_q_workspace_bytes", "cce_backward_q",
)


class CceQuantHead(ctypes.Structure):
    """Mirror of ``CceQuantHead`` (include/cce_b200.h)."""
    _fields_ = [("wq", ctypes.c_void_p), ("scales", ctypes.c_void_p), ("biases", ctypes.c_void_p),
                ("scale_dtype", ctypes.c_int32), ("group_size", ctypes.c_int32), ("bits", ctypes.c_int32)]


class CcePeerGroup(ctypes.Structure):
    """Mirror of ``CcePeerGroup`` (include/cce_b200.h)."""
    _fields_ = [("rank", ctypes.c_int32), ("world", ctypes.c_int32), ("wait_limit_ns", ctypes.c_int64),
                ("bytes", ctypes.c_size_t), ("bases", ctypes.c_void_p * CCE_PEER_MAX_WORLD)]

_DTYPE_CODE = {torch.float32: CCE_F32, torch.float16: CCE_F16, torch.bfloat16: CCE_BF16}


def _load():
    if not _LIB_PATH.exists():
        raise ImportError(
            f"{_LIB_PATH} is missing: build it with `python mlx-cross-entropy_b200/mlx_cce/build.py` "
            "(there is no fallback implementation)")
    lib = ctypes.CDLL(str(_LIB_PATH))
    c_i64, c_int, c_vp, c_sz, c_f = (ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
                                      ctypes.c_size_t, ctypes.c_float)
    lib.cce_version.restype = c_int
    lib.cce_version.argtypes = []
    lib.cce_last_error.restype = ctypes.c_char_p
    lib.cce_last_error.argtypes = []
    lib.cce_launch_count.restype = ctypes.c_uint64
    lib.cce_launch_count.argtypes = []
    lib.cce_device_status.restype = c_int
    lib.cce_device_status.argtypes = [c_int]
    lib.cce_num_stat_tiles.restype = c_i64
    lib.cce_num_stat_tiles.argtypes = [c_i64]
    lib.cce_forward_workspace_bytes.restype = c_sz
    lib.cce_forward_workspace_bytes.argtypes = [c_i64, c_i64, c_i64, c_int]
    lib.cce_forward.restype = c_int
    lib.cce_forward.argtypes = [c_vp, c_vp, c_vp, c_int, c_vp, c_i64, c_i64, c_i64, c_i64, c_int,
                                c_vp, c_vp, c_vp, c_vp, c_sz, c_vp]
    lib.cce_forward_noalloc.restype = c_int
    lib.cce_forward_noalloc.argtypes = [c_vp, c_vp, c_vp, c_int, c_vp, c_i64, c_i64, c_i64, c_i64,
                                        c_int, c_vp, c_vp, c_vp, c_vp]
    lib.cce_lse_combine.restype = c_int
    lib.cce_lse_combine.argtypes = [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp]
    lib.cce_backward_workspace_bytes.restype = c_sz
    lib.cce_backward_workspace_bytes.argtypes = [c_i64, c_i64, c_i64, c_int, c_int]
    lib.cce_backward.restype = c_int
    lib.cce_backward.argtypes = [c_vp, c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64,
                                 c_i64, c_i64, c_int, c_int, c_f, c_vp, c_vp, c_vp, c_vp, c_vp,
                                 c_sz, c_vp]
    lib.cce_selftest_wait_timeout.restype = c_int
    lib.cce_selftest_wait_timeout.argtypes = [c_i64, c_vp]
    lib.cce_dequantize.restype = c_int
    lib.cce_dequantize.argtypes = [c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_int, c_int, c_int, c_vp, c_vp]
    lib.cce_peer_buffer_bytes.restype = c_sz
    lib.cce_peer_buffer_bytes.argtypes = [c_i64, c_i64, c_int, c_int]
    lib.cce_peer_buffer_alloc.restype = c_int
    lib.cce_peer_buffer_alloc.argtypes = [c_sz, ctypes.POINTER(c_vp), ctypes.POINTER(c_int)]
    lib.cce_peer_buffer_open.restype = c_int
    lib.cce_peer_buffer_open.argtypes = [c_int, c_sz, ctypes.POINTER(c_vp)]
    lib.cce_peer_buffer_close.restype = c_int
    lib.cce_peer_buffer_close.argtypes = [c_vp]
    lib.cce_peer_buffer_free.restype = c_int
    lib.cce_peer_buffer_free.argtypes = [c_vp]
    lib.cce_forward_q_workspace_bytes.restype = c_sz
    lib.cce_forward_q_workspace_bytes.argtypes = [c_i64, c_i64, c_i64, c_int]
    lib.cce_forward_q.restype = c_int
    lib.cce_forward_q.argtypes = [c_vp, ctypes.POINTER(CceQuantHead), c_vp, c_int, c_vp, c_i64, c_i64, c_i64,
                                  c_i64, c_int, c_vp, c_vp, c_vp, c_vp, c_sz, c_vp]
    lib.cce_backward_q_workspace_bytes.restype = c_sz
    lib.cce_backward_q_workspace_bytes.argtypes = [c_i64, c_i64, c_i64, c_int, c_int]
    lib.cce_backward_q.restype = c_int
    lib.cce_backward_q.argtypes = [c_vp, ctypes.POINTER(CceQuantHead), c_vp, c_int, c_vp, c_vp, c_vp, c_vp,
                                   c_i64, c_i64, c_i64, c_i64, c_int, c_int, c_f, c_vp, c_vp, c_vp, c_vp, c_sz,
                                   c_vp]
    lib.cce_mma_flops.restype = c_int
    lib.cce_mma_flops.argtypes = [ctypes.POINTER(ctypes.c_uint64), c_int]
    lib.cce_backward_peer.restype = c_int
    lib.cce_backward_peer.argtypes = [c_vp, c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64,
                                      c_i64, c_i64, c_int, c_int, c_f, c_vp, c_vp, c_vp, c_vp, c_vp,
                                      c_sz, ctypes.POINTER(CcePeerGroup), c_vp]
    return lib


lib = _load()


def version() -> int:
    return lib.cce_version()


def device_status(reset: bool = False):
    """Raise RuntimeError if a kernel abandoned a pipeline wait (synchronous)."""
    _check(lib.cce_device_status(1 if reset else 0), "cce_device_status")


def mma_flops(reset: bool = False):
    """Executed tensor-core FLOPs since the last reset (synchronous):
    {"forward", "dlogits", "grad_e", "grad_c"} -> FLOPs."""
    out = (ctypes.c_uint64 * 4)()
    _check(lib.cce_mma_flops(out, 1 if reset else 0), "cce_mma_flops")
    return dict(zip(("forward", "dlogits", "grad_e", "grad_c"), (int(x) for x in out)))


def launch_count() -> int:
    """Kernels launched by the library in this process so far."""
    return int(lib.cce_launch_count())


# Optional CUDA-event timing of the C-ABI calls (off by default; used by the
# benchmark to time the forward / backward kernels on their own stream).
_timing = None


def set_timing(enabled: bool):
    """Start (True) or stop (False) recording (name, start, end) CUDA events."""
    global _timing
    _timing = [] if enabled else None


def timings():
    """Recorded (name, start_event, end_event) triples since set_timing(True)."""
    return list(_timing or [])


class _Timed:
    def __init__(self, name, stream):
        self.name, self.stream = name, stream

    def __enter__(self):
        if _timing is not None:
            self.ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            self.ev[0].record(self.stream)
        return self

    def __exit__(self, *exc):
        if _timing is not None:
            self.ev[1].record(self.stream)
            _timing.append((self.name, self.ev[0], self.ev[1]))
        return False


def _torch_stream(stream):
    if stream is None:
        return torch.cuda.current_stream()
    if isinstance(stream, torch.cuda.Stream):
        return stream
    return torch.cuda.ExternalStream(int(stream))


def _check(rc: int, what: str):
    if rc == CCE_OK:
        return
    msg = lib.cce_last_error().decode(errors="replace")
    if rc in (CCE_ERR_SHAPE, CCE_ERR_DTYPE, CCE_ERR_ARG, CCE_ERR_ALIGN):
        raise ValueError(f"[{what}] {msg}")
    raise RuntimeError(f"[{what}] {msg} (status {rc})")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _alloc_on(stream):
    """Context in which outputs and workspaces for a call on ``stream`` are allocated.

    The caching allocator ties a block to the stream that allocated it: a
    workspace freed when the call returns may be handed to the next
    allocation on that same stream only.  Allocating on the launch stream
    (not torch's current stream) keeps a kernel still running there from
    sharing its memory with work on another stream.
    """
    if stream is None:
        return contextlib.nullcontext()
    return torch.cuda.stream(_torch_stream(stream))


def _stream(stream=None):
    if stream is None:
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, torch.cuda.Stream):
        return ctypes.c_void_p(stream.cuda_stream)
    return ctypes.c_void_p(int(stream))


def dtype_code(dt: torch.dtype, what: str) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise ValueError(f"[{what}] unsupported dtype {dt}; expected float32, float16 or bfloat16")


def _require_cuda(what: str, **tensors):
    dev = None
    for name, t in tensors.items():
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError(f"[{what}] {name} must be a CUDA tensor (no CPU implementation exists)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"[{what}] {name} is on {t.device}, expected {dev}")
        if not t.is_contiguous():
            raise ValueError(f"[{what}] {name} must be contiguous")
    return dev


def num_stat_tiles(V: int) -> int:
    return int(lib.cce_num_stat_tiles(V))


def forward(e, c, targets, bias=None, v_offset: int = 0, stream=None):
    """Raw fused forward over this call's vocabulary rows.

    e [N, D], c [V, D] (same 16/32-bit float dtype), targets int32 [N]
    (sanitised global ids), bias [V] or None.
    Returns (tile_max [nVt, N] fp32, lse [N] fp32, tgt [N] fp32).
    """
    what = "cce_forward"
    if e.dim() != 2 or c.dim() != 2:
        raise ValueError(f"[{what}] e must be [N, D] and c [V, D], got {tuple(e.shape)} and {tuple(c.shape)}")
    N, D = e.shape
    V = c.shape[0]
    if c.shape[1] != D:
        raise ValueError(f"[{what}] c.shape[1] ({c.shape[1]}) must equal e.shape[1] ({D})")
    if targets.dim() != 1 or targets.shape[0] != N:
        raise ValueError(f"[{what}] targets must be [N={N}], got {tuple(targets.shape)}")
    if targets.dtype != torch.int32:
        raise ValueError(f"[{what}] targets must be int32, got {targets.dtype}")
    if e.dtype != c.dtype:
        raise ValueError(f"[{what}] e and c must share a dtype, got {e.dtype} and {c.dtype}")
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != V):
        raise ValueError(f"[{what}] bias must be [V={V}], got {tuple(bias.shape)}")
    dev = _require_cuda(what, e=e, c=c, targets=targets, bias=bias)
    dt = dtype_code(e.dtype, what)
    bdt = dtype_code(bias.dtype, what) if bias is not None else 0
    nvt = num_stat_tiles(V)
    ws_bytes = int(lib.cce_forward_workspace_bytes(N, D, V, dt))
    with _alloc_on(stream):
        tile_max = torch.empty((nvt, N), dtype=torch.float32, device=dev)
        lse = torch.empty((N,), dtype=torch.float32, device=dev)
        tgt = torch.empty((N,), dtype=torch.float32, device=dev)
        ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
    with _Timed("forward", _torch_stream(stream) if _timing is not None else None):
        rc = lib.cce_forward(_ptr(e), _ptr(c), _ptr(bias), bdt, _ptr(targets), N, D, V, int(v_offset),
                             dt, _ptr(tile_max), _ptr(lse), _ptr(tgt), _ptr(ws), ws_bytes,
                             _stream(stream))
    _check(rc, what)
    return tile_max, lse, tgt


def lse_combine(part_lse, part_tgt=None, stream=None):
    """Merge P partial rows: part_lse [P, N] (any row stride, unit column stride).

    Returns (lse [N], tgt [N] or None, nll [N] or None).
    """
    what = "cce_lse_combine"
    if part_lse.dim() != 2 or part_lse.stride(1) != 1:
        raise ValueError(f"[{what}] part_lse must be [P, N] with unit column stride")
    P, N = part_lse.shape
    if part_tgt is not None and (part_tgt.shape != part_lse.shape or part_tgt.stride() != part_lse.stride()):
        raise ValueError(f"[{what}] part_tgt must match part_lse in shape and strides")
    if part_lse.dtype != torch.float32 or (part_tgt is not None and part_tgt.dtype != torch.float32):
        raise ValueError(f"[{what}] partials must be float32")
    if not part_lse.is_cuda:
        raise ValueError(f"[{what}] partials must be CUDA tensors")
    dev = part_lse.device
    with _alloc_on(stream):
        lse = torch.empty((N,), dtype=torch.float32, device=dev)
        tgt = torch.empty((N,), dtype=torch.float32, device=dev) if part_tgt is not None else None
        nll = torch.empty((N,), dtype=torch.float32, device=dev) if part_tgt is not None else None
    rc = lib.cce_lse_combine(_ptr(part_lse), _ptr(part_tgt), P, N, part_lse.stride(0), _ptr(lse),
                             _ptr(tgt), _ptr(nll), _stream(stream))
    _check(rc, what)
    return lse, tgt, nll


def backward(e, c, targets, lse, d_nll, tile_max, bias=None, *, v_offset: int = 0,
             need_e: bool = True, need_c: bool = False, need_bias: bool = False,
             grad_e_f32: bool = False, filter_log_eps: float = FILTER_LOG_EPS,
             no_filter: bool = False, skip_stats=None, peer_group=None, stream=None):
    """Raw backward.  Returns (grad_e, grad_c, grad_bias); absent ones are None.

    grad_e is in e's dtype (fp32 with ``grad_e_f32``), grad_c in c's dtype,
    grad_bias in fp32.  With ``peer_group`` (a ``CcePeerGroup`` describing
    the exchange buffers of a vocabulary-sharded group, see ``_peer``) this
    runs ``cce_backward_peer``: grad_e comes back summed over the group.
    """
    what = "cce_backward_peer" if peer_group is not None else "cce_backward"
    N, D = e.shape
    V = c.shape[0]
    dev = _require_cuda(what, e=e, c=c, targets=targets, lse=lse, d_nll=d_nll, tile_max=tile_max,
                        bias=bias)
    if targets.dtype != torch.int32:
        raise ValueError(f"[{what}] targets must be int32")
    for name, t in (("lse", lse), ("d_nll", d_nll), ("tile_max", tile_max)):
        if t.dtype != torch.float32:
            raise ValueError(f"[{what}] {name} must be float32")
    if lse.numel() != N or d_nll.numel() != N or tile_max.numel() != num_stat_tiles(V) * N:
        raise ValueError(f"[{what}] lse/d_nll must hold N={N} values and tile_max {num_stat_tiles(V)}x{N}")
    if need_bias and bias is None:
        raise ValueError(f"[{what}] need_bias without bias")
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != V):
        raise ValueError(f"[{what}] bias must be [V={V}], got {tuple(bias.shape)}")
    dt = dtype_code(e.dtype, what)
    bdt = dtype_code(bias.dtype, what) if bias is not None else 0
    flags = (CCE_NEED_DE if need_e else 0) | (CCE_NEED_DC if need_c else 0) | \
            (CCE_NEED_DBIAS if need_bias else 0) | (CCE_DE_F32 if grad_e_f32 else 0) | \
            (CCE_NO_FILTER if no_filter else 0)
    ws_bytes = int(lib.cce_backward_workspace_bytes(N, D, V, dt, flags))
    with _alloc_on(stream):
        grad_e = None
        if need_e:
            grad_e = torch.empty((N, D), dtype=torch.float32 if grad_e_f32 else e.dtype, device=dev)
        grad_c = torch.empty((V, D), dtype=c.dtype, device=dev) if need_c else None
        grad_b = torch.empty((V,), dtype=torch.float32, device=dev) if need_bias else None
        ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
    if skip_stats is not None and (skip_stats.dtype != torch.int64 or skip_stats.numel() < 2
                                   or not skip_stats.is_cuda):
        raise ValueError(f"[{what}] skip_stats must be a CUDA int64 tensor with 2 entries")
    with _Timed("backward", _torch_stream(stream) if _timing is not None else None):
        if peer_group is not None:
            rc = lib.cce_backward_peer(_ptr(e), _ptr(c), _ptr(bias), bdt, _ptr(targets), _ptr(lse),
                                       _ptr(d_nll), _ptr(tile_max), N, D, V, int(v_offset), dt, flags,
                                       float(filter_log_eps), _ptr(grad_e), _ptr(grad_c), _ptr(grad_b),
                                       _ptr(skip_stats), _ptr(ws), ws_bytes, ctypes.byref(peer_group),
                                       _stream(stream))
        else:
            rc = lib.cce_backward(_ptr(e), _ptr(c), _ptr(bias), bdt, _ptr(targets), _ptr(lse),
                                  _ptr(d_nll), _ptr(tile_max), N, D, V, int(v_offset), dt, flags,
                                  float(filter_log_eps), _ptr(grad_e), _ptr(grad_c), _ptr(grad_b),
                                  _ptr(skip_stats), _ptr(ws), ws_bytes, _stream(stream))
    _check(rc, what)
    return grad_e, grad_c, grad_b


def _quant_head(what, wq, scales, biases, group_size, bits, D):
    if wq.dim() != 2 or scales.dim() != 2 or biases.shape != scales.shape:
        raise ValueError(f"[{what}] wq must be 2D and scales / biases 2D of equal shape")
    if wq.dtype not in (torch.int32, torch.uint32):
        raise ValueError(f"[{what}] wq must hold 32-bit words, got {wq.dtype}")
    V = wq.shape[0]
    if wq.shape[1] * 32 != D * bits or scales.shape != (V, D // group_size):
        raise ValueError(f"[{what}] quantised head shapes do not match D={D}, bits={bits}, group_size={group_size}")
    h = CceQuantHead()
    h.wq, h.scales, h.biases = wq.data_ptr(), scales.data_ptr(), biases.data_ptr()
    h.scale_dtype = dtype_code(scales.dtype, what)
    h.group_size, h.bits = int(group_size), int(bits)
    return h, V


def forward_q(e, wq, scales, biases, group_size: int, bits: int, targets, bias=None, stream=None):
    """Fused forward with a quantised classifier (``cce_forward_q``): the head
    is expanded one chunk at a time inside the library.  Returns (tile_max, lse, tgt)."""
    what = "cce_forward_q"
    if e.dim() != 2:
        raise ValueError(f"[{what}] e must be [N, D]")
    N, D = e.shape
    h, V = _quant_head(what, wq, scales, biases, group_size, bits, D)
    if targets.dim() != 1 or targets.shape[0] != N or targets.dtype != torch.int32:
        raise ValueError(f"[{what}] targets must be int32 [N={N}]")
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != V):
        raise ValueError(f"[{what}] bias must be [V={V}]")
    dev = _require_cuda(what, e=e, wq=wq, scales=scales, biases=biases, targets=targets, bias=bias)
    dt = dtype_code(e.dtype, what)
    bdt = dtype_code(bias.dtype, what) if bias is not None else 0
    ws_bytes = int(lib.cce_forward_q_workspace_bytes(N, D, V, dt))
    with _alloc_on(stream):
        tile_max = torch.empty((num_stat_tiles(V), N), dtype=torch.float32, device=dev)
        lse = torch.empty((N,), dtype=torch.float32, device=dev)
        tgt = torch.empty((N,), dtype=torch.float32, device=dev)
        ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
    with _Timed("forward", _torch_stream(stream) if _timing is not None else None):
        rc = lib.cce_forward_q(_ptr(e), ctypes.byref(h), _ptr(bias), bdt, _ptr(targets), N, D, V, 0, dt,
                               _ptr(tile_max), _ptr(lse), _ptr(tgt), _ptr(ws), ws_bytes, _stream(stream))
    _check(rc, what)
    return tile_max, lse, tgt


def backward_q(e, wq, scales, biases, group_size: int, bits: int, targets, lse, d_nll, tile_max, bias=None, *,
               need_e=True, need_bias=False, filter_log_eps: float = FILTER_LOG_EPS, stream=None):
    """Backward with a quantised (frozen) classifier (``cce_backward_q``).
    Returns (grad_e in e's dtype or None, grad_bias fp32 or None)."""
    what = "cce_backward_q"
    N, D = e.shape
    h, V = _quant_head(what, wq, scales, biases, group_size, bits, D)
    dev = _require_cuda(what, e=e, targets=targets, lse=lse, d_nll=d_nll, tile_max=tile_max, bias=bias)
    if need_bias and bias is None:
        raise ValueError(f"[{what}] need_bias without bias")
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != V):
        raise ValueError(f"[{what}] bias must be [V={V}]")
    if tile_max.numel() != num_stat_tiles(V) * N:
        raise ValueError(f"[{what}] tile_max must hold {num_stat_tiles(V)}x{N} values")
    dt = dtype_code(e.dtype, what)
    bdt = dtype_code(bias.dtype, what) if bias is not None else 0
    flags = (CCE_NEED_DE if need_e else 0) | (CCE_NEED_DBIAS if need_bias else 0)
    ws_bytes = int(lib.cce_backward_q_workspace_bytes(N, D, V, dt, flags))
    with _alloc_on(stream):
        grad_e = torch.empty((N, D), dtype=e.dtype, device=dev) if need_e else None
        grad_b = torch.empty((V,), dtype=torch.float32, device=dev) if need_bias else None
        ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
    with _Timed("backward", _torch_stream(stream) if _timing is not None else None):
        rc = lib.cce_backward_q(_ptr(e), ctypes.byref(h), _ptr(bias), bdt, _ptr(targets), _ptr(lse), _ptr(d_nll),
                                _ptr(tile_max), N, D, V, 0, dt, flags, float(filter_log_eps), _ptr(grad_e),
                                _ptr(grad_b), None, _ptr(ws), ws_bytes, _stream(stream))
    _check(rc, what)
    return grad_e, grad_b


def dequantize(wq, scales, biases, group_size: int, bits: int, dtype, out=None, stream=None):
    """Expand rows of an affine group-quantised matrix (``cce_dequantize``).

    wq uint32 [rows, D * bits / 32] (32 / bits values per word, low bits
    first; torch.int32 storage is accepted as the same bits), scales / biases
    [rows, D / group_size]; returns ``scales * q + biases`` as ``dtype``
    [rows, D] (into ``out`` when given).
    """
    what = "cce_dequantize"
    if wq.dim() != 2 or scales.dim() != 2 or biases.shape != scales.shape:
        raise ValueError(f"[{what}] wq must be 2D and scales / biases 2D of equal shape")
    if wq.dtype not in (torch.int32, torch.uint32):
        raise ValueError(f"[{what}] wq must hold 32-bit words, got {wq.dtype}")
    if bits not in (2, 4, 8):
        raise ValueError(f"[{what}] bits must be 2, 4 or 8, got {bits}")
    rows = wq.shape[0]
    D = wq.shape[1] * 32 // bits
    if scales.shape != (rows, D // group_size):
        raise ValueError(f"[{what}] scales must be [{rows}, {D // group_size}], got {tuple(scales.shape)}")
    dev = _require_cuda(what, wq=wq, scales=scales, biases=biases)
    if out is None:
        with _alloc_on(stream):
            out = torch.empty((rows, D), dtype=dtype, device=dev)
    elif out.shape != (rows, D) or out.dtype != dtype or not out.is_contiguous():
        raise ValueError(f"[{what}] out must be a contiguous [{rows}, {D}] {dtype} tensor")
    rc = lib.cce_dequantize(_ptr(wq), _ptr(scales), _ptr(biases), dtype_code(scales.dtype, what), rows, D,
                            int(group_size), int(bits), dtype_code(dtype, what), _ptr(out), _stream(stream))
    _check(rc, what)
    return out


# ---------------------------------------------------------------------------
# The reference's three module-level entry points (csrc/bindings.cpp:15-86).
# ---------------------------------------------------------------------------

def _as_i32_targets(targets):
    return targets.to(torch.int32).contiguous()


def cce_forward_raw(e, c, targets, bias=None, *, stream=None):
    """Mirror of ``cce_forward_raw`` (csrc/bindings.cpp:58-69, cce.cpp:123-145).

    Returns ``[tile_max_flat, tile_sum_exp_flat, neg_target_logit, lse]`` like
    the reference, except that the 32-column tile maxima are in tile-major
    order (``[ceil(V/32) * N]``, the reference's is row-major) and
    ``tile_sum_exp`` is not kept (it is folded into ``lse`` on the device), so
    an empty tensor stands in.
    """
    tile_max, lse, tgt = forward(e, c, _as_i32_targets(targets), bias, stream=stream)
    return [tile_max.reshape(-1), tile_max.new_empty((0,)), -tgt, lse]


def cce_backward_raw(e, c, lse, targets, d_nll, tile_max, bias=None, *, stream=None,
                     compute_all_grads=False):
    """Mirror of ``cce_backward_raw`` (csrc/bindings.cpp:71-86, cce.cpp:152-179).

    Returns dE in e's dtype; with ``compute_all_grads=True`` returns
    ``(dE, dC, dBias)`` (the reference's CutCrossEntropy::vjp path,
    cce.cpp:424-450).
    """
    V = c.shape[0]
    tm = tile_max.reshape(num_stat_tiles(V), e.shape[0])
    ge, gc, gb = backward(e, c, _as_i32_targets(targets), lse.float().contiguous(),
                          d_nll.float().contiguous(), tm.contiguous(), bias, need_e=True,
                          need_c=compute_all_grads, need_bias=compute_all_grads and bias is not None,
                          stream=stream)
    if compute_all_grads:
        return ge, gc, (gb.to(bias.dtype) if gb is not None else None)
    return ge


def cut_cross_entropy(e, c, targets, bias=None, reduction="mean", ignore_index=-100,
                      compute_all_grads=False, *, stream=None):
    """Mirror of ``cut_cross_entropy`` (csrc/bindings.cpp:15-56, cce.cpp:31-116).

    Differentiable; gradients flow to c and bias whenever they require grad
    (``compute_all_grads`` is accepted for signature compatibility).
    """
    from . import cce_loss
    if e.dim() != 2:
        raise ValueError(f"[cut_cross_entropy] e must be 2D [B, D], got {e.dim()}D")
    if c.dim() != 2:
        raise ValueError(f"[cut_cross_entropy] c must be 2D [V, D], got {c.dim()}D")
    if targets.dim() != 1:
        raise ValueError(f"[cut_cross_entropy] targets must be 1D [B], got {targets.dim()}D")
    if stream is not None:
        with torch.cuda.stream(stream):
            return cce_loss(e, c, targets, bias=bias, reduction=reduction, ignore_index=ignore_index)
    return cce_loss(e, c, targets, bias=bias, reduction=reduction, ignore_index=ignore_index)
