"""CPU tests of the C-ABI library and the host-side API logic (no kernel runs)."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

import mlx_cce
from mlx_cce import _ext
from mlx_cce._autograd import sanitize_targets
from mlx_cce.distributed import vocab_shard

REPO = Path(__file__).resolve().parent.parent


def _header_symbols():
    text = "\n".join(p.read_text() for p in (REPO / "include").glob("*.h"))
    return set(re.findall(r"CCE_API\s+[\w\s\*]+?\b(cce_\w+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    declared = _header_symbols()
    assert declared, "no CCE_API declarations found in include/*.h"
    lib = ctypes.CDLL(str(_ext._LIB_PATH))
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert set(_ext.EXPORTED_SYMBOLS) == declared


def test_version_and_tile_count():
    assert _ext.version() == 100
    assert _ext.num_stat_tiles(128256) == 4008
    assert _ext.num_stat_tiles(32) == 1
    assert _ext.num_stat_tiles(33) == 2
    assert _ext.num_stat_tiles(0) == 0


def test_workspace_sizes():
    lib = _ext.lib
    f = lib.cce_forward_workspace_bytes(4096, 4096, 128256, _ext.CCE_BF16)
    assert f >= 2 * 1002 * 4096 * 4 and f % 256 == 0
    flags = _ext.CCE_NEED_DE | _ext.CCE_NEED_DC
    b = lib.cce_backward_workspace_bytes(4096, 4096, 128256, _ext.CCE_BF16, flags)
    # mask + a bounded dlogits chunk (never [N, V]) + two fp32 grad_e accumulator slabs
    assert b < 4096 * 128256 * 2
    assert b >= 2 * 4096 * 4096 * 4
    b32 = lib.cce_backward_workspace_bytes(4096, 4096, 128256, _ext.CCE_BF16,
                                           flags | _ext.CCE_DE_F32)
    assert b32 <= b
    # the fp32 (CUDA-core) path accumulates in grad_e itself when it is fp32
    f = lib.cce_backward_workspace_bytes(512, 512, 32000, _ext.CCE_F32, flags)
    f32 = lib.cce_backward_workspace_bytes(512, 512, 32000, _ext.CCE_F32, flags | _ext.CCE_DE_F32)
    assert f32 == f - 512 * 512 * 4


def test_error_codes_without_gpu_work():
    lib = _ext.lib
    # bad dtype / sizes are rejected before any CUDA call
    rc = lib.cce_forward(None, None, None, 0, None, 4, 8, 16, 0, 7, None, None, None, None, 0, None)
    assert rc == _ext.CCE_ERR_DTYPE
    assert b"dtype" in lib.cce_last_error()
    rc = lib.cce_forward(None, None, None, 0, None, -1, 8, 16, 0, 0, None, None, None, None, 0, None)
    assert rc == _ext.CCE_ERR_SHAPE
    rc = lib.cce_backward(None, None, None, 0, None, None, None, None, 4, 8, 16, 0, 0, 1 << 9,
                          -8.0, None, None, None, None, None, 0, None)
    assert rc == _ext.CCE_ERR_ARG
    rc = lib.cce_backward(None, None, None, 0, None, None, None, None, 4, 8, 16, 0, 0,
                          _ext.CCE_NEED_DE, -8.0, None, None, None, None, None, 0, None)
    assert rc == _ext.CCE_ERR_ARG
    rc = lib.cce_lse_combine(None, None, 0, 4, 4, None, None, None, None)
    assert rc == _ext.CCE_ERR_SHAPE
    # the bounded-wait self-test takes a limit in (0, 2 s]
    assert lib.cce_selftest_wait_timeout(0, None) == _ext.CCE_ERR_ARG
    assert lib.cce_selftest_wait_timeout(3_000_000_000, None) == _ext.CCE_ERR_ARG


def test_peer_buffer_layout_and_argument_checks():
    """Exchange buffer of the sharded backward: a 4 KB control block, then
    world x 2 fp32 receive slots of R rows (R = 128 * ceil(ceil(N / 128) /
    world)), then R rows of the output dtype; each part 256-byte aligned."""
    lib = _ext.lib

    def expect(N, D, world, esize):
        mt = -(-N // 128)
        R = 128 * -(-mt // world)
        up = lambda x: -(-x // 256) * 256
        return 4096 + up(world * 2 * R * D * 4) + up(R * D * esize)

    assert lib.cce_peer_buffer_bytes(4096, 4096, 8, _ext.CCE_BF16) == expect(4096, 4096, 8, 2)
    assert lib.cce_peer_buffer_bytes(640, 256, 2, _ext.CCE_BF16) == expect(640, 256, 2, 2)
    assert lib.cce_peer_buffer_bytes(200, 100, 2, _ext.CCE_F32) == expect(200, 100, 2, 4)
    assert lib.cce_peer_buffer_bytes(32768, 8192, 8, _ext.CCE_BF16) == expect(32768, 8192, 8, 2)
    assert lib.cce_peer_buffer_bytes(100, 64, 0, _ext.CCE_BF16) == 0
    assert lib.cce_peer_buffer_bytes(100, 64, 17, _ext.CCE_BF16) == 0
    # rejected before any CUDA call
    args = [None, None, None, 0, None, None, None, None, 4, 8, 16, 0, 0, _ext.CCE_NEED_DE, -8.0,
            None, None, None, None, None, 0]
    assert lib.cce_backward_peer(*args, None, None) == _ext.CCE_ERR_ARG
    g = _ext.CcePeerGroup()
    g.rank, g.world = 0, 17
    assert lib.cce_backward_peer(*args, ctypes.byref(g), None) == _ext.CCE_ERR_ARG
    g.world = 2   # bases left NULL
    assert lib.cce_backward_peer(*args, ctypes.byref(g), None) == _ext.CCE_ERR_ARG
    assert b"NULL" in lib.cce_last_error()
    assert lib.cce_peer_buffer_alloc(1 << 20, None, None) == _ext.CCE_ERR_ARG
    assert lib.cce_peer_buffer_open(-1, 1 << 20, None) == _ext.CCE_ERR_ARG


def test_python_api_rejects_cpu_tensors_and_bad_args():
    e = torch.randn(8, 16)
    c = torch.randn(32, 16)
    t = torch.randint(0, 32, (8,))
    with pytest.raises(ValueError, match="Unknown reduction"):
        mlx_cce.linear_cross_entropy(e, c, t, reduction="avg")
    with pytest.raises(ValueError, match="CUDA tensor"):
        mlx_cce.linear_cross_entropy(e, c, t)
    with pytest.raises(ValueError, match="2D"):
        mlx_cce.cce_loss(e[None], c, t)
    with pytest.raises(ValueError):
        _ext.forward(e, c[:, :8], t.to(torch.int32))
    with pytest.raises(ValueError, match="int32"):
        _ext.forward(e, c, t)
    with pytest.raises(ValueError, match="share a dtype"):
        _ext.forward(e, c.half(), t.to(torch.int32))
    with pytest.raises(ValueError, match="unsupported dtype"):
        _ext.dtype_code(torch.float64, "x")


def test_sanitize_targets():
    t = torch.tensor([[3, -100, 7], [-100, 0, 5]])
    safe, valid = sanitize_targets(t, -100)
    assert safe.dtype == torch.int32
    assert safe.tolist() == [3, 0, 7, 0, 0, 5]
    assert valid.tolist() == [True, False, True, False, True, True]
    safe, valid = sanitize_targets(torch.tensor([1, 2]), None)
    assert valid.all() and safe.tolist() == [1, 2]


@pytest.mark.parametrize("V,world", [(128256, 8), (128256, 3), (10, 4), (7, 8)])
def test_vocab_shard_partition(V, world):
    spans = [vocab_shard(V, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == V
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0 and a1 >= a0
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1
