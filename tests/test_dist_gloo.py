"""Multi-rank (world_size 2 / 4) CPU tests of the vocabulary-sharded exchange.

The ranks are gloo processes on the CPU.  Each rank computes its shard's
per-row (lse_r, tgt_r) and grad_e partial with the CPU oracle (these ranks
have no GPU), then runs the SAME exchange code the GPU path uses
(mlx_cce._exchange): the all-gather of the [2, N] statistics and the
all-reduce of grad_e.  The merged results must equal the unsharded oracle.
A rank that fails before the collective must make its peer fail with an
error within the process-group timeout, not hang.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _inputs():
    g = torch.Generator().manual_seed(123)
    N, D, V = 48, 24, 1000
    e = torch.randn(N, D, generator=g, dtype=torch.float64)
    c = torch.randn(V, D, generator=g, dtype=torch.float64) * 0.3
    b = torch.randn(V, generator=g, dtype=torch.float64) * 0.1
    t = torch.randint(0, V, (N,), generator=g)
    t[::7] = -100
    return e, c, b, t


def _worker_exchange(rank, world, port, q):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo))
    sys.path.insert(0, str(repo / "mlx-cross-entropy_b200"))
    from oracle import cce_oracle as O
    from mlx_cce._exchange import gather_shard_stats, sum_grad_e
    from mlx_cce.distributed import vocab_shard
    try:
        _init(rank, world, port)
        e, c, b, t = _inputs()
        V = c.shape[0]
        v0, v1 = vocab_shard(V, rank, world)
        safe, valid = O.sanitize(t.numpy())
        en, cn, bn = e.numpy(), c.numpy(), b.numpy()
        # this rank's shard: local LSE and target logit (0 when the target is elsewhere)
        z = en @ cn[v0:v1].T + bn[None, v0:v1]
        m = z.max(axis=1)
        lse_r = m + np.log(np.exp(z - m[:, None]).sum(axis=1))
        local = (safe >= v0) & (safe < v1)
        tgt_r = np.where(local, z[np.arange(len(safe)), np.clip(safe - v0, 0, v1 - v0 - 1)], 0.0)
        gathered = gather_shard_stats(torch.from_numpy(lse_r).float(), torch.from_numpy(tgt_r).float())
        assert gathered.shape == (world, 2, len(safe))
        g = gathered.double().numpy()
        M = g[:, 0].max(axis=0)
        lse = M + np.log(np.exp(g[:, 0] - M).sum(axis=0))
        tgt = g[:, 1].sum(axis=0)
        # backward with the GLOBAL lse: this rank's grad_e partial, then the sum
        d = O.d_nll_from_reduction(valid, "mean")
        p = np.exp(z - lse[:, None])
        p[local, safe[local] - v0] -= 1.0
        ge_r = (d[:, None] * p) @ cn[v0:v1]
        ge = sum_grad_e(torch.from_numpy(ge_r).float()).double().numpy()
        nll_full, lse_full, tgt_full, _ = O.dense_forward(en, cn, t.numpy(), bn)
        dE_full, _, _ = O.backward_full(en, cn, lse_full, safe, d, bn)
        ok = (np.allclose(lse, lse_full, rtol=1e-5) and np.allclose(tgt, tgt_full, rtol=1e-5, atol=1e-5)
              and O.rel_max_abs(ge, dE_full) < 1e-5)
        q.put((rank, ok, float(np.abs(lse - lse_full).max()), O.rel_max_abs(ge, dE_full)))
    except Exception as exc:  # pragma: no cover - reported through the queue
        q.put((rank, False, repr(exc), None))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_exchange_matches_unsharded(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_exchange, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, a, b in sorted(results):
        assert ok, f"rank {rank}: {a} {b}"


def _worker_fail(rank, world, port, q):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "mlx-cross-entropy_b200"))
    from mlx_cce._exchange import gather_shard_stats
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            raise RuntimeError("rank 1 fails before the exchange")
        gather_shard_stats(torch.zeros(4), torch.zeros(4))
        q.put((rank, "no error"))
    except Exception as exc:
        q.put((rank, type(exc).__name__))
    finally:
        if rank == 1 and dist.is_initialized():
            dist.destroy_process_group()


def test_failed_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_fail, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():  # pragma: no cover
            p.kill()
    assert results[1] == "RuntimeError"
    assert results[0] != "no error"


def _worker_fd_exchange(rank, world, port, q):
    """Ranks send each other a descriptor of a file holding their rank id, with
    the code the GPU exchange buffers use (mlx_cce._peer.PeerGroup._exchange_fds)."""
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "mlx-cross-entropy_b200"))
    from mlx_cce import _peer
    try:
        _init(rank, world, port)
        pg = _peer.PeerGroup(dist.group.WORLD, torch.device("cpu"))
        fd = os.memfd_create(f"cce-test-{rank}")
        os.write(fd, b"rank %d" % rank)
        got = _peer.PeerGroup._exchange_fds(pg, fd)
        os.close(fd)
        seen = {}
        for r, rfd in got.items():
            seen[r] = os.pread(rfd, 16, 0).decode()
            os.close(rfd)
        q.put((rank, "ok", seen))
    except Exception as exc:  # reported through the queue
        q.put((rank, "error", repr(exc)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 12])
def test_exchange_buffer_descriptors_reach_every_rank(world):
    """12 ranks exceed the datagram queue length of 10: the receiving thread
    must drain while the sends go out."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_fd_exchange, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, status, seen in out:
        assert status == "ok", (rank, seen)
        assert seen == {r: f"rank {r}" for r in range(world) if r != rank}
