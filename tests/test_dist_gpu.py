"""Vocabulary-sharded CCE on 2 GPUs over NCCL (one process per GPU).

Each rank holds e, targets and its contiguous shard of c / bias; the
distributed wrapper all-gathers the per-row (lse, target logit) rows and
all-reduces grad_e.  The loss and gradients must equal the unsharded
single-GPU path on the same inputs.  Needs >= 2 GPUs; on a 1-GPU machine the
test is skipped with that reason (the sharded composition itself is covered
on one GPU by test_parity_gpu.py::test_vocab_sharded_composition).
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(77)
    N, D, V = 640, 256, 10007
    e = torch.randn(N, D, generator=g).to(torch.bfloat16)
    c = (torch.randn(V, D, generator=g) * D ** -0.5).to(torch.bfloat16)
    b = torch.randn(V, generator=g) * 0.2
    t = torch.randint(0, V, (N,), generator=g)
    t[::9] = -100
    return e, c, b, t


def _worker(rank, world, port, q):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "mlx-cross-entropy_b200"))
    import torch.distributed as dist
    import mlx_cce
    from mlx_cce import distributed as mdist
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        e, c, b, t = _inputs()
        V = c.shape[0]
        v0, v1 = mdist.vocab_shard(V, rank, world)
        res = {}
        for reduction in ("mean", "none"):
            e_ = e.to(dev).requires_grad_(True)
            c_ = c[v0:v1].contiguous().to(dev).requires_grad_(True)
            b_ = b[v0:v1].contiguous().to(dev).requires_grad_(True)
            loss = mdist.linear_cross_entropy(e_, c_, t.to(dev), b_, reduction=reduction, v_offset=v0)
            go = torch.linspace(-1, 1, loss.numel(), device=dev).reshape(loss.shape) \
                if reduction == "none" else None
            loss.backward(go)
            # unsharded reference on the same GPU
            e2 = e.to(dev).requires_grad_(True)
            c2 = c.to(dev).requires_grad_(True)
            b2 = b.to(dev).requires_grad_(True)
            ref = mlx_cce.linear_cross_entropy(e2, c2, t.to(dev), b2, reduction=reduction)
            ref.backward(go)
            torch.cuda.synchronize()
            rel = lambda x, y: float((x.float() - y.float()).abs().max() / (y.float().abs().max() + 1e-30))
            res[reduction] = dict(
                loss=rel(loss.detach(), ref.detach()),
                de=rel(e_.grad, e2.grad),
                dc=rel(c_.grad, c2.grad[v0:v1]),
                db=rel(b_.grad, b2.grad[v0:v1]))
        q.put((rank, "ok", res))
    except Exception as exc:  # reported through the queue
        q.put((rank, "error", repr(exc)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_vocab_sharded_two_gpus_match_unsharded():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs (this machine has %d)" % torch.cuda.device_count())
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, status, res in sorted(out, key=lambda x: x[0]):
        assert status == "ok", f"rank {rank}: {res}"
        for reduction, errs in res.items():
            assert errs["loss"] < 1e-3, (rank, reduction, errs)
            for k in ("de", "dc", "db"):
                assert errs[k] < 2e-2, (rank, reduction, k, errs)
