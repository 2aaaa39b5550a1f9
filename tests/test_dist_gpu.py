"""Vocabulary-sharded CCE on 2 GPUs (one process per GPU).

Each rank holds e, targets and its contiguous shard of c / bias.  The forward
all-gathers the per-row (lse, target logit) over NCCL; the backward sums
grad_e across the ranks inside ``cce_backward_peer`` over NVLink peer memory
(the default), or with one NCCL all-reduce of fp32 partials
(``CCE_GRAD_E_EXCHANGE=nccl``, the unfused baseline).  Both must reproduce the
float64 oracle (loss, grad_e, each rank's grad_c / grad_bias rows), and the
large case the unsharded single-GPU path on the same inputs.  Needs >= 2 GPUs;
on a 1-GPU machine the test is skipped with that reason (the sharded
composition is covered on one GPU by
test_parity_gpu.py::test_vocab_sharded_composition and the exchange by
test_peer_gpu.py).
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CASES = {
    # name: (N, D, V, dtype, bias, oracle)
    "bf16_bias": (640, 256, 10007, torch.bfloat16, True, True),
    "fp32_cuda_cores": (200, 100, 3000, torch.float32, False, True),
    "bf16_two_chunks_per_rank": (8300, 64, 40000, torch.bfloat16, False, False),
}


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(N, D, V, dtype, bias, seed=77):
    g = torch.Generator().manual_seed(seed)
    e = torch.randn(N, D, generator=g).to(dtype)
    c = (torch.randn(V, D, generator=g) * D ** -0.5).to(dtype)
    b = torch.randn(V, generator=g) * 0.2 if bias else None
    t = torch.randint(0, V, (N,), generator=g)
    t[::9] = -100
    return e, c, b, t


def _worker(rank, world, port, mode, q):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "mlx-cross-entropy_b200"))
    sys.path.insert(0, str(repo))
    os.environ["CCE_GRAD_E_EXCHANGE"] = mode
    os.environ["CCE_BWD_CHUNK_ROWS"] = "16384"   # several vocabulary chunks per rank in the big case
    import torch.distributed as dist
    import mlx_cce
    from mlx_cce import distributed as mdist, _peer
    from oracle import cce_oracle as O
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        res = {}
        for name, (N, D, V, dtype, bias, use_oracle) in CASES.items():
            e, c, b, t = _inputs(N, D, V, dtype, bias)
            v0, v1 = mdist.vocab_shard(V, rank, world)
            for reduction in ("mean", "none"):
                go = torch.linspace(-1, 1, N) if reduction == "none" else None
                e_ = e.to(dev).requires_grad_(True)
                c_ = c[v0:v1].contiguous().to(dev).requires_grad_(True)
                b_ = b[v0:v1].contiguous().to(dev).requires_grad_(True) if bias else None
                loss = mdist.linear_cross_entropy(e_, c_, t.to(dev), b_, reduction=reduction, v_offset=v0)
                loss.backward(go.to(dev) if go is not None else None)
                torch.cuda.synchronize()
                f = lambda x: x.detach().double().cpu().numpy()
                if use_oracle:
                    ref_loss, _lse, dE, dC, dB = O.loss_and_grads(
                        e.double().numpy(), c.double().numpy(), t.numpy(),
                        None if b is None else b.double().numpy(), reduction, -100,
                        None if go is None else go.double().numpy())
                    ref_c = dC[v0:v1]
                    ref_b = None if dB is None else dB[v0:v1]
                else:   # the unsharded single-GPU path on the same inputs
                    e2 = e.to(dev).requires_grad_(True)
                    c2 = c.to(dev).requires_grad_(True)
                    ref = mlx_cce.linear_cross_entropy(e2, c2, t.to(dev), reduction=reduction)
                    ref.backward(go.to(dev) if go is not None else None)
                    ref_loss, dE, ref_c, ref_b = f(ref), f(e2.grad), f(c2.grad)[v0:v1], None
                loss_err = float(np.abs(f(loss).reshape(-1) - np.asarray(ref_loss).reshape(-1)).max()
                                 / max(np.abs(ref_loss).max(), 1e-30))
                errs = dict(loss=loss_err, de=O.rel_max_abs(f(e_.grad), dE),
                            dc=O.rel_max_abs(f(c_.grad), ref_c))
                if ref_b is not None:
                    errs["db"] = O.rel_max_abs(f(b_.grad), ref_b)
                assert e_.grad.dtype == dtype
                res[f"{name}/{reduction}"] = errs
        _ext_status = mlx_cce._ext.lib.cce_device_status(0)
        res["device_status"] = int(_ext_status)
        _peer.release_all()
        q.put((rank, "ok", res))
    except Exception as exc:  # reported through the queue
        import traceback
        q.put((rank, "error", repr(exc) + traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["peer", "nccl"])
def test_vocab_sharded_two_gpus_match_oracle(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs (this machine has %d)" % torch.cuda.device_count())
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, status, res in sorted(out, key=lambda x: x[0]):
        assert status == "ok", f"rank {rank}: {res}"
        assert res.pop("device_status") == 0, f"rank {rank}: a bounded wait ran out"
        for case, errs in res.items():
            tol = 1e-5 if case.startswith("fp32") else 1e-3
            assert errs["loss"] < tol, (rank, case, errs)
            for k in ("de", "dc", "db"):
                if k in errs:
                    assert errs[k] < 2e-2, (rank, case, k, errs)
