#!/usr/bin/env python
"""Benchmark: Cut Cross-Entropy forward+backward tokens/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 3] [--impl ours|reference]

One step = forward + backward of the fused linear + cross-entropy over one
batch of the synthetic workload (default: config 3, the Llama-3.1-8B head,
N=4096 tokens, D=4096, V=128256, bf16, peaked logits, Zipf targets, 5%
ignored, reduction='mean'), producing grad_e and grad_c.  With N GPUs (one
process per GPU under torchrun) the vocabulary is split across the ranks
(strong scaling: the same N tokens per step, V/N classifier rows per GPU);
the per-row statistics are all-gathered and grad_e all-reduced over NCCL.

Prints ONE JSON line on rank 0.  ``--impl reference`` times the CPU
restatement of the reference's pure-MLX path (oracle/cce_oracle.py) on the
host cores instead, on a bounded row sample of the same workload.
"""

from __future__ import annotations

import argparse
import csv
import datetime
import io
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "mlx-cross-entropy_b200"))

import torch  # noqa: E402

METRIC = "CCE fwd+bwd tokens/s (Llama-3-8B head, bf16) and % of BF16 tensor peak"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
DTYPE_NAMES = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}
N_SMS = 148


def fp32_nominal_tflops(sm_mhz):
    """FP32 FFMA peak of one B200: 128 lanes per SM, one FMA (2 FLOP) per cycle."""
    return N_SMS * 128 * 2 * sm_mhz * 1e6 / 1e12


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# DRAM bytes (read + write) of one forward launch, measured by ncu on config 3
# at full size (profiles/forward_cfg3_dram_traffic.txt): e is read once
# (33.6 MB); c and the per-row statistics grow with the local vocabulary.
def forward_traffic_bytes(N, D, V_local):
    if (N, D) != (4096, 4096):
        return None
    return 33.55e6 + (1168.373248e6 - 33.55e6) * V_local / 128256


def load_synthetic():
    """The workload generator, loaded from its file without importing the
    ``mlx_cce`` package (whose import loads the CUDA library): the reference
    arm must map none of this repository's native code."""
    import importlib.util
    path = REPO / "mlx-cross-entropy_b200" / "mlx_cce" / "synthetic.py"
    spec = importlib.util.spec_from_file_location("cce_synthetic", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["cce_synthetic"] = mod  # dataclasses resolve the module by name
    spec.loader.exec_module(mod)
    return mod


def workload_config(w, N, D, V, world, scaled):
    """The ``config`` object of both arms' JSON lines (identical for one workload)."""
    return {"workload": f"cfg{w.cfg} {w.name}" + (" (scaled)" if scaled else ""),
            "N": N, "D": D, "V": V,
            "global_batch": N, "seq_len": w.batch[-1] if len(w.batch) > 1 and not scaled else N,
            "reduction": w.reduction,
            "parallelism": f"vocab-sharded x{world}" if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (c is %.2f GB), no flush" % (V * D * 2 / 1e9)}


def probe_mlx():
    """Whether the reference's own array library imports here (it never has:
    MLX targets Apple silicon and is not in this image).  Returns the outcome
    as one line for the reference arm's note."""
    try:
        import mlx.core  # noqa: F401
        return "import mlx.core succeeded"
    except Exception as exc:  # ImportError / ModuleNotFoundError expected
        return f"import mlx.core failed: {type(exc).__name__}: {exc}"


def env_int(name, default):
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self, gpus):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r for r in csv.reader(io.StringIO(out)) if len(r) >= 9]
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                idx = int(r[0])
            except ValueError:
                continue
            if idx not in gpus:
                continue
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
            except ValueError:
                pass
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        busy = [s for s in sm if s > 0.5 * max(sm)]
        return {"sm_mhz": statistics.median(busy or sm), "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# reference arm: the CPU restatement of the reference's pure-MLX path
# ---------------------------------------------------------------------------

def cpu_reference_step_fn(cfg, rows):
    """Returns (step(), sample description, cores) timing the oracle on a row sample."""
    sys.path.insert(0, str(REPO))
    from oracle import cce_oracle as O
    synthetic = load_synthetic()
    e, c, t, bias, go, w = synthetic.make_inputs(cfg)
    rows = min(rows, w.N)
    e2 = e.reshape(-1, w.D)[:rows].float().numpy()
    t2 = t.reshape(-1)[:rows].numpy()
    c32 = c.float().numpy()
    b32 = None if bias is None else bias.float().numpy()
    red = w.reduction if w.reduction != "none" else "sum"

    def step():
        O.cpu_fwd_bwd_step(e2, c32, t2, b32, reduction=red)

    try:
        from threadpoolctl import threadpool_info
        cores = max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
    except Exception:
        cores = os.cpu_count() or 1
    what = f"all {rows} rows" if rows == w.N else f"first {rows} of {w.N} rows"
    sample = (f"{what} of config {cfg} against the full V={w.V} x D={w.D} "
              f"classifier: chunked online-LSE forward + analytic dE/dC backward, float32 numpy")
    return step, sample, cores, w, rows


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    # torchrun limits every process to one OpenMP thread; the CPU reference
    # runs alone on rank 0 and may use every host thread
    from threadpoolctl import threadpool_limits
    ncpu = os.cpu_count() or 1
    torch.set_num_threads(ncpu)
    mlx_note = probe_mlx()
    with threadpool_limits(limits=ncpu):
        step, sample, cores, w, rows = cpu_reference_step_fn(args.config, args.ref_rows)
        for _ in range(args.warmup):
            step()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step()
        dt = (time.perf_counter() - t0) / args.steps
    value = rows / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": workload_config(w, w.N, w.D, w.V, world, False),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": (f"{mlx_note}; the reference's pure-MLX path (reference/_chunked.py + "
                 "reference/_metal_backward.py) is therefore timed through its CPU restatement "
                 "(oracle/cce_oracle.py) on a row sample of the same workload; tokens/s = sample "
                 "rows / step time"),
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# parity of the benchmarked step (checker leg: reads the oracle's fixtures)
# ---------------------------------------------------------------------------

LOSS_RTOL_16 = 1e-3   # BASELINE's loss tolerance for 16-bit inputs (1e-5 for fp32)
GRAD_TOL = 2e-2       # relative max-abs gradient tolerance


def parity_block(w, scaled, loss, lse, e_grad, c_grad, e_dev, c_dev, b_dev, e_cpu, t_cpu, c_full,
                 b_full, go_cpu, v0, v1, rank, world, dev):
    """Loss and sampled gradients of one benchmarked step against the float64 oracle.

    With a committed fixture (tests/golden/cfg{1..4}.npz, the oracle's
    outputs on the same seeded inputs) the loss, the sampled grad_e rows and
    the sampled grad_c vocabulary rows of this rank's shard are compared with
    it.  Without one (config 5, scaled runs) the oracle runs here on sampled
    rows: rank 0 checks the LSE and grad_e of 8 rows against the full
    classifier (``c_full``, ``b_full``), every rank the grad_c of sampled vocabulary rows
    of its shard (given the GPU's global LSE), and the loss is compared with
    the reduction of (GPU LSE - target logit), the target logits recomputed
    in float64.  Every rank takes the same collective steps; each error is the
    maximum over ranks.
    """
    import numpy as np
    import torch.distributed as dist
    sys.path.insert(0, str(REPO))
    from oracle import cce_oracle as O

    def allreduce(vals, op):
        tt = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(tt, op=op)
        return tt.tolist()

    MAX = dist.ReduceOp.MAX if world > 1 else None
    fixture = REPO / "tests" / "golden" / f"cfg{w.cfg}.npz"
    safe, valid = O.sanitize(t_cpu.numpy())
    got_loss = loss.detach().double().cpu().numpy().reshape(-1)
    rtol_loss = 1e-5 if w.dtype == torch.float32 else LOSS_RTOL_16
    if fixture.exists() and not scaled:
        ref = np.load(fixture)
        ref_loss = np.asarray(ref["loss"], np.float64).reshape(-1)
        loss_rel = float(np.abs(got_loss - ref_loss).max() / max(np.abs(ref_loss).max(), 1e-30))
        rows = ref["rows"]
        de = e_grad[torch.as_tensor(rows, device=dev)].double().cpu().numpy()
        de_rel = O.rel_max_abs(de, ref["dE_rows"])
        cols = ref["cols"]
        mine = (cols >= v0) & (cols < v1)
        num = 0.0
        if mine.any():
            got = c_grad[torch.as_tensor(cols[mine] - v0, device=dev)].double().cpu().numpy()
            num = float(np.abs(got - ref["dC_cols"][mine]).max())
        den = float(np.abs(ref["dC_cols"]).max()) or 1.0
        loss_rel, de_rel, num = allreduce([loss_rel, de_rel, num], MAX)
        out = {"loss_rel": loss_rel, "dE_rel": de_rel, "dC_rel": num / den,
               "rows": int(len(rows)), "cols": int(len(cols)),
               "source": f"tests/golden/{fixture.name}: float64 oracle on the same seeded inputs"}
    else:
        gw = go_cpu.reshape(-1).double().numpy() if go_cpu is not None else np.ones(len(safe))
        d_nll = valid * gw
        if w.reduction == "mean":
            d_nll = d_nll / max(valid.sum(), 1)
        lse_g = lse.detach().double().cpu().numpy()
        e32 = e_cpu.float().numpy()
        rng = np.random.default_rng(1000 + w.cfg)
        lse_rel = de_rel = 0.0
        if rank == 0:
            rows = np.sort(rng.choice(len(safe), 8, replace=False))
            cf = c_full.float().numpy()
            bf = None if b_full is None else b_full.float().numpy()
            lse_ref, _ = O.rows_lse_tgt(e32, cf, safe, rows, bias=bf)
            lse_rel = float(np.abs(lse_g[rows] - lse_ref).max() / np.abs(lse_ref).max())
            de_ref = O.rows_grad_e(e32, cf, safe, lse_ref, d_nll[rows], rows, bias=bf)
            de = e_grad[torch.as_tensor(rows, device=dev)].double().cpu().numpy()
            de_rel = O.rel_max_abs(de, de_ref)
        # target logits in float64: each rank adds those of its shard's targets
        tl = safe - v0
        on = np.nonzero((tl >= 0) & (tl < v1 - v0))[0]
        tgt = torch.zeros(len(safe), dtype=torch.float64, device=dev)
        if len(on):
            r_on = torch.as_tensor(on, device=dev)
            c_on = c_dev.detach()[torch.as_tensor(tl[on], device=dev)].double()
            tgt[r_on] = (e_dev[r_on].double() * c_on).sum(dim=1)
            if b_dev is not None:
                tgt[r_on] += b_dev.detach()[torch.as_tensor(tl[on], device=dev)].double()
        if world > 1:
            dist.all_reduce(tgt, op=dist.ReduceOp.SUM)
        ref_loss = O.reduce(lse_g - tgt.cpu().numpy(), valid, w.reduction)
        ref_loss = np.asarray(ref_loss, np.float64).reshape(-1)
        loss_rel = float(np.abs(got_loss - ref_loss).max() / max(np.abs(ref_loss).max(), 1e-30))
        # grad_c on 6 sampled vocabulary rows of this shard plus 2 target rows in it
        vr = v1 - v0
        pick = rng.choice(vr, min(6, vr), replace=False) + v0
        tgts = np.unique(safe[valid][(safe[valid] >= v0) & (safe[valid] < v1)])[:2]
        cols = np.unique(np.concatenate([pick, tgts])).astype(np.int64)
        c_sub = c_dev.detach()[torch.as_tensor(cols - v0, device=dev)].float().cpu().numpy()
        tmap = np.full(len(safe), -1, np.int64)
        for j, col in enumerate(cols):
            tmap[safe == col] = j
        b_sub = None
        if b_dev is not None:
            b_sub = b_dev.detach()[torch.as_tensor(cols - v0, device=dev)].float().cpu().numpy()
        dc_ref, _ = O.cols_grad_c(e32, c_sub, tmap, lse_g, d_nll, np.arange(len(cols)),
                                  bias=b_sub)
        got = c_grad[torch.as_tensor(cols - v0, device=dev)].double().cpu().numpy()
        num, den = float(np.abs(got - dc_ref).max()), float(np.abs(dc_ref).max())
        loss_rel, lse_rel, de_rel, num, den = allreduce([loss_rel, lse_rel, de_rel, num, den], MAX)
        out = {"loss_rel": loss_rel, "lse_rel": lse_rel, "dE_rel": de_rel,
               "dC_rel": num / (den or 1.0), "rows": 8, "cols_per_rank": int(len(cols)),
               "source": ("float64 oracle on sampled rows; loss = reduction of (GPU lse - float64 "
                          "target logit), the GPU lse checked on the sampled rows")}
    out["tol"] = {"loss_rel": rtol_loss, "grad_rel": GRAD_TOL}
    out["ok"] = bool(out["loss_rel"] < rtol_loss and out["dE_rel"] < GRAD_TOL
                     and out["dC_rel"] < GRAD_TOL and out.get("lse_rel", 0.0) < rtol_loss)
    return out


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args, rank, world, local_rank):
    import torch.distributed as dist
    import mlx_cce
    from mlx_cce import _ext, synthetic
    from mlx_cce import distributed as mdist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    scaled = args.N is not None or args.V is not None or args.D is not None
    e_cpu, c_cpu, t_cpu, b_cpu, go_cpu, w = synthetic.make_inputs(args.config, N=args.N, V=args.V,
                                                                  D=args.D)
    N, D, V = e_cpu.reshape(-1, e_cpu.shape[-1]).shape[0], e_cpu.shape[-1], c_cpu.shape[0]
    v0, v1 = mdist.vocab_shard(V, rank, world)
    e_cpu = e_cpu.reshape(N, D)
    t_cpu = t_cpu.reshape(N)
    e = e_cpu.to(dev)
    t = t_cpu.to(dev)
    c = c_cpu[v0:v1].contiguous().to(dev).requires_grad_(True)
    bias = b_cpu[v0:v1].contiguous().to(dev).requires_grad_(True) if b_cpu is not None else None
    go = go_cpu.reshape(N).to(dev) if go_cpu is not None else None
    # the parity leg's sampled oracle needs the whole classifier on rank 0
    # when no fixture covers the workload
    fixture = (REPO / "tests" / "golden" / f"cfg{w.cfg}.npz").exists() and not scaled
    keep_full = not args.no_parity and not fixture and rank == 0
    c_full = c_cpu if keep_full else None
    b_full = b_cpu if keep_full else None
    del c_cpu
    skip = torch.zeros(2, dtype=torch.int64, device=dev)

    def step(e_in, t_in, full=False):
        e_in = e_in.detach().requires_grad_(True)
        c.grad = None
        if bias is not None:
            bias.grad = None
        if world > 1:
            loss, lse = mdist.linear_cross_entropy(e_in, c, t_in, bias, reduction=w.reduction,
                                                   v_offset=v0, skip_stats=skip, return_lse=True)
        else:
            loss, lse = mlx_cce.linear_cross_entropy(e_in, c, t_in, bias, reduction=w.reduction,
                                                     skip_stats=skip, return_lse=True)
        if w.reduction == "none":
            loss.backward(go)
        else:
            loss.backward()
        return (loss, lse, e_in) if full else loss

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        tt = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    # Warm-up: W eager steps on the stream the eager regions time (the caching
    # allocator keeps blocks per stream, and a first allocation while the
    # exchange buffers are mapped has stalled the host for up to ~0.5 s), then
    # one on a side stream (as CUDA-graph capture wants); then capture one whole
    # fwd+bwd step.  Every replay recomputes everything from e, c, targets.
    for _ in range(args.warmup):
        step(e, t)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step(e, t)
    torch.cuda.current_stream().wait_stream(side)
    barrier()
    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step(e, t)
        barrier()

    # ---- device-resident timed region: graph replays (eager steps with --no-graph) ----
    sampler = ClockSampler()
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        if graph is not None:
            graph.replay()
        else:
            step(e, t)
    ev1.record()
    torch.cuda.synchronize()
    elapsed_ms = max_over_ranks(ev0.elapsed_time(ev1))
    clocks = sampler.stop(set(range(world))) if rank == 0 else None

    # ---- eager timed region: per-call kernel times, launches, skipped blocks ----
    skip.zero_()
    _ext.mma_flops(reset=True)
    launches0 = _ext.launch_count()
    _ext.set_timing(True)
    barrier()
    ev4, ev5 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev4.record()
    for _ in range(args.steps):
        step(e, t)
    ev5.record()
    torch.cuda.synchronize()
    eager_ms = max_over_ranks(ev4.elapsed_time(ev5))
    launches = _ext.launch_count() - launches0
    recs = _ext.timings()
    _ext.set_timing(False)
    fwd_ms = [a.elapsed_time(b) for name, a, b in recs if name == "forward"]
    bwd_ms = [a.elapsed_time(b) for name, a, b in recs if name == "backward"]
    fwd_avg = max_over_ranks(statistics.mean(fwd_ms)) if fwd_ms else float("nan")
    bwd_avg = max_over_ranks(statistics.mean(bwd_ms)) if bwd_ms else float("nan")
    skipped, total = skip.tolist()
    # tensor-core work the kernels issued (filter-skipped blocks excluded), all ranks
    mma = _ext.mma_flops(reset=True)
    mma_t = torch.tensor([mma[k] / args.steps for k in ("forward", "dlogits", "grad_e", "grad_c")],
                         dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(mma_t)
    mma_step = dict(zip(("forward", "dlogits", "grad_e", "grad_c"), mma_t.tolist()))

    # ---- end-to-end through the public API with host buffers ----
    # Every step copies its inputs from pinned host memory and reads its loss
    # back, inside the timed region.  As in a training loop with a prefetching
    # data loader, step i + 1's inputs are copied on a copy stream (into the
    # other of two device buffers) while step i computes; a buffer is
    # overwritten only after the loss read-back of the step that last read it.
    # With N GPUs every rank needs all of e: each copies its 1/N of the rows
    # over PCIe and the rows are all-gathered over NVLink (NCCL) in the step,
    # so the job moves e across PCIe once, not N times.
    split = world > 1 and N % world == 0
    rows = N // world if split else N
    e_host = (e_cpu[rank * rows:(rank + 1) * rows] if split else e_cpu).contiguous().pin_memory()
    t_host = t_cpu.pin_memory()
    e_dev = [torch.empty_like(e), torch.empty_like(e)]
    e_part = [torch.empty((rows, D), dtype=e.dtype, device=dev) for _ in range(2)] if split else e_dev
    t_dev = [torch.empty_like(t), torch.empty_like(t)]
    copy_stream = torch.cuda.Stream(device=dev)
    ready = [torch.cuda.Event(), torch.cuda.Event()]

    def prefetch(i):
        with torch.cuda.stream(copy_stream):
            e_part[i % 2].copy_(e_host, non_blocking=True)
            t_dev[i % 2].copy_(t_host, non_blocking=True)
            ready[i % 2].record(copy_stream)

    def inputs(i):
        torch.cuda.current_stream().wait_event(ready[i % 2])
        if split:
            dist.all_gather_into_tensor(e_dev[i % 2], e_part[i % 2])
        return e_dev[i % 2], t_dev[i % 2]

    # two untimed passes of the loop body (its buffers, copies and collective warm)
    for i in range(2):
        prefetch(i)
        step(*inputs(i)).detach().cpu()
    barrier()
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev2.record()
    copy_stream.wait_event(ev2)
    d2h = 0
    prefetch(0)
    for i in range(args.steps):
        loss = step(*inputs(i))
        if i + 1 < args.steps:
            prefetch(i + 1)
        host = loss.detach().cpu()
        d2h = host.numel() * host.element_size()
    ev3.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(ev2.elapsed_time(ev3))
    # bytes the whole job moves per step: e once (split over the ranks), the
    # targets to every rank; the loss back to the host on every rank
    h2d = e_cpu.numel() * e_cpu.element_size() * (1 if split else world) + \
        t_host.numel() * t_host.element_size() * world
    d2h *= world

    # ---- parity of the benchmarked step (every rank, every N) ----
    parity = None
    if not args.no_parity:
        loss_p, lse_p, e_p = step(e, t, full=True)
        torch.cuda.synchronize()
        parity = parity_block(w, scaled, loss_p, lse_p, e_p.grad, c.grad, e, c, bias, e_cpu, t_cpu,
                              c_full, b_full, go_cpu, v0, v1, rank, world, dev)
        del loss_p, lse_p, e_p

    # ---- CPU baseline (rank 0 at N=1 only) ----
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        stepc, sample, cores, _, crow = cpu_reference_step_fn(args.config, args.cpu_rows)
        stepc()  # warm-up
        runs = []
        for _ in range(3):  # median of three
            t0 = time.perf_counter()
            stepc()
            runs.append(time.perf_counter() - t0)
        dtc = statistics.median(runs)
        cpu = {"value": crow / dtc, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": sample + "; median of 3 runs after 1 warm-up"}

    if world > 1:
        dist.barrier()
    if rank == 0:
        peaks, src = load_peaks()
        ms = elapsed_ms / args.steps
        value = N / (ms / 1e3)
        flops = 8.0 * N * V * D
        tflops = flops / (ms / 1e3) / 1e12
        peak_sus = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
        peak_burst = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
        # a timed region under a second never reaches the power-capped steady state
        long_run = elapsed_ms > 1000.0
        peak = peak_sus if long_run else peak_burst
        vl = v1 - v0
        fwd_tflops = 2.0 * N * vl * D / (fwd_avg / 1e3) / 1e12
        traffic = forward_traffic_bytes(N, D, vl)
        fp32 = w.dtype == torch.float32
        if fp32:
            # float32 inputs run on the CUDA cores (FFMA): TF32 tensor cores
            # cannot meet the 1e-5 loss tolerance.  No measured FP32 peak
            # exists for this pool, so the denominator is the nominal one.
            sm_mhz = peaks.get("sm_max_mhz", 1965.0)
            peak = fp32_nominal_tflops(sm_mhz)
            peak_kind = f"nominal FP32 FFMA: {N_SMS} SMs x 128 lanes x 2 FLOP x {sm_mhz:.0f} MHz"
        else:
            peak_kind = f"{src} bf16 {'sustained' if long_run else 'burst'}"
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": DTYPE_NAMES.get(w.dtype, str(w.dtype)),
            "data": "synthetic (seeded, see mlx_cce/synthetic.py)",
            "config": workload_config(w, N, D, V, world, scaled),
            # whole-job TFLOP/s against the peak of all N GPUs together
            "tflops": tflops, "pct_bf16_peak": tflops / (peak_burst * world),
            "pct_bf16_peak_sustained": tflops / (peak_sus * world),
            # against the 2.25 PFLOP/s dense-BF16 figure NVIDIA quotes per B200
            "pct_bf16_spec": tflops / (2250.0 * world),
            "flops_per_step": flops,
            # what the tensor cores executed: the nominal 8 N V D minus the
            # blocks the filter skipped (tile padding included)
            "executed_flops_per_step": sum(mma_step.values()),
            "executed_flops_by_kernel": mma_step,
            "pct_bf16_peak_executed": sum(mma_step.values()) / (ms / 1e3) / 1e12 / (peak_burst * world),
            "skipped_blocks_frac": (skipped / total) if total else None,
            "fwd_ms": fwd_avg, "bwd_ms": bwd_avg,
            "roofline": {"bound": "fp32 (CUDA cores)" if fp32 else "tensor",
                         "kernel": "forward (logits + online LSE)",
                         "achieved": fwd_tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": fwd_tflops / peak,
                         "peak_kind": peak_kind,
                         "traffic": traffic,
                         # e and c once, a max per row per 32-column statistics tile,
                         # a (max, sum-exp) pair per row per 256-column kernel tile
                         "algorithmic_bytes": (2.0 * (N * D + vl * D) + 4.0 * N * (-(-vl // 32))
                                               + 8.0 * N * (-(-vl // 256)))},
            "e2e": {"value": N * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            # library kernels per K steps (counted in the eager region; a graph
            # replay launches the same kernels)
            "gpu_launches": int(launches),
            "timing": ("CUDA-graph replay of the whole fwd+bwd step" if graph is not None
                       else "eager steps"),
            "eager_ms_per_step": eager_ms / args.steps,
            "clocks": clocks,
        }
        if fp32:
            line["pct_fp32_peak_nominal"] = tflops / (peak * world)
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if parity is not None:
            line["parity"] = parity
        print(json.dumps(line), flush=True)
    # a graph holding NCCL calls must be released before the process group,
    # and the exchange buffers (a collective) while it still exists
    del graph
    torch.cuda.synchronize()
    if world > 1:
        from mlx_cce import _peer
        _peer.release_all()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_quantized(args):
    """Frozen quantised head (the reference's mlx-lm LoRA recipe, README.md:84-95):
    tokens/s of fwd + bwd (grad_e only) with the classifier kept group-quantised
    in HBM, beside the same step on the dense head with c frozen.  Eager steps,
    CUDA events on the launching stream; one GPU."""
    import mlx_cce
    from mlx_cce import synthetic
    from mlx_cce.quantized import linear_cross_entropy_quantized, quantize
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    e_cpu, c_cpu, t_cpu, b_cpu, go_cpu, w = synthetic.make_inputs(args.config, N=args.N, V=args.V, D=args.D)
    N, D = e_cpu.reshape(-1, e_cpu.shape[-1]).shape
    e = e_cpu.reshape(N, D).to(dev)
    t = t_cpu.reshape(N).to(dev)
    c = c_cpu.to(dev)
    q = quantize(c, args.group_size, args.quantized_bits)
    V = c.shape[0]
    c_deq = q.dequantize(c.dtype)          # the dense head the quantised one stands for
    del c

    def dense():
        ei = e.detach().requires_grad_(True)
        loss = mlx_cce.linear_cross_entropy(ei, c_deq, t, reduction=w.reduction)
        (loss.sum() if w.reduction == "none" else loss).backward()

    def quant():
        ei = e.detach().requires_grad_(True)
        loss = linear_cross_entropy_quantized(ei, q, t, reduction=w.reduction)
        (loss.sum() if w.reduction == "none" else loss).backward()

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / args.steps

    dense_ms = timed(dense)
    quant_ms = timed(quant)
    line = {
        "metric": "CCE fwd+bwd tokens/s with a frozen quantised classifier", "value": N / (quant_ms / 1e3),
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": quant_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded, see mlx_cce/synthetic.py)",
        "config": dict(workload_config(w, N, D, V, 1, args.N is not None or args.V is not None),
                       classifier=f"{args.quantized_bits}-bit affine, groups of {args.group_size}, frozen",
                       gradients="grad_e only"),
        "dense_frozen_ms_per_step": dense_ms,
        "quantized_over_dense": quant_ms / dense_ms,
        "timing": "eager steps, CUDA events",
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ref-rows", type=int, default=1 << 30,
                    help="rows of the workload in one step of the reference arm (--impl reference; "
                         "default: all of them)")
    ap.add_argument("--cpu-rows", type=int, default=256,
                    help="rows of the workload in the cpu_baseline leg of our arm")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the check of one step against the float64 oracle")
    ap.add_argument("--no-graph", action="store_true", help="time eager steps instead of graph replays")
    ap.add_argument("--quantized-bits", type=int, default=0,
                    help="time a frozen classifier quantised to 2/4/8 bits beside the dense frozen one")
    ap.add_argument("--group-size", type=int, default=64, help="quantisation group size")
    ap.add_argument("--N", type=int, default=None, help="scaled-down rows (profiling captures)")
    ap.add_argument("--V", type=int, default=None, help="scaled-down vocabulary (profiling captures)")
    ap.add_argument("--D", type=int, default=None, help="scaled-down hidden size (profiling captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        print("warning: --warmup below 3 does not meet the timing rules", file=sys.stderr)
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.quantized_bits:
        if world > 1:
            raise SystemExit("--quantized-bits runs on one GPU")
        return run_quantized(args)
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
