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
    from mlx_cce import synthetic
    e, c, t, bias, go, w = synthetic.make_inputs(cfg)
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
    sample = (f"first {rows} of {w.N} rows of config {cfg} against the full V={w.V} x D={w.D} "
              f"classifier: chunked online-LSE forward + analytic dE/dC backward, float32 numpy")
    return step, sample, cores, w


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    # torchrun limits every process to one OpenMP thread; the CPU reference
    # runs alone on rank 0 and may use every host thread
    from threadpoolctl import threadpool_limits
    ncpu = os.cpu_count() or 1
    torch.set_num_threads(ncpu)
    with threadpool_limits(limits=ncpu):
        rows = args.ref_rows
        step, sample, cores, w = cpu_reference_step_fn(args.config, rows)
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
        "config": {"workload": f"cfg{w.cfg} {w.name}", "N": w.N, "D": w.D, "V": w.V,
                   "global_batch": w.N, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "MLX is not installable here: the reference's pure-MLX path is timed through its "
                "CPU restatement (oracle/cce_oracle.py).",
    }
    print(json.dumps(line), flush=True)
    return 0


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
    del c_cpu
    skip = torch.zeros(2, dtype=torch.int64, device=dev)

    def step(e_in, t_in):
        e_in = e_in.detach().requires_grad_(True)
        c.grad = None
        if bias is not None:
            bias.grad = None
        if world > 1:
            loss = mdist.linear_cross_entropy(e_in, c, t_in, bias, reduction=w.reduction,
                                              v_offset=v0, skip_stats=skip)
        else:
            loss = mlx_cce.linear_cross_entropy(e_in, c, t_in, bias, reduction=w.reduction,
                                                skip_stats=skip)
        if w.reduction == "none":
            loss.backward(go)
        else:
            loss.backward()
        return loss

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

    # warm-up on a side stream (as CUDA-graph capture wants), then capture one
    # whole fwd+bwd step; every replay recomputes everything from e, c, targets
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(args.warmup):
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

    # ---- end-to-end through the public API with host buffers ----
    # Every step copies its inputs from pinned host memory and reads its loss
    # back, inside the timed region.  As in a training loop with a prefetching
    # data loader, step i + 1's inputs are copied on a copy stream (into the
    # other of two device buffers) while step i computes; a buffer is
    # overwritten only after the loss read-back of the step that last read it.
    e_host = e_cpu.pin_memory()
    t_host = t_cpu.pin_memory()
    e_dev = [torch.empty_like(e), torch.empty_like(e)]
    t_dev = [torch.empty_like(t), torch.empty_like(t)]
    copy_stream = torch.cuda.Stream(device=dev)
    ready = [torch.cuda.Event(), torch.cuda.Event()]

    def prefetch(i):
        with torch.cuda.stream(copy_stream):
            e_dev[i % 2].copy_(e_host, non_blocking=True)
            t_dev[i % 2].copy_(t_host, non_blocking=True)
            ready[i % 2].record(copy_stream)

    barrier()
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev2.record()
    copy_stream.wait_event(ev2)
    d2h = 0
    prefetch(0)
    for i in range(args.steps):
        torch.cuda.current_stream().wait_event(ready[i % 2])
        loss = step(e_dev[i % 2], t_dev[i % 2])
        if i + 1 < args.steps:
            prefetch(i + 1)
        host = loss.detach().cpu()
        d2h = host.numel() * host.element_size()
    ev3.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(ev2.elapsed_time(ev3))
    h2d = e_host.numel() * e_host.element_size() + t_host.numel() * t_host.element_size()

    # ---- CPU baseline (rank 0 at N=1 only) ----
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        stepc, sample, cores, _ = cpu_reference_step_fn(args.config, args.ref_rows)
        stepc()  # warm-up
        runs = []
        for _ in range(3):  # median of three
            t0 = time.perf_counter()
            stepc()
            runs.append(time.perf_counter() - t0)
        dtc = statistics.median(runs)
        cpu = {"value": args.ref_rows / dtc, "unit": "tokens/s", "cores": cores, "kind": "port",
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
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16" if w.dtype == torch.bfloat16 else str(w.dtype),
            "data": "synthetic (seeded, see mlx_cce/synthetic.py)",
            "config": {"workload": f"cfg{w.cfg} {w.name}" + (" (scaled)" if scaled else ""),
                       "N": N, "D": D, "V": V,
                       "global_batch": N, "seq_len": w.batch[-1] if len(w.batch) > 1 and not scaled else N,
                       "reduction": w.reduction,
                       "parallelism": f"vocab-sharded x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (c is %.2f GB), no flush" % (V * D * 2 / 1e9)},
            # whole-job TFLOP/s against the peak of all N GPUs together
            "tflops": tflops, "pct_bf16_peak": tflops / (peak_burst * world),
            "pct_bf16_peak_sustained": tflops / (peak_sus * world),
            # against the 2.25 PFLOP/s dense-BF16 figure NVIDIA quotes per B200
            "pct_bf16_spec": tflops / (2250.0 * world),
            "flops_per_step": flops,
            "skipped_blocks_frac": (skipped / total) if total else None,
            "fwd_ms": fwd_avg, "bwd_ms": bwd_avg,
            "roofline": {"bound": "tensor", "kernel": "forward (logits + online LSE)",
                         "achieved": fwd_tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": fwd_tflops / peak,
                         "peak_kind": f"{src} bf16 {'sustained' if long_run else 'burst'}",
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
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    # a graph holding NCCL calls must be released before the process group
    del graph
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ref-rows", type=int, default=256,
                    help="rows of the workload in one CPU-reference step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="time eager steps instead of graph replays")
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
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
