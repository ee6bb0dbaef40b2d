"""Benchmark of the scan hot path: tokens/s of one forward+backward step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c4] [--impl ours|reference]

A step is one forward and one backward pass of the configured scan through
the public API (torch.autograd over libmlrec.so) on one batch of synthetic
inputs. The default workload is config c4 (SSD, bf16, B=32, L=16384, H=32,
Dh=64, N=128, seg=32), the configuration the scaling target is quoted on.
Under torchrun (N > 1) every rank takes a contiguous batch range of the same
global problem (strong scaling, no collective on the data path); the timed
region is bracketed by a barrier and device synchronisation and the reported
time is the maximum over ranks.

Printed (rank 0, one JSON line): value = whole-job tokens/s with inputs
resident in HBM; e2e = the same step with host->device copies of the inputs
from pinned memory and a device->host read of the result inside the timed
region; roofline of the dominant kernel (algorithmic bytes / CUDA-event time);
cpu_baseline = the float32 C restatement of the reference algorithm
(oracle/ckpt_scan.c) on a bounded sample; clocks sampled during timing.

``--impl reference`` times that CPU restatement on this host's cores (the
reference itself is MLX/Metal and cannot run here) on the same metric.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def _env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# --------------------------------------------------------------------------- #
# algorithmic bytes per step (compulsory traffic; checkpoints excluded)
# --------------------------------------------------------------------------- #

def algorithmic_bytes(cfg, batch):
    """(forward_bytes, backward_bytes): inputs read once and y written (fp32)
    in the forward; inputs and grad_y (fp32) read and every gradient written
    in the input dtype in the backward."""
    es = 4 if cfg["dtype"].itemsize == 4 else 2
    B, L = batch, cfg["L"]
    k = cfg["kind"]
    if k == "ssd":
        H, Dh, N = cfg["H"], cfg["Dh"], cfg["N"]
        inp = B * L * H * (Dh + 1 + 2 * N) * es
        y = B * L * H * Dh * 4
    elif k == "gla":
        H, Dh = cfg["H"], cfg["Dh"]
        inp = B * L * H * (3 * Dh + 1) * es
        y = B * L * H * Dh * 4
    elif k == "gdn":  # q, k, v and alpha, beta per head
        H, Dh = cfg["H"], cfg["Dh"]
        inp = B * L * H * (3 * Dh + 2) * es
        y = B * L * H * Dh * 4
    elif k == "rglru":
        inp = B * L * cfg["D"] * 2 * es
        y = B * L * cfg["D"] * 4
    elif k == "rglru_gated":  # x, r, i (lam: one value per channel)
        inp = B * L * cfg["D"] * 3 * es
        y = B * L * cfg["D"] * 4
    elif k == "rotlru_angle":  # a, theta, x (two values per pair)
        Dp = cfg["Dp"]
        inp = B * L * Dp * 4 * es
        y = B * L * 2 * Dp * 4
    else:
        Dp = cfg["Dp"]
        inp = B * L * Dp * 5 * es
        y = B * L * 2 * Dp * 4
    return inp + y, inp + y + inp


# DRAM bytes (read + write) per launch measured by ncu, per batch row: the
# kernels' traffic grows linearly with the independent units. Chunk kernels
# (c4, c5) from a B=2 instance of the same configuration, diagonal scans (c2,
# c3) from the full configuration.
_NCU_TRAFFIC_PER_BATCH_ROW = {
    ("c4", "backward"): (1.208137e9 + 0.629970e9) / 2,
    ("c4", "forward"): (0.677076e9 + 0.496836e9) / 2,
    ("c5", "backward"): (0.806439e9 + 0.363859e9) / 2,
    ("c5", "forward"): (0.407030e9 + 0.357562e9) / 2,
    ("c2", "backward"): (674.370e6 + 309.851e6) / 8,
    ("c2", "forward"): (336.269e6 + 298.693e6) / 8,
    ("c3", "backward"): (2.516725e9 + 1.315607e9) / 16,
    ("c3", "forward"): (1.342216e9 + 1.059618e9) / 16,
}


def _traffic(name, which, nb, cfg):
    v = _NCU_TRAFFIC_PER_BATCH_ROW.get((name, which))
    return None if v is None else v * nb


# --------------------------------------------------------------------------- #
# clocks sampled during the timed region
# --------------------------------------------------------------------------- #

class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []  # (wall time, csv line)

    def _reader(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line))

    def __enter__(self):
        import threading
        try:
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                   "-lms", "50"]
            if self.gpu_id is not None:
                cmd.insert(1, f"--id={self.gpu_id}")
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._reader, daemon=True).start()
            t_end = time.time() + 3.0
            while not self.lines and time.time() < t_end and self.proc.poll() is None:
                time.sleep(0.01)
        except (OSError, ValueError):
            self.proc = None
        self.t0 = time.time()
        return self

    def __exit__(self, *a):
        self.t1 = time.time()
        time.sleep(0.06)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        inside = [l for ts, l in self.lines if self.t0 - 0.03 <= ts <= self.t1 + 0.06]
        if not inside:  # region shorter than the sampling interval: nearest sample after start
            inside = [l for ts, l in self.lines if ts >= self.t0][:1]
        for line in inside:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def _gpu_uuid(dev):
    import torch
    try:
        u = torch.cuda.get_device_properties(dev).uuid
        return f"GPU-{u}"
    except Exception:
        return None


# --------------------------------------------------------------------------- #
# CPU baseline: the C restatement of the reference algorithm on a sample
# --------------------------------------------------------------------------- #

def cpu_sample(name):
    """(inputs, grad_y, fraction of the config's units, description)."""
    import numpy as np
    import torch
    W = importlib.import_module("mlx-recurrence_b200.workloads")
    cfg = W.CONFIGS[name]
    k = cfg["kind"]
    threads = os.cpu_count() or 1
    if k in ("ssd", "gla", "gdn") and cfg["B"] * cfg["H"] > 2 * threads and cfg["L"] * cfg["Dh"] > 2 ** 18:
        hs = min(cfg["H"], max(1, threads))
        ins = W.make_inputs(name, "cpu", seed=1000, batch=1)
        ins = [t[:, :, :hs] if t.dim() >= 3 else t[:hs] for t in ins]
        frac = hs / (cfg["B"] * cfg["H"])
        desc = f"1 batch row x {hs} of {cfg['H']} heads (full L), scaled by units"
    elif k in ("rglru", "rglru_gated", "rotlru", "rotlru_angle") and cfg["B"] > 1 and cfg["B"] * cfg["L"] > 2 ** 15:
        nb = 1
        ins = W.make_inputs(name, "cpu", seed=1000, batch=nb)
        frac = nb / cfg["B"]
        desc = f"{nb} of {cfg['B']} batch rows (full L and width), scaled by units"
    else:
        ins = W.make_inputs(name, "cpu", seed=1000)
        frac = 1.0
        desc = "full config"
    ins = [t.float().contiguous().numpy() for t in ins]
    g = torch.Generator().manual_seed(7)
    yshape = ins[3].shape if k == "rotlru" else ins[2].shape if k == "rotlru_angle" else ins[0].shape
    gy = torch.randn(yshape, generator=g).numpy()
    return ins, gy, frac, desc


def _cpu_run(c_oracle, W, cfg, ins, gy):
    """One forward+backward of the C restatement; for the gated RG-LRU the
    reference's host-side gating (rglru.py:8-27), for the rotLRU angle input
    its host-side cos/sin (rotlru.py:18-22), runs first, in numpy."""
    if cfg["kind"] == "rglru_gated":
        a, b = W.gated_to_plain(*ins)
        return c_oracle.run("rglru", [a, b], cfg["seg"], gy=gy)
    if cfg["kind"] == "rotlru_angle":
        return c_oracle.run("rotlru", list(W.angle_to_plain(*ins)), cfg["seg"], gy=gy)
    return c_oracle.run(cfg["kind"], ins, cfg["seg"], gy=gy)


def cpu_baseline(name, reps=1):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import c_oracle  # float32 C restatement (test infrastructure)
    W = importlib.import_module("mlx-recurrence_b200.workloads")
    cfg = W.CONFIGS[name]
    ins, gy, frac, desc = cpu_sample(name)
    c_oracle.lib()
    _cpu_run(c_oracle, W, cfg, ins, gy)  # warm-up
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        _cpu_run(c_oracle, W, cfg, ins, gy)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    tok = W.tokens(cfg) * frac
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return {"value": tok / t, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{desc}; fwd+bwd of oracle/ckpt_scan.c (float32, OpenMP), median of {reps}",
            "seconds_per_sample": t}


# --------------------------------------------------------------------------- #
# GPU arm
# --------------------------------------------------------------------------- #

def run_ours(args):
    import torch
    import torch.distributed as dist

    pkg = importlib.import_module("mlx-recurrence_b200")
    W = importlib.import_module("mlx-recurrence_b200.workloads")
    lib = importlib.import_module("mlx-recurrence_b200._lib").load()
    rank, world = _env_int("RANK", 0), _env_int("WORLD_SIZE", 1)
    local = _env_int("LOCAL_RANK", 0)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    name = args.config
    cfg = dict(W.CONFIGS[name])
    if args.batch:
        cfg["B"] = args.batch
    b0, b1 = W.shard_batch(cfg["B"], rank, world)
    nb = b1 - b0
    ins = W.make_inputs(name, dev, seed=1000 + rank, batch=nb)
    gen = torch.Generator(device=dev).manual_seed(2000 + rank)
    gy = torch.randn(W.output_shape(name, nb), generator=gen, device=dev, dtype=torch.float32)
    fn = W.scan_fn(pkg, name)
    leaves = [t.detach().requires_grad_(True) if t.dtype.is_floating_point else t for t in ins]
    # A_neg as an expanded view: differentiate w.r.t. its base
    stream = torch.cuda.current_stream(dev)

    def step(xs, g):
        y = fn(*xs)
        torch.autograd.backward(y, g)
        return y

    ev = lambda: torch.cuda.Event(enable_timing=True)

    # ---- warm-up
    for _ in range(args.warmup):
        for x in leaves:
            x.grad = None
        step(leaves, gy)
    torch.cuda.synchronize()

    # ---- timed: inputs resident in HBM
    fwd_ms, bwd_ms = [], []
    n_launch0 = lib.mr_launch_count()
    torch.cuda.reset_peak_memory_stats(dev)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(_gpu_uuid(dev)) as clk:
        e_start, e_end = ev(), ev()
        e_start.record(stream)
        marks = []
        for _ in range(args.steps):
            for x in leaves:
                x.grad = None
            a, b, c = ev(), ev(), ev()
            a.record(stream)
            y = fn(*leaves)
            b.record(stream)
            torch.autograd.backward(y, gy)
            c.record(stream)
            marks.append((a, b, c))
            del y
        e_end.record(stream)
        torch.cuda.synchronize()
        barrier()
    launches = lib.mr_launch_count() - n_launch0
    total_ms = e_start.elapsed_time(e_end)
    for a, b, c in marks:
        fwd_ms.append(a.elapsed_time(b))
        bwd_ms.append(b.elapsed_time(c))
    peak_mb = torch.cuda.max_memory_allocated(dev) / 2 ** 20

    # ---- timed: end to end from pinned host memory
    e2e_ms = None
    h2d = d2h = 0
    if not args.no_e2e:
        e2e_ms, h2d, d2h = _e2e(args, fn, ins, gy, dev, stream, barrier, ev)

    # ---- max over ranks
    t = torch.tensor([total_ms, e2e_ms or 0.0, statistics.mean(fwd_ms), statistics.mean(bwd_ms)],
                     dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms_max, f_ms, b_ms = t.tolist()
    if e2e_ms is not None:
        e2e_ms = e2e_ms_max
    _report(args, rank, world, W, name, cfg, nb, total_ms, e2e_ms, f_ms, b_ms, h2d, d2h, peak_mb, launches, clk)
    if args.check:
        _check(args, rank, world, W, fn, ins, leaves, gy, cfg, nb)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _check(args, rank, world, W, fn, ins, leaves, gy, cfg, nb):
    """After timing: every rank's outputs and gradients gathered over the process
    group (NCCL), the replicated parameters' gradients summed over ranks, and rank 0
    runs the whole batch on its GPU and compares (max|diff| / max|ref|). The units
    are independent, so the gathered results equal the 1-GPU run up to the order
    of the cross-rank sums."""
    import torch
    import torch.distributed as dist
    S = importlib.import_module("mlx-recurrence_b200.sharding")
    B = cfg["B"]
    for x in leaves:
        x.grad = None
    y = fn(*leaves)
    torch.autograd.backward(y, gy)
    sharded = [x.dim() > 0 and x.shape[0] == nb and x.dim() >= 3 for x in ins]
    full_in = [S.gather_rows(x.detach(), B) if sh else x.detach() for x, sh in zip(ins, sharded)]
    y_all = S.gather_rows(y.detach(), B)
    gy_all = S.gather_rows(gy, B)
    g_all = []
    for x, sh in zip(leaves, sharded):
        g = x.grad
        if g is None:
            g_all.append(None)
        elif sh:
            g_all.append(S.gather_rows(g, B))
        else:  # a replicated parameter: its gradient is the sum of the ranks' partial sums
            g = g.float().contiguous()
            if world > 1:
                dist.all_reduce(g)
            g_all.append(g)
    if rank != 0:
        return
    # (detach keeps a broadcast parameter's stride-0 view, so the same kernel path runs)
    ref = [x.detach().requires_grad_(True) if x.dtype.is_floating_point else x for x in full_in]
    y_ref = fn(*ref)
    torch.autograd.backward(y_ref, gy_all)

    def rel(a, b):
        a, b = a.detach().float(), b.detach().float()
        return float((a - b).abs().max() / (b.abs().max() + 1e-30))
    errs = {"y": rel(y_all, y_ref)}
    for i, (g, r) in enumerate(zip(g_all, ref)):
        if g is not None and r.grad is not None:
            errs[f"grad{i}"] = rel(g, r.grad)
    print(json.dumps({"check": {"world": world, "config": args.config, "max_rel_err": max(errs.values()),
                                "rel_err": errs}}), flush=True)


def _e2e(args, fn, ins, gy, dev, stream, barrier, ev):
    """Same step through the public API with host buffers: per step, H2D copies
    of every input from pinned memory, forward+backward, D2H of the last
    step's outputs. Returns (ms for all steps, H2D bytes/step, D2H bytes/step)."""
    import torch
    # A tensor broadcast along its last axis (SSD's per-head A_neg) travels as
    # its [.., 1] base and is re-expanded on the device, as a caller would.
    def compact(t):
        t = t.detach()
        if t.dim() > 0 and t.stride(-1) == 0:
            return t[..., :1].contiguous(), tuple(t.shape)
        return t.contiguous(), None

    packed = [compact(t) for t in ins]
    host_ins = [c.to("cpu").pin_memory() for c, _ in packed]
    shapes = [s for _, s in packed]
    host_gy = gy.to("cpu").pin_memory()
    dev_ins = [torch.empty_like(h, device=dev) for h in host_ins]
    dev_gy = torch.empty_like(gy)
    with torch.no_grad():
        y_probe = fn(*(t.detach() for t in ins))  # only for the result's shape and dtype
    res_host = torch.empty(y_probe[:, -1].shape, dtype=y_probe.dtype, pin_memory=True)
    del y_probe
    h2d = sum(t.numel() * t.element_size() for t in host_ins) + host_gy.numel() * 4
    d2h = res_host.numel() * res_host.element_size()
    with torch.no_grad():
        for _ in range(2):  # warm the copy path
            for d, h in zip(dev_ins, host_ins):
                d.copy_(h, non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e2e_s, e2e_e = ev(), ev()
    e2e_s.record(stream)
    for _ in range(args.steps):
        with torch.no_grad():
            for d, h in zip(dev_ins, host_ins):
                d.copy_(h, non_blocking=True)
            dev_gy.copy_(host_gy, non_blocking=True)
        xs = []
        for d, s in zip(dev_ins, shapes):
            x = d.detach().requires_grad_(True)
            xs.append(x.expand(s) if s is not None else x)
        y = fn(*xs)
        torch.autograd.backward(y, dev_gy)
        res_host.copy_(y[:, -1].detach(), non_blocking=True)
        del y
    e2e_e.record(stream)
    torch.cuda.synchronize()
    barrier()
    return e2e_s.elapsed_time(e2e_e), h2d, d2h


def _report(args, rank, world, W, name, cfg, nb, total_ms, e2e_ms, f_ms, b_ms, h2d, d2h, peak_mb, launches, clk):
    if rank == 0:
        hbm, tc, peak_kind = _peaks()
        tok = W.tokens(cfg)  # whole job: all ranks together process the config
        fb, bb = algorithmic_bytes(cfg, nb)
        dom = ("backward", bb, b_ms) if b_ms >= f_ms else ("forward", fb, f_ms)
        achieved = dom[1] / (dom[2] * 1e-3) / 1e9
        out = {
            "metric": "tokens/s fwd+bwd",
            "value": tok * args.steps / (total_ms * 1e-3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": {4: "f32", 2: "bf16"}[cfg["dtype"].itemsize] + " inputs, f32 state",
            "data": "synthetic (seeded, BASELINE config distributions)",
            "config": {"workload": W.DESCRIPTION[name], "name": name, "global_batch": cfg["B"],
                       "seq_len": cfg["L"], "parallelism": f"batch-shard x{world}",
                       "l2": "inputs larger than L2" if fb > 126e6 else "inputs smaller than L2 (no flush)"},
            "fwd_ms": f_ms,
            "bwd_ms": b_ms,
            "fwd_tokens_per_s": tok / (f_ms * 1e-3),
            "peak_mb": peak_mb,
            "e2e": None if e2e_ms is None else {
                "value": tok * args.steps / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": {"bound": "hbm", "kernel": f"{cfg['kind']} {dom[0]}",
                         "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": _traffic(name, dom[0], nb, cfg),
                         "algorithmic_bytes_per_launch": dom[1],
                         "peak_source": f"{peak_kind} hbm_gbs"},
            **({"note": "per-step delta-rule recurrence: bound by FP32 issue and per-step latency on the "
                        "CUDA cores, not by HBM"} if cfg["kind"] == "gdn" else {}),
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_baseline(name)
        print(json.dumps(out), flush=True)


def run_reference(args):
    rank = _env_int("RANK", 0)
    if rank != 0:
        return
    W = importlib.import_module("mlx-recurrence_b200.workloads")
    name = args.config
    cfg = W.CONFIGS[name]
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import c_oracle
    ins, gy, frac, desc = cpu_sample(name)
    c_oracle.lib()
    for _ in range(args.warmup):
        _cpu_run(c_oracle, W, cfg, ins, gy)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _cpu_run(c_oracle, W, cfg, ins, gy)
    dt = time.perf_counter() - t0
    tok = W.tokens(cfg) * frac
    v = tok * args.steps / dt
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    out = {
        "impl": "reference",
        "metric": "tokens/s fwd+bwd",
        "value": v,
        "unit": "tokens/s",
        "n_gpus": _env_int("WORLD_SIZE", 1),
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded, BASELINE config distributions)",
        "config": {"workload": W.DESCRIPTION[name], "name": name, "global_batch": cfg["B"],
                   "seq_len": cfg["L"]},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{desc}; the reference (MLX/Metal) cannot run on this host, so its "
                                   "algorithm is timed as the float32 C restatement oracle/ckpt_scan.c"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c4", choices=["c0", "c1", "c2", "c3", "c4", "c5", "c2g", "c3a", "c6"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffer) timing")
    ap.add_argument("--check", action="store_true",
                    help="after timing, gather every rank's outputs and gradients and compare them on "
                         "rank 0 with the whole batch run on one GPU")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the config's batch (a smaller instance, e.g. for profiler captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
