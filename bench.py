"""Benchmark of the scan hot path: tokens/s of one forward+backward step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c4] [--impl ours|reference]

A step is one forward and one backward pass of the configured scan through
the public API (torch.autograd over libmlrec.so) on one batch of synthetic
inputs. The default workload is config c4 (SSD, bf16, B=32, L=16384, H=32,
Dh=64, N=128, seg=32), the configuration the scaling target is quoted on; the
default run also measures the GLA shape of the same target (c5) and the RG-LRU
(c2) and rotLRU (c3) configurations with the same steps and warm-up and reports
them under "extra" (every plug-in measured). Under torchrun (N > 1) every
rank takes a block of the same global problem - a range of batch rows, and of
heads (channels) when N does not divide the batch - with no collective on the
data path (strong scaling); the timed region is bracketed by a barrier and
device synchronisation and the reported time is the maximum over ranks.

Printed (rank 0, one JSON line): value = whole-job tokens/s with inputs
resident in HBM; e2e = the same step with host->device copies of every input
(and the upstream gradient) from pinned memory and device->host copies of y
and every input gradient into pinned memory inside the timed region; roofline
of the dominant kernel (algorithmic bytes / CUDA-event time), with the whole
step's and the forward's fractions of the same roofline; cpu_baseline =
the float32 C restatement of the reference algorithm (oracle/ckpt_scan.c) on
a bounded sample (median of three runs); clocks sampled during timing.

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
    ("c4d", "backward"): (1.210163e9 + 0.632409e9) / 2,
    ("c4d", "forward"): (0.676261e9 + 0.497439e9) / 2,
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


def cpu_baseline(name, reps=3):
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

def _setup():
    import torch
    import torch.distributed as dist

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

    return dict(pkg=importlib.import_module("mlx-recurrence_b200"),
                W=importlib.import_module("mlx-recurrence_b200.workloads"),
                lib=importlib.import_module("mlx-recurrence_b200._lib").load(),
                rank=rank, world=world, dev=dev, stream=torch.cuda.current_stream(dev), barrier=barrier)


def _prepare(ctx, name, batch=0):
    """The rank's block of config ``name``: inputs, upstream gradient, leaves."""
    import torch
    W = ctx["W"]
    cfg = dict(W.CONFIGS[name])
    if batch:
        cfg["B"] = batch
    blk = W.rank_block(name, ctx["rank"], ctx["world"], batch=cfg["B"])
    lcfg = W.local_config(name, blk)
    ins = W.make_inputs(name, ctx["dev"], seed=1000 + ctx["rank"], block=blk)
    gen = torch.Generator(device=ctx["dev"]).manual_seed(2000 + ctx["rank"])
    gy = torch.randn(W.output_shape(name, block=blk), generator=gen, device=ctx["dev"], dtype=torch.float32)
    leaves = [t.detach().requires_grad_(True) if t.dtype.is_floating_point else t for t in ins]
    return dict(name=name, cfg=cfg, lcfg=lcfg, blk=blk, ins=ins, gy=gy, leaves=leaves,
                fn=W.scan_fn(ctx["pkg"], name))


def _time_steps(ctx, P, steps, warmup):
    """W untimed warm-up steps, then K timed forward+backward steps bracketed by
    a barrier and device synchronisation, with CUDA events on the launching
    stream and clocks sampled meanwhile."""
    import torch
    fn, leaves, gy, stream, lib = P["fn"], P["leaves"], P["gy"], ctx["stream"], ctx["lib"]
    ev = lambda: torch.cuda.Event(enable_timing=True)
    for _ in range(warmup):
        for x in leaves:
            x.grad = None
        torch.autograd.backward(fn(*leaves), gy)
    torch.cuda.synchronize()
    n_launch0 = lib.mr_launch_count()
    torch.cuda.reset_peak_memory_stats(ctx["dev"])
    ctx["barrier"]()
    torch.cuda.synchronize()
    with ClockSampler(_gpu_uuid(ctx["dev"])) as clk:
        e_start, e_end = ev(), ev()
        e_start.record(stream)
        marks = []
        for _ in range(steps):
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
        ctx["barrier"]()
    return dict(total_ms=e_start.elapsed_time(e_end), steps=steps,
                f_ms=statistics.mean(a.elapsed_time(b) for a, b, _ in marks),
                b_ms=statistics.mean(b.elapsed_time(c) for _, b, c in marks),
                launches=lib.mr_launch_count() - n_launch0,
                peak_mb=torch.cuda.max_memory_allocated(ctx["dev"]) / 2 ** 20, clk=clk)


def _max_over_ranks(ctx, vals):
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device=ctx["dev"])
    if ctx["world"] > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def run_ours(args):
    import torch
    import torch.distributed as dist
    ctx = _setup()
    P = _prepare(ctx, args.config, args.batch)
    M = _time_steps(ctx, P, args.steps, args.warmup)
    e2e_ms, h2d, d2h = None, 0, 0
    if not args.no_e2e:
        e2e_ms, h2d, d2h = _e2e(args, P["fn"], P["ins"], P["gy"], ctx["dev"], ctx["stream"], ctx["barrier"],
                                lambda: torch.cuda.Event(enable_timing=True))
    mx = _max_over_ranks(ctx, [M["total_ms"], e2e_ms or 0.0, M["f_ms"], M["b_ms"]])
    M["total_ms"], M["f_ms"], M["b_ms"] = mx[0], mx[2], mx[3]
    e2e_ms = mx[1] if e2e_ms is not None else None
    if args.check:
        _check(args, ctx, P)
    meta = {k: P[k] for k in ("name", "cfg", "lcfg")}
    extra = {}
    if args.config == "c4" and not args.no_extra:
        # the GLA half of the target shape (B=32, L=16384, H=32, Dh=64), then the two diagonal
        # scans at their configurations (c2 RG-LRU, c3 rotLRU): every plug-in measured with the
        # same warm-up; c5 with the same steps, the diagonal scans (0.4 and 1.3 ms a step) with
        # ten times as many, so that their timed regions are not a few milliseconds (args.batch
        # applies to c4 and c5 only)
        del P
        for name, mult in (("c5", 1), ("c2", 10), ("c3", 10)):
            torch.cuda.empty_cache()
            Pk = _prepare(ctx, name, args.batch if name == "c5" else 0)
            Mk = _time_steps(ctx, Pk, args.steps * mult, args.warmup)
            Mk["total_ms"], Mk["f_ms"], Mk["b_ms"] = _max_over_ranks(ctx, [Mk["total_ms"], Mk["f_ms"], Mk["b_ms"]])
            extra[name] = ({k: Pk[k] for k in ("name", "cfg", "lcfg")}, Mk)
            del Pk
    if ctx["rank"] == 0:
        out = _report(args, ctx, meta, M, e2e_ms, h2d, d2h)
        if extra:
            out["extra"] = {k: _metrics(args, ctx, Pk, Mk) for k, (Pk, Mk) in extra.items()}
        if ctx["world"] == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_baseline(args.config)
        print(json.dumps(out), flush=True)
    if ctx["world"] > 1:
        dist.barrier()
        dist.destroy_process_group()


def _check(args, ctx, P):
    """After timing: every rank's outputs and gradients gathered over the process
    group (NCCL), the shared parameters' gradients summed over ranks, and rank 0
    runs the whole problem on its GPU and compares (max|diff| / max|ref|). The
    units are independent, so the gathered results equal the 1-GPU run up to the
    order of the cross-rank sums."""
    import torch
    S = importlib.import_module("mlx-recurrence_b200.sharding")
    W = ctx["W"]
    fn, ins, leaves, gy, cfg = P["fn"], P["ins"], P["leaves"], P["gy"], P["cfg"]
    ax, q = W.UNIT_AXIS[cfg["kind"]]
    B, U = cfg["B"], cfg[ax]
    for x in leaves:
        x.grad = None
    y = fn(*leaves)
    torch.autograd.backward(y, gy)
    blocked = lambda x: x.dim() >= 3  # [B, L, units (x values), ...]; lower ranks: per-unit parameters

    def gather_param(x):  # a per-unit parameter, re-expanded like the caller's view
        if x.dim() == 2 and x.stride(1) == 0:
            return _gather_param(S, x[:, :1].detach(), B, U, q).expand(U, x.shape[1])
        return _gather_param(S, x.detach(), B, U, q)

    full_in = [S.gather_blocks(x.detach(), B, U, q) if blocked(x) else gather_param(x) for x in ins]
    y_all = S.gather_blocks(y.detach(), B, U, q)
    gy_all = S.gather_blocks(gy, B, U, q)
    g_all = []
    for x in leaves:
        g = x.grad
        if g is None:
            g_all.append(None)
        elif blocked(x):
            g_all.append(S.gather_blocks(g, B, U, q))
        else:  # a shared parameter: the sum of the ranks' partial sums
            g_all.append(S.sum_unit_param(g.contiguous(), B, U, q))
    if ctx["rank"] != 0:
        return
    # (a broadcast parameter keeps its stride-0 view, so the same kernel path runs)
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
    print(json.dumps({"check": {"world": ctx["world"], "config": args.config, "max_rel_err": max(errs.values()),
                                "rel_err": errs}}), flush=True)


def _gather_param(S, x, B, U, q):
    """A per-unit parameter slice [u0:u1, ...] of every rank assembled into [U, ...]
    (ranks sharing a unit range hold the same values)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return x
    _, _, u0, u1 = S.block_of(B, U, dist.get_rank(), dist.get_world_size(), q)
    full = torch.zeros((U,) + tuple(x.shape[1:]), dtype=torch.float64, device=x.device)
    cnt = torch.zeros((U,), dtype=torch.float64, device=x.device)
    full[u0:u1] = x.double()
    cnt[u0:u1] = 1
    dist.all_reduce(full)
    dist.all_reduce(cnt)
    return (full / cnt.view((U,) + (1,) * (x.dim() - 1))).to(x.dtype).contiguous()


def _e2e(args, fn, ins, gy, dev, stream, barrier, ev):
    """Same step through the public API with host buffers: per step, H2D copies
    of every input and of the upstream gradient from pinned memory,
    forward+backward, and D2H copies into pinned memory of the step's output
    y and of every input gradient (what a caller holding host buffers reads
    back). The copies are pipelined as a data loader would: each step's batch
    goes through in slices of whole batch rows (every scan is independent per
    batch row), slice i+1's inputs stream in on one copy stream (into the other
    of two device buffers) while slice i computes and slice i-1's results
    stream out on a second copy stream, so the two PCIe directions run
    concurrently except for one slice at each end of the run. The gradients of
    the shared parameters (SSD's A_neg) are summed over a step's slices on the
    device and read back once per step. Every step's copies happen inside the
    timed region, which ends once the last step's results are in host memory.
    Returns (ms for all steps, H2D bytes/step, D2H bytes/step)."""
    import torch
    # A tensor broadcast along its last axis (SSD's per-head A_neg) travels as
    # its [.., 1] base and is re-expanded on the device, as a caller would.
    def compact(t):
        t = t.detach()
        if t.dim() > 0 and t.stride(-1) == 0:
            return t[..., :1].contiguous(), tuple(t.shape)
        return t.contiguous(), None

    B = gy.shape[0]
    parts = next(p for p in (4, 2, 1) if B % p == 0)
    rows = B // parts
    per_row = [x.dim() >= 3 for x in ins]  # [B, L, ...] tensors; lower ranks: shared parameters
    packed = [compact(t) for t in ins]
    host_ins = [c.to("cpu").pin_memory() for c, _ in packed]
    shapes = [s for _, s in packed]
    host_gy = gy.to("cpu").pin_memory()

    def part_of(t, p, rowwise=True):  # batch rows of slice p (a view; contiguous for [B, ...])
        return t[p * rows:(p + 1) * rows] if rowwise else t

    bufs = [([torch.empty_like(part_of(h, 0, r), device=dev) for h, r in zip(host_ins, per_row)],
             torch.empty_like(part_of(gy, 0))) for _ in range(2)]
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event(), torch.cuda.Event()]
    buf_free = [torch.cuda.Event(), torch.cuda.Event()]
    out_ready = torch.cuda.Event()

    def h2d(p, j):  # slice p's inputs into device buffer j once the slice before last has read it
        h2d_s.wait_event(buf_free[j])
        with torch.cuda.stream(h2d_s), torch.no_grad():
            for d, h, r in zip(bufs[j][0], host_ins, per_row):
                d.copy_(part_of(h, p, r), non_blocking=True)
            bufs[j][1].copy_(part_of(host_gy, p), non_blocking=True)
        in_ready[j].record(h2d_s)

    def compute(p, j, host_out, acc):  # forward+backward of slice p on the main stream, results out
        stream.wait_event(in_ready[j])
        leaves, xs = [], []
        for d, s_ in zip(bufs[j][0], shapes):
            x = d.detach().requires_grad_(True)
            leaves.append(x)
            xs.append(x.expand(s_) if s_ is not None else x)
        y = fn(*xs)
        torch.autograd.backward(y, bufs[j][1])
        buf_free[j].record(stream)
        grads = [x.grad for x in leaves]
        if host_out is None:  # untimed first call: the host result buffers (whole batch)
            outs = [y.detach()] + grads
            return [torch.empty((o.shape[0] * parts,) + tuple(o.shape[1:]) if r else o.shape, dtype=o.dtype,
                                pin_memory=True) for o, r in zip(outs, [True] + per_row)], None
        # the shared parameters' gradients, summed over the step's slices (a fresh sum each step:
        # the allocator keeps the previous one until its copy is done)
        with torch.no_grad():
            acc = [None if r else (g.clone() if p == 0 else a.add_(g)) for g, r, a in
                   zip(grads, per_row, acc if acc is not None else [None] * len(grads))]
        out_ready.record(stream)
        d2h_s.wait_event(out_ready)
        outs = [y.detach()] + [g for g, r in zip(grads, per_row) if r]
        hosts = [host_out[0]] + [h for h, r in zip(host_out[1:], per_row) if r]
        with torch.cuda.stream(d2h_s), torch.no_grad():
            for h, o in zip(hosts, outs):
                part_of(h, p).copy_(o, non_blocking=True)
            if p == parts - 1:  # the step's shared-parameter gradients, once
                for h, a in zip(host_out[1:], acc):
                    if a is not None:
                        h.copy_(a, non_blocking=True)
        for o in outs + ([a for a in acc if a is not None] if p == parts - 1 else []):
            o.record_stream(d2h_s)  # the allocator keeps them until the copies are done
        return host_out, acc

    def run(n):
        for e in buf_free:
            e.record(stream)
        pieces = [p for _ in range(n) for p in range(parts)]
        acc = None
        h2d(0, 0)
        for i, p in enumerate(pieces):
            if i + 1 < len(pieces):
                h2d(pieces[i + 1], (i + 1) % 2)
            _, acc = compute(p, i % 2, host_out, acc)
        stream.wait_stream(d2h_s)

    for e in buf_free:
        e.record(stream)
    h2d(0, 0)
    host_out, _ = compute(0, 0, None, None)
    run(2)  # warm the copy paths
    # the bytes copied: every batch row once, the shared parameters once per slice
    h2d_b = sum(part_of(t, 0, r).numel() * t.element_size() * parts
                for t, r in zip(host_ins, per_row)) + host_gy.numel() * host_gy.element_size()
    d2h_b = sum(t.numel() * t.element_size() for t in host_out)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e2e_s, e2e_e = ev(), ev()
    e2e_s.record(stream)
    run(args.steps)
    e2e_e.record(stream)
    torch.cuda.synchronize()
    barrier()
    return e2e_s.elapsed_time(e2e_e), h2d_b, d2h_b


def _ckpt_spacing(ctx, cfg):
    """Checkpoint spacing the plug-in wrappers use for this config (the fastest
    path's; the final state is the same for any spacing)."""
    L = importlib.import_module("mlx-recurrence_b200._lib")
    code = L.DTYPE_CODE[cfg["dtype"]]
    if cfg["kind"] == "ssd":  # one rate per head (the stride-0 view along N), or dense
        asn = 1 if cfg.get("dense_a") else 0
        return int(ctx["lib"].mr_ssd_preferred_seg(code, cfg["L"], cfg["Dh"], cfg["N"], cfg["seg"], asn))
    if cfg["kind"] == "gla":
        return int(ctx["lib"].mr_gla_preferred_seg(code, cfg["L"], cfg["Dh"], cfg["seg"]))
    return cfg["seg"]


def _metrics(args, ctx, P, M):
    """Throughput, per-phase times and the dominant kernel's roofline."""
    W = ctx["W"]
    name, cfg, lcfg = P["name"], P["cfg"], P["lcfg"]
    hbm, tc, peak_kind = _peaks()
    tok = W.tokens(cfg)  # whole job: all ranks together process the config
    fb, bb = algorithmic_bytes(lcfg, lcfg["B"])
    f_ms, b_ms = M["f_ms"], M["b_ms"]
    dom = ("backward", bb, b_ms) if b_ms >= f_ms else ("forward", fb, f_ms)
    achieved = dom[1] / (dom[2] * 1e-3) / 1e9
    ax, _ = W.UNIT_AXIS[cfg["kind"]]
    traffic = _traffic(name, dom[0], lcfg["B"] * lcfg[ax] / cfg[ax], cfg)
    wb, wu = importlib.import_module("mlx-recurrence_b200.sharding").rank_grid(
        cfg["B"], cfg[ax], ctx["world"], W.UNIT_AXIS[cfg["kind"]][1])
    unit = {"H": "head", "D": "channel", "Dp": "pair"}[ax]
    return {
        "value": tok * M["steps"] / (M["total_ms"] * 1e-3),
        "unit": "tokens/s",
        "ms_per_step": M["total_ms"] / M["steps"],
        "steps": M["steps"],
        "config": {"workload": W.DESCRIPTION[name], "name": name, "global_batch": cfg["B"], "seq_len": cfg["L"],
                   "ckpt_spacing": _ckpt_spacing(ctx, cfg),
                   "parallelism": f"{wb} batch x {wu} {unit} blocks over {ctx['world']} GPU(s), no collective",
                   "l2": "inputs larger than L2" if fb > 126e6 else "inputs smaller than L2 (no flush)"},
        "fwd_ms": f_ms,
        "bwd_ms": b_ms,
        "fwd_tokens_per_s": tok / (f_ms * 1e-3),
        "peak_mb": M["peak_mb"],
        "roofline": {"bound": "hbm", "kernel": f"{cfg['kind']} {dom[0]}",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": traffic,
                     "algorithmic_bytes_per_launch": dom[1],
                     "peak_source": f"{peak_kind} hbm_gbs",
                     # the whole forward+backward step against the same roofline (this rank's
                     # algorithmic bytes over its share of the step time), and the forward alone
                     "step_frac": (fb + bb) / (M["total_ms"] / M["steps"] * 1e-3) / 1e9 / hbm,
                     "fwd_frac": fb / (f_ms * 1e-3) / 1e9 / hbm},
        **({"note": "per-step delta-rule recurrence: bound by FP32 issue and per-step latency on the "
                    "CUDA cores, not by HBM"} if cfg["kind"] == "gdn" else {}),
        "gpu_launches": int(M["launches"]),
        "clocks": M["clk"].summary(),
    }


# The reference's only published numbers for this path (Apple M3 Max through Metal,
# README.md:86-88 and docs/validation/V3_VALIDATION_REPORT_20260610.md:32-34): one
# forward+backward step at B=3, L=512, H=12, Dh=64, seg=32 (SSD's N not stated), in ms.
_PUBLISHED_STEP_MS = {"c0": 17.34, "c1": 12.06}


def _report(args, ctx, P, M, e2e_ms, h2d, d2h):
    cfg = P["cfg"]
    m = _metrics(args, ctx, P, M)
    tok = ctx["W"].tokens(cfg)
    pub = _PUBLISHED_STEP_MS.get(P["name"])
    out = {
        "metric": "tokens/s fwd+bwd",
        "value": m["value"],
        "unit": m.pop("unit"),
        "n_gpus": ctx["world"],
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": m.pop("ms_per_step"),
        "higher_is_better": True,
        "scaling": "strong",
        # value over the published tokens/s of the same shape (c0, c1 only)
        "vs_baseline": None if pub is None else m["value"] / (tok / (pub * 1e-3)),
        **({} if pub is None else {"vs_baseline_note": f"published: {pub} ms per fwd+bwd step on an Apple M3 Max "
                                                       "(Metal), same shape"}),
        "dtype": {4: "f32", 2: "bf16"}[cfg["dtype"].itemsize] + " inputs, f32 state",
        "data": "synthetic (seeded, BASELINE config distributions)",
        "config": m.pop("config"),
        "e2e": None if e2e_ms is None else {
            "value": tok * args.steps / (e2e_ms * 1e-3), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "copies": "H2D of every input and grad_y from pinned memory; D2H of y and every input gradient "
                      "into pinned memory; inside the timed region, each step's batch in row slices "
                      "pipelined on two copy streams (double-buffered device inputs)"},
    }
    m.pop("value")
    out.update(m)
    return out


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
    ap.add_argument("--config", default="c4", choices=["c0", "c1", "c2", "c3", "c4", "c4d", "c5", "c2g", "c3a", "c6"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffer) timing")
    ap.add_argument("--no-extra", action="store_true",
                    help="with the default c4, skip the extra measurements (c5 GLA at the same shape, c2 RG-LRU, c3 rotLRU)")
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
