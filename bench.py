#!/usr/bin/env python
"""Benchmark: slice+deslice coupling round, forward + backward, in Mpoints/s.

A step is one coupling round over one batch of synthetic points: slice
forward, token normalisation z_num / (s + 1e-5) (identity mix), deslice
forward, and the backward of sum(out * r) (deslice backward, the mix's
backward, slice backward). Workload: B=1, N=1,048,576
points per GPU, H=8, D=DV=32, G=32, fp32, ieee dot level, per-head W (H, G, D)
~ N(0, 1/D), b (H, G) ~ N(0, 0.02^2), tau ~ U[0.3, 1.0], x_mid, fx_mid, r
~ N(0, 1), seeded. Inputs are larger than L2 (1 GiB each), so no L2 flush is
needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...

One JSON line on rank 0. With N > 1 GPUs each rank holds its own N points
(weak scaling); the per-rank slice partials and token gradients are summed
across ranks in rank order (all-gather + ordered sum over NCCL) and the
parameter gradients likewise, inside the timed step.

``--impl reference`` times the reference's own CPU implementation of the
round -- its eager op math, restated in ``oracle/eager_torch.py`` -- on the
host cores, on a bounded sample of the workload (rank 0 only).
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "slice+deslice fwd+bwd Mpoints/s at N=1M,G=32 (1–8 GPU); % of HBM roofline"
UNIT = "Mpoints/s"
EPS = 1e-5

CONFIGS = {
    # configs[1] of the baseline: per-GPU shard of 2^20 points (weak scaling)
    "cfg2": dict(B=1, N=1 << 20, H=8, D=32, DV=32, G=32, weight="hgd", tau="uniform",
                 dtype=torch.float32, dot="ieee", split=False),
    # config 2's shape with bf16 point tensors (a bf16 layer's x_mid / fx_mid)
    "cfg2-bf16": dict(B=1, N=1 << 20, H=8, D=32, DV=32, G=32, weight="hgd", tau="uniform",
                      dtype=torch.bfloat16, dot="bf16", split=False),
    "cfg1": dict(B=1, N=16384, H=8, D=32, DV=32, G=32, weight="gd", tau="half",
                 dtype=torch.float32, dot="ieee", split=False),
    "cfg3": dict(B=2, N=262144, H=8, D=32, DV=64, G=1024, weight="bhgd", tau="half",
                 dtype=torch.bfloat16, dot="bf16", split=False, bias=False),
    # 2^24 points split over the ranks (strong scaling)
    "cfg5": dict(B=1, N=1 << 24, H=8, D=32, DV=32, G=64, weight="hgd", tau="half",
                 dtype=torch.float32, dot="ieee", split=True),
}
# (N, H, 32) fp32 tensors each op of the tied round reads or writes: slice
# forward x, fx; deslice forward x, out; dtokens pass x, d_out; coupled
# backward x, fx, d_out, dx, dfx -- 11 in all, the round's credited bytes
# (the reference's own count, bench_kernels.py:45: 2 + 2 + 4 + 3).
UNITS = {"slice_fwd": 2, "deslice_fwd": 2, "dtokens": 2, "coupled_bwd": 5}
# the kernel each op runs (for the traffic of the committed ncu capture)
KERNEL_OF = {"slice_fwd": "slice_fwd", "deslice_fwd": "deslice_fwd", "dtokens": "slice_fwd",
             "coupled_bwd": "coupled_bwd"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference", "reference-triton"), default="ours",
                    help="reference: the reference's CPU path (the driver's arm); "
                         "reference-triton: the unmodified reference's own Triton GPU kernels "
                         "from baseline/_ref on this GPU, the GPU bar")
    ap.add_argument("--config", choices=sorted(CONFIGS) + ["cfg4"], default="cfg2")
    ap.add_argument("--n", type=int, default=None, help="override the point count")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--bf16-autocast", action="store_true",
                    help="config 4: train under torch.autocast(bfloat16) (bf16 activations, "
                         "the coupling ops on bf16 point tensors)")
    ap.add_argument("--tf32-gemms", action="store_true",
                    help="config 4: let the model's torch GEMMs use TF32 (the coupling ops "
                         "stay exact fp32 either way)")
    ap.add_argument("--compile", action="store_true",
                    help="config 4: run both models under torch.compile(fullgraph=True)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the op-by-op and reverse-order figures")
    ap.add_argument("--cpu-sample", type=int, default=None,
                    help="points per CPU step (default: the workload's points per GPU, "
                         "at most 2^20)")
    return ap.parse_args()


# --------------------------------------------------------------------------- inputs

def make_inputs(cfg, n, device, seed):
    """Seeded synthetic leaves of one shard: x_mid, fx_mid, W, b, tau, r."""
    gen = torch.Generator(device=device).manual_seed(seed)
    B, H, D, DV, G = cfg["B"], cfg["H"], cfg["D"], cfg["DV"], cfg["G"]
    dt = cfg["dtype"]
    rn = lambda *s: torch.randn(*s, generator=gen, device=device)  # noqa: E731
    x = rn(B, n, H, D).to(dt)
    fx = rn(B, n, H, DV).to(dt)
    r = rn(B, n, H, DV).to(dt)
    if cfg["weight"] == "gd":
        W, b = rn(G, D) / D ** 0.5, 0.02 * rn(G)
    elif cfg["weight"] == "hgd":
        W, b = rn(H, G, D) / D ** 0.5, 0.02 * rn(H, G)
    else:  # tokens projected by a random linear map (parity_ops.Case), scaled to N(0, 1/D)
        Ht = 64
        Wk = rn(Ht, H * D) / (Ht * D) ** 0.5
        W = (rn(B, G, Ht) @ Wk).view(B, G, H, D).permute(0, 2, 1, 3).contiguous()
        b = None
    if not cfg.get("bias", True):
        b = None
    if cfg["tau"] == "uniform":
        tau = 0.3 + 0.7 * torch.rand(H, generator=gen, device=device)
    else:
        tau = torch.full((H,), 0.5, device=device)
    W = W.to(dt) if dt != torch.float32 else W
    return x, fx, W, b, tau, r


# --------------------------------------------------------------------------- steps

def coupling_step(K, x, fx, W, b, tau, r, group=None):
    """Forward + backward of one round through the public API: one
    ``fused_coupling`` (slice -> z_num / (s + eps) -> deslice, tied backward),
    points sharded over ``group``."""
    from flashslice_b200 import sharded
    out = K.fused_coupling(x, fx, W, b, tau, eps=EPS, group=group)
    out.backward(r)
    if group is not None:
        sharded.reduce_grads([W, b, tau], group)
    return out


def zero_grads(*ts):
    for t in ts:
        if t is not None:
            t.grad = None


def op_by_op_step(K, x, fx, W, b, tau, r):
    """The same round through the reference's own surface: ``fused_slice``,
    the normalisation, ``fused_deslice`` and autograd's backward of the two
    ops (deslice backward, slice backward, and the sum of their dx)."""
    z, s = K.fused_slice(x, fx, W, b, tau)
    out = K.fused_deslice(x, W, b, tau, z / (s + EPS)[..., None])
    out.backward(r)
    return out


def reverse_step(K, x, fx, W, b, tau, tok, r, rz, rs):
    """The reverse call order of config 2: deslice first (tokens given, the
    per-point statistics returned), then the slice of the same points with
    those statistics handed in, forward and backward of
    sum(out r) + sum(z_num rz) + sum(s rs)."""
    out, st = K.fused_deslice(x, W, b, tau, tok, return_stats=True)
    z, s = K.fused_slice(x, fx, W, b, tau, stats=st)
    torch.autograd.backward([out, z, s], [r, rz, rs])
    return out


def timed_rounds(step, steps, warmup=2):
    """Mean device time (ms) of ``steps`` calls of ``step`` after ``warmup``."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


PROFILE_SUMMARY = os.path.join(ROOT, "profiles", "tc_kernels_ncu_full_small.md")


def profile_traffic(op, rows):
    """DRAM bytes (read + write) of one launch of `op`'s kernel, from the
    committed ncu capture summary (measured at 8M point rows and scaled by
    the rows processed, traffic growing in proportion); None without it."""
    try:
        with open(PROFILE_SUMMARY) as f:
            lines = f.read().splitlines()
    except OSError:
        return None
    for ln in lines:
        cells = [c.strip() for c in ln.strip().strip("|").split("|")]
        if len(cells) == 2 and cells[0] == op:
            try:
                return int(int(cells[1]) * rows / float(8 << 20))
            except ValueError:
                return None
    return None


# Each per-op timing rep starts on an idle GPU (a synchronize ends the last
# one); a device-side sleep of about 2 ms enqueued before the first event
# keeps the GPU busy while the host dispatches the first op, so that its
# time, like the others', is device time and not the host's dispatch
# latency.
_HIDE_DISPATCH_CYCLES = 4_000_000


def op_timings(K, x, fx, W, b, tau, r, dot, reps=3):
    """Per-op device time (ms) of one tied round, each op launched directly
    on the current stream between CUDA events; median over reps. The ops are
    the ones ``fused_coupling`` runs: slice forward, deslice forward, the
    dtokens pass (a slice forward of d_out) and the coupled backward."""
    ops = torch.ops.flashslice
    bb = b if b is not None else W.new_zeros(W.shape[-2])
    Wd, bd, td = W.detach(), bb.detach(), tau.detach()
    xd, fd = x.detach(), fx.detach()
    times = {k: [] for k in UNITS}
    for _ in range(reps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
        torch.cuda._sleep(_HIDE_DISPATCH_CYCLES)
        ev[0].record()
        z, s = ops.flash_slice(xd, fd, Wd, bd, td, dot)
        ev[1].record()
        den = (s + EPS)[..., None]
        tok = z / den
        ev[2].record()
        ops.flash_deslice(xd, Wd, bd, td, tok, dot)
        ev[3].record()
        dtok, _ = ops.flash_slice(xd, r, Wd, bd, td, dot)
        ev[4].record()
        dz = dtok / den
        ds = -(dtok * z).sum(-1) / (s + EPS) ** 2
        ev[5].record()
        ops.coupled_bwd(xd, fd, r, Wd, bd, td, tok, dz, ds, dot)
        ev[6].record()
        torch.cuda.synchronize()
        times["slice_fwd"].append(ev[0].elapsed_time(ev[1]))
        times["deslice_fwd"].append(ev[2].elapsed_time(ev[3]))
        times["dtokens"].append(ev[3].elapsed_time(ev[4]))
        times["coupled_bwd"].append(ev[5].elapsed_time(ev[6]))
    return {k: statistics.median(v) for k, v in times.items()}


def op_timings_blocked(x, fx, W, b, tau, r, dot, reps=3):
    """Per-op device time (ms) of one round on the blocked family, the ops
    ``fused_coupling`` runs there: slice forward (statistics out), deslice
    forward (statistics in), and the two backward ops. Median over reps."""
    from flashslice_b200.kernels import blocked  # noqa: F401  (registers the ops)
    ops = torch.ops.flashslice
    bb = b if b is not None else W.new_zeros(W.shape[-2])
    Wd, bd, td = W.detach(), bb.detach(), tau.detach()
    xd, fd = x.detach(), fx.detach()
    times = {k: [] for k in BLK_FLOPS}
    for _ in range(reps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
        torch.cuda._sleep(_HIDE_DISPATCH_CYCLES)
        ev[0].record()
        z, s, st = ops.slice_blk(xd, fd, Wd, bd, td, None, dot)
        ev[1].record()
        den = (s + EPS)[..., None]
        tok = z / den
        ev[2].record()
        ops.deslice_blk(xd, Wd, bd, td, tok, st, dot)
        ev[3].record()
        dx1, dtok, _, _, _ = ops.deslice_blk_bwd(xd, Wd, bd, td, tok, st, r, dot)
        ev[4].record()
        dz = dtok / den
        ds = -(dtok * z).sum(-1) / (s + EPS) ** 2
        ev[5].record()
        ops.slice_blk_bwd(xd, fd, Wd, bd, td, st, dz, ds, dot)
        ev[6].record()
        torch.cuda.synchronize()
        times["slice_fwd"].append(ev[0].elapsed_time(ev[1]))
        times["deslice_fwd"].append(ev[2].elapsed_time(ev[3]))
        times["deslice_bwd"].append(ev[3].elapsed_time(ev[4]))
        times["slice_bwd"].append(ev[5].elapsed_time(ev[6]))
    return {k: statistics.median(v) for k, v in times.items()}


# Algorithmic flops per point-head of each blocked op, in units of 2 G
# (multiply-adds of the minimal dots): slice forward logits + pool (D + DV),
# deslice forward logits + scatter (D + DV), each backward logits, two value
# dots, dx and dW (3 D + 2 DV): 2 G (8 D + 6 DV) for the round.
BLK_FLOPS = {"slice_fwd": lambda D, DV: D + DV, "deslice_fwd": lambda D, DV: D + DV,
             "deslice_bwd": lambda D, DV: 3 * D + 2 * DV,
             "slice_bwd": lambda D, DV: 3 * D + 2 * DV}


# --------------------------------------------------------------------------- clocks

class ClockSampler:
    """SM clock and clock-event reasons of this rank's GPU over the timed
    region: NVML read every 5 ms by a thread (the timed region of a few
    tens of ms holds no sample of nvidia-smi's 200 ms loop), or nvidia-smi
    samples when NVML cannot be loaded. Read-only queries."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    # NVML clock-event reason bits of the names above, and the power brake
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}
    PERIOD_S = 0.005

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None
        self.nvml = None
        self.samples = []

    def _handle(self, nv):
        try:
            pr = torch.cuda.get_device_properties(self.index)
            bus = "%08x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.index)

    def _sample(self):
        nv, h = self.nvml
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        self.samples.append((float(sm), float(mx), int(rs)))

    def _loop(self):
        while not self.done.is_set():
            try:
                self._sample()
            except Exception:
                return
            self.done.wait(self.PERIOD_S)

    def start(self):
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            self.nvml = (nv, self._handle(nv))
            self.done = threading.Event()
            self.thread = threading.Thread(target=self._loop, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.nvml = None
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "200", "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def _summary(self, sm, mx, reasons, source):
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm), "source": source}

    def stop(self):
        if self.nvml is not None:
            self.done.set()
            self.thread.join(timeout=5)
            nv = self.nvml[0]
            try:
                if not self.samples:
                    self._sample()
            except Exception:
                pass
            try:
                nv.nvmlShutdown()
            except Exception:
                pass
            reasons = {name for name, bit in self.BITS.items()
                       if any(r & bit for _, _, r in self.samples)}
            return self._summary([s[0] for s in self.samples], [s[1] for s in self.samples],
                                 reasons, "nvml every %d ms" % round(1e3 * self.PERIOD_S))
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) < 9:
                        continue
                    try:
                        sm.append(float(parts[1]))
                        mx.append(float(parts[2]))
                    except ValueError:
                        continue
                    for name, val in zip(self.NAMES, parts[5:9]):
                        if val.lower() == "active":
                            reasons.add(name)
        finally:
            os.unlink(self.path)
        return self._summary(sm, mx, reasons, "nvidia-smi every 200 ms")


# --------------------------------------------------------------------------- CPU legs

def cpu_round_time(cfg, n, threads, reps, seed=0):
    """Median seconds of one eager coupling round (the reference's op math on
    the CPU, ``oracle/eager_torch.py``) over ``n`` points."""
    from oracle import eager_torch as E
    torch.set_num_threads(threads)
    x, fx, W, b, tau, r = make_inputs(cfg, n, "cpu", seed)
    x, fx = x.float(), fx.float()
    W = W.float()
    times = []
    for i in range(reps + 1):
        leaves = [t.detach().requires_grad_(True) if t is not None else None
                  for t in (x, fx, W, b, tau)]
        t0 = time.perf_counter()
        E.coupling_round(*leaves, r.float(), eps=EPS)
        if i:
            times.append(time.perf_counter() - t0)
    return statistics.median(times)


def cpu_baseline(cfg, sample, reps=3):
    threads = os.cpu_count() or 1
    sec = cpu_round_time(cfg, sample, threads, reps)
    return {"value": round(cfg["B"] * sample / sec / 1e6, 4), "unit": UNIT, "cores": threads,
            "kind": "port",
            "sample": "one eager coupling round (oracle/eager_torch.py, the reference's op math) "
                      "over %d points of the same shape, median of %d" % (sample, reps)}


def cpu_sample(args, cfg):
    """Points per CPU step: the workload's points per GPU (config 2: all
    2^20, so the CPU arm runs the same configuration), at most 2^20."""
    if args.cpu_sample is not None:
        return args.cpu_sample
    return min(cfg["N"], 1 << 20)


def run_reference_triton(args, cfg):
    """The same round through the unmodified reference (``baseline/_ref``,
    installed from the reference's source tree) on one GPU: its public
    ``fused_slice`` / ``fused_deslice`` and autograd, its Triton kernels at
    its own default settings (ieee dot mode, the tile table it picks for
    this GPU). Device-resident inputs, CUDA-event timing, the same metric,
    config and seeds as our arm."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    ref = os.path.join(ROOT, "baseline", "_ref")
    why = None
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        why = "the reference has no multi-GPU path; this leg runs on one GPU"
    elif not os.path.isdir(os.path.join(ref, "flashslice")):
        why = "baseline/_ref is not installed (pip install --target baseline/_ref <reference>)"
    elif not torch.cuda.is_available():
        why = "no CUDA device"
    if why:
        print(json.dumps({"impl": "reference-triton", "unavailable": why}), flush=True)
        return
    sys.path.insert(0, ref)
    import flashslice.kernels as R  # the reference's own package
    device = torch.device("cuda", 0)
    torch.backends.cuda.matmul.allow_tf32 = False
    n = cfg["N"]
    x, fx, W, b, tau, r = make_inputs(cfg, n, device, 1234)
    _, _, W, b, tau, _ = make_inputs(cfg, 1, device, 99)
    for t in (x, fx, W, b, tau):
        if t is not None:
            t.requires_grad_(True)

    def step():
        zero_grads(x, fx, W, b, tau)
        z, s = R.fused_slice(x, fx, W, b, tau)
        out = R.fused_deslice(x, W, b, tau, z / (s + EPS)[..., None])
        out.backward(r)

    ms = timed_rounds(step, args.steps, max(args.warmup, 1))
    points = cfg["B"] * n
    value = points / (ms * 1e-3) / 1e6
    unit_bytes = points * cfg["H"] * cfg["D"] * x.element_size()
    peak = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = json.load(f).get("hbm_gbs")
    except (OSError, ValueError):
        pass
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32" if cfg["dtype"] == torch.float32 else "bf16",
            "data": "synthetic (seeded torch.Generator on the device)",
            "impl": "reference-triton",
            "config": {"workload": args.config, "B": cfg["B"], "N": n, "H": cfg["H"],
                       "D": cfg["D"], "DV": cfg["DV"], "G": cfg["G"], "weight": cfg["weight"],
                       "dot": "the reference's default (ieee)",
                       "path": "flashslice.kernels.fused_slice + fused_deslice + autograd "
                               "(its Triton kernels), unmodified, from baseline/_ref"},
            "round_frac": (round(11 * unit_bytes / (ms * 1e-3) / 1e9 / peak, 4)
                           if peak and cfg["G"] <= 64 else None)}
    print(json.dumps(line), flush=True)


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    sample = cpu_sample(args, cfg)
    from oracle import eager_torch as E
    torch.set_num_threads(threads)
    x, fx, W, b, tau, r = make_inputs(cfg, sample, "cpu", 0)
    x, fx, W, r = x.float(), fx.float(), W.float(), r.float()

    def step():
        leaves = [t.detach().requires_grad_(True) if t is not None else None
                  for t in (x, fx, W, b, tau)]
        E.coupling_round(*leaves, r, eps=EPS)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    sec = (time.perf_counter() - t0) / args.steps
    value = cfg["B"] * sample / sec / 1e6
    line = {"metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": args.config if sample == cfg["N"] else
                       args.config + " (CPU sample)", "B": cfg["B"], "N": sample,
                       "H": cfg["H"], "D": cfg["D"], "DV": cfg["DV"], "G": cfg["G"],
                       "same_config": sample == cfg["N"]},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads,
                             "kind": "port",
                             "sample": "eager coupling round over %d points per step" % sample},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- config 4

MODEL4 = dict(space_dim=3, fun_dim=1, out_dim=4, n_hidden=256, n_heads=8, n_layers=8,
              slice_num=32)


def run_model(args):
    """Config 4: one training step (forward, MSE backward, Adam) of the
    Transolver with the fused ops, on one GPU, next to the same model on its
    eager slice/deslice path (identical weights and data)."""
    from flashslice_b200 import Transolver
    torch.backends.cuda.matmul.allow_tf32 = bool(args.tf32_gemms)
    device = torch.device("cuda", 0)
    n = args.n or 200_000
    g = torch.Generator(device="cpu").manual_seed(0)
    xs = torch.rand(1, n, 3, generator=g).to(device)
    fs = torch.randn(1, n, 1, generator=g).to(device)
    ys = torch.randn(1, n, 4, generator=g).to(device)
    torch.manual_seed(0)
    fused = Transolver(**MODEL4, use_fused_slice=True).to(device)
    eager = Transolver(**MODEL4, use_fused_slice=False).to(device)
    eager.load_state_dict(fused.state_dict())
    lib = __import__("flashslice_b200.kernels._native", fromlist=["load"]).load()

    def timed(model):
        opt = torch.optim.Adam(model.parameters(), lr=1e-4)
        fwd = torch.compile(model, fullgraph=True) if args.compile else model

        def step():
            opt.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16, enabled=bool(args.bf16_autocast)):
                loss = torch.nn.functional.mse_loss(fwd(xs, fs).float(), ys)
            loss.backward()
            opt.step()

        for _ in range(max(args.warmup, 1)):
            step()
        torch.cuda.synchronize()
        launches0 = lib.fs_launch_count()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps, lib.fs_launch_count() - launches0

    clocks = ClockSampler(0)
    clocks.start()
    ms, launches = timed(fused)
    clk = clocks.stop()
    ms_eager, _ = timed(eager)
    line = {"metric": METRIC, "value": round(n / (ms * 1e-3) / 1e6, 3), "unit": UNIT,
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if args.bf16_autocast else "f32",
            "data": "synthetic (seeded, U[0,1]^3 points)",
            "config": {"workload": "cfg4", "model": "Transolver", **MODEL4, "N": n,
                       "step": "forward + MSE backward + Adam", "l2": "activations larger "
                       "than L2, no flush", "gemms": "tf32" if args.tf32_gemms else "fp32",
                       "compiled": bool(args.compile),
                       "eager_ms_per_step": round(ms_eager, 4),
                       "speedup_vs_eager": round(ms_eager / ms, 3)},
            "gpu_launches": launches,
            "roofline": None, "roofline_note": "a whole model step: projection GEMMs and "
            "MLPs (cuBLAS) dominate; the coupling ops are measured by the default workload",
            "cpu_baseline": None, "e2e": None, "clocks": clk}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- main

def main():
    args = parse()
    if args.config == "cfg4":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "config 4 is a model step; "
                              "the reference arm times the coupling round (default config)"}))
            return None
        return run_model(args)
    cfg = dict(CONFIGS[args.config])
    if args.n is not None:
        cfg["N"] = args.n
    if args.impl == "reference":
        return run_reference(args, cfg)
    if args.impl == "reference-triton":
        return run_reference_triton(args, cfg)
    if not torch.cuda.is_available():
        raise SystemExit("bench.py: no CUDA device (the fused ops have no CPU implementation)")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)
        group = dist.group.WORLD
    torch.backends.cuda.matmul.allow_tf32 = False

    import flashslice_b200.kernels as K
    from flashslice_b200.kernels import _native
    lib = _native.load()
    K.set_dot_mode(cfg["dot"])

    if cfg["split"]:
        from flashslice_b200.sharded import shard_range
        lo, hi = shard_range(cfg["N"], rank, world)
        n_local = hi - lo
    else:
        n_local = cfg["N"]
    x, fx, W, b, tau, r = make_inputs(cfg, n_local, device, 1234 + rank)
    # replicated parameters: identical on every rank
    _, _, W, b, tau, _ = make_inputs(cfg, 1, device, 99)
    leaves = [t.requires_grad_(True) for t in (x, fx, W, tau)]
    if b is not None:
        b.requires_grad_(True)

    def step():
        zero_grads(x, fx, W, b, tau)
        coupling_step(K, x, fx, W, b, tau, r, group)

    def barrier():
        if group is not None:
            import torch.distributed as dist
            dist.barrier(group=group)

    for _ in range(max(args.warmup, 1)):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = lib.fs_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    launches = lib.fs_launch_count() - launches0
    ms = e0.elapsed_time(e1) / args.steps
    barrier()
    clk = clocks.stop()
    if group is not None:
        import torch.distributed as dist
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        ms = t.item()
    points = cfg["B"] * (cfg["N"] if cfg["split"] else n_local * world)
    value = points / (ms * 1e-3) / 1e6

    # end to end: inputs from pinned host memory; every result back to pinned
    # host memory -- the round's output and the point gradients dx, dfx (the
    # op's results are point tensors: a host caller wants them on the host)
    # and the parameter gradients
    e2e = None
    if not args.no_e2e:
        xh = x.detach().cpu().pin_memory()
        fh = fx.detach().cpu().pin_memory()
        params = (W, tau) + ((b,) if b is not None else ())
        res_bytes = sum(t.numel() * t.element_size() for t in params)
        outs = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in params]
        pt_host = [torch.empty(x.shape, dtype=x.dtype, pin_memory=True) for _ in range(3)]
        res_bytes += sum(t.numel() * t.element_size() for t in pt_host)
        # Two sets of device inputs: the host copy of step i + 1's inputs runs
        # on a copy stream while step i computes, and step i's results go back
        # on a third stream while step i + 1 computes (PCIe is full duplex);
        # every step still copies its own inputs in and its results out
        # inside the timed region.
        sets = [(x, fx), (x.detach().clone().requires_grad_(True),
                          fx.detach().clone().requires_grad_(True))]
        main = torch.cuda.current_stream()
        copy_stream = torch.cuda.Stream(device=device)
        back_stream = torch.cuda.Stream(device=device)
        ready = [torch.cuda.Event() for _ in sets]
        free = [torch.cuda.Event() for _ in sets]
        done = torch.cuda.Event()

        def load(k, after_use):
            with torch.cuda.stream(copy_stream):
                if after_use:
                    copy_stream.wait_event(free[k])
                with torch.no_grad():
                    sets[k][0].copy_(xh, non_blocking=True)
                    sets[k][1].copy_(fh, non_blocking=True)
                ready[k].record(copy_stream)

        def e2e_steps(n):
            copy_stream.wait_stream(main)
            back_stream.wait_stream(main)
            for k in range(min(n, 2)):
                load(k, False)
            for i in range(n):
                k = i % 2
                main.wait_event(ready[k])
                xs, fs = sets[k]
                zero_grads(xs, fs, W, b, tau)
                out = coupling_step(K, xs, fs, W, b, tau, r, group)
                free[k].record(main)
                done.record(main)
                with torch.cuda.stream(back_stream):
                    back_stream.wait_event(done)
                    with torch.no_grad():
                        res = [out, xs.grad, fs.grad] + [t.grad for t in params]
                        for o, t in zip(pt_host + outs, res):
                            # the allocator keeps t's memory until the copy is done
                            t.record_stream(back_stream)
                            o.copy_(t, non_blocking=True)
                if i + 2 < n:
                    load(k, True)
            main.wait_stream(back_stream)

        e2e_steps(2)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        e2e_steps(args.steps)
        f1.record()
        torch.cuda.synchronize()
        ems = f0.elapsed_time(f1) / args.steps
        if group is not None:
            import torch.distributed as dist
            t = torch.tensor([ems], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
            ems = t.item()
        e2e = {"value": round(points / (ems * 1e-3) / 1e6, 3), "unit": UNIT,
               "h2d_bytes_per_step": (xh.numel() * xh.element_size()
                                      + fh.numel() * fh.element_size()),
               "d2h_bytes_per_step": res_bytes,
               "path": "fused_coupling + autograd; every step copies x_mid and fx_mid in "
                       "from pinned host memory and copies out, dx_mid, dfx_mid and the "
                       "parameter gradients back to pinned host memory (the next step's "
                       "inputs and the last step's results cross PCIe while a step "
                       "computes)"}

    # per-op device times of the same round, for the roofline
    dot = K.slice_ops._dot_mode(x)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    elem = x.element_size()
    unit_bytes = cfg["B"] * n_local * cfg["H"] * cfg["D"] * elem
    if K.slice_ops._use_blocked(cfg["D"], cfg["G"], cfg["DV"], dot, x.device):
        # the blocked family (G > 32): dots of 2 G (8 D + 6 DV) flops a
        # point-head, bound by the tensor cores (bf16) or the FMA pipes
        opt = op_timings_blocked(x, fx, W, b, tau, r, dot)
        top = max(opt, key=opt.get)
        heads = cfg["B"] * n_local * cfg["H"]
        flops = {k: 2 * cfg["G"] * f(cfg["D"], cfg["DV"]) * heads for k, f in BLK_FLOPS.items()}
        peak = peaks.get("bf16_tflops")
        peak_src = "measured (cuBLAS bf16, burst)" if peak else "fallback"
        peak = peak or 1590.0
        achieved = flops[top] / (opt[top] * 1e-3) / 1e12
        roofline = {"bound": "tensor", "kernel": top, "achieved": round(achieved, 2),
                    "peak": peak, "peak_source": peak_src, "unit": "TFLOP/s",
                    "frac": round(achieved / peak, 4), "traffic": None,
                    "algorithmic_flops_per_launch": flops[top],
                    "op_ms": {k: round(v, 4) for k, v in opt.items()},
                    "round_frac": round(sum(flops.values()) / (ms * 1e-3) / 1e12 / peak, 4)}
    else:
        opt = op_timings(K, x, fx, W, b, tau, r, dot)
        top = max(opt, key=opt.get)
        peak = peaks.get("hbm_gbs")
        peak_src = "measured" if peak else "fallback"
        peak = peak or 6650.0
        algo = UNITS[top] * unit_bytes
        achieved = algo / (opt[top] * 1e-3) / 1e9
        round_bytes = sum(UNITS.values()) * unit_bytes
        roofline = {"bound": "hbm", "kernel": top, "achieved": round(achieved, 1),
                    "peak": peak, "peak_source": peak_src, "unit": "GB/s",
                    "frac": round(achieved / peak, 4),
                    "traffic": profile_traffic(KERNEL_OF[top], cfg["B"] * n_local * cfg["H"]),
                    "algorithmic_bytes_per_launch": algo,
                    "op_ms": {k: round(v, 4) for k, v in opt.items()},
                    "round_frac": round(round_bytes / (ms * 1e-3) / 1e9 / peak, 4)}

    # the reference's surface (op by op) and the reverse call order, same inputs
    extra = {}
    if world == 1 and not args.no_extras and \
            not K.slice_ops._use_blocked(cfg["D"], cfg["G"], cfg["DV"], dot, x.device):
        def obo():
            zero_grads(x, fx, W, b, tau)
            op_by_op_step(K, x, fx, W, b, tau, r)

        t = timed_rounds(obo, args.steps)
        extra["op_by_op"] = {
            "value": round(points / (t * 1e-3) / 1e6, 3), "unit": UNIT, "ms_per_step": round(t, 4),
            "round_frac": round(sum(UNITS.values()) * unit_bytes / (t * 1e-3) / 1e9 / peak, 4),
            "path": "fused_slice + fused_deslice + autograd (the reference's surface: slice "
                    "forward, deslice forward, deslice backward, slice backward, dx summed)"}
        gen = torch.Generator(device=device).manual_seed(4321)
        shp = (cfg["B"], cfg["H"], cfg["G"], cfg["DV"])
        tok = torch.randn(*shp, generator=gen, device=device).requires_grad_(True)
        rz = torch.randn(*shp, generator=gen, device=device)
        rs = torch.randn(*shp[:3], generator=gen, device=device)

        def rev():
            zero_grads(x, fx, W, b, tau, tok)
            reverse_step(K, x, fx, W, b, tau, tok, r, rz, rs)

        t = timed_rounds(rev, args.steps)
        extra["reverse_order"] = {
            "value": round(points / (t * 1e-3) / 1e6, 3), "unit": UNIT,
            "ms_per_step": round(t, 4),
            "path": "fused_deslice(return_stats=True) then fused_slice(stats=...) of the same "
                    "points, forward and backward; tokens ~ N(0, 1)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(cfg, cpu_sample(args, cfg))

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
                "higher_is_better": True, "scaling": "strong" if cfg["split"] else "weak",
                "vs_baseline": None,
                "dtype": "f32" if cfg["dtype"] == torch.float32 else "bf16",
                "data": "synthetic (seeded torch.Generator on the device)",
                "config": {"workload": args.config, "B": cfg["B"], "N_per_gpu": n_local,
                           "H": cfg["H"], "D": cfg["D"], "DV": cfg["DV"], "G": cfg["G"],
                           "weight": cfg["weight"], "dot": cfg["dot"],
                           "parallelism": "point-shard x%d" % world,
                           "l2": "inputs larger than L2 (%d MiB per point tensor), no flush"
                                 % (unit_bytes >> 20)},
                "e2e": e2e, "gpu_launches": int(launches), "roofline": roofline,
                "cpu_baseline": cpu, "clocks": clk, **extra}
        print(json.dumps(line), flush=True)
    if group is not None:
        import torch.distributed as dist
        dist.barrier(group=group)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
