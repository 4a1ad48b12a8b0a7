#!/usr/bin/env python
"""Benchmark: joint VAE + motion-net training, frame-pairs/s at 854x480 (padded
to 856) on N B200s, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

N > 1 is launched with torch.distributed.run (one rank per GPU); ranks join a
torch.distributed group (NCCL) for the barriers and the max-over-ranks timing,
and the library's own NCCL communicator for the gradient all-reduce.

Timed regions (device time, CUDA events on the trainer's stream, barrier +
synchronize on both sides, max over ranks):
  value -- K steps with the step's frames already resident in device memory;
  e2e   -- K steps through yl_trainer_step_host: host->device copy of the
           step's frames from pinned memory, the step, device->host read of
           the two losses, every step.
Per-kernel-class and per-template times come from CUDA events the library
records around every conv / GroupNorm launch, in K further steps run after
the `value` region (so the value itself carries no per-launch events).

Roofline denominators: the dense TF32 rate is measured at the start of the
run on the same GPU (cuBLAS fp32 GEMM with TF32 tensor cores, burst and
sustained); HBM bandwidth comes from the driver's MEASURED_PEAKS.json.

--impl reference times the reference's arithmetic on the CPU instead: the
oracle (a C restatement of the reference's own kernels, oracle/) running the
same joint step on one full 480x856 frame-pair per step (the metric's unit),
with the thread count set explicitly to every CPU the process may use.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "train frame-pairs/s @854x480 at 1/2/4/8 B200; conv TFLOP/s vs tensor peak"
# Algorithmic conv work per frame-pair (2*MACs over every conv of the frozen
# layer tables; dX and dW each equal the forward): VAE train on frame k +
# encoder forward on frames 0 and 16 + motion U-Net train.
VAE_FWD_PER_FRAME = 2.5980e12
ENC_FWD_PER_FRAME = 1.1100e12
MOTION_TRAIN_PER_SAMPLE = 0.1433e12
# DRAM bytes (read + write) of one conv_tma_fprop_kernel<128, 2, 1, 1> launch
# per image of 480x856 (3x3, 128 -> 128): ncu capture of a 2-image launch,
# 421.5 MB read + 374.6 MB written.
DOM_TRAFFIC_PER_IMAGE = (421.5e6 + 374.6e6) / 2
WORKLOAD = ("joint VAE + motion-net train step at 854x480: VAE fwd+bwd on frame k, encoder fwd "
            "on frames 0/16, U-Net fwd+bwd, all-reduce, Adam")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--batch", type=int, default=8, help="frame-pair samples per GPU")
    ap.add_argument("--height", type=int, default=480)
    ap.add_argument("--width", type=int, default=856)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = Path(f"/tmp/yl_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.device)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = [r.split(",") for r in self.path.read_text().strip().splitlines() if r.strip()]
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except (ValueError, IndexError):
                continue
            for i, nm in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower().startswith("active"):
                    reasons.add(nm)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU arm
def host_threads() -> int:
    """CPUs this process may run on (torch.distributed.run sets OMP_NUM_THREADS=1
    for every rank; the CPU baseline sets its thread count explicitly instead)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def _oracle():
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle_ctypes  # the oracle: a C restatement of the reference's kernels (CPU)
    L = oracle_ctypes.load_oracle()
    L.orc_set_num_threads(host_threads())
    return oracle_ctypes, L


def cpu_sample(steps: int, warmup: int, rows: int = 480, width: int = 856):
    """The oracle's joint step (VAE fwd+bwd on frame k, encoder fwd on frames 0
    and 16, motion U-Net fwd+bwd, Adam) on one full frame-pair, all host
    threads.  A 16-row crop step first pages in the code paths untimed."""
    _, L = _oracle()
    import nets  # the oracle's composition of the reference's kernels (CPU)
    from yumelayers_b200 import synth
    js = nets.standalone_joint_step(seed=0, ops=nets.Ops(L))
    clip = synth.make_clip(7, h=rows, w=width - 2, width_padded=width)
    frames = np.ascontiguousarray(np.stack([clip[0][None], clip[16][None], clip[5][None]]))
    t = np.array([5 / 16.0], np.float32)
    small = np.ascontiguousarray(frames[:, :, :, :16])
    js.step(small, t)
    for _ in range(warmup):
        js.step(frames, t)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        js.step(frames, t)
        times.append(time.perf_counter() - t0)
    per_step = statistics.median(times)
    return {"value": 1.0 / per_step, "unit": "frame-pairs/s", "cores": L.orc_num_threads(),
            "kind": "port",
            "sample": (f"oracle joint step (VAE train on frame k, encoder fwd on frames 0/16, "
                       f"motion U-Net train, Adam) on one full {rows}x{width} frame-pair, "
                       f"{L.orc_num_threads()} host threads; median of {steps} timed steps "
                       f"({per_step:.1f} s each) after {warmup} full-size warm-up steps; "
                       "no scaling"),
            "seconds_per_sample_step": per_step}


def cpu_configs(reps_conv: int = 10, reps_block: int = 3):
    """The two single-op workloads timed in full on the host cores with the
    oracle: conv3x3 N=2 32->32 64x64 forward + dX + dW + db, and the ResNet
    block N=8 C=128 128x128 forward + backward (GroupNorm32 eps 1e-6, SiLU)."""
    oc_, L = _oracle()
    from yumelayers_b200 import config_bench as cbm
    rng = np.random.default_rng(0)
    out = {}
    d = cbm.CONV1
    x = oc_.f32(rng.standard_normal((d["n"], d["c"], d["h"], d["w"])))
    w = oc_.f32(rng.uniform(-0.08, 0.08, (d["oc"], d["c"], 3, 3)))
    dy = oc_.f32(rng.standard_normal((d["n"], d["oc"], d["h"], d["w"])))
    ts = []
    for _ in range(reps_conv + 1):
        t0 = time.perf_counter()
        oc_.conv2d_fwd(L, x, w, None)
        oc_.conv2d_bwd(L, x, w, dy)
        ts.append(time.perf_counter() - t0)
    out["conv1"] = statistics.median(ts[1:]) * 1e3
    b = cbm.BLOCK
    n, c, h, wd, g, eps = b["n"], b["c"], b["h"], b["w"], b["groups"], b["eps"]
    x = oc_.f32(rng.standard_normal((n, c, h, wd)))
    dy = oc_.f32(rng.standard_normal((n, c, h, wd)))
    ga, be = oc_.f32(1 + 0.02 * rng.standard_normal(c)), oc_.f32(0.02 * rng.standard_normal(c))
    w1 = oc_.f32(rng.uniform(-0.03, 0.03, (c, c, 3, 3)))
    w2 = oc_.f32(rng.uniform(-0.03, 0.03, (c, c, 3, 3)))
    ts = []
    for _ in range(reps_block + 1):
        t0 = time.perf_counter()
        h1, _, _ = oc_.gn_silu_fwd(L, x, g, eps, ga, be)
        c1 = oc_.conv2d_fwd(L, h1, w1, None)
        h2, _, _ = oc_.gn_silu_fwd(L, c1, g, eps, ga, be)
        oc_.conv2d_fwd(L, h2, w2, None, residual=x)
        dh2, _, _, _ = oc_.conv2d_bwd(L, h2, w2, dy)
        dc1, _, _ = oc_.gn_silu_bwd(L, c1, dh2, g, eps, ga, be)
        dh1, _, _, _ = oc_.conv2d_bwd(L, h1, w1, dc1)
        oc_.gn_silu_bwd(L, x, dh1, g, eps, ga, be, addend=dy)
        ts.append(time.perf_counter() - t0)
    out["block"] = statistics.median(ts[1:]) * 1e3
    out["cores"] = L.orc_num_threads()
    return out


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    # one full frame-pair step takes tens of seconds on the host cores: at most
    # 2 timed and 1 warm-up steps keep the run within a few minutes
    steps, warmup = max(1, min(args.steps, 2)), max(0, min(args.warmup, 1))
    cb = cpu_sample(steps, warmup)
    line = {"metric": METRIC, "value": cb["value"], "unit": "frame-pairs/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": steps, "warmup": warmup,
            "ms_per_step": 1000 * cb["seconds_per_sample_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded 17-frame clips: blobs + gratings + 4 moving sprites)",
            "config": {"workload": WORKLOAD, "frame": "480x856 (854 padded to 856)",
                       "per_gpu_batch": 8, "global_batch": 8,
                       "parallelism": "host threads on rank 0 (the oracle's CPU path)",
                       "sample": "one frame-pair per step (the metric's unit), full frame"},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": "frame-pairs/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def measure_tf32_peak(device: int) -> dict:
    """Dense TF32 tensor-core rate of this GPU the way the driver measures bf16:
    torch.matmul on 8192^3 fp32 operands with TF32 allowed (cuBLAS), best of 10
    single launches (burst) and back to back for >= 4 s (sustained, under the
    power cap), with the SM clocks sampled during the sustained loop."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        n = 8192
        dev = f"cuda:{device}"
        g = torch.Generator(device=dev).manual_seed(0)
        a = torch.randn(n, n, device=dev, generator=g)
        b = torch.randn(n, n, device=dev, generator=g)
        c = torch.empty(n, n, device=dev)
        flops = 2.0 * n ** 3
        for _ in range(3):
            torch.matmul(a, b, out=c)
        torch.cuda.synchronize(dev)
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        iters = max(10, int(4000.0 / best) + 1)
        with ClockSampler(device) as clk:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                torch.matmul(a, b, out=c)
            e1.record()
            e1.synchronize()
        sustained_ms = e0.elapsed_time(e1) / iters
        del a, b, c
        torch.cuda.empty_cache()
        return {"tf32_tflops": flops / (best * 1e-3) / 1e12,
                "tf32_tflops_sustained": flops / (sustained_ms * 1e-3) / 1e12,
                "sustained_seconds": iters * sustained_ms / 1e3, "clocks": clk.summary()}
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


# ------------------------------------------------------------------ native arm
def run_native(args):
    import torch
    import torch.distributed as dist
    from yumelayers_b200 import synth
    from yumelayers_b200._lib import lib
    from yumelayers_b200.session import Context
    from yumelayers_b200.trainer import (Comm, Trainer, default_config, max_over_ranks,
                                         share_unique_id)

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    # this GPU's dense TF32 rate, measured before the trainer holds its memory
    tf32 = measure_tf32_peak(local)
    ctx = Context(local)
    comm = None
    if world > 1:
        def bcast(obj):
            dist.broadcast_object_list(obj, src=0)
        uid = share_unique_id(rank, Comm.unique_id, bcast)
        comm = Comm(ctx, uid, rank, world)
    B, H, W = args.batch, args.height, args.width
    tr = Trainer(default_config(batch=B, height=H, width=W, seed=0), ctx=ctx, comm=comm)

    # synthetic 17-frame clips, a few distinct step batches
    clips = [synth.make_clip(1000 * rank + c, h=H, w=854 if W == 856 else W, width_padded=W)
             for c in range(2)]
    nb = 3
    host, tvals = [], []
    for i in range(nb):
        pinned = torch.empty((3, B, 3, H, W), dtype=torch.float32, pin_memory=True)
        fr, t = synth.sample_batch(clips, B, seed=97 * rank + i, out=pinned.numpy())
        host.append(pinned)
        tvals.append(torch.from_numpy(t).pin_memory())
    dev = [h.to(f"cuda:{local}", non_blocking=False) for h in host]
    tdev = [t.to(f"cuda:{local}") for t in tvals]
    losses_dev = torch.zeros(2, dtype=torch.float32, device=f"cuda:{local}")
    stream = torch.cuda.ExternalStream(ctx.stream, device=f"cuda:{local}")
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        tr.step_device(dev[i % nb].data_ptr(), tdev[i % nb].data_ptr(), losses_dev.data_ptr())
    barrier()

    # ---- value: device-resident inputs, no per-launch events in the step
    tr.set_config(profile=0)
    launches0 = lib().yl_kernel_launch_count()
    barrier()
    with ClockSampler(local) as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for i in range(args.steps):
            tr.step_device(dev[i % nb].data_ptr(), tdev[i % nb].data_ptr(), losses_dev.data_ptr())
        ev1.record(stream)
        ev1.synchronize()
    barrier()
    launches = lib().yl_kernel_launch_count() - launches0
    ms = max_over_ranks(ev0.elapsed_time(ev1), f"cuda:{local}")
    clocks = clk.summary()
    losses = losses_dev.cpu().numpy().tolist()

    # ---- the same steps again with CUDA events around every conv / GroupNorm
    # launch: per-class and per-template times, exposed communication
    tr.set_config(profile=1)
    tr.kernel_stats(reset=True)
    tr.comm_stats(reset=True)
    barrier()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    for i in range(args.steps):
        tr.step_device(dev[i % nb].data_ptr(), tdev[i % nb].data_ptr(), losses_dev.data_ptr())
    p1.record(stream)
    p1.synchronize()
    barrier()
    prof_ms = max_over_ranks(p0.elapsed_time(p1), f"cuda:{local}")
    stats = tr.kernel_stats(reset=True)
    comm_ms, comm_steps = tr.comm_stats(reset=True)
    # every rank profiled the same steps: at N > 1 all ranks take part in the max
    exposed = (max_over_ranks(comm_ms / comm_steps, f"cuda:{local}") if comm_steps else None)
    tr.set_config(profile=0)

    # ---- e2e: host buffers through the public step call
    out = np.zeros(2, np.float32)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e0.record(stream)
    for i in range(args.steps):
        tr.step_host_ptr(host[i % nb].data_ptr(), tvals[i % nb].data_ptr(), out)
    e1.record(stream)
    e1.synchronize()
    wall = time.perf_counter() - w0
    barrier()
    e2e_ms = max_over_ranks(max(e0.elapsed_time(e1), 1000 * wall), f"cuda:{local}")

    value = world * B * args.steps / (ms / 1000.0)
    e2e_value = world * B * args.steps / (e2e_ms / 1000.0)
    peaks = measured_peaks()
    hbm = peaks.get("hbm_gbs") or 6650.0
    hbm_src = "measured (MEASURED_PEAKS.json)" if peaks.get("hbm_gbs") else "fallback"
    # the convs run inside a step of a few hundred ms: the sustained TF32 rate
    tf32_peak = tf32["tf32_tflops_sustained"]
    templates = tr.template_stats()
    kernels = {}
    for k, v in stats.items():
        if v["ms"] <= 0:
            continue
        ent = {"ms_per_step": v["ms"] / args.steps, "launches_per_step": v["launches"] / args.steps,
               "share_of_step": v["ms"] / prof_ms}
        if v["flops"]:
            ent["tflops_algorithmic"] = v["flops"] / (v["ms"] * 1e-3) / 1e12
            ent["tflops_executed"] = v["exec_flops"] / (v["ms"] * 1e-3) / 1e12
            ent["frac_tf32_executed"] = ent["tflops_executed"] / tf32_peak
        if v["bytes"]:
            ent["gbs"] = v["bytes"] / (v["ms"] * 1e-3) / 1e9
            ent["frac_hbm"] = ent["gbs"] / hbm
        kernels[k] = ent
    conv_templates = []
    for name, v in sorted(templates.items(), key=lambda kv: -kv[1]["ms"]):
        if v["ms"] <= 0:
            continue
        ex = v["exec_flops"] / (v["ms"] * 1e-3) / 1e12
        conv_templates.append({
            "kernel": name, "launches_per_step": v["launches"] / args.steps,
            "ms_per_step": v["ms"] / args.steps, "share_of_step": v["ms"] / prof_ms,
            "tflops_algorithmic": v["flops"] / (v["ms"] * 1e-3) / 1e12,
            "tflops_executed": ex, "frac_tf32_executed": ex / tf32_peak})
    classes = ("conv_fprop", "conv_dgrad", "conv_wgrad", "gn_silu_fwd", "gn_silu_bwd")
    top = max(classes, key=lambda k: stats[k]["ms"])
    conv_flops = sum(stats[k]["flops"] for k in ("conv_fprop", "conv_dgrad", "conv_wgrad"))
    conv_exec = sum(stats[k]["exec_flops"] for k in ("conv_fprop", "conv_dgrad", "conv_wgrad"))
    conv_ms = sum(stats[k]["ms"] for k in ("conv_fprop", "conv_dgrad", "conv_wgrad"))
    dom = stats.get("conv_3x3_128_frame", {"ms": 0.0})
    if dom["ms"] > 0 and dom["launches"] > 0:
        # the dominant launch type: one stride-1 3x3 128->128 pass over the batch
        # at the frame resolution (forward or dX, the same kernel; algorithmic
        # and executed FLOPs are equal for it)
        achieved = dom["flops"] / (dom["ms"] * 1e-3) / 1e12
        per_launch_flops = dom["flops"] / dom["launches"]
        per_launch_bytes = 2.0 * B * H * W * 128 * 4 + 128 * 128 * 9 * 4
        kernel = (f"conv_tma_fprop_kernel<128, 2, 1, 1> (3x3 128->128, {B}x{H}x{W}, "
                  "forward and dX passes)")
        traffic = DOM_TRAFFIC_PER_IMAGE * B if (H, W) == (480, 856) else None
    else:
        achieved = stats[top]["exec_flops"] / (stats[top]["ms"] * 1e-3) / 1e12
        per_launch_flops = per_launch_bytes = None
        kernel, traffic = top, None
    roofline = {"bound": "tensor", "kernel": kernel, "achieved": achieved, "peak": tf32_peak,
                "unit": "TFLOP/s", "frac": achieved / tf32_peak, "traffic": traffic,
                "flops_per_launch": per_launch_flops,
                "algorithmic_bytes_per_launch": per_launch_bytes,
                "peak_note": ("measured in this run on this GPU: cuBLAS fp32 GEMM with TF32 "
                              f"tensor cores, 8192^3, back to back for "
                              f"{tf32['sustained_seconds']:.1f} s (sustained; burst "
                              f"{tf32['tf32_tflops']:.1f} TFLOP/s), SM clock median "
                              f"{tf32['clocks'].get('sm_mhz')} MHz, reasons "
                              f"{tf32['clocks'].get('reasons')}"),
                "peak_burst": tf32["tf32_tflops"], "frac_burst": achieved / tf32["tf32_tflops"],
                "flops_note": ("achieved = 2*N*Cout*Cin*9*OH*OW per launch over the summed "
                               "CUDA-event time of those launches in the timed steps"),
                "traffic_note": ("DRAM read + write bytes per launch from an ncu capture of "
                                 "the same kernel on 2 images, scaled to the batch; below "
                                 "the algorithmic bytes because part of the output is "
                                 "still in L2 when the kernel ends"),
                "all_convs": {"tflops_algorithmic": conv_flops / (conv_ms * 1e-3) / 1e12,
                              "tflops_executed": conv_exec / (conv_ms * 1e-3) / 1e12,
                              "frac_executed": conv_exec / (conv_ms * 1e-3) / 1e12 / tf32_peak},
                "hbm_peak_gbs": hbm, "hbm_peak_source": hbm_src}
    act_gb = tr.activation_bytes() / 1e9
    if rank == 0:
        cpu, configs = None, None
        if world == 1:
            configs = config_lines(ctx, args.no_cpu_baseline)
        if world == 1 and not args.no_cpu_baseline:
            try:
                cb = cpu_sample(steps=1, warmup=0)
                cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
            except Exception as exc:  # reported, not fatal
                cpu = {"value": None, "error": str(exc)}
        h2d = 3 * B * 3 * H * W * 4 + B * 4
        line = {
            "metric": METRIC, "value": value, "unit": "frame-pairs/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "tf32",
            "data": "synthetic (seeded 17-frame clips: blobs + gratings + 4 moving sprites)",
            "config": {"workload": WORKLOAD,
                       "frame": f"{H}x{W} (854 padded to 856)", "per_gpu_batch": B,
                       "global_batch": B * world, "parallelism": f"dp{world}",
                       "l2": (f"working set {act_gb:.0f} GB per GPU >> 126 MB L2; "
                              "no explicit flush"),
                       "conv_tflop_per_step": conv_flops / 1e12 / args.steps},
            "e2e": {"value": e2e_value, "unit": "frame-pairs/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": 8, "ms_per_step": e2e_ms / args.steps},
            "roofline": roofline, "kernels": kernels, "conv_templates": conv_templates,
            "configs": configs, "cpu_baseline": cpu,
            "exposed_comm_ms_per_step": exposed,
            "profiled_ms_per_step": prof_ms / args.steps,
            "clocks": clocks, "gpu_launches": int(launches),
            "losses_last_step": losses,
        }
        print(json.dumps(line), flush=True)
    tr.close()
    if comm:
        comm.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def config_lines(ctx, no_cpu: bool) -> dict:
    """The two single-op workloads: GPU device time through the C ABI (NCHW,
    L2 evicted before each repetition) and the oracle timed in full on the host
    cores."""
    from yumelayers_b200 import config_bench as cbm
    out = {}
    try:
        g1 = cbm.conv1_gpu_ms(ctx)
        g2 = cbm.block_gpu_ms(ctx)
        cpu = None if no_cpu else cpu_configs()
        for key, gms, flops, what in (
                ("conv3x3_n2_c32_64x64", g1, cbm.CONV1_FLOPS,
                 "Conv2d 3x3 s1 p1, N=2, 32->32, 64x64: forward + dX + dW + db"),
                ("resblock_n8_c128_128x128", g2, cbm.BLOCK_FLOPS,
                 "ResNet block N=8 C=128 128x128 (GN32 eps 1e-6 + SiLU, two 3x3 convs, "
                 "identity residual): forward + backward")):
            ent = {"workload": what, "gpu_ms": gms, "gpu_tflops": flops / (gms * 1e-3) / 1e12,
                   "conv_gflop": flops / 1e9,
                   "gpu_note": "C-ABI calls on NCHW device buffers incl. layout conversions; "
                               "median of the repetitions, L2 evicted before each"}
            if cpu:
                cms = cpu["conv1" if key.startswith("conv") else "block"]
                ent.update({"cpu_ms": cms, "cpu_cores": cpu["cores"], "cpu_kind": "port",
                            "cpu_note": "the oracle (C restatement of the reference's "
                                        "kernels) timed in full, median of repetitions"})
            out[key] = ent
    except Exception as exc:  # reported, not fatal
        out["error"] = str(exc)
    return out


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_native(args)


if __name__ == "__main__":
    main()
