#!/usr/bin/env python
"""Benchmark of the splax_b200 hot path on its headline workload.

Metric: fwd+bwd frames/s of config 2 (N=1,000,000 gaussians, 8 ring cameras, 1080x1920,
MSE against seeded targets, gradients of all five gaussian parameter arrays). One step renders
all 8 cameras forward, takes the loss and runs the full backward. With --gpus N (torchrun)
the 8 cameras are split across the N ranks (strong scaling) and the gaussian gradients are
summed with one NCCL all-reduce per step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl splax_b200|reference]

``--impl reference`` times the CPU restatement of the path (the C oracle, with every host
thread) because the reference's own runtime (warp-lang + jax) cannot be installed here; rank 0
alone runs it. Each of its steps renders one camera of the workload forward and backward, the
steps rotating through all the cameras (a bounded sample of the same 8-camera mix).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fwd+bwd frames/s (1M gaussians, 1080p, 8 cams) at 1/2/4/8 B200; % roofline"
CONFIG = 2
WORKLOAD = "config 2: 1M gaussians, 8 ring cams, 1080x1920, MSE fwd+bwd, grads of 5 param arrays"
# the other fwd+bwd configurations of the benchmark (not the headline): metric, workload, options
FWD_BWD = {
    0: ("config 0 forward frames/s (10k gaussians, 256x256, 1 cam)",
        "config 0: 10k gaussians, 1 cam, 256x256, white background, forward render only",
        dict(viewmat_grad=False, antialiased=False, forward_only=True)),
    1: ("config 1 fwd+bwd frames/s (200k gaussians, 800x800, 1 cam)",
        "config 1: 200k gaussians, 1 cam, 800x800, MSE fwd+bwd, grads of 5 param arrays + "
        "viewmat", dict(viewmat_grad=True, antialiased=False)),
    2: (METRIC, WORKLOAD, dict(viewmat_grad=False, antialiased=False)),
    4: ("config 4 fwd+bwd frames/s (6M gaussians, 2160x3840, 64 cams, antialiased)",
        "config 4: 6M gaussians, 64 sphere cams, 2160x3840, antialiased, MSE fwd+bwd, grads of "
        "5 param arrays + viewmats", dict(viewmat_grad=True, antialiased=True)),
}
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
NCCL_LABEL = "nccl (its NVLS algorithm off): one all-reduce of the gradients and the loss"
NCCL_SPLIT_LABEL = ("nccl (its NVLS algorithm off): two all-reduces, the colour and opacity "
                    "gradients' overlapped with the projection backward")
L2_BYTES = 126 << 20
# algorithmic work per unit: FLOPs per blend evaluation / contribution (FMA = 2), restated from
# the reference blend loop (splax/_rasterize/_kernels.py:185-197) and vjp (:1235-1253)
# DRAM bytes (read + write) per launch of the full config-2 workload from single-pass ncu
# captures (dram__bytes_read.sum + dram__bytes_write.sum)
TRAFFIC_BYTES_PER_LAUNCH = {"raster_bwd": 571.82e6, "raster_fwd": 491.21e6,
                            "emit_keys": 811.68e6}
FWD_FLOPS_PER_EVAL = 22
BWD_FLOPS_PER_EVAL = 12
BWD_FLOPS_PER_CONTRIB = 45


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="splax_b200", choices=["splax_b200", "reference"])
    ap.add_argument("--n", type=int, default=None, help="override the gaussian count (debug)")
    ap.add_argument("--overlap", action="store_true",
                    help="N>1 with NCCL: two all-reduces, the colour / opacity part started "
                         "while the projection backward runs, instead of one after the backward")
    ap.add_argument("--cams", type=int, default=None,
                    help="render only the first K cameras of the configuration (debug: one "
                         "rank's share of a sharded run on one GPU)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--collective", default="nccl", choices=["nccl", "nvls", "auto"],
                    help="gradient all-reduce for N>1: NCCL (default; 'auto' is the same), or "
                         "the library's NVLS kernel, opt-in")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--forward-only", action="store_true",
                    help="time the forward render alone (configs 1, 2, 4)")
    ap.add_argument("--config", type=int, default=CONFIG, choices=[0, 1, 2, 3, 4],
                    help="2: the headline fwd+bwd step (default); 0: forward render only; 1: one "
                         "camera with the viewmat "
                         "gradient; 3: the batched training step; 4: the antialiased 64-camera "
                         "4K stress step (8 GPUs)")
    return ap.parse_args()


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return FALLBACK_PEAKS, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled while the timed region runs: NVML
    read every 20 ms from a thread (read-only queries; faster polling slowed the launch-bound
    small configurations), else nvidia-smi every 200 ms."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.thread = None
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None

    def _start_nvml(self) -> bool:
        import threading

        try:
            import pynvml
            pynvml.nvmlInit()
            h = (pynvml.nvmlDeviceGetHandleByUUID(self.uuid) if self.uuid
                 else pynvml.nvmlDeviceGetHandleByIndex(0))
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons",
                              getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons", None))
            self.bits = (getattr(pynvml, "nvmlClocksEventReasonHwSlowdown", 0x8),
                         getattr(pynvml, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
                         getattr(pynvml, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
                         getattr(pynvml, "nvmlClocksEventReasonSwPowerCap", 0x4))
        except Exception:
            return False
        self.stop_flag = threading.Event()

        def loop():
            while not self.stop_flag.is_set():
                try:
                    self.samples.append((float(pynvml.nvmlDeviceGetClockInfo(
                        h, pynvml.NVML_CLOCK_SM)), int(reasons(h)) if reasons else 0))
                except Exception:
                    pass
                time.sleep(0.02)

        self.thread = threading.Thread(target=loop, daemon=True)
        self.thread.start()
        return True

    def start(self) -> None:
        if self._start_nvml():
            return
        try:
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                   "-lms", "200"]
            if self.uuid:
                cmd += ["-i", self.uuid]
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict | None:
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join(timeout=5)
            if not self.samples:
                return None
            sm = [c for c, _ in self.samples]
            reasons = sorted({n for _, r in self.samples for n, b in zip(self.NAMES, self.bits)
                              if r & b})
            return {"sm_mhz": statistics.median(sm), "sm_max_mhz": self.max_mhz,
                    "reasons": reasons, "samples": len(sm), "source": "nvml, 20 ms"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(", ") for r in out.strip().splitlines() if r.count(",") >= 9]
        if not rows:
            return None
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        reasons = sorted({self.NAMES[k] for r in rows for k in range(4)
                          if r[6 + k].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows), "source": "nvidia-smi, 200 ms"}


def cpu_baseline(scene: dict, threads: int, forward_only: bool = False, cam_index: int = 0,
                 target: np.ndarray | None = None) -> dict:
    """One camera of the workload (camera ``cam_index``, against ``target``, its (H, W, 3)
    image), forward + backward (or forward only), through the C oracle."""
    import oracle

    oracle.build()
    n, H, W, f = scene["means"].shape[0], scene["H"], scene["W"], scene["f"]
    cam = dict(img_shape=(H, W), f=(f, f), c=(W / 2, H / 2))
    xyzw = np.roll(scene["quats"], -1, -1)
    vm = scene["viewmats"][cam_index]
    t0 = time.perf_counter()
    xys, d, r, cn, nth, cum = oracle.project(scene["means"], scene["scales"], xyzw, vm,
                                             scene["opacities"], n=n, nthreads=threads, **cam)
    op = scene["opacities"]
    fT, fi, img, _, _ = oracle.rasterize(scene["colors"], op, op, scene["background"], xys, d, r,
                                         cn, cum, n=n, B=1, img_shape=(H, W), nthreads=threads)
    if forward_only:
        return {"seconds": time.perf_counter() - t0, "counters": oracle.counters()}
    v_img = 2.0 * (img.reshape(H * W, 3) - target.reshape(H * W, 3)) / (scene["B"] * H * W * 3)
    vc, vo, vxy, vcon, _ = oracle.rasterize_bwd(scene["colors"], op, op, scene["background"], xys,
                                                d, r, cn, cum, fT, fi, v_img, n=n, B_out=1,
                                                B_geom=1, img_shape=(H, W), nthreads=threads)
    oracle.project_bwd(scene["means"], scene["scales"], xyzw, vm, r, cn, vxy,
                       np.zeros(n, np.float32), vcon, n=n, B=1, f=(f, f), nthreads=threads)
    dt = time.perf_counter() - t0
    return {"seconds": dt, "counters": oracle.counters()}


def arm_config(workload: str, n: int, per: int, world: int, input_bytes: int, flush: bool,
               collective: str | None) -> dict:
    """The ``config`` object of a bench line; both arms print the same one for a workload."""
    return {"workload": workload, "cams_per_gpu": per, "gaussians": n,
            "l2": (f"inputs {input_bytes / 1e6:.0f} MB per rank, below 2x the 126 MB L2: L2 "
                   "flushed (256 MB write) between timed steps" if flush else
                   f"inputs {input_bytes / 1e6:.0f} MB per rank (targets + parameters) plus the "
                   "per-step sort scratch exceed the 126 MB L2"),
            "parallelism": f"camera-sharded dp{world}", "collective": collective}


def reference_arm(args) -> None:
    """The reference arm: the CPU restatement of the path on the host cores, on the same
    workload and config object as this repo's arm. Step k renders camera k mod B (forward and
    backward for the fwd+bwd configurations), so the steps cover the workload's camera mix."""
    from splax_b200 import utils

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = max(args.gpus, 1)
    config = args.config if args.config in (0, 1, 2) else CONFIG
    metric, workload, opts = FWD_BWD[config]
    fwd_only = bool(opts.get("forward_only")) or args.forward_only
    if args.forward_only and not opts.get("forward_only"):
        metric = metric.replace("fwd+bwd", "forward")
        workload += " (forward render only)"
    scene = utils.synthetic_scene(config, n=args.n)
    B, H, W = scene["B"], scene["H"], scene["W"]
    n = scene["means"].shape[0]
    per = B // world if B % world == 0 else B
    targets = None if fwd_only else utils.target_images(scene)
    threads = os.cpu_count() or 1

    def one(k):
        c = k % B
        return cpu_baseline(scene, threads, forward_only=fwd_only, cam_index=c,
                            target=None if targets is None else targets[c])["seconds"]

    for k in range(min(args.warmup, 1)):
        one(k)
    times = [one(k) for k in range(args.steps)]
    total = sum(times)
    value = args.steps / total  # one frame per step
    sample = (f"one camera per step, cameras 0..{B - 1} in turn (N={n}, {H}x{W}, "
              f"{'forward' if fwd_only else 'fwd+bwd'}), C oracle with {threads} threads")
    input_bytes = 4 * (14 * n + per * H * W * 3)
    collective = None if world == 1 else ("nvls (library kernel)" if args.collective == "nvls"
                                          else NCCL_SPLIT_LABEL if args.overlap
                                          else NCCL_LABEL)
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": "frames/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seeded, config {config} distributions)",
        "config": arm_config(workload, n, per, world, input_bytes, input_bytes < 2 * L2_BYTES,
                             collective),
        "implementation": "C oracle: the CPU restatement of the path (warp-lang/jax, the "
                          "reference's runtime, cannot be installed here)",
        "cpu_baseline": {"value": value, "unit": "frames/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# Config 3 training step: the reference's per-group learning rates (scripts/train_colmap.py:
# 867-871), scaled by sqrt(B) for batched training (:609-610), and its D-SSIM weight (:872)
TRAIN_LRS = {"means": 1.5e-3, "log_scales": 5e-3, "quats": 1e-3, "colors_logit": 1e-2,
             "opac_logit": 5e-2}
SSIM_LAMBDA = 0.2


def nccl_environment(args) -> None:
    """Before the process group exists: NCCL's own NVLS all-reduce off unless the caller set
    NCCL_NVLS_ENABLE. On an NVSwitch B200 box NCCL otherwise picks NVLS for the 56 MB gradient
    all-reduce, which binds its buffers to NVLink multicast objects for the whole run; its ring
    measured faster there (8 ranks, 56 MB: 0.229 ms vs 0.257 ms). The opt-in library exchange
    (--collective nvls) keeps NCCL's default."""
    if args.collective != "nvls":
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")


def make_reducer(args, params, dev, world):
    """The library's NVLS gradient all-reduce over the parameters' gradients plus the loss when
    --collective nvls asks for it, else None (NCCL). NVLS stays opt-in: it measured 2% faster
    than NCCL at 4 ranks, and its symmetric buffers are bound to an NVLink multicast object for
    the life of the run."""
    if world == 1 or args.collective != "nvls":
        return None
    from splax_b200._collective import GradAllReduce

    return GradAllReduce([p.shape for p in params] + [(1,)], dev)


def teardown(world: int, closers: list) -> None:
    """End a multi-rank run on every path, the error path included: wait for this rank's queued
    work, release the collective objects (each waits for every rank before its symmetric memory
    may go), then leave the process group. A rank that raised thus keeps its memory bound until
    the others have left their kernels, or until the group's timeout ends the barrier."""
    if world <= 1:
        return
    import torch
    import torch.distributed as dist

    try:
        torch.cuda.synchronize()
        for c in closers:
            c.close()
        if not closers:
            dist.barrier()
    finally:
        dist.destroy_process_group()


class SplitAllReduce:
    """NCCL gradient exchange in two parts. The colour and opacity gradients are final once the
    rasterize backward has run: a hook on their accumulation starts their all-reduce on NCCL's
    stream while the projection backward computes the means / scales / quats gradients, which
    follow, with the loss, in a second all-reduce. Every rank issues the two collectives in the
    same order (the early one first), whether or not its hook fired."""

    def __init__(self, params, early):
        self.params = list(params)
        self.early = list(early)
        self.rest = [k for k in range(len(self.params)) if k not in self.early]
        self.ready: set = set()
        self.work = None
        self.flat_early = None
        self.armed = False
        for k in self.early:
            self.params[k].register_post_accumulate_grad_hook(self._hook(k))

    def _hook(self, k):
        def hook(p):
            if not self.armed:
                return
            self.ready.add(k)
            if len(self.ready) == len(self.early) and self.work is None:
                self._start_early()
        return hook

    def _start_early(self):
        import torch
        import torch.distributed as dist

        self.flat_early = torch.cat([self.params[k].grad.reshape(-1) for k in self.early])
        self.work = dist.all_reduce(self.flat_early, async_op=True)

    def arm(self):
        self.ready.clear()
        self.work = None
        self.armed = True

    def finish(self, loss):
        """Second all-reduce, then p.grad becomes a view of the summed buffers; returns the summed
        loss."""
        import torch
        import torch.distributed as dist

        self.armed = False
        if self.work is None:
            self._start_early()
        flat = torch.cat([self.params[k].grad.reshape(-1) for k in self.rest] +
                         [loss.detach().reshape(1)])
        dist.all_reduce(flat)
        self.work.wait()
        for bufs, idx in ((self.flat_early, self.early), (flat, self.rest)):
            o = 0
            for k in idx:
                p = self.params[k]
                p.grad = bufs[o:o + p.numel()].view_as(p)
                o += p.numel()
        self.work = None
        return flat[-1].reshape(())


def reduce_grads(reducer, params, loss, dev):
    """Sum the gradients and the loss over the ranks in one collective; p.grad becomes a view of
    the summed buffer. Returns the summed loss."""
    import torch
    import torch.distributed as dist

    if reducer is None:
        flat = torch.cat([p.grad.reshape(-1) for p in params] + [loss.detach().reshape(1)])
        dist.all_reduce(flat)
        sums, o = [], 0
        for p in params:
            sums.append(flat[o:o + p.numel()].view_as(p))
            o += p.numel()
        sums.append(flat[o:])
    else:
        sums = reducer.reduce([p.grad for p in params] + [loss.detach().reshape(1)])
    for p, g in zip(params, sums):
        p.grad = g
    return sums[-1].reshape(())


def train_bench(args) -> None:
    """Config 3: one batched training step = render_log fwd+bwd of B views, fused L1 + D-SSIM
    loss and gradient, on camera shards the gradient exchange (NCCL or the library's NVLS
    all-reduce, or with --collective nvls the exchange fused with Adam), per-group Adam."""
    import torch
    import torch.distributed as dist

    import splax_b200 as sx
    from splax_b200 import _lib, utils

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        nccl_environment(args)
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    closers: list = []
    try:
        scene = utils.synthetic_scene(3, n=args.n)
        B, H, W, f = scene["B"], scene["H"], scene["W"], scene["f"]
        n = scene["means"].shape[0]
        if B % world:
            raise SystemExit(f"{B} cameras do not split over {world} ranks")
        per = B // world
        cams = slice(rank * per, (rank + 1) * per)
        targets_np = utils.target_images(scene, range(rank * per, (rank + 1) * per))
        logit = lambda x: np.log(x) - np.log1p(-x)  # noqa: E731
        host = {"means": scene["means"], "log_scales": np.log(scene["scales"]),
                "quats": scene["quats"], "colors_logit": logit(np.clip(scene["colors"], 1e-4, 1 - 1e-4)),
                "opac_logit": logit(scene["opacities"])}
        params = [torch.tensor(host[k].astype(np.float32), device=dev).requires_grad_()
                  for k in TRAIN_LRS]
        lrs = [lr * float(np.sqrt(B)) for lr in TRAIN_LRS.values()]
        views = torch.tensor(scene["viewmats"][cams], device=dev)
        target = torch.tensor(targets_np, device=dev)
        bg = torch.tensor(scene["background"], device=dev)
        kw = dict(background=bg, img_shape=(H, W), f=(f, f))
        # with --collective nvls the exchange and the update fuse into one NVLS kernel (sharded
        # moments); otherwise an all-reduce, then Adam on every rank
        fused = None
        if world > 1 and args.collective == "nvls":
            from splax_b200._collective import NvlsAdam
            fused = NvlsAdam(params, lrs, dev)
            closers.append(fused)
            params = fused.params
        opt = None if fused is not None else sx.Adam(params, lrs)
        reducer = None if fused is not None else make_reducer(args, params, dev, world)
        if reducer is not None:
            closers.append(reducer)

        def step(vm, tgt):
            for p in params:
                p.grad = None
            imgs, _ = sx.render_log(*params, viewmat=vm, **kw)
            loss = sx.l1_dssim_loss(imgs, tgt, ssim_lambda=SSIM_LAMBDA, views_total=B)
            loss.backward()
            if fused is not None:
                fused.step([p.grad for p in params])
                dist.all_reduce(loss.detach())
                return loss
            if world > 1:  # the shared gradients (and the loss) summed over the ranks
                loss = reduce_grads(reducer, params, loss, dev)
            opt.step([p.grad for p in params])
            return loss

        for _ in range(args.warmup):
            step(views, target)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        uuid = None
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
        except Exception:
            pass
        sampler = ClockSampler(uuid) if rank == 0 else None
        _lib.profile_enable(timing=True, count_work=False)
        _lib.profile_reset()
        if sampler:
            sampler.start()
            if sampler.thread is None:
                time.sleep(0.3)  # nvidia-smi's first sample
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            loss = step(views, target)
        t1.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        clocks = sampler.stop() if sampler else None
        prof = _lib.profile_report()
        _lib.profile_enable(timing=False, count_work=False)
        ms_t = torch.tensor([t0.elapsed_time(t1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        ms = float(ms_t.item())
        loss_v = float(loss.item())
        if not np.isfinite(loss_v):
            raise SystemExit("non-finite training loss")
        if rank == 0:
            kern = prof["kernels"]
            total_ms = {k: v["ms"] for k, v in kern.items()}
            line = {
                "metric": "config 3 batched training step frames/s (3M gaussians, 840x1297, 32 cams)",
                "value": B * args.steps / (ms / 1e3), "unit": "frames/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
                "steps_per_s": args.steps / (ms / 1e3), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded, config 3 distributions)",
                "config": {"workload": "config 3: render_log fwd+bwd, L1 + 0.2 D-SSIM, all-reduce, "
                                       "per-group Adam", "gaussians": n, "cams_per_gpu": per,
                           "parallelism": f"camera-sharded dp{world}",
                           "collective": None if world == 1 else
                           ("nvls exchange fused with Adam (library kernel)" if fused is not None
                            else "nvls (library kernel)" if reducer is not None else "nccl")},
                "loss": loss_v,
                "kernels": {k: {**v, "share": v["ms"] / max(sum(total_ms.values()), 1e-9)}
                            for k, v in kern.items()},
                "clocks": clocks,
                "gpu_launches": int(sum(k["kernels"] for k in kern.values())),
            }
            print(json.dumps(line), flush=True)
    finally:
        teardown(world, closers)


def main() -> None:
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.config == 3:
        train_bench(args)
        return

    import torch
    import torch.distributed as dist

    import splax_b200 as sx
    from splax_b200 import _lib, utils

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        nccl_environment(args)
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    closers: list = []
    try:

        metric, workload, opts = FWD_BWD[args.config]
        if args.forward_only and not opts.get("forward_only"):
            opts = dict(opts, forward_only=True, viewmat_grad=False)
            metric = metric.replace("fwd+bwd", "forward")
            workload += " (forward render only)"
        scene = utils.synthetic_scene(args.config, n=args.n)
        if args.cams:
            scene["viewmats"] = scene["viewmats"][:args.cams]
            scene["B"] = int(scene["viewmats"].shape[0])
            workload += f" (debug: first {scene['B']} cameras only)"
        B, H, W, f = scene["B"], scene["H"], scene["W"], scene["f"]
        n = scene["means"].shape[0]
        if B % world:
            raise SystemExit(f"{B} cameras do not split over {world} ranks")
        per = B // world
        cams = slice(rank * per, (rank + 1) * per)
        targets_np = utils.target_images(scene, range(rank * per, (rank + 1) * per))
        host = {k: scene[k] for k in ("means", "scales", "quats", "colors", "opacities")}
        params = [torch.tensor(host[k], device=dev).requires_grad_() for k in host]
        views = torch.tensor(scene["viewmats"][cams], device=dev)
        if opts["viewmat_grad"]:
            views.requires_grad_()
        target = torch.tensor(targets_np, device=dev)
        bg = torch.tensor(scene["background"], device=dev)
        kw = dict(background=bg, img_shape=(H, W), f=(f, f), antialiased=opts["antialiased"])
        denom = float(B * H * W * 3)
        reducer = None if opts.get("forward_only") else make_reducer(args, params, dev, world)
        if reducer is not None:
            closers.append(reducer)
        # --overlap: colours and opacities (params 3, 4) summed while the projection backward runs
        split = (SplitAllReduce(params, early=(3, 4))
                 if world > 1 and reducer is None and not opts.get("forward_only")
                 and args.overlap else None)

        def step(vm, tgt, ps=params, tgt_ready=None, xev=None):
            """One step; returns the rendered images (forward only) or the loss. tgt_ready: an
            event the loss waits for (the targets' copy may overlap the forward render). xev: a
            pair of events recorded around the gradient exchange (N>1)."""
            if opts.get("forward_only"):
                with torch.no_grad():
                    imgs, _ = sx.render(*ps, viewmat=vm, **kw)
                return imgs
            for p in ps:
                p.grad = None
            if vm.requires_grad:
                vm.grad = None
            imgs, _ = sx.render(*ps, viewmat=vm, **kw)
            if tgt_ready is not None:
                torch.cuda.current_stream(dev).wait_event(tgt_ready)
            loss = sx.mse_loss(imgs, tgt, denom=denom)
            if split is not None:
                split.arm()
            loss.backward()
            if split is not None:  # the second half of the NCCL exchange (the first overlapped)
                return split.finish(loss)
            if world > 1:  # the gradients of the shared gaussians (and the loss) summed over ranks
                if xev is not None:
                    xev[0].record()
                loss = reduce_grads(reducer, ps, loss, dev)
                if xev is not None:
                    xev[1].record()
            return loss

        for _ in range(args.warmup):
            step(views, target)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

        # Per-stage breakdown: K untimed steps with every stage bracketed by CUDA events. The
        # events add a few microseconds per stage to the stream (6% of a one-camera step), so
        # the timed steps below bracket only the dominant stage, whose roofline they report.
        _lib.profile_enable(timing=True, count_work=False)
        _lib.profile_stages(None)
        _lib.profile_reset()
        for _ in range(args.steps):
            step(views, target)
        torch.cuda.synchronize()
        prof = _lib.profile_report()
        totals = {k: v["ms"] for k, v in prof["kernels"].items()}
        dominant = max(totals, key=totals.get)
        if world > 1:
            dist.barrier()

        uuid = None
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
        except Exception:
            pass
        sampler = ClockSampler(uuid) if rank == 0 else None
        _lib.profile_stages([dominant])
        _lib.profile_reset()
        if sampler:
            sampler.start()
            if sampler.thread is None:
                time.sleep(0.3)  # nvidia-smi's first sample
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        # Inputs smaller than L2 (config 1): time each step alone and flush L2 between steps by
        # writing a 256 MB buffer outside the timed events; otherwise from the first step's start
        # event to the last step's end event.
        input_bytes = 4 * (sum(p.numel() for p in params) + target.numel())
        flush = input_bytes < 2 * L2_BYTES
        # N>1: events around each step's exchange split this rank's time into its own work
        # (step start to exchange start) and the exchange as its stream sees it (waiting for
        # the slowest rank included)
        xevs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in range(args.steps)] if world > 1 and split is None else None
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        if flush:
            scratch = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
            for k, (a, b) in enumerate(evs):
                scratch.fill_(1)
                a.record()
                step(views, target, xev=xevs[k] if xevs else None)
                b.record()
            torch.cuda.synchronize()
            ms = sum(a.elapsed_time(b) for a, b in evs)
        else:
            for k, (a, b) in enumerate(evs):
                a.record()
                step(views, target, xev=xevs[k] if xevs else None)
                b.record()
            torch.cuda.synchronize()
            ms = evs[0][0].elapsed_time(evs[-1][1])
        rank_split = None
        if xevs:
            own = sum(a.elapsed_time(x0) for (a, _), (x0, _) in zip(evs, xevs)) / args.steps
            xch = sum(x0.elapsed_time(x1) for x0, x1 in xevs) / args.steps
            mine = torch.tensor([ms / args.steps, own, xch], device=dev, dtype=torch.float64)
            every = [torch.zeros_like(mine) for _ in range(world)]
            dist.all_gather(every, mine)
            rank_split = {"ms_per_step": [round(float(t[0]), 4) for t in every],
                          "own_work_ms": [round(float(t[1]), 4) for t in every],
                          "exchange_ms": [round(float(t[2]), 4) for t in every],
                          "how": "per rank, mean over the timed steps: CUDA events at the step's "
                                 "start, around the gradient exchange (the concatenation of the "
                                 "gradients and the wait for the slowest rank included) and at "
                                 "its end"}
        if world > 1:
            dist.barrier()
        clocks = sampler.stop() if sampler else None
        live = _lib.profile_report()["kernels"][dominant]
        _lib.profile_enable(timing=False, count_work=False)
        _lib.profile_stages(None)
        ms_t = torch.tensor([ms], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        ms = float(ms_t.item())
        value = B * args.steps / (ms / 1e3)

        # the exchange alone, outside the timed region: one all-reduce of the step's gradient
        # and loss floats (CUDA events on the launching stream, max over ranks)
        exchange = None
        if world > 1 and reducer is None and not opts.get("forward_only"):
            buf = torch.ones(sum(p.numel() for p in params) + 1, device=dev)
            for _ in range(3):
                dist.all_reduce(buf)
            xe = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(10)]
            torch.cuda.synchronize()
            for a0, a1 in xe:
                a0.record()
                dist.all_reduce(buf)
                a1.record()
            torch.cuda.synchronize()
            x_t = torch.tensor([statistics.median(a0.elapsed_time(a1) for a0, a1 in xe)],
                               device=dev, dtype=torch.float64)
            dist.all_reduce(x_t, op=dist.ReduceOp.MAX)
            exchange = {"bytes": int(4 * buf.numel()), "allreduce_ms": float(x_t.item()),
                        "how": "median of 10 back-to-back NCCL all-reduces, max over ranks"}
            del buf

        # one instrumented step outside the timed region: exact work units per step
        _lib.profile_enable(timing=False, count_work=True)
        _lib.profile_reset()
        step(views, target)
        torch.cuda.synchronize()
        work = _lib.profile_report()["units"]
        _lib.profile_enable(timing=False, count_work=False)

        # end to end through the public API from pinned host buffers. Every step copies its batch
        # from pinned host memory -- its cameras and, with a backward, its target images -- and
        # reads its result back: the loss, or for a forward-only step the rendered images. The
        # gaussians are the model: like a training loop, the step keeps them resident on the device.
        # A copy stream fills one of two device slots with step k+1's batch while step k computes
        # (a prefetching data loader; a step's loss waits for its targets, its render only for its
        # cameras) and drains the images of forward-only steps; every copy is inside the timed region.
        e2e = None
        if not args.no_e2e:
            fwd_only = bool(opts.get("forward_only"))
            v_host = torch.from_numpy(np.ascontiguousarray(scene["viewmats"][cams])).pin_memory()
            t_host = torch.from_numpy(np.ascontiguousarray(targets_np)).pin_memory()
            loss_host = torch.empty((args.steps + 1,), dtype=torch.float32).pin_memory()
            img_host = ([torch.empty((per, H, W, 3), dtype=torch.float32).pin_memory()
                         for _ in range(2)] if fwd_only else None)
            slots = [(torch.empty_like(views).requires_grad_(views.requires_grad),
                      torch.empty_like(target)) for _ in range(2)]
            h2d = v_host.numel() * 4 + (0 if fwd_only else t_host.numel() * 4)
            d2h = per * H * W * 3 * 4 if fwd_only else 4
            compute = torch.cuda.current_stream(dev)
            copier = torch.cuda.Stream(dev)
            copied = [torch.cuda.Event() for _ in range(2)]      # cameras on the device
            copied_tgt = [torch.cuda.Event() for _ in range(2)]  # targets on the device
            released = [torch.cuda.Event() for _ in range(2)]

            def load(k):
                s = k % 2
                with torch.cuda.stream(copier), torch.no_grad():
                    copier.wait_event(released[s])
                    slots[s][0].copy_(v_host, non_blocking=True)
                    copied[s].record(copier)
                    if not fwd_only:
                        slots[s][1].copy_(t_host, non_blocking=True)
                    copied_tgt[s].record(copier)

            def run(k):
                # the render waits for the cameras only; the loss waits for the targets, whose copy
                # overlaps the forward of the same step
                s = k % 2
                compute.wait_event(copied[s])
                out = step(slots[s][0], slots[s][1], tgt_ready=copied_tgt[s])
                if fwd_only:
                    rendered = torch.cuda.Event()
                    rendered.record(compute)
                    with torch.cuda.stream(copier):
                        copier.wait_event(rendered)
                        img_host[s].copy_(out, non_blocking=True)
                        out.record_stream(copier)
                else:
                    loss_host[k].copy_(out.detach(), non_blocking=True)
                released[s].record(compute)

            for s in range(2):
                released[s].record(compute)
            load(0)
            run(0)
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(compute)
            copier.wait_event(e0)
            load(1)
            for k in range(1, args.steps + 1):
                if k + 1 <= args.steps:
                    load(k + 1)
                run(k)
            compute.wait_stream(copier)  # the last images are on the host
            e1.record(compute)
            torch.cuda.synchronize()
            ems = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
            if world > 1:
                dist.all_reduce(ems, op=dist.ReduceOp.MAX)
            if fwd_only:
                if not bool(torch.isfinite(img_host[args.steps % 2]).all()):
                    raise SystemExit("non-finite image in the end-to-end steps")
            elif not bool(torch.isfinite(loss_host[1:]).all()):
                raise SystemExit("non-finite loss in the end-to-end steps")
            e2e = {"value": B * args.steps / (float(ems.item()) / 1e3), "unit": "frames/s",
                   "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                   "inputs": "per-step cameras" + ("" if fwd_only else " and target images") +
                             " from pinned host memory; gaussians resident (the model)",
                   "result": "rendered images to pinned host memory" if fwd_only else "loss",
                   "pipelining": "copy stream, two input slots"}

        cpu = None
        if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config in (0, 1, 2):
            threads = os.cpu_count() or 1
            fo = bool(opts.get("forward_only"))
            res = cpu_baseline(scene, threads, forward_only=fo, cam_index=0,
                               target=None if fo else targets_np[0])
            cpu = {"value": 1.0 / res["seconds"], "unit": "frames/s", "cores": threads,
                   "kind": "port",
                   "sample": f"camera 0 of {B} (one frame), N={n}, {H}x{W}, "
                             f"{'forward' if fo else 'fwd+bwd'}, C oracle"}

        if rank == 0:
            peaks, peak_src = load_peaks()
            props = torch.cuda.get_device_properties(dev)
            sm_mhz = (clocks or {}).get("sm_mhz") or 1965.0
            fp32_peak = props.multi_processor_count * 128 * 2 * sm_mhz * 1e6 / 1e12  # TFLOP/s
            kern = prof["kernels"]
            steps = args.steps
            rows = {}

            def avg_ms(name):
                k = kern[name]
                return k["ms"] / k["launches"] if k["launches"] else None

            units = prof["units"]
            per_launch = lambda key, name: units[key] / max(kern[name]["launches"], 1)  # noqa: E731
            I = work["intersections"]
            # HBM-bound stages: algorithmic bytes per launch
            kb = work["key_bytes"] / max(I, 1)
            passes = work["sort_pass_keys"] / max(I, 1)
            pairs = per_launch("pairs_fwd", "project_fwd")
            V = work["pairs_sorted"]  # pairs that hit a tile (exact, from the instrumented step)
            kbp = work["pair_key_bytes"] / max(V, 1)
            pp = work["pair_pass_keys"] / max(V, 1)
            bytes_est = {
                "project_fwd": 44 * n + 36 * pairs,
                "emit_keys": per_launch("intersections", "emit_keys") * (kb + 4) + 36 * pairs,
                "radix_sort": per_launch("intersections", "radix_sort") * kb
                + 2 * passes * per_launch("intersections", "radix_sort") * (kb + 4),
                "tile_bins": per_launch("key_bytes", "tile_bins") + 8 * per_launch("bins", "tile_bins"),
                # depth-order sort: the histogram and first pass read all P pair keys and keep the
                # V that hit a tile; the other passes move V keys and values
                "pair_sort": pairs * kbp + pairs * (kbp + 4) + V * (kbp + 4)
                + 2 * max(pp - 1, 0) * V * (kbp + 4),
                # prep pass: reads depth, radius, cum pair, xy, conic, both opacities, colour
                # (56 B); writes key, value, walk record, blend record (88 B)
                "pair_keys": 144 * pairs,
                # the scan of the V sorted pairs' counts: perm, gathered count, offset
                "pair_scan": 12 * V,
                # per pair: radius, conic, v_xy, v_conic (36 B); per gaussian: means, scales,
                # quats read and their cotangents written once, summed over the cameras (80 B)
                "project_bwd": 36 * per_launch("pairs_bwd", "project_bwd") + 80 * n,
                "depth_minmax": 8 * pairs,
            }
            for name, b in bytes_est.items():
                t = avg_ms(name)
                if t:
                    gbs = b / (t / 1e3) / 1e9
                    rows[name] = {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"],
                                  "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"], "ms": t}
            fwd_flops = FWD_FLOPS_PER_EVAL * work["fwd_evals"]
            bwd_flops = BWD_FLOPS_PER_EVAL * work["bwd_evals"] + BWD_FLOPS_PER_CONTRIB * work["bwd_contribs"]
            for name, fl in (("raster_fwd", fwd_flops), ("raster_bwd", bwd_flops)):
                t = avg_ms(name)
                if t:
                    tf = fl / (t / 1e3) / 1e12
                    rows[name] = {"bound": "fp32", "achieved": tf, "peak": fp32_peak,
                                  "unit": "TFLOP/s", "frac": tf / fp32_peak, "ms": t}
            total_ms = {k: v["ms"] for k, v in kern.items()}
            dom = dominant
            for name, t in TRAFFIC_BYTES_PER_LAUNCH.items():
                if name in rows and args.config == 2 and args.n is None and world == 1:
                    rows[name]["traffic"] = t
            roof = dict(rows.get(dom, {}))
            if roof and live["launches"]:
                # the dominant kernel's time as measured live inside the timed steps
                t_live = live["ms"] / live["launches"]
                scale = roof["ms"] / t_live
                roof["achieved"] *= scale
                roof["frac"] *= scale
                roof["ms_per_launch"] = t_live
            roof.pop("ms", None)
            roof.update({"kernel": dom, "traffic": roof.get("traffic"),
                         "timing": "CUDA events around this kernel on its stream during the "
                                   "timed steps (the only stage timed there)",
                         "peak_source": peak_src if roof.get("bound") == "hbm"
                         else f"derived: {props.multi_processor_count} SMs x 128 FP32 lanes x 2 x "
                              f"{sm_mhz:.0f} MHz sampled SM clock"})
            launches = sum(k["kernels"] for k in kern.values())
            line = {
                "metric": metric, "value": value, "unit": "frames/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": f"synthetic (seeded, config {args.config} distributions)",
                "config": arm_config(workload, n, per, world, input_bytes, flush,
                                     None if world == 1 else
                                     ("nvls (library kernel)" if reducer is not None
                                      else NCCL_SPLIT_LABEL if split is not None
                                      else NCCL_LABEL)),
                "roofline": roof,
                "kernels": {k: {**v, "share": v["ms"] / max(sum(total_ms.values()), 1e-9)}
                            for k, v in kern.items()},
                "kernels_source": "a pass of the same K steps right before the timed ones, with "
                                  "every stage bracketed by CUDA events",
                "kernel_rooflines": rows,
                "work_per_step": work,
                "clocks": clocks,
                "exchange": exchange,
                "ranks": rank_split,
                "host": {"cpus": os.cpu_count(),
                         "cpus_usable": len(os.sched_getaffinity(0))
                         if hasattr(os, "sched_getaffinity") else None},
                "e2e": e2e,
                "cpu_baseline": cpu,
                "gpu_launches": int(launches),
            }
            print(json.dumps(line), flush=True)
    finally:
        teardown(world, closers)


if __name__ == "__main__":
    main()
