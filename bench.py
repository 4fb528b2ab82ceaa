"""Forward + backward throughput of the Gabor splatting render path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

One step = render (public API, projection + binning + compositing) of one batch of
the synthetic workload, the benchmark loss, and backward to every input.  Prints one
JSON line (rank 0).  Metric: fwd+bwd Mpix/s = pixels rendered / (forward + backward
time), whole job, max over ranks.

Default workload: config 1 (classic Gabor, SH degree 3, N=500k surfels, 4 cameras at
1920x1080).  With N GPUs each rank renders its own independent scene of that size
(scene sharding, weak scaling, no collective in the step).  Config 3 (32 scenes x 8
cameras) shards its scenes across ranks (strong scaling).

--impl reference times the reference algorithm's CPU restatement (the oracle; the
reference has no CPU renderer of its own) on a bounded pixel window of the same
workload, on the host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from diff_gabor_splatting_b200.workloads import crop, loss_of, make_workload  # noqa: E402

METRIC = "fwd+bwd Mpix/s"
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
# my kernels launched per C entry point (CUB library kernels are not counted)
OWN_KERNELS = {"gs_project_forward": 1, "gs_project_backward": 1, "gs_bin_count": 2,
               "gs_bin_sort": 2, "gs_composite_forward": 1, "gs_composite_backward": 1,
               "gs_sh_forward": 1, "gs_sh_backward": 1, "gs_pack_geometry": 1,
               "gs_pack_rows": 1, "gs_unpack_geometry_grads": 1, "gs_unpack_rows": 1}


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--config", type=int, default=1, choices=[0, 1, 2, 3, 4])
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    p.add_argument("--cpu-window", type=int, default=64, help="CPU sample window (pixels)")
    p.add_argument("--surfels", type=int, default=None, help="override N (profiling cases)")
    p.add_argument("--cameras", type=int, default=None, help="override C (profiling cases)")
    p.add_argument("--scenes", type=int, default=None, help="override S (profiling cases)")
    return p.parse_args()


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.distributed.init_process_group(
            "nccl" if args.impl == "ours" else "gloo", timeout=timedelta(seconds=300))
    return world, rank, local


def shard(workload_config, rank, world, overrides):
    """This rank's scenes: config 3 splits its 32 scenes, others give each rank a scene."""
    if workload_config in (3,):
        full = make_workload(workload_config, **overrides)
        S = full.scenes
        lo, hi = rank * S // world, (rank + 1) * S // world
        inputs = {k: v[lo:hi].contiguous() for k, v in full.inputs.items()}
        full.inputs, full.scenes = inputs, hi - lo
        return full, "strong"
    return make_workload(workload_config, seed=rank, **overrides), "weak"


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                try:
                    rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
                except ValueError:
                    continue
        if not rows:
            return None
        sm = [r[0] for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[2]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def device_inputs(w, device):
    return {k: v.to(device).requires_grad_() for k, v in w.inputs.items()}


def step(fn, w, values):
    rgb, alpha, meta = fn(**values, **w.kwargs(), validate=False)
    loss = loss_of(rgb, alpha, meta, w.depth_normal_loss)
    loss.backward()
    return loss


def max_over_ranks(value, world, device):
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def peaks():
    if PEAKS_FILE.exists():
        data = json.loads(PEAKS_FILE.read_text())
        return data, "measured"
    return FALLBACK_PEAKS, "fallback"


def roofline(stage_ms, counts, w, steps):
    """Roofline of the dominant stage (largest total device time)."""
    from diff_gabor_splatting_b200 import perfmodel

    name, (calls, total) = max(stage_ms.items(), key=lambda kv: kv[1][1])
    per_launch_ms = total / max(calls, 1)
    model = perfmodel.stage_model(name, counts, w)
    data, source = peaks()
    out = {"kernel": name, "launches": calls, "ms_per_launch": per_launch_ms,
           "bound": model["bound"], "unit": model["unit"], "traffic": None}
    if model["bound"] == "hbm":
        achieved = model["work"] / (per_launch_ms * 1e-3) / 1e9
        peak = data["hbm_gbs"]
        out["peak_source"] = f"hbm_gbs of {source}"
    else:
        achieved = model["work"] / (per_launch_ms * 1e-3) / 1e12
        peak = perfmodel.FP32_NOMINAL_TFLOPS
        out["peak_source"] = "nominal FP32 (148 SM x 128 lanes x 2 x 1.965 GHz); no measured FP32 peak"
    out.update(achieved=achieved, peak=peak, frac=achieved / peak, work_per_launch=model["work"],
               work_basis=model["basis"])
    return out


def cpu_baseline(w, window, cores=None):
    """Oracle fwd+bwd on a window of camera 0 (tile-aligned, centred); Mpix/s."""
    from oracle import gabor_oracle as O

    if cores:
        torch.set_num_threads(cores)
    x0 = ((w.width - window) // 2) // 16 * 16
    y0 = ((w.height - window) // 2) // 16 * 16
    sample = crop(w, x0, y0, min(window, w.width), min(window, w.height), camera_ids=[0])
    names = (["input_weights", "input_biases", "output_weights", "output_biases"]
             if w.method == "neural" else
             ["colors", "secondary_colors", "frequency_weights", "frequency_magnitudes", "phases"])
    leaves = {k: v.clone().requires_grad_() for k, v in sample.inputs.items()}
    t0 = time.perf_counter()
    rgb, alpha, meta = O.render(leaves["means"], leaves["quaternions"], leaves["scales"],
                                leaves["opacities"], [leaves[k] for k in names],
                                leaves["view_matrices"], leaves["intrinsics"], sample.width,
                                sample.height, backgrounds=leaves["backgrounds"],
                                packed=sample.packed, neural=w.method == "neural",
                                sh_degree=sample.sh_degree)
    loss_of(rgb, alpha, meta, w.depth_normal_loss).backward()
    seconds = time.perf_counter() - t0
    desc = (f"config {w.config}, camera 0, {sample.width}x{sample.height} window at "
            f"({x0},{y0}), all {w.surfels} surfels projected; fwd+bwd with autograd")
    return sample.pixels / seconds / 1e6, seconds, desc


def run_reference(args, world, rank):
    """CPU arm: the oracle (reference algorithm restated on the CPU), rank 0 only."""
    if rank != 0:
        return
    w = make_workload(args.config, surfels=args.surfels, cameras=args.cameras, scenes=args.scenes)
    cores = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_baseline(w, args.cpu_window, cores)
    rates, seconds, desc = [], 0.0, ""
    for _ in range(args.steps):
        rate, sec, desc = cpu_baseline(w, args.cpu_window, cores)
        rates.append(rate)
        seconds += sec
    pixels = args.steps * (min(args.cpu_window, w.width) * min(args.cpu_window, w.height))
    value = pixels / seconds / 1e6
    line = {"metric": METRIC, "value": value, "unit": "Mpix/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": seconds / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_desc(w, "cpu"),
            "cpu_baseline": {"value": value, "unit": "Mpix/s", "cores": torch.get_num_threads(),
                             "kind": "port", "sample": desc},
            "e2e": {"value": value, "unit": "Mpix/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_desc(w, parallelism):
    return {"workload": f"config {w.config}: {w.method}"
            + (f" SH{w.sh_degree}" if w.sh_degree is not None else "")
            + f", {w.scenes} scene(s) x {w.cameras} camera(s) {w.width}x{w.height}, "
              f"N={w.surfels} surfels/scene" + (", packed" if w.packed else ""),
            "global_batch": w.scenes * w.cameras, "pixels_per_step": w.pixels,
            "parallelism": parallelism,
            "l2": "working set larger than L2 (records, sort buffers and maps exceed 126 MB)"}


def main():
    args = parse()
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    from diff_gabor_splatting_b200 import _native as nat
    from diff_gabor_splatting_b200 import perfmodel, rasterize_gabors, rasterize_neural_gabors

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    overrides = dict(surfels=args.surfels, cameras=args.cameras, scenes=args.scenes)
    w, scaling = shard(args.config, rank, world, overrides)
    fn = rasterize_gabors if w.method == "classic" else rasterize_neural_gabors
    values = device_inputs(w, device)
    for _ in range(max(args.warmup, 3)):
        for v in values.values():
            v.grad = None
        step(fn, w, values)
    torch.cuda.synchronize()
    counts = perfmodel.count_work(fn, w, values)
    # timed region: K steps, inputs resident in HBM
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks, nat.StageTimer() as timer:
        start.record()
        for _ in range(args.steps):
            for v in values.values():
                v.grad = None
            step(fn, w, values)
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world, device)
    stage = timer.totals()
    launches = sum(OWN_KERNELS.get(name, 1) * calls for name, (calls, _) in stage.items())
    pixels_all = w.pixels * world if scaling == "weak" else make_workload_pixels(args.config,
                                                                                  overrides)
    value = pixels_all * args.steps / (ms * 1e-3) / 1e6
    # end to end: host (pinned) inputs copied in every step, loss read back
    e2e = None
    if not args.no_e2e:
        host = {k: v.pin_memory() for k, v in w.inputs.items()}
        h2d = sum(v.numel() * v.element_size() for v in host.values())
        for _ in range(2):
            dev = {k: v.to(device, non_blocking=True).requires_grad_() for k, v in host.items()}
            step(fn, w, dev).item()
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            dev = {k: v.to(device, non_blocking=True).requires_grad_() for k, v in host.items()}
            step(fn, w, dev).item()
        e1.record()
        torch.cuda.synchronize()
        barrier(world)
        ems = max_over_ranks(e0.elapsed_time(e1), world, device)
        e2e = {"value": pixels_all * args.steps / (ems * 1e-3) / 1e6, "unit": "Mpix/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
               "ms_per_step": ems / args.steps}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        rate, sec, desc = cpu_baseline(w, args.cpu_window, cores)
        cpu = {"value": rate, "unit": "Mpix/s", "cores": torch.get_num_threads(),
               "kind": "port", "sample": desc, "seconds": sec}
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "Mpix/s", "n_gpus": world,
                "steps": args.steps, "warmup": max(args.warmup, 3),
                "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": scaling,
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, config shapes)",
                "config": config_desc(w, f"scene-sharded x{world}" if world > 1 else "single"),
                "gpu_launches": launches,
                "roofline": roofline(stage, counts, w, args.steps),
                "stages_ms_per_step": {k: v[1] / args.steps for k, v in stage.items()},
                "work": counts, "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks.summary()}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def make_workload_pixels(config, overrides):
    w = make_workload(config, **dict(overrides, surfels=1))
    return w.pixels


if __name__ == "__main__":
    main()
