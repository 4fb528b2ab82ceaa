"""Forward + backward throughput of the Gabor splatting render path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

One step = render (public API, projection + binning + compositing) of one batch of
the synthetic workload, the benchmark loss, and backward to every input.  Prints one
JSON line (rank 0).  Metric: fwd+bwd Mpix/s = pixels rendered / (forward + backward
time), whole job, max over ranks.  `value` has the inputs resident in HBM; `e2e` is
the same metric with every step's inputs copied from pinned host memory (on a side
stream, overlapping the previous step, as a prefetching loader does) and the loss read
back.

Default workload: config 3 (classic Gabor, SH degree 1, a fused batch of 32 independent
scenes x 8 cameras at 256x256, N=50k surfels per scene, packed=True), the batched
configuration the scaling target names.  It is strong-scaled: the 32 scenes are split
into contiguous blocks over the N ranks (N=1 renders all 32), with no collective in the
step; each rank renders its block in one call.  Config 4 shards the same way (cameras of
a scene split over ranks, with an NCCL all-reduce of its parameter gradients, when there
are more ranks than scenes); configs 0-2 (one scene) run one independent replica per
rank (weak scaling), and --split-cameras splits config 1's cameras instead.

Besides `value` (tight bins, the library's default) the line carries `square_bins`, the
same step with the reference's square tile rectangles (point lists identical to the
reference's), and, at N=1, `reference_cuda`: the reference's own CUDA extension
(compiled unmodified into oracle/_ref) timed on the same workload, steps and loss in a
child process after the timed region (oracle/ref_gpu_bench.py), with `vs_reference_cuda`
= value / its value.  Renders run with validate=False on both sides (the reference's
numerical checks cost one host synchronisation per call).

--impl reference times the reference algorithm's CPU restatement (the oracle; the
reference has no CPU renderer of its own) on a bounded pixel window of one camera of one
scene of the same workload, on the host cores, rank 0 only.
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
               "gs_bin_sort": 8, "gs_composite_forward": 1, "gs_composite_backward": 1,
               "gs_composite_forward_split": 1, "gs_composite_backward_split": 1,
               "gs_sh_forward": 1, "gs_sh_backward": 1, "gs_pack_geometry": 1,
               "gs_pack_rows": 1, "gs_unpack_geometry_grads": 1, "gs_unpack_rows": 1,
               "gs_adam_step": 1, "gs_adam_step_capturable": 2, "gs_bin_arena": 6,
               "gs_pair_ids": 1, "gs_pack_surfel_rows": 1, "gs_unpack_surfel_rows": 1}


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--config", type=int, default=3, choices=[0, 1, 2, 3, 4])
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    p.add_argument("--no-square", action="store_true",
                   help="skip the square-bins leg (the reference's tile rectangles)")
    p.add_argument("--no-reference-cuda", action="store_true",
                   help="skip timing the reference CUDA extension (N=1 only)")
    p.add_argument("--cpu-window", type=int, default=64, help="CPU sample window (pixels)")
    p.add_argument("--surfels", type=int, default=None, help="override N (profiling cases)")
    p.add_argument("--cameras", type=int, default=None, help="override C (profiling cases)")
    p.add_argument("--scenes", type=int, default=None, help="override S (profiling cases)")
    p.add_argument("--optimizer", choices=["none", "fused", "torch"], default="none",
                   help="add an Adam step (lr 1e-3) over every parameter to each step: this\n"
                        "build's fused kernel or torch.optim.Adam (the reference's loop);\n"
                        "reported under 'optimizer' (the e2e leg is skipped)")
    p.add_argument("--pixels", type=int, default=None,
                   help="render only this many seeded random pixels per camera (selected-\n"
                        "pixel mode); the metric counts the selected pixels")
    p.add_argument("--graph", action="store_true",
                   help="also time the step captured as one CUDA graph (arena binning, no\n"
                        "host sync): reported under 'graph' beside the eager value")
    p.add_argument("--split-cameras", action="store_true",
                   help="shard one workload over the ranks, splitting a scene's cameras "
                        "(gradient all-reduce) when there are more ranks than scenes")
    p.add_argument("--scenes-per-call", type=int, default=None,
                   help="scenes per render call (config 4 defaults to 1)")
    return p.parse_args()


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        if args.impl == "ours":
            torch.cuda.set_device(local)
            torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300),
                                                 device_id=torch.device("cuda", local))
        else:
            torch.distributed.init_process_group("gloo", timeout=timedelta(seconds=300))
    return world, rank, local


class Job:
    """This rank's share of one step: render calls (each a scene block) + collectives."""

    def __init__(self, args, rank, world):
        from diff_gabor_splatting_b200 import sharding

        overrides = dict(surfels=args.surfels, cameras=args.cameras, scenes=args.scenes)
        self.sharding = sharding
        if args.config in (3, 4) or args.split_cameras:
            # one workload sharded over the ranks (strong scaling)
            full = make_workload(args.config, **overrides)
            self.scaling = "strong"
            self.total_pixels = full.pixels
            shards = sharding.plan(full.scenes, full.cameras, world)
            self.groups = sharding.groups_for(shards) if world > 1 else {}
            self.shard = shards[rank]
            part = sharding.take(full.inputs, self.shard)
            self.workload = full
        else:
            # every rank renders its own independent scene of the config (weak scaling)
            full = make_workload(args.config, seed=rank, **overrides)
            self.scaling = "weak"
            self.total_pixels = full.pixels * world
            self.groups, self.shard = {}, None
            part = full.inputs
            self.workload = full
        per_call = args.scenes_per_call or (1 if args.config == 4 else None)
        S = next(iter(part.values())).shape[0]
        step = per_call or S
        self.calls = [{k: v[s:s + step] for k, v in part.items()} for s in range(0, S, step)]
        self.local_pixels = sum(c["view_matrices"].shape[0] * c["view_matrices"].shape[1]
                                for c in self.calls) * full.width * full.height
        self.pixel_count = args.pixels
        self.pixels = None
        self.timing = False          # collect the camera-split all-reduce's CUDA events
        self.allreduce_events = []
        if args.pixels:   # selected-pixel mode: the metric counts selected pixels
            scale = args.pixels / (full.width * full.height)
            self.total_pixels = round(self.total_pixels * scale)
            self.local_pixels = round(self.local_pixels * scale)

    def pixels_on(self, device, seed=0):
        """Seeded random (x, y) per camera for every call (selected-pixel mode)."""
        if not self.pixel_count:
            return None
        w = self.workload
        g = torch.Generator().manual_seed(seed)
        out = []
        for c in self.calls:
            shape = tuple(c["view_matrices"].shape[:-2]) + (self.pixel_count,)
            xy = torch.stack((torch.randint(0, w.width, shape, generator=g),
                              torch.randint(0, w.height, shape, generator=g)), -1)
            out.append(xy.to(torch.int32).to(device))
        return out

    def inputs_on(self, device):
        return [{k: v.to(device).contiguous().requires_grad_() for k, v in c.items()}
                for c in self.calls]


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index, interval_ms=50):
        self.index = index
        self.interval_ms = interval_ms
        self.proc = None
        self.lines = []
        self.first = 0   # samples before this index precede the timed region
        self.live = threading.Event()

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", str(self.interval_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            self.live.wait(timeout=5)   # sampling has started before the timer does
        except (OSError, ValueError):
            self.proc = None
        self.first = len(self.lines)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())
            self.live.set()

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        for line in self.lines[self.first:] or self.lines[-1:]:
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


class OptimizerStep:
    """The optional Adam step of a training step, timed with CUDA events."""

    def __init__(self, kind, calls):
        from diff_gabor_splatting_b200.optim import FusedAdam

        self.kind = kind
        self.params = [t for c in calls for t in c.values() if t.requires_grad]
        cls = FusedAdam if kind == "fused" else torch.optim.Adam
        self.optimizer = cls(self.params, lr=1e-3)
        self.events = []
        self.timing = False

    def __call__(self):
        if self.timing:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            self.optimizer.step()
            end.record()
            self.events.append((start, end))
        else:
            self.optimizer.step()

    def summary(self, steps, hbm_gbs):
        ms = sum(a.elapsed_time(b) for a, b in self.events) / max(len(self.events), 1)
        numel = sum(t.numel() for t in self.params)
        moved = 28 * numel   # read p, g, m, v; write p, m, v (float32)
        gbs = moved / (ms * 1e-3) / 1e9
        return {"impl": "fused gs_adam_step" if self.kind == "fused" else "torch.optim.Adam",
                "params": numel, "tensors": len(self.params), "ms_per_step": ms,
                "bytes_per_step": moved, "achieved_gbs": gbs, "peak_gbs": hbm_gbs,
                "frac": gbs / hbm_gbs}


def step(fn, job, calls, optimizer=None):
    """Render every call of this rank, backward with the batch-mean loss, sum parameter
    gradients over the camera-split group when the scene is split, and take the
    optional optimizer step."""
    w = job.workload
    total = None
    for i, values in enumerate(calls):
        for v in values.values():
            v.grad = None
        extra = {} if job.pixels is None else {"pixels": job.pixels[i]}
        rgb, alpha, meta = fn(**values, **w.kwargs(), **extra, validate=False)
        pixels = rgb.shape[:-1].numel()
        loss = loss_of(rgb, alpha, meta, w.depth_normal_loss) * (pixels / job.total_pixels)
        loss.backward()
        total = loss.detach() if total is None else total + loss.detach()
    if job.shard is not None and job.shard.split:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for values in calls:
            params = [t for k, t in values.items() if k not in job.sharding.PER_CAMERA]
            job.sharding.allreduce_gradients(params, job.groups[job.shard.group_ranks])
        t1.record()
        if job.timing:
            job.allreduce_events.append((t0, t1))
    if optimizer is not None:
        optimizer()
    return total


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


def fp32_peak(device):
    """FP32 multiply-add throughput of this GPU (TFLOP/s), measured with gs_fp32_probe:
    148 x 8 blocks of 256 threads, eight independent FFMA chains each, best of three
    launches of ~6 ms (CUDA events); also the paired FFMA2 form."""
    from diff_gabor_splatting_b200 import _native as nat

    sms = torch.cuda.get_device_properties(device).multi_processor_count
    blocks, iterations = sms * 8, 100_000
    out = torch.zeros(blocks, device=device)
    result = {}
    for paired in (0, 1):
        flops = blocks * 256 * iterations * 8 * (4 if paired else 2)
        best = 0.0
        for i in range(4):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            nat.call("gs_fp32_probe", blocks, iterations, paired, nat.ptr(out),
                     nat.stream_of(device))
            b.record()
            torch.cuda.synchronize()
            if i:   # the first launch warms up
                best = max(best, flops / (a.elapsed_time(b) * 1e-3) / 1e12)
        result["ffma2_tflops" if paired else "ffma_tflops"] = best
    return result


def roofline(stage_ms, counts, w, steps, calls_per_step, fp32=None):
    """Roofline of the dominant stage (largest total device time in the timed region).

    achieved = algorithmic work of every launch of that stage in the timed region
    (the counted work of one render call x calls per step x steps) / their summed
    CUDA-event time.
    """
    from diff_gabor_splatting_b200 import perfmodel

    name, (launches, total_ms) = max(stage_ms.items(), key=lambda kv: kv[1][1])
    model = perfmodel.stage_model(name, counts, w)
    work = model["work"] * calls_per_step * steps
    data, source = peaks()
    dram = perfmodel.traffic(name, counts, w.config)
    out = {"kernel": name, "launches": launches, "ms_per_launch": total_ms / max(launches, 1),
           "bound": model["bound"], "unit": model["unit"],
           "traffic": dram * calls_per_step * steps / max(launches, 1) if dram else None}
    if dram:
        out["traffic_basis"] = ("DRAM read+write bytes of one ncu-profiled small-case launch of "
                                "the same config (config 1 otherwise), scaled by accepted samples")
    if model["bound"] == "hbm":
        achieved = work / (total_ms * 1e-3) / 1e9
        peak = data["hbm_gbs"]
        out["peak_source"] = f"hbm_gbs of {source}"
    else:
        achieved = work / (total_ms * 1e-3) / 1e12
        if fp32:
            peak = fp32["ffma_tflops"]
            out["peak_source"] = ("measured on this GPU by gs_fp32_probe (FFMA chains, "
                                  f"{fp32['ffma_tflops']:.1f} TFLOP/s; paired FFMA2 "
                                  f"{fp32['ffma2_tflops']:.1f}); nominal "
                                  f"{perfmodel.FP32_NOMINAL_TFLOPS:.1f}")
        else:
            peak = perfmodel.FP32_NOMINAL_TFLOPS
            out["peak_source"] = "nominal FP32 (148 SM x 128 lanes x 2 flop x 1.965 GHz)"
    out.update(achieved=achieved, peak=peak, frac=achieved / peak,
               work_per_launch=model["work"] * calls_per_step * steps / max(launches, 1),
               work_basis=model["basis"])
    return out


def cpu_baseline(w, window, cores=None):
    """Oracle fwd+bwd on a window of camera 0 (tile-aligned, centred); Mpix/s."""
    from oracle import gabor_oracle as O

    if cores:
        torch.set_num_threads(cores)
    x0 = ((w.width - window) // 2) // 16 * 16
    y0 = ((w.height - window) // 2) // 16 * 16
    sample = crop(w, x0, y0, min(window, w.width), min(window, w.height), camera_ids=[0],
                  scene_ids=[0])
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
    desc = (f"config {w.config}, scene 0, camera 0, {sample.width}x{sample.height} window at "
            f"({x0},{y0}), all {w.surfels} surfels of the scene projected (the projection is "
            f"part of the per-window cost); fwd+bwd with autograd")
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
            "validate": False,
            "validate_note": "renders called with validate=False (both this build and the "
                             "reference CUDA arm); the reference's default validate=True adds "
                             "its numerical checks and one host synchronisation per call",
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
    job = Job(args, rank, world)
    w = job.workload
    fn = rasterize_gabors if w.method == "classic" else rasterize_neural_gabors
    calls = job.inputs_on(device)
    job.pixels = job.pixels_on(device)
    opt = OptimizerStep(args.optimizer, calls) if args.optimizer != "none" else None
    for _ in range(max(args.warmup, 3)):
        step(fn, job, calls, opt)
    torch.cuda.synchronize()
    counts = perfmodel.count_work(fn, w, calls[0])
    # timed region: K steps, inputs resident in HBM
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks, nat.StageTimer() as timer:
        if opt is not None:
            opt.timing = True
        job.timing = True
        start.record()
        for _ in range(args.steps):
            step(fn, job, calls, opt)
        end.record()
        torch.cuda.synchronize()
        job.timing = False
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world, device)
    stage = timer.totals()
    allreduce = None
    if job.allreduce_events:
        ar_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in job.allreduce_events)
                               / len(job.allreduce_events), world, device)
        bucket = sum(t.numel() * 4 for c in calls for k, t in c.items()
                     if k not in job.sharding.PER_CAMERA)
        group = len(job.shard.group_ranks)
        allreduce = {"ms_per_step": ar_ms, "bucket_bytes": bucket, "group_ranks": group,
                     "bus_gbs": bucket * 2 * (group - 1) / group / (ar_ms * 1e-3) / 1e9,
                     "timing": "CUDA events around the NCCL all-reduce of each step, mean over "
                               "the timed steps, max over ranks"}
    own = dict(OWN_KERNELS)
    if w.sh_degree is not None and w.sh_degree >= 2:   # plus its SH coefficient kernel
        own["gs_project_backward"] = 2
    launches = sum(own.get(name, 1) * n for name, (n, _) in stage.items() if name in own)
    pixels_all = job.total_pixels
    value = pixels_all * args.steps / (ms * 1e-3) / 1e6
    # end to end: every step's inputs copied from pinned host memory and its loss read
    # back, as a training loop with a prefetching loader does it: step k+1's inputs are
    # copied on a side stream while step k computes (each step waits for its own copy;
    # the first copy starts after the opening event, so all K copies are timed)
    e2e = None
    if not args.no_e2e and opt is None:
        host = [{k: v.pin_memory() for k, v in c.items()} for c in job.calls]
        h2d = sum(v.numel() * v.element_size() for c in host for v in c.values())
        copies = torch.cuda.Stream(device)

        def upload():
            copies.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(copies):
                dev = [{k: v.to(device, non_blocking=True) for k, v in c.items()} for c in host]
                ready = torch.cuda.Event()
                ready.record(copies)
            return dev, ready

        def e2e_steps(n):
            pending = upload()
            for i in range(n):
                dev, ready = pending
                torch.cuda.current_stream().wait_event(ready)
                for c in dev:
                    for v in c.values():
                        v.record_stream(torch.cuda.current_stream())
                        v.requires_grad_()
                if i + 1 < n:
                    pending = upload()
                step(fn, job, dev).item()

        e2e_steps(2)
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        e2e_steps(args.steps)
        e1.record()
        torch.cuda.synchronize()
        barrier(world)
        ems = max_over_ranks(e0.elapsed_time(e1), world, device)
        e2e = {"value": pixels_all * args.steps / (ems * 1e-3) / 1e6, "unit": "Mpix/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
               "ms_per_step": ems / args.steps,
               "copies": "pinned host -> device on a side stream, overlapping the previous step",
               "read_back": "the step's loss (4 bytes); images and gradients stay on the "
                            "device, as in an on-device training loop"}
    square = None
    if not args.no_square and opt is None:
        square = square_leg(args, job, fn, calls, device, world, pixels_all)
    graph = graph_leg(args, job, fn, calls, device, world, pixels_all) if args.graph else None
    fp32 = fp32_peak(device) if rank == 0 else None
    ref_cuda = None
    if rank == 0 and world == 1 and not args.no_reference_cuda and not args.pixels:
        ref_cuda = reference_cuda(args)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        rate, sec, desc = cpu_baseline(w, args.cpu_window, cores)
        cpu = {"value": rate, "unit": "Mpix/s", "cores": torch.get_num_threads(),
               "kind": "port", "sample": desc, "seconds": sec}
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "Mpix/s", "n_gpus": world,
                "steps": args.steps, "warmup": max(args.warmup, 3),
                "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": job.scaling,
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, config shapes)",
                "config": config_desc(w, parallelism(job, world)),
                "gpu_launches": launches,
                "roofline": roofline(stage, counts, w, args.steps, len(job.calls), fp32),
                "stages_ms_per_step": {k: v[1] / args.steps for k, v in stage.items()},
                "work": counts, "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks.summary()}
        if args.pixels:
            line["config"]["selected_pixels_per_camera"] = args.pixels
            line["config"]["pixels_per_step"] = pixels_all
            line["roofline"]["note"] = "kernel work counted on a full render of the workload"
        if allreduce is not None:
            line["allreduce"] = allreduce
        if square is not None:
            line["square_bins"] = square
        if ref_cuda is not None:
            line["reference_cuda"] = ref_cuda
            if ref_cuda.get("value"):
                line["vs_reference_cuda"] = value / ref_cuda["value"]
                if e2e is not None:
                    line["e2e_vs_reference_cuda"] = e2e["value"] / ref_cuda["value"]
        if graph is not None:
            line["graph"] = graph
        if opt is not None:
            line["optimizer"] = opt.summary(args.steps, peaks()[0]["hbm_gbs"])
            line["config"]["step"] = "render + backward + Adam step (lr 1e-3) on every parameter"
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def square_leg(args, job, fn, calls, device, world, pixels_all):
    """The same step with the reference's square tile rectangles (``TIGHT_BINNING =
    False``): point lists identical to the reference's, so the gain of tight binning is
    separable from the kernels'.  Timed like the main loop (device events, max over
    ranks)."""
    from diff_gabor_splatting_b200 import rendering

    previous = rendering.TIGHT_BINNING
    rendering.TIGHT_BINNING = False
    try:
        for _ in range(2):
            step(fn, job, calls)
        rendering.WORK = {}
        try:
            step(fn, job, calls)
            torch.cuda.synchronize()
            intersections = rendering.WORK.get("intersections", 0)
        finally:
            rendering.WORK = None
        barrier(world)
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(args.steps):
            step(fn, job, calls)
        s1.record()
        torch.cuda.synchronize()
        barrier(world)
        sms = max_over_ranks(s0.elapsed_time(s1), world, device)
    finally:
        rendering.TIGHT_BINNING = previous
    return {"value": pixels_all * args.steps / (sms * 1e-3) / 1e6, "unit": "Mpix/s",
            "ms_per_step": sms / args.steps, "intersections_rank0": intersections,
            "binning": "square tile rectangles (the reference's bins; point lists identical "
                       "to the reference's)"}


def reference_cuda(args):
    """The reference's CUDA extension (oracle/_ref, compiled unmodified for sm_100a) on
    the same workload, steps, warm-up and loss, timed in a child process after this
    process's timed region (oracle/ref_gpu_bench.py).  Measurement only: nothing of the
    reference runs in this build's step."""
    script = ROOT / "oracle" / "ref_gpu_bench.py"
    ref_pkg = ROOT / "oracle" / "_ref" / "gabor_splatting"
    if not ref_pkg.exists():
        return {"unavailable": "the compiled reference is not in oracle/_ref"}
    cmd = [sys.executable, str(script), "--config", str(args.config), "--steps",
           str(args.steps), "--warmup", str(max(args.warmup, 3))]
    for flag, value in (("--surfels", args.surfels), ("--cameras", args.cameras),
                        ("--scenes", args.scenes)):
        if value:
            cmd += [flag, str(value)]
    torch.cuda.empty_cache()   # leave the device memory to the child
    try:
        out = subprocess.run(cmd, capture_output=True, text=True, timeout=1500)
    except subprocess.TimeoutExpired:
        return {"unavailable": "reference timing exceeded 1500 s"}
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    if out.returncode != 0 or not lines:
        return {"unavailable": f"reference timing failed (rc {out.returncode}): "
                               + (out.stderr.strip().splitlines() or [""])[-1][:300]}
    return json.loads(lines[-1])


def graph_leg(args, job, fn, calls, device, world, pixels_all):
    """The same step as one CUDA graph replay (``GraphedStep``: arena binning sized 1.25x
    the live counts, no host synchronisation), timed like the eager loop, plus its
    end-to-end form (host inputs copied into the captured tensors, loss read back)."""
    from diff_gabor_splatting_b200.graphs import GraphedStep

    if len(calls) != 1 or (job.shard is not None and job.shard.split):
        return {"unavailable": "graph leg needs one render call per rank and no camera split"}
    w = job.workload
    static = calls[0]
    # with --optimizer fused the graph records the whole training step: render, loss,
    # backward and the Adam step (FusedAdam with device step counts)
    optimizer = None
    if args.optimizer == "torch":
        return {"unavailable": "the graph leg records FusedAdam(capturable=True) only"}
    if args.optimizer == "fused":
        from diff_gabor_splatting_b200.optim import FusedAdam
        optimizer = FusedAdam([t for t in static.values() if t.requires_grad], lr=1e-3,
                              capturable=True)
    # packing counts visible pairs on the host; images and gradients are the same dense
    step_graph = GraphedStep(fn, static,
                             lambda rgb, alpha, meta: loss_of(rgb, alpha, meta,
                                                              w.depth_normal_loss),
                             optimizer=optimizer, **dict(w.kwargs(), packed=False))
    for _ in range(3):
        step_graph.replay()
    barrier(world)
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record()
    for _ in range(args.steps):
        step_graph.replay()
    g1.record()
    torch.cuda.synchronize()
    barrier(world)
    gms = max_over_ranks(g0.elapsed_time(g1), world, device)
    out = {"value": pixels_all * args.steps / (gms * 1e-3) / 1e6, "unit": "Mpix/s",
           "ms_per_step": gms / args.steps, "overflow": step_graph.arena.overflowed(),
           "arena": [step_graph.arena.max_intersections, step_graph.arena.max_spans],
           "packed": False,
           "optimizer": "FusedAdam(capturable=True) in the graph" if optimizer else None}
    host = {k: v.detach().cpu().pin_memory() for k, v in static.items()}
    h2d = sum(v.numel() * v.element_size() for v in host.values())

    def e2e_replay():
        with torch.no_grad():
            for k, v in host.items():
                static[k].copy_(v, non_blocking=True)
        return step_graph.replay().item()

    for _ in range(2):
        e2e_replay()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_replay()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    ems = max_over_ranks(e0.elapsed_time(e1), world, device)
    out["e2e"] = {"value": pixels_all * args.steps / (ems * 1e-3) / 1e6, "unit": "Mpix/s",
                  "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                  "ms_per_step": ems / args.steps}
    return out


def parallelism(job, world):
    if world == 1:
        return "single GPU" + (f", {len(job.calls)} render calls per step"
                               if len(job.calls) > 1 else "")
    if job.scaling == "weak":
        return f"scene replicas x{world} (one independent scene per GPU, no collective)"
    if job.shard.split:
        return (f"camera split x{world} (ranks per scene {len(job.shard.group_ranks)}, "
                "NCCL all-reduce of parameter gradients)")
    return f"scene sharded x{world} (contiguous scene blocks, no collective)"


if __name__ == "__main__":
    main()
