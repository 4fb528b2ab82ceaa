"""Time the reference CUDA extension (oracle/_ref, built by oracle/build_ref.sh) on a
B200 through its own public API, on the same seeded workloads as bench.py.

    python oracle/ref_gpu_bench.py [--config 1] [--steps 10] [--warmup 3]

Measurement infrastructure only (the reference is the thing being timed here, never
part of this library).  Prints one JSON line: fwd+bwd Mpix/s of the reference with
the same loss, inputs resident on the device, CUDA-event timing of K steps.
Config 4 exceeds the reference's int32 intersection limit as one call; it is run one
scene per call (the reference's own batching limit), and the line says so.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from oracle import reference  # noqa: E402

ref = reference.load()   # the compiled reference package, as module gs_reference

from diff_gabor_splatting_b200.workloads import loss_of, make_workload  # noqa: E402


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--config", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--surfels", type=int, default=None)
    p.add_argument("--cameras", type=int, default=None)
    p.add_argument("--scenes", type=int, default=None)
    args = p.parse_args()
    w = make_workload(args.config, surfels=args.surfels, cameras=args.cameras, scenes=args.scenes)
    fn = ref.rasterize_gabors if w.method == "classic" else ref.rasterize_neural_gabors
    values = {k: v.cuda().requires_grad_() for k, v in w.inputs.items()}
    chunks = [slice(s, s + 1) for s in range(w.scenes)] if args.config == 4 else [slice(None)]

    def step():
        for v in values.values():
            v.grad = None
        for sl in chunks:
            part = {k: v[sl] for k, v in values.items()}
            rgb, alpha, meta = fn(**part, **w.kwargs(), validate=False)
            loss_of(rgb, alpha, meta, w.depth_normal_loss).backward()

    for _ in range(max(args.warmup, 1)):
        step()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    print(json.dumps({"impl": "reference CUDA extension (oracle/_ref, sm_100a)",
                      "config": args.config, "metric": "fwd+bwd Mpix/s",
                      "value": w.pixels / (ms * 1e-3) / 1e6, "ms_per_step": ms,
                      "pixels_per_step": w.pixels, "steps": args.steps,
                      "calls_per_step": len(chunks), "surfels": w.surfels, "scenes": w.scenes,
                      "cameras": w.cameras, "validate": False,
                      "chunking": ("one scene per call: the batch exceeds the reference's "
                                   "int32 tile-intersection limit (rasterize.cu:469)"
                                   if len(chunks) > 1 else "one call per step")}), flush=True)


if __name__ == "__main__":
    main()
