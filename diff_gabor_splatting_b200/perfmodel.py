"""Algorithmic work per stage, for roofline fractions.

Memory-bound stages are charged the bytes they must move (HBM roofline).  The
compositors are charged floating-point work (FP32 roofline): per-event constants times
event counts measured by the kernels' own counters (tests: (pixel, record) samples
tested; accepts: samples blended forward / differentiated backward).

The constants are executed FP32 flops per event (2 x FFMA + FADD + FMUL thread
instructions with the predicate on, ncu), fitted over two classic workloads whose
test/accept ratios differ (config 1 with 100k surfels and one camera: 1.45 tests per
accept; config 3 with two scenes: 2.84), which both fit to 0.1%; the neural accept cost
follows from a neural workload (config 2, 50k surfels) given the classic test cost.
They include the backward's reduction adds (the per-warp transpose sums its lanes'
fields), which an accept pays in proportion to its warp's accepting lanes.  The
backward has two variants: without a normal-map gradient (configs 0-3) its kernel has
no normal fields; with one (config 4's loss) it keeps them.

  forward:  33 flop per test + 141 (classic) / 220 (neural) per accept
  backward: 43 flop per test + 308 (classic) / 512 (neural) per accept,
            with a normal-map gradient 45 + 325 / 523

With warp accept masks the backward tests only the records its warp accepted in the
forward (the rest are skipped, not counted), so the tests it does execute are the
costlier ones: 57 flop per executed test, fitted on the masked config-3 workload with
the accept cost held at 308.
"""

from __future__ import annotations

import torch

FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12   # 74.4 nominal; bench.py measures it

TEST_FLOP = {"forward": 33, "backward": 43, "backward_normals": 45, "backward_masked": 57}
ACCEPT_FLOP = {"classic": 141, "neural": 220}
BACKWARD_ACCEPT_FLOP = {"classic": 308, "neural": 512}
BACKWARD_ACCEPT_FLOP_NORMALS = {"classic": 325, "neural": 523}


# DRAM bytes (read + write) of one launch measured with ncu on small cases of two
# workloads -- config 1 (N=100k surfels, 1 camera) and config 3 (2 of its 32 scenes) --
# with the accepted samples of that launch.  A full-size launch is estimated by scaling
# the matching workload's bytes with its own accepted samples (the compositors' DRAM
# traffic is the record batches, gradient atomics and pixel buffers, all of which grow
# with the accepted work); other workloads use the config-1 figures.
PROFILED_TRAFFIC = {
    1: {"gs_composite_forward": (16.188672e6 + 52.855296e6, 130426868),
        "gs_composite_backward": (88.078080e6 + 3.940096e6, 130426868)},
    3: {"gs_composite_forward": (87.757056e6 + 26.615808e6, 74378371),
        "gs_composite_backward": (148.364288e6 + 18.006272e6, 74378371)},
}


def traffic(name: str, counts: dict, config: int = 1):
    """Estimated DRAM bytes per launch of ``name`` (None when not profiled)."""
    name = name.removesuffix("_split")
    table = PROFILED_TRAFFIC.get(config, PROFILED_TRAFFIC[1])
    if name not in table:
        return None
    stage = "forward" if name.endswith("forward") else "backward"
    accepts = counts.get(f"{stage}_accepts", 0)
    bytes_small, accepts_small = table[name]
    return bytes_small * accepts / accepts_small


def count_work(fn, workload, values) -> dict:
    """Run one render + backward with the kernels' counters on; return event counts."""
    from . import rendering
    from .workloads import loss_of

    rendering.WORK = {}
    try:
        for v in values.values():
            v.grad = None
        rgb, alpha, meta = fn(**values, **workload.kwargs(), validate=False)
        loss_of(rgb, alpha, meta, workload.depth_normal_loss).backward()
        torch.cuda.synchronize()
        work = rendering.WORK
    finally:
        rendering.WORK = None
    out = {k: int(v) for k, v in work.items() if k != "_counters"}
    for stage, t in work.get("_counters", []):
        tests, accepts = (int(x) for x in t.tolist())
        out[f"{stage}_tests"] = out.get(f"{stage}_tests", 0) + tests
        out[f"{stage}_accepts"] = out.get(f"{stage}_accepts", 0) + accepts
    for v in values.values():
        v.grad = None
    return out


def stage_model(name: str, counts: dict, w) -> dict:
    """{'bound', 'unit', 'work' (bytes or flop per launch), 'basis'} for one entry point."""
    name = name.removesuffix("_split")   # same kernels, maps as separate planes
    R = counts.get("records", 0)
    I = counts.get("intersections", 0)
    S, C, N = w.scenes, w.cameras, w.surfels
    K = 0 if w.sh_degree is None else (w.sh_degree + 1) ** 2
    pixels = w.pixels
    if name == "gs_composite_forward":
        flop = TEST_FLOP["forward"] * counts.get("forward_tests", 0) + \
            ACCEPT_FLOP[w.method] * counts.get("forward_accepts", 0)
        return dict(bound="fp32", unit="TFLOP/s", work=flop,
                    basis=f"{TEST_FLOP['forward']} flop/test x tests + {ACCEPT_FLOP[w.method]} "
                          "flop/accept x accepts (kernel counters; constants = executed FP32 "
                          "flops per event, ncu-fitted)")
    if name == "gs_composite_backward":
        normals = bool(w.depth_normal_loss)   # a normal-map gradient: the kernel keeps its fields
        masked = counts.get("masked_intersections", 0) > 0   # warp accept masks were used
        per_test = TEST_FLOP["backward_masked" if masked and not normals else
                             "backward_normals" if normals else "backward"]
        per_accept = (BACKWARD_ACCEPT_FLOP_NORMALS if normals else BACKWARD_ACCEPT_FLOP)[w.method]
        flop = per_test * counts.get("backward_tests", 0) + \
            per_accept * counts.get("backward_accepts", 0)
        return dict(bound="fp32", unit="TFLOP/s", work=flop,
                    basis=f"{per_test} flop/test x tests + {per_accept} flop/accept x accepts "
                          "(kernel counters; constants = executed FP32 flops per event, "
                          "ncu-fitted)")
    if name == "gs_bin_sort":
        # per record: the span writer reads the fields its region uses (T, xy, opacity:
        # 48 B), radius, depth order and span offset (16 B); per row span: 12 B written
        # (row key + packed span), sorted by row over 2 passes of 12 B read + written,
        # read by the count and write kernels (8 B each); per intersection the 4-byte
        # point-list entry
        Sp = counts.get("spans", 0)
        return dict(bound="hbm", unit="GB/s", work=R * 64 + Sp * (12 + 48 + 16) + I * 4,
                    basis="64 B per record + 76 B per row span + 4 B per intersection")
    if name == "gs_bin_count":
        # depth keys 8 B written/record; 32-bit key-value depth sort, 4 passes of 16 B +
        # 4 B histogram read; tile counting reads the record fields its region uses and
        # the radius (52 B) and writes tile and span counts (16 B); two scans 32 B
        return dict(bound="hbm", unit="GB/s", work=R * (8 + 4 * 16 + 4 + 52 + 16 + 32),
                    basis="176 B per record (keys, 4-pass depth sort, region fields, counts, scans)")
    surfel_in = 4 * (3 + 4 + 2 + 1 + (2 * K * 3 + 12 if K else 0))
    if name == "gs_project_forward":
        pair_out = 4 * (20 + 2 + 1 + (20 if K else 0))
        return dict(bound="hbm", unit="GB/s", work=S * N * surfel_in + S * C * N * pair_out,
                    basis=f"{surfel_in} B per surfel read + {pair_out} B per pair written")
    if name == "gs_project_backward":
        pair_in = 4 * (20 + 2 + (20 if K else 0))
        return dict(bound="hbm", unit="GB/s",
                    work=S * N * 2 * surfel_in + S * C * N * pair_in,
                    basis=f"{pair_in} B per pair read + surfel inputs read and grads written")
    return dict(bound="hbm", unit="GB/s", work=pixels * 4, basis="unmodelled")
