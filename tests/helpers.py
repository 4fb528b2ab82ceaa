"""Shared inputs and comparisons for the test suite."""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
CLASSIC_APPEARANCE = ["colors", "secondary_colors", "frequency_weights", "frequency_magnitudes",
                      "phases"]
NEURAL_APPEARANCE = ["input_weights", "input_biases", "output_weights", "output_biases"]


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / name) as data:
        return {k: data[k] for k in data.files}


def golden_cases():
    """Render cases of golden/render.npz: name -> (method, loss, inputs, maps, grads)."""
    g = load_golden("render.npz")
    cases = {}
    for key in sorted({k.split("/")[0] for k in g}):
        inputs = {k.split("/")[2]: g[k] for k in g if k.startswith(f"{key}/in/")}
        grads = {k.split("/")[2]: g[k] for k in g if k.startswith(f"{key}/grad/")}
        cases[key] = (str(g[f"{key}/method"]), str(g[f"{key}/loss"]), inputs,
                      g[f"{key}/maps"], grads)
    return cases


def small_inputs(method, scenes=1, cameras=2, primitives=3, seed=7, device="cuda"):
    """The overlapping-surface workload of the reference tests (one 9x9 tile)."""
    g = torch.Generator().manual_seed(seed)
    means = torch.randn(scenes, primitives, 3, generator=g) * 0.08
    means[..., 2] = torch.linspace(2.4, 3.5, primitives)
    quats = torch.tensor([1.0, 0.08, -0.05, 0.02])
    quats = (quats / quats.norm()).expand(scenes, primitives, 4).clone()
    views = torch.eye(4).expand(scenes, cameras, 4, 4).clone()
    views[..., 0, 3] = torch.linspace(-0.03, 0.04, cameras)
    K = torch.tensor([[16.0, 0.0, 4.0], [0.0, 17.0, 4.0], [0.0, 0.0, 1.0]])
    v = dict(means=means, quaternions=quats, scales=torch.full((scenes, primitives, 2), 0.37),
             opacities=torch.full((scenes, primitives), 0.32), view_matrices=views,
             intrinsics=K.expand(scenes, cameras, 3, 3).clone(),
             backgrounds=torch.full((scenes, cameras, 3), 0.13))
    if method == "classic":
        v.update(colors=torch.rand(scenes, primitives, 3, generator=g),
                 secondary_colors=torch.rand(scenes, primitives, 3, generator=g),
                 frequency_weights=torch.full((scenes, primitives, 4), 0.25),
                 frequency_magnitudes=torch.full((scenes, primitives, 4), 0.4),
                 phases=torch.rand(scenes, primitives, 4, generator=g))
    else:
        for name, shape in [("input_weights", (6, 5)), ("input_biases", (6,)),
                            ("output_weights", (3, 6)), ("output_biases", (3,))]:
            v[name] = torch.randn(scenes, primitives, *shape, generator=g) * 0.08
    return {k: t.to(device).requires_grad_() for k, t in v.items()}


def random_scene(method="classic", scenes=1, cameras=2, n=256, width=64, height=48, seed=0,
                 sh_degree=None, device="cuda", spread=1.0, focal=80.0, conditioned=False):
    """Seeded multi-tile scene in the style of the benchmark config 0 inputs.

    conditioned=True keeps surfaces within ~35 degrees of facing the camera and the
    Gabor magnitudes low (like the reference tests' workloads), so float32-vs-float64
    gradient comparisons are not dominated by near-grazing samples.
    """
    g = torch.Generator().manual_seed(seed)
    means = torch.empty(scenes, n, 3)
    means[..., :2] = (torch.rand(scenes, n, 2, generator=g) * 2 - 1) * spread
    means[..., 2] = torch.rand(scenes, n, generator=g) * 2 + 2
    quats = torch.randn(scenes, n, 4, generator=g)
    if conditioned:
        quats = quats * 0.15
        quats[..., 0] = 1.0
    quats = quats / quats.norm(dim=-1, keepdim=True)
    scales = torch.exp(torch.empty(scenes, n, 2).uniform_(math.log(0.02), math.log(0.2),
                                                            generator=g))
    views = torch.eye(4).expand(scenes, cameras, 4, 4).clone()
    for c in range(cameras):
        a = 0.15 * c
        views[:, c, 0, 0], views[:, c, 0, 2] = math.cos(a), math.sin(a)
        views[:, c, 2, 0], views[:, c, 2, 2] = -math.sin(a), math.cos(a)
        views[:, c, 0, 3] = 0.05 * c
    K = torch.tensor([[focal, 0.0, (width - 1) / 2], [0.0, focal, (height - 1) / 2],
                      [0.0, 0.0, 1.0]])
    v = dict(means=means, quaternions=quats, scales=scales,
             opacities=torch.rand(scenes, n, generator=g) * 0.8 + 0.1,
             view_matrices=views, intrinsics=K.expand(scenes, cameras, 3, 3).clone(),
             backgrounds=torch.rand(scenes, cameras, 3, generator=g))
    if method == "classic":
        if sh_degree is None:
            v["colors"] = torch.rand(scenes, n, 3, generator=g)
            v["secondary_colors"] = torch.rand(scenes, n, 3, generator=g)
        else:
            k = (sh_degree + 1) ** 2
            for name in ("colors", "secondary_colors"):
                c = torch.randn(scenes, n, k, 3, generator=g) * 0.3
                c[..., 0, :] = torch.rand(scenes, n, 3, generator=g)
                v[name] = c
        w = torch.rand(scenes, n, 4, generator=g)
        v["frequency_weights"] = w / w.sum(-1, keepdim=True)
        v["frequency_magnitudes"] = torch.rand(scenes, n, 4, generator=g) * (
            1.5 if conditioned else 7.5) + 0.5
        v["phases"] = torch.rand(scenes, n, 4, generator=g) * 2 * math.pi
    else:
        v["input_weights"] = (torch.rand(scenes, n, 6, 5, generator=g) * 2 - 1) / 5
        v["input_biases"] = torch.zeros(scenes, n, 6)
        v["output_weights"] = (torch.rand(scenes, n, 3, 6, generator=g) * 2 - 1) / 30
        v["output_biases"] = torch.zeros(scenes, n, 3)
    return {k: t.to(device).contiguous() for k, t in v.items()}


def maps_from_result(result):
    """Every differentiable output in one [..., 9] tensor (reference test helper)."""
    rgb, alpha, meta = result
    return torch.cat((rgb, alpha, meta["accumulated_depth"], meta["normals"],
                      meta["distortion"]), -1)


def appearance_names(method):
    return NEURAL_APPEARANCE if method == "neural" else CLASSIC_APPEARANCE


def ordered(values, method):
    """Input dict in the order of the public signature."""
    names = ["means", "quaternions", "scales", "opacities", *appearance_names(method),
             "view_matrices", "intrinsics", "backgrounds"]
    return {k: values[k] for k in names if k in values}


def assert_images_close(actual, expected, rtol, atol, max_bad_pixels=0.01, msg=""):
    """Image maps [..., H, W, 9] equal within tolerance except at a bounded fraction of
    pixels.

    Used against the CPU oracle: the kernels (like the reference's CUDA) round the
    ill-conditioned ray/plane intersection differently from plain CPU float32 (fused
    multiply-adds), which flips the alpha >= 1/255 acceptance or the T < 1e-4 stop
    for a few samples; each flip changes one pixel by up to one small contribution.
    """
    a = actual.detach().cpu().double()
    e = expected.detach().cpu().double()
    assert a.shape == e.shape, (a.shape, e.shape)
    bad = ((a - e).abs() > atol + rtol * e.abs()).reshape(-1, a.shape[-1]).any(-1)
    frac = bad.double().mean().item()
    assert frac <= max_bad_pixels, (
        f"{msg}: {frac:.3%} of pixels outside rtol={rtol} atol={atol} "
        f"(max abs diff {(a - e).abs().max().item():.3g})")
    return frac


def assert_grads_close(actual, expected, name, elementwise=2e-3, norm=None):
    """Gradient parity: every element within `elementwise` of the gradient's scale, and
    optionally the relative L2 error below `norm`."""
    a = actual.detach().cpu().double()
    e = expected.detach().cpu().double()
    scale = e.abs().max().item() + 1e-12
    err = (a - e).abs().max().item() / scale
    assert err <= elementwise, f"{name}: max error {err:.2e} of the gradient's scale"
    if norm is not None:
        rel = (a - e).norm().item() / (e.norm().item() + 1e-12)
        assert rel <= norm, f"{name}: relative L2 error {rel:.2e}"
