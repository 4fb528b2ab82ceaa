"""Generate the committed golden fixtures from the reference's own Python code.

Run in the build container (it needs the reference source tree; the GPU box never
runs this):

    python tests/golden/make_golden.py [/path/to/reference]

The reference is luisrodolfo10/diff_gabor_splatting v0.1.1.  Everything it is asked
to compute here is pure PyTorch and runs on the CPU:

* ``gabor_splatting.rendering.project_surfaces`` / ``quaternion_matrix``
  (src/gabor_splatting/rendering.py:156-218) on seeded inputs, including the
  culling edge cases (behind the camera, beyond the far plane, edge-on, degenerate
  conic, off-screen);
* ``gabor_splatting.rendering.check_values`` (rendering.py:88-153): the exact
  ValueError message for each invalid input;
* the float64 test oracle ``reference`` of tests/test_rendering.py:64-171 (images and,
  by autograd, every input gradient) on the workloads of that test file's cases;
* the SH polynomial oracle ``evaluate_sh_reference`` of
  tests/test_spherical_harmonics.py:10-69 (values and gradients, degrees 0-3).

The test oracle hard-codes ``device="cuda"``; its source is loaded with that one
string replaced by ``"cpu"`` (no other change).  The native extension is not
needed: if it is not importable, a stub module stands in for it, because none of
the functions above call it.
"""

from __future__ import annotations

import importlib
import inspect
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def import_reference(root: Path):
    """Import the reference package and its two test modules from ``root``."""
    sys.path.insert(0, str(root / "src"))
    try:
        importlib.import_module("gabor_splatting._C")
    except ImportError:
        sys.modules["gabor_splatting._C"] = types.ModuleType("gabor_splatting._C")
    rendering = importlib.import_module("gabor_splatting.rendering")
    sys.path.insert(0, str(root / "tests"))
    test_rendering = importlib.import_module("test_rendering")
    test_sh = importlib.import_module("test_spherical_harmonics")
    source = inspect.getsource(test_rendering.reference).replace('device="cuda"', 'device="cpu"')
    namespace = {"torch": torch}
    exec(compile(source, "reference_cpu", "exec"), namespace)
    return rendering, namespace["reference"], test_sh.evaluate_sh_reference


def small_inputs(method, scenes=1, cameras=2, primitives=3, seed=7):
    """The deterministic overlapping-surface workload of the reference tests, on CPU.

    Same structure and constants as tests/test_rendering.py:11-48 (one 9x9 tile,
    depths increasing with the primitive index); random draws use a CPU generator.
    """
    g = torch.Generator().manual_seed(seed)
    means = torch.randn(scenes, primitives, 3, generator=g) * 0.08
    means[..., 2] = torch.linspace(2.4, 3.5, primitives)
    quats = torch.tensor([1.0, 0.08, -0.05, 0.02])
    quats = (quats / quats.norm()).expand(scenes, primitives, 4).clone()
    views = torch.eye(4).expand(scenes, cameras, 4, 4).clone()
    views[..., 0, 3] = torch.linspace(-0.03, 0.04, cameras)
    K = torch.tensor([[16.0, 0.0, 4.0], [0.0, 17.0, 4.0], [0.0, 0.0, 1.0]])
    v = dict(
        means=means, quaternions=quats,
        scales=torch.full((scenes, primitives, 2), 0.37),
        opacities=torch.full((scenes, primitives), 0.32),
        view_matrices=views, intrinsics=K.expand(scenes, cameras, 3, 3).clone(),
        backgrounds=torch.full((scenes, cameras, 3), 0.13),
    )
    if method == "classic":
        v.update(
            colors=torch.rand(scenes, primitives, 3, generator=g),
            secondary_colors=torch.rand(scenes, primitives, 3, generator=g),
            frequency_weights=torch.full((scenes, primitives, 4), 0.25),
            frequency_magnitudes=torch.full((scenes, primitives, 4), 0.4),
            phases=torch.rand(scenes, primitives, 4, generator=g),
        )
    else:
        for name, shape in [("input_weights", (6, 5)), ("input_biases", (6,)),
                            ("output_weights", (3, 6)), ("output_biases", (3,))]:
            v[name] = torch.randn(scenes, primitives, *shape, generator=g) * 0.08
    return v


def render_cases():
    """The image/gradient cases of tests/test_rendering.py restated as workloads."""
    cases = []
    for method in ("classic", "neural"):
        cases.append((f"{method}_basic", method, small_inputs(method), "weighted"))
        v = small_inputs(method, cameras=1, primitives=65)
        v["opacities"].fill_(0.03)
        cases.append((f"{method}_batch65", method, v, "weighted"))
        for opacity in (0.0, 1.0):
            v = small_inputs(method, cameras=1, primitives=7)
            v["opacities"].fill_(0.85 if opacity == 1.0 else opacity)
            v["opacities"][..., 0] = opacity
            v["quaternions"].zero_()
            v["quaternions"][..., 0] = 1
            v["means"][..., :2] = 0
            cases.append((f"{method}_opacity{int(opacity)}", method, v, "sum"))
        v = small_inputs(method, cameras=1, primitives=1)
        v["scales"].fill_(0.02)
        v["quaternions"].zero_()
        v["quaternions"][..., 0] = 1
        cases.append((f"{method}_tiny", method, v, "sum"))
        cases.append((f"{method}_scenes2", method,
                      small_inputs(method, scenes=2, cameras=3), "weighted"))
    return cases


def projection_inputs(seed=0, n=96, cameras=3):
    """Seeded config-0-style surfels plus hand-made culling edge cases."""
    g = torch.Generator().manual_seed(seed)
    means = torch.empty(1, n, 3)
    means[..., :2] = torch.rand(1, n, 2, generator=g) * 2 - 1
    means[..., 2] = torch.rand(1, n, generator=g) * 2 + 2
    quats = torch.randn(1, n, 4, generator=g)
    quats = quats / quats.norm(dim=-1, keepdim=True)
    scales = torch.exp(torch.empty(1, n, 2).uniform_(np.log(0.02), np.log(0.2), generator=g))
    # edge cases in the last rows
    means[0, -1] = torch.tensor([0.0, 0.0, -2.0])       # behind the camera
    means[0, -2] = torch.tensor([0.0, 0.0, 150.0])      # beyond the far plane
    means[0, -3] = torch.tensor([50.0, 0.0, 2.0])       # far off screen
    means[0, -4] = torch.tensor([0.0, 0.0, 3.0])        # edge-on (normal _|_ view ray)
    quats[0, -4] = torch.tensor([0.5, 0.5, 0.5, 0.5])
    means[0, -5] = torch.tensor([0.1, 0.0, 3.0])        # degenerate conic (rendering.py:191)
    quats[0, -5] = torch.tensor([0.5, 0.5, 0.5, 0.5])
    scales[0, -5] = 1.0
    views = torch.eye(4).expand(1, cameras, 4, 4).clone()
    views[0, 1, 0, 3] = 0.3
    angle = torch.tensor(0.4)
    views[0, 2, 0, 0], views[0, 2, 0, 2] = torch.cos(angle), torch.sin(angle)
    views[0, 2, 2, 0], views[0, 2, 2, 2] = -torch.sin(angle), torch.cos(angle)
    views[0, 2, 1, 3] = -0.2
    K = torch.tensor([[80.0, 0.0, 32.0], [0.0, 80.0, 32.0], [0.0, 0.0, 1.0]])
    K = K.expand(1, cameras, 3, 3).clone()
    K[0, 2, 0, 1] = 1.5                                  # skew is allowed
    return means, quats, scales, views, K


def main():
    # the reference checkout: argument, else $GS_REFERENCE_DIR, else a checkout named
    # `reference` beside this repository
    default = os.environ.get("GS_REFERENCE_DIR",
                             Path(__file__).resolve().parents[3] / "reference")
    root = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(default)
    rendering, reference_render, evaluate_sh_reference = import_reference(root)
    torch.set_grad_enabled(True)
    out = {}

    # projection (rendering.py:156-218)
    means, quats, scales, views, K = projection_inputs()
    T, xy, normals, dirs, radii = rendering.project_surfaces(
        means, quats, scales, views, K, 64, 64, 0.2, 100.0)
    for name, value in dict(means=means, quaternions=quats, scales=scales,
                            view_matrices=views, intrinsics=K, transform=T, xy=xy,
                            normals=normals, directions=dirs, radii=radii,
                            rotation=rendering.quaternion_matrix(quats)).items():
        out[f"projection/{name}"] = value.detach().numpy()
    np.savez_compressed(HERE / "projection.npz", **{k.split("/")[1]: v for k, v in out.items()})

    # check_values messages (rendering.py:88-153)
    messages = {}
    base = small_inputs("classic")
    invalid = {
        "nonfinite_means": ("means", lambda v: v.__setitem__((0, 0, 0), float("nan"))),
        "negative_scales": ("scales", lambda v: v.neg_()),
        "zero_quaternions": ("quaternions", lambda v: v.zero_()),
        "opacity_two": ("opacities", lambda v: v.fill_(2.0)),
        "transposed_intrinsics": ("intrinsics", lambda v: v.copy_(v.transpose(-1, -2).clone())),
        "view_last_row": ("view_matrices", lambda v: v.__setitem__((0, 0, 3, 0), 0.5)),
        "view_scaled": ("view_matrices", lambda v: v[..., :3, :3].mul_(1.1)),
        "view_reflection": ("view_matrices", lambda v: v[..., 0, :3].neg_()),
        "negative_focal": ("intrinsics", lambda v: v[..., 0, 0].neg_()),
        "weights_sum": ("frequency_weights", lambda v: v.fill_(0.3)),
        "negative_weights": ("frequency_weights", lambda v: v.__setitem__((0, 0, 0), -0.25)),
        "negative_magnitudes": ("frequency_magnitudes", lambda v: v.neg_()),
    }
    names = ["colors", "secondary_colors", "frequency_weights", "frequency_magnitudes", "phases"]
    for case, (name, mutate) in invalid.items():
        v = {k: t.clone() for k, t in base.items()}
        mutate(v[name])
        tensors = {k: (t, None) for k, t in v.items()}
        try:
            rendering.check_values(tensors, v["quaternions"], v["scales"], v["opacities"],
                                   v["view_matrices"], v["intrinsics"],
                                   [v[k] for k in names], False)
            messages[case] = ""
        except ValueError as error:
            messages[case] = str(error)
    np.savez_compressed(HERE / "check_values.npz",
                        cases=np.array(list(messages)), messages=np.array(list(messages.values())))

    # float64 test oracle images and gradients (tests/test_rendering.py:64-171)
    render = {}
    for case, method, values, loss in render_cases():
        leaves = {k: t.double().requires_grad_() for k, t in values.items()}
        expected = reference_render(method, leaves)
        if loss == "weighted":
            weights = torch.linspace(-0.4, 0.7, expected.numel(), dtype=torch.float64)
            objective = (expected * weights.reshape(expected.shape)).sum()
        else:
            objective = expected.sum()
        grads = torch.autograd.grad(objective, tuple(leaves.values()))
        render[f"{case}/method"] = np.array(method)
        render[f"{case}/loss"] = np.array(loss)
        render[f"{case}/maps"] = expected.detach().numpy()
        for (name, value), grad in zip(values.items(), grads):
            render[f"{case}/in/{name}"] = value.numpy()
            render[f"{case}/grad/{name}"] = grad.numpy()
    np.savez_compressed(HERE / "render.npz", **render)

    # SH polynomial oracle (tests/test_spherical_harmonics.py:10-95)
    sh = {}
    g = torch.Generator().manual_seed(31)
    for degree in range(4):
        for cameras in (1, 3):
            first = torch.randn(2, 7, (degree + 1) ** 2, 3, generator=g, dtype=torch.float64)
            second = torch.randn(first.shape, generator=g, dtype=torch.float64)
            d = torch.randn(2, cameras, 7, 3, generator=g, dtype=torch.float64)
            d = d / d.norm(dim=-1, keepdim=True)
            w = torch.randn(2, cameras, 7, 6, generator=g, dtype=torch.float64)
            f_, s_, d_ = (t.clone().requires_grad_() for t in (first, second, d))
            expected = torch.cat([evaluate_sh_reference(degree, c[:, None], d_).expand(
                2, cameras, 7, 3) for c in (f_, s_)], -1)
            grads = torch.autograd.grad((expected * w).sum() + d_.sum() * 0, (f_, s_, d_))
            key = f"d{degree}c{cameras}"
            sh.update({f"{key}/first": first.numpy(), f"{key}/second": second.numpy(),
                       f"{key}/directions": d.numpy(), f"{key}/weights": w.numpy(),
                       f"{key}/colors": expected.detach().numpy(),
                       f"{key}/grad_first": grads[0].numpy(),
                       f"{key}/grad_second": grads[1].numpy(),
                       f"{key}/grad_directions": grads[2].numpy()})
    np.savez_compressed(HERE / "sh.npz", **sh)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
