"""Seeded synthetic scenes with the shapes and distributions of the benchmark configs.

Config numbering follows the benchmark's list (0-4).  No dataset is involved (the
reference's own benchmark is synthetic too); every tensor is drawn from a
``torch.Generator`` seeded per (config, seed) on the host, so the same call always
yields the same scene.

    0  classic, 1 scene, N=1024, one 64x64 camera (identity view, f=80, c=32), SH 0
    1  classic, SH degree 3, N=500k, 4 cameras 1920x1080 on a radius-5 ring, f=1100
    2  neural, N=200k, one 1280x720 camera (ring angle 0), f=900, packed
    3  classic, SH degree 1, 32 scenes x 8 cameras, N=50k, 256x256, radius-4 sphere,
       f=220, packed
    4  classic, SH degree 3, 8 scenes x 16 cameras, N=2M, 1024x1024, radius-5 sphere,
       f=900; depth and normals also feed the loss
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass
class Workload:
    config: int
    method: str
    scenes: int
    cameras: int
    surfels: int
    width: int
    height: int
    sh_degree: int | None
    packed: bool
    depth_normal_loss: bool
    inputs: dict = field(default_factory=dict)   # host tensors, public-API names

    @property
    def pixels(self) -> int:
        return self.scenes * self.cameras * self.width * self.height

    def kwargs(self) -> dict:
        out = dict(width=self.width, height=self.height, packed=self.packed)
        if self.method == "classic":
            out["sh_degree"] = self.sh_degree
        return out


CONFIGS = {
    0: dict(method="classic", scenes=1, cameras=1, surfels=1024, width=64, height=64,
            sh_degree=0, packed=False, focal=80.0, rig="identity", loss_extra=False),
    1: dict(method="classic", scenes=1, cameras=4, surfels=500_000, width=1920, height=1080,
            sh_degree=3, packed=False, focal=1100.0, rig="ring5", loss_extra=False),
    2: dict(method="neural", scenes=1, cameras=1, surfels=200_000, width=1280, height=720,
            sh_degree=None, packed=True, focal=900.0, rig="ring5", loss_extra=False),
    3: dict(method="classic", scenes=32, cameras=8, surfels=50_000, width=256, height=256,
            sh_degree=1, packed=True, focal=220.0, rig="sphere4", loss_extra=False),
    4: dict(method="classic", scenes=8, cameras=16, surfels=2_000_000, width=1024, height=1024,
            sh_degree=3, packed=False, focal=900.0, rig="sphere5", loss_extra=True),
}


def look_at(eye: torch.Tensor) -> torch.Tensor:
    """World-to-camera [4,4] looking at the origin: +x right, +y down, +z forward."""
    f = -eye / eye.norm()
    up = torch.tensor([0.0, 0.0, 1.0], dtype=torch.float64)
    if abs(float(f @ up)) > 0.99:
        up = torch.tensor([0.0, 1.0, 0.0], dtype=torch.float64)
    x = torch.linalg.cross(f, up)
    x = x / x.norm()
    y = torch.linalg.cross(f, x)
    R = torch.stack((x, y, f))
    V = torch.eye(4, dtype=torch.float64)
    V[:3, :3] = R
    V[:3, 3] = -R @ eye
    return V


def camera_rig(rig: str, count: int, width: int, height: int, focal: float,
               g: torch.Generator):
    """View matrices [count,4,4] and intrinsics [count,3,3] (float32)."""
    if rig == "identity":
        views = torch.eye(4, dtype=torch.float64).expand(count, 4, 4).clone()
        K = torch.tensor([[focal, 0, 32.0], [0, focal, 32.0], [0, 0, 1]], dtype=torch.float64)
        return views.float(), K.expand(count, 3, 3).clone().float()
    if rig == "ring5":
        angles = [2 * math.pi * i / 4 for i in range(count)]
        eyes = [torch.tensor([5 * math.cos(a), 5 * math.sin(a), 0.0], dtype=torch.float64)
                for a in angles]
    else:
        radius = 4.0 if rig == "sphere4" else 5.0
        d = torch.randn(count, 3, generator=g, dtype=torch.float64)
        d = d / d.norm(dim=-1, keepdim=True)
        eyes = list(radius * d)
    views = torch.stack([look_at(e) for e in eyes]).float()
    K = torch.tensor([[focal, 0, (width - 1) / 2], [0, focal, (height - 1) / 2], [0, 0, 1]])
    return views, K.expand(count, 3, 3).clone().float()


def make_workload(config: int, seed: int = 0, surfels: int | None = None,
                  scenes: int | None = None, cameras: int | None = None) -> Workload:
    """Build config ``config`` on the host (optionally fewer surfels/scenes/cameras)."""
    c = dict(CONFIGS[config])
    S = scenes or c["scenes"]
    N = surfels or c["surfels"]
    C = cameras or c["cameras"]
    g = torch.Generator().manual_seed(seed * 1000 + config)
    if config == 0:
        means = torch.empty(S, N, 3)
        means[..., :2] = torch.rand(S, N, 2, generator=g) * 2 - 1
        means[..., 2] = torch.rand(S, N, generator=g) * 2 + 2
    else:
        means = torch.randn(S, N, 3, generator=g) * 1.5
        norm = means.norm(dim=-1, keepdim=True)
        means = torch.where(norm > 3, means * (3 / norm), means)
    quats = torch.randn(S, N, 4, generator=g)
    quats = quats / quats.norm(dim=-1, keepdim=True)
    scales = torch.exp(torch.empty(S, N, 2).uniform_(math.log(0.02), math.log(0.2), generator=g))
    opacities = torch.rand(S, N, generator=g) * 0.8 + 0.1
    inputs = dict(means=means, quaternions=quats, scales=scales, opacities=opacities)
    if c["method"] == "classic":
        deg = c["sh_degree"]
        if deg is None:
            inputs["colors"] = torch.rand(S, N, 3, generator=g)
            inputs["secondary_colors"] = torch.rand(S, N, 3, generator=g)
        else:
            k = (deg + 1) ** 2
            for name in ("colors", "secondary_colors"):
                coeffs = torch.randn(S, N, k, 3, generator=g) * 0.3
                coeffs[..., 0, :] = torch.rand(S, N, 3, generator=g)
                inputs[name] = coeffs
        w = torch.rand(S, N, 4, generator=g)
        inputs["frequency_weights"] = w / w.sum(-1, keepdim=True)
        inputs["frequency_magnitudes"] = torch.rand(S, N, 4, generator=g) * 7.5 + 0.5
        inputs["phases"] = torch.rand(S, N, 4, generator=g) * (2 * math.pi)
    else:
        inputs["input_weights"] = (torch.rand(S, N, 6, 5, generator=g) * 2 - 1) / 5
        inputs["input_biases"] = torch.zeros(S, N, 6)
        inputs["output_weights"] = (torch.rand(S, N, 3, 6, generator=g) * 2 - 1) / 30
        inputs["output_biases"] = torch.zeros(S, N, 3)
    views, Ks = [], []
    for _ in range(S):
        v, k = camera_rig(c["rig"], C, c["width"], c["height"], c["focal"], g)
        views.append(v)
        Ks.append(k)
    inputs["view_matrices"] = torch.stack(views)
    inputs["intrinsics"] = torch.stack(Ks)
    inputs["backgrounds"] = torch.zeros(S, C, 3)
    inputs = {k: v.contiguous() for k, v in inputs.items()}
    return Workload(config=config, method=c["method"], scenes=S, cameras=C, surfels=N,
                    width=c["width"], height=c["height"], sh_degree=c["sh_degree"],
                    packed=c["packed"], depth_normal_loss=c["loss_extra"], inputs=inputs)


def loss_of(rgb, alpha, meta, depth_normal: bool):
    """rgb.mean() + alpha.mean() + 0.01 distortion.mean() (+ depth.mean() + normals.mean())."""
    loss = rgb.mean() + alpha.mean() + 0.01 * meta["distortion"].mean()
    if depth_normal:
        loss = loss + meta["accumulated_depth"].mean() + meta["normals"].mean()
    return loss


def crop(w: Workload, x0: int, y0: int, width: int, height: int,
         camera_ids=None, scene_ids=None) -> Workload:
    """The same scenes seen through a pixel window of some cameras.

    Shifting the principal point by (-x0, -y0) makes pixel (x, y) of the crop
    the pixel (x0 + x, y0 + y) of the full image: the same rays, so the same values.
    Used to time the CPU oracle on a bounded sample of a large workload.
    """
    cams = list(range(w.cameras)) if camera_ids is None else list(camera_ids)
    scenes = list(range(w.scenes)) if scene_ids is None else list(scene_ids)
    inputs = {k: v[scenes].contiguous() for k, v in w.inputs.items()}
    views = inputs["view_matrices"][:, cams].clone()
    K = inputs["intrinsics"][:, cams].clone()
    K[..., 0, 2] -= x0
    K[..., 1, 2] -= y0
    inputs["view_matrices"], inputs["intrinsics"] = views.contiguous(), K.contiguous()
    inputs["backgrounds"] = inputs["backgrounds"][:, cams].contiguous()
    return Workload(config=w.config, method=w.method, scenes=len(scenes), cameras=len(cams),
                    surfels=w.surfels, width=width, height=height, sh_degree=w.sh_degree,
                    packed=w.packed, depth_normal_loss=w.depth_normal_loss, inputs=inputs)
