"""Ragged scene batches (row "next" 3): scenes with different surfel counts in one
call equal each scene rendered on its own."""

import pytest
import torch

from diff_gabor_splatting_b200 import rasterize_gabors, rasterize_neural_gabors
from diff_gabor_splatting_b200.ragged import (rasterize_gabors_ragged,
                                              rasterize_neural_gabors_ragged)
from helpers import appearance_names, assert_grads_close, ordered, random_scene

pytestmark = pytest.mark.gpu

W, H = 70, 45
PER_SURFEL = ("means", "quaternions", "scales", "opacities")


@pytest.mark.parametrize("method,sh_degree", [("classic", None), ("classic", 2), ("neural", None)])
def test_ragged_batch_equals_scenes_alone(method, sh_degree):
    counts = [150, 0, 400, 275]
    scenes = [ordered(random_scene(method, scenes=1, cameras=2, n=max(n, 1), width=W, height=H,
                                   sh_degree=sh_degree, conditioned=True), method)
              for n in counts]
    per_surfel = list(PER_SURFEL) + appearance_names(method)
    fn = rasterize_gabors if method == "classic" else rasterize_neural_gabors
    ragged_fn = rasterize_gabors_ragged if method == "classic" else rasterize_neural_gabors_ragged
    kw = dict(width=W, height=H)
    if method == "classic":
        kw["sh_degree"] = sh_degree
    # ragged inputs: per-surfel tensors concatenated, cameras stacked
    flat = {}
    for name in scenes[0]:
        if name in per_surfel:
            flat[name] = torch.cat([s[name][0, :n] for s, n in zip(scenes, counts)]).contiguous()
        else:
            flat[name] = torch.cat([s[name] for s in scenes]).contiguous()
    flat = {k: t.clone().requires_grad_() for k, t in flat.items()}
    rgb, alpha, meta = ragged_fn(**flat, **kw, counts=counts, median_depth=True)
    assert rgb.shape == (4, 2, H, W, 3)
    weights = torch.linspace(0.2, 1.0, rgb.numel(), device="cuda").reshape(rgb.shape)
    ((rgb * weights).sum() + meta["distortion"].sum() + meta["median_depth"].sum()).backward()
    offset = 0
    for i, (s, n) in enumerate(zip(scenes, counts)):
        mine = {k: (t[:, :n] if k in per_surfel else t).clone().requires_grad_()
                for k, t in s.items()}
        e_rgb, e_alpha, e_meta = fn(**mine, **kw, median_depth=True)
        assert torch.equal(rgb[i], e_rgb[0]), i
        assert torch.equal(alpha[i], e_alpha[0]), i
        for key in ("accumulated_depth", "normals", "distortion", "median_depth"):
            assert torch.equal(meta[key][i], e_meta[key][0]), (i, key)
        ((e_rgb * weights[i:i + 1]).sum() + e_meta["distortion"].sum()
         + e_meta["median_depth"].sum()).backward()
        for name, t in mine.items():
            got = flat[name].grad[offset:offset + n] if name in per_surfel else flat[name].grad[i:i + 1]
            if t.grad is None or got.numel() == 0:
                continue
            expected = t.grad[0] if name in per_surfel else t.grad
            assert_grads_close(got, expected, f"scene {i} {name}", elementwise=1e-4)
        offset += n
    # flat pair metadata: C * sum(N) pairs in scene, camera, surfel order
    assert meta["radii"].shape == (2 * sum(counts),)
    assert torch.equal(meta["scene_ids"][:300], torch.zeros(300, dtype=torch.int64, device="cuda"))
    assert int(meta["camera_ids"][150]) == 1 and int(meta["primitive_ids"][151]) == 1
