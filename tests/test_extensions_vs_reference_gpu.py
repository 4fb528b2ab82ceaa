"""The additions outside the reference's release, pinned to the reference itself.

The reference has no ragged scene batches and no selected-pixel rendering
(README.md:267-270 lists both outside its release), but it renders each scene on its
own and renders full images, so both additions are checked against those:

* ragged batches: each scene of one ragged call equals the reference rendering that
  scene alone, images and input gradients;
* selected pixels: the listed pixels equal the same pixels of the reference's full
  render, and the gradients of a loss on them equal the reference's gradients of the
  same loss written on its full images.

"Alone" means as the reference computes a batch: for one small scene PyTorch's einsum
inside the reference's projection switches to separately rounded products and its
images then depend on the batch shape (tests/test_reference_ext_gpu.py,
test_reference_varies_with_batch_shape); the reference renders each scene here as
scene 0 of a batch of two copies, which is the rounding this build follows.

With exact appearance and square bins every value must be bit-identical; gradients
within 1e-4 of their scale (float atomics sum in an unspecified order on both sides).
"""

import pytest
import torch

from diff_gabor_splatting_b200 import rasterize_gabors, rasterize_neural_gabors, rendering
from diff_gabor_splatting_b200.ragged import (rasterize_gabors_ragged,
                                              rasterize_neural_gabors_ragged)
from helpers import appearance_names, assert_grads_close, maps_from_result, ordered, random_scene
from oracle import reference as reference_loader

try:
    ref = reference_loader.load()
except ImportError:   # pragma: no cover - depends on the build container
    ref = None

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(ref is None, reason="compiled reference not in oracle/_ref")]

W, H = 70, 45
PER_SURFEL = ("means", "quaternions", "scales", "opacities")


@pytest.fixture(autouse=True)
def reference_modes(monkeypatch):
    monkeypatch.setattr(rendering, "EXACT_APPEARANCE", True)
    monkeypatch.setattr(rendering, "TIGHT_BINNING", False)


def reference_alone(method, values, kw, weights):
    """The reference's images and input gradients of one scene ([1, ...] inputs),
    rendered as scene 0 of a batch of two copies; the loss sees scene 0 only."""
    fn = ref.rasterize_gabors if method == "classic" else ref.rasterize_neural_gabors
    leaves = {k: t.detach().clone().requires_grad_() for k, t in values.items()}
    two = {k: torch.cat([t, t.detach()], 0) for k, t in leaves.items()}
    maps = maps_from_result(fn(**two, **kw))[:1]
    (maps * weights).sum().backward()
    return maps.detach(), {k: t.grad for k, t in leaves.items()}


@pytest.mark.parametrize("method,sh_degree",
                         [("classic", None), ("classic", 2), ("classic", 3), ("neural", None)])
def test_ragged_batch_equals_reference_per_scene(method, sh_degree):
    counts = [150, 0, 400, 275]
    scenes = [ordered(random_scene(method, scenes=1, cameras=2, n=max(n, 1), width=W, height=H,
                                   sh_degree=sh_degree, conditioned=True, seed=i), method)
              for i, n in enumerate(counts)]
    per_surfel = list(PER_SURFEL) + appearance_names(method)
    ragged_fn = rasterize_gabors_ragged if method == "classic" else rasterize_neural_gabors_ragged
    kw = dict(width=W, height=H)
    if method == "classic":
        kw["sh_degree"] = sh_degree
    flat = {}
    for name in scenes[0]:
        if name in per_surfel:
            flat[name] = torch.cat([s[name][0, :n] for s, n in zip(scenes, counts)]).contiguous()
        else:
            flat[name] = torch.cat([s[name] for s in scenes]).contiguous()
    flat = {k: t.clone().requires_grad_() for k, t in flat.items()}
    maps = maps_from_result(ragged_fn(**flat, **kw, counts=counts))
    weights = torch.linspace(-0.3, 0.8, maps.numel(), device="cuda").reshape(maps.shape)
    (maps * weights).sum().backward()
    offset = 0
    for i, (s, n) in enumerate(zip(scenes, counts)):
        alone = {k: (t[:, :n] if k in per_surfel else t).contiguous() for k, t in s.items()}
        e_maps, e_grads = reference_alone(method, alone, kw, weights[i:i + 1])
        assert torch.equal(maps[i:i + 1].detach(), e_maps), f"scene {i}: images differ"
        for name, expected in e_grads.items():
            got = (flat[name].grad[offset:offset + n][None] if name in per_surfel
                   else flat[name].grad[i:i + 1])
            if expected is None or got.numel() == 0:
                continue
            assert_grads_close(got, expected, f"scene {i} {name}", elementwise=1e-4)
        offset += n


@pytest.mark.parametrize("method", ["classic", "neural"])
def test_selected_pixels_equal_reference_full_render(method):
    Wd, Hd, P = 70, 45, 600
    v = ordered(random_scene(method, scenes=2, cameras=2, n=300, width=Wd, height=Hd,
                             conditioned=True), method)
    fn = rasterize_gabors if method == "classic" else rasterize_neural_gabors
    ref_fn = ref.rasterize_gabors if method == "classic" else ref.rasterize_neural_gabors
    g = torch.Generator(device="cuda").manual_seed(9)
    xs = torch.randint(0, Wd, (2, 2, P), device="cuda", generator=g)
    ys = torch.randint(0, Hd, (2, 2, P), device="cuda", generator=g)
    xs[..., :20] = xs[..., 20:40]   # duplicated pixels
    ys[..., :20] = ys[..., 20:40]
    pixels = torch.stack((xs, ys), -1).to(torch.int32)
    weights = torch.rand((2, 2, P, 9), device="cuda", generator=g) - 0.3

    sel = {k: t.clone().requires_grad_() for k, t in v.items()}
    maps = maps_from_result(fn(**sel, width=Wd, height=Hd, pixels=pixels))
    assert maps.shape == (2, 2, P, 9)
    full = {k: t.clone().requires_grad_() for k, t in v.items()}
    f_maps = maps_from_result(ref_fn(**full, width=Wd, height=Hd))
    s, c = torch.meshgrid(torch.arange(2, device="cuda"), torch.arange(2, device="cuda"),
                          indexing="ij")
    index = (s[..., None].expand_as(xs), c[..., None].expand_as(xs), ys.long(), xs.long())
    assert torch.equal(maps.detach(), f_maps.detach()[index])
    (maps * weights).sum().backward()
    dense = torch.zeros_like(f_maps)
    dense.index_put_(index, weights, accumulate=True)   # the same loss on the full images
    (f_maps * dense).sum().backward()
    for name in sel:
        assert_grads_close(sel[name].grad, full[name].grad, name, elementwise=1e-4)
