"""CPU: pin the oracle to the reference's own outputs (tests/golden/*.npz).

The fixtures were produced by running the reference's Python code on the CPU
(tests/golden/make_golden.py).  Tolerances: the projection is bit-exact; the render
oracle matches the reference's float64 test oracle to 1e-7 (that oracle builds its
rotation with a float32 identity matrix, so it carries ~1e-8 of float32 rounding).
"""

import numpy as np
import pytest
import torch

from helpers import appearance_names, golden_cases, load_golden
from oracle import gabor_oracle as O

GOLDEN = golden_cases()


def test_projection_bit_exact_with_reference():
    p = load_golden("projection.npz")
    T, xy, normals, dirs, radii = O.project_surfaces(
        *(torch.from_numpy(p[k]) for k in ("means", "quaternions", "scales", "view_matrices",
                                          "intrinsics")), 64, 64, 0.2, 100.0)
    np.testing.assert_array_equal(T.numpy(), p["transform"])
    np.testing.assert_array_equal(xy.numpy(), p["xy"])
    np.testing.assert_array_equal(normals.numpy(), p["normals"])
    np.testing.assert_array_equal(dirs.numpy(), p["directions"])
    np.testing.assert_array_equal(radii.numpy(), p["radii"])
    np.testing.assert_array_equal(O.quaternion_matrix(torch.from_numpy(p["quaternions"])).numpy(),
                                  p["rotation"])
    # the culling edge cases in the last five surfels are culled from the first camera
    assert (p["radii"][0, 0, -5:] == 0).all()


@pytest.mark.parametrize("case", sorted(GOLDEN))
def test_render_oracle_matches_reference_test_oracle(case):
    method, loss, inputs, maps, grads = GOLDEN[case]
    vals = {k: torch.from_numpy(v).double().requires_grad_() for k, v in inputs.items()}
    rgb, alpha, meta = O.render(vals["means"], vals["quaternions"], vals["scales"],
                                vals["opacities"], [vals[k] for k in appearance_names(method)],
                                vals["view_matrices"], vals["intrinsics"], 9, 9,
                                backgrounds=vals["backgrounds"], neural=method == "neural",
                                dtype=torch.float64)
    out = torch.cat((rgb, alpha, meta["accumulated_depth"], meta["normals"],
                     meta["distortion"]), -1)
    np.testing.assert_allclose(out.detach().numpy(), maps, atol=1e-7, rtol=1e-6)
    if loss == "weighted":
        w = torch.linspace(-0.4, 0.7, out.numel(), dtype=torch.float64).reshape(out.shape)
        objective = (out * w).sum()
    else:
        objective = out.sum()
    got = torch.autograd.grad(objective, tuple(vals.values()), allow_unused=True)
    for (name, value), g in zip(vals.items(), got):
        g = torch.zeros_like(value) if g is None else g
        scale = np.abs(grads[name]).max() + 1e-12
        assert np.abs(g.numpy() - grads[name]).max() <= 1e-6 * scale + 1e-9, name


@pytest.mark.parametrize("key", sorted({k.split("/")[0] for k in load_golden("sh.npz")}))
def test_sh_oracle_matches_reference_polynomials(key):
    g = load_golden("sh.npz")
    degree = int(key[1])
    first, second, dirs = (torch.from_numpy(g[f"{key}/{n}"]).requires_grad_()
                           for n in ("first", "second", "directions"))
    colors = O.evaluate_sh(first, second, dirs, degree)
    np.testing.assert_allclose(colors.detach().numpy(), g[f"{key}/colors"], rtol=1e-12, atol=1e-12)
    objective = (colors * torch.from_numpy(g[f"{key}/weights"])).sum() + dirs.sum() * 0
    grads = torch.autograd.grad(objective, (first, second, dirs))
    for name, a in zip(("grad_first", "grad_second", "grad_directions"), grads):
        np.testing.assert_allclose(a.numpy(), g[f"{key}/{name}"], rtol=1e-10, atol=1e-12)


def test_binning_matches_brute_force():
    """bin_tiles equals a per-tile scan of every record (ordered by depth, then index)."""
    gen = torch.Generator().manual_seed(5)
    Q, W, H, images = 300, 70, 45, 2
    geometry = torch.zeros(Q, 17)
    geometry[:, 9] = torch.rand(Q, generator=gen) * 90 - 10
    geometry[:, 10] = torch.rand(Q, generator=gen) * 65 - 10
    geometry[:, 8] = torch.randint(1, 6, (Q,), generator=gen).float()   # many depth ties
    radii = torch.randint(0, 25, (Q,), generator=gen, dtype=torch.int32)
    image_ids = torch.randint(0, images, (Q,), generator=gen)
    out = O.bin_tiles(geometry, radii, image_ids, images, W, H)
    tw, th = (W + 15) // 16, (H + 15) // 16
    x0, y0, x1, y1 = O.tile_rects(geometry.numpy(), radii.numpy(), tw, th)
    for tile in range(images * tw * th):
        img, local = divmod(tile, tw * th)
        ty, tx = divmod(local, tw)
        members = [q for q in range(Q) if radii[q] > 0 and image_ids[q] == img
                   and x0[q] <= tx < x1[q] and y0[q] <= ty < y1[q]]
        members.sort(key=lambda q: (geometry[q, 8].item(), q))
        s, e = out["ranges"][tile]
        assert list(out["point_list"][s:e]) == members
