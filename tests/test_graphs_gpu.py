"""Binning without a host synchronisation (gs_bin_arena) and the render step captured
as a CUDA graph (row "next" 2: a step that CUDA graphs can capture)."""

import ctypes

import numpy as np
import pytest
import torch

from diff_gabor_splatting_b200 import _native as nat
from diff_gabor_splatting_b200 import rasterize_gabors, rasterize_neural_gabors, rendering
from diff_gabor_splatting_b200.graphs import GraphedStep
from helpers import assert_grads_close, maps_from_result, ordered, random_scene

pytestmark = pytest.mark.gpu

W, H = 70, 45


def _records(method="classic", scenes=2, cameras=3, n=400):
    v = random_scene(method, scenes=scenes, cameras=cameras, n=n, width=W, height=H)
    with torch.no_grad():
        records, _, _, radii = rendering.Projection.apply(
            v["means"], v["quaternions"], v["scales"], v["opacities"], v["view_matrices"],
            v["intrinsics"], None, None, None, None, None, None, W, H, 0.2, 100.0)
    return records, radii, scenes * cameras, n


def _arena_bin(records, radii, images, n, flags, max_i, max_s):
    size = ctypes.c_size_t()
    nat.call("gs_bin_arena_workspace", records.shape[0], max_i, max_s, images, W, H,
             ctypes.byref(size))
    ws = torch.empty(size.value, dtype=torch.uint8, device="cuda")
    point_list = torch.full((max_i,), -7, dtype=torch.int32, device="cuda")
    tw, th = (W + 15) // 16, (H + 15) // 16
    ranges = torch.full((images * tw * th, 2), -7, dtype=torch.int32, device="cuda")
    totals = torch.zeros(2, dtype=torch.int64, device="cuda")
    nat.call("gs_bin_arena", nat.ptr(records), 20, nat.ptr(radii), None, records.shape[0], n,
             images, W, H, flags, nat.ptr(ws), size.value, max_i, max_s, nat.ptr(point_list),
             nat.ptr(ranges), nat.ptr(totals), nat.stream_of(records.device))
    return point_list, ranges, totals


@pytest.mark.parametrize("flags", [0, nat.BIN_TIGHT])
def test_arena_binning_equals_counted_binning(flags):
    records, radii, images, n = _records()
    point_list, ranges = rendering.bin_records(records, 20, radii, None, n, images, W, H, flags)
    I = point_list.shape[0]
    # spans are at most the intersections; give the arena room for both
    for slack in (0, 1, 5000):
        a_list, a_ranges, totals = _arena_bin(records, radii, images, n, flags, I + slack,
                                              I + slack)
        assert int(totals[0]) == I
        assert torch.equal(a_ranges, ranges)
        assert torch.equal(a_list[:I], point_list)


def test_arena_overflow_bins_nothing_and_reports_the_counts():
    records, radii, images, n = _records()
    point_list, _ = rendering.bin_records(records, 20, radii, None, n, images, W, H, 0)
    I = point_list.shape[0]
    _, a_ranges, totals = _arena_bin(records, radii, images, n, 0, I - 1, I - 1)
    assert int(totals[0]) == I
    assert bool((a_ranges == 0).all())


def _loss(rgb, alpha, meta):
    return rgb.mean() + alpha.mean() + 0.01 * meta["distortion"].mean()


@pytest.mark.parametrize("method", ["classic", "neural"])
def test_graph_replay_matches_eager_steps(method):
    v = random_scene(method, scenes=2, cameras=2, n=300, width=W, height=H, conditioned=True)
    fn = rasterize_gabors if method == "classic" else rasterize_neural_gabors
    static = {k: t.clone().requires_grad_() for k, t in ordered(v, method).items()}
    step = GraphedStep(fn, static, _loss, width=W, height=H)

    def eager(values):
        mine = {k: t.detach().clone().requires_grad_() for k, t in values.items()}
        rgb, alpha, meta = fn(**mine, width=W, height=H)
        loss = _loss(rgb, alpha, meta)
        loss.backward()
        return loss.detach(), {k: t.grad for k, t in mine.items()}

    g = torch.Generator(device="cuda").manual_seed(5)
    for replay in range(3):
        if replay:   # new inputs, written in place into the captured tensors
            with torch.no_grad():
                static["means"].add_(0.01 * torch.randn(static["means"].shape, device="cuda",
                                                        generator=g))
                static["opacities"].mul_(0.98)
        loss = step.replay()
        torch.cuda.synchronize()
        assert not step.arena.overflowed()
        expected_loss, expected_grads = eager(static)
        torch.testing.assert_close(loss, expected_loss, rtol=1e-6, atol=1e-7)
        for name, t in static.items():
            assert_grads_close(t.grad, expected_grads[name], name, elementwise=1e-4)


def test_graph_overflow_is_reported():
    v = random_scene("classic", scenes=1, cameras=2, n=300, width=W, height=H)
    static = {k: t.clone().requires_grad_() for k, t in ordered(v, "classic").items()}
    step = GraphedStep(rasterize_gabors, static, _loss, width=W, height=H,
                       max_intersections=16, max_spans=16)
    step.replay()
    assert step.arena.overflowed()
    needed = step.arena.needed()
    assert needed[0] > 16
    with pytest.raises(ValueError, match="packed=False"):
        GraphedStep(rasterize_gabors, static, _loss, width=W, height=H, packed=True)


def test_graphed_training_step_skips_adam_when_the_arena_overflows():
    """A replay whose binning overflowed renders background only; the recorded Adam step
    then leaves parameters, moments and device step counts unchanged."""
    from diff_gabor_splatting_b200.optim import FusedAdam

    v = random_scene("classic", scenes=1, cameras=2, n=300, width=W, height=H)
    static = {k: t.clone().requires_grad_() for k, t in ordered(v, "classic").items()}
    trained = [k for k in static if k not in ("view_matrices", "intrinsics", "backgrounds")]
    opt = FusedAdam([static[k] for k in trained], lr=1e-2, capturable=True)
    step = GraphedStep(rasterize_gabors, static, _loss, optimizer=opt, width=W, height=H,
                       max_intersections=16, max_spans=16)
    before = {k: static[k].detach().clone() for k in trained}
    for _ in range(2):
        step.replay()
    torch.cuda.synchronize()
    assert step.arena.overflowed()
    for k in trained:
        assert torch.equal(static[k].detach(), before[k]), k
        state = opt.state[static[k]]
        assert float(state["step"]) == 0.0, k
        assert state["exp_avg"].count_nonzero() == 0 and state["exp_avg_sq"].count_nonzero() == 0
    # the same graph machinery with room in the arena does train
    roomy = GraphedStep(rasterize_gabors, static, _loss, optimizer=opt, width=W, height=H)
    roomy.replay()
    torch.cuda.synchronize()
    assert not roomy.arena.overflowed()
    assert float(opt.state[static["means"]]["step"]) == 1.0
    assert not torch.equal(static["means"].detach(), before["means"])


@pytest.mark.parametrize("method", ["classic", "neural"])
def test_graphed_training_step_matches_eager_training(method):
    """Render + loss + backward + FusedAdam(capturable) captured as one graph: three
    replays leave the parameters where three eager training steps do, and building the
    graph leaves the parameters and optimizer state untouched."""
    from diff_gabor_splatting_b200.optim import FusedAdam

    v = random_scene(method, scenes=1, cameras=2, n=300, width=W, height=H, conditioned=True)
    fn = rasterize_gabors if method == "classic" else rasterize_neural_gabors
    static = {k: t.clone().requires_grad_() for k, t in ordered(v, method).items()}
    eager = {k: t.detach().clone().requires_grad_() for k, t in static.items()}
    trained = [k for k in static if k not in ("view_matrices", "intrinsics", "backgrounds")]
    opt = FusedAdam([static[k] for k in trained], lr=1e-3, capturable=True)
    ref = FusedAdam([eager[k] for k in trained], lr=1e-3)
    step = GraphedStep(fn, static, _loss, optimizer=opt, width=W, height=H)
    for k in static:   # the warm-up steps were undone
        torch.testing.assert_close(static[k].detach(), eager[k].detach(), rtol=0, atol=0)
    assert int(opt.state[static[trained[0]]]["step"]) == 0
    losses = []
    for _ in range(3):
        losses.append(step.replay().clone())
        for t in eager.values():
            t.grad = None
        # trained quaternions and wave weights leave the reference's validation ranges
        rgb, alpha, meta = fn(**eager, width=W, height=H, validate=False)
        loss = _loss(rgb, alpha, meta)
        loss.backward()
        ref.step()
        torch.testing.assert_close(losses[-1], loss.detach(), rtol=1e-5, atol=1e-7)
    torch.cuda.synchronize()
    assert not step.arena.overflowed()
    assert int(opt.state[static[trained[0]]]["step"]) == 3
    for k in trained:
        scale = float(eager[k].detach().abs().max()) + 1e-12
        err = float((static[k].detach() - eager[k].detach()).abs().max()) / scale
        assert err < 1e-5, f"{k}: {err:.2e} of its scale after three training steps"
    with pytest.raises(ValueError, match="capturable"):
        GraphedStep(fn, static, _loss, optimizer=FusedAdam([static["means"]]), width=W,
                    height=H)
