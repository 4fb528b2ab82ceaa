"""Fused Adam (row "next" 1: the optimiser step of the reference's fitting loop,
examples/fit_texture.py:50-61) against torch.optim.Adam on the same gradients."""

import math

import pytest
import torch

from diff_gabor_splatting_b200 import rasterize_gabors, rasterize_neural_gabors
from diff_gabor_splatting_b200.optim import FusedAdam

pytestmark = pytest.mark.gpu


def _pair(shapes, seed, **kw):
    g = torch.Generator(device="cuda").manual_seed(seed)
    base = [torch.randn(s, device="cuda", generator=g) for s in shapes]
    ours = [t.clone().requires_grad_() for t in base]
    theirs = [t.clone().requires_grad_() for t in base]
    return ours, theirs, FusedAdam(ours, **kw), torch.optim.Adam(theirs, **kw), g


@pytest.mark.parametrize("kw", [dict(lr=0.01), dict(lr=3e-3, betas=(0.8, 0.99), eps=1e-6,
                                                    weight_decay=0.01)])
def test_matches_torch_adam(kw):
    # sizes: single elements, odd tails, a misaligned view-free mix, and a large tensor
    shapes = [(1,), (3,), (5, 7), (1000,), (4097,), (2_000_003,), (64, 16, 3)]
    ours, theirs, fused, reference, g = _pair(shapes, 0, **kw)
    for step in range(6):
        for a, b in zip(ours, theirs):
            grad = torch.randn(a.shape, device="cuda", generator=g) * (10.0 ** (step - 3))
            a.grad, b.grad = grad.clone(), grad.clone()
        ours[2].grad = None if step == 3 else ours[2].grad   # a parameter without a gradient
        theirs[2].grad = None if step == 3 else theirs[2].grad
        fused.step()
        reference.step()
    for a, b in zip(ours, theirs):
        torch.testing.assert_close(a, b, rtol=2e-6, atol=1e-7)
        sa, sb = fused.state[a], reference.state[b]
        assert int(sa["step"]) == int(sb["step"])
        torch.testing.assert_close(sa["exp_avg"], sb["exp_avg"], rtol=1e-6, atol=1e-9)
        torch.testing.assert_close(sa["exp_avg_sq"], sb["exp_avg_sq"], rtol=1e-6, atol=1e-12)


def test_param_groups_and_state_dict():
    a = torch.randn(100, device="cuda", requires_grad=True)
    b = torch.randn(37, device="cuda", requires_grad=True)
    opt = FusedAdam([{"params": [a], "lr": 0.1}, {"params": [b]}], lr=1e-3)
    ref_a, ref_b = a.detach().clone().requires_grad_(), b.detach().clone().requires_grad_()
    ref = torch.optim.Adam([{"params": [ref_a], "lr": 0.1}, {"params": [ref_b]}], lr=1e-3)
    for _ in range(3):
        for x, y in ((a, ref_a), (b, ref_b)):
            grad = torch.randn_like(x)
            x.grad, y.grad = grad, grad.clone()
        opt.step()
        ref.step()
    torch.testing.assert_close(a, ref_a, rtol=2e-6, atol=1e-7)
    torch.testing.assert_close(b, ref_b, rtol=2e-6, atol=1e-7)
    state = opt.state_dict()
    assert set(state["state"][0]) == {"step", "exp_avg", "exp_avg_sq"}
    with pytest.raises(RuntimeError, match="contiguous float32 CUDA"):
        bad = torch.randn(4, 4, device="cuda").t().requires_grad_()
        bad.grad = torch.ones_like(bad)
        FusedAdam([bad]).step()


@pytest.mark.parametrize("method", ["classic", "neural"])
def test_fit_texture_loop_matches_torch_adam(method):
    """The reference example's loop (examples/fit_texture.py:13-70), run with both
    optimisers: the loss curves agree."""
    def run(optimizer_class):
        torch.manual_seed(3)
        geometry = {
            "means": torch.tensor([[0.0, 0.0, 3.0]], device="cuda"),
            "quaternions": torch.tensor([[1.0, 0.0, 0.0, 0.0]], device="cuda"),
            "scales": torch.tensor([[0.7, 0.7]], device="cuda"),
            "opacities": torch.tensor([0.9], device="cuda"),
            "view_matrices": torch.eye(4, device="cuda")[None],
            "intrinsics": torch.tensor([[[40.0, 0.0, 15.5], [0.0, 40.0, 15.5], [0.0, 0.0, 1.0]]],
                                       device="cuda"),
            "width": 32,
            "height": 32,
        }
        x = torch.arange(32, device="cuda")[None, None, :, None].expand(1, 32, 32, 3)
        target = (0.5 + 0.4 * torch.cos(x * 0.7)).contiguous()
        if method == "classic":
            values = {
                "colors": torch.tensor([[0.6, 0.4, 0.5]], device="cuda", requires_grad=True),
                "secondary_colors": torch.tensor([[0.3, 0.5, 0.4]], device="cuda",
                                                 requires_grad=True),
                "frequency_weights": torch.tensor([[1.0, 0.0, 0.0, 0.0]], device="cuda"),
                "frequency_magnitudes": torch.full((1, 4), 1.0, device="cuda",
                                                   requires_grad=True),
                "phases": torch.zeros(1, 4, device="cuda", requires_grad=True),
            }
            function = rasterize_gabors
        else:
            values = {
                "input_weights": torch.empty(1, 6, 5, device="cuda").uniform_(-1 / 5, 1 / 5)
                .requires_grad_(),
                "input_biases": torch.zeros(1, 6, device="cuda", requires_grad=True),
                "output_weights": torch.empty(1, 3, 6, device="cuda")
                .uniform_(-1 / 30, 1 / 30).requires_grad_(),
                "output_biases": torch.zeros(1, 3, device="cuda", requires_grad=True),
            }
            function = rasterize_neural_gabors
        optimizer = optimizer_class([v for v in values.values() if v.requires_grad], lr=0.01)
        losses = []
        for _ in range(40):
            optimizer.zero_grad(set_to_none=True)
            rgb, alpha, _ = function(**geometry, **values)
            loss = ((rgb - target * alpha.detach()).square()).mean()
            loss.backward()
            optimizer.step()
            if method == "classic":
                with torch.no_grad():
                    values["frequency_magnitudes"].clamp_min_(0)
            losses.append(loss.item())
        return losses

    ours, theirs = run(FusedAdam), run(torch.optim.Adam)
    assert all(math.isfinite(v) for v in ours)
    assert ours[-1] < ours[0]
    for a, b in zip(ours, theirs):
        assert abs(a - b) <= 1e-5 * max(abs(b), 1e-6) + 1e-9, (a, b)


@pytest.mark.parametrize("kw", [dict(lr=0.01), dict(lr=3e-3, betas=(0.8, 0.99), eps=1e-6,
                                                    weight_decay=0.01)])
def test_capturable_matches_torch_adam(kw):
    """Device step counts (gs_adam_step_capturable) give torch.optim.Adam's update, with
    the counts advanced on the device (a parameter without a gradient keeps its count)."""
    shapes = [(1,), (5, 7), (4097,), (300_001,)]
    ours, theirs, fused, reference, g = _pair(shapes, 1, **kw)
    fused = FusedAdam(ours, capturable=True, **kw)
    for step in range(6):
        for a, b in zip(ours, theirs):
            grad = torch.randn(a.shape, device="cuda", generator=g) * (10.0 ** (step - 3))
            a.grad, b.grad = grad.clone(), grad.clone()
        if step == 2:
            ours[1].grad = theirs[1].grad = None
        fused.step()
        reference.step()
    for a, b in zip(ours, theirs):
        torch.testing.assert_close(a, b, rtol=2e-6, atol=1e-7)
        sa, sb = fused.state[a], reference.state[b]
        assert sa["step"].is_cuda and int(sa["step"]) == int(sb["step"])
        torch.testing.assert_close(sa["exp_avg"], sb["exp_avg"], rtol=1e-6, atol=1e-9)


def test_capturable_step_replays_in_a_cuda_graph():
    """The capturable step recorded once in a CUDA graph and replayed on gradients written
    in place equals eager steps (the step count advancing on every replay)."""
    g = torch.Generator(device="cuda").manual_seed(2)
    base = [torch.randn(s, device="cuda", generator=g) for s in [(33,), (1000, 3)]]
    graphed = [t.clone() for t in base]
    eager = [t.clone() for t in base]
    grads = [torch.zeros_like(t) for t in base]
    for p, gr in zip(graphed, grads):
        p.grad = gr
    opt = FusedAdam(graphed, lr=0.05, capturable=True)
    opt.init_state()
    ref = FusedAdam(eager, lr=0.05)
    warm = torch.zeros(8, device="cuda")   # load the kernels before capturing
    warm.grad = torch.ones_like(warm)
    FusedAdam([warm], capturable=True).step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side), torch.cuda.graph(graph):
        opt.step()
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(5):
        step_grads = [torch.randn(t.shape, device="cuda", generator=g) for t in base]
        for gr, new in zip(grads, step_grads):
            gr.copy_(new)
        for p, new in zip(eager, step_grads):
            p.grad = new.clone()
        graph.replay()
        ref.step()
    torch.cuda.synchronize()
    for a, b in zip(graphed, eager):
        torch.testing.assert_close(a, b, rtol=2e-6, atol=1e-7)
    assert int(opt.state[graphed[0]]["step"]) == 5
