"""CPU: host-side logic of the optimiser, the graph-captured step and the work model
(no GPU needed: every check here runs before any kernel would)."""

import dataclasses

import pytest
import torch

from diff_gabor_splatting_b200 import perfmodel
from diff_gabor_splatting_b200.graphs import GraphedStep
from diff_gabor_splatting_b200.optim import FusedAdam
from diff_gabor_splatting_b200.workloads import Workload


@pytest.mark.parametrize("kw,message", [
    (dict(lr=-1.0), "Invalid learning rate"),
    (dict(eps=-1e-8), "Invalid epsilon value"),
    (dict(betas=(1.0, 0.999)), "Invalid beta parameter at index 0"),
    (dict(betas=(0.9, -0.1)), "Invalid beta parameter at index 1"),
    (dict(weight_decay=-0.1), "Invalid weight_decay value"),
])
def test_fused_adam_rejects_what_torch_adam_rejects(kw, message):
    p = [torch.zeros(3, requires_grad=True)]
    with pytest.raises(ValueError, match=message):
        torch.optim.Adam(p, **kw)
    with pytest.raises(ValueError, match=message):
        FusedAdam(p, **kw)


@pytest.mark.parametrize("capturable", [False, True])
def test_init_state_allocates_zero_state_without_stepping(capturable):
    a, b = torch.ones(5, requires_grad=True), torch.ones(2, 3, requires_grad=True)
    opt = FusedAdam([a, b], capturable=capturable)
    opt.init_state()
    for p in (a, b):
        state = opt.state[p]
        assert set(state) == {"step", "exp_avg", "exp_avg_sq"}
        assert float(state["step"]) == 0.0 and state["step"].dtype == torch.float32
        assert state["exp_avg"].shape == p.shape and not state["exp_avg"].any()
        assert not state["exp_avg_sq"].any()
        assert torch.equal(p.detach(), torch.ones_like(p))
    assert opt.param_groups[0]["capturable"] is capturable
    first = opt.state[a]["exp_avg"]
    opt.init_state()   # idempotent: existing state is kept
    assert opt.state[a]["exp_avg"] is first


def test_graphed_step_validates_before_any_gpu_work():
    inputs = {"means": torch.zeros(1, 4, 3, requires_grad=True)}
    loss = lambda rgb, alpha, meta: rgb.sum()   # noqa: E731
    with pytest.raises(ValueError, match="packed=False"):
        GraphedStep(None, inputs, loss, packed=True)
    with pytest.raises(ValueError, match="capturable"):
        GraphedStep(None, inputs, loss, optimizer=torch.optim.SGD(inputs.values(), lr=0.1))
    with pytest.raises(ValueError, match="capturable"):
        GraphedStep(None, inputs, loss, optimizer=FusedAdam(inputs.values(), capturable=False))


def test_work_model_is_positive_and_scales_with_the_counts():
    w = Workload(config=1, method="classic", scenes=1, cameras=4, surfels=500_000,
                 width=1920, height=1080, sh_degree=3, packed=False, depth_normal_loss=False)
    counts = dict(records=2_000_000, intersections=69_386_971, spans=12_307_690,
                  forward_tests=916_009_984, forward_accepts=647_833_643,
                  backward_tests=905_160_015, backward_accepts=647_833_643)
    names = ["gs_project_forward", "gs_bin_count", "gs_bin_sort", "gs_composite_forward_split",
             "gs_composite_backward_split", "gs_project_backward"]
    for name in names:
        m = perfmodel.stage_model(name, counts, w)
        assert m["work"] > 0 and m["bound"] in ("hbm", "fp32"), name
        doubled = perfmodel.stage_model(name, {k: 2 * v for k, v in counts.items()}, w)
        if name.startswith(("gs_bin", "gs_composite")):
            assert doubled["work"] == 2 * m["work"], name
    backward = perfmodel.stage_model("gs_composite_backward_split", counts, w)
    assert backward["unit"] == "TFLOP/s"
    assert perfmodel.traffic("gs_composite_backward_split", counts) > 0
    assert perfmodel.traffic("gs_bin_sort", counts) is None
    # a loss with a normal-map gradient runs the backward variant that keeps the normal
    # fields, which executes more flops per event
    with_normals = perfmodel.stage_model("gs_composite_backward_split", counts,
                                         dataclasses.replace(w, depth_normal_loss=True))
    assert with_normals["work"] > backward["work"]
    assert backward["work"] == (perfmodel.TEST_FLOP["backward"] * counts["backward_tests"] +
                                perfmodel.BACKWARD_ACCEPT_FLOP["classic"] *
                                counts["backward_accepts"])
    # with warp accept masks the executed tests are charged the masked per-test cost
    masked = perfmodel.stage_model("gs_composite_backward_split",
                                   dict(counts, masked_intersections=1), w)
    assert masked["work"] == (perfmodel.TEST_FLOP["backward_masked"] * counts["backward_tests"] +
                              perfmodel.BACKWARD_ACCEPT_FLOP["classic"] *
                              counts["backward_accepts"])


def test_product_package_never_imports_the_oracle():
    """The oracle is test infrastructure: only tests/, __graft_entry__.smoke() and
    bench.py's CPU baseline may use it.  No module of the package imports it, and
    importing the package does not load it."""
    import ast
    import subprocess
    import sys
    from pathlib import Path

    package = Path(__file__).resolve().parents[1] / "diff_gabor_splatting_b200"
    for path in sorted(package.glob("*.py")):
        tree = ast.parse(path.read_text())
        for node in ast.walk(tree):
            names = []
            if isinstance(node, ast.Import):
                names = [a.name for a in node.names]
            elif isinstance(node, ast.ImportFrom):
                names = [node.module or ""]
            assert not any(n == "oracle" or n.startswith("oracle.") for n in names), path.name
    code = ("import sys, diff_gabor_splatting_b200 as g; g.rasterize_gabors; "
            "print(any(m == 'oracle' or m.startswith('oracle.') for m in sys.modules))")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         cwd=package.parent, timeout=300)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "False"


def test_missing_library_fails_loudly():
    """Without the built library the package raises ImportError with build instructions
    (no CPU or alternative-backend fallback)."""
    import subprocess
    import sys
    from pathlib import Path

    code = (
        "import pathlib\n"
        "exists = pathlib.Path.exists\n"
        "pathlib.Path.exists = lambda self: False if self.name == 'libgabor_b200.so' "
        "else exists(self)\n"
        "try:\n"
        "    import diff_gabor_splatting_b200 as g\n"
        "    g.rasterize_gabors\n"
        "    print('loaded')\n"
        "except ImportError as error:\n"
        "    print('ImportError:', error)\n")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         cwd=Path(__file__).resolve().parents[1], timeout=300)
    assert out.returncode == 0, out.stderr
    assert out.stdout.startswith("ImportError:"), out.stdout
    assert "no CPU or alternative-backend fallback" in out.stdout


def test_selection_groups_pixels_by_tile():
    """Selected-pixel grouping (host side of the compositor's selected-pixel mode): every
    pixel lands in exactly one group of at most 256 pixels of its own tile, in the stable
    tile order, and per-chunk views rebase tiles and output indices."""
    from diff_gabor_splatting_b200.rendering import Selection

    g = torch.Generator().manual_seed(3)
    W, H, images, P = 70, 45, 3, 900
    x = torch.randint(0, W, (images, P), generator=g)
    y = torch.randint(0, H, (images, P), generator=g)
    x[1, :400], y[1, :400] = 5, 7   # one tile with more than 256 pixels (duplicates too)
    pixels = torch.stack((x, y), -1)
    sel = Selection(pixels, W, H)
    tw, th = (W + 15) // 16, (H + 15) // 16
    image = torch.arange(images).repeat_interleave(P)
    tile = image * tw * th + (y.reshape(-1) // 16) * tw + x.reshape(-1) // 16
    expected_order = torch.argsort(tile, stable=True)
    assert torch.equal(sel.sel_index, expected_order)
    seen = torch.zeros(images * P, dtype=torch.long)
    for t, first, count in zip(sel.group_tile.tolist(), sel.group_first.tolist(),
                               sel.group_count.tolist()):
        assert 1 <= count <= 256
        members = sel.sel_index[first:first + count]
        assert bool((tile[members] == t).all())
        seen[members] += 1
    assert bool((seen == 1).all())
    assert int(sel.group_count.sum()) == images * P
    selected, groups = sel.for_images(1, 2)   # images 1-2 as one chunk
    assert bool((groups[:, 0] >= 0).all()) and bool((groups[:, 0] < 2 * tw * th).all())
    assert int(groups[:, 2].sum()) == 2 * P
    for local_tile, first, count, _ in groups.tolist():
        out = selected[first:first + count, 2].long()
        assert bool((out >= 0).all()) and bool((out < 2 * P).all())
        assert bool((tile[out + P] == local_tile + tw * th).all())
