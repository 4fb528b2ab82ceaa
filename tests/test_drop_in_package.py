"""The ``gabor_splatting`` import path serves this build (no GPU needed).

The reference's callers import ``gabor_splatting`` (src/gabor_splatting/__init__.py:1-5),
``gabor_splatting.rendering`` (tests/test_spherical_harmonics.py:5) and monkeypatch
``gabor_splatting.rendering.check_values`` (tests/test_rendering.py:405-414).
"""

import inspect

import gabor_splatting
import gabor_splatting._C as drop_in_C
import gabor_splatting.rendering as drop_in_rendering
from gabor_splatting import rasterize_gabors, rasterize_neural_gabors
from gabor_splatting.rendering import SHColors, check_tensor, check_values

import diff_gabor_splatting_b200
from diff_gabor_splatting_b200 import _C, rendering


def test_modules_are_this_builds():
    assert drop_in_rendering is rendering
    assert drop_in_C is _C
    assert gabor_splatting.rendering is rendering and gabor_splatting._C is _C
    assert rasterize_gabors is diff_gabor_splatting_b200.rasterize_gabors
    assert rasterize_neural_gabors is diff_gabor_splatting_b200.rasterize_neural_gabors
    assert SHColors is rendering.SHColors and check_tensor is rendering.check_tensor
    assert check_values is rendering.check_values
    assert gabor_splatting.__all__ == ["rasterize_gabors", "rasterize_neural_gabors"]
    for name in ("rasterize_forward", "rasterize_backward", "evaluate_sh_forward",
                 "evaluate_sh_backward"):
        assert callable(getattr(drop_in_C, name)), name


def test_check_values_patch_reaches_the_renderer(monkeypatch):
    """render looks check_values up at call time, so patching it under the drop-in name
    replaces the one the renderer calls (the reference's trusted-path test relies on it)."""
    calls = []
    monkeypatch.setattr(drop_in_rendering, "check_values", lambda *a: calls.append(a))
    assert rendering.check_values is not check_values
    source = inspect.getsource(rendering.render)
    assert "check_values(" in source


def test_public_signatures_match_the_reference_keywords():
    for fn, extra in ((rasterize_gabors, ["sh_degree"]), (rasterize_neural_gabors, [])):
        params = inspect.signature(fn).parameters
        for name in ["backgrounds", "packed", "near_plane", "far_plane", *extra, "validate"]:
            assert params[name].kind is inspect.Parameter.KEYWORD_ONLY, name
        assert params["packed"].default is False and params["validate"].default is True
        assert params["near_plane"].default == 0.2 and params["far_plane"].default == 100.0
