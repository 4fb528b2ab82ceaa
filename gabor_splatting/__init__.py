"""The reference's import path, served by this build.

luisrodolfo10/diff_gabor_splatting v0.1.1 is imported as ``gabor_splatting``
(src/gabor_splatting/__init__.py:1-5); its callers and tests write
``from gabor_splatting import rasterize_gabors, rasterize_neural_gabors``,
``from gabor_splatting.rendering import SHColors`` and monkeypatch
``gabor_splatting.rendering.check_values``.  This package answers those imports with
this build's own modules -- it holds no second implementation:

* ``gabor_splatting.rendering`` is the module object ``diff_gabor_splatting_b200.rendering``
  under a second name, so a monkeypatch of ``gabor_splatting.rendering.check_values``
  reaches the renderer (which looks the function up at call time, as the reference's
  ``render`` does, rendering.py:320-321);
* ``gabor_splatting._C`` is ``diff_gabor_splatting_b200._C``, the mirror of the
  reference's pybind11 module (csrc/bindings.cpp:6-10) over the C ABI.
"""

import sys

from diff_gabor_splatting_b200 import _C, rendering
from diff_gabor_splatting_b200.rendering import rasterize_gabors, rasterize_neural_gabors

sys.modules[__name__ + ".rendering"] = rendering
sys.modules[__name__ + "._C"] = _C

__all__ = ["rasterize_gabors", "rasterize_neural_gabors"]
