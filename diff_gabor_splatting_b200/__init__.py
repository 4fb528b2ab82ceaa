"""B200-native differentiable classic and neural Gabor surface rasterization.

Drop-in for the render path of ``gabor_splatting`` (luisrodolfo10/diff_gabor_splatting
v0.1.1): ``rasterize_gabors`` and ``rasterize_neural_gabors`` keep the reference's
signatures and contracts; projection, binning and compositing run as hand-written
sm_100a kernels in ``libgabor_b200.so`` behind a C ABI (include/gabor_b200.h).

The renderers are imported on first use, so ``python -m diff_gabor_splatting_b200.build``
runs before the shared library exists; using them without the library raises ImportError.
"""

__all__ = ["rasterize_gabors", "rasterize_neural_gabors"]


def __getattr__(name):
    if name in __all__:
        from . import rendering

        return getattr(rendering, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
