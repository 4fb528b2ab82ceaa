"""A render + loss + backward step captured as one CUDA graph.

The reference's render call cannot be captured: its binning reads the tile
intersection count on the host (rasterize.cu:466-468; docs/contracts.md:136-138).
Here binning can run in an arena sized ahead of time (``rendering.Arena``,
``gs_bin_arena``) with every count kept on the device, so the whole step -- projection,
binning, both compositors, the projection backward and the caller's loss -- replays as
one graph launch, with no host synchronisation and no per-kernel launch overhead.
"""

from __future__ import annotations

import math

import torch

from . import rendering


class GraphedStep:
    """Capture ``loss_fn(*fn(**inputs, **kwargs)).backward()`` as a CUDA graph.

    ``inputs`` are static CUDA tensors: update them in place (``copy_``) between
    replays.  After ``replay()`` the inputs' ``.grad`` hold the step's gradients and
    the returned tensor the loss.  Arena capacities default to ``margin`` times the
    counts of an eager binning of the initial inputs; after replays on changed inputs
    check ``arena.overflowed()`` (one host read) and rebuild with a larger margin when
    it is true (the overflowing step rendered background only).  ``packed`` must be
    False (packing counts visible pairs on the host); values are not validated.
    """

    def __init__(self, fn, inputs: dict, loss_fn, *, margin: float = 1.25,
                 max_intersections: int | None = None, max_spans: int | None = None,
                 warmup: int = 2, **kwargs):
        if kwargs.get("packed", False):
            raise ValueError("GraphedStep needs packed=False (packing syncs with the host)")
        kwargs = dict(kwargs, validate=False)
        self.fn, self.inputs, self.loss_fn, self.kwargs = fn, inputs, loss_fn, kwargs
        device = next(iter(inputs.values())).device
        if max_intersections is None or max_spans is None:
            work = self._eager_counts()
            max_intersections = max_intersections or max(1, math.ceil(margin * work[0]))
            max_spans = max_spans or max(1, math.ceil(margin * work[1]))
            max_spans = min(max_spans, max_intersections)
        self.arena = rendering.Arena(max_intersections, max_spans, device)
        self.graph = torch.cuda.CUDAGraph()
        previous = rendering.ARENA
        rendering.ARENA = self.arena
        try:
            side = torch.cuda.Stream(device)
            side.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(side):
                for _ in range(warmup):
                    self._step()
            torch.cuda.current_stream(device).wait_stream(side)
            self._zero_grads()
            with torch.cuda.graph(self.graph):
                self.loss = self._step()
        finally:
            rendering.ARENA = previous

    def _zero_grads(self):
        for t in self.inputs.values():
            t.grad = None

    def _step(self):
        self._zero_grads()
        rgb, alpha, meta = self.fn(**self.inputs, **self.kwargs)
        loss = self.loss_fn(rgb, alpha, meta)
        loss.backward()
        return loss.detach()

    def _eager_counts(self):
        previous = rendering.WORK
        rendering.WORK = {}
        try:
            with torch.no_grad():
                self.fn(**self.inputs, **self.kwargs)
            work = rendering.WORK
        finally:
            rendering.WORK = previous
        return work.get("intersections", 0), work.get("spans", 0)

    def replay(self) -> torch.Tensor:
        """Run the captured step; returns the (static) loss tensor."""
        self.graph.replay()
        return self.loss
