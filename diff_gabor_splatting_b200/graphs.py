"""A render + loss + backward step captured as one CUDA graph.

The reference's render call cannot be captured: its binning reads the tile
intersection count on the host (rasterize.cu:466-468; docs/contracts.md:136-138).
Here binning can run in an arena sized ahead of time (``rendering.Arena``,
``gs_bin_arena``) with every count kept on the device, so the whole step -- projection,
binning, both compositors, the projection backward and the caller's loss -- replays as
one graph launch, with no host synchronisation and no per-kernel launch overhead.
With ``optimizer=FusedAdam(..., capturable=True)`` the optimizer step is recorded too, so
one replay is a whole training step (the reference's loop, examples/fit_texture.py:50-61:
render, loss, backward, Adam).
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

    ``optimizer`` (a ``FusedAdam`` with ``capturable=True``) is stepped after the
    backward inside the graph: every replay updates its parameters and advances its
    device step counts, except a replay whose binning overflowed the arena, which
    leaves them as they were.  The warm-up steps that precede the capture leave the
    parameters and the optimizer's state as they were.
    """

    def __init__(self, fn, inputs: dict, loss_fn, *, margin: float = 1.25,
                 max_intersections: int | None = None, max_spans: int | None = None,
                 warmup: int = 2, optimizer=None, **kwargs):
        if kwargs.get("packed", False):
            raise ValueError("GraphedStep needs packed=False (packing syncs with the host)")
        if optimizer is not None and not (
                hasattr(optimizer, "init_state")
                and all(g.get("capturable", False) for g in optimizer.param_groups)):
            raise ValueError("GraphedStep's optimizer must be FusedAdam(capturable=True)")
        kwargs = dict(kwargs, validate=False)
        self.fn, self.inputs, self.loss_fn, self.kwargs = fn, inputs, loss_fn, kwargs
        self.optimizer = optimizer
        saved = self._save_training_state()
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
            self._restore_training_state(saved)
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
        if self.optimizer is not None:
            # a replay whose binning overflowed the arena rendered background only: its
            # gradients are not the step's, so the recorded Adam step skips itself on
            # the device (parameters, moments and step counts stay as they were)
            self.optimizer.skip_flag = self.arena.overflow_flag()
            try:
                self.optimizer.step()
            finally:
                self.optimizer.skip_flag = None
        return loss.detach()

    def _save_training_state(self):
        """Copies of the optimizer's parameters and state (allocated first, so the
        tensors the graph records are the ones training continues with)."""
        if self.optimizer is None:
            return None
        self.optimizer.init_state()
        params = [p for g in self.optimizer.param_groups for p in g["params"]]
        return [(p, p.detach().clone(),
                 {k: v.clone() for k, v in self.optimizer.state[p].items() if torch.is_tensor(v)})
                for p in params]

    def _restore_training_state(self, saved):
        if saved is None:
            return
        with torch.no_grad():
            for p, value, state in saved:
                p.copy_(value)
                for k, v in state.items():
                    self.optimizer.state[p][k].copy_(v)

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
