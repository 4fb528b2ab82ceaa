"""Fused Adam for the renderer's parameters.

The reference's optimisation loop (examples/fit_texture.py:50-61) steps
``torch.optim.Adam(params, lr=...)`` after every render backward.  ``FusedAdam`` is a
drop-in for that optimizer (same constructor arguments without ``amsgrad``,
``maximize``, ``foreach``, ``capturable``, ``differentiable`` and ``fused``; same
state keys ``step``, ``exp_avg``, ``exp_avg_sq``; same update), whose ``step()`` is one
launch of ``gs_adam_step`` per parameter group (48 tensors per launch) instead of
torch's ~10 element-wise passes over every parameter, gradient and moment.

``capturable=True`` mirrors ``torch.optim.Adam(capturable=True)``: each parameter's step
count is a float32 tensor on its device, advanced and read by the kernels
(``gs_adam_step_capturable``), so ``step()`` makes no host round trip and can be recorded
in a CUDA graph (``graphs.GraphedStep(optimizer=...)``).
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as nat


class FusedAdam(torch.optim.Optimizer):
    """Adam (Kingma & Ba) with L2 weight decay, as ``torch.optim.Adam`` computes it.

    Parameters must be contiguous float32 CUDA tensors.  Parameters without a
    gradient are skipped (their state is untouched), as torch does.
    """

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, capturable: bool = False):
        if not lr >= 0.0:
            raise ValueError(f"Invalid learning rate: {lr}")
        if not eps >= 0.0:
            raise ValueError(f"Invalid epsilon value: {eps}")
        if not 0.0 <= betas[0] < 1.0:
            raise ValueError(f"Invalid beta parameter at index 0: {betas[0]}")
        if not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"Invalid beta parameter at index 1: {betas[1]}")
        if not weight_decay >= 0.0:
            raise ValueError(f"Invalid weight_decay value: {weight_decay}")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                                      capturable=capturable))
        # capturable steps only: a device int32 flag read when the step runs; nonzero
        # leaves parameters, moments and step counts unchanged (set by GraphedStep to
        # its arena's overflow flag)
        self.skip_flag = None

    def init_state(self):
        """Create every parameter's state (zero moments, step 0) without stepping, so a
        CUDA graph can record ``step()`` with the state tensors already allocated."""
        for group in self.param_groups:
            for p in group["params"]:
                state = self.state[p]
                if len(state) == 0:
                    state["step"] = (torch.zeros((), dtype=torch.float32, device=p.device)
                                     if group["capturable"] else torch.tensor(0.0))
                    state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            if group["capturable"]:
                self._step_capturable(group)
                continue
            by_step = {}
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise RuntimeError("FusedAdam does not support sparse gradients")
                if not (p.is_cuda and p.dtype == torch.float32 and p.is_contiguous()):
                    raise RuntimeError("FusedAdam needs contiguous float32 CUDA parameters")
                grad = p.grad if p.grad.is_contiguous() else p.grad.contiguous()
                state = self.state[p]
                if len(state) == 0:
                    state["step"] = torch.tensor(0.0)
                    state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                state["step"] += 1
                key = (p.device, int(state["step"].item()))
                by_step.setdefault(key, []).append((p, grad, state))
            beta1, beta2 = group["betas"]
            for (device, step), items in by_step.items():
                params, params_ptr = nat.host_array(ctypes.c_void_p, [p.data_ptr() for p, _, _ in items])
                grads, grads_ptr = nat.host_array(ctypes.c_void_p, [g.data_ptr() for _, g, _ in items])
                m1, m1_ptr = nat.host_array(ctypes.c_void_p,
                                            [s["exp_avg"].data_ptr() for _, _, s in items])
                m2, m2_ptr = nat.host_array(ctypes.c_void_p,
                                            [s["exp_avg_sq"].data_ptr() for _, _, s in items])
                sizes, sizes_ptr = nat.host_array(ctypes.c_int64, [p.numel() for p, _, _ in items])
                with torch.cuda.device(device):
                    nat.call("gs_adam_step", len(items), params_ptr, grads_ptr, m1_ptr, m2_ptr,
                             sizes_ptr, float(group["lr"]), float(beta1), float(beta2),
                             float(group["eps"]), float(group["weight_decay"]), step,
                             nat.stream_of(device))
        return loss

    def _step_capturable(self, group):
        """One ``gs_adam_step_capturable`` call per device: step counts stay on the device."""
        by_device = {}
        for p in group["params"]:
            if p.grad is None:
                continue
            if p.grad.is_sparse:
                raise RuntimeError("FusedAdam does not support sparse gradients")
            if not (p.is_cuda and p.dtype == torch.float32 and p.is_contiguous()):
                raise RuntimeError("FusedAdam needs contiguous float32 CUDA parameters")
            if not p.grad.is_contiguous():
                raise RuntimeError("FusedAdam(capturable=True) needs contiguous gradients")
            state = self.state[p]
            if len(state) == 0:
                state["step"] = torch.zeros((), dtype=torch.float32, device=p.device)
                state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            if not (state["step"].is_cuda and state["step"].device == p.device):
                raise RuntimeError("FusedAdam(capturable=True) needs step counts on the "
                                   "parameters' device")
            by_device.setdefault(p.device, []).append((p, state))
        beta1, beta2 = group["betas"]
        flag = self.skip_flag
        if flag is not None and not (flag.is_cuda and flag.dtype == torch.int32
                                     and flag.numel() == 1):
            raise RuntimeError("FusedAdam.skip_flag must be a one-element int32 CUDA tensor")
        for device, items in by_device.items():
            skip = nat.ptr(flag) if flag is not None and flag.device == device else None
            arrays = [nat.host_array(ctypes.c_void_p, ptrs) for ptrs in (
                [p.data_ptr() for p, _ in items], [p.grad.data_ptr() for p, _ in items],
                [s["exp_avg"].data_ptr() for _, s in items],
                [s["exp_avg_sq"].data_ptr() for _, s in items],
                [s["step"].data_ptr() for _, s in items])]
            sizes = nat.host_array(ctypes.c_int64, [p.numel() for p, _ in items])
            with torch.cuda.device(device):
                nat.call("gs_adam_step_capturable", len(items), arrays[0][1], arrays[1][1],
                         arrays[2][1], arrays[3][1], sizes[1], arrays[4][1], float(group["lr"]),
                         float(beta1), float(beta2), float(group["eps"]),
                         float(group["weight_decay"]), skip, nat.stream_of(device))
