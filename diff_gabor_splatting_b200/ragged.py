"""Ragged scene batches: scenes with different surfel counts in one render call.

The reference renders batches ``[..., N, ...]`` whose scenes all have N surfels and
lists ragged scene batches outside its release (README.md:267-270).  Here the
per-surfel inputs of S scenes are concatenated (``[N_0 + ... + N_{S-1}, ...]``) with
``counts`` giving each scene's N_s; cameras stay ``[S, C, ...]``.  Projection runs
over the ragged layout directly (``gs_project_forward_ragged``: scene s owns surfels
``[o_s, o_s + N_s)`` and pairs ``[C o_s, C (o_s + N_s))``), binning takes each pair's
image from an explicit image-id array, and the compositor reads each record's
appearance row through an explicit row index -- no padding to the largest scene.

Outputs are ``[S, C, H, W, k]`` like a dense batch; pair metadata (radii,
projected_means, scene/camera/primitive ids) is flat over the pairs in scene, camera,
surfel order, as in packed mode.
"""

from __future__ import annotations

from typing import Any

import torch
from torch.autograd.function import once_differentiable

from . import _native as nat
from . import rendering
from .rendering import Chunk, Composite, SurfelRows, bin_records, check_tensor, check_values


class RaggedProjection(torch.autograd.Function):
    """``gs_project_forward_ragged`` / ``gs_project_backward_ragged`` (the dense
    Projection's kernels with per-scene surfel ranges)."""

    @staticmethod
    def forward(ctx, means, quaternions, scales, opacities, view_matrices, intrinsics,
                sh_first, sh_second, frequency_weights, frequency_magnitudes, phases,
                offsets, max_surfels, sh_degree, width, height, near_plane, far_plane):
        S, C = view_matrices.shape[0], view_matrices.shape[1]
        total = means.shape[0]
        P = C * total
        device = means.device
        records = torch.empty((P, nat.RECORD_FLOATS), device=device, dtype=torch.float32)
        xy = torch.empty((P, 2), device=device, dtype=torch.float32)
        radii = torch.empty((P,), device=device, dtype=torch.int32)
        sh = sh_degree is not None
        rows = torch.empty((P if sh else 0, nat.CLASSIC_ROW_FLOATS), device=device,
                           dtype=torch.float32)
        nat.call("gs_project_forward_ragged", nat.ptr(means), nat.ptr(quaternions),
                 nat.ptr(scales), nat.ptr(opacities), nat.ptr(view_matrices),
                 nat.ptr(intrinsics), nat.ptr(sh_first), nat.ptr(sh_second),
                 nat.ptr(frequency_weights), nat.ptr(frequency_magnitudes), nat.ptr(phases),
                 -1 if sh_degree is None else sh_degree, S, C, nat.ptr(offsets), max_surfels,
                 width, height, near_plane, far_plane, nat.ptr(records), nat.ptr(xy),
                 nat.ptr(rows), nat.ptr(radii), nat.stream_of(device))
        ctx.save_for_backward(means, quaternions, scales, view_matrices, intrinsics, sh_first,
                              sh_second, offsets)
        ctx.options = (sh_degree, max_surfels)
        ctx.mark_non_differentiable(radii)
        return records, xy, rows, radii

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_records, grad_xy, grad_rows, _grad_radii):
        means, quaternions, scales, view_matrices, intrinsics, sh_first, sh_second, offsets = \
            ctx.saved_tensors
        sh_degree, max_surfels = ctx.options
        S, C = view_matrices.shape[0], view_matrices.shape[1]
        total = means.shape[0]
        P = C * total
        device = means.device
        sh = sh_degree is not None
        zeros = (lambda *shape: torch.zeros(shape, device=device, dtype=torch.float32))
        grad_records = zeros(P, nat.RECORD_FLOATS) if grad_records is None else grad_records
        grad_xy = zeros(P, 2) if grad_xy is None else grad_xy
        if sh and grad_rows is None:
            grad_rows = zeros(P, nat.CLASSIC_ROW_FLOATS)
        grad_records, grad_xy = grad_records.contiguous(), grad_xy.contiguous()
        if grad_rows is not None:
            grad_rows = grad_rows.contiguous()
        g_means = torch.zeros_like(means)
        g_quats = torch.zeros_like(quaternions)
        g_scales = torch.zeros_like(scales)
        g_opac = torch.zeros((total,), device=device, dtype=torch.float32)
        g_views = torch.empty_like(view_matrices)
        g_intr = torch.empty_like(intrinsics)
        g_sh1 = torch.empty_like(sh_first) if sh else None
        g_sh2 = torch.empty_like(sh_second) if sh else None
        g_w = torch.zeros((total, 4), device=device) if sh else None
        g_m = torch.zeros((total, 4), device=device) if sh else None
        g_p = torch.zeros((total, 4), device=device) if sh else None
        nat.call("gs_project_backward_ragged", nat.ptr(means), nat.ptr(quaternions),
                 nat.ptr(scales), nat.ptr(view_matrices), nat.ptr(intrinsics), nat.ptr(sh_first),
                 nat.ptr(sh_second), -1 if sh_degree is None else sh_degree, S, C,
                 nat.ptr(offsets), max_surfels, total, nat.ptr(grad_records), nat.ptr(grad_xy),
                 nat.ptr(grad_rows), nat.ptr(g_means), nat.ptr(g_quats), nat.ptr(g_scales),
                 nat.ptr(g_opac), nat.ptr(g_views), nat.ptr(g_intr), nat.ptr(g_sh1),
                 nat.ptr(g_sh2), nat.ptr(g_w), nat.ptr(g_m), nat.ptr(g_p), nat.stream_of(device))
        return (g_means, g_quats, g_scales, g_opac, g_views, g_intr, g_sh1, g_sh2, g_w, g_m,
                g_p) + (None,) * 7


def _render_ragged(means, quaternions, scales, opacities, appearance, view_matrices,
                   intrinsics, width, height, counts, backgrounds, near_plane, far_plane, neural,
                   sh_degree, validate, median_depth):
    if not isinstance(view_matrices, torch.Tensor) or view_matrices.ndim != 4:
        raise ValueError("view_matrices must have shape [S, C, 4, 4]")
    S, C = view_matrices.shape[0], view_matrices.shape[1]
    counts = [int(n) for n in (counts.tolist() if isinstance(counts, torch.Tensor) else counts)]
    if len(counts) != S or any(n < 0 for n in counts):
        raise ValueError("counts must give a non-negative surfel count for each of the S scenes")
    if type(width) is not int or type(height) is not int or not (0 < width < 2**30
                                                               and 0 < height < 2**30):
        raise ValueError("width and height must be positive integers smaller than 2**30")
    if not 0 < near_plane < far_plane:
        raise ValueError("clipping planes must be finite and satisfy 0 < near_plane < far_plane")
    if type(median_depth) is not bool or type(validate) is not bool:
        raise TypeError("validate and median_depth must be bool")
    total = sum(counts)
    if not isinstance(means, torch.Tensor):
        raise TypeError("means must be a torch.Tensor")
    device = means.device
    tensors = {
        "means": (means, (total, 3)),
        "quaternions": (quaternions, (total, 4)),
        "scales": (scales, (total, 2)),
        "opacities": (opacities, (total,)),
        "view_matrices": (view_matrices, (S, C, 4, 4)),
        "intrinsics": (intrinsics, (S, C, 3, 3)),
    }
    if backgrounds is None:
        backgrounds = means.new_zeros((S, C, 3))
    tensors["backgrounds"] = backgrounds, (S, C, 3)
    if neural:
        shapes, names = [(6, 5), (6,), (3, 6), (3,)], ["input_weights", "input_biases",
                                                       "output_weights", "output_biases"]
    else:
        if sh_degree is not None and (type(sh_degree) is not int or not 0 <= sh_degree <= 3):
            raise ValueError("sh_degree must be None or an integer from 0 to 3")
        color = (3,) if sh_degree is None else ((sh_degree + 1) ** 2, 3)
        shapes = [color, color, (4,), (4,), (4,)]
        names = ["colors", "secondary_colors", "frequency_weights", "frequency_magnitudes",
                 "phases"]
    for name, tensor, shape in zip(names, appearance, shapes):
        tensors[name] = tensor, (total,) + shape
    for name, (tensor, shape) in tensors.items():
        check_tensor(name, tensor, shape, device)
    if validate:
        check_values(tensors, quaternions, scales, opacities, view_matrices, intrinsics,
                     appearance, neural)
    with torch.cuda.device(device):
        counts_t = torch.tensor(counts, dtype=torch.int64, device=device)
        offsets = torch.zeros(S + 1, dtype=torch.int64, device=device)
        offsets[1:] = torch.cumsum(counts_t, 0)
        images = S * C
        sh = sh_degree is not None
        sh_args = tuple(appearance) if sh else (None,) * 5
        records, xy, sh_rows, radii = RaggedProjection.apply(
            means, quaternions, scales, opacities, view_matrices, intrinsics, *sh_args, offsets,
            max(counts) if counts else 0, sh_degree, width, height, float(near_plane),
            float(far_plane))
        P = C * total
        # per pair: scene, camera, surfel within the scene, image and appearance row
        scene = torch.repeat_interleave(torch.arange(S, device=device), C * counts_t)
        local = torch.arange(P, device=device) - C * offsets[scene]
        n_s = counts_t[scene].clamp_min(1)
        camera = local // n_s
        primitive = local % n_s
        image_ids = scene * C + camera
        if sh:
            rows, row_mode, row_ids = sh_rows, nat.ROWS_PER_RECORD, None
        else:
            rows = SurfelRows.apply(neural, *(t.reshape(total, k) for t, k in
                                              zip(appearance, SurfelRows.widths(neural))))
            row_mode, row_ids = nat.ROWS_EXPLICIT, (offsets[scene] + primitive).contiguous()
        chunk = Chunk(0, images, 0, True)
        chunk.record0, chunk.record_count = 0, P
        if P:
            chunk.point_list, chunk.ranges = bin_records(
                records, nat.RECORD_FLOATS, radii, image_ids.contiguous(), 1, images, width,
                height, rendering._bin_flags())
        else:
            tw, th = (width + 15) // 16, (height + 15) // 16
            chunk.point_list = torch.empty((0,), device=device, dtype=torch.int32)
            chunk.ranges = torch.zeros((images * tw * th, 2), device=device, dtype=torch.int32)
        outputs = Composite.apply(records, xy, rows, backgrounds.reshape(-1, 3), None, [chunk],
                                  row_mode, C, max(counts + [1]), images, width, height, neural,
                                  float(near_plane), float(far_plane), median_depth, None,
                                  row_ids)
        rgb, alpha, depth, normals, distortion = (
            plane.reshape(S, C, height, width, plane.shape[-1]) for plane in outputs[:5])
        meta = {
            "radii": radii,
            "projected_means": xy,
            "scene_ids": scene,
            "camera_ids": camera,
            "primitive_ids": primitive,
            "packed": False,
            "accumulated_depth": depth,
            "normals": normals,
            "distortion": distortion,
        }
        if median_depth:
            meta["median_depth"] = outputs[5].reshape(S, C, height, width, 1)
        return rgb, alpha, meta


def rasterize_gabors_ragged(means, quaternions, scales, opacities, colors, secondary_colors,
                            frequency_weights, frequency_magnitudes, phases, view_matrices,
                            intrinsics, width: int, height: int, *, counts,
                            backgrounds=None, near_plane: float = 0.2, far_plane: float = 100.0,
                            sh_degree: int | None = None, validate: bool = True,
                            median_depth: bool = False
                            ) -> tuple[torch.Tensor, torch.Tensor, dict[str, Any]]:
    """``rasterize_gabors`` over scenes of different sizes.

    Per-surfel inputs concatenated over the S scenes (``means [sum N_s, 3]`` and so on),
    ``counts`` the S surfel counts, cameras ``[S, C, 4, 4]`` / ``[S, C, 3, 3]``,
    backgrounds ``[S, C, 3]``.  Returns RGB ``[S, C, H, W, 3]``, alpha
    ``[S, C, H, W, 1]`` and metadata with flat pair arrays (radii, projected_means and
    scene/camera/primitive ids over the C * sum N_s pairs, scene by scene, camera-major).
    Images equal rendering each scene on its own.
    """
    return _render_ragged(means, quaternions, scales, opacities,
                          (colors, secondary_colors, frequency_weights, frequency_magnitudes,
                           phases), view_matrices, intrinsics, width, height, counts,
                          backgrounds, near_plane, far_plane, False, sh_degree, validate,
                          median_depth)


def rasterize_neural_gabors_ragged(means, quaternions, scales, opacities, input_weights,
                                   input_biases, output_weights, output_biases, view_matrices,
                                   intrinsics, width: int, height: int, *, counts,
                                   backgrounds=None, near_plane: float = 0.2,
                                   far_plane: float = 100.0, validate: bool = True,
                                   median_depth: bool = False
                                   ) -> tuple[torch.Tensor, torch.Tensor, dict[str, Any]]:
    """``rasterize_neural_gabors`` over scenes of different sizes (layout as
    ``rasterize_gabors_ragged``)."""
    return _render_ragged(means, quaternions, scales, opacities,
                          (input_weights, input_biases, output_weights, output_biases),
                          view_matrices, intrinsics, width, height, counts, backgrounds,
                          near_plane, far_plane, True, None, validate, median_depth)
