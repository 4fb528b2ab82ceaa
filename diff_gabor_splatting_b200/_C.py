"""The reference's native module interface, over the C ABI.

Same four functions, argument order, tensor layouts, return values and error type
(RuntimeError) as the pybind11 module ``gabor_splatting._C``
(src/gabor_splatting/csrc/bindings.cpp:6-10, rasterize.h:5-21):

    rasterize_forward(geometry[Q,17], appearance[P,18|57], opacities[P],
                      primitive_ids[Q] int64, image_ids[Q] int64, radii[Q] int32,
                      backgrounds[images,3], width, height, neural, near, far)
        -> [maps[images,H,W,9], point_list[I] int32, ranges[tiles,2] int32,
            state[images,H,W,3], contributors[images,H,W] int32]
    rasterize_backward(geometry, appearance, opacities, primitive_ids, backgrounds,
                       point_list, ranges, state, contributors, grad_maps,
                       width, height, neural, near, far)
        -> [grad_geometry, grad_appearance, grad_opacities, grad_backgrounds]
    evaluate_sh_forward(first, second, directions, degree) -> colors[B,C,N,6]
    evaluate_sh_backward(first, second, directions, grad_colors, degree) -> 3 grads

Records are repacked into the library's 80-byte rows (opacity folded in) by a
kernel; binning and compositing are the same kernels the public renderers use.
"""

from __future__ import annotations

import torch

from . import _native as nat
from .rendering import SHColors, _check_sh, _composite_flags, bin_records

TILE = 16


def _check_float(value, geometry):
    if not (value.is_cuda and value.dtype == torch.float32):
        raise RuntimeError("native rendering requires CUDA float32 tensors")
    if value.device != geometry.device or not value.is_contiguous():
        raise RuntimeError("native buffers must be contiguous on the geometry device")


def _check_buffers(geometry, appearance, opacities, primitive_ids, backgrounds, neural):
    """rasterize.cu:401-422."""
    for t in (geometry, appearance, opacities, backgrounds):
        _check_float(t, geometry)
    if geometry.dim() != 2 or geometry.shape[1] != 17:
        raise RuntimeError("invalid geometry shape")
    if geometry.shape[0] > 2**31 - 1:
        raise RuntimeError("too many projected primitives")
    if appearance.dim() != 2 or appearance.shape[1] != (57 if neural else 18):
        raise RuntimeError("invalid appearance shape")
    if opacities.dim() != 1 or opacities.shape[0] != appearance.shape[0]:
        raise RuntimeError("invalid opacity shape")
    if backgrounds.dim() != 2 or backgrounds.shape[1] != 3 or backgrounds.shape[0] == 0:
        raise RuntimeError("invalid backgrounds")
    if not (primitive_ids.device == geometry.device and primitive_ids.is_contiguous()
            and primitive_ids.dtype == torch.int64 and primitive_ids.dim() == 1
            and primitive_ids.shape[0] == geometry.shape[0]):
        raise RuntimeError("invalid primitive IDs")


def _pack(geometry, appearance, opacities, primitive_ids, neural):
    device = geometry.device
    stream = nat.stream_of(device)
    Q, A = geometry.shape[0], appearance.shape[0]
    records = torch.empty((Q, nat.RECORD_FLOATS), device=device, dtype=torch.float32)
    width = 57 if neural else 18
    rows = torch.empty((A, nat.NEURAL_ROW_FLOATS if neural else nat.CLASSIC_ROW_FLOATS),
                       device=device, dtype=torch.float32)
    nat.call("gs_pack_geometry", nat.ptr(geometry), nat.ptr(opacities), nat.ptr(primitive_ids),
             Q, opacities.shape[0], nat.ptr(records), stream)
    nat.call("gs_pack_rows", nat.ptr(appearance), A, width, nat.ptr(rows), stream)
    return records, rows


def rasterize_forward(geometry, appearance, opacities, primitive_ids, image_ids, radii,
                      backgrounds, width, height, neural, near_plane, far_plane):
    """Mirror of rasterizeForward (rasterize.cu:425-503)."""
    _check_buffers(geometry, appearance, opacities, primitive_ids, backgrounds, neural)
    if not (0 < width < 2**31 - 1 - TILE and 0 < height < 2**31 - 1 - TILE):
        raise RuntimeError("invalid image dimensions")
    if not (near_plane > 0 and far_plane > near_plane):
        raise RuntimeError("invalid clipping planes")
    if not (image_ids.device == geometry.device and image_ids.is_contiguous()
            and image_ids.dtype == torch.int64 and image_ids.dim() == 1
            and image_ids.shape[0] == geometry.shape[0]):
        raise RuntimeError("invalid image IDs")
    if not (radii.device == geometry.device and radii.is_contiguous()
            and radii.dtype == torch.int32 and radii.dim() == 1
            and radii.shape[0] == geometry.shape[0]):
        raise RuntimeError("invalid radii")
    device = geometry.device
    with torch.cuda.device(device):
        images = backgrounds.shape[0]
        records, rows = _pack(geometry, appearance, opacities, primitive_ids, neural)
        point_list, ranges = bin_records(records, nat.RECORD_FLOATS, radii, image_ids, 1, images,
                                         width, height)
        maps = torch.empty((images, height, width, 9), device=device, dtype=torch.float32)
        state = torch.empty((images, height, width, 3), device=device, dtype=torch.float32)
        contributors = torch.empty((images, height, width), device=device, dtype=torch.int32)
        nat.call("gs_composite_forward", nat.ptr(records), nat.ptr(rows), nat.ROWS_EXPLICIT,
                 nat.ptr(primitive_ids), 1, 1, records.shape[0], rows.shape[0],
                 nat.ptr(backgrounds), nat.ptr(point_list), nat.ptr(ranges), images, width,
                 height, int(neural), _composite_flags(), float(near_plane), float(far_plane),
                 nat.ptr(maps),
                 nat.ptr(state), nat.ptr(contributors), None, nat.stream_of(device))
    return [maps, point_list, ranges, state, contributors]


def rasterize_backward(geometry, appearance, opacities, primitive_ids, backgrounds, point_list,
                       ranges, state, contributors, grad_maps, width, height, neural, near_plane,
                       far_plane):
    """Mirror of rasterizeBackward (rasterize.cu:505-529)."""
    _check_buffers(geometry, appearance, opacities, primitive_ids, backgrounds, neural)
    _check_float(grad_maps, geometry)
    device = geometry.device
    with torch.cuda.device(device):
        stream = nat.stream_of(device)
        images = backgrounds.shape[0]
        records, rows = _pack(geometry, appearance, opacities, primitive_ids, neural)
        g_records = torch.zeros_like(records)
        g_rows = torch.zeros_like(rows)
        g_bg = torch.zeros_like(backgrounds)
        nat.call("gs_composite_backward", nat.ptr(records), nat.ptr(rows), nat.ROWS_EXPLICIT,
                 nat.ptr(primitive_ids), 1, 1, records.shape[0], rows.shape[0],
                 nat.ptr(backgrounds), nat.ptr(point_list), nat.ptr(ranges), nat.ptr(state),
                 nat.ptr(contributors), nat.ptr(grad_maps), images, width, height, int(neural),
                 float(near_plane), float(far_plane), nat.ptr(g_records), None,
                 nat.ptr(g_rows), nat.ptr(g_bg), None, stream)
        gg = torch.empty_like(geometry)
        go = torch.empty_like(opacities)
        ga = torch.empty_like(appearance)
        if records.shape[0] == 0:
            gg.zero_()
        nat.call("gs_unpack_geometry_grads", nat.ptr(g_records), nat.ptr(primitive_ids),
                 geometry.shape[0], opacities.shape[0], nat.ptr(gg), nat.ptr(go), stream)
        nat.call("gs_unpack_rows", nat.ptr(g_rows), rows.shape[0], 57 if neural else 18,
                 nat.ptr(ga), stream)
    return [gg, ga, go, g_bg]


def evaluate_sh_forward(first, second, directions, degree):
    """Mirror of evaluateSHForward (spherical_harmonics.cu:106-126)."""
    _check_sh(first, second, directions, degree)
    with torch.no_grad():
        return SHColors.forward(_Ctx(), first, second, directions, degree)


def evaluate_sh_backward(first, second, directions, grad_colors, degree):
    """Mirror of evaluateSHBackward (spherical_harmonics.cu:128-150)."""
    _check_sh(first, second, directions, degree)
    if not (grad_colors.device == first.device and grad_colors.dtype == torch.float32
            and grad_colors.is_contiguous()
            and tuple(grad_colors.shape) == tuple(directions.shape[:3]) + (6,)):
        raise RuntimeError("invalid SH color gradients")
    B, C, N = directions.shape[:3]
    gf, gs, gd = (torch.zeros_like(first), torch.zeros_like(second),
                  torch.zeros_like(directions))
    with torch.cuda.device(first.device):
        nat.call("gs_sh_backward", nat.ptr(first), nat.ptr(second), nat.ptr(directions),
                 nat.ptr(grad_colors), degree, B, C, N, nat.ptr(gf), nat.ptr(gs), nat.ptr(gd),
                 nat.stream_of(first.device))
    return [gf, gs, gd]


class _Ctx:
    """Minimal stand-in for an autograd context when calling SHColors.forward directly."""

    def save_for_backward(self, *tensors):
        self.saved = tensors
