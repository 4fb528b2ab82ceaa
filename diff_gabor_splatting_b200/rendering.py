"""Public renderers with the reference's contracts, over the sm_100a kernels.

Mirrors ``gabor_splatting.rendering`` of luisrodolfo10/diff_gabor_splatting v0.1.1
(src/gabor_splatting/rendering.py): the same two public functions with the same
signatures, defaults, validation messages, outputs and metadata, and the same
module-level names tests reach into (``check_tensor``, ``check_values``,
``SHColors``).  What changes is underneath: projection, SH colours and record
packing run as one fused kernel (``gs_project_forward``) with a hand-derived
reverse kernel instead of ~30 PyTorch ops and their autograd graph; binning and
compositing run in libgabor_b200.so.  There is no CPU fallback: inputs must be
CUDA float32, exactly as in the reference.
"""

from __future__ import annotations

import ctypes
import math
from typing import Any

import torch
from torch.autograd.function import once_differentiable

from . import _native as nat

TILE = 16

# Work accounting for benchmarks: when WORK is a dict, the next renders record their
# record and intersection counts and the compositors' sample/accept counters in it.
WORK = None


def _counters(stage: str, device) -> torch.Tensor | None:
    if WORK is None:
        return None
    t = torch.zeros(2, dtype=torch.int64, device=device)
    WORK.setdefault("_counters", []).append((stage, t))
    return t


# ----------------------------------------------------------------------------------
# autograd bridges
# ----------------------------------------------------------------------------------
class Projection(torch.autograd.Function):
    """Fused splat setup (rendering.py:156-218, 334-374) and its reverse kernel.

    Returns per-pair records [P, 20], conic centres [P, 2], per-pair appearance rows
    [P, 20] (SH mode; empty otherwise) and int32 radii [P] (not differentiable).
    """

    @staticmethod
    def forward(ctx, means, quaternions, scales, opacities, view_matrices, intrinsics,
                sh_first, sh_second, frequency_weights, frequency_magnitudes, phases,
                sh_degree, width, height, near_plane, far_plane):
        S, N = means.shape[0], means.shape[1]
        C = view_matrices.shape[1]
        P = S * C * N
        device = means.device
        records = torch.empty((P, nat.RECORD_FLOATS), device=device, dtype=torch.float32)
        xy = torch.empty((P, 2), device=device, dtype=torch.float32)
        radii = torch.empty((P,), device=device, dtype=torch.int32)
        sh = sh_degree is not None
        rows = torch.empty((P if sh else 0, nat.CLASSIC_ROW_FLOATS), device=device,
                           dtype=torch.float32)
        nat.call("gs_project_forward", nat.ptr(means), nat.ptr(quaternions), nat.ptr(scales),
                 nat.ptr(opacities), nat.ptr(view_matrices), nat.ptr(intrinsics),
                 nat.ptr(sh_first), nat.ptr(sh_second), nat.ptr(frequency_weights),
                 nat.ptr(frequency_magnitudes), nat.ptr(phases),
                 -1 if sh_degree is None else sh_degree, S, C, N, width, height,
                 near_plane, far_plane, nat.ptr(records), nat.ptr(xy), nat.ptr(rows),
                 nat.ptr(radii), nat.stream_of(device))
        ctx.save_for_backward(means, quaternions, scales, view_matrices, intrinsics,
                              sh_first, sh_second)
        ctx.sh_degree = sh_degree
        ctx.mark_non_differentiable(radii)
        return records, xy, rows, radii

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_records, grad_xy, grad_rows, _grad_radii):
        means, quaternions, scales, view_matrices, intrinsics, sh_first, sh_second = \
            ctx.saved_tensors
        S, N = means.shape[0], means.shape[1]
        C = view_matrices.shape[1]
        P = S * C * N
        device = means.device
        sh = ctx.sh_degree is not None
        zeros = (lambda *shape: torch.zeros(shape, device=device, dtype=torch.float32))
        if grad_records is None:
            grad_records = zeros(P, nat.RECORD_FLOATS)
        if grad_xy is None:
            grad_xy = zeros(P, 2)
        if sh and grad_rows is None:
            grad_rows = zeros(P, nat.CLASSIC_ROW_FLOATS)
        grad_records, grad_xy = grad_records.contiguous(), grad_xy.contiguous()
        if grad_rows is not None:
            grad_rows = grad_rows.contiguous()
        g_means = torch.empty_like(means)
        g_quats = torch.empty_like(quaternions)
        g_scales = torch.empty_like(scales)
        g_opac = torch.empty((S, N), device=device, dtype=torch.float32)
        g_views = torch.empty_like(view_matrices)
        g_intr = torch.empty_like(intrinsics)
        g_sh1 = torch.empty_like(sh_first) if sh else None
        g_sh2 = torch.empty_like(sh_second) if sh else None
        g_w = torch.empty((S, N, 4), device=device) if sh else None
        g_m = torch.empty((S, N, 4), device=device) if sh else None
        g_p = torch.empty((S, N, 4), device=device) if sh else None
        nat.call("gs_project_backward", nat.ptr(means), nat.ptr(quaternions), nat.ptr(scales),
                 nat.ptr(view_matrices), nat.ptr(intrinsics), nat.ptr(sh_first),
                 nat.ptr(sh_second), -1 if ctx.sh_degree is None else ctx.sh_degree, S, C, N,
                 nat.ptr(grad_records), nat.ptr(grad_xy), nat.ptr(grad_rows), nat.ptr(g_means),
                 nat.ptr(g_quats), nat.ptr(g_scales), nat.ptr(g_opac), nat.ptr(g_views),
                 nat.ptr(g_intr), nat.ptr(g_sh1), nat.ptr(g_sh2), nat.ptr(g_w), nat.ptr(g_m),
                 nat.ptr(g_p), nat.stream_of(device))
        if N == 0:
            g_means.zero_(), g_quats.zero_(), g_scales.zero_(), g_opac.zero_()
            if sh:
                g_w.zero_(), g_m.zero_(), g_p.zero_()
        return (g_means, g_quats, g_scales, g_opac, g_views, g_intr, g_sh1, g_sh2, g_w, g_m,
                g_p, None, None, None, None, None)


class PackedRows(torch.autograd.Function):
    """``values[selected]`` for the packed metadata, whose backward scatters into zeros.

    ``selected`` holds distinct, increasing pair indices, so the adjoint is a plain
    scatter (``index_copy_``); autograd's generic indexing backward would sort the
    indices and accumulate (about 2.5 ms per call for a 10M-pair batch).
    """

    @staticmethod
    def forward(ctx, values, selected):
        ctx.save_for_backward(selected)
        ctx.rows = values.shape[0]
        return values.index_select(0, selected)

    @staticmethod
    @once_differentiable
    def backward(ctx, grad):
        (selected,) = ctx.saved_tensors
        out = grad.new_zeros((ctx.rows,) + tuple(grad.shape[1:]))
        return out.index_copy_(0, selected, grad.contiguous()), None


class SurfelRows(torch.autograd.Function):
    """Per-surfel appearance rows of the renderers without SH: the reference concatenates
    the appearance tensors (rendering.py:347-356); here one kernel packs them into the
    library's padded 20- / 60-float rows (``gs_pack_surfel_rows``) and one kernel writes
    the rows' gradients back as contiguous per-tensor gradients
    (``gs_unpack_surfel_rows``).  Inputs are contiguous [A, k] views.
    """

    @staticmethod
    def widths(neural):
        """Floats per surfel of each appearance tensor, in row order."""
        return (30, 6, 18, 3) if neural else (3, 3, 4, 4, 4)

    @staticmethod
    def forward(ctx, neural, *appearance):
        device = appearance[0].device
        count = appearance[0].shape[0]
        width = nat.NEURAL_ROW_FLOATS if neural else nat.CLASSIC_ROW_FLOATS
        rows = torch.empty((count, width), device=device, dtype=torch.float32)
        inputs, inputs_ptr = nat.host_array(ctypes.c_void_p, [t.data_ptr() for t in appearance])
        nat.call("gs_pack_surfel_rows", int(neural), inputs_ptr, count, nat.ptr(rows),
                 nat.stream_of(device))
        ctx.neural = neural
        ctx.shapes = [t.shape for t in appearance]
        return rows

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_rows):
        grad_rows = grad_rows.contiguous()
        grads = [grad_rows.new_empty(shape) for shape in ctx.shapes]
        outs, outs_ptr = nat.host_array(ctypes.c_void_p, [g.data_ptr() for g in grads])
        nat.call("gs_unpack_surfel_rows", int(ctx.neural), nat.ptr(grad_rows), grad_rows.shape[0],
                 outs_ptr, nat.stream_of(grad_rows.device))
        return (None, *grads)


# channels of the five map planes the compositor writes: rgb, alpha, accumulated depth,
# normals, distortion (together the reference's [..][9] maps, in that order)
PLANES = (3, 1, 1, 3, 1)


class Selection:
    """Selected pixels of every image, grouped for the compositor's selected-pixel mode.

    ``pixels`` [images, P, 2] integer (x, y) inside the image.  Pixels are sorted
    (stably) by tile and cut into groups of at most 256 pixels of one tile; the kernels
    write each pixel's outputs at its original index image * P + p.
    """

    def __init__(self, pixels: torch.Tensor, width: int, height: int):
        images, count = pixels.shape[0], pixels.shape[1]
        device = pixels.device
        self.count = count
        self.tw, self.th = (width + TILE - 1) // TILE, (height + TILE - 1) // TILE
        tiles_per_image = self.tw * self.th
        x = pixels[..., 0].reshape(-1).long()
        y = pixels[..., 1].reshape(-1).long()
        image = torch.arange(images, device=device).repeat_interleave(count)
        tile = image * tiles_per_image + (y // TILE) * self.tw + x // TILE
        order = torch.argsort(tile, stable=True)
        ordered_tiles = tile[order]
        n = ordered_tiles.numel()
        index = torch.arange(n, device=device)
        run_start = torch.ones(n, dtype=torch.bool, device=device)
        run_start[1:] = ordered_tiles[1:] != ordered_tiles[:-1]
        first_of_run = torch.cummax(torch.where(run_start, index, torch.zeros_like(index)), 0)[0]
        new_group = run_start | ((index - first_of_run) % (TILE * TILE) == 0)
        firsts = torch.nonzero(new_group).reshape(-1)
        counts = torch.diff(firsts, append=torch.tensor([n], device=device))
        self.tiles_per_image = tiles_per_image
        self.group_tile = ordered_tiles[firsts]
        self.group_first = firsts
        self.group_count = counts
        self.sel_xy = torch.stack((x[order], y[order]), -1)
        self.sel_index = order

    def for_images(self, image0: int, images: int):
        """(selected int32 [n, 4], groups int32 [g, 4]) for images [image0, image0 + images),
        with chunk-local tiles and output indices."""
        low, high = image0 * self.tiles_per_image, (image0 + images) * self.tiles_per_image
        keep = (self.group_tile >= low) & (self.group_tile < high)
        groups = torch.stack((self.group_tile[keep] - low, self.group_first[keep],
                              self.group_count[keep], torch.zeros_like(self.group_first[keep])),
                             -1).to(torch.int32).contiguous()
        selected = torch.cat((self.sel_xy, (self.sel_index - image0 * self.count)[:, None],
                              torch.zeros_like(self.sel_index)[:, None]), -1)
        return selected.to(torch.int32).contiguous(), groups


class Composite(torch.autograd.Function):
    """Tile compositor forward/backward (rasterize.cu:229-399) over binned records.

    ``chunks`` is the list of image chunks from ``bin_chunks``; each is composited
    with its own point list and ranges, and the backward adds every chunk into the
    same gradient buffers.  ``projected_means`` receives the screen-centre gradient
    (record slots 9-10), so it can be inspected with ``retain_grad`` like the
    reference's.  The maps come out as the five planes of ``PLANES`` (the reference
    slices one [..][9] array into the same five outputs): each output's gradient goes
    to the kernel as autograd delivers it -- broadcast, strided or absent -- with no
    [..][9] gradient assembled.  With a ``Selection`` only the selected pixels are
    composited and every per-pixel output is [images, P, ...].
    """

    @staticmethod
    def forward(ctx, records, projected_means, rows, backgrounds, selected, chunks, row_mode,
                cameras, surfels, images, width, height, neural, near_plane, far_plane,
                median=False, selection=None, row_ids=None):
        device = records.device
        pixel_shape = (height, width) if selection is None else (selection.count,)
        per_image = math.prod(pixel_shape)
        planes = [torch.empty((images,) + pixel_shape + (k,), device=device, dtype=torch.float32)
                  for k in PLANES]
        # optional median depth plane and the 1-based list position it came from
        median_depth = torch.empty((images,) + pixel_shape + (1,) if median else (0,),
                                   device=device, dtype=torch.float32)
        median_index = torch.empty((images,) + pixel_shape if median else (0,), device=device,
                                   dtype=torch.int32)
        state = torch.empty((images,) + pixel_shape + (3,), device=device, dtype=torch.float32)
        contributors = torch.empty((images,) + pixel_shape, device=device, dtype=torch.int32)
        stream = nat.stream_of(device)
        strides, strides_ptr = nat.host_array(ctypes.c_int64, PLANES)
        chunk_selection, chunk_masks = [], []
        for ch in chunks:
            a = _chunk_args(ch, records, rows, row_mode, cameras, surfels, width, height)
            pixel0 = ch.image0 * per_image
            sel = selection.for_images(ch.image0, ch.images) if selection is not None else None
            chunk_selection.append(sel)
            masks = _warp_masks(ch, device)
            chunk_masks.append(masks)
            outs, outs_ptr = nat.host_array(
                ctypes.c_void_p, [_at(t, pixel0 * k) for t, k in zip(planes, PLANES)])
            nat.call("gs_composite_forward_split", a["records"], a["rows"], row_mode,
                     _at(row_ids, ch.record0),
                     a["cameras"], surfels, ch.record_count, a["rows_count"],
                     _at(backgrounds, ch.image0 * 3), nat.ptr(ch.point_list),
                     nat.ptr(ch.ranges), ch.images, width, height, int(neural),
                     _composite_flags(), near_plane, far_plane, outs_ptr, strides_ptr,
                     _at(median_depth, pixel0), 1, _at(median_index, pixel0),
                     None if sel is None else nat.ptr(sel[0]),
                     None if sel is None else nat.ptr(sel[1]),
                     0 if sel is None else sel[1].shape[0],
                     _at(state, pixel0 * 3), _at(contributors, pixel0),
                     None if masks is None else nat.ptr(masks),
                     0 if masks is None else masks.shape[1],
                     nat.ptr(_counters("forward", device)), stream)
        ctx.save_for_backward(records, rows, backgrounds, selected, state, contributors,
                              median_index)
        ctx.set_materialize_grads(False)   # an unused output's gradient stays None (zero)
        ctx.chunks = chunks
        ctx.row_ids = row_ids
        ctx.chunk_selection = chunk_selection
        ctx.chunk_masks = chunk_masks
        ctx.pixel_shape = pixel_shape
        ctx.options = (row_mode, cameras, surfels, images, width, height, neural, near_plane,
                       far_plane)
        return tuple(planes) + (median_depth,)

    @staticmethod
    @once_differentiable
    def backward(ctx, *grad_outputs):
        records, rows, backgrounds, selected, state, contributors, median_index = \
            ctx.saved_tensors
        grad_planes, grad_median = grad_outputs[:5], grad_outputs[5]
        if median_index.numel() == 0:
            grad_median = None
        row_mode, cameras, surfels, images, width, height, neural, near_plane, far_plane = \
            ctx.options
        device = records.device
        pixel_shape = ctx.pixel_shape
        per_image = math.prod(pixel_shape)
        grads = [_pixel_linear(g, pixel_shape) for g in grad_planes]
        g_median, median_px, _ = _pixel_linear(grad_median, pixel_shape)
        g_records = torch.zeros_like(records)
        g_xy = torch.zeros((records.shape[0], 2), device=device, dtype=torch.float32)
        g_rows = torch.zeros_like(rows)
        g_bg = torch.zeros_like(backgrounds)
        stream = nat.stream_of(device)
        strides, strides_ptr = nat.host_array(
            ctypes.c_int64, [x for _, px, ch in grads for x in (px, ch)])
        for ch, sel, masks in zip(ctx.chunks, ctx.chunk_selection, ctx.chunk_masks):
            a = _chunk_args(ch, records, rows, row_mode, cameras, surfels, width, height)
            pixel0 = ch.image0 * per_image
            ins, ins_ptr = nat.host_array(
                ctypes.c_void_p, [None if g is None else g.data_ptr() + pixel0 * px * 4
                                  for g, px, _ in grads])
            nat.call("gs_composite_backward_split", a["records"], a["rows"], row_mode,
                     _at(ctx.row_ids, ch.record0),
                     a["cameras"], surfels, ch.record_count, a["rows_count"],
                     _at(backgrounds, ch.image0 * 3), nat.ptr(ch.point_list),
                     nat.ptr(ch.ranges), _at(state, pixel0 * 3),
                     _at(contributors, pixel0), ins_ptr, strides_ptr,
                     _at(median_index, pixel0) if g_median is not None else None,
                     None if g_median is None else g_median.data_ptr() + pixel0 * median_px * 4,
                     median_px, None if sel is None else nat.ptr(sel[0]),
                     None if sel is None else nat.ptr(sel[1]),
                     0 if sel is None else sel[1].shape[0], ch.images, width, height,
                     int(neural), near_plane, far_plane,
                     _at(g_records, ch.record0 * nat.RECORD_FLOATS), _at(g_xy, ch.record0 * 2),
                     _at(g_rows, a["row0"] * rows.shape[1]), _at(g_bg, ch.image0 * 3),
                     None if masks is None else nat.ptr(masks),
                     0 if masks is None else masks.shape[1],
                     nat.ptr(_counters("backward", device)), stream)
        g_pm = g_xy if selected is None else g_xy.index_select(0, selected)
        return (g_records, g_pm, g_rows, g_bg) + (None,) * 14


def _pixel_linear(g, pixel_shape):
    """(tensor, pixel stride, channel stride) of a per-pixel gradient [images, *pixel_shape, k].

    The kernel reads element (pixel p, channel c) at p * pixel_stride + c * channel_stride,
    which fits a contiguous gradient and a broadcast one (all strides 0, as a mean's
    gradient arrives); any other layout is made contiguous first.  None stays None
    (a zero gradient).
    """
    if g is None:
        return None, 0, 0
    if g.dtype != torch.float32:
        g = g.float()
    k = g.shape[-1]
    dims = (g.shape[0],) + tuple(pixel_shape)
    strides = g.stride()
    px = strides[len(dims) - 1]
    fits, expect = True, px
    for size, stride in zip(reversed(dims), reversed(strides[:len(dims)])):
        if size != 1 and stride != expect:
            fits = False
            break
        expect = expect * size
    ch = strides[-1]
    if not fits:
        g = g.contiguous()
        px, ch = k, 1
    return g, px, (ch if k > 1 else 0)


def _at(t: torch.Tensor, offset: int) -> int | None:
    """Device address of element ``offset`` of a contiguous tensor."""
    if t is None or t.numel() == 0:
        return None
    return t.data_ptr() + offset * t.element_size()


def _chunk_args(ch, records, rows, row_mode, cameras, surfels, width, height):
    """Pointers and appearance-row addressing of one image chunk.

    Chunks are either whole scenes or a camera range of one scene, so with rows
    addressed per surfel the chunk's rows start at its first scene and the per-chunk
    camera count keeps the kernel's record -> row arithmetic local.
    """
    if row_mode == nat.ROWS_PER_SURFEL:
        row0 = (ch.image0 // cameras) * surfels
        cams = cameras if ch.whole_scenes else ch.images
        rows_count = (ch.images // cameras if ch.whole_scenes else 1) * surfels
    else:
        row0, cams, rows_count = ch.record0, cameras, ch.record_count
    return dict(records=_at(records, ch.record0 * nat.RECORD_FLOATS),
                rows=_at(rows, row0 * rows.shape[1]), cameras=cams, rows_count=rows_count,
                row0=row0, pixel0=ch.image0 * height * width)


# Appearance evaluation in the forward compositor: False (default) uses the SFU forms
# (images within 1e-6 of exact), True the reference's full-precision cosf/sinf/expf
# (images bit-identical to the reference's).
EXACT_APPEARANCE = False


def _composite_flags() -> int:
    return nat.COMPOSITE_EXACT if EXACT_APPEARANCE else 0


# The public renderers bin tightly: tiles that no sample of a record can reach with
# alpha >= 1/255 are dropped (identical images, shorter lists).  False restores the
# reference's square 3-sigma bins.
TIGHT_BINNING = True


def _bin_flags() -> int:
    return nat.BIN_TIGHT if TIGHT_BINNING else 0


# Warp accept masks: the forward records, per tile-list entry and warp of its tile
# CTA, whether any pixel of the warp accepted the entry, and the backward skips the
# entries its warp accepted nowhere (same images and gradients).  They pay when splats
# are small against a tile (few tiles per record: most entries reach few of a tile's
# 8x4-pixel warp blocks) and cost the forward's bookkeeping otherwise.  "auto" uses them
# below MASK_TILES_PER_RECORD tile intersections per record; True / False force them.
WARP_MASKS = "auto"
MASK_TILES_PER_RECORD = 8.0


def _warp_masks(ch, device):
    """Zeroed accept masks for one binned chunk of I list entries (8 planes of
    I // 32 + 2 words, at least one word per 32 positions), or None when this chunk
    does without."""
    entries = ch.point_list.shape[0]
    use = WARP_MASKS is True or (WARP_MASKS == "auto" and ARENA is None and
                                 entries < MASK_TILES_PER_RECORD * max(ch.record_count, 1))
    if not use or entries == 0:
        return None
    if WORK is not None:   # work accounting: the backward's tests count executed ones
        WORK["masked_intersections"] = WORK.get("masked_intersections", 0) + entries
    words = entries // 32 + 2
    return torch.zeros((8, words), device=device, dtype=torch.int32)


# Largest number of tile intersections binned in one pass.  Larger batches are split
# into image chunks (whole scenes, or camera ranges of one scene), each binned and
# composited on its own; this bounds the sort workspace (~20 bytes per intersection)
# and keeps indices within int32.
MAX_CHUNK_INTERSECTIONS = 1 << 30
GS_ERR_LIMIT = 2
INT32_MAX = 2**31 - 1


class Chunk:
    """One image chunk: images [image0, image0 + images), records likewise."""

    def __init__(self, image0, images, surfels, whole_scenes):
        self.image0, self.images, self.whole_scenes = image0, images, whole_scenes
        self.record0, self.record_count = image0 * surfels, images * surfels
        self.point_list = self.ranges = None


def _count(records, radii, R, per_image, images, width, height):
    """gs_bin_count on a record range (``_Ptr`` addresses); returns (workspace, bytes,
    intersections); the count is returned even when it exceeds int32."""
    device = records.device
    bytes1 = ctypes.c_size_t()
    nat.call("gs_bin_count_workspace", R, ctypes.byref(bytes1))
    ws1 = torch.empty((max(bytes1.value, 1),), device=device, dtype=torch.uint8)
    total, spans = ctypes.c_int64(), ctypes.c_int64()
    status = nat.call_status("gs_bin_count", records.address, nat.RECORD_FLOATS, radii.address,
                             None, R, per_image, images, width, height, _bin_flags(),
                             nat.ptr(ws1), bytes1.value, ctypes.byref(total), ctypes.byref(spans),
                             nat.stream_of(device))
    if status not in (0, GS_ERR_LIMIT) or (status == GS_ERR_LIMIT and total.value <= INT32_MAX):
        nat.check(status, "gs_bin_count")
    return ws1, bytes1.value, total.value, spans.value


def _bin_chunk(ch, records, radii, surfels, width, height, counted=None):
    """Sort one chunk's (record, tile) slots; ``counted`` reuses a finished count."""
    device = records.device
    rec = _at(records, ch.record0 * nat.RECORD_FLOATS)
    rad = _at(radii, ch.record0)
    if counted is None:
        counted = _count(_Ptr(rec, device), _Ptr(rad, device), ch.record_count, surfels,
                         ch.images, width, height)
    ws1, bytes1, total, spans = counted
    tw, th = (width + TILE - 1) // TILE, (height + TILE - 1) // TILE
    bytes2 = ctypes.c_size_t()
    nat.call("gs_bin_sort_workspace", ch.record_count, total, spans, ch.images, width, height,
             ctypes.byref(bytes2))
    ws2 = torch.empty((max(bytes2.value, 1),), device=device, dtype=torch.uint8)
    ch.point_list = torch.empty((total,), device=device, dtype=torch.int32)
    ch.ranges = torch.empty((ch.images * tw * th, 2), device=device, dtype=torch.int32)
    nat.call("gs_bin_sort", rec, nat.RECORD_FLOATS, rad, None, ch.record_count, surfels,
             ch.images, width, height, _bin_flags(), nat.ptr(ws1), bytes1, nat.ptr(ws2),
             bytes2.value, total, spans,
             nat.ptr(ch.point_list), nat.ptr(ch.ranges), nat.stream_of(device))
    if WORK is not None:
        WORK["records"] = WORK.get("records", 0) + ch.record_count
        WORK["intersections"] = WORK.get("intersections", 0) + total
        WORK["spans"] = WORK.get("spans", 0) + spans
        WORK["tiles"] = WORK.get("tiles", 0) + ch.images * tw * th
        # intersections x 8-bit radix passes of the tile-id sort
        passes = -(-max(1, (ch.images * tw * th - 1).bit_length()) // 8)
        WORK["sort_passes"] = WORK.get("sort_passes", 0) + total * passes
    return ch


class _Ptr:
    """A raw device address standing in for a tensor argument of ``_count``."""

    def __init__(self, address, device):
        self.address, self.device = address, device


class Arena:
    """Capacities for binning without a host synchronisation (``gs_bin_arena``).

    While installed as ``rendering.ARENA`` every render bins all its images in one
    arena of ``max_intersections`` (record, tile) slots and ``max_spans`` row spans,
    with no host read of the counts, so render steps can be captured in CUDA graphs.
    ``totals`` (device int64[2]) holds the live counts of the latest binning; when they
    exceed the capacities that binning produced empty tile lists (background only):
    check with ``overflowed()`` (one host read) and grow the arena.
    """

    def __init__(self, max_intersections: int, max_spans: int, device=None):
        if not (1 <= max_spans <= max_intersections <= INT32_MAX):
            raise ValueError("arena capacities must satisfy 1 <= max_spans <= "
                             "max_intersections <= 2^31 - 1")
        self.max_intersections, self.max_spans = int(max_intersections), int(max_spans)
        self.totals = torch.zeros(2, dtype=torch.int64,
                                  device=device if device is not None else "cuda")

    def overflowed(self) -> bool:
        live = self.totals.tolist()
        return live[0] > self.max_intersections or live[1] > self.max_spans

    def overflow_flag(self) -> torch.Tensor:
        """Device int32 scalar, 1 when the latest binning exceeded the capacities
        (computed on the device: no host read, so it can be recorded in a graph)."""
        over = (self.totals[0] > self.max_intersections) | (self.totals[1] > self.max_spans)
        return over.to(torch.int32).reshape(1)

    def needed(self) -> tuple[int, int]:
        """Live (intersections, spans) of the latest binning (one host read)."""
        return tuple(self.totals.tolist())


ARENA = None


def _bin_arena(arena, records, radii, images, surfels, width, height):
    device = records.device
    tw, th = (width + TILE - 1) // TILE, (height + TILE - 1) // TILE
    whole = Chunk(0, images, surfels, True)
    R = whole.record_count
    nbytes = ctypes.c_size_t()
    nat.call("gs_bin_arena_workspace", R, arena.max_intersections, arena.max_spans, images,
             width, height, ctypes.byref(nbytes))
    workspace = torch.empty((max(nbytes.value, 1),), device=device, dtype=torch.uint8)
    whole.point_list = torch.empty((arena.max_intersections,), device=device, dtype=torch.int32)
    whole.ranges = torch.empty((images * tw * th, 2), device=device, dtype=torch.int32)
    nat.call("gs_bin_arena", nat.ptr(records), nat.RECORD_FLOATS, nat.ptr(radii), None, R,
             surfels, images, width, height, _bin_flags(), nat.ptr(workspace), nbytes.value,
             arena.max_intersections, arena.max_spans, nat.ptr(whole.point_list),
             nat.ptr(whole.ranges), nat.ptr(arena.totals), nat.stream_of(device))
    return [whole]


def bin_chunks(records, radii, scenes, cameras, surfels, width, height):
    """Bin the dense records of S scenes x C cameras x N surfels in image chunks (one
    arena-binned chunk when ``ARENA`` is set)."""
    device = records.device
    images = scenes * cameras
    if ARENA is not None and records.shape[0] > 0:
        return _bin_arena(ARENA, records, radii, images, surfels, width, height)
    whole = Chunk(0, images, surfels, True)
    if records.shape[0] == 0:
        whole.record_count = 0
        whole.point_list = torch.empty((0,), device=device, dtype=torch.int32)
        tw, th = (width + TILE - 1) // TILE, (height + TILE - 1) // TILE
        whole.ranges = torch.zeros((images * tw * th, 2), device=device, dtype=torch.int32)
        return [whole]

    def count_of(image0, count):
        rec = _Ptr(_at(records, image0 * surfels * nat.RECORD_FLOATS), device)
        rad = _Ptr(_at(radii, image0 * surfels), device)
        return _count(rec, rad, count * surfels, surfels, count, width, height)

    counted = count_of(0, images)
    if counted[2] <= MAX_CHUNK_INTERSECTIONS:
        return [_bin_chunk(whole, records, radii, surfels, width, height, counted)]
    del counted
    chunks, group, group_total = [], [], 0

    def flush():
        nonlocal group, group_total
        if group:
            chunks.append(Chunk(group[0] * cameras, len(group) * cameras, surfels, True))
        group, group_total = [], 0

    for s in range(scenes):
        total = count_of(s * cameras, cameras)[2]
        if total > MAX_CHUNK_INTERSECTIONS:
            flush()
            pending = [(s * cameras, cameras)]
            while pending:   # split the scene's cameras until each range fits
                image0, count = pending.pop(0)
                if count > 1 and count_of(image0, count)[2] > MAX_CHUNK_INTERSECTIONS:
                    half = count // 2
                    pending[:0] = [(image0, half), (image0 + half, count - half)]
                else:
                    chunks.append(Chunk(image0, count, surfels, count == cameras))
        elif group_total + total > MAX_CHUNK_INTERSECTIONS:
            flush()
            group, group_total = [s], total
        else:
            group.append(s)
            group_total += total
    flush()
    return [_bin_chunk(ch, records, radii, surfels, width, height) for ch in chunks]


def bin_records(records, record_stride, radii, image_ids, records_per_image, images, width,
                height, flags=0):
    """Depth-ordered per-tile record lists (rasterize.cu:454-493): point_list, ranges.

    One pass (no chunking): used by the reference-layout entry points and the tests.
    flags=0 gives the reference's bins exactly; nat.BIN_TIGHT drops unreachable tiles.
    """
    device = records.device
    stream = nat.stream_of(device)
    R = records.shape[0]
    tw, th = (width + TILE - 1) // TILE, (height + TILE - 1) // TILE
    bytes1 = ctypes.c_size_t()
    nat.call("gs_bin_count_workspace", R, ctypes.byref(bytes1))
    ws1 = torch.empty((max(bytes1.value, 1),), device=device, dtype=torch.uint8)
    total, spans = ctypes.c_int64(), ctypes.c_int64()
    nat.call("gs_bin_count", nat.ptr(records), record_stride, nat.ptr(radii), nat.ptr(image_ids),
             R, records_per_image, images, width, height, flags, nat.ptr(ws1), bytes1.value,
             ctypes.byref(total), ctypes.byref(spans), stream)
    intersections = total.value
    bytes2 = ctypes.c_size_t()
    nat.call("gs_bin_sort_workspace", R, intersections, spans.value, images, width, height,
             ctypes.byref(bytes2))
    ws2 = torch.empty((max(bytes2.value, 1),), device=device, dtype=torch.uint8)
    point_list = torch.empty((intersections,), device=device, dtype=torch.int32)
    ranges = torch.empty((images * tw * th, 2), device=device, dtype=torch.int32)
    nat.call("gs_bin_sort", nat.ptr(records), record_stride, nat.ptr(radii), nat.ptr(image_ids),
             R, records_per_image, images, width, height, flags, nat.ptr(ws1), bytes1.value,
             nat.ptr(ws2), bytes2.value, intersections, spans.value, nat.ptr(point_list),
             nat.ptr(ranges), stream)
    return point_list, ranges


# ----------------------------------------------------------------------------------
# contracts (rendering.py:74-153)
# ----------------------------------------------------------------------------------
def check_tensor(name: str, value: torch.Tensor, shape: tuple[int, ...],
                 device: torch.device) -> None:
    """Require a contiguous float32 CUDA tensor with an exact shape and device."""
    if not isinstance(value, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if value.device != device or value.dtype != torch.float32 or not value.is_cuda:
        raise ValueError(f"{name} must be float32 on {device}")
    if value.shape != shape:
        raise ValueError(f"{name} must have shape {shape}, got {tuple(value.shape)}")
    if not value.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


@torch.no_grad()
def check_values(tensors, quaternions, scales, opacities, view_matrices, intrinsics,
                 appearance, neural):
    """Validate the numerical contracts with one synchronisation (rendering.py:88-153).

    Raises ValueError naming every violated contract, joined by "; ", in the
    reference's order and wording.
    """
    checks = [(f"{name} must contain only finite values", torch.isfinite(t).all())
              for name, (t, _) in tensors.items()]
    eye = torch.eye(3, device=view_matrices.device, dtype=view_matrices.dtype)
    rotation = view_matrices[..., :3, :3]
    checks += [
        ("scales must be strictly positive", (scales > 0).all()),
        ("opacities must lie in [0, 1]", ((opacities >= 0) & (opacities <= 1)).all()),
        ("quaternions must be unit wxyz vectors",
         torch.isclose(quaternions.square().sum(-1), quaternions.new_tensor(1),
                       atol=1e-4, rtol=1e-4).all()),
        ("view_matrices must have last row [0, 0, 0, 1]",
         torch.isclose(view_matrices[..., 3, :], view_matrices.new_tensor([0, 0, 0, 1])).all()),
        ("intrinsics must have last row [0, 0, 1]",
         torch.isclose(intrinsics[..., 2, :], intrinsics.new_tensor([0, 0, 1])).all()),
        ("intrinsics fx and fy must be positive",
         ((intrinsics[..., 0, 0] > 0) & (intrinsics[..., 1, 1] > 0)).all()),
        ("view_matrices rotations must be orthonormal",
         torch.isclose(rotation.transpose(-1, -2) @ rotation, eye, atol=1e-4, rtol=1e-4).all()),
        ("view_matrices rotations must have determinant +1",
         torch.isclose(torch.linalg.det(rotation), rotation.new_tensor(1),
                       atol=1e-4, rtol=1e-4).all()),
    ]
    if not neural:
        weights, magnitudes = appearance[2], appearance[3]
        checks += [
            ("frequency_weights must be nonnegative", (weights >= 0).all()),
            ("frequency_magnitudes must be nonnegative", (magnitudes >= 0).all()),
            ("frequency_weights must sum to one",
             torch.isclose(weights.sum(-1), weights.new_tensor(1), atol=1e-4, rtol=1e-4).all()),
        ]
    passed = torch.stack([ok for _, ok in checks]).tolist()
    if not all(passed):
        raise ValueError("; ".join(message for (message, _), ok in zip(checks, passed) if not ok))


class SHColors(torch.autograd.Function):
    """Both SH colour sets per (scene, camera, surfel) pair (rendering.py:221-238).

    first/second [B, N, K, 3], directions [B, C, N, 3] -> colours [B, C, N, 6].
    """

    @staticmethod
    def forward(ctx, first, second, directions, degree):
        _check_sh(first, second, directions, degree)
        B, C, N = directions.shape[:3]
        colors = torch.empty((B, C, N, 6), device=first.device, dtype=torch.float32)
        nat.call("gs_sh_forward", nat.ptr(first), nat.ptr(second), nat.ptr(directions), degree,
                 B, C, N, nat.ptr(colors), nat.stream_of(first.device))
        ctx.save_for_backward(first, second, directions)
        ctx.degree = degree
        return colors

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_colors):
        first, second, directions = ctx.saved_tensors
        B, C, N = directions.shape[:3]
        grad_colors = grad_colors.contiguous()
        gf, gs, gd = (torch.zeros_like(first), torch.zeros_like(second),
                      torch.zeros_like(directions))
        nat.call("gs_sh_backward", nat.ptr(first), nat.ptr(second), nat.ptr(directions),
                 nat.ptr(grad_colors), ctx.degree, B, C, N, nat.ptr(gf), nat.ptr(gs),
                 nat.ptr(gd), nat.stream_of(first.device))
        return gf, gs, gd, None


def _check_sh(first, second, directions, degree):
    """Structural SH checks (spherical_harmonics.cu:88-103), raising RuntimeError."""
    if not (isinstance(degree, int) and 0 <= degree <= 3):
        raise RuntimeError("SH degree must be 0 through 3")
    for t in (first, second, directions):
        if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()
                and t.device == first.device):
            raise RuntimeError("SH tensors must be contiguous float32 on the same CUDA device")
    if not (first.dim() == 4 and second.shape == first.shape
            and first.shape[2] == (degree + 1) ** 2 and first.shape[3] == 3):
        raise RuntimeError("SH coefficients must have shape [B, N, K, 3]")
    if not (directions.dim() == 4 and directions.shape[0] == first.shape[0]
            and directions.shape[2] == first.shape[1] and directions.shape[3] == 3):
        raise RuntimeError("SH directions must have shape [B, C, N, 3]")


# ----------------------------------------------------------------------------------
# render (rendering.py:241-400)
# ----------------------------------------------------------------------------------
def render(means, quaternions, scales, opacities, appearance, view_matrices, intrinsics, width,
           height, backgrounds, packed, near_plane, far_plane, neural, sh_degree, validate,
           median_depth=False, pixels=None):
    """Validate inputs, project scene/camera pairs, bin, and composite in one call."""
    if not isinstance(means, torch.Tensor) or means.ndim < 2 or means.shape[-1] != 3:
        raise ValueError("means must have shape [..., N, 3]")
    if not means.is_cuda or means.dtype != torch.float32:
        raise ValueError("means must be a CUDA float32 tensor")
    if (type(width) is not int or type(height) is not int
            or not (0 < width < 2**30 and 0 < height < 2**30)):
        raise ValueError("width and height must be positive integers smaller than 2**30")
    if (not math.isfinite(near_plane) or not math.isfinite(far_plane)
            or not 0 < near_plane < far_plane):
        raise ValueError("clipping planes must be finite and satisfy 0 < near_plane < far_plane")
    if type(packed) is not bool:
        raise TypeError("packed must be bool")
    batch = tuple(means.shape[:-2])
    n = means.shape[-2]
    if not isinstance(view_matrices, torch.Tensor) or view_matrices.ndim != len(batch) + 3:
        raise ValueError("view_matrices must have shape [..., C, 4, 4]")
    cameras = view_matrices.shape[-3]
    scenes = math.prod(batch)
    if scenes < 1 or cameras < 1:
        raise ValueError("scene and camera dimensions must be nonempty")
    device = means.device
    tensors = {
        "means": (means, batch + (n, 3)),
        "quaternions": (quaternions, batch + (n, 4)),
        "scales": (scales, batch + (n, 2)),
        "opacities": (opacities, batch + (n,)),
        "view_matrices": (view_matrices, batch + (cameras, 4, 4)),
        "intrinsics": (intrinsics, batch + (cameras, 3, 3)),
    }
    if backgrounds is None:
        backgrounds = means.new_zeros(batch + (cameras, 3))
    tensors["backgrounds"] = backgrounds, batch + (cameras, 3)
    if neural:
        shapes = [(6, 5), (6,), (3, 6), (3,)]
        names = ["input_weights", "input_biases", "output_weights", "output_biases"]
    else:
        if sh_degree is not None and (type(sh_degree) is not int or not 0 <= sh_degree <= 3):
            raise ValueError("sh_degree must be None or an integer from 0 to 3")
        color_shape = (3,) if sh_degree is None else ((sh_degree + 1) ** 2, 3)
        shapes = [color_shape, color_shape, (4,), (4,), (4,)]
        names = ["colors", "secondary_colors", "frequency_weights", "frequency_magnitudes",
                 "phases"]
    for name, tensor, shape in zip(names, appearance, shapes):
        tensors[name] = tensor, batch + (n,) + shape
    for name, (tensor, shape) in tensors.items():
        check_tensor(name, tensor, shape, device)
    if type(median_depth) is not bool:
        raise TypeError("median_depth must be bool")
    if pixels is not None:
        if (not isinstance(pixels, torch.Tensor) or pixels.dtype not in (torch.int32, torch.int64)
                or pixels.device != device or pixels.ndim < 2 or pixels.shape[-1] != 2
                or tuple(pixels.shape[:-2]) != batch + (cameras,)):
            raise ValueError("pixels must be an integer tensor [..., C, P, 2] on the scene's "
                             "device")
        if pixels.numel() and bool(((pixels[..., 0] < 0) | (pixels[..., 0] >= width)
                                    | (pixels[..., 1] < 0) | (pixels[..., 1] >= height))
                                   .any()):
            raise ValueError("pixels must lie inside the image")
    if type(validate) is not bool:
        raise TypeError("validate must be bool")
    if validate:
        check_values(tensors, quaternions, scales, opacities, view_matrices, intrinsics,
                     appearance, neural)
    with torch.cuda.device(device):
        return _render(means, quaternions, scales, opacities, appearance, view_matrices,
                       intrinsics, width, height, backgrounds, packed, near_plane, far_plane,
                       neural, sh_degree, batch, scenes, cameras, n, median_depth, pixels)


def _render(means, quaternions, scales, opacities, appearance, view_matrices, intrinsics, width,
            height, backgrounds, packed, near_plane, far_plane, neural, sh_degree, batch, scenes,
            cameras, n, median_depth=False, pixels=None):
    device = means.device
    S, C, N = scenes, cameras, n
    P = S * C * N
    sh = sh_degree is not None
    flat = (lambda t, *shape: t.reshape(S, *shape))
    sh_args = (flat(appearance[0], N, (sh_degree + 1) ** 2, 3),
               flat(appearance[1], N, (sh_degree + 1) ** 2, 3),
               flat(appearance[2], N, 4), flat(appearance[3], N, 4),
               flat(appearance[4], N, 4)) if sh else (None,) * 5
    records, xy, sh_rows, radii = Projection.apply(
        flat(means, N, 3), flat(quaternions, N, 4), flat(scales, N, 2), flat(opacities, N),
        flat(view_matrices, C, 4, 4), flat(intrinsics, C, 3, 3), *sh_args, sh_degree, width,
        height, float(near_plane), float(far_plane))
    if sh:
        rows, row_mode = sh_rows, nat.ROWS_PER_RECORD
    else:
        rows = SurfelRows.apply(neural, *(t.reshape(S * N, k) for t, k in
                                          zip(appearance, SurfelRows.widths(neural))))
        row_mode = nat.ROWS_PER_SURFEL
    images = S * C
    visible_count = None
    if packed:
        # The packed metadata needs the number of visible pairs on the host.  Count them
        # on the device and copy the count to pinned memory ahead of binning: binning
        # reads its own totals back with one stream synchronisation per call (as the
        # reference's does, rasterize.cu:466-468), after which the count is readable, so
        # packing adds no second synchronisation (torch.nonzero would).
        visible = radii > 0
        visible_count = torch.empty((), dtype=torch.int64, pin_memory=True)
        visible_count.copy_(visible.sum(), non_blocking=True)
    chunks = bin_chunks(records, radii, S, C, max(N, 1), width, height)
    selected = None
    projected_means = xy
    if packed:
        if ARENA is not None or P == 0:   # binning made no host synchronisation
            torch.cuda.current_stream(device).synchronize()
        selected = torch.nonzero_static(visible, size=int(visible_count)).reshape(-1)
        projected_means = PackedRows.apply(xy, selected)
    selection = None
    pixel_shape = (height, width)
    if pixels is not None:
        selection = Selection(pixels.reshape(images, -1, 2), width, height)
        pixel_shape = (selection.count,)
    outputs = Composite.apply(records, projected_means, rows, backgrounds.reshape(-1, 3),
                              selected, chunks, row_mode, C, max(N, 1), images, width, height,
                              neural, float(near_plane), float(far_plane), median_depth,
                              selection)
    rgb, alpha, depth, normals, distortion = (
        plane.reshape(batch + (C,) + pixel_shape + (plane.shape[-1],)) for plane in outputs[:5])
    count = selected.shape[0] if packed else P
    scene_ids, camera_ids, primitive_ids = (torch.empty((count,), device=device, dtype=torch.int64)
                                            for _ in range(3))
    nat.call("gs_pair_ids", nat.ptr(selected) if packed else None, count, C, max(N, 1),
             nat.ptr(scene_ids), nat.ptr(camera_ids), nat.ptr(primitive_ids),
             nat.stream_of(device))
    meta = {
        "radii": radii.index_select(0, selected) if packed else radii.reshape(batch + (C, N)),
        "projected_means": projected_means,
        "scene_ids": scene_ids,
        "camera_ids": camera_ids,
        "primitive_ids": primitive_ids,
        "packed": packed,
        "accumulated_depth": depth,
        "normals": normals,
        "distortion": distortion,
    }
    if median_depth:
        meta["median_depth"] = outputs[5].reshape(batch + (C,) + pixel_shape + (1,))
    return rgb, alpha, meta


def rasterize_gabors(
    means: torch.Tensor,
    quaternions: torch.Tensor,
    scales: torch.Tensor,
    opacities: torch.Tensor,
    colors: torch.Tensor,
    secondary_colors: torch.Tensor,
    frequency_weights: torch.Tensor,
    frequency_magnitudes: torch.Tensor,
    phases: torch.Tensor,
    view_matrices: torch.Tensor,
    intrinsics: torch.Tensor,
    width: int,
    height: int,
    *,
    backgrounds: torch.Tensor | None = None,
    packed: bool = False,
    near_plane: float = 0.2,
    far_plane: float = 100.0,
    sh_degree: int | None = None,
    validate: bool = True,
    median_depth: bool = False,
    pixels: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor, dict[str, Any]]:
    """Render four-frequency Gabor surfaces over arbitrary scene and camera batches.

    Same contract as the reference (rendering.py:403-456): means [..., N, 3], unit
    wxyz quaternions [..., N, 4], positive scales [..., N, 2], opacities [..., N];
    colors and secondary_colors [..., N, 3] (or [..., N, (degree+1)**2, 3] SH
    coefficients with ``sh_degree``); frequency weights (summing to one),
    magnitudes and phases [..., N, 4]; cameras [..., C, 4, 4] and [..., C, 3, 3].
    All tensors contiguous CUDA float32.  Returns RGB [..., C, H, W, 3], alpha
    [..., C, H, W, 1] and metadata (radii, projected_means, scene/camera/primitive
    ids, packed, accumulated_depth, normals, distortion).

    ``median_depth=True`` (an addition: the reference lists median depth outside its
    release) also returns ``meta["median_depth"]`` [..., C, H, W, 1]: per pixel the depth
    of the last contribution made while the transmittance before it exceeded 0.5 (the
    2DGS convention; 0 without contributions), differentiable through that
    contribution's depth.  ``pixels`` (also an addition: selected-pixel rendering is
    outside the reference's release), integer [..., C, P, 2] (x, y) inside the image,
    composites only those pixels: every per-pixel output is then [..., C, P, k], with
    values identical to the same pixels of a full render.
    """
    return render(means, quaternions, scales, opacities,
                  (colors, secondary_colors, frequency_weights, frequency_magnitudes, phases),
                  view_matrices, intrinsics, width, height, backgrounds, packed, near_plane,
                  far_plane, False, sh_degree, validate, median_depth, pixels)


def rasterize_neural_gabors(
    means: torch.Tensor,
    quaternions: torch.Tensor,
    scales: torch.Tensor,
    opacities: torch.Tensor,
    input_weights: torch.Tensor,
    input_biases: torch.Tensor,
    output_weights: torch.Tensor,
    output_biases: torch.Tensor,
    view_matrices: torch.Tensor,
    intrinsics: torch.Tensor,
    width: int,
    height: int,
    *,
    backgrounds: torch.Tensor | None = None,
    packed: bool = False,
    near_plane: float = 0.2,
    far_plane: float = 100.0,
    validate: bool = True,
    median_depth: bool = False,
    pixels: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor, dict[str, Any]]:
    """Render per-surface 5->6->3 SIRENs (sine frequency 30, sigmoid RGB).

    Same contract as the reference (rendering.py:459-502): per-primitive input
    weights/biases [..., N, 6, 5] / [..., N, 6], output weights/biases
    [..., N, 3, 6] / [..., N, 3]; network input (u/3, v/3, world view direction).
    ``median_depth`` and ``pixels`` as for ``rasterize_gabors``.
    """
    return render(means, quaternions, scales, opacities,
                  (input_weights, input_biases, output_weights, output_biases),
                  view_matrices, intrinsics, width, height, backgrounds, packed, near_plane,
                  far_plane, True, None, validate, median_depth, pixels)
