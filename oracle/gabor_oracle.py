"""CPU oracle for the Gabor surface-splatting render path.  TEST INFRASTRUCTURE ONLY.

This module restates, on the CPU and in plain PyTorch/numpy, the algorithm of the
reference package luisrodolfo10/diff_gabor_splatting v0.1.1.  It is the checker for
the CUDA product path (tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg only).  Nothing in ``diff_gabor_splatting_b200`` imports it, and the
product path never falls back to it.

Pinned against: golden vectors produced by the reference's own Python code
(``project_surfaces``, ``quaternion_matrix``, ``check_values`` of
``src/gabor_splatting/rendering.py`` and the float64 test oracles of
``tests/test_rendering.py:64-171`` / ``tests/test_spherical_harmonics.py:10-69``), run
on the CPU in the build container and committed under ``tests/golden/`` together
with the script that made them (``tests/golden/make_golden.py``).

Every function cites the reference lines it restates.  All arithmetic follows the
reference's float32 operation order where the CUDA kernels fix one (tile bounds,
sampling, compositing recurrences), so the oracle's integer outputs (tile counts,
keys, sort order, tile ranges, contributor counts) are exact for identical inputs
and its float outputs agree to rounding.  The compositor is written as a
sequential front-to-back recurrence vectorised over (tiles x 256 pixels); it is
differentiable with torch autograd, which is how gradients are obtained (the
reference tests obtain theirs the same way from their float64 oracle).
"""

from __future__ import annotations

import math

import numpy as np
import torch

TILE = 16
GEOMETRY_SIZE = 17
MAP_SIZE = 9
# float32(3 * 0.707106): minimum screen radius, rendering.py:208
MIN_RADIUS = 3 * 0.707106


# ----------------------------------------------------------------------------------
# projection: rendering.py:156-218
# ----------------------------------------------------------------------------------
def quaternion_matrix(q: torch.Tensor) -> torch.Tensor:
    """Normalise wxyz quaternions and build rotation matrices (rendering.py:156-173)."""
    q = q / torch.linalg.vector_norm(q, dim=-1, keepdim=True)
    w, x, y, z = q.unbind(-1)
    rows = (
        1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
        2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
        2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y),
    )
    return torch.stack(rows, -1).reshape(*q.shape[:-1], 3, 3)


def project_surfaces(means, quaternions, scales, view_matrices, intrinsics,
                     width, height, near_plane, far_plane):
    """Per (scene, camera, surfel) splat setup (rendering.py:176-218).

    Shapes: means [S,N,3], quaternions [S,N,4], scales [S,N,2], view_matrices
    [S,C,4,4], intrinsics [S,C,3,3].  Returns the homogeneous plane transform
    T = K [R_c t_u s_u, R_c t_v s_v, mean_c] as [S,C,N,3,3], the conic centre xy
    [S,C,N,2], camera-facing normals [S,C,N,3], unit world view directions
    [S,C,N,3] and int32 screen radii [S,C,N] (0 = culled).
    """
    rotation = quaternion_matrix(quaternions)
    tangent = rotation[..., :2] * scales.unsqueeze(-2)                 # [S,N,3,2]
    cam_rot = view_matrices[..., :3, :3]
    cam_means = torch.einsum("scij,snj->scni", cam_rot, means)
    cam_means = cam_means + view_matrices[..., None, :3, 3]
    cam_tangent = torch.einsum("scij,snjk->scnik", cam_rot, tangent)
    plane = torch.cat((cam_tangent, cam_means.unsqueeze(-1)), dim=-1)  # [S,C,N,3,3]
    T = torch.einsum("scij,scnjk->scnik", intrinsics, plane)
    # Perspective conic of the 3-sigma disk (t = (9, 9, -1)), rendering.py:189-196.
    t = T.new_tensor([9.0, 9.0, -1.0])
    denom = (t * T[..., 2, :].square()).sum(-1)
    valid_conic = denom != 0
    f = t / torch.where(valid_conic, denom, torch.ones_like(denom)).unsqueeze(-1)
    xy = (f.unsqueeze(-2) * T[..., :2, :] * T[..., 2:3, :]).sum(-1)
    extent_sq = xy.square() - (f.unsqueeze(-2) * T[..., :2, :].square()).sum(-1)
    extent = extent_sq.clamp_min(1e-4).sqrt()
    normals = torch.einsum("scij,snj->scni", cam_rot, rotation[..., 2])
    facing = -(cam_means * normals).sum(-1)
    sign = torch.where(facing > 0, torch.ones_like(facing), -torch.ones_like(facing))
    normals = normals * sign.unsqueeze(-1)
    centers = -torch.einsum("scji,scj->sci", cam_rot, view_matrices[..., :3, 3])
    direction = means[:, None] - centers[:, :, None]
    directions = direction / torch.linalg.vector_norm(
        direction, dim=-1, keepdim=True).clamp_min(1e-12)
    with torch.no_grad():
        radius = torch.maximum(extent.amax(-1), extent.new_tensor(MIN_RADIUS)).ceil()
        tw, th = (width + TILE - 1) // TILE, (height + TILE - 1) // TILE
        lower = torch.trunc((xy - radius.unsqueeze(-1)) / TILE).clamp_min(0)
        upper = torch.trunc((xy + radius.unsqueeze(-1) + (TILE - 1)) / TILE).clamp_min(0)
        visible = valid_conic & (facing != 0) & (cam_means[..., 2] > near_plane)
        visible &= cam_means[..., 2] < far_plane
        visible &= torch.isfinite(radius) & (radius < 2**30) & torch.isfinite(xy).all(-1)
        visible &= upper[..., 0].clamp_max(tw) > lower[..., 0].clamp_max(tw)
        visible &= upper[..., 1].clamp_max(th) > lower[..., 1].clamp_max(th)
        radii = torch.where(visible, radius, torch.zeros_like(radius)).to(torch.int32)
    return T, xy, normals, directions, radii


# ----------------------------------------------------------------------------------
# spherical harmonics: spherical_harmonics.cu:11-85
# ----------------------------------------------------------------------------------
SH_C0 = 0.28209479177387814
SH_C1 = 0.4886025119029199
SH_C2 = (1.0925484305920792, 0.31539156525252005, 0.5462742152960396)
SH_C3 = (-0.5900435899266435, 2.890611442640554, -0.4570457994644658,
         0.3731763325901154, 1.445305721320277)


def sh_basis(degree: int, directions: torch.Tensor) -> torch.Tensor:
    """Real SH basis (Inria ordering) up to ``degree`` (spherical_harmonics.cu:11-42).

    directions [..., 3] -> basis [..., (degree+1)**2], differentiable.
    """
    x, y, z = directions.unbind(-1)
    b = [torch.full_like(x, SH_C0)]
    if degree > 0:
        b += [-SH_C1 * y, SH_C1 * z, -SH_C1 * x]
    if degree > 1:
        a, c, d = SH_C2
        b += [a * x * y, -a * y * z, c * (2 * z * z - x * x - y * y), -a * x * z,
              d * (x * x - y * y)]
    if degree > 2:
        a, b1, c, d, e = SH_C3
        b += [a * y * (3 * x * x - y * y), b1 * x * y * z, c * y * (4 * z * z - x * x - y * y),
              d * z * (2 * z * z - 3 * x * x - 3 * y * y), c * x * (4 * z * z - x * x - y * y),
              e * z * (x * x - y * y), a * x * (x * x - 3 * y * y)]
    return torch.stack(b, -1)


def evaluate_sh(first, second, directions, degree):
    """Both SH colour sets per pair, clamp(SH(dir).c + 0.5, 0) (spherical_harmonics.cu:45-85).

    first/second [S,N,K,3] coefficients shared by the cameras of a scene;
    directions [S,C,N,3]; returns colours [S,C,N,6] = (first rgb, second rgb).
    """
    basis = sh_basis(degree, directions)                       # [S,C,N,K]
    out = []
    for coeffs in (first, second):
        raw = 0.5 + torch.einsum("scnk,snkr->scnr", basis, coeffs)
        out.append(raw.clamp_min(0.0))
    return torch.cat(out, -1)


# ----------------------------------------------------------------------------------
# packing: rendering.py:334-381
# ----------------------------------------------------------------------------------
def pack(transform, xy, normals, directions, radii, opacities, appearance,
         neural, sh_degree, packed):
    """Build the compositor's flat records (rendering.py:334-381).

    Returns dict(geometry [Q,17], parameters [P,18|57], opacities [P],
    primitive_ids [Q] int64, image_ids [Q] int64, radii [Q] int32, selected [Q],
    projected_means [Q,2]).  ``appearance`` is the tuple of user tensors with the
    scene dims flattened to one ([S,N,...]).
    """
    S, C, N = radii.shape
    dev = radii.device
    if sh_degree is not None:
        colors = evaluate_sh(appearance[0], appearance[1], directions, sh_degree)
        rest = [t.reshape(S, 1, N, 4).expand(S, C, N, 4) for t in appearance[2:]]
        parameters = torch.cat((colors, *rest), -1).reshape(-1, 18)
        opacity_parameters = opacities.reshape(S, 1, N).expand(S, C, N).reshape(-1)
        primitive_ids = torch.arange(S * C * N, device=dev)
    else:
        width = 57 if neural else 18
        parameters = torch.cat([t.reshape(S, N, -1) for t in appearance], -1).reshape(S * N, width)
        opacity_parameters = opacities.reshape(S * N)
        primitive_ids = torch.arange(S * N, device=dev).reshape(S, 1, N).expand(S, C, N).reshape(-1)
    image_ids = torch.arange(S * C, device=dev).reshape(S, C, 1).expand(S, C, N).reshape(-1)
    selected = torch.arange(S * C * N, device=dev)
    if packed:
        selected = selected[radii.reshape(-1) > 0]
    projected_means = xy.reshape(-1, 2)[selected]
    geometry = torch.cat((transform.reshape(-1, 9)[selected], projected_means,
                          normals.reshape(-1, 3)[selected],
                          directions.reshape(-1, 3)[selected]), -1)
    return dict(geometry=geometry, parameters=parameters, opacities=opacity_parameters,
                primitive_ids=primitive_ids[selected], image_ids=image_ids[selected],
                radii=radii.reshape(-1)[selected].contiguous(), selected=selected,
                projected_means=projected_means)


# ----------------------------------------------------------------------------------
# tile binning: rasterize.cu:24-69 and the host driver rasterize.cu:454-493
# ----------------------------------------------------------------------------------
def tile_rects(geometry: np.ndarray, radii: np.ndarray, tw: int, th: int):
    """Integer tile rectangle [x0,y0,x1,y1) per record (rasterize.cu:24-30).

    float32 (x - r)/16 and (x + r + 15)/16, truncated toward zero, clamped to the grid.
    """
    g = np.asarray(geometry, dtype=np.float32)
    r = np.asarray(radii).astype(np.float32)
    x, y = g[:, 9], g[:, 10]
    sixteen, fifteen = np.float32(TILE), np.float32(TILE - 1)

    def trunc_clamp(v, hi):
        with np.errstate(invalid="ignore", over="ignore"):
            v = np.trunc(v.astype(np.float64))
        v = np.nan_to_num(v, nan=0.0, posinf=2**31 - 1, neginf=-(2**31))
        v = np.clip(v, -(2**31), 2**31 - 1)            # cvt.rzi.s32 saturates
        return np.clip(v, 0, hi).astype(np.int64)

    x0 = trunc_clamp((x - r) / sixteen, tw)
    y0 = trunc_clamp((y - r) / sixteen, th)
    x1 = trunc_clamp((x + r + fifteen) / sixteen, tw)
    y1 = trunc_clamp((y + r + fifteen) / sixteen, th)
    return x0, y0, x1, y1


def bin_tiles(geometry, radii, image_ids, images, width, height):
    """Count, emit, stable-sort and range the (image, tile, depth) keys.

    Restates countTiles/emitTiles/findRanges (rasterize.cu:32-69) and the
    CUB SortPairs over all 64 key bits (rasterize.cu:478-487): a stable sort, so
    equal keys keep emission order (record index, then row-major tile order).
    Returns dict(counts int64 [Q], keys uint64 [I] (sorted), point_list int32 [I],
    ranges int32 [images*tw*th, 2]).
    """
    g = np.ascontiguousarray(torch.as_tensor(geometry).detach().to(torch.float32).numpy())
    r = torch.as_tensor(radii).numpy().astype(np.int64)
    img = torch.as_tensor(image_ids).numpy().astype(np.int64)
    tw, th = (width + TILE - 1) // TILE, (height + TILE - 1) // TILE
    n_tiles = images * tw * th
    Q = g.shape[0]
    ranges = np.zeros((n_tiles, 2), np.int32)
    if Q == 0:
        return dict(counts=np.zeros(0, np.int64), keys=np.zeros(0, np.uint64),
                    point_list=np.zeros(0, np.int32), ranges=ranges)
    x0, y0, x1, y1 = tile_rects(g, r, tw, th)
    counts = np.where(r > 0, (x1 - x0) * (y1 - y0), 0).astype(np.int64)
    total = int(counts.sum())
    if total == 0:
        return dict(counts=counts, keys=np.zeros(0, np.uint64),
                    point_list=np.zeros(0, np.int32), ranges=ranges)
    owner = np.repeat(np.arange(Q), counts)
    start = np.cumsum(counts) - counts
    local = np.arange(total) - start[owner]
    w = (x1 - x0)[owner]
    tx = x0[owner] + local % w
    ty = y0[owner] + local // w
    tile = img[owner].astype(np.uint64) * np.uint64(tw * th) + (ty * tw + tx).astype(np.uint64)
    depth_bits = g[:, 8].view(np.uint32).astype(np.uint64)[owner]
    keys = (tile << np.uint64(32)) | depth_bits
    order = np.argsort(keys, kind="stable")
    keys = keys[order]
    point_list = owner[order].astype(np.int32)
    tiles = (keys >> np.uint64(32)).astype(np.int64)
    uniq, first, cnt = np.unique(tiles, return_index=True, return_counts=True)
    ranges[uniq, 0] = first
    ranges[uniq, 1] = first + cnt
    return dict(counts=counts, keys=keys, point_list=point_list, ranges=ranges)


# ----------------------------------------------------------------------------------
# compositor: rasterize.cu:71-138 (sample, appearance), 229-281 (forward)
# ----------------------------------------------------------------------------------
def _appearance(a, g, s0, s1, neural, dtype):
    """Per (pixel, record) RGB (rasterize.cu:105-138); a/g are [T,1,*] batches."""
    if neural:
        inp = [s0 / 3, s1 / 3, g[..., 14], g[..., 15], g[..., 16]]
        hidden = []
        for h in range(6):
            z = a[..., 30 + h]
            for k in range(5):
                z = z + a[..., h * 5 + k] * inp[k]
            hidden.append(torch.sin(30 * z))
        color = []
        for c in range(3):
            z = a[..., 54 + c]
            for h in range(6):
                z = z + a[..., 36 + c * 6 + h] * hidden[h]
            color.append(1 / (1 + torch.exp(-z)))
        return color
    pi = torch.tensor(math.pi, dtype=dtype)
    h1 = torch.zeros((), dtype=dtype)
    h2 = torch.zeros((), dtype=dtype)
    for f in range(4):
        ang = pi * f / 4
        dot = torch.cos(ang) * s0 + torch.sin(ang) * s1
        wave = torch.cos(2 * pi * a[..., 10 + f] * dot + a[..., 14 + f])
        h1 = h1 + a[..., 6 + f] * 0.5 * (1 + wave)
        h2 = h2 + a[..., 6 + f] * 0.5 * (1 - wave)
    return [h1 * a[..., c] + h2 * a[..., 3 + c] for c in range(3)]


def composite(geometry, appearance, opacities, primitive_ids, backgrounds, point_list,
              ranges, width, height, neural, near_plane, far_plane, tiles=None,
              dtype=torch.float32):
    """Front-to-back compositing of every image tile (rasterize.cu:229-281).

    Vectorised over (selected tiles x 16x16 pixels), sequential over each tile's
    depth-sorted record list, with the reference's per-pixel stopping rule: a pixel
    stops *before* a record whose contribution would take T below 1e-4.  The
    sample test follows sampleSurface (rasterize.cu:84-103).  Differentiable by
    autograd through geometry, appearance, opacities and backgrounds.

    Returns dict(maps [n,256,9], state [n,256,3], contributors [n,256] int32,
    inside [n,256] bool, tiles [n]) for the ``tiles`` processed (all by default).
    """
    geometry = geometry.to(dtype)
    appearance = appearance.to(dtype)
    opacities = opacities.to(dtype)
    backgrounds = backgrounds.to(dtype)
    images = backgrounds.shape[0]
    tw, th = (width + TILE - 1) // TILE, (height + TILE - 1) // TILE
    per_image = tw * th
    ranges = torch.as_tensor(np.asarray(ranges)).to(torch.int64).reshape(-1, 2)
    plist = torch.as_tensor(np.asarray(point_list)).to(torch.int64)
    if tiles is None:
        tiles = torch.arange(images * per_image)
    tiles = torch.as_tensor(tiles).to(torch.int64)
    n = tiles.numel()
    starts, ends = ranges[tiles, 0], ranges[tiles, 1]
    lens = ends - starts
    image = tiles // per_image
    local = tiles % per_image
    px = torch.arange(TILE * TILE) % TILE
    py = torch.arange(TILE * TILE) // TILE
    X = ((local % tw) * TILE)[:, None] + px[None]
    Y = ((local // tw) * TILE)[:, None] + py[None]
    inside = (X < width) & (Y < height)
    Xf, Yf = X.to(dtype), Y.to(dtype)
    near = torch.tensor(near_plane, dtype=dtype)
    far = torch.tensor(far_plane, dtype=dtype)
    mscale = far / (far - near)
    threshold = torch.tensor(1.0, dtype=dtype) / 255
    cap = torch.tensor(0.99, dtype=dtype)
    T = torch.ones((n, TILE * TILE), dtype=dtype)
    m1 = torch.zeros_like(T)
    m2 = torch.zeros_like(T)
    out = [torch.zeros_like(T) for _ in range(MAP_SIZE)]
    done = ~inside
    last = torch.zeros((n, TILE * TILE), dtype=torch.int64)
    # median depth: the depth of the last contribution made while the transmittance
    # before it exceeds 0.5 (the 2DGS convention; an addition beyond the reference)
    median = torch.zeros_like(T)
    # test support: per pixel, the smallest |T - 0.5| over accepted contributions (the
    # transmittance before each); a median that differs between two roundings of the
    # same pixel needs a contribution this close to the 0.5 threshold
    median_margin = torch.full_like(T, float("inf"))
    max_len = int(lens.max()) if n else 0
    one = torch.ones((), dtype=dtype)
    for j in range(max_len):
        has = (j < lens)[:, None]
        live = has & ~done
        if not bool(live.any()):
            break
        ids = plist[(starts + j).clamp_max(max(plist.numel() - 1, 0))] if plist.numel() else starts
        ids = torch.where(has[:, 0], ids, torch.zeros_like(ids))
        g = geometry[ids][:, None, :]
        prim = primitive_ids[ids]
        o = opacities[prim][:, None]
        a = appearance[prim][:, None, :]
        k = [Xf * g[..., 6 + i] - g[..., i] for i in range(3)]
        l_ = [Yf * g[..., 6 + i] - g[..., 3 + i] for i in range(3)]
        p0 = k[1] * l_[2] - k[2] * l_[1]
        p1 = k[2] * l_[0] - k[0] * l_[2]
        p2 = k[0] * l_[1] - k[1] * l_[0]
        nonzero = p2 != 0
        p2s = torch.where(nonzero, p2, one)
        s0, s1 = p0 / p2s, p1 / p2s
        rho3 = s0 * s0 + s1 * s1
        dx, dy = g[..., 9] - Xf, g[..., 10] - Yf
        rho2 = 2 * (dx * dx + dy * dy)
        surface = rho3 <= rho2
        zsurf = s0 * g[..., 6] + s1 * g[..., 7] + g[..., 8]
        depth = zsurf if neural else torch.where(surface, zsurf, g[..., 8].expand_as(zsurf))
        ok = nonzero & (depth >= near) & torch.isfinite(depth)
        rho = torch.where(ok, torch.minimum(rho3, rho2), torch.zeros_like(rho3))
        expo = torch.exp(-0.5 * rho)
        alpha = torch.minimum(cap, o * expo)
        accept = live & ok & (alpha >= threshold)
        nxt = T * (1 - alpha)
        stop = accept & (nxt < 1e-4)
        done = done | stop
        accept = accept & ~stop
        if not bool(accept.any()):
            continue
        color = _appearance(a, g, torch.where(accept, s0, 0 * s0),
                            torch.where(accept, s1, 0 * s1), neural, dtype)
        w = torch.where(accept, T * alpha, torch.zeros_like(T))
        dsafe = torch.where(accept, depth, one.expand_as(depth))
        m = mscale * (1 - near / dsafe)
        for c in range(3):
            out[c] = out[c] + w * color[c]
            out[5 + c] = out[5 + c] + w * g[..., 11 + c]
        out[4] = out[4] + w * dsafe
        out[8] = out[8] + w * (m * m * (1 - T) + m2 - 2 * m * m1)
        m1 = m1 + w * m
        m2 = m2 + w * m * m
        median = torch.where(accept & (T > 0.5), dsafe, median)
        median_margin = torch.where(accept, torch.minimum(median_margin, (T - 0.5).abs()),
                                    median_margin)
        T = torch.where(accept, nxt, T)
        last = torch.where(accept, torch.full_like(last, j + 1), last)
    bg = backgrounds[image][:, None, :]
    for c in range(3):
        out[c] = out[c] + T * bg[..., c]
    out[3] = 1 - T
    maps = torch.stack(out, -1)
    zero = torch.zeros((), dtype=dtype)
    maps = torch.where(inside[..., None], maps, zero)
    state = torch.where(inside[..., None], torch.stack((T, m1, m2), -1), zero)
    contributors = torch.where(inside, last, torch.zeros_like(last)).to(torch.int32)
    median = torch.where(inside, median, zero)
    return dict(maps=maps, state=state, contributors=contributors, inside=inside, tiles=tiles,
                median_depth=median, median_margin=median_margin.detach())


def tiles_to_images(tile_values, images, width, height):
    """Reassemble per-tile pixel values [images*tw*th, 256, ...] into [images, H, W, ...]."""
    tw, th = (width + TILE - 1) // TILE, (height + TILE - 1) // TILE
    rest = tile_values.shape[2:]
    v = tile_values.reshape(images, th, tw, TILE, TILE, *rest)
    v = v.permute(0, 1, 3, 2, 4, *range(5, 5 + len(rest)))
    return v.reshape(images, th * TILE, tw * TILE, *rest)[:, :height, :width]


# ----------------------------------------------------------------------------------
# whole render: rendering.py:241-400 (without the CUDA-only input checks)
# ----------------------------------------------------------------------------------
def render(means, quaternions, scales, opacities, appearance, view_matrices, intrinsics,
           width, height, backgrounds=None, packed=False, near_plane=0.2, far_plane=100.0,
           neural=False, sh_degree=None, dtype=torch.float32, return_internals=False):
    """CPU restatement of ``render`` (rendering.py:241-400), differentiable by autograd.

    Inputs follow the public API (leading scene dims [...], cameras C).  Returns
    (rgb, alpha, meta) like the reference; with ``return_internals`` also the packed
    records and the binning result.
    """
    batch = tuple(means.shape[:-2])
    n = means.shape[-2]
    cameras = view_matrices.shape[-3]
    scenes = math.prod(batch)
    cast = (lambda t: t.to(dtype))
    if backgrounds is None:
        backgrounds = torch.zeros(batch + (cameras, 3), dtype=means.dtype)
    transform, xy, normals, directions, radii = project_surfaces(
        cast(means).reshape(scenes, n, 3), cast(quaternions).reshape(scenes, n, 4),
        cast(scales).reshape(scenes, n, 2), cast(view_matrices).reshape(scenes, cameras, 4, 4),
        cast(intrinsics).reshape(scenes, cameras, 3, 3), width, height, near_plane, far_plane)
    if neural:
        shapes = [(6, 5), (6,), (3, 6), (3,)]
    else:
        cs = (3,) if sh_degree is None else ((sh_degree + 1) ** 2, 3)
        shapes = [cs, cs, (4,), (4,), (4,)]
    app = [cast(t).reshape((scenes, n) + s) for t, s in zip(appearance, shapes)]
    rec = pack(transform, xy, normals, directions, radii, cast(opacities), app,
               neural, sh_degree, packed)
    images = scenes * cameras
    binned = bin_tiles(rec["geometry"], rec["radii"], rec["image_ids"], images, width, height)
    comp = composite(rec["geometry"], rec["parameters"], rec["opacities"], rec["primitive_ids"],
                     cast(backgrounds).reshape(-1, 3), binned["point_list"], binned["ranges"],
                     width, height, neural, near_plane, far_plane, dtype=dtype)
    maps = tiles_to_images(comp["maps"], images, width, height)
    maps = maps.reshape(batch + (cameras, height, width, MAP_SIZE))
    selected = rec["selected"]
    meta = {
        "radii": rec["radii"] if packed else radii.reshape(batch + (cameras, n)),
        "projected_means": rec["projected_means"],
        "scene_ids": selected // (cameras * max(n, 1)),
        "camera_ids": selected // max(n, 1) % cameras,
        "primitive_ids": selected % max(n, 1),
        "packed": packed,
        "accumulated_depth": maps[..., 4:5],
        "normals": maps[..., 5:8],
        "distortion": maps[..., 8:9],
        "median_depth": tiles_to_images(comp["median_depth"], images, width, height).reshape(
            batch + (cameras, height, width, 1)),
    }
    if return_internals:
        meta["_records"] = rec
        meta["_binning"] = binned
        meta["_state"] = tiles_to_images(comp["state"], images, width, height)
        meta["_contributors"] = tiles_to_images(comp["contributors"], images, width, height)
        meta["_median_margin"] = tiles_to_images(comp["median_margin"], images, width, height)
    return maps[..., :3], maps[..., 3:4], meta
