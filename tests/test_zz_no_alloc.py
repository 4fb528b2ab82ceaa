"""gs_bin_static: the binning entry point that allocates nothing.

It exists for callers that cannot allocate device memory when they bin: a host
application whose own allocator owns every device byte (an engine or DCC plugin with
a fixed memory budget), or a real-time loop that forbids allocation after start-up.
Its scratch is an array compiled into the library.  Checked through the C ABI against
the allocating pair gs_bin_count + gs_bin_sort: point lists and tile ranges are
integers, so they must be identical, on two calls in a row (the array keeps the
previous call's contents; nothing may leak from one call into the next), and on a
16-pixel-wide image where nearly every intersection is its own row span, close to the
documented limits.

This file is collected last on purpose (its name sorts after the others).
"""

import ctypes

import pytest
import torch

from diff_gabor_splatting_b200 import _native as nat
from diff_gabor_splatting_b200 import rendering
from helpers import random_scene

pytestmark = pytest.mark.gpu

W, H = 70, 45
SCRATCH_BYTES = 80 << 20
_p, _i, _l = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64


def _bin_static():
    fn = nat.lib.gs_bin_static
    fn.argtypes = [_p, _i, _p, _p, _l, _l, _l, _i, _i, _p, _l, _p, ctypes.POINTER(_l), _p]
    fn.restype = _i
    return fn


def _records(seed, scenes=2, cameras=2, n=400):
    v = random_scene("classic", scenes=scenes, cameras=cameras, n=n, width=W, height=H, seed=seed)
    with torch.no_grad():
        records, _, _, radii = rendering.Projection.apply(
            v["means"], v["quaternions"], v["scales"], v["opacities"], v["view_matrices"],
            v["intrinsics"], None, None, None, None, None, None, W, H, 0.2, 100.0)
    return records, radii, n, scenes * cameras


def _check_against_allocating(fn, records, radii, per_image, images, width, height):
    expected_points, expected_ranges = rendering.bin_records(
        records, nat.RECORD_FLOATS, radii, None, per_image, images, width, height)
    capacity = expected_points.numel() + 1000
    points = torch.full((capacity,), -7, dtype=torch.int32, device="cuda")
    ranges = torch.full_like(expected_ranges, -7)
    total = ctypes.c_int64(-1)
    status = fn(nat.ptr(records), nat.RECORD_FLOATS, nat.ptr(radii), None, records.shape[0],
                per_image, images, width, height, nat.ptr(points), capacity, nat.ptr(ranges),
                ctypes.byref(total), nat.stream_of(records.device))
    assert status == 0, nat.lib.gs_last_error().decode()
    torch.cuda.synchronize()
    assert total.value == expected_points.numel()
    assert torch.equal(points[:total.value], expected_points)
    assert torch.equal(ranges, expected_ranges)
    assert (points[total.value:] == -7).all()   # nothing written past the count
    return total.value


def test_static_binning_matches_allocating_binning_twice():
    fn = _bin_static()
    for seed in (3, 4):   # two calls in a row, different scenes
        records, radii, n, images = _records(seed)
        _check_against_allocating(fn, records, radii, n, images, W, H)


def test_static_binning_narrow_image_near_the_limits():
    """A 16-px-wide, 4096-tile-tall image: every record's tiles are one column, so the
    row spans equal the intersections (the sort workspace's largest case) -- 921,152 of
    them, within the 1,048,576 limit."""
    fn = _bin_static()
    width, height, count = 16, 16 * 4096, 61440
    g = torch.Generator().manual_seed(9)
    records = torch.zeros(count, nat.RECORD_FLOATS)
    records[:, 9] = 8.0                                                   # x: tile column 0
    records[:, 10] = (torch.arange(count) % 4081).float() * 16 + 8.5      # y: rows 0..4080
    records[:, 8] = torch.rand(count, generator=g) * 5 + 1               # depth (T[2][2])
    records[:, 17] = 0.5
    radii = torch.full((count,), 120, dtype=torch.int32)                  # 8-15 tile rows each
    total = _check_against_allocating(fn, records.cuda(), radii.cuda(), count, 1, width,
                                      height)
    assert 900_000 < total <= 1 << 20


def test_static_scratch_fits_the_worst_case_within_the_limits():
    """The two workspaces (CUB temporary storage included, sized on the GPU) fit the
    80 MiB array at the corners of the limits: 2^20 spans over 128 columns, or over
    2^18 tiles of one column."""
    b1, b2 = ctypes.c_size_t(), ctypes.c_size_t()
    assert nat.lib.gs_bin_count_workspace(ctypes.c_int64(65536), ctypes.byref(b1)) == 0
    align = lambda v: (v + 255) // 256 * 256   # noqa: E731
    for images, width, height in [(1, 2048, 2048 * 16), (32, 2048, 1024), (64, 16, 4096 * 16),
                                  (1, 16, 16 << 18), (2048, 2048, 16)]:
        assert images * -(-width // 16) * -(-height // 16) <= 1 << 18
        st = nat.lib.gs_bin_sort_workspace(ctypes.c_int64(65536), ctypes.c_int64(1 << 20),
                                           ctypes.c_int64(1 << 20), ctypes.c_int64(images),
                                           width, height, ctypes.byref(b2))
        assert st == 0
        assert align(b1.value) + b2.value <= SCRATCH_BYTES, (images, width, height, b2.value)


def test_static_binning_rejects_sizes_beyond_its_scratch():
    fn = _bin_static()
    records, radii, n, images = _records(5)
    total = ctypes.c_int64(-1)
    stream = nat.stream_of(records.device)
    status = fn(nat.ptr(records), nat.RECORD_FLOATS, nat.ptr(radii), None, 65537, n, images, W,
                H, None, 0, None, ctypes.byref(total), stream)
    assert status == 2 and b"65536" in nat.lib.gs_last_error()
    status = fn(nat.ptr(records), nat.RECORD_FLOATS, nat.ptr(radii), None, records.shape[0], n,
                images, 2064, H, None, 0, None, ctypes.byref(total), stream)
    assert status == 2 and b"2048" in nat.lib.gs_last_error()
    status = fn(nat.ptr(records), nat.RECORD_FLOATS, nat.ptr(radii), None, records.shape[0], 1,
                records.shape[0], 1024, 1024, None, 0, None, ctypes.byref(total), stream)
    assert status == 2 and b"262144" in nat.lib.gs_last_error()
    points = torch.empty(1, dtype=torch.int32, device="cuda")
    ranges = torch.empty(images * 5 * 3, 2, dtype=torch.int32, device="cuda")
    status = fn(nat.ptr(records), nat.RECORD_FLOATS, nat.ptr(radii), None, records.shape[0], n,
                images, W, H, nat.ptr(points), 1, nat.ptr(ranges), ctypes.byref(total), stream)
    assert status == 1 and b"capacity" in nat.lib.gs_last_error()
    assert total.value > 1
