"""gs_bin_static: the binning entry point that allocates nothing.

It exists for callers that cannot allocate device memory when they bin (a host
application whose allocator owns every device byte, code running while a stream is
captured into a CUDA graph, real-time loops that forbid allocation after start-up);
its scratch is an array compiled into the library.  Checked through the C ABI
against the allocating pair gs_bin_count + gs_bin_sort: point lists and tile ranges
are integers, so they must be identical, on two calls in a row (the array keeps the
previous call's contents; nothing may leak from one call into the next).

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


def test_static_binning_matches_allocating_binning_twice():
    fn = _bin_static()
    for seed in (3, 4):   # two calls in a row, different scenes
        records, radii, n, images = _records(seed)
        expected_points, expected_ranges = rendering.bin_records(records, nat.RECORD_FLOATS,
                                                                 radii, None, n, images, W, H)
        capacity = expected_points.numel() + 1000
        points = torch.full((capacity,), -7, dtype=torch.int32, device="cuda")
        ranges = torch.full_like(expected_ranges, -7)
        total = ctypes.c_int64(-1)
        status = fn(nat.ptr(records), nat.RECORD_FLOATS, nat.ptr(radii), None, records.shape[0],
                    n, images, W, H, nat.ptr(points), capacity, nat.ptr(ranges),
                    ctypes.byref(total), nat.stream_of(records.device))
        assert status == 0, nat.lib.gs_last_error().decode()
        torch.cuda.synchronize()
        assert total.value == expected_points.numel()
        assert torch.equal(points[:total.value], expected_points)
        assert torch.equal(ranges, expected_ranges)
        assert (points[total.value:] == -7).all()   # nothing written past the count


def test_static_binning_rejects_sizes_beyond_its_scratch():
    fn = _bin_static()
    records, radii, n, images = _records(5)
    total = ctypes.c_int64(-1)
    status = fn(nat.ptr(records), nat.RECORD_FLOATS, nat.ptr(radii), None, 65537, n, images, W,
                H, None, 0, None, ctypes.byref(total), nat.stream_of(records.device))
    assert status == 2 and b"65536" in nat.lib.gs_last_error()
    points = torch.empty(1, dtype=torch.int32, device="cuda")
    ranges = torch.empty(images * 5 * 3, 2, dtype=torch.int32, device="cuda")
    status = fn(nat.ptr(records), nat.RECORD_FLOATS, nat.ptr(radii), None, records.shape[0], n,
                images, W, H, nat.ptr(points), 1, nat.ptr(ranges), ctypes.byref(total),
                nat.stream_of(records.device))
    assert status == 1 and b"capacity" in nat.lib.gs_last_error()
    assert total.value > 1
