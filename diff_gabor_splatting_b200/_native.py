"""ctypes binding of libgabor_b200.so (the C ABI declared in include/gabor_b200.h).

The library is loaded once, from this package directory.  There is no fallback:
if the shared library is missing or cannot be loaded, importing the package fails
with an explanation of how to build it.  Every call checks the returned status and
raises RuntimeError with the library's message (the reference's native layer raises
RuntimeError through TORCH_CHECK in the same situations).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIBRARY_PATH = Path(__file__).resolve().parent / "libgabor_b200.so"

_p = ctypes.c_void_p
_i = ctypes.c_int
_l = ctypes.c_int64
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> argument types (all return int status)
SIGNATURES = {
    "gs_project_forward": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _l, _l, _l, _i, _i, _f,
                           _f, _p, _p, _p, _p, _p],
    "gs_project_backward": [_p, _p, _p, _p, _p, _p, _p, _i, _l, _l, _l, _p, _p, _p, _p, _p, _p,
                            _p, _p, _p, _p, _p, _p, _p, _p, _p],
    "gs_project_forward_ragged": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _l, _l, _p, _l,
                                  _i, _i, _f, _f, _p, _p, _p, _p, _p],
    "gs_project_backward_ragged": [_p, _p, _p, _p, _p, _p, _p, _i, _l, _l, _p, _l, _l, _p, _p, _p,
                                   _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p],
    "gs_bin_count_workspace": [_l, ctypes.POINTER(_sz)],
    "gs_bin_count": [_p, _i, _p, _p, _l, _l, _l, _i, _i, _i, _p, _sz, ctypes.POINTER(_l),
                     ctypes.POINTER(_l), _p],
    "gs_bin_sort_workspace": [_l, _l, _l, _l, _i, _i, ctypes.POINTER(_sz)],
    "gs_bin_sort": [_p, _i, _p, _p, _l, _l, _l, _i, _i, _i, _p, _sz, _p, _sz, _l, _l, _p, _p, _p],
    "gs_bin_arena_workspace": [_l, _l, _l, _l, _i, _i, ctypes.POINTER(_sz)],
    "gs_bin_arena": [_p, _i, _p, _p, _l, _l, _l, _i, _i, _i, _p, _sz, _l, _l, _p, _p, _p, _p],
    "gs_composite_forward": [_p, _p, _i, _p, _l, _l, _l, _l, _p, _p, _p, _l, _i, _i, _i, _i, _f,
                             _f, _p, _p, _p, _p, _p],
    "gs_composite_backward": [_p, _p, _i, _p, _l, _l, _l, _l, _p, _p, _p, _p, _p, _p, _l, _i, _i,
                              _i, _f, _f, _p, _p, _p, _p, _p, _p],
    "gs_composite_forward_split": [_p, _p, _i, _p, _l, _l, _l, _l, _p, _p, _p, _l, _i, _i, _i, _i,
                                   _f, _f, _p, _p, _p, _l, _p, _p, _p, _l, _p, _p, _p, _l, _p,
                                   _p],
    "gs_composite_backward_split": [_p, _p, _i, _p, _l, _l, _l, _l, _p, _p, _p, _p, _p, _p, _p, _p,
                                    _p, _l, _p, _p, _l, _l, _i, _i, _i, _f, _f, _p, _p, _p, _p,
                                    _p, _l, _p, _p],
    "gs_adam_step": [_i, _p, _p, _p, _p, _p, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                     ctypes.c_double, ctypes.c_double, _l, _p],
    "gs_adam_step_capturable": [_i, _p, _p, _p, _p, _p, _p, ctypes.c_double, ctypes.c_double,
                                ctypes.c_double, ctypes.c_double, ctypes.c_double, _p, _p],
    "gs_pack_geometry": [_p, _p, _p, _l, _l, _p, _p],
    "gs_pack_rows": [_p, _l, _i, _p, _p],
    "gs_unpack_geometry_grads": [_p, _p, _l, _l, _p, _p, _p],
    "gs_unpack_rows": [_p, _l, _i, _p, _p],
    "gs_pair_ids": [_p, _l, _l, _l, _p, _p, _p, _p],
    "gs_pack_surfel_rows": [_i, _p, _l, _p, _p],
    "gs_unpack_surfel_rows": [_i, _p, _l, _p, _p],
    "gs_fp32_probe": [_i, _i, _i, _p, _p],
    "gs_sh_forward": [_p, _p, _p, _i, _l, _l, _l, _p, _p],
    "gs_sh_backward": [_p, _p, _p, _p, _i, _l, _l, _l, _p, _p, _p, _p],
}

ROWS_PER_RECORD, ROWS_PER_SURFEL, ROWS_EXPLICIT = 0, 1, 2
BIN_TIGHT = 1
COMPOSITE_EXACT = 1
RECORD_FLOATS, CLASSIC_ROW_FLOATS, NEURAL_ROW_FLOATS = 20, 20, 60


def _load() -> ctypes.CDLL:
    if not LIBRARY_PATH.exists():
        raise ImportError(
            f"{LIBRARY_PATH} is missing: build it with "
            "`python -m diff_gabor_splatting_b200.build` (nvcc, sm_100a). "
            "There is no CPU or alternative-backend fallback.")
    lib = ctypes.CDLL(str(LIBRARY_PATH))
    lib.gs_version.restype = _i
    lib.gs_last_error.restype = ctypes.c_char_p
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _i
    return lib


lib = _load()


def check(status: int, name: str) -> None:
    """Raise RuntimeError for a nonzero library status."""
    if status != 0:
        message = lib.gs_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed (status {status}): {message}")


# Optional stage timer: when set (see ``StageTimer``), every call is bracketed by
# CUDA events on the caller's current stream.
TIMER = None


def call(name: str, *args) -> None:
    """Call one C entry point and check its status."""
    check(call_status(name, *args), name)


def call_status(name: str, *args) -> int:
    """Call one C entry point and return its status (timed when a timer is set)."""
    if TIMER is None:
        return getattr(lib, name)(*args)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    status = getattr(lib, name)(*args)
    end.record()
    TIMER.add(name, start, end)
    return status


class StageTimer:
    """Collects per-entry-point CUDA-event durations while installed as ``TIMER``."""

    def __init__(self):
        self.events = []

    def __enter__(self):
        global TIMER
        TIMER = self
        return self

    def __exit__(self, *exc):
        global TIMER
        TIMER = None

    def add(self, name, start, end):
        self.events.append((name, start, end))

    def totals(self) -> dict:
        """name -> (calls, total milliseconds); call after synchronising."""
        out = {}
        for name, start, end in self.events:
            calls, ms = out.get(name, (0, 0.0))
            out[name] = (calls + 1, ms + start.elapsed_time(end))
        return out


def ptr(t: torch.Tensor | None) -> int | None:
    """Device pointer of a tensor (None for a missing or empty optional buffer)."""
    if t is None:
        return None
    return t.data_ptr() if t.numel() else None


def host_array(ctype, values):
    """A host C array of ``values`` (keep it alive across the call) and its address."""
    array = (ctype * len(values))(*[0 if v is None else v for v in values])
    return array, ctypes.cast(array, ctypes.c_void_p)


def stream_of(device: torch.device) -> int:
    """The caller's current CUDA stream on ``device`` as a raw handle."""
    return torch.cuda.current_stream(device).cuda_stream
