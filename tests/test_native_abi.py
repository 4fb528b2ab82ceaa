"""CPU: the C-ABI library and the host-side contracts, without a GPU.

* libgabor_b200.so loads and exports every entry point include/gabor_b200.h declares;
* entry points reject invalid sizes and options before touching the GPU, with the
  documented status codes and a message;
* numerical validation (check_values) raises the reference's exact messages, read
  from tests/golden/check_values.npz (produced by the reference's own check_values);
* the public renderers' structural checks raise the reference's exception types.
"""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from diff_gabor_splatting_b200 import _native as nat
from diff_gabor_splatting_b200 import rasterize_gabors, rasterize_neural_gabors
from diff_gabor_splatting_b200.rendering import check_tensor, check_values
from helpers import load_golden, small_inputs

HEADER = Path(__file__).resolve().parents[1] / "include" / "gabor_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(gs_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    names = declared_symbols()
    assert len(names) >= 17
    for name in names:
        assert hasattr(nat.lib, name), name
    assert nat.lib.gs_version() >= 1
    # every binding the package uses is declared in the header
    assert set(nat.SIGNATURES) <= set(names)


def test_bindings_match_header_prototypes():
    """Every ctypes binding has as many arguments as the header's prototype, and pointer
    / integer / floating kinds line up argument by argument."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    kinds = {ctypes.c_void_p: "pointer", ctypes.c_char_p: "pointer", ctypes.c_int: "int",
             ctypes.c_int64: "int", ctypes.c_uint64: "int", ctypes.c_size_t: "int",
             ctypes.c_float: "float", ctypes.c_double: "float"}
    for name, argtypes in nat.SIGNATURES.items():
        match = re.search(r"\b" + name + r"\s*\(([^;]*?)\)\s*;", text, re.S)
        assert match, name
        params = [p.strip() for p in match.group(1).split(",") if p.strip() not in ("", "void")]
        assert len(params) == len(argtypes), f"{name}: header {len(params)}, binding {len(argtypes)}"
        for param, argtype in zip(params, argtypes):
            declared = "pointer" if "*" in param else (
                "float" if re.match(r"(const\s+)?(float|double)\b", param) else "int")
            kind = "pointer" if issubclass(argtype, ctypes._Pointer) else kinds[argtype]
            assert kind == declared, f"{name}: '{param}' bound as {argtype.__name__}"


def test_invalid_arguments_fail_before_any_gpu_work():
    lib = nat.lib
    size = ctypes.c_size_t()
    assert lib.gs_bin_count_workspace(-1, ctypes.byref(size)) == 1
    assert lib.gs_bin_count_workspace(2**31, ctypes.byref(size)) == 2
    assert b"too many" in lib.gs_last_error()
    assert lib.gs_project_forward(*([None] * 11), -1, 0, 1, 1, 8, 8, 0.2, 100.0,
                                  None, None, None, None, None) == 1
    assert lib.gs_project_forward(*([None] * 11), 4, 1, 1, 1, 8, 8, 0.2, 100.0,
                                  None, None, None, None, None) == 1
    assert b"SH degree" in lib.gs_last_error()
    # projection buffers moved as vectors must be aligned (checked before any GPU work)
    a16, a8, odd = ctypes.c_void_p(4096), ctypes.c_void_p(4104), ctypes.c_void_p(4100)
    assert lib.gs_project_forward(a16, odd, a8, a16, a16, a16, *([None] * 5), -1, 1, 1, 4, 8, 8,
                                  0.2, 100.0, a16, a8, None, a16, None) == 1
    assert b"16-byte aligned" in lib.gs_last_error()
    assert lib.gs_project_forward(a16, a16, odd, a16, a16, a16, *([None] * 5), -1, 1, 1, 4, 8,
                                  8, 0.2, 100.0, a16, a8, None, a16, None) == 1
    assert b"8-byte aligned" in lib.gs_last_error()
    assert lib.gs_project_backward(a16, a16, a8, a16, a16, None, None, -1, 1, 1, 4, a8, a8,
                                   None, *([a16] * 11), None) == 1
    assert b"16-byte aligned" in lib.gs_last_error()
    # ragged projection: the per-scene surfel offsets are required
    assert lib.gs_project_forward_ragged(*([None] * 11), 0, 1, 1, None, 1, 8, 8, 0.2, 100.0,
                                         None, None, None, None, None) == 1
    assert b"NULL offsets" in lib.gs_last_error()
    assert lib.gs_project_backward_ragged(*([None] * 7), 0, 1, 1, None, 1, 1,
                                          *([None] * 14), None) == 1
    assert b"invalid offsets" in lib.gs_last_error()
    assert lib.gs_pack_rows(None, 4, 17, None, None) == 1
    assert lib.gs_sh_forward(None, None, None, 4, 1, 1, 1, None, None) == 1
    assert lib.gs_composite_forward(None, None, 0, None, 1, 1, 0, 0, None, None, None, 0, 8, 8, 0,
                                    0, 0.2, 100.0, None, None, None, None, None) == 1
    assert lib.gs_composite_forward(None, None, 7, None, 1, 1, 0, 0, ctypes.c_void_p(16),
                                     None, ctypes.c_void_p(16), 1, 8, 8, 0, 0, 0.2, 100.0,
                                     None, None, None, None, None) == 1
    assert b"row mode" in lib.gs_last_error()
    # split-plane compositor: a missing plane or a plane stride below its channel count
    fake = ctypes.c_void_p(16)
    planes, planes_ptr = nat.host_array(ctypes.c_void_p, [16, 16, None, 16, 16])
    strides, strides_ptr = nat.host_array(ctypes.c_int64, [3, 1, 1, 3, 1])
    assert lib.gs_composite_forward_split(None, None, 0, None, 1, 1, 0, 0, fake, None, fake, 1,
                                          8, 8, 0, 0, 0.2, 100.0, planes_ptr, strides_ptr, None,
                                          0, None, None, None, 0, fake, fake, None, 0, None,
                                          None) == 1
    assert b"bad plane 2" in lib.gs_last_error()
    planes, planes_ptr = nat.host_array(ctypes.c_void_p, [16] * 5)
    strides, strides_ptr = nat.host_array(ctypes.c_int64, [2, 1, 1, 3, 1])
    assert lib.gs_composite_forward_split(None, None, 0, None, 1, 1, 0, 0, fake, None, fake, 1,
                                          8, 8, 0, 0, 0.2, 100.0, planes_ptr, strides_ptr, None,
                                          0, None, None, None, 0, fake, fake, None, 0, None,
                                          None) == 1
    assert b"bad plane 0" in lib.gs_last_error()
    strides, strides_ptr = nat.host_array(ctypes.c_int64, [3, 1, 1, 3, 1])
    assert lib.gs_composite_forward_split(None, None, 0, None, 1, 1, 0, 0, fake, None, fake, 1,
                                          8, 8, 0, 0, 0.2, 100.0, planes_ptr, strides_ptr, fake,
                                          1, None, None, None, 0, fake, fake, None, 0, None,
                                          None) == 1
    assert b"median depth needs its index" in lib.gs_last_error()
    assert lib.gs_composite_forward_split(None, None, 0, None, 1, 1, 0, 0, fake, None, fake, 1,
                                          8, 8, 0, 0, 0.2, 100.0, planes_ptr, strides_ptr, None,
                                          0, None, fake, None, 0, fake, fake, None, 0, None,
                                          None) == 1
    assert b"selected-pixel groups" in lib.gs_last_error()
    grad_strides, grad_strides_ptr = nat.host_array(ctypes.c_int64, [3, 1, 1, 0, 1, 0, 3, -1, 1, 0])
    assert lib.gs_composite_backward_split(None, None, 0, None, 1, 1, 0, 0, fake, None, fake, fake,
                                           fake, planes_ptr, grad_strides_ptr, None, None, 0, None,
                                           None, 0, 1, 8, 8, 0, 0.2, 100.0, None, None, None, fake,
                                           None, 0, None, None) == 1
    assert b"negative stride" in lib.gs_last_error()
    # warp accept masks need a positive plane size
    assert lib.gs_composite_forward_split(None, None, 0, None, 1, 1, 0, 0, fake, None, fake, 1,
                                          8, 8, 0, 0, 0.2, 100.0, planes_ptr, strides_ptr, None,
                                          0, None, None, None, 0, fake, fake, fake, 0, None,
                                          None) == 1
    assert b"warp masks" in lib.gs_last_error()
    grad_strides, grad_strides_ptr = nat.host_array(ctypes.c_int64, [3, 1, 1, 0, 1, 0, 3, 1, 1, 0])
    assert lib.gs_composite_backward_split(None, None, 0, None, 1, 1, 0, 0, fake, None, fake, fake,
                                           fake, planes_ptr, grad_strides_ptr, None, None, 0, None,
                                           None, 0, 1, 8, 8, 0, 0.2, 100.0, None, None, None, fake,
                                           fake, 0, None, None) == 1
    assert b"warp masks" in lib.gs_last_error()
    # metadata ids and the FP32 probe: sizes checked before any GPU work
    assert lib.gs_pair_ids(None, -1, 2, 3, None, None, None, None) == 1
    assert lib.gs_pair_ids(None, 4, 0, 3, None, None, None, None) == 1
    assert b"gs_pair_ids" in lib.gs_last_error()
    assert lib.gs_pair_ids(None, 0, 2, 3, None, None, None, None) == 0   # nothing to do
    assert lib.gs_fp32_probe(0, 10, 0, fake, None) == 1
    assert lib.gs_fp32_probe(1, 10, 0, None, None) == 1
    assert b"gs_fp32_probe" in lib.gs_last_error()
    # arena binning: capacities checked before any GPU work
    assert lib.gs_bin_arena_workspace(10, 0, 0, 1, 8, 8, ctypes.byref(size)) == 1
    assert lib.gs_bin_arena_workspace(10, 5, 6, 1, 8, 8, ctypes.byref(size)) == 1   # spans > slots
    assert lib.gs_bin_arena_workspace(10, 2**31, 6, 1, 8, 8, ctypes.byref(size)) == 2
    # fused Adam: table and hyper-parameter checks
    assert lib.gs_adam_step(-1, None, None, None, None, None, 0.1, 0.9, 0.999, 1e-8, 0.0, 1,
                            None) == 1
    assert lib.gs_adam_step(0, None, None, None, None, None, 0.1, 0.9, 0.999, 1e-8, 0.0, 0,
                            None) == 1
    assert b"step counts from 1" in lib.gs_last_error()
    assert lib.gs_adam_step(0, None, None, None, None, None, 0.1, 1.0, 0.999, 1e-8, 0.0, 1,
                            None) == 1
    assert lib.gs_adam_step(0, None, None, None, None, None, 0.1, 0.9, 0.999, 1e-8, 0.0, 1,
                            None) == 0   # nothing to do
    # capturable Adam: step table required, same hyper-parameter checks
    one, one_ptr = nat.host_array(ctypes.c_int64, [1])
    ptrs, ptrs_ptr = nat.host_array(ctypes.c_void_p, [16])
    assert lib.gs_adam_step_capturable(1, ptrs_ptr, ptrs_ptr, ptrs_ptr, ptrs_ptr, one_ptr, None,
                                       0.1, 0.9, 0.999, 1e-8, 0.0, None, None) == 1
    assert b"NULL step table" in lib.gs_last_error()
    assert lib.gs_adam_step_capturable(0, None, None, None, None, None, None, 0.1, 0.9, 1.5,
                                       1e-8, 0.0, None, None) == 1
    assert b"hyper-parameters" in lib.gs_last_error()
    assert lib.gs_adam_step_capturable(0, None, None, None, None, None, None, 0.1, 0.9, 0.999,
                                       1e-8, 0.0, None, None) == 0   # nothing to do
    # tiles beyond int32
    assert lib.gs_bin_sort_workspace(10, 10**10, 10, 1, 8, 8, ctypes.byref(size)) == 2
    assert lib.gs_bin_sort_workspace(10, 5, 6, 1, 8, 8, ctypes.byref(size)) == 1   # spans > slots


def test_check_values_messages_match_reference():
    golden = load_golden("check_values.npz")
    base = small_inputs("classic", device="cpu")
    base = {k: v.detach() for k, v in base.items()}
    mutations = {
        "nonfinite_means": ("means", lambda v: v.__setitem__((0, 0, 0), float("nan"))),
        "negative_scales": ("scales", lambda v: v.neg_()),
        "zero_quaternions": ("quaternions", lambda v: v.zero_()),
        "opacity_two": ("opacities", lambda v: v.fill_(2.0)),
        "transposed_intrinsics": ("intrinsics", lambda v: v.copy_(v.transpose(-1, -2).clone())),
        "view_last_row": ("view_matrices", lambda v: v.__setitem__((0, 0, 3, 0), 0.5)),
        "view_scaled": ("view_matrices", lambda v: v[..., :3, :3].mul_(1.1)),
        "view_reflection": ("view_matrices", lambda v: v[..., 0, :3].neg_()),
        "negative_focal": ("intrinsics", lambda v: v[..., 0, 0].neg_()),
        "weights_sum": ("frequency_weights", lambda v: v.fill_(0.3)),
        "negative_weights": ("frequency_weights", lambda v: v.__setitem__((0, 0, 0), -0.25)),
        "negative_magnitudes": ("frequency_magnitudes", lambda v: v.neg_()),
    }
    names = ["colors", "secondary_colors", "frequency_weights", "frequency_magnitudes", "phases"]
    for case, expected in zip(golden["cases"], golden["messages"]):
        name, mutate = mutations[str(case)]
        v = {k: t.clone() for k, t in base.items()}
        mutate(v[name])
        tensors = {k: (t, None) for k, t in v.items()}
        if not str(expected):
            check_values(tensors, v["quaternions"], v["scales"], v["opacities"],
                         v["view_matrices"], v["intrinsics"], [v[k] for k in names], False)
            continue
        with pytest.raises(ValueError) as info:
            check_values(tensors, v["quaternions"], v["scales"], v["opacities"],
                         v["view_matrices"], v["intrinsics"], [v[k] for k in names], False)
        assert str(info.value) == str(expected), case


def test_structural_checks_raise_reference_exception_types():
    v = {k: t.detach() for k, t in small_inputs("classic", device="cpu").items()}
    with pytest.raises(ValueError, match="CUDA float32"):
        rasterize_gabors(**v, width=9, height=9)
    with pytest.raises(ValueError, match="shape"):
        rasterize_gabors(**dict(v, means=v["means"][0, 0]), width=9, height=9)
    n = {k: t.detach() for k, t in small_inputs("neural", device="cpu").items()}
    with pytest.raises(ValueError):
        rasterize_neural_gabors(**n, width=9, height=9)
    with pytest.raises(TypeError):
        check_tensor("means", [1.0], (1,), torch.device("cpu"))
    with pytest.raises(ValueError, match="x must be float32 on cpu"):
        check_tensor("x", torch.zeros(2), (2,), torch.device("cpu"))


def test_golden_fixture_inventory():
    """Every fixture file the parity tests rely on is present and non-trivial."""
    for name in ("projection.npz", "render.npz", "sh.npz", "check_values.npz"):
        data = load_golden(name)
        assert len(data) >= 2 and all(np.asarray(v).size for v in data.values()), name
