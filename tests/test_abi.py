"""The C-ABI library: it loads, exports what the header declares, and rejects bad arguments
before touching a device (no GPU needed)."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

import rocmkernels_b200
from rocmkernels_b200 import attention as api

REPO = Path(__file__).resolve().parent.parent
HEADERS = sorted((REPO / "include").glob("*.h"))


def declared_functions():
    names = []
    for header in HEADERS:
        text = header.read_text()
        names += re.findall(r"ROCMKERNELS_C_EXPORT\s+[\w\s\*]+?\b(\w+)\s*\(", text)
    return names


def test_library_loads_and_reports_sm100a():
    assert "sm_100a" in rocmkernels_b200.build_info()


def test_every_declared_symbol_is_exported():
    names = declared_functions()
    assert len(names) >= 14
    library = rocmkernels_b200.lib()
    for name in names:
        assert hasattr(library, name), name
    exported = subprocess.run(["nm", "-D", "--defined-only", str(api.LIBRARY_PATH)], capture_output=True, text=True,
                              check=True).stdout
    for name in names:
        assert re.search(rf"\bT {name}$", exported, re.M), name


def test_reference_entry_points_all_declared():
    reference_names = {
        "attention_fp32_forward", "attention_fp32_forward_tiled", "attention_fp32_backward", "attention_fp32_backward_tiled",
        "attention_fp32_statistics", "attention_fp32_forward_tuned", "attention_fp32_forward_flash",
        "attention_fp32_forward_flash_tuned", "attention_fp32_backward_tuned", "attention64_fp32_forward",
        "attention64_fp32_backward", "attention_fp32_backward_profile", "attention_fp32_query_profile",
        "attention_generic_forward", "rotary_fp32",
    }
    assert reference_names <= set(declared_functions())
    assert reference_names == set(api.ENTRY_POINTS)


def test_strides_struct_layout():
    assert ctypes.sizeof(api.Strides) == 12


S = api.Strides(0, 0, 0)
FWD = dict(q=1, k=1, v=1, mask=1, output=1, lse=1)


def forward_args(**override):
    a = dict(FWD, batch=1, heads=1, queries=4, keys=4, radius=-1)
    a.update(override)
    return [a["q"], a["k"], a["v"], a["mask"], a["output"], a["lse"], a["batch"], a["heads"], a["queries"], a["keys"], a["radius"]]


@pytest.mark.parametrize("entry", ["attention_fp32_forward", "attention_fp32_forward_tiled", "attention_fp32_forward_flash",
                                   "attention64_fp32_forward"])
@pytest.mark.parametrize("override", [dict(q=None), dict(k=None), dict(v=None), dict(mask=None), dict(output=None),
                                      dict(lse=None), dict(batch=0), dict(heads=-1), dict(queries=0), dict(keys=0)])
def test_forward_rejects_invalid_arguments(entry, override):
    assert getattr(api, entry)(*forward_args(**override), S, S, S, S) == api.INVALID_VALUE


def test_radius_validation_matches_reference():
    # Flash and statistics reject radius < -1 (Attention.hip:376, :255); simple/tiled/64 do not check it.
    assert api.attention_fp32_forward_flash(*forward_args(radius=-2), S, S, S, S) == api.INVALID_VALUE
    assert api.attention_fp32_statistics(1, 1, 1, 1, 1, 1, 4, 4, -2, S, S) == api.INVALID_VALUE
    assert api.attention_fp32_forward_flash_tuned(*forward_args(radius=-2), 13, S, S, S, S) == api.INVALID_VALUE


@pytest.mark.parametrize("variant", [-1, 19, 100])
def test_flash_variant_out_of_range(variant):
    assert api.attention_fp32_forward_flash_tuned(*forward_args(), variant, S, S, S, S) == api.INVALID_VALUE


@pytest.mark.parametrize("group", [0, 1, 3, 16, 1165])
def test_unknown_tuning_groups(group):
    assert api.attention_fp32_forward_tuned(*forward_args(), group, S, S, S, S) == api.INVALID_VALUE
    bwd = [1] * 11 + [1, 1, 4, 4, -1]
    assert api.attention_fp32_backward_tuned(*bwd, group, S, S, S, S, S) == api.INVALID_VALUE


@pytest.mark.parametrize("entry", ["attention_fp32_backward", "attention_fp32_backward_tiled", "attention64_fp32_backward"])
@pytest.mark.parametrize("null_index", range(11))
def test_backward_rejects_null_pointers(entry, null_index):
    pointers = [1] * 11
    pointers[null_index] = None
    assert getattr(api, entry)(*pointers, 1, 1, 4, 4, -1, S, S, S, S, S) == api.INVALID_VALUE


def test_profile_entries_validate_like_reference():
    ok = [1] * 11
    # stage outside 1..3, queries < 32, radius < -1 (Attention.hip:331-334)
    assert api.attention_fp32_backward_profile(*ok, 1, 1, 64, 64, -1, 0, S, S, S, S, S) == api.INVALID_VALUE
    assert api.attention_fp32_backward_profile(*ok, 1, 1, 64, 64, -1, 4, S, S, S, S, S) == api.INVALID_VALUE
    assert api.attention_fp32_backward_profile(*ok, 1, 1, 31, 64, -1, 1, S, S, S, S, S) == api.INVALID_VALUE
    assert api.attention_fp32_backward_profile(*ok, 1, 1, 64, 64, -2, 1, S, S, S, S, S) == api.INVALID_VALUE
    # tuning ids accepted by the reference are 14, 18, 24, 28, 44, 116 (Attention.hip:346-353)
    assert api.attention_fp32_query_profile(*ok, 1, 1, 64, 64, -1, 15, S, S, S, S, S) == api.INVALID_VALUE
    assert api.attention_fp32_query_profile(*ok, 1, 1, 16, 64, -1, 14, S, S, S, S, S) == api.INVALID_VALUE


def test_throwing_wrappers_raise_hip_error():
    with pytest.raises(api.HipError) as error:
        api.AttentionForwardFlash(*forward_args(q=None), S, S, S, S)
    assert error.value.status == api.INVALID_VALUE


def generic_args(head_width=32, dtype=api.DType.Float32, **override):
    return [*forward_args(**override)[:10], head_width, override.get("radius", -1), S, S, S, S, dtype]


@pytest.mark.parametrize("override", [dict(q=None), dict(k=None), dict(v=None), dict(mask=None), dict(output=None),
                                      dict(lse=None), dict(batch=0), dict(heads=-1), dict(queries=0), dict(keys=0),
                                      dict(radius=-2)])
@pytest.mark.parametrize("dtype", list(api.DType))
def test_generic_forward_rejects_invalid_arguments(override, dtype):
    # AttentionGeneric.hip:295-297: null pointers, non-positive sizes, radius < -1
    assert api.attention_generic_forward(*generic_args(dtype=dtype, **override)) == api.INVALID_VALUE


@pytest.mark.parametrize("head_width", [0, 8, 17, 48, 128])
def test_generic_forward_rejects_head_width(head_width):
    # AttentionGeneric.hip:296: only 16, 32 and 64
    assert api.attention_generic_forward(*generic_args(head_width=head_width)) == api.INVALID_VALUE


@pytest.mark.parametrize("dtype", [2, 3, 255])
def test_generic_forward_rejects_unknown_dtype(dtype):
    # AttentionGeneric.hip:306-307: any other DType value
    assert api.attention_generic_forward(*generic_args(dtype=dtype)) == api.INVALID_VALUE


def test_generic_wrapper_raises_hip_error():
    with pytest.raises(api.HipError) as error:
        api.AttentionGenericForward(*generic_args(head_width=24))
    assert error.value.status == api.INVALID_VALUE


@pytest.mark.parametrize("head_width", [16, 32, 64])
def test_generic_dispatch_names(head_width):
    # Contiguous tensors: FP16 storage on the FP16 tensor-core kernel, FP32 on the split one.
    assert api.generic_kernel_name(2, 8, 512, 512, head_width, api.DType.Float16) == f"tcgen05-f16-flash-d{head_width}"
    assert api.generic_kernel_name(2, 8, 512, 512, head_width, api.DType.Float32) == f"tcgen05-f16x2-flash-d{head_width}"
    assert api.generic_kernel_name(1, 1, 4, 4, 24, api.DType.Float16) == "unsupported"


@pytest.mark.parametrize("null_index", range(6))
def test_rotary_rejects_null_pointers(null_index):
    # Rotary.hip:47-48: any null pointer, non-positive batch, heads or length
    pointers = [1] * 6
    pointers[null_index] = None
    assert api.rotary_fp32(*pointers, 1, 1, 1, 0, S, S, S, S) == api.INVALID_VALUE


@pytest.mark.parametrize("sizes", [(0, 1, 1), (1, 0, 1), (1, 1, 0), (-1, 2, 2)])
def test_rotary_rejects_sizes(sizes):
    assert api.rotary_fp32(1, 1, 1, 1, 1, 1, *sizes, 1, S, S, S, S) == api.INVALID_VALUE
    with pytest.raises(api.HipError):
        api.Rotary(1, 1, 1, 1, 1, 1, *sizes, True, S, S, S, S)


@pytest.mark.parametrize("null_index", range(8))
def test_fused_rotary_flash_rejects_null_pointers(null_index):
    pointers = [1] * 8  # q, k, v, cos, sin, mask, output, lse
    pointers[null_index] = None
    assert api.attention_fp32_forward_flash_rotary(*pointers, 1, 1, 4, 4, -1, S, S, S, S, S, S) == api.INVALID_VALUE


def test_fused_rotary_flash_rejects_radius():
    assert api.attention_fp32_forward_flash_rotary(*[1] * 8, 1, 1, 4, 4, -2, S, S, S, S, S, S) == api.INVALID_VALUE


def _cuda_device_visible() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.mark.skipif(_cuda_device_visible(), reason="boundary probe needs a machine without a CUDA device: the accepted "
                                                   "case would otherwise launch on stand-in pointers")
def test_static_delta_row_limit_boundary():
    """attention_fp32_backward_static_delta holds delta for at most 4,194,304 (batch, head, query)
    rows. Exactly that many pass the size check (the call then stops at the device lookup, which
    fails without a driver: an error other than 1); one more row is rejected with error 1 before
    any CUDA call."""
    limit = 1 << 22
    for (batch, heads, queries) in [(2, 16, 131072), (1, 1, limit), (4, 8, limit // 32)]:
        assert batch * heads * queries == limit
        status = api.attention_fp32_backward_static_delta(1, 1, 1, 1, 1, 1, 1, 1, 1, 1, batch, heads, queries, 64, -1, S, S, S, S, S)
        assert status not in (0, api.INVALID_VALUE), (batch, heads, queries, status)
    for (batch, heads, queries) in [(2, 16, 131073), (1, 1, limit + 1), (4097, 1024, 1)]:
        status = api.attention_fp32_backward_static_delta(1, 1, 1, 1, 1, 1, 1, 1, 1, 1, batch, heads, queries, 64, -1, S, S, S, S, S)
        assert status == api.INVALID_VALUE, (batch, heads, queries, status)


def test_fused_backward_workspace_size():
    """256 bytes per query (queries padded to 64 per (batch, head)) plus a 528-byte record per
    64 queries; 0 for non-positive sizes."""
    size = api.attention_fp32_backward_fused_workspace_size
    for batch, heads, queries in [(1, 1, 1), (2, 3, 64), (2, 3, 65), (64, 12, 4096), (1, 1, 1000)]:
        tiles = batch * heads * ((queries + 63) // 64)
        assert size(batch, heads, queries) == tiles * (64 * 256 + 528)
    assert size(0, 1, 1) == 0 and size(1, -1, 1) == 0 and size(1, 1, 0) == 0


@pytest.mark.parametrize("null_index", range(12))
def test_fused_backward_rejects_null_pointers_and_small_workspace(null_index):
    pointers = [1] * 12  # q, k, v, mask, output, lse, upstream, gradients, delta, workspace
    pointers[null_index] = None
    lib = api.lib()
    needed = api.attention_fp32_backward_fused_workspace_size(1, 1, 4)
    assert lib.attention_fp32_backward_fused(*pointers, needed, 1, 1, 4, 4, -1, S, S, S, S, S, None) == api.INVALID_VALUE
    # a workspace smaller than the size query asks for: error 1 before any CUDA call
    assert lib.attention_fp32_backward_fused(*[1] * 12, needed - 1, 1, 1, 4, 4, -1, S, S, S, S, S, None) == api.INVALID_VALUE


def test_forward_workspace_size():
    """16,400 bytes per 64-key tile of every (batch, head): the split K and V images (16,384) and
    a 16-byte stage header; 0 for non-positive sizes."""
    size = api.attention_fp32_forward_flash_workspace_size
    for batch, heads, keys in [(1, 1, 1), (2, 3, 64), (2, 3, 65), (8, 3, 1024), (64, 12, 4096)]:
        assert size(batch, heads, keys) == batch * heads * ((keys + 63) // 64) * 16400
    assert size(0, 1, 1) == 0 and size(1, -1, 1) == 0 and size(1, 1, 0) == 0


@pytest.mark.parametrize("rotary", [False, True], ids=["plain", "rotary"])
@pytest.mark.parametrize("null_index", range(9))
def test_forward_workspace_entries_reject_null_pointers_and_small_workspace(null_index, rotary):
    count = 9 if rotary else 7  # q, k, v, [cos, sin,] mask, output, lse, workspace
    if null_index >= count:
        pytest.skip("no such pointer")
    lib = api.lib()
    needed = api.attention_fp32_forward_flash_workspace_size(1, 1, 4)
    pointers = [1] * count
    pointers[null_index] = None
    if rotary:
        call = lambda ptrs, capacity: lib.attention_fp32_forward_flash_rotary_workspace(
            *ptrs[:8], 1, 1, 4, 4, -1, S, S, S, S, S, S, ptrs[8], capacity, None)
    else:
        call = lambda ptrs, capacity: lib.attention_fp32_forward_flash_workspace(
            *ptrs[:6], 1, 1, 4, 4, -1, S, S, S, S, ptrs[6], capacity, None)
    assert call(pointers, needed) == api.INVALID_VALUE
    # a workspace smaller than the size query asks for: error 1 before any CUDA call
    assert call([1] * count, needed - 1) == api.INVALID_VALUE
