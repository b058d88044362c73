"""Python binding of librocmkernels_attention.so (ctypes), mirroring the reference's interface.

The reference's host API is C++: ``extern "C"`` launchers plus namespaced wrappers that throw
``ROCmKernels::HipError`` (ROCmKernels.Kernels/include/ROCmKernels/Kernels/Attention/Attention.hpp:44-108,
Attention64.hpp:19-32, Generic/AttentionGeneric.hpp:15-25, Positional/Rotary.hpp:13-22). This
module exposes both layers under the same names:

* ``lib()`` returns the loaded library whose ``attention_fp32_*`` / ``attention64_fp32_*``
  functions return the raw status code (0 = success, 1 = invalid value, else a CUDA error);
* ``AttentionForward``, ``AttentionForwardFlash``, ... call them and raise :class:`HipError`
  on a non-zero status, with the same argument order and a default ``stream=None`` (the legacy
  default stream).

Pointer arguments accept an ``int`` device address or any object with ``data_ptr()`` (a torch
CUDA tensor). Strides are :class:`Strides` or 3-tuples ``(batch, head, token)`` in elements.
There is no CPU fallback: if the CUDA library is missing, :func:`lib` raises.
"""
from __future__ import annotations

import ctypes
import enum
import os
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
LIBRARY_PATH = PACKAGE_DIR / "librocmkernels_attention.so"

SUCCESS = 0
INVALID_VALUE = 1  # cudaErrorInvalidValue == hipErrorInvalidValue


class Strides(ctypes.Structure):
    """Element strides of a [batch][head][token] tensor (ROCmKernels::Kernels::Strides)."""

    _fields_ = [("batch", ctypes.c_int), ("head", ctypes.c_int), ("token", ctypes.c_int)]

    def __repr__(self) -> str:
        return f"Strides(batch={self.batch}, head={self.head}, token={self.token})"


class DType(enum.IntEnum):
    """Storage type of the generic forward (ROCmKernels::Kernels::DType, passed as one byte)."""

    Float32 = 0
    Float16 = 1


class HipError(RuntimeError):
    """Raised by the wrappers when an entry point returns a non-zero status (ROCmKernels::HipError)."""

    def __init__(self, status: int, function: str):
        self.status = int(status)
        super().__init__(f"{function} returned status {self.status} ({_error_name(self.status)})")


_POINTER = ctypes.c_void_p
_INT = ctypes.c_int
_FORWARD_ARGS = [_POINTER] * 6 + [_INT] * 5 + [Strides] * 4 + [_POINTER]
_FORWARD_SELECT_ARGS = [_POINTER] * 6 + [_INT] * 6 + [Strides] * 4 + [_POINTER]
_BACKWARD_ARGS = [_POINTER] * 11 + [_INT] * 5 + [Strides] * 5 + [_POINTER]
_BACKWARD_SELECT_ARGS = [_POINTER] * 11 + [_INT] * 6 + [Strides] * 5 + [_POINTER]
_SIGNATURES = {
    "attention_fp32_forward": _FORWARD_ARGS,
    "attention_fp32_forward_tiled": _FORWARD_ARGS,
    "attention_fp32_forward_flash": _FORWARD_ARGS,
    "attention64_fp32_forward": _FORWARD_ARGS,
    "attention_fp32_forward_tuned": _FORWARD_SELECT_ARGS,
    "attention_fp32_forward_flash_tuned": _FORWARD_SELECT_ARGS,
    "attention_fp32_backward": _BACKWARD_ARGS,
    "attention_fp32_backward_tiled": _BACKWARD_ARGS,
    "attention64_fp32_backward": _BACKWARD_ARGS,
    "attention_fp32_backward_tuned": _BACKWARD_SELECT_ARGS,
    "attention_fp32_backward_profile": _BACKWARD_SELECT_ARGS,
    "attention_fp32_query_profile": _BACKWARD_SELECT_ARGS,
    "attention_fp32_statistics": [_POINTER] * 4 + [_INT] * 5 + [Strides] * 2 + [_POINTER],
    "attention_generic_forward": [_POINTER] * 6 + [_INT] * 6 + [Strides] * 4 + [ctypes.c_ubyte, _POINTER],
    "rotary_fp32": [_POINTER] * 6 + [_INT] * 4 + [Strides] * 4 + [_POINTER],
}
ENTRY_POINTS = tuple(_SIGNATURES)

_lib = None


def lib() -> ctypes.CDLL:
    """Loads the in-tree CUDA library (once). Raises if it has not been built."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("ROCMKERNELS_ATTENTION_LIBRARY", LIBRARY_PATH))
        if not path.exists():
            raise RuntimeError(f"{path} is missing: build the sm_100a library with `python -m rocmkernels_b200.build`")
        library = ctypes.CDLL(str(path))
        for name, argtypes in _SIGNATURES.items():
            function = getattr(library, name)
            function.argtypes = argtypes
            function.restype = ctypes.c_int
        library.rocmkernels_attention_build_info.argtypes = []
        library.rocmkernels_attention_build_info.restype = ctypes.c_char_p
        library.rocmkernels_attention_flash_kernel.argtypes = [ctypes.c_int] * 5
        library.rocmkernels_attention_flash_kernel.restype = ctypes.c_char_p
        library.rocmkernels_attention_generic_kernel.argtypes = [ctypes.c_int] * 5 + [ctypes.c_ubyte]
        library.rocmkernels_attention_generic_kernel.restype = ctypes.c_char_p
        library.rocmkernels_attention_device_status.argtypes = [ctypes.c_int]
        library.rocmkernels_attention_device_status.restype = ctypes.c_uint
        library.attention_fp32_forward_flash_workspace.argtypes = ([_POINTER] * 6 + [_INT] * 5 + [Strides] * 4 +
                                                                   [_POINTER, ctypes.c_ulonglong, _POINTER])
        library.attention_fp32_forward_flash_workspace.restype = ctypes.c_int
        library.attention_fp32_forward_flash_rotary_workspace.argtypes = ([_POINTER] * 8 + [_INT] * 5 + [Strides] * 6 +
                                                                          [_POINTER, ctypes.c_ulonglong, _POINTER])
        library.attention_fp32_forward_flash_rotary_workspace.restype = ctypes.c_int
        library.attention_fp32_forward_flash_workspace_size.argtypes = [_INT] * 3
        library.attention_fp32_forward_flash_workspace_size.restype = ctypes.c_ulonglong
        library.rocmkernels_attention_flash_workspace_kernel.argtypes = [ctypes.c_int] * 4
        library.rocmkernels_attention_flash_workspace_kernel.restype = ctypes.c_char_p
        library.attention_fp32_backward_static_delta.argtypes = [_POINTER] * 10 + [_INT] * 5 + [Strides] * 5 + [_POINTER]
        library.attention_fp32_backward_static_delta.restype = ctypes.c_int
        library.attention_fp32_backward_fused.argtypes = ([_POINTER] * 12 + [ctypes.c_ulonglong] + [_INT] * 5 + [Strides] * 5
                                                          + [_POINTER])
        library.attention_fp32_backward_fused.restype = ctypes.c_int
        library.attention_fp32_backward_fused_workspace_size.argtypes = [_INT] * 3
        library.attention_fp32_backward_fused_workspace_size.restype = ctypes.c_ulonglong
        library.attention_fp32_forward_flash_rotary.argtypes = [_POINTER] * 8 + [_INT] * 5 + [Strides] * 6 + [_POINTER]
        library.attention_fp32_forward_flash_rotary.restype = ctypes.c_int
        _lib = library
    return _lib


def build_info() -> str:
    return lib().rocmkernels_attention_build_info().decode()


def flash_kernel_name(batch: int, heads: int, queries: int, keys: int, head_width: int = 32) -> str:
    """Name of the kernel attention_fp32_forward_flash runs for contiguous, 16-byte aligned inputs."""
    return lib().rocmkernels_attention_flash_kernel(batch, heads, queries, keys, head_width).decode()


def generic_kernel_name(batch: int, heads: int, queries: int, keys: int, head_width: int, dtype: DType) -> str:
    """Name of the kernel attention_generic_forward runs for contiguous, 16-byte aligned inputs."""
    return lib().rocmkernels_attention_generic_kernel(batch, heads, queries, keys, head_width, int(dtype)).decode()


def device_status(clear: bool = True) -> int:
    """Status word of the tensor-core kernels on the current device (0 = no failed pipeline wait).
    Synchronizes with the device."""
    return int(lib().rocmkernels_attention_device_status(int(clear)))


def _error_name(status: int) -> str:
    try:
        import torch  # noqa: F401  (cudart is linked into the library, torch only helps naming)
        from torch.cuda import cudart

        return str(cudart().cudaGetErrorString(status))
    except Exception:  # pragma: no cover - naming is best effort
        return "see cudaError_t"


def ptr(value) -> int | None:
    """Device address of a tensor / int / None."""
    if value is None:
        return None
    if isinstance(value, int):
        return value
    return int(value.data_ptr())


def strides(value) -> Strides:
    if isinstance(value, Strides):
        return value
    batch, head, token = value
    return Strides(int(batch), int(head), int(token))


def strides_of(tensor) -> Strides:
    """Strides of a [batch, heads, tokens, D] tensor whose feature stride is 1."""
    if tensor.dim() != 4 or tensor.stride(3) != 1:
        raise ValueError("expected a [batch, heads, tokens, D] tensor with unit feature stride")
    return Strides(tensor.stride(0), tensor.stride(1), tensor.stride(2))


def _stream(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


def _call(name: str, *args) -> int:
    return getattr(lib(), name)(*args)


def _forward(name, q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream, *select):
    return _call(name, ptr(q), ptr(k), ptr(v), ptr(mask), ptr(output), ptr(lse), batch, heads, queries, keys, radius,
                 *select, strides(qs), strides(ks), strides(vs), strides(os_), _stream(stream))


def _backward(name, q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, qs, ks,
              vs, os_, us, stream, *select):
    return _call(name, ptr(q), ptr(k), ptr(v), ptr(mask), ptr(output), ptr(lse), ptr(upstream), ptr(gq), ptr(gk),
                 ptr(gv), ptr(delta), batch, heads, queries, keys, radius, *select, strides(qs), strides(ks), strides(vs),
                 strides(os_), strides(us), _stream(stream))


# Raw entry points: return the status code like the C functions.
def attention_fp32_forward(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream=None):
    return _forward("attention_fp32_forward", q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream)


def attention_fp32_forward_tiled(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream=None):
    return _forward("attention_fp32_forward_tiled", q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream)


def attention_fp32_forward_flash(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream=None):
    return _forward("attention_fp32_forward_flash", q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream)


def attention64_fp32_forward(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream=None):
    return _forward("attention64_fp32_forward", q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream)


def attention_fp32_forward_tuned(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, group, qs, ks, vs, os_, stream=None):
    return _forward("attention_fp32_forward_tuned", q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream, group)


def attention_fp32_forward_flash_tuned(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, variant, qs, ks, vs, os_,
                                       stream=None):
    return _forward("attention_fp32_forward_flash_tuned", q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs,
                    os_, stream, variant)


def attention_fp32_statistics(q, k, mask, lse, batch, heads, queries, keys, radius, qs, ks, stream=None):
    return _call("attention_fp32_statistics", ptr(q), ptr(k), ptr(mask), ptr(lse), batch, heads, queries, keys, radius,
                 strides(qs), strides(ks), _stream(stream))


def attention_fp32_backward(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, qs, ks, vs,
                            os_, us, stream=None):
    return _backward("attention_fp32_backward", q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys,
                     radius, qs, ks, vs, os_, us, stream)


def attention_fp32_backward_static_delta(q, k, v, mask, output, lse, upstream, gq, gk, gv, batch, heads, queries, keys, radius,
                                         qs, ks, vs, os_, us, stream=None):
    """attention_fp32_backward with the delta scratch held by the library (no delta argument)."""
    return _call("attention_fp32_backward_static_delta", ptr(q), ptr(k), ptr(v), ptr(mask), ptr(output), ptr(lse),
                 ptr(upstream), ptr(gq), ptr(gk), ptr(gv), batch, heads, queries, keys, radius, strides(qs), strides(ks),
                 strides(vs), strides(os_), strides(us), _stream(stream))


def attention_fp32_backward_fused_workspace_size(batch, heads, queries) -> int:
    """Bytes of device workspace attention_fp32_backward_fused needs for these sizes."""
    return int(lib().attention_fp32_backward_fused_workspace_size(batch, heads, queries))


def attention_fp32_backward_fused(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, qs, ks,
                                  vs, os_, us, stream=None, workspace=None):
    """attention_fp32_backward in one key-major pass (dQ added with FP32 atomics: its summation
    order over key tiles is not fixed). `workspace`: a device buffer (a torch tensor or a pointer)
    of attention_fp32_backward_fused_workspace_size bytes; None allocates one with torch on q's
    device (the caching allocator reuses it across calls)."""
    size = attention_fp32_backward_fused_workspace_size(batch, heads, queries)
    if workspace is None:
        import torch

        workspace = torch.empty(max(size, 1), dtype=torch.uint8, device=q.device)
    capacity = workspace.numel() * workspace.element_size() if hasattr(workspace, "numel") else size
    return _call("attention_fp32_backward_fused", ptr(q), ptr(k), ptr(v), ptr(mask), ptr(output), ptr(lse), ptr(upstream), ptr(gq),
                 ptr(gk), ptr(gv), ptr(delta), ptr(workspace), capacity, batch, heads, queries, keys, radius, strides(qs), strides(ks),
                 strides(vs), strides(os_), strides(us), _stream(stream))


def attention_fp32_backward_tiled(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, qs, ks,
                                  vs, os_, us, stream=None):
    return _backward("attention_fp32_backward_tiled", q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries,
                     keys, radius, qs, ks, vs, os_, us, stream)


def attention64_fp32_backward(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, qs, ks, vs,
                              os_, us, stream=None):
    return _backward("attention64_fp32_backward", q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys,
                     radius, qs, ks, vs, os_, us, stream)


def attention_fp32_backward_tuned(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, group,
                                  qs, ks, vs, os_, us, stream=None):
    return _backward("attention_fp32_backward_tuned", q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries,
                     keys, radius, qs, ks, vs, os_, us, stream, group)


def attention_fp32_backward_profile(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, stage,
                                    qs, ks, vs, os_, us, stream=None):
    return _backward("attention_fp32_backward_profile", q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries,
                     keys, radius, qs, ks, vs, os_, us, stream, stage)


def attention_fp32_query_profile(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, tuning,
                                 qs, ks, vs, os_, us, stream=None):
    return _backward("attention_fp32_query_profile", q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries,
                     keys, radius, qs, ks, vs, os_, us, stream, tuning)


def attention_generic_forward(q, k, v, mask, output, lse, batch, heads, queries, keys, head_width, radius, qs, ks, vs, os_, dtype,
                              stream=None):
    return _call("attention_generic_forward", ptr(q), ptr(k), ptr(v), ptr(mask), ptr(output), ptr(lse), batch, heads, queries,
                 keys, head_width, radius, strides(qs), strides(ks), strides(vs), strides(os_), int(dtype), _stream(stream))


def rotary_fp32(q, k, cos, sin, oq, ok, batch, heads, length, backward, qs, ks, cs, ss, stream=None):
    return _call("rotary_fp32", ptr(q), ptr(k), ptr(cos), ptr(sin), ptr(oq), ptr(ok), batch, heads, length, int(bool(backward)),
                 strides(qs), strides(ks), strides(cs), strides(ss), _stream(stream))


def attention_fp32_forward_flash_workspace_size(batch, heads, keys) -> int:
    """Bytes of device workspace attention_fp32_forward_flash_workspace needs for these sizes."""
    return int(lib().attention_fp32_forward_flash_workspace_size(batch, heads, keys))


def flash_workspace_kernel_name(batch: int, heads: int, queries: int, keys: int) -> str:
    """Name of the kernel attention_fp32_forward_flash_workspace runs for contiguous, 16-byte
    aligned inputs ("...-prepared": the operand pre-pass and the forward)."""
    return lib().rocmkernels_attention_flash_workspace_kernel(batch, heads, queries, keys).decode()


def _forward_workspace(q, workspace, size):
    if workspace is None:
        import torch

        workspace = torch.empty(max(size, 1), dtype=torch.uint8, device=q.device)
    capacity = workspace.numel() * workspace.element_size() if hasattr(workspace, "numel") else size
    return workspace, capacity


def attention_fp32_forward_flash_workspace(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_,
                                           stream=None, workspace=None):
    """attention_fp32_forward_flash with caller scratch for the split K/V operands (see the C
    header). `workspace`: a device buffer (a torch tensor or a pointer) of
    attention_fp32_forward_flash_workspace_size bytes; None allocates one with torch on q's device."""
    workspace, capacity = _forward_workspace(q, workspace, attention_fp32_forward_flash_workspace_size(batch, heads, keys))
    return _call("attention_fp32_forward_flash_workspace", ptr(q), ptr(k), ptr(v), ptr(mask), ptr(output), ptr(lse), batch, heads,
                 queries, keys, radius, strides(qs), strides(ks), strides(vs), strides(os_), ptr(workspace), capacity,
                 _stream(stream))


def attention_fp32_forward_flash_rotary_workspace(q, k, v, cos, sin, mask, output, lse, batch, heads, queries, keys, radius, qs, ks,
                                                  vs, cs, ss, os_, stream=None, workspace=None):
    """attention_fp32_forward_flash_rotary with caller scratch, as attention_fp32_forward_flash_workspace."""
    workspace, capacity = _forward_workspace(q, workspace, attention_fp32_forward_flash_workspace_size(batch, heads, keys))
    return _call("attention_fp32_forward_flash_rotary_workspace", ptr(q), ptr(k), ptr(v), ptr(cos), ptr(sin), ptr(mask), ptr(output),
                 ptr(lse), batch, heads, queries, keys, radius, strides(qs), strides(ks), strides(vs), strides(cs), strides(ss),
                 strides(os_), ptr(workspace), capacity, _stream(stream))


def attention_fp32_forward_flash_rotary(q, k, v, cos, sin, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, cs,
                                        ss, os_, stream=None):
    """Flash forward with the rotary prologue (no reference counterpart): rotary_fp32 forward on q
    and k, then attention_fp32_forward_flash, in one kernel."""
    return _call("attention_fp32_forward_flash_rotary", ptr(q), ptr(k), ptr(v), ptr(cos), ptr(sin), ptr(mask), ptr(output),
                 ptr(lse), batch, heads, queries, keys, radius, strides(qs), strides(ks), strides(vs), strides(cs), strides(ss),
                 strides(os_), _stream(stream))


def _check(status: int, function: str) -> None:
    if status != SUCCESS:
        raise HipError(status, function)


# Throwing wrappers with the reference's C++ names (Attention.hpp:44-108, Attention64.hpp:19-32).
def AttentionForward(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream=None):
    _check(attention_fp32_forward(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream),
           "attention_fp32_forward")


def AttentionForwardTiled(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream=None):
    _check(attention_fp32_forward_tiled(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream),
           "attention_fp32_forward_tiled")


def AttentionForwardFlash(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream=None):
    _check(attention_fp32_forward_flash(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream),
           "attention_fp32_forward_flash")


def AttentionForwardTuned(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, group, qs, ks, vs, os_, stream=None):
    _check(attention_fp32_forward_tuned(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, group, qs, ks, vs, os_, stream),
           "attention_fp32_forward_tuned")


def AttentionForwardFlashTuned(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, variant, qs, ks, vs, os_, stream=None):
    _check(attention_fp32_forward_flash_tuned(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, variant, qs, ks, vs, os_,
                                              stream), "attention_fp32_forward_flash_tuned")


def AttentionStatistics(q, k, mask, lse, batch, heads, queries, keys, radius, qs, ks, stream=None):
    _check(attention_fp32_statistics(q, k, mask, lse, batch, heads, queries, keys, radius, qs, ks, stream), "attention_fp32_statistics")


def AttentionBackward(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, qs, ks, vs, os_, us,
                      stream=None):
    _check(attention_fp32_backward(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, qs, ks,
                                   vs, os_, us, stream), "attention_fp32_backward")


def AttentionBackwardTiled(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, qs, ks, vs, os_,
                           us, stream=None):
    _check(attention_fp32_backward_tiled(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius,
                                         qs, ks, vs, os_, us, stream), "attention_fp32_backward_tiled")


def AttentionBackwardTuned(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, group, qs, ks,
                           vs, os_, us, stream=None):
    _check(attention_fp32_backward_tuned(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius,
                                         group, qs, ks, vs, os_, us, stream), "attention_fp32_backward_tuned")


def Attention64Forward(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream=None):
    _check(attention64_fp32_forward(q, k, v, mask, output, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream),
           "attention64_fp32_forward")


def Attention64Backward(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, qs, ks, vs, os_,
                        us, stream=None):
    _check(attention64_fp32_backward(q, k, v, mask, output, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, qs,
                                     ks, vs, os_, us, stream), "attention64_fp32_backward")


def AttentionGenericForward(q, k, v, mask, output, lse, batch, heads, queries, keys, head_width, radius, qs, ks, vs, os_, dtype,
                            stream=None):
    _check(attention_generic_forward(q, k, v, mask, output, lse, batch, heads, queries, keys, head_width, radius, qs, ks, vs, os_,
                                     dtype, stream), "attention_generic_forward")


def Rotary(q, k, cos, sin, oq, ok, batch, heads, length, backward, qs, ks, cs, ss, stream=None):
    _check(rotary_fp32(q, k, cos, sin, oq, ok, batch, heads, length, backward, qs, ks, cs, ss, stream), "rotary_fp32")
