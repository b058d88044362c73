"""attention_fp32_backward_static_delta: the backward whose delta scratch is held by the library.

Collected last (file name) so that it also runs after every other GPU test in one process; it
passes alone as well. Each case calls the entry twice in a row and compares both results with
attention_fp32_backward given a caller-owned delta buffer, through the C ABI. Both run the same
deterministic kernels, so the gradients must agree bit for bit. The size limit itself is checked
on the CPU (tests/test_abi.py), never with a GPU call on invalid pointers.
"""
from __future__ import annotations

import os
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest

from attention_cases import make_inputs

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parent.parent


def _device_copy(torch, array, cuda, layout):
    """[B, H, S, D] tensor on the device; "padded" stores it with token stride D + 1 (not
    TMA-addressable: the SIMT kernels run)."""
    tensor = torch.from_numpy(np.ascontiguousarray(array)).to(cuda)
    if layout != "padded":
        return tensor
    B, H, S, D = tensor.shape
    storage = torch.zeros((B, H, S, D + 1), device=cuda)
    storage[..., :D] = tensor
    return storage[..., :D]


def _run_pair(cuda, batch, heads, queries, keys, radius, mask_fraction, layout="bhsd"):
    import torch

    from rocmkernels_b200 import attention as api

    q, k, v, upstream, mask = make_inputs(batch, heads, queries, keys, 32, dist="normal", mask_fraction=mask_fraction)
    q, k, v, upstream = (_device_copy(torch, x, cuda, layout) for x in (q, k, v, upstream))
    mask = torch.from_numpy(mask).to(cuda)
    out = _device_copy(torch, np.zeros((batch, heads, queries, 32), np.float32), cuda, layout)
    lse = torch.empty(batch, heads, queries, 2, device=cuda)
    st = [api.strides_of(t) for t in (q, k, v, out, upstream)]
    assert api.attention_fp32_forward_flash(q, k, v, mask, out, lse, batch, heads, queries, keys, radius, *st[:4]) == 0

    expected = [torch.full((batch, heads, n, 32), float("nan"), device=cuda) for n in (queries, keys, keys)]
    delta = torch.empty(batch, heads, queries, device=cuda)
    assert api.attention_fp32_backward(q, k, v, mask, out, lse, upstream, *expected, delta, batch, heads, queries, keys,
                                       radius, *st) == 0
    results = []
    for _ in range(2):  # two calls in a row: the shared array keeps the last call's contents
        grads = [torch.full_like(x, float("nan")) for x in expected]
        assert api.attention_fp32_backward_static_delta(q, k, v, mask, out, lse, upstream, *grads, batch, heads, queries,
                                                        keys, radius, *st) == 0
        torch.cuda.synchronize(cuda)
        results.append([g.cpu().numpy() for g in grads])
    assert api.device_status() == 0
    reference = [g.cpu().numpy() for g in expected]
    for grads in results:
        for name, got, want in zip(("dQ", "dK", "dV"), grads, reference):
            assert np.isfinite(got).all(), name
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"{name} differs from attention_fp32_backward"


@pytest.mark.parametrize("batch,heads,queries,keys,radius,mask_fraction,layout",
                         [(2, 3, 300, 333, -1, 0.2, "bhsd"), (1, 2, 1024, 1024, 64, 0.0, "bhsd"),
                          (2, 12, 128, 128, -1, 0.0, "bhsd"), (2, 3, 150, 200, 17, 0.2, "padded")])
def test_static_delta_backward_matches_backward(cuda, batch, heads, queries, keys, radius, mask_fraction, layout):
    _run_pair(cuda, batch, heads, queries, keys, radius, mask_fraction, layout)


# Child process for the reset case. It holds its buffers through the CUDA driver API (libcuda), not
# torch: ROCmKernels::ResetDevice destroys the primary context, and the driver-API buffers can be
# allocated again in the context that follows, where torch's cached allocations would be stale.
_RESET_CHILD = textwrap.dedent(r"""
    import ctypes, sys
    import numpy as np
    sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/tests")
    from attention_cases import make_inputs
    from rocmkernels_b200 import attention as api

    cu = ctypes.CDLL("libcuda.so.1")
    def check(status, what):
        if status != 0:
            raise SystemExit(f"{what} failed with CUresult {status}")
    check(cu.cuInit(0), "cuInit")
    device = ctypes.c_int()
    check(cu.cuDeviceGet(ctypes.byref(device), 0), "cuDeviceGet")

    def make_current():
        context = ctypes.c_void_p()
        check(cu.cuDevicePrimaryCtxRetain(ctypes.byref(context), device), "cuDevicePrimaryCtxRetain")
        check(cu.cuCtxSetCurrent(context), "cuCtxSetCurrent")

    def upload(array):
        array = np.ascontiguousarray(array)
        pointer = ctypes.c_uint64()
        check(cu.cuMemAlloc_v2(ctypes.byref(pointer), ctypes.c_size_t(array.nbytes)), "cuMemAlloc")
        check(cu.cuMemcpyHtoD_v2(pointer, array.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(array.nbytes)), "HtoD")
        return pointer.value

    def download(pointer, shape):
        out = np.empty(shape, np.float32)
        check(cu.cuCtxSynchronize(), "cuCtxSynchronize")
        check(cu.cuMemcpyDtoH_v2(out.ctypes.data_as(ctypes.c_void_p), ctypes.c_uint64(pointer), ctypes.c_size_t(out.nbytes)), "DtoH")
        return out

    B, H, S, D = 2, 3, 256, 32
    q, k, v, u, mask = make_inputs(B, H, S, S, D, dist="normal", mask_fraction=0.1)
    s = api.Strides(H * S * D, S * D, D)

    def gradients(static):
        dq, dk, dv, uu, m = (upload(x) for x in (q, k, v, u, mask))
        out, lse = upload(np.zeros((B, H, S, D), np.float32)), upload(np.zeros((B, H, S, 2), np.float32))
        assert api.attention_fp32_forward_flash(dq, dk, dv, m, out, lse, B, H, S, S, -1, s, s, s, s) == 0
        grads = [upload(np.full((B, H, S, D), np.nan, np.float32)) for _ in range(3)]
        if static:
            status = api.attention_fp32_backward_static_delta(dq, dk, dv, m, out, lse, uu, *grads, B, H, S, S, -1, s, s, s, s, s)
        else:
            delta = upload(np.zeros((B, H, S), np.float32))
            status = api.attention_fp32_backward(dq, dk, dv, m, out, lse, uu, *grads, delta, B, H, S, S, -1, s, s, s, s, s)
        assert status == 0, status
        return [download(g, (B, H, S, D)) for g in grads]

    reset = api.lib()._ZN11ROCmKernels11ResetDeviceEi
    reset.argtypes, reset.restype = [ctypes.c_int], None
    make_current()
    before = gradients(static=True)       # caches the array's address in this context
    reset(0)                              # ROCmKernels::ResetDevice: the context and its module are gone
    make_current()
    after = gradients(static=True)        # must look the address up again in the new context
    plain = gradients(static=False)
    assert api.device_status() == 0
    for a, b, c in zip(before, after, plain):
        assert np.isfinite(a).all()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        assert np.array_equal(b.view(np.uint32), c.view(np.uint32))
    print("reset ok")
""")


def test_static_delta_after_device_reset(cuda):
    """A device reset between two calls: the second call must use the array of the new context."""
    env = dict(os.environ)
    result = subprocess.run([sys.executable, "-c", _RESET_CHILD, str(REPO)], capture_output=True, text=True, timeout=300,
                            env=env)
    assert result.returncode == 0, result.stdout[-2000:] + result.stderr[-4000:]
    assert "reset ok" in result.stdout
