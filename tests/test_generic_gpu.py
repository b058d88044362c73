"""attention_generic_forward (AttentionGeneric.hip:292-309) on the GPU through the C ABI.

The checker is the oracle's forward in double precision over the values the device reads: FP16
inputs are rounded to FP16 first and widened, which is the reference test's ComputeReference
(AttentionGenericTests.cpp:45-104; the same statements as AttentionTests.cpp:47-92 for any head
width). Bars:
  * the reference test's own: max absolute difference <= 5e-4 (FP32) / 2e-3 (FP16) on O and
    lse (AttentionGenericTests.cpp:146-148, CheckClose in TestSupport.hpp:24-38);
  * this library's normwise bars: FP32 storage 1e-5 (every FP32 entry's bar); FP16 storage 2e-3
    (P is rounded to FP16 once for P.V, as in the reference, and O is rounded to FP16);
  * selection exact: fully masked rows give O = 0 and lse = {-inf, 0}.
"""
from __future__ import annotations

import numpy as np
import pytest

from attention_cases import make_inputs, max_abs, normwise
from oracle import oracle

pytestmark = pytest.mark.gpu

FLOAT32, FLOAT16 = 0, 1
ABS_TOL = {FLOAT32: 5e-4, FLOAT16: 2e-3}
NORM_TOL = {FLOAT32: 1e-5, FLOAT16: 2e-3}
DTYPES = [FLOAT32, FLOAT16]
WIDTHS = [16, 32, 64]


def stored(x, dtype):
    """The values the device holds for a float32 array stored as `dtype` (FP16: round to nearest even)."""
    return x.astype(np.float16).astype(np.float32) if dtype == FLOAT16 else x.astype(np.float32)


def run_generic(cuda, q, k, v, mask, radius, dtype, layout="bhsd"):
    import torch

    from rocmkernels_b200 import attention as api

    tdtype = torch.float16 if dtype == FLOAT16 else torch.float32
    B, H, Q, D = q.shape
    K = k.shape[2]

    def place(x):
        t = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(cuda).to(tdtype)
        if layout == "bshd":  # token-major storage, strided heads
            return t.transpose(1, 2).contiguous().transpose(1, 2)
        if layout == "padded":  # token stride D + 1: not TMA-addressable, not vector-loadable
            storage = torch.zeros(*t.shape[:3], D + 1, device=cuda, dtype=tdtype)
            storage[..., :D] = t
            return storage[..., :D]
        return t

    dq, dk, dv = place(q), place(k), place(v)
    out = place(np.full((B, H, Q, D), np.nan, np.float32))
    lse = torch.full((B, H, Q, 2), float("nan"), device=cuda)
    dmask = torch.from_numpy(np.ascontiguousarray(mask, np.uint8)).to(cuda)
    status = api.attention_generic_forward(dq, dk, dv, dmask, out, lse, B, H, Q, K, D, radius, api.strides_of(dq),
                                           api.strides_of(dk), api.strides_of(dv), api.strides_of(out), dtype)
    torch.cuda.synchronize(cuda)
    assert api.device_status() == 0
    return status, out.float().cpu().numpy(), lse.cpu().numpy()


def expected_forward(q, k, v, mask, radius, dtype):
    q, k, v = (stored(x, dtype) for x in (q, k, v))
    return oracle.attention(q, k, v, mask, None, radius, forward_only=True, threads=oracle.cpu_count())


def check(output, lse, expected, dtype, label):
    assert normwise(output, expected["output"]) <= NORM_TOL[dtype], f"{label} O"
    assert max_abs(output, expected["output"]) <= ABS_TOL[dtype], f"{label} O abs"
    for i, name in ((0, "max"), (1, "sum")):
        assert normwise(lse[..., i], expected["lse"][..., i]) <= NORM_TOL[dtype], f"{label} lse {name}"
    assert max_abs(lse, expected["lse"]) <= ABS_TOL[dtype], f"{label} lse abs"
    dead = expected["lse"][..., 1] == 0  # rows without a visible key
    assert np.all(lse[..., 0][dead] == -np.inf) and np.all(lse[..., 1][dead] == 0.0), label
    assert np.all(output[dead] == 0.0), label


# AttentionGenericTests.cpp:152-188: RandomValues seeds 101/102/103 in [-1, 1), mask[3] = 0.
REFERENCE_CASES = [(1, 2, 40, 48, -1), (2, 1, 33, 37, 3)]


@pytest.mark.parametrize("width", WIDTHS)
@pytest.mark.parametrize("dtype", DTYPES, ids=["fp32", "fp16"])
@pytest.mark.parametrize("case", REFERENCE_CASES, ids=lambda c: "b{}h{}q{}k{}r{}".format(*c))
def test_generic_reference_cases(cuda, case, dtype, width):
    batch, heads, queries, keys, radius = case
    q, k, v, _, mask = make_inputs(batch, heads, queries, keys, width, seed=101)
    status, output, lse = run_generic(cuda, q, k, v, mask, radius, dtype)
    assert status == 0
    check(output, lse, expected_forward(q, k, v, mask, radius, dtype), dtype, f"d{width}")


EXTRA_CASES = [  # batch, heads, queries, keys, radius, masked fraction, fully masked batches, distribution
    (2, 3, 300, 333, -1, 0.2, (), "normal"),
    (1, 2, 700, 900, 100, 0.1, (), "uniform"),
    (3, 2, 129, 65, -1, 0.0, (1,), "uniform"),
    (1, 1, 1, 1, -1, 0.0, (), "uniform"),
    (2, 2, 257, 130, 0, 0.3, (), "normal"),
]


@pytest.mark.parametrize("layout", ["bhsd", "bshd", "padded"])
@pytest.mark.parametrize("width", WIDTHS)
@pytest.mark.parametrize("dtype", DTYPES, ids=["fp32", "fp16"])
@pytest.mark.parametrize("case", EXTRA_CASES, ids=lambda c: "b{}h{}q{}k{}r{}m{}".format(*c[:6]))
def test_generic_extra_cases(cuda, case, dtype, width, layout):
    batch, heads, queries, keys, radius, fraction, dead, dist = case
    q, k, v, _, mask = make_inputs(batch, heads, queries, keys, width, seed=7 + width, dist=dist, mask_fraction=fraction,
                                   masked_batches=dead)
    status, output, lse = run_generic(cuda, q, k, v, mask, radius, dtype, layout)
    assert status == 0
    check(output, lse, expected_forward(q, k, v, mask, radius, dtype), dtype, f"{layout} d{width}")


@pytest.mark.parametrize("width", WIDTHS)
@pytest.mark.parametrize("dtype", DTYPES, ids=["fp32", "fp16"])
def test_generic_benchmark_inputs(cuda, dtype, width):
    """The reference benchmark's inputs (AttentionGenericBenchmarks.cpp:35-54: q = 0.5, k = v =
    0.25, b2 h8 l512): every score is sqrt(D) / 8, so O = 0.25 and lse = {sqrt(D) / 8, 512}."""
    batch, heads, tokens = 2, 8, 512
    q = np.full((batch, heads, tokens, width), 0.5, np.float32)
    kv = np.full((batch, heads, tokens, width), 0.25, np.float32)
    mask = np.ones((batch, tokens), np.uint8)
    status, output, lse = run_generic(cuda, q, kv, kv, mask, -1, dtype)
    assert status == 0
    assert np.all(output == 0.25)
    score = np.float32(width * 0.125) * np.float32(1.0 / np.sqrt(np.float32(width)))
    assert np.allclose(lse[..., 0], score, rtol=1e-6, atol=0)
    assert np.allclose(lse[..., 1], tokens, rtol=1e-5, atol=0)


@pytest.mark.parametrize("width", [16, 32])
@pytest.mark.parametrize("dtype", DTYPES, ids=["fp32", "fp16"])
def test_generic_nan_conventions(cuda, dtype, width):
    """NaN in masked key rows changes nothing; a NaN in a visible key gives every row that sees
    it O = 0 and lse = {-inf, 0} (the reference's epilogue: total > 0 fails for a NaN total,
    AttentionGeneric.hip:119-128); other rows are unaffected."""
    batch, heads, queries, keys, radius = 2, 2, 150, 140, 20
    q, k, v, _, mask = make_inputs(batch, heads, queries, keys, width, seed=31)
    masked_key = 3  # mask[0, 3] == 0
    k[0, :, masked_key, :] = np.nan
    v[0, :, masked_key, :] = np.nan
    expected = expected_forward(q, k, v, mask, radius, dtype)
    visible_key = 100
    k[1, 1, visible_key, 5] = np.nan
    sees = np.abs(np.arange(queries) - visible_key) <= radius
    expected["output"][1, 1, sees] = 0.0
    expected["lse"][1, 1, sees] = (-np.inf, 0.0)
    status, output, lse = run_generic(cuda, q, k, v, mask, radius, dtype)
    assert status == 0
    assert np.isfinite(output).all()
    check(output, lse, expected, dtype, "nan")


@pytest.mark.parametrize("width", WIDTHS)
def test_generic_runs_on_tensor_cores(cuda, width):
    """The tensor maps of the tensor-core kernels (boxes wider than the rows for FP16 d16/d32 and
    FP32 d16, the TMA zero-filling the rest) are accepted by the driver here, so contiguous
    problems do not fall back to SIMT."""
    from rocmkernels_b200 import attention as api

    assert api.generic_kernel_name(2, 8, 512, 512, width, api.DType.Float16) == f"tcgen05-f16-flash-d{width}"
    assert api.generic_kernel_name(2, 8, 512, 512, width, api.DType.Float32) == f"tcgen05-f16x2-flash-d{width}"
