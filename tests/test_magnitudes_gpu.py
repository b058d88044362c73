"""Extreme input magnitudes through the split-FP16 tensor-core kernels.

Every FP32 operand enters the tensor cores as two FP16 terms after an exact power-of-two scale
(per Q row, per K/V tile, per column tile in the backward) that brings its largest magnitude into
[2^14, 2^15); the exponents are clamped to [-100, 100]. These cases scale Q, K, V and dO by factors
from 1e-20 to 1e20 -- far outside FP16's range, inside the clamp -- and check the results against
the oracle (double accumulation) with the normwise bars (forward 1e-5, gradients 1e-4; the
reference test's absolute 5e-4 is meant for U(-1, 1) inputs and does not apply at these
magnitudes): if a scale were lost or applied twice, the outputs would be off by powers of two, far
beyond the bars. Also a very peaked softmax (scores in
the hundreds), where almost every P underflows to zero.
"""
from __future__ import annotations

import numpy as np
import pytest

from attention_cases import FORWARD_TOL, GRADIENT_TOL, Device, make_inputs, normwise
from oracle import oracle

pytestmark = pytest.mark.gpu

# (q scale, k scale, v scale, dO scale): the products q.k stay moderate or grow, V and dO move O and
# the gradients by many orders of magnitude.
SCALES = [
    (1e-20, 1e20, 1.0, 1.0),
    (1e20, 1e-20, 1e10, 1e-10),
    (1.0, 1.0, 1e-20, 1e15),
    (30.0, 1.0, 1.0, 1.0),  # scores ~ +-170: a very peaked softmax
]


@pytest.fixture(scope="module")
def dev(cuda):
    return Device(cuda)


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("scales", SCALES, ids=lambda s: "q{:g}_k{:g}_v{:g}_do{:g}".format(*s))
def test_scaled_inputs_forward_backward(dev, width, scales):
    qs, ks, vs, us = scales
    B, H, Q, K = 2, 3, 200, 333
    q, k, v, upstream, mask = make_inputs(B, H, Q, K, width, seed=801 + width, dist="normal", mask_fraction=0.2)
    q, k, v, upstream = (x * np.float32(f) for x, f in ((q, qs), (k, ks), (v, vs), (upstream, us)))
    expected = oracle.attention(q, k, v, mask, upstream, -1, threads=oracle.cpu_count())
    forward = "attention_fp32_forward_flash" if width == 32 else "attention64_fp32_forward"
    backward = "attention_fp32_backward" if width == 32 else "attention64_fp32_backward"
    status, out, lse = dev.forward(forward, q, k, v, mask)
    assert status == 0
    assert np.isfinite(out).all()
    label = f"scaled {scales} d{width}"
    assert normwise(out, expected["output"]) <= FORWARD_TOL, label
    assert normwise(lse[..., 0], expected["lse"][..., 0]) <= FORWARD_TOL, label
    assert normwise(lse[..., 1], expected["lse"][..., 1]) <= FORWARD_TOL, label
    # d = 32 also through the fused single-pass backward (one K and dS exponent per 128-key tile)
    for entry in [backward] + (["attention_fp32_backward_fused"] if width == 32 else []):
        status, grads = dev.backward(entry, q, k, v, mask, upstream, out, lse)
        assert status == 0
        for name in ("grad_q", "grad_k", "grad_v"):
            assert normwise(grads[name], expected[name]) <= GRADIENT_TOL, f"{label} {entry} {name}"


@pytest.mark.parametrize("scales", SCALES[:2], ids=lambda s: "q{:g}_k{:g}".format(*s[:2]))
def test_scaled_inputs_statistics(cuda, scales):
    from test_statistics_gpu import check, run_statistics

    qs, ks = scales[:2]
    B, H, Q, K = 2, 3, 200, 333
    q, k, v, _, mask = make_inputs(B, H, Q, K, 32, seed=811, dist="normal", mask_fraction=0.2)
    q, k = q * np.float32(qs), k * np.float32(ks)
    expected = oracle.attention(q, k, v, mask, None, -1, forward_only=True, threads=oracle.cpu_count())
    status, lse = run_statistics(cuda, q, k, mask, -1)
    assert status == 0
    check(lse, expected, f"statistics scaled {scales[:2]}")
