"""The fused single-pass backward (attention_fp32_backward_fused): one key-major kernel computes dK
and dV per key and adds each 128-key tile's share of dQ with FP32 atomics, after a pre-pass that
writes delta and zeroes dQ.

Against the oracle with the gradient bars of attention_cases.py, on shapes with many key tiles
per head (so that dQ rows collect atomics from several CTAs), key padding, fully masked batches,
local radii that leave query rows without any visible key, and ragged tile edges. Also: dK and dV
are bitwise repeatable (their sums have a fixed order), dQ's summation order over key tiles is
not fixed but stays within the bars, query rows without a visible key get dQ = 0 exactly, masked
keys dK = dV = 0 exactly, and the result agrees with the two-pass attention_fp32_backward.
"""
from __future__ import annotations

import numpy as np
import pytest

from attention_cases import (
    GRADIENT_TOL,
    Device,
    assert_gradients_close,
    expected_delta,
    make_inputs,
    normwise,
)
from oracle import oracle

pytestmark = pytest.mark.gpu

FUSED = "attention_fp32_backward_fused"

CASES = [
    # batch, heads, queries, keys, radius, mask_fraction, masked_batches
    (2, 3, 700, 1000, -1, 0.2, ()),
    (1, 2, 1000, 700, 100, 0.1, ()),
    (3, 2, 333, 517, 7, 0.4, (1,)),
    (2, 2, 64, 1300, -1, 0.0, ()),
    (1, 1, 1, 129, -1, 0.0, ()),
    (2, 1, 257, 1, -1, 0.0, ()),
]


@pytest.fixture(scope="module")
def dev(cuda):
    return Device(cuda)


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b{}h{}q{}k{}r{}m{}".format(*c[:6]))
def test_fused_backward_matches_oracle(dev, case):
    B, H, Q, K, radius, fraction, masked = case
    q, k, v, upstream, mask = make_inputs(B, H, Q, K, 32, seed=901 + Q, dist="normal", mask_fraction=fraction,
                                          masked_batches=masked)
    expected = oracle.attention(q, k, v, mask, upstream, radius, threads=oracle.cpu_count())
    status, out, lse = dev.forward("attention_fp32_forward_flash", q, k, v, mask, radius)
    assert status == 0
    status, grads = dev.backward(FUSED, q, k, v, mask, upstream, out, lse, radius)
    assert status == 0
    assert_gradients_close(grads, expected, f"fused {case}")
    assert normwise(grads["delta"], expected_delta(upstream, out)) <= GRADIENT_TOL
    # selection: masked keys and query rows without a visible key get exact zeros
    hidden = mask == 0
    for b in range(B):
        assert np.all(grads["grad_k"][b][:, hidden[b]] == 0.0) and np.all(grads["grad_v"][b][:, hidden[b]] == 0.0)
    dead = expected["lse"][..., 1] == 0
    assert np.all(grads["grad_q"][dead] == 0.0)


def test_fused_backward_repeatable_and_agrees_with_two_pass(dev):
    B, H, Q, K, radius = 2, 4, 900, 1100, -1
    q, k, v, upstream, mask = make_inputs(B, H, Q, K, 32, seed=931, dist="normal", mask_fraction=0.15)
    status, out, lse = dev.forward("attention_fp32_forward_flash", q, k, v, mask, radius)
    assert status == 0
    runs = []
    for _ in range(3):
        status, grads = dev.backward(FUSED, q, k, v, mask, upstream, out, lse, radius)
        assert status == 0
        runs.append(grads)
    for grads in runs[1:]:
        assert np.array_equal(grads["grad_k"].view(np.uint32), runs[0]["grad_k"].view(np.uint32))
        assert np.array_equal(grads["grad_v"].view(np.uint32), runs[0]["grad_v"].view(np.uint32))
        assert np.array_equal(grads["delta"].view(np.uint32), runs[0]["delta"].view(np.uint32))
        assert normwise(grads["grad_q"], runs[0]["grad_q"]) <= 1e-6
    status, two_pass = dev.backward("attention_fp32_backward", q, k, v, mask, upstream, out, lse, radius)
    assert status == 0
    for name in ("grad_q", "grad_k", "grad_v"):
        assert normwise(runs[0][name], two_pass[name]) <= GRADIENT_TOL, name


def test_fused_backward_strided_and_padded_layouts(dev):
    """Token-major storage (strided heads, still TMA-addressable) and a padded token stride (not
    TMA-addressable: the call takes the two-pass SIMT path) give the same bars."""
    B, H, Q, K, radius = 2, 3, 300, 450, 60
    q, k, v, upstream, mask = make_inputs(B, H, Q, K, 32, seed=941, dist="normal", mask_fraction=0.2)
    expected = oracle.attention(q, k, v, mask, upstream, radius, threads=oracle.cpu_count())
    for layout in ("bshd", "padded"):
        status, out, lse = dev.forward("attention_fp32_forward", q, k, v, mask, radius, layout=layout)
        assert status == 0
        status, grads = dev.backward(FUSED, q, k, v, mask, upstream, out, lse, radius, layout=layout)
        assert status == 0
        assert_gradients_close(grads, expected, f"fused {layout}")


def test_fused_backward_workspace_reuse_and_unaligned_fallback(dev):
    """One workspace serves calls of different sizes ordered on one stream; a workspace that is not
    128-byte aligned takes the two-pass path, whose results equal attention_fp32_backward's bit
    for bit."""
    import torch

    import rocmkernels_b200.attention as api

    big = api.attention_fp32_backward_fused_workspace_size(2, 3, 900)
    storage = torch.empty(big + 256, dtype=torch.uint8, device=dev.device)
    for (B, H, Q, K) in [(2, 3, 900, 700), (1, 2, 130, 260), (2, 3, 900, 700)]:
        q, k, v, upstream, mask = make_inputs(B, H, Q, K, 32, seed=951 + Q + K, dist="normal", mask_fraction=0.1)
        expected = oracle.attention(q, k, v, mask, upstream, -1, threads=oracle.cpu_count())
        status, out, lse = dev.forward("attention_fp32_forward_flash", q, k, v, mask)
        assert status == 0
        t = [dev.put(x) for x in (q, k, v, out, upstream)]
        dmask, dlse = dev.put(mask), dev.put(lse)
        grads = [torch.full((B, H, n, 32), float("nan"), device=dev.device) for n in (Q, K, K)]
        delta = torch.full((B, H, Q), float("nan"), device=dev.device)
        st = [api.strides_of(x) for x in t]
        assert api.attention_fp32_backward_fused(*t[:3], dmask, t[3], dlse, t[4], *grads, delta, B, H, Q, K, -1, *st,
                                                 workspace=storage[:big]) == 0
        torch.cuda.synchronize()
        got = {n: dev.get(x) for n, x in zip(("grad_q", "grad_k", "grad_v"), grads)}
        assert_gradients_close(got, expected, f"reused workspace B{B} Q{Q} K{K}")
    # unaligned (the last call's problem again): the two-pass path
    status, two_pass = dev.backward("attention_fp32_backward", q, k, v, mask, upstream, out, lse)
    assert status == 0
    assert api.attention_fp32_backward_fused(*t[:3], dmask, t[3], dlse, t[4], *grads, delta, B, H, Q, K, -1, *st,
                                             workspace=storage[16:16 + big]) == 0
    torch.cuda.synchronize()
    for name, x in zip(("grad_q", "grad_k", "grad_v"), grads):
        assert np.array_equal(dev.get(x).view(np.uint32), two_pass[name].view(np.uint32)), name
