"""Parity of every entry point, called through the C ABI on the GPU, with the CPU oracle.

The oracle is the C restatement of the reference's ReferenceAttention, itself pinned
bit-for-bit to the reference (tests/test_oracle.py). Bars: see attention_cases.py.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from attention_cases import (
    Device,
    assert_forward_close,
    assert_gradients_close,
    expected_delta,
    make_inputs,
    normwise,
    GRADIENT_TOL,
)
from oracle import oracle

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"

FORWARD_32 = [
    ("attention_fp32_forward", None),
    ("attention_fp32_forward_tiled", None),
    ("attention_fp32_forward_flash", None),
    ("attention_fp32_forward_flash_tuned", 13),
    ("attention_fp32_forward_flash_tuned", 8),
    ("attention_fp32_forward_flash_tuned", 1),
    ("attention_fp32_forward_tuned", 164),
    ("attention_fp32_forward_tuned", 1164),
]
BACKWARD_32 = [
    ("attention_fp32_backward", None),
    ("attention_fp32_backward_tiled", None),
    ("attention_fp32_backward_fused", None),
    ("attention_fp32_backward_tuned", 4),
    ("attention_fp32_backward_tuned", 1264),
]


@pytest.fixture(scope="module")
def dev(cuda):
    return Device(cuda)


def forward_entries(width):
    return FORWARD_32 if width == 32 else [("attention64_fp32_forward", None)]


def backward_entries(width):
    return BACKWARD_32 if width == 32 else [("attention64_fp32_backward", None)]


@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("*.npz")
                                         if p.stem != "normal_pin" and not p.stem.startswith("rotary_")))
def test_golden_vectors_all_entries(dev, name):
    """The reference's own test sections (and extras), expected outputs from its own code."""
    case = np.load(GOLDEN / f"{name}.npz")
    q, k, v, mask, upstream, radius = case["q"], case["k"], case["v"], case["mask"], case["upstream"], int(case["radius"])
    width = q.shape[-1]
    for entry, selector in forward_entries(width):
        status, out, lse = dev.forward(entry, q, k, v, mask, radius, selector)
        assert status == 0, entry
        assert_forward_close(out, lse, case, f"{name}/{entry}/{selector}")
    if not np.any(upstream):
        return
    _, out, lse = dev.forward("attention_fp32_forward" if width == 32 else "attention64_fp32_forward", q, k, v, mask, radius)
    for entry, selector in backward_entries(width):
        status, grads = dev.backward(entry, q, k, v, mask, upstream, out, lse, radius, selector)
        assert status == 0, entry
        assert_gradients_close(grads, case, f"{name}/{entry}/{selector}")
        assert normwise(grads["delta"], expected_delta(upstream, out)) <= GRADIENT_TOL


SHAPES = [
    # batch, heads, queries, keys, width, radius, mask_fraction, masked_batches
    (1, 1, 1, 1, 32, -1, 0.0, ()),
    (2, 2, 1, 77, 32, -1, 0.0, ()),
    (1, 3, 31, 33, 32, -1, 0.2, ()),
    (2, 1, 64, 64, 32, 0, 0.0, ()),
    (1, 2, 65, 130, 32, 9, 0.3, ()),
    (2, 2, 127, 200, 32, -1, 0.5, (1,)),
    (1, 1, 200, 31, 32, 64, 0.1, ()),
    (3, 2, 129, 129, 64, -1, 0.25, ()),
    (1, 2, 100, 70, 64, 17, 0.0, (0,)),
    (2, 1, 1, 300, 64, -1, 0.4, ()),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "b{}h{}q{}k{}d{}r{}m{}".format(*s[:7]))
@pytest.mark.parametrize("layout", ["bhsd", "bshd", "padded"])
def test_random_shapes_forward_backward(dev, shape, layout):
    B, H, Q, K, D, radius, fraction, masked = shape
    q, k, v, upstream, mask = make_inputs(B, H, Q, K, D, seed=7 + Q, dist="normal", mask_fraction=fraction,
                                          masked_batches=masked)
    expected = oracle.attention(q, k, v, mask, upstream, radius, threads=4)
    for entry, selector in forward_entries(D):
        status, out, lse = dev.forward(entry, q, k, v, mask, radius, selector, layout=layout)
        assert status == 0
        assert_forward_close(out, lse, expected, f"{entry}/{selector}/{layout}")
    _, out, lse = dev.forward(forward_entries(D)[0][0], q, k, v, mask, radius, layout=layout)
    for entry, selector in backward_entries(D):
        status, grads = dev.backward(entry, q, k, v, mask, upstream, out, lse, radius, selector, layout=layout)
        assert status == 0
        assert_gradients_close(grads, expected, f"{entry}/{selector}/{layout}")


@pytest.mark.parametrize("width", [32, 64])
def test_selection_is_bit_exact(dev, width):
    """With Q = 0 every visible score is 0: max must be exactly 0, sum the exact count of visible
    keys, fully masked rows {-inf, 0} with O = 0."""
    B, H, Q, K, radius = 2, 2, 150, 170, 23
    q, k, v, upstream, mask = make_inputs(B, H, Q, K, width, mask_fraction=0.3, masked_batches=(1,))
    q[:] = 0
    rows = np.arange(Q)[:, None]
    keys = np.arange(K)[None, :]
    window = np.abs(rows - keys) <= radius
    counts = np.einsum("qk,bk->bq", window.astype(np.int64), mask.astype(np.int64))
    for entry, selector in forward_entries(width):
        status, out, lse = dev.forward(entry, q, k, v, mask, radius, selector)
        assert status == 0
        for b in range(B):
            for h in range(H):
                visible = counts[b] > 0
                assert np.all(lse[b, h, visible, 0] == 0.0), entry
                assert np.array_equal(lse[b, h, visible, 1], counts[b][visible].astype(np.float32)), entry
                assert np.all(lse[b, h, ~visible, 0] == -np.inf) and np.all(lse[b, h, ~visible, 1] == 0.0)
                assert not np.any(out[b, h, ~visible])


def test_statistics_entry_matches_forward_lse(dev):
    import rocmkernels_b200.attention as api
    import torch

    q, k, v, upstream, mask = make_inputs(2, 3, 97, 130, 32, mask_fraction=0.2)
    expected = oracle.attention(q, k, v, mask, None, 11, forward_only=True)
    dq, dk, dmask = dev.put(q), dev.put(k), dev.put(mask)
    lse = torch.full((2, 3, 97, 2), float("nan"), device=dev.device)
    status = api.attention_fp32_statistics(dq, dk, dmask, lse, 2, 3, 97, 130, 11, api.strides_of(dq), api.strides_of(dk))
    torch.cuda.synchronize()
    assert status == 0
    got = dev.get(lse)
    assert normwise(got[..., 0], expected["lse"][..., 0]) <= 1e-5
    assert normwise(got[..., 1], expected["lse"][..., 1]) <= 1e-5


@pytest.mark.parametrize("entry", ["attention_fp32_backward", "attention_fp32_backward_fused"])
def test_masked_keys_get_zero_gradients_bitwise(dev, entry):
    q, k, v, upstream, mask = make_inputs(2, 2, 90, 110, 32, dist="normal", mask_fraction=0.4)
    k[0][:, mask[0] == 0] = np.nan  # garbage in masked rows must not leak (the reference zeroes them)
    v[0][:, mask[0] == 0] = np.inf
    _, out, lse = dev.forward("attention_fp32_forward", q, k, v, mask)
    status, grads = dev.backward(entry, q, k, v, mask, upstream, out, lse)
    assert status == 0
    for b in range(2):
        hidden = mask[b] == 0
        assert np.all(grads["grad_k"][b][:, hidden] == 0.0) and np.all(grads["grad_v"][b][:, hidden] == 0.0)
    assert np.all(np.isfinite(grads["grad_q"])) and np.all(np.isfinite(grads["grad_k"]))


def test_profile_stages_compose_to_the_full_backward(dev):
    import rocmkernels_b200.attention as api
    import torch

    B, H, Q, K = 1, 2, 96, 80
    q, k, v, upstream, mask = make_inputs(B, H, Q, K, 32, dist="normal", mask_fraction=0.1)
    expected = oracle.attention(q, k, v, mask, upstream, 5)
    _, out, lse = dev.forward("attention_fp32_forward", q, k, v, mask, 5)
    t = [dev.put(x) for x in (q, k, v, out, upstream)]
    dmask, dlse = dev.put(mask), dev.put(lse)
    gq, gk, gv = (torch.zeros(B, H, n, 32, device=dev.device) for n in (Q, K, K))
    delta = torch.zeros(B, H, Q, device=dev.device)
    s = [api.strides_of(x) for x in t]
    for stage in (1, 2, 3):
        assert api.attention_fp32_backward_profile(*t[:3], dmask, t[3], dlse, t[4], gq, gk, gv, delta, B, H, Q, K, 5, stage, *s) == 0
    torch.cuda.synchronize()
    assert normwise(dev.get(delta), expected_delta(upstream, out)) <= GRADIENT_TOL
    assert_gradients_close({"grad_q": dev.get(gq), "grad_k": dev.get(gk), "grad_v": dev.get(gv)}, expected, "profile")
    gq2 = torch.zeros_like(gq)
    for tuning in (14, 18, 24, 28, 44, 116):
        assert api.attention_fp32_query_profile(*t[:3], dmask, t[3], dlse, t[4], gq2, gk, gv, delta, B, H, Q, K, 5, tuning, *s) == 0
    torch.cuda.synchronize()
    assert normwise(dev.get(gq2), expected["grad_q"]) <= GRADIENT_TOL


def test_nan_propagates_like_reference(dev):
    q, k, v, upstream, mask = make_inputs(1, 1, 64, 64, 32)
    k[0, 0, 10, 5] = np.nan
    for entry, selector in FORWARD_32:
        status, out, lse = dev.forward(entry, q, k, v, mask, 3, selector)
        assert status == 0
        seeing = np.abs(np.arange(64) - 10) <= 3
        assert np.all(np.isnan(out[0, 0, seeing])) and np.all(np.isnan(lse[0, 0, seeing]))
        assert np.all(np.isfinite(out[0, 0, ~seeing])) and np.all(np.isfinite(lse[0, 0, ~seeing]))
