"""The d = 32 split-FP32 flash forward runs 128-query CTAs when that grid fits in one wave (at most
one CTA per SM), 256-query CTAs (two Q tiles sharing each K/V tile) above that, and -- when the
grid of 128-query CTAs fills two per SM -- 128-query CTAs with two threads per query row, two CTAs
per SM (not with the rotary prologue). The shapes here sit just below and just above the one-wave
threshold and just above the two-per-SM one, computed from the device's SM count, so every CTA
form is checked. Entries: attention_fp32_forward_flash (the plain kernel),
attention_fp32_forward_flash_workspace (above one wave: the operand pre-pass and the prepared
kernel in the same three forms; the Python wrapper allocates the workspace), the fused rotary
forward and attention_generic_forward with 16-wide FP32 heads (the narrow-row instantiation).

Bars: the forward's (attention_cases.py) against the oracle, selection bit-exact on rows without
a visible key; the fused rotary forward bit-identical to rotary_fp32 followed by the flash forward.
"""
from __future__ import annotations

import numpy as np
import pytest

from attention_cases import Device, assert_forward_close, make_inputs
from oracle import oracle
from test_generic_gpu import FLOAT32, check, expected_forward, run_generic
from test_rotary_gpu import composition, fused, tables

pytestmark = pytest.mark.gpu

SIDES = ["one_wave", "two_waves", "two_per_sm"]


def batch_for(cuda, side, heads, queries):
    """Batch so that the 128-query grid has at most / just over one CTA per SM, or at least two."""
    import torch

    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    per_batch = heads * ((queries + 127) // 128)
    if side == "one_wave":
        return sms // per_batch
    if side == "two_waves":
        return sms // per_batch + 1
    return -(-2 * sms // per_batch)


def padded_mask(batch, keys, seed):
    lengths = np.random.default_rng(seed).integers(0, keys + 1, size=batch)
    lengths[0] = keys
    mask = np.zeros((batch, keys), np.uint8)
    for b, length in enumerate(lengths):
        mask[b, :length] = 1
    return mask


FLASH_CASES = [  # heads, queries, keys, radius
    (6, 600, 700, -1),
    (8, 128, 300, 40),
    (5, 333, 517, 100),
]


@pytest.fixture(scope="module")
def dev(cuda):
    return Device(cuda)


@pytest.mark.parametrize("entry", ["attention_fp32_forward_flash", "attention_fp32_forward_flash_workspace"],
                         ids=["plain", "workspace"])
@pytest.mark.parametrize("side", SIDES)
@pytest.mark.parametrize("case", FLASH_CASES, ids=lambda c: "h{}q{}k{}r{}".format(*c))
def test_flash_forward_either_cta_shape(dev, cuda, side, case, entry):
    H, Q, K, radius = case
    B = batch_for(cuda, side, H, Q)
    q, k, v, _, _ = make_inputs(B, H, Q, K, 32, seed=611 + Q, dist="normal", mask3=False)
    mask = padded_mask(B, K, 613 + Q)
    expected = oracle.attention(q, k, v, mask, None, radius, forward_only=True, threads=oracle.cpu_count())
    status, out, lse = dev.forward(entry, q, k, v, mask, radius)
    assert status == 0
    assert_forward_close(out, lse, expected, f"B{B} {side} {entry}")
    dead = expected["lse"][..., 1] == 0
    assert np.all(lse[..., 0][dead] == -np.inf) and np.all(lse[..., 1][dead] == 0.0)
    assert not np.any(out[dead])


@pytest.mark.parametrize("side", SIDES)
def test_fused_rotary_either_cta_shape(cuda, side):
    H, Q, K, radius = 4, 400, 450, -1
    B = batch_for(cuda, side, H, Q)
    q, k, v, _, mask = make_inputs(B, H, Q, K, 32, seed=621, dist="normal", mask_fraction=0.25)
    cos, sin = tables(B, max(Q, K), 625)
    status, out, lse = fused(cuda, q, k, v, mask, cos, sin, radius)
    assert status == 0
    ref_out, ref_lse, rq, rk = composition(cuda, q, k, v, mask, cos, sin, radius)
    assert np.array_equal(out.view(np.uint32), ref_out.view(np.uint32))
    assert np.array_equal(lse.view(np.uint32), ref_lse.view(np.uint32))
    expected = oracle.attention(rq, rk, v, mask, None, radius, forward_only=True, threads=oracle.cpu_count())
    assert_forward_close(out, lse, expected, f"fused rotary B{B} {side}")


@pytest.mark.parametrize("side", SIDES)
def test_generic_fp32_d16_either_cta_shape(cuda, side):
    H, Q, K, radius = 3, 512, 512, 30
    B = batch_for(cuda, side, H, Q)
    q, k, v, _, _ = make_inputs(B, H, Q, K, 16, seed=631, dist="normal", mask3=False)
    mask = padded_mask(B, K, 633)
    status, out, lse = run_generic(cuda, q, k, v, mask, radius, FLOAT32)
    assert status == 0
    check(out, lse, expected_forward(q, k, v, mask, radius, FLOAT32), FLOAT32, f"generic d16 B{B} {side}")
