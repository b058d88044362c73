"""Key-padding masks (each sequence's keys valid up to a length, the rest masked) on the tensor-core
paths: the forward and the query-rows backward visit key tiles only up to the last visible key of
their window, and the key-rows backward skips key tiles whose keys are all masked. This is the
mask shape of BASELINE configs 2 and 3 (valid lengths drawn per sequence).

Bars: the forward's and the gradients' (attention_cases.py) against the oracle; selection
bit-exact (Q = 0: lse max exactly 0 and lse sum the exact count of visible keys, rows with none
O = 0 and {-inf, 0}); masked keys dK = dV = 0.0 exactly.
"""
from __future__ import annotations

import numpy as np
import pytest

from attention_cases import Device, assert_forward_close, assert_gradients_close, make_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu

CASES = [  # batch, heads, queries, keys, width, radius, valid key lengths per sequence
    (4, 2, 300, 700, 32, -1, (700, 517, 64, 0)),
    (3, 2, 1100, 1100, 32, 128, (1100, 600, 130)),
    (2, 1, 129, 2100, 32, -1, (2100, 65)),
    (3, 2, 400, 530, 64, -1, (530, 263, 1)),
    (2, 3, 257, 900, 64, 50, (900, 300)),
]


def padded_inputs(case, seed):
    B, H, Q, K, D, radius, lengths = case
    q, k, v, upstream, _ = make_inputs(B, H, Q, K, D, seed=seed, dist="normal", mask3=False)
    mask = np.zeros((B, K), np.uint8)
    for b, length in enumerate(lengths):
        mask[b, :length] = 1
    return q, k, v, upstream, mask


def entries(width):
    if width == 32:
        return "attention_fp32_forward_flash", "attention_fp32_backward"
    return "attention64_fp32_forward", "attention64_fp32_backward"


@pytest.fixture(scope="module")
def dev(cuda):
    return Device(cuda)


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b{}h{}q{}k{}d{}r{}".format(*c[:6]))
def test_padded_forward_backward(dev, case):
    B, H, Q, K, D, radius, lengths = case
    q, k, v, upstream, mask = padded_inputs(case, seed=401 + Q)
    expected = oracle.attention(q, k, v, mask, upstream, radius, threads=oracle.cpu_count())
    forward, backward = entries(D)
    status, out, lse = dev.forward(forward, q, k, v, mask, radius)
    assert status == 0
    assert_forward_close(out, lse, expected, forward)
    status, grads = dev.backward(backward, q, k, v, mask, upstream, out, lse, radius)
    assert status == 0
    assert_gradients_close(grads, expected, backward)
    for b, length in enumerate(lengths):
        assert not np.any(grads["grad_k"][b, :, length:]) and not np.any(grads["grad_v"][b, :, length:])


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b{}h{}q{}k{}d{}r{}".format(*c[:6]))
def test_padded_selection_is_bit_exact(dev, case):
    B, H, Q, K, D, radius, lengths = case
    q, k, v, _, mask = padded_inputs(case, seed=411)
    q[:] = 0
    rows = np.arange(Q)[:, None]
    keys = np.arange(K)[None, :]
    window = np.ones((Q, K), bool) if radius < 0 else np.abs(rows - keys) <= radius
    counts = np.einsum("qk,bk->bq", window.astype(np.int64), mask.astype(np.int64))
    status, out, lse = dev.forward(entries(D)[0], q, k, v, mask, radius)
    assert status == 0
    for b in range(B):
        visible = counts[b] > 0
        for h in range(H):
            rows_lse, rows_out = lse[b, h], out[b, h]
            assert np.all(rows_lse[visible, 0] == 0.0)
            assert np.array_equal(rows_lse[visible, 1], counts[b][visible].astype(np.float32))
            assert np.all(rows_lse[~visible, 0] == -np.inf) and np.all(rows_lse[~visible, 1] == 0.0)
            assert not np.any(rows_out[~visible])
