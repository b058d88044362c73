"""attention_fp32_statistics (Attention.hip:252-261): {row max, sum} per query from Q, K and the
mask, no V and no output. With K TMA-addressable it runs the split-FP16 flash forward without the
P.V products (row sums in FP32); other layouts take the SIMT kernel.

Bars: the forward's lse bar (attention_cases.py) against the oracle; selection bit-exact (Q = 0:
max exactly 0 and sum the exact count of visible keys, rows without one {-inf, 0}); garbage in
masked key rows never leaks.
"""
from __future__ import annotations

import numpy as np
import pytest

from attention_cases import FORWARD_TOL, REFERENCE_ABS_TOL, make_inputs, max_abs, normwise
from oracle import oracle
from test_cta_tiles_gpu import batch_for, padded_mask

pytestmark = pytest.mark.gpu


def run_statistics(cuda, q, k, mask, radius, layout="bhsd"):
    import torch

    from rocmkernels_b200 import attention as api

    B, H, Q, _ = q.shape
    K = k.shape[2]

    def place(x):
        t = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(cuda)
        if layout == "padded":  # token stride 33: not TMA-addressable, the SIMT kernel
            storage = torch.zeros(*t.shape[:3], 33, device=cuda)
            storage[..., :32] = t
            return storage[..., :32]
        return t

    dq, dk = place(q), place(k)
    dmask = torch.from_numpy(np.ascontiguousarray(mask, np.uint8)).to(cuda)
    lse = torch.full((B, H, Q, 2), float("nan"), device=cuda)
    status = api.attention_fp32_statistics(dq, dk, dmask, lse, B, H, Q, K, radius, api.strides_of(dq), api.strides_of(dk))
    torch.cuda.synchronize(cuda)
    assert api.device_status() == 0
    return status, lse.cpu().numpy()


def check(lse, expected, label):
    for i, name in ((0, "max"), (1, "sum")):
        err = normwise(lse[..., i], expected["lse"][..., i])
        assert err <= FORWARD_TOL, f"{label} lse {name} normwise error {err:.3e}"
    assert max_abs(lse, expected["lse"]) <= REFERENCE_ABS_TOL * max(1.0, float(np.nanmax(np.abs(expected["lse"][..., 1]))))


CASES = [  # heads, queries, keys, radius, layout
    (3, 300, 333, -1, "bhsd"),
    (6, 600, 700, 64, "bhsd"),
    (2, 129, 1100, -1, "bhsd"),
    (3, 200, 170, 7, "padded"),
]


@pytest.mark.parametrize("side", ["one_wave", "two_waves"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "h{}q{}k{}r{}_{}".format(*c))
def test_statistics_matches_oracle(cuda, side, case):
    H, Q, K, radius, layout = case
    B = batch_for(cuda, side, H, Q)
    q, k, v, _, _ = make_inputs(B, H, Q, K, 32, seed=701 + Q, dist="normal", mask3=False)
    mask = padded_mask(B, K, 703 + K)
    expected = oracle.attention(q, k, v, mask, None, radius, forward_only=True, threads=oracle.cpu_count())
    status, lse = run_statistics(cuda, q, k, mask, radius, layout)
    assert status == 0
    check(lse, expected, f"B{B} {side} {layout}")


@pytest.mark.parametrize("radius", [-1, 40])
def test_statistics_selection_is_bit_exact(cuda, radius):
    B, H, Q, K = 3, 2, 333, 517
    q, k, v, _, _ = make_inputs(B, H, Q, K, 32, seed=711, dist="normal", mask3=False)
    q[:] = 0
    mask = padded_mask(B, K, 713)
    mask[2, :] = 0  # a sequence without visible keys
    rows = np.arange(Q)[:, None]
    keys = np.arange(K)[None, :]
    window = np.ones((Q, K), bool) if radius < 0 else np.abs(rows - keys) <= radius
    counts = np.einsum("qk,bk->bq", window.astype(np.int64), mask.astype(np.int64))
    status, lse = run_statistics(cuda, q, k, mask, radius)
    assert status == 0
    for b in range(B):
        visible = counts[b] > 0
        for h in range(H):
            assert np.all(lse[b, h, visible, 0] == 0.0)
            assert np.array_equal(lse[b, h, visible, 1], counts[b][visible].astype(np.float32))
            assert np.all(lse[b, h, ~visible, 0] == -np.inf) and np.all(lse[b, h, ~visible, 1] == 0.0)


def test_statistics_ignore_masked_key_rows(cuda):
    B, H, Q, K = 2, 3, 256, 300
    q, k, v, _, mask = make_inputs(B, H, Q, K, 32, seed=721, dist="normal", mask_fraction=0.3)
    expected = oracle.attention(q, k, v, mask, None, -1, forward_only=True, threads=oracle.cpu_count())
    k_garbage = k.copy()
    for b in range(B):
        k_garbage[b][:, mask[b] == 0] = np.nan
    status, lse = run_statistics(cuda, q, k_garbage, mask, -1)
    assert status == 0
    check(lse, expected, "masked rows hold NaN")


@pytest.mark.parametrize("side", ["one_wave", "two_waves"])
@pytest.mark.parametrize("key_tiles", [1, 2, 3, 4, 5])
def test_statistics_short_windows_repeated(cuda, side, key_tiles):
    """Windows of one to five key tiles, called repeatedly: the MMA warp's handling of the last
    two tiles (their releases are not waited for in statistics mode) must never leave a pipeline
    wait to run out, whatever the timing between the softmax and MMA warps."""
    H, Q = 2, 129
    K = 64 * key_tiles - 7  # a ragged last tile
    B = batch_for(cuda, side, H, Q)
    q, k, v, _, _ = make_inputs(B, H, Q, K, 32, seed=741 + key_tiles, dist="normal", mask3=False)
    mask = padded_mask(B, K, 743 + key_tiles)
    expected = oracle.attention(q, k, v, mask, None, -1, forward_only=True, threads=oracle.cpu_count())
    for _ in range(8):  # run_statistics asserts the device status word after every call
        status, lse = run_statistics(cuda, q, k, mask, -1)
        assert status == 0
    check(lse, expected, f"B{B} {side} {key_tiles} tiles")
