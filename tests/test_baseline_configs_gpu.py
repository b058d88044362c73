"""Parity on BASELINE.json's five configurations, through the C ABI on the GPU, against the oracle.

Inputs are the configurations' own seeded synthetic tensors, drawn with the reference's generator
(std::mt19937 + libstdc++ normal_distribution, restated in oracle/attention_oracle.c and pinned in
tests/test_oracle.py): Q, K, V, dO ~ N(0, 1) from seeds 101, 102, 103, 104; key-padding lengths
from seed 105 (oracle.lengths).

  C1  B2 H12 S128 d32, keys 112..127 of batch 1 masked: every 32-wide entry point
  C2  B8 H3 S1024 d32, the headline: attention_fp32_forward_flash
  C3  B8 H6 S1024 d64, lengths U[512, 1024]: attention64_fp32_forward / _backward
  C4  B16 H12 S2048 d32, radius 128, lengths U[1024, 2048]: flash forward + backward
  C5  B64 H12 S4096 d32: flash forward + backward on the whole problem, compared with the oracle
      on the declared (batch, head) slices C5_SLICES (the oracle needs ~7 s per slice)

Bars (attention_cases.py): forward O and lse normwise <= 1e-5, gradients normwise <= 1e-4, plus
the reference test's absolute 5e-4. Key selection is checked bit for bit with Q = 0 (every visible
score is 0, so each row's max is exactly 0 and its sum the exact count of visible keys; rows with
no visible key give O = 0 and {-inf, 0}), and masked keys must get dK = dV = 0.0 exactly.
The errors measured are printed as `PARITY <config> ...` lines (run pytest with -s to see them).
"""
from __future__ import annotations

import concurrent.futures

import numpy as np
import pytest

from attention_cases import (FORWARD_TOL, Device, assert_forward_close,
                             assert_gradients_close, max_abs, normwise)
from oracle import oracle

pytestmark = pytest.mark.gpu

# Declared deterministic subset of C5's 64 x 12 (batch, head) slices checked against the oracle.
C5_SLICES = [(0, 0), (21, 5), (42, 7), (63, 11)]


def config_inputs(batch, heads, seq, dim, lengths=None, backward=True):
    """Q, K, V, dO from seeds 101..104 and the [batch, seq] mask of the given visible lengths."""
    count = batch * heads * seq * dim
    seeds = (101, 102, 103, 104) if backward else (101, 102, 103)
    with concurrent.futures.ThreadPoolExecutor(len(seeds)) as pool:  # ctypes releases the GIL
        tensors = list(pool.map(lambda s: oracle.normal(count, s).reshape(batch, heads, seq, dim), seeds))
    mask = np.ones((batch, seq), np.uint8)
    if lengths is not None:
        for b, length in enumerate(lengths):
            mask[b, length:] = 0
    if not backward:
        tensors.append(None)
    return (*tensors, mask)


def visible_counts(mask, radius):
    """[batch, queries] number of keys each query sees (mask x radius window)."""
    seq = mask.shape[1]
    rows = np.arange(seq)[:, None]
    keys = np.arange(seq)[None, :]
    window = np.ones((seq, seq), bool) if radius < 0 else np.abs(rows - keys) <= radius
    return np.einsum("qk,bk->bq", window.astype(np.int64), mask.astype(np.int64))


def assert_selection_exact(lse, out, counts, label):
    """lse/out of a Q = 0 run: max exactly 0 and sum the exact visible count per row."""
    for b in range(lse.shape[0]):
        visible = counts[b] > 0
        assert np.all(lse[b][:, visible, 0] == 0.0), label
        assert np.all(lse[b][:, visible, 1] == counts[b][visible].astype(np.float32)), label
        assert np.all(lse[b][:, ~visible, 0] == -np.inf) and np.all(lse[b][:, ~visible, 1] == 0.0), label
        assert not np.any(out[b][:, ~visible]), label


def report(config, **errors):
    print(f"PARITY {config} " + " ".join(f"{k}={v:.3e}" for k, v in errors.items()), flush=True)


@pytest.fixture(scope="module")
def dev(cuda):
    return Device(cuda)


# ---------------------------------------------------------------------------------------------- C1
C1 = dict(batch=2, heads=12, seq=128, dim=32)
C1_FORWARD = ([("attention_fp32_forward", None), ("attention_fp32_forward_tiled", None), ("attention_fp32_forward_flash", None)]
              + [("attention_fp32_forward_flash_tuned", v) for v in range(19)]
              + [("attention_fp32_forward_tuned", g) for g in (2, 4, 8, 84, 164, 1164, 1264)])
C1_BACKWARD = ([("attention_fp32_backward", None), ("attention_fp32_backward_tiled", None),
                ("attention_fp32_backward_fused", None)]
               + [("attention_fp32_backward_tuned", g) for g in (2, 4, 8, 84, 164, 1164, 1264)])


@pytest.fixture(scope="module")
def c1():
    q, k, v, u, mask = config_inputs(**C1)
    mask[1, 112:] = 0  # the last 16 keys of batch 1 masked
    return q, k, v, u, mask, oracle.attention(q, k, v, mask, u, -1, threads=8)


@pytest.mark.parametrize("entry,selector", C1_FORWARD, ids=lambda x: str(x))
def test_c1_forward_entries(dev, c1, entry, selector):
    q, k, v, u, mask, expected = c1
    status, out, lse = dev.forward(entry, q, k, v, mask, -1, selector)
    assert status == 0
    assert_forward_close(out, lse, expected, f"C1 {entry} {selector}")
    status, out0, lse0 = dev.forward(entry, np.zeros_like(q), k, v, mask, -1, selector)
    assert status == 0
    assert_selection_exact(lse0, out0, visible_counts(mask, -1), f"C1 selection {entry} {selector}")


def test_c1_statistics(dev, c1):
    import torch

    import rocmkernels_b200.attention as api

    q, k, v, u, mask, expected = c1
    dq, dk, dmask = dev.put(q), dev.put(k), dev.put(mask)
    lse = torch.full((2, 12, 128, 2), float("nan"), device=dev.device)
    assert api.attention_fp32_statistics(dq, dk, dmask, lse, 2, 12, 128, 128, -1, api.strides_of(dq), api.strides_of(dk)) == 0
    torch.cuda.synchronize()
    got = dev.get(lse)
    assert normwise(got[..., 0], expected["lse"][..., 0]) <= FORWARD_TOL
    assert normwise(got[..., 1], expected["lse"][..., 1]) <= FORWARD_TOL


@pytest.mark.parametrize("entry,selector", C1_BACKWARD, ids=lambda x: str(x))
def test_c1_backward_entries(dev, c1, entry, selector):
    q, k, v, u, mask, expected = c1
    _, out, lse = dev.forward("attention_fp32_forward_flash", q, k, v, mask)
    status, grads = dev.backward(entry, q, k, v, mask, u, out, lse, -1, selector)
    assert status == 0
    assert_gradients_close(grads, expected, f"C1 {entry} {selector}")
    assert np.all(grads["grad_k"][1][:, 112:] == 0.0) and np.all(grads["grad_v"][1][:, 112:] == 0.0)
    report(f"C1/{entry}/{selector}", **{n: normwise(grads[n], expected[n]) for n in ("grad_q", "grad_k", "grad_v")})


# ---------------------------------------------------------------------------------------------- C2
def test_c2_headline_flash_forward(dev):
    q, k, v, _, mask = config_inputs(8, 3, 1024, 32, backward=False)
    expected = oracle.attention(q, k, v, mask, None, -1, threads=oracle.cpu_count(), forward_only=True)
    status, out, lse = dev.forward("attention_fp32_forward_flash", q, k, v, mask)
    assert status == 0
    assert_forward_close(out, lse, expected, "C2")
    report("C2", O=normwise(out, expected["output"]), lse_max=normwise(lse[..., 0], expected["lse"][..., 0]),
           lse_sum=normwise(lse[..., 1], expected["lse"][..., 1]), O_abs=max_abs(out, expected["output"]))
    status, out0, lse0 = dev.forward("attention_fp32_forward_flash", np.zeros_like(q), k, v, mask)
    assert status == 0
    assert_selection_exact(lse0, out0, visible_counts(mask, -1), "C2 selection")


# ------------------------------------------------------------------------------------------ C3, C4
def _forward_backward_config(dev, label, batch, heads, seq, dim, radius, low, high):
    lengths = oracle.lengths(batch, 105, low, high)
    q, k, v, u, mask = config_inputs(batch, heads, seq, dim, lengths)
    expected = oracle.attention(q, k, v, mask, u, radius, threads=oracle.cpu_count())
    forward = "attention_fp32_forward_flash" if dim == 32 else "attention64_fp32_forward"
    backwards = ["attention_fp32_backward", "attention_fp32_backward_fused"] if dim == 32 else ["attention64_fp32_backward"]
    status, out, lse = dev.forward(forward, q, k, v, mask, radius)
    assert status == 0
    assert_forward_close(out, lse, expected, label)
    report(label, O=normwise(out, expected["output"]), lse_max=normwise(lse[..., 0], expected["lse"][..., 0]),
           lse_sum=normwise(lse[..., 1], expected["lse"][..., 1]))
    for backward in backwards:
        status, grads = dev.backward(backward, q, k, v, mask, u, out, lse, radius)
        assert status == 0
        assert_gradients_close(grads, expected, f"{label} {backward}")
        for b, length in enumerate(lengths):  # masked keys: exact zeros
            assert np.all(grads["grad_k"][b][:, length:] == 0.0) and np.all(grads["grad_v"][b][:, length:] == 0.0)
        report(f"{label}/{backward}", **{n: normwise(grads[n], expected[n]) for n in ("grad_q", "grad_k", "grad_v")})
    status, out0, lse0 = dev.forward(forward, np.zeros_like(q), k, v, mask, radius)
    assert status == 0
    assert_selection_exact(lse0, out0, visible_counts(mask, radius), f"{label} selection")


def test_c3_64_wide_forward_backward(dev):
    _forward_backward_config(dev, "C3", 8, 6, 1024, 64, -1, 512, 1024)


def test_c4_local_radius_forward_backward(dev):
    _forward_backward_config(dev, "C4", 16, 12, 2048, 32, 128, 1024, 2048)


# ---------------------------------------------------------------------------------------------- C5
def test_c5_declared_slices(dev):
    import torch

    import rocmkernels_b200.attention as api

    B, H, S, D = 64, 12, 4096, 32
    q, k, v, u, mask = config_inputs(B, H, S, D)
    device = dev.device
    dq, dk, dv, du = (torch.from_numpy(x).to(device) for x in (q, k, v, u))
    dmask = torch.from_numpy(mask).to(device)
    out = torch.full_like(dq, float("nan"))
    lse = torch.full((B, H, S, 2), float("nan"), device=device)
    gq, gk, gv = (torch.full_like(dq, float("nan")) for _ in range(3))
    delta = torch.full((B, H, S), float("nan"), device=device)
    st = api.strides_of(dq)
    assert api.attention_fp32_forward_flash(dq, dk, dv, dmask, out, lse, B, H, S, S, -1, st, st, st, st) == 0
    assert api.attention_fp32_backward(dq, dk, dv, dmask, out, lse, du, gq, gk, gv, delta, B, H, S, S, -1, st, st, st, st, st) == 0
    fq, fk, fv = (torch.full_like(dq, float("nan")) for _ in range(3))  # the fused single-pass backward
    fdelta = torch.full((B, H, S), float("nan"), device=device)
    assert api.attention_fp32_backward_fused(dq, dk, dv, dmask, out, lse, du, fq, fk, fv, fdelta, B, H, S, S, -1,
                                             st, st, st, st, st) == 0
    torch.cuda.synchronize()
    assert api.device_status() == 0
    assert bool(torch.isfinite(out).all()) and bool(torch.isfinite(gq).all()) and bool(torch.isfinite(gk).all())
    assert bool(torch.isfinite(fq).all()) and bool(torch.isfinite(fk).all()) and bool(torch.isfinite(fv).all())

    def slice_check(bh):
        b, h = bh
        view = lambda x: np.ascontiguousarray(x[b:b + 1, h:h + 1])  # noqa: E731
        return oracle.attention(view(q), view(k), view(v), mask[b:b + 1], view(u), -1)

    with concurrent.futures.ThreadPoolExecutor(len(C5_SLICES)) as pool:
        expected = list(pool.map(slice_check, C5_SLICES))
    for (b, h), exp in zip(C5_SLICES, expected):
        got_out = out[b:b + 1, h:h + 1].cpu().numpy()
        got_lse = lse[b:b + 1, h:h + 1].cpu().numpy()
        grads = {n: t[b:b + 1, h:h + 1].cpu().numpy() for n, t in (("grad_q", gq), ("grad_k", gk), ("grad_v", gv))}
        label = f"C5 slice b{b} h{h}"
        assert_forward_close(got_out, got_lse, exp, label)
        assert_gradients_close(grads, exp, label)
        report(label, O=normwise(got_out, exp["output"]), lse_max=normwise(got_lse[..., 0], exp["lse"][..., 0]),
               lse_sum=normwise(got_lse[..., 1], exp["lse"][..., 1]),
               **{n: normwise(grads[n], exp[n]) for n in ("grad_q", "grad_k", "grad_v")})
        fused = {n: t[b:b + 1, h:h + 1].cpu().numpy() for n, t in (("grad_q", fq), ("grad_k", fk), ("grad_v", fv))}
        assert_gradients_close(fused, exp, f"{label} fused")
        report(f"{label} fused", **{n: normwise(fused[n], exp[n]) for n in ("grad_q", "grad_k", "grad_v")})
    # Selection on the whole problem: Q = 0 gives max 0 and sum 4096 in every row.
    dq.zero_()
    assert api.attention_fp32_forward_flash(dq, dk, dv, dmask, out, lse, B, H, S, S, -1, st, st, st, st) == 0
    torch.cuda.synchronize()
    assert bool((lse[..., 0] == 0).all()) and bool((lse[..., 1] == float(S)).all())
    del dq, dk, dv, du, out, lse, gq, gk, gv, delta, fq, fk, fv, fdelta
    torch.cuda.empty_cache()
