"""Helpers shared by the parity tests: input generation, calls through the C ABI, metrics.

Parity bars (written here once, used by every test):
  * forward O and lse: normwise max|x - ref| / max|ref| <= FORWARD_TOL, and the reference
    test's own absolute bar REFERENCE_ABS_TOL (TestSupport.hpp:23-39 with 5e-4);
  * gradients and delta: normwise <= GRADIENT_TOL;
  * key selection: bit-exact (non-finite lse entries must match exactly, masked keys give
    dK = dV = 0.0 exactly).
The tensor-core (split-FP16, kind::f16) paths are held to the same bars as the SIMT path.
"""
from __future__ import annotations

import numpy as np

from oracle import oracle

FORWARD_TOL = 1e-5
GRADIENT_TOL = 1e-4
REFERENCE_ABS_TOL = 5e-4


def make_inputs(batch, heads, queries, keys, width, *, seed=101, dist="uniform", mask_fraction=0.0, masked_batches=(),
                mask3=True):
    """Seeded inputs in the reference's style: q, k, v, dO from seeds seed..seed+3."""
    gen = oracle.uniform if dist == "uniform" else oracle.normal
    q = gen(batch * heads * queries * width, seed).reshape(batch, heads, queries, width)
    k = gen(batch * heads * keys * width, seed + 1).reshape(batch, heads, keys, width)
    v = gen(batch * heads * keys * width, seed + 2).reshape(batch, heads, keys, width)
    upstream = gen(batch * heads * queries * width, seed + 3).reshape(batch, heads, queries, width)
    mask = np.ones((batch, keys), np.uint8)
    if mask3 and mask.size > 3:
        mask.flat[3] = 0
    if mask_fraction > 0:
        draws = oracle.uniform(batch * keys, seed + 4, 0.0, 1.0).reshape(batch, keys)
        mask[draws < mask_fraction] = 0
    for b in masked_batches:
        mask[b, :] = 0
    return q, k, v, upstream, mask


def normwise(actual: np.ndarray, expected: np.ndarray) -> float:
    """max|actual - expected| / max|expected| over finite expected entries; inf if the
    non-finite pattern differs (NaN where NaN, +-inf where +-inf)."""
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    finite = np.isfinite(expected)
    if not np.array_equal(finite, np.isfinite(actual)):
        return float("inf")
    nonfinite = ~finite
    if nonfinite.any():
        same = (np.isnan(expected[nonfinite]) & np.isnan(actual[nonfinite])) | (expected[nonfinite] == actual[nonfinite])
        if not same.all():
            return float("inf")
    if not finite.any():
        return 0.0
    scale = np.max(np.abs(expected[finite]))
    diff = np.max(np.abs(actual[finite] - expected[finite]))
    return float(diff / scale) if scale > 0 else float(diff)


def max_abs(actual, expected) -> float:
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    finite = np.isfinite(e) & np.isfinite(a)
    return float(np.max(np.abs(a[finite] - e[finite]))) if finite.any() else 0.0


def assert_forward_close(output, lse, expected, label=""):
    o_err = normwise(output, expected["output"])
    m_err = normwise(lse[..., 0], expected["lse"][..., 0])
    s_err = normwise(lse[..., 1], expected["lse"][..., 1])
    assert o_err <= FORWARD_TOL, f"{label} O normwise error {o_err:.3e}"
    assert m_err <= FORWARD_TOL, f"{label} lse max normwise error {m_err:.3e}"
    assert s_err <= FORWARD_TOL, f"{label} lse sum normwise error {s_err:.3e}"
    assert max_abs(output, expected["output"]) <= REFERENCE_ABS_TOL
    assert max_abs(lse, expected["lse"]) <= REFERENCE_ABS_TOL * max(1.0, float(np.nanmax(np.abs(expected["lse"][..., 1]))))


def assert_gradients_close(grads, expected, label=""):
    for name in ("grad_q", "grad_k", "grad_v"):
        err = normwise(grads[name], expected[name])
        assert err <= GRADIENT_TOL, f"{label} {name} normwise error {err:.3e}"
        assert max_abs(grads[name], expected[name]) <= REFERENCE_ABS_TOL * max(1.0, float(np.max(np.abs(expected[name]))))


class Device:
    """Torch-backed device buffers and calls through the C ABI (rocmkernels_b200.attention)."""

    def __init__(self, device):
        import torch

        self.torch = torch
        self.device = device

    def put(self, array):
        return self.torch.from_numpy(np.ascontiguousarray(array)).to(self.device)

    @staticmethod
    def get(tensor):
        return tensor.detach().cpu().numpy()

    def padded(self, array):
        """[B, H, S, D] view of [B, H, S, D + 1] storage (token stride D + 1 floats)."""
        B, H, S, D = array.shape
        storage = self.torch.zeros((B, H, S, D + 1), device=self.device)
        storage[..., :D] = self.put(array)
        return storage[..., :D]

    def forward(self, entry, q, k, v, mask, radius=-1, selector=None, layout="bhsd", queries_first=False):
        """Runs a forward entry point. layout="bshd" stores q/k/v/O token-major (strided heads)."""
        import rocmkernels_b200.attention as api

        torch = self.torch
        B, H, Q, D = q.shape
        K = k.shape[2]
        if layout == "bhsd":
            dq, dk, dv = self.put(q), self.put(k), self.put(v)
            out = torch.full((B, H, Q, D), float("nan"), device=self.device)
            views = dq, dk, dv, out
        elif layout == "padded":  # token stride D + 1: not TMA-addressable, exercises the SIMT fallbacks
            dq, dk, dv = (self.padded(x) for x in (q, k, v))
            out = self.padded(np.full((B, H, Q, D), np.nan, np.float32))
            views = dq, dk, dv, out
        else:  # [B, S, H, D] storage viewed as [B, H, S, D]
            dq, dk, dv = (self.put(np.ascontiguousarray(x.transpose(0, 2, 1, 3))).transpose(1, 2) for x in (q, k, v))
            out = torch.full((B, Q, H, D), float("nan"), device=self.device).transpose(1, 2)
            views = dq, dk, dv, out
        dmask = self.put(mask)
        lse = torch.full((B, H, Q, 2), float("nan"), device=self.device)
        s = [api.strides_of(t) for t in views]
        args = [dq, dk, dv, dmask, out, lse, B, H, Q, K, radius]
        if selector is not None:
            args.append(selector)
        status = getattr(api, entry)(*args, *s)
        torch.cuda.synchronize()
        return status, self.get(out), self.get(lse)

    def backward(self, entry, q, k, v, mask, upstream, output, lse, radius=-1, selector=None, layout="bhsd"):
        import rocmkernels_b200.attention as api

        torch = self.torch
        B, H, Q, D = q.shape
        K = k.shape[2]
        if layout == "bhsd":
            tensors = [self.put(x) for x in (q, k, v, output, upstream)]
        elif layout == "padded":
            tensors = [self.padded(x) for x in (q, k, v, output, upstream)]
        else:
            tensors = [self.put(np.ascontiguousarray(x.transpose(0, 2, 1, 3))).transpose(1, 2) for x in (q, k, v, output, upstream)]
        dq_, dk_, dv_, do_, du_ = tensors
        dmask, dlse = self.put(mask), self.put(lse)
        gq = torch.full((B, H, Q, D), float("nan"), device=self.device)
        gk = torch.full((B, H, K, D), float("nan"), device=self.device)
        gv = torch.full((B, H, K, D), float("nan"), device=self.device)
        delta = torch.full((B, H, Q), float("nan"), device=self.device)
        s = [api.strides_of(t) for t in (dq_, dk_, dv_, do_, du_)]
        args = [dq_, dk_, dv_, dmask, do_, dlse, du_, gq, gk, gv, delta, B, H, Q, K, radius]
        if selector is not None:
            args.append(selector)
        status = getattr(api, entry)(*args, *s)
        torch.cuda.synchronize()
        return status, {"grad_q": self.get(gq), "grad_k": self.get(gk), "grad_v": self.get(gv), "delta": self.get(delta)}


def expected_delta(upstream, output):
    return np.einsum("bhqd,bhqd->bhq", upstream.astype(np.float64), output.astype(np.float64))
