"""rotary_fp32 (Rotary.hip:44-56) and the fused rotary flash forward on the GPU, through the C ABI.

Checkers: the rotary oracle (ReferenceRotary, PositionalTests.cpp:18-50, pinned bit-exact against
the reference's own function) and the golden vectors it produced. Bars:
  * rotary: the reference test's own max absolute difference 1e-6 (PositionalTests.cpp:94-95);
    the device uses one fused multiply-add per output where the CPU rounds twice, so the two
    differ by at most an ulp or two;
  * fused forward: bit-identical to rotary_fp32 followed by attention_fp32_forward_flash, and
    within the forward bars of the oracle on the rotated inputs;
  * autograd with rotary tables: values and gradients against torch in float64.
"""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest

from attention_cases import FORWARD_TOL, GRADIENT_TOL, assert_forward_close, make_inputs, max_abs, normwise
from oracle import oracle

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
ROTARY_TOL = 1e-6


def tables(batch, tokens, seed):
    cos = oracle.uniform(batch * tokens * 32, seed).reshape(batch, tokens, 32)
    sin = oracle.uniform(batch * tokens * 32, seed + 1).reshape(batch, tokens, 32)
    return cos, sin


def put(cuda, array):
    import torch

    return torch.from_numpy(np.ascontiguousarray(array, np.float32)).to(cuda)


def table_strides(t):
    """[batch, tokens, 32] tables; a [tokens, 32] table is one table shared by every sequence."""
    from rocmkernels_b200 import attention as api

    return api.Strides(t.stride(0), 0, t.stride(1)) if t.dim() == 3 else api.Strides(0, 0, t.stride(0))


def run_rotary(cuda, q, k, cos, sin, backward, layout="token"):
    """q, k token-major [B, L, H, 32] numpy arrays stored in `layout`; returns (status, oq, ok)."""
    import torch

    from rocmkernels_b200 import attention as api

    B, L, H, _ = q.shape

    def place(x):
        if layout == "token":
            t = put(cuda, x)
            return t, api.Strides(t.stride(0), t.stride(2), t.stride(1))
        if layout == "head":  # [B, H, L, 32] storage
            t = put(cuda, x.transpose(0, 2, 1, 3))
            return t, api.Strides(t.stride(0), t.stride(1), t.stride(2))
        # "odd": [B, H, L, 33] storage, rows 4-byte aligned only (scalar path)
        storage = torch.zeros(B, H, L, 33, device=cuda)
        storage[..., :32] = put(cuda, x.transpose(0, 2, 1, 3))
        return storage, api.Strides(storage.stride(0), storage.stride(1), storage.stride(2))

    dq, qs = place(q)
    dk, ks = place(k)
    dcos, dsin = put(cuda, cos), put(cuda, sin)
    oq = torch.full((B, L, H, 32), float("nan"), device=cuda)
    ok = torch.full((B, L, H, 32), float("nan"), device=cuda)
    status = api.rotary_fp32(dq, dk, dcos, dsin, oq, ok, B, H, L, backward, qs, ks, table_strides(dcos), table_strides(dsin))
    torch.cuda.synchronize(cuda)
    return status, oq.cpu().numpy(), ok.cpu().numpy()


@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("rotary_*.npz")))
def test_rotary_golden(cuda, name):
    case = np.load(GOLDEN / f"{name}.npz")
    status, oq, ok = run_rotary(cuda, case["q"], case["k"], case["cos"], case["sin"], bool(case["backward"]))
    assert status == 0
    assert max_abs(oq, case["out_q"]) <= ROTARY_TOL and max_abs(ok, case["out_k"]) <= ROTARY_TOL


@pytest.mark.parametrize("layout", ["token", "head", "odd"])
@pytest.mark.parametrize("backward", [False, True])
@pytest.mark.parametrize("shape", [(2, 12, 1024), (3, 5, 77), (1, 1, 1)], ids=lambda s: "b{}h{}l{}".format(*s))
def test_rotary_layouts(cuda, shape, backward, layout):
    B, H, L = shape
    q = oracle.uniform(B * L * H * 32, 81, -2, 2).reshape(B, L, H, 32)
    k = oracle.uniform(B * L * H * 32, 82, -2, 2).reshape(B, L, H, 32)
    cos, sin = tables(B, L, 83)
    status, oq, ok = run_rotary(cuda, q, k, cos, sin, backward, layout)
    assert status == 0
    assert np.isfinite(oq).all() and np.isfinite(ok).all()
    assert max_abs(oq, oracle.rotary(q, cos, sin, backward)) <= ROTARY_TOL
    assert max_abs(ok, oracle.rotary(k, cos, sin, backward)) <= ROTARY_TOL


def test_rotary_shared_tables(cuda):
    """cos/sin with batch stride 0 (one table for every sequence), as a caller with fixed positions passes them."""
    import torch

    from rocmkernels_b200 import attention as api

    B, H, L = 3, 4, 50
    q = oracle.uniform(B * L * H * 32, 91, -2, 2).reshape(B, L, H, 32)
    cos1, sin1 = tables(1, L, 92)
    dq = put(cuda, q)
    dcos, dsin = put(cuda, cos1[0]), put(cuda, sin1[0])
    oq = torch.empty(B, L, H, 32, device=cuda)
    ok = torch.empty_like(oq)
    st = api.Strides(dq.stride(0), dq.stride(2), dq.stride(1))
    shared = api.Strides(0, 0, 32)
    assert api.rotary_fp32(dq, dq, dcos, dsin, oq, ok, B, H, L, 0, st, st, shared, shared) == 0
    torch.cuda.synchronize(cuda)
    expected = oracle.rotary(q, np.repeat(cos1, B, 0), np.repeat(sin1, B, 0), False)
    assert max_abs(oq.cpu().numpy(), expected) <= ROTARY_TOL
    assert np.array_equal(oq.cpu().numpy(), ok.cpu().numpy())


def composition(cuda, q, k, v, mask, cos, sin, radius):
    """rotary_fp32 (forward) on q and k, then attention_fp32_forward_flash on the rotated tensors."""
    import torch

    from rocmkernels_b200 import attention as api

    B, H, Q, D = q.shape
    K = k.shape[2]
    dcos, dsin = put(cuda, cos), put(cuda, sin)

    def rotated(x):
        dx = put(cuda, x)
        out = torch.empty(B, x.shape[2], H, 32, device=cuda)
        spare = torch.empty_like(out)
        s = api.strides_of(dx)
        assert api.rotary_fp32(dx, dx, dcos, dsin, out, spare, B, H, x.shape[2], 0, s, s, table_strides(dcos),
                               table_strides(dsin)) == 0
        return out.transpose(1, 2)

    rq, rk, dv = rotated(q), rotated(k), put(cuda, v)
    torch.cuda.synchronize(cuda)
    out = torch.empty(B, H, Q, D, device=cuda)
    lse = torch.empty(B, H, Q, 2, device=cuda)
    st = [api.strides_of(t) for t in (rq, rk, dv, out)]
    assert api.attention_fp32_forward_flash(rq, rk, dv, put(cuda, mask).to(torch.uint8), out, lse, B, H, Q, K, radius, *st) == 0
    torch.cuda.synchronize(cuda)
    return out.cpu().numpy(), lse.cpu().numpy(), rq.cpu().numpy(), rk.cpu().numpy()


def fused(cuda, q, k, v, mask, cos, sin, radius, layout="bhsd"):
    import torch

    from rocmkernels_b200 import attention as api

    B, H, Q, D = q.shape
    K = k.shape[2]

    def place(x):
        if layout == "bhsd":
            return put(cuda, x)
        storage = torch.zeros(*x.shape[:3], D + 1, device=cuda)  # token stride 33: not TMA-addressable
        storage[..., :D] = put(cuda, x)
        return storage[..., :D]

    dq, dk, dv = place(q), place(k), place(v)
    dcos, dsin = put(cuda, cos), put(cuda, sin)
    out = torch.full((B, H, Q, D), float("nan"), device=cuda)
    lse = torch.full((B, H, Q, 2), float("nan"), device=cuda)
    st = [api.strides_of(t) for t in (dq, dk, dv)]
    status = api.attention_fp32_forward_flash_rotary(dq, dk, dv, dcos, dsin, put(cuda, mask).to(torch.uint8), out, lse, B, H, Q, K,
                                                     radius, *st, table_strides(dcos), table_strides(dsin), api.strides_of(out))
    torch.cuda.synchronize(cuda)
    assert api.device_status() == 0
    return status, out.cpu().numpy(), lse.cpu().numpy()


FUSED_CASES = [  # batch, heads, queries, keys, radius, masked fraction
    (2, 3, 300, 333, -1, 0.2),
    (1, 2, 1024, 1024, 64, 0.0),
    (2, 2, 129, 65, -1, 0.5),
]


@pytest.mark.parametrize("case", FUSED_CASES, ids=lambda c: "b{}h{}q{}k{}r{}m{}".format(*c))
def test_fused_rotary_forward_equals_composition(cuda, case):
    B, H, Q, K, radius, fraction = case
    q, k, v, _, mask = make_inputs(B, H, Q, K, 32, seed=201, dist="normal", mask_fraction=fraction)
    cos, sin = tables(B, max(Q, K), 205)
    status, out, lse = fused(cuda, q, k, v, mask, cos, sin, radius)
    assert status == 0
    ref_out, ref_lse, rq, rk = composition(cuda, q, k, v, mask, cos, sin, radius)
    assert np.array_equal(out.view(np.uint32), ref_out.view(np.uint32))
    assert np.array_equal(lse.view(np.uint32), ref_lse.view(np.uint32))
    expected = oracle.attention(rq, rk, v, mask, None, radius, forward_only=True, threads=oracle.cpu_count())
    assert_forward_close(out, lse, expected, "fused rotary")


def test_fused_rotary_forward_shared_table(cuda):
    """One [tokens, 32] table for every sequence (batch stride 0)."""
    B, H, Q, K, radius = 3, 2, 200, 260, -1
    q, k, v, _, mask = make_inputs(B, H, Q, K, 32, seed=221, dist="normal", mask_fraction=0.1)
    cos, sin = tables(1, max(Q, K), 225)
    status, out, lse = fused(cuda, q, k, v, mask, cos[0], sin[0], radius)
    assert status == 0
    ref_out, ref_lse, _, _ = composition(cuda, q, k, v, mask, cos[0], sin[0], radius)
    assert np.array_equal(out.view(np.uint32), ref_out.view(np.uint32))
    assert np.array_equal(lse.view(np.uint32), ref_lse.view(np.uint32))


@pytest.mark.parametrize("case", FUSED_CASES[::2], ids=lambda c: "b{}h{}q{}k{}r{}m{}".format(*c))
def test_fused_rotary_forward_simt_fallback(cuda, case):
    """Strides the tensor maps cannot describe: the exact SIMT kernel with the same prologue."""
    B, H, Q, K, radius, fraction = case
    q, k, v, _, mask = make_inputs(B, H, Q, K, 32, seed=211, dist="normal", mask_fraction=fraction)
    cos, sin = tables(B, max(Q, K), 215)
    status, out, lse = fused(cuda, q, k, v, mask, cos, sin, radius, layout="padded")
    assert status == 0
    rq = oracle.rotary(q.transpose(0, 2, 1, 3), cos[:, :Q], sin[:, :Q]).transpose(0, 2, 1, 3)
    rk = oracle.rotary(k.transpose(0, 2, 1, 3), cos[:, :K], sin[:, :K]).transpose(0, 2, 1, 3)
    expected = oracle.attention(rq, rk, v, mask, None, radius, forward_only=True, threads=oracle.cpu_count())
    assert_forward_close(out, lse, expected, "fused rotary simt")


def torch_rotate(x, cos, sin):
    """The forward rotation in torch ([B, H, T, 32] x, [B, T, 32] tables)."""
    c, s = cos[:, None, : x.shape[2]], sin[:, None, : x.shape[2]]
    lo, hi = x[..., :16], x[..., 16:]
    return torch_cat(lo * c[..., :16] - hi * s[..., :16], hi * c[..., 16:] + lo * s[..., 16:])


def torch_cat(a, b):
    import torch

    return torch.cat([a, b], dim=-1)


@pytest.mark.parametrize("case", [(2, 3, 200, 233, -1, 0.2), (1, 2, 300, 300, 40, 0.0)],
                         ids=lambda c: "b{}h{}q{}k{}r{}m{}".format(*c))
def test_autograd_with_rotary_matches_torch(cuda, case):
    import torch

    from rocmkernels_b200.autograd import attention

    B, H, Q, K, radius, fraction = case
    generator = torch.Generator(device=cuda)
    generator.manual_seed(4242 + Q)
    q, k, v = (torch.randn(B, H, n, 32, device=cuda, generator=generator).requires_grad_() for n in (Q, K, K))
    angle = torch.rand(B, max(Q, K), 16, device=cuda, generator=generator) * 6.0
    cos = torch.cat([torch.cos(angle)] * 2, dim=-1).contiguous()
    sin = torch.cat([torch.sin(angle)] * 2, dim=-1).contiguous()
    mask = (torch.rand(B, K, device=cuda, generator=generator) >= fraction).to(torch.uint8)
    weights = torch.randn(B, H, Q, 32, device=cuda, generator=generator)

    out = attention(q, k, v, mask, radius, cos=cos, sin=sin)
    (out * weights).sum().backward()
    grads = [t.grad.detach().cpu().numpy() for t in (q, k, v)]

    q64, k64, v64 = (t.detach().double().requires_grad_() for t in (q, k, v))
    rq, rk = torch_rotate(q64, cos.double(), sin.double()), torch_rotate(k64, cos.double(), sin.double())
    scores = (rq @ rk.transpose(-1, -2)) / math.sqrt(32)
    visible = mask.bool()[:, None, None, :]
    if radius >= 0:
        rows = torch.arange(Q, device=cuda)[:, None]
        cols = torch.arange(K, device=cuda)[None, :]
        visible = visible & ((rows - cols).abs() <= radius)
    probabilities = torch.nan_to_num(torch.softmax(scores.masked_fill(~visible, float("-inf")), dim=-1), nan=0.0)
    expected = probabilities @ v64
    (expected * weights.double()).sum().backward()

    assert normwise(out.detach().cpu().numpy(), expected.detach().cpu().numpy()) <= FORWARD_TOL
    for name, got, want in zip("qkv", grads, (q64.grad, k64.grad, v64.grad)):
        assert np.isfinite(got).all(), name
        assert normwise(got, want.cpu().numpy()) <= GRADIENT_TOL, name
