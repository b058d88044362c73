"""attention_fp32_backward_static_delta: the backward whose delta scratch is held by the library.

Collected last (file name) so that it also runs after every other GPU test in one process; it
passes alone as well. Each case calls the entry twice in a row and compares both results with
attention_fp32_backward given a caller-owned delta buffer, through the C ABI.
"""
from __future__ import annotations

import numpy as np
import pytest

from attention_cases import GRADIENT_TOL, make_inputs, normwise

pytestmark = pytest.mark.gpu


def _run_pair(cuda, batch, heads, queries, keys, radius, mask_fraction):
    import torch

    from rocmkernels_b200 import attention as api

    q, k, v, upstream, mask = make_inputs(batch, heads, queries, keys, 32, dist="normal", mask_fraction=mask_fraction)
    put = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    q, k, v, upstream, mask = put(q), put(k), put(v), put(upstream), put(mask)
    out = torch.empty_like(q)
    lse = torch.empty(batch, heads, queries, 2, device=cuda)
    st = [api.strides_of(t) for t in (q, k, v, out, upstream)]
    assert api.attention_fp32_forward_flash(q, k, v, mask, out, lse, batch, heads, queries, keys, radius, *st[:4]) == 0

    expected = [torch.full_like(x, float("nan")) for x in (q, k, v)]
    delta = torch.empty(batch, heads, queries, device=cuda)
    assert api.attention_fp32_backward(q, k, v, mask, out, lse, upstream, *expected, delta, batch, heads, queries, keys,
                                       radius, *st) == 0
    results = []
    for _ in range(2):  # two calls in a row: no state may carry over between them
        grads = [torch.full_like(x, float("nan")) for x in (q, k, v)]
        assert api.attention_fp32_backward_static_delta(q, k, v, mask, out, lse, upstream, *grads, batch, heads, queries,
                                                        keys, radius, *st) == 0
        torch.cuda.synchronize(cuda)
        results.append([g.cpu().numpy() for g in grads])
    assert api.device_status() == 0
    reference = [g.cpu().numpy() for g in expected]
    for grads in results:
        for name, got, want in zip(("dQ", "dK", "dV"), grads, reference):
            assert np.isfinite(got).all(), name
            assert normwise(got, want) <= GRADIENT_TOL, name


@pytest.mark.parametrize("batch,heads,queries,keys,radius,mask_fraction",
                         [(2, 3, 300, 333, -1, 0.2), (1, 2, 1024, 1024, 64, 0.0), (2, 12, 128, 128, -1, 0.0)])
def test_static_delta_backward_matches_backward(cuda, batch, heads, queries, keys, radius, mask_fraction):
    _run_pair(cuda, batch, heads, queries, keys, radius, mask_fraction)


def test_static_delta_rejects_oversized_problem(cuda):
    from rocmkernels_b200 import attention as api

    s = api.Strides(0, 0, 0)
    # 2 * 16 * 131073 rows > 4194304: rejected with error 1 before any pointer is used.
    status = api.attention_fp32_backward_static_delta(1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 2, 16, 131073, 64, -1, s, s, s, s, s)
    assert status == 1
