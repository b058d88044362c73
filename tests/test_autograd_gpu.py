"""rocmkernels_b200.autograd.attention against plain PyTorch attention in float64 (values and
gradients of q, k and v through torch.autograd)."""
from __future__ import annotations

import math

import numpy as np
import pytest

from attention_cases import FORWARD_TOL, GRADIENT_TOL, normwise

pytestmark = pytest.mark.gpu


def torch_reference(q, k, v, mask, radius):
    import torch

    width = q.shape[-1]
    scores = (q @ k.transpose(-1, -2)) / math.sqrt(width)
    visible = mask.bool()[:, None, None, :]
    if radius >= 0:
        rows = torch.arange(q.shape[2], device=q.device)[:, None]
        cols = torch.arange(k.shape[2], device=q.device)[None, :]
        visible = visible & ((rows - cols).abs() <= radius)
    scores = scores.masked_fill(~visible, float("-inf"))
    probabilities = torch.nan_to_num(torch.softmax(scores, dim=-1), nan=0.0)  # rows without keys: 0
    return probabilities @ v


CASES = [  # batch, heads, queries, keys, width, radius, masked fraction, layout
    (2, 3, 200, 333, 32, -1, 0.2, "bhsd"),
    (1, 2, 300, 300, 32, 40, 0.0, "bshd"),
    (2, 2, 129, 257, 64, -1, 0.3, "bhsd"),
    (1, 3, 256, 256, 64, 17, 0.0, "bshd"),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b{}h{}q{}k{}d{}r{}m{}{}".format(*c))
def test_autograd_matches_torch(cuda, case):
    import torch

    from rocmkernels_b200.autograd import attention

    batch, heads, queries, keys, width, radius, fraction, layout = case
    generator = torch.Generator(device=cuda)
    generator.manual_seed(1234 + queries + width)

    def make(tokens):
        x = torch.randn(batch, heads, tokens, width, device=cuda, generator=generator)
        if layout == "bshd":  # token-major storage viewed as [batch, heads, tokens, width]
            x = x.transpose(1, 2).contiguous().transpose(1, 2)
        return x.requires_grad_()

    q, k, v = make(queries), make(keys), make(keys)
    mask = (torch.rand(batch, keys, device=cuda, generator=generator) >= fraction).to(torch.uint8)
    weights = torch.randn(batch, heads, queries, width, device=cuda, generator=generator)

    out = attention(q, k, v, mask, radius)
    (out * weights).sum().backward()
    grads = [t.grad.detach().cpu().numpy() for t in (q, k, v)]

    q64, k64, v64 = (t.detach().double().requires_grad_() for t in (q, k, v))
    expected = torch_reference(q64, k64, v64, mask, radius)
    (expected * weights.double()).sum().backward()

    assert normwise(out.detach().cpu().numpy(), expected.detach().cpu().numpy()) <= FORWARD_TOL
    for name, got, want in zip("qkv", grads, (q64.grad, k64.grad, v64.grad)):
        assert np.isfinite(got).all(), name
        assert normwise(got, want.cpu().numpy()) <= GRADIENT_TOL, name


def test_deterministic_mode_takes_the_two_pass_backward(cuda):
    """Under torch.use_deterministic_algorithms(True) the D = 32 backward is the two-pass
    attention_fp32_backward: q.grad is bitwise repeatable; by default it is the fused backward,
    whose gradients agree with it within the bars."""
    import torch

    from rocmkernels_b200.autograd import attention

    generator = torch.Generator(device=cuda)
    generator.manual_seed(77)
    q, k, v = (torch.randn(2, 4, 700, 32, device=cuda, generator=generator) for _ in range(3))
    mask = torch.ones(2, 700, dtype=torch.uint8, device=cuda)
    weights = torch.randn(2, 4, 700, 32, device=cuda, generator=generator)

    def grads():
        leaves = [t.detach().clone().requires_grad_() for t in (q, k, v)]
        (attention(*leaves, mask) * weights).sum().backward()
        return [t.grad.cpu().numpy() for t in leaves]

    previous = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True)
    try:
        first, second = grads(), grads()
    finally:
        torch.use_deterministic_algorithms(previous)
    for a, b in zip(first, second):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    fused = grads()
    for a, b in zip(fused, first):
        assert normwise(a, b) <= GRADIENT_TOL
