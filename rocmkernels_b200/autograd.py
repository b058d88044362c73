"""torch.autograd binding of the attention entry points (the reference's "external training loop"
use, README.md:67-81, bound through ctypes like tools/TorchCompare/compare_ops.py:29-60).

``attention(q, k, v, mask=None, radius=-1)`` returns softmax(Q K^T / sqrt(D), masked) V for
float32 CUDA tensors shaped [batch, heads, tokens, D] (D = 32 or 64, feature stride 1, any other
strides) and differentiates with respect to q, k and v through the library's backward. The
calls run on torch's current stream and allocate their outputs through torch.
"""
from __future__ import annotations

import torch

from . import attention as api

__all__ = ["AttentionFunction", "attention"]


def _entries(width: int):
    if width == 32:
        return api.AttentionForwardFlash, api.AttentionBackward
    if width == 64:
        return api.Attention64Forward, api.Attention64Backward
    raise ValueError(f"head width {width} is not supported (32 or 64)")


def _check(name: str, tensor: torch.Tensor) -> None:
    if not tensor.is_cuda or tensor.dtype != torch.float32 or tensor.dim() != 4 or tensor.stride(3) != 1:
        raise ValueError(f"{name} must be a float32 CUDA tensor [batch, heads, tokens, D] with unit feature stride")


class AttentionFunction(torch.autograd.Function):
    """Forward: the flash entry (D = 32) or attention64_fp32_forward (D = 64); backward: the
    matching backward entry, recomputing P from the saved {max, sum}."""

    @staticmethod
    def forward(ctx, q, k, v, mask, radius):
        for name, tensor in (("q", q), ("k", k), ("v", v)):
            _check(name, tensor)
        batch, heads, queries, width = q.shape
        keys = k.shape[2]
        forward, _ = _entries(width)
        out = torch.empty(batch, heads, queries, width, device=q.device, dtype=torch.float32)
        lse = torch.empty(batch, heads, queries, 2, device=q.device, dtype=torch.float32)
        stream = torch.cuda.current_stream(q.device)
        forward(q, k, v, mask, out, lse, batch, heads, queries, keys, radius, api.strides_of(q), api.strides_of(k),
                api.strides_of(v), api.strides_of(out), stream)
        ctx.save_for_backward(q, k, v, mask, out, lse)
        ctx.radius = radius
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, mask, out, lse = ctx.saved_tensors
        batch, heads, queries, width = q.shape
        keys = k.shape[2]
        _, backward = _entries(width)
        if grad_out.stride(3) != 1:
            grad_out = grad_out.contiguous()
        grad_q = torch.empty(batch, heads, queries, width, device=q.device, dtype=torch.float32)
        grad_k = torch.empty(batch, heads, keys, width, device=q.device, dtype=torch.float32)
        grad_v = torch.empty(batch, heads, keys, width, device=q.device, dtype=torch.float32)
        delta = torch.empty(batch, heads, queries, device=q.device, dtype=torch.float32)
        stream = torch.cuda.current_stream(q.device)
        backward(q, k, v, mask, out, lse, grad_out, grad_q, grad_k, grad_v, delta, batch, heads, queries, keys, ctx.radius,
                 api.strides_of(q), api.strides_of(k), api.strides_of(v), api.strides_of(out), api.strides_of(grad_out),
                 stream)
        return grad_q, grad_k, grad_v, None, None


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor | None = None,
              radius: int = -1) -> torch.Tensor:
    """Masked attention with gradients for q, k and v.

    mask: [batch, keys] (nonzero = visible), default all visible. radius: keys with |i - j| <=
    radius are visible to query i (-1 = all). Rows without any visible key give 0.
    """
    batch, _, _, _ = q.shape
    keys = k.shape[2]
    if mask is None:
        mask = torch.ones(batch, keys, dtype=torch.uint8, device=q.device)
    else:
        mask = mask.to(device=q.device, dtype=torch.uint8).contiguous()
        if mask.shape != (batch, keys):
            raise ValueError(f"mask must be [batch, keys] = {(batch, keys)}")
    return AttentionFunction.apply(q, k, v, mask, int(radius))
