"""torch.autograd binding of the attention entry points (the reference's "external training loop"
use, README.md:67-81, bound through ctypes like tools/TorchCompare/compare_ops.py:29-60).

``attention(q, k, v, mask=None, radius=-1, cos=None, sin=None)`` returns softmax(Q K^T / sqrt(D),
masked) V for float32 CUDA tensors shaped [batch, heads, tokens, D] (D = 32 or 64, feature
stride 1, any other strides) and differentiates with respect to q, k and v through the
library's backward: for D = 32 the fused single-pass backward (attention_fp32_backward_fused, dQ
summed with atomics), or the deterministic two-pass attention_fp32_backward when
torch.are_deterministic_algorithms_enabled(); for D = 64 attention64_fp32_backward. With rotary
tables cos/sin ([batch, tokens, 32], D = 32) q and k are rotated
first (rotary_fp32's forward, Positional/Rotary.hip) inside the fused flash forward; the backward
rebuilds the rotated q and k with rotary_fp32, runs the attention backward on them and applies
the transposed rotation (rotary_fp32 with backward = 1) to their gradients. For D = 32 the
forward is the flash entry with a workspace (attention_fp32_forward_flash_workspace: K and V split
once by an operand pre-pass where that pays). The calls run on torch's current stream and
allocate their outputs and workspaces through torch.
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


def _table_strides(table: torch.Tensor) -> api.Strides:
    """Strides of a [batch, tokens, 32] rotary table (no head stride)."""
    return api.Strides(table.stride(0), 0, table.stride(1))


def _rotate(x: torch.Tensor, cos, sin, backward: bool) -> torch.Tensor:
    """rotary_fp32 on a [batch, heads, tokens, 32] tensor; the result is a [batch, heads, tokens, 32]
    view of token-major [batch, tokens, heads, 32] storage."""
    batch, heads, tokens, _ = x.shape
    out = torch.empty(batch, tokens, heads, 32, device=x.device, dtype=torch.float32)
    spare = torch.empty_like(out)  # rotary_fp32 always rotates two tensors; the second copy is discarded
    stream = torch.cuda.current_stream(x.device)
    status = api.rotary_fp32(x, x, cos, sin, out, spare, batch, heads, tokens, backward, api.strides_of(x), api.strides_of(x),
                             _table_strides(cos), _table_strides(sin), stream)
    if status != 0:
        raise api.HipError(status, "rotary_fp32")
    return out.transpose(1, 2)


class AttentionFunction(torch.autograd.Function):
    """Forward: the flash entry (D = 32; with rotary tables the fused rotary flash entry) or
    attention64_fp32_forward (D = 64); backward: the fused single-pass backward (D = 32; the
    two-pass one under torch's deterministic mode) or attention64_fp32_backward, recomputing P
    from the saved {max, sum}."""

    @staticmethod
    def forward(ctx, q, k, v, mask, radius, cos=None, sin=None):
        for name, tensor in (("q", q), ("k", k), ("v", v)):
            _check(name, tensor)
        batch, heads, queries, width = q.shape
        keys = k.shape[2]
        forward, _ = _entries(width)
        out = torch.empty(batch, heads, queries, width, device=q.device, dtype=torch.float32)
        lse = torch.empty(batch, heads, queries, 2, device=q.device, dtype=torch.float32)
        stream = torch.cuda.current_stream(q.device)
        if cos is None and width == 32:
            status = api.attention_fp32_forward_flash_workspace(q, k, v, mask, out, lse, batch, heads, queries, keys, radius,
                                                                api.strides_of(q), api.strides_of(k), api.strides_of(v),
                                                                api.strides_of(out), stream)
            if status != 0:
                raise api.HipError(status, "attention_fp32_forward_flash_workspace")
        elif cos is None:
            forward(q, k, v, mask, out, lse, batch, heads, queries, keys, radius, api.strides_of(q), api.strides_of(k),
                    api.strides_of(v), api.strides_of(out), stream)
        else:
            status = api.attention_fp32_forward_flash_rotary_workspace(q, k, v, cos, sin, mask, out, lse, batch, heads, queries, keys,
                                                                       radius, api.strides_of(q), api.strides_of(k),
                                                                       api.strides_of(v), _table_strides(cos), _table_strides(sin),
                                                                       api.strides_of(out), stream)
            if status != 0:
                raise api.HipError(status, "attention_fp32_forward_flash_rotary_workspace")
        ctx.save_for_backward(q, k, v, mask, out, lse, cos, sin)
        ctx.radius = radius
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, mask, out, lse, cos, sin = ctx.saved_tensors
        batch, heads, queries, width = q.shape
        keys = k.shape[2]
        _, backward = _entries(width)
        rotary = cos is not None
        if rotary:  # gradients with respect to the rotated q and k first
            q, k = _rotate(q, cos, sin, False), _rotate(k, cos, sin, False)
        if grad_out.stride(3) != 1:
            grad_out = grad_out.contiguous()
        grad_q = torch.empty(batch, heads, queries, width, device=q.device, dtype=torch.float32)
        grad_k = torch.empty(batch, heads, keys, width, device=q.device, dtype=torch.float32)
        grad_v = torch.empty(batch, heads, keys, width, device=q.device, dtype=torch.float32)
        delta = torch.empty(batch, heads, queries, device=q.device, dtype=torch.float32)
        stream = torch.cuda.current_stream(q.device)
        strides = (api.strides_of(q), api.strides_of(k), api.strides_of(v), api.strides_of(out), api.strides_of(grad_out))
        if width == 32 and not torch.are_deterministic_algorithms_enabled():
            status = api.attention_fp32_backward_fused(q, k, v, mask, out, lse, grad_out, grad_q, grad_k, grad_v, delta, batch,
                                                       heads, queries, keys, ctx.radius, *strides, stream)
            if status != 0:
                raise api.HipError(status, "attention_fp32_backward_fused")
        else:
            backward(q, k, v, mask, out, lse, grad_out, grad_q, grad_k, grad_v, delta, batch, heads, queries, keys, ctx.radius,
                     *strides, stream)
        if rotary:
            grad_q, grad_k = _rotate(grad_q, cos, sin, True), _rotate(grad_k, cos, sin, True)
        return grad_q, grad_k, grad_v, None, None, None, None


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor | None = None,
              radius: int = -1, cos: torch.Tensor | None = None, sin: torch.Tensor | None = None) -> torch.Tensor:
    """Masked attention with gradients for q, k and v.

    mask: [batch, keys] (nonzero = visible), default all visible. radius: keys with |i - j| <=
    radius are visible to query i (-1 = all). Rows without any visible key give 0.
    cos, sin: optional rotary tables [batch, tokens, 32] (float32, unit last stride, tokens >=
    max(queries, keys)); q and k are rotated before the attention (D = 32 only).
    """
    if (cos is None) != (sin is None):
        raise ValueError("pass both rotary tables or neither")
    if cos is not None:
        if q.shape[-1] != 32:
            raise ValueError("the rotary prologue is defined for 32-wide heads")
        for name, table in (("cos", cos), ("sin", sin)):
            if not table.is_cuda or table.dtype != torch.float32 or table.dim() != 3 or table.shape[2] != 32 or \
                    table.stride(2) != 1 or table.shape[0] != q.shape[0] or table.shape[1] < max(q.shape[2], k.shape[2]):
                raise ValueError(f"{name} must be a float32 CUDA tensor [batch, tokens >= max(queries, keys), 32]")
    batch, _, _, _ = q.shape
    keys = k.shape[2]
    if mask is None:
        mask = torch.ones(batch, keys, dtype=torch.uint8, device=q.device)
    else:
        mask = mask.to(device=q.device, dtype=torch.uint8).contiguous()
        if mask.shape != (batch, keys):
            raise ValueError(f"mask must be [batch, keys] = {(batch, keys)}")
    return AttentionFunction.apply(q, k, v, mask, int(radius), cos, sin)
