"""Host-side partitioning of the attention path across GPUs (one process per GPU).

(batch, head) slices of the attention are independent: no slice reads another's queries, keys
or values, so a multi-GPU run splits them and needs no collective on the data path. Each rank
calls the unchanged C entry points on its slices with pointers offset into the full tensors:
q/k/v/dO/O by b*strides.batch + h*strides.head, the mask by b*keys, and the packed lse,
delta and gradients by (b*heads + h) rows.

``shard_plan`` returns the calls one rank makes: contiguous batch ranges when there are at
least as many sequences as ranks, otherwise one call per sequence over a contiguous head range
(a single sequence's heads are contiguous in every packed output).

``shard_offsets`` turns one call into the element offset of every tensor argument, and
``run_forward`` / ``run_backward`` make a rank's calls through the library's entry points
(``rocmkernels_b200.attention``) with those offsets applied to the full tensors' device
addresses. The offsets are plain integers, so the same function drives the CPU check in
tests/test_sharding.py.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ShardCall:
    """One entry-point call: sequences [b0, b1) x heads [h0, h1)."""

    b0: int
    b1: int
    h0: int
    h1: int

    @property
    def batch(self) -> int:
        return self.b1 - self.b0

    @property
    def heads(self) -> int:
        return self.h1 - self.h0


def even_ranges(total: int, parts: int) -> list[tuple[int, int]]:
    """[start, end) ranges splitting `total` items into `parts` contiguous, near-equal pieces."""
    if parts <= 0:
        raise ValueError("parts must be positive")
    base, extra = divmod(total, parts)
    ranges, start = [], 0
    for index in range(parts):
        end = start + base + (1 if index < extra else 0)
        ranges.append((start, end))
        start = end
    return ranges


def shard_plan(batch: int, heads: int, world: int, rank: int) -> list[ShardCall]:
    """The calls rank `rank` of `world` makes so that all ranks together cover every slice once."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    if batch >= world:
        b0, b1 = even_ranges(batch, world)[rank]
        return [ShardCall(b0, b1, 0, heads)] if b1 > b0 else []
    # Fewer sequences than ranks: split the flattened (sequence, head) slices, one call per sequence.
    s0, s1 = even_ranges(batch * heads, world)[rank]
    calls = []
    for b in range(batch):
        lo, hi = max(s0, b * heads), min(s1, (b + 1) * heads)
        if hi > lo:
            calls.append(ShardCall(b, b + 1, lo - b * heads, hi - b * heads))
    return calls


# Tensor arguments by role: strided [batch][heads][tokens][D] inputs/outputs, the [batch][keys]
# mask, and the packed outputs (their row counts per (batch, head) slice and row width).
STRIDED = ("q", "k", "v", "out", "upstream")


def shard_offsets(call: ShardCall, *, heads: int, queries: int, keys: int, width: int, strides: dict) -> dict:
    """Element offsets of every tensor argument for `call` into the full problem's tensors.

    `strides` maps the strided roles present (q, k, v, out, upstream) to (batch, head, token)
    element strides. Packed outputs: lse [B][H][Q][2], delta [B][H][Q], grad_q [B][H][Q][D],
    grad_k and grad_v [B][H][K][D]."""
    first_row = call.b0 * heads + call.h0  # flattened (batch, head) slice of the call's first row block
    offsets = {"mask": call.b0 * keys, "lse": first_row * queries * 2, "delta": first_row * queries,
               "grad_q": first_row * queries * width, "grad_k": first_row * keys * width,
               "grad_v": first_row * keys * width}
    for role, s in strides.items():
        sb, sh = (s.batch, s.head) if hasattr(s, "batch") else (s[0], s[1])
        offsets[role] = call.b0 * sb + call.h0 * sh
    return offsets


def _address(tensor) -> int:
    return tensor if isinstance(tensor, int) else int(tensor.data_ptr())


def _shifted(tensors: dict, offsets: dict, element_bytes: dict) -> dict:
    return {role: _address(t) + offsets[role] * element_bytes.get(role, 4) for role, t in tensors.items()}


def run_forward(entry, tensors: dict, plan: list[ShardCall], *, heads: int, queries: int, keys: int, width: int, radius: int,
                strides: dict, stream=None, workspace=None) -> int:
    """One rank's forward calls: `entry` is a forward entry point of rocmkernels_b200.attention
    (same argument order as attention_fp32_forward_flash); `tensors` holds the full problem's q,
    k, v, mask, out, lse (torch tensors or device addresses). `workspace`
    (attention_fp32_forward_flash_workspace: a device buffer sized for the largest call of the
    plan, see forward_workspace_bytes) is passed to every call, which are ordered on `stream`.
    Returns the first non-zero status."""
    extra = {} if workspace is None else {"workspace": workspace}
    for call in plan:
        offsets = shard_offsets(call, heads=heads, queries=queries, keys=keys, width=width,
                                strides={r: strides[r] for r in ("q", "k", "v", "out")})
        p = _shifted(tensors, offsets, {"mask": 1})
        status = entry(p["q"], p["k"], p["v"], p["mask"], p["out"], p["lse"], call.batch, call.heads, queries, keys, radius,
                       strides["q"], strides["k"], strides["v"], strides["out"], stream, **extra)
        if status != 0:
            return status
    return 0


def run_backward(entry, tensors: dict, plan: list[ShardCall], *, heads: int, queries: int, keys: int, width: int, radius: int,
                 strides: dict, stream=None, workspace=None) -> int:
    """One rank's backward calls (argument order of attention_fp32_backward); `tensors` holds the
    full problem's q, k, v, mask, out, lse, upstream, grad_q, grad_k, grad_v, delta. `workspace`
    (attention_fp32_backward_fused: a device buffer sized for the largest call of the plan, see
    workspace_bytes) is passed to every call, which are ordered on `stream`."""
    extra = {} if workspace is None else {"workspace": workspace}
    for call in plan:
        offsets = shard_offsets(call, heads=heads, queries=queries, keys=keys, width=width,
                                strides={r: strides[r] for r in STRIDED})
        p = _shifted(tensors, offsets, {"mask": 1})
        status = entry(p["q"], p["k"], p["v"], p["mask"], p["out"], p["lse"], p["upstream"], p["grad_q"], p["grad_k"],
                       p["grad_v"], p["delta"], call.batch, call.heads, queries, keys, radius, strides["q"], strides["k"],
                       strides["v"], strides["out"], strides["upstream"], stream, **extra)
        if status != 0:
            return status
    return 0


def forward_workspace_bytes(size_of, plan: list[ShardCall], keys: int) -> int:
    """Workspace for run_forward with attention_fp32_forward_flash_workspace: `size_of(batch,
    heads, keys)` (attention_fp32_forward_flash_workspace_size) of the plan's largest call."""
    return max((size_of(call.batch, call.heads, keys) for call in plan), default=0)


def workspace_bytes(size_of, plan: list[ShardCall], queries: int) -> int:
    """Workspace for run_backward with the fused backward: `size_of(batch, heads, queries)` (e.g.
    attention_fp32_backward_fused_workspace_size) of the plan's largest call."""
    return max((size_of(call.batch, call.heads, queries) for call in plan), default=0)
