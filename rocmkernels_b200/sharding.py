"""Host-side partitioning of the attention path across GPUs (one process per GPU).

(batch, head) slices of the attention are independent: no slice reads another's queries, keys
or values, so a multi-GPU run splits them and needs no collective on the data path. Each rank
calls the unchanged C entry points on its slices with pointers offset into the full tensors:
q/k/v/dO/O by b*strides.batch + h*strides.head, the mask by b*keys, and the packed lse,
delta and gradients by (b*heads + h) rows.

``shard_plan`` returns the calls one rank makes: contiguous batch ranges when there are at
least as many sequences as ranks, otherwise one call per sequence over a contiguous head range
(a single sequence's heads are contiguous in every packed output).
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
