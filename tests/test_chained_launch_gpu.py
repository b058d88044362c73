"""Chained launches keep stream order.

A flash forward whose grid is one wave of one-Q-tile CTAs is launched as a programmatic
dependent of the kernel before it in the stream: its CTAs may be scheduled while that kernel still
runs, and they touch global memory only after it has completed. Checked here with a chain of
forwards on one stream, each one's output the next one's Q (read after write), written back into
the buffer the call before read (write after read), with torch kernels between some calls; the
chain is run once without any synchronisation and once with a synchronise after every call, and
the two must agree bit for bit. The same chain captured in a CUDA graph (where the launches become
programmatic edges) replays to the same bits. Shapes: 32-wide split FP32, 64-wide, and the 16-wide
FP16 generic forward, all one-wave grids on a 148-SM B200.
"""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

FLOAT16 = 1  # attention_generic_forward's dtype selector for FP16 storage


def api():
    from rocmkernels_b200 import attention

    return attention


def run_chain(cuda, width, start, k, v, mask, steps, synchronise, torch_ops=True):
    a = api()
    batch, heads, seq, _ = start.shape
    buffers = [start.clone(), torch.empty_like(start)]
    lse = torch.empty(batch, heads, seq, 2, device=cuda)
    st = a.strides_of(buffers[0])
    entry = a.attention_fp32_forward_flash if width == 32 else a.attention64_fp32_forward
    for i in range(steps):
        q, out = buffers[i % 2], buffers[(i + 1) % 2]
        assert entry(q, k, v, mask, out, lse, batch, heads, seq, seq, -1, st, st, st, st) == 0
        if torch_ops and i % 3 == 2:
            out.mul_(1.5)  # a torch kernel (not a programmatic dependent) between two forwards
        if synchronise:
            torch.cuda.synchronize(cuda)
    torch.cuda.synchronize(cuda)
    return buffers[steps % 2], lse


@pytest.mark.parametrize("width", [32, 64])
def test_forward_chain_keeps_stream_order(cuda, width):
    batch, heads, seq = 2, 8, 512
    gen = torch.Generator(device="cpu").manual_seed(901 + width)
    q, k, v = (torch.randn(batch, heads, seq, width, generator=gen).to(cuda) for _ in range(3))
    mask = torch.ones(batch, seq, dtype=torch.uint8, device=cuda)
    chained, chained_lse = run_chain(cuda, width, q, k, v, mask, 24, synchronise=False)
    ordered, ordered_lse = run_chain(cuda, width, q, k, v, mask, 24, synchronise=True)
    assert torch.isfinite(chained).all()
    assert torch.equal(chained.view(torch.int32), ordered.view(torch.int32))
    assert torch.equal(chained_lse.view(torch.int32), ordered_lse.view(torch.int32))
    assert api().device_status(clear=True) == 0


def test_generic_fp16_chain_keeps_stream_order(cuda):
    a = api()
    batch, heads, seq, width = 2, 8, 512, 16
    gen = torch.Generator(device="cpu").manual_seed(911)
    q, k, v = (torch.randn(batch, heads, seq, width, generator=gen).to(cuda).half() for _ in range(3))
    mask = torch.ones(batch, seq, dtype=torch.uint8, device=cuda)
    st = a.strides_of(q)

    def chain(synchronise):
        buffers = [q.clone(), torch.empty_like(q)]
        lse = torch.empty(batch, heads, seq, 2, device=cuda)
        for i in range(24):
            src, dst = buffers[i % 2], buffers[(i + 1) % 2]
            assert a.attention_generic_forward(src, k, v, mask, dst, lse, batch, heads, seq, seq, width, -1, st, st, st, st,
                                               FLOAT16) == 0
            if synchronise:
                torch.cuda.synchronize(cuda)
        torch.cuda.synchronize(cuda)
        return buffers[0], lse

    chained, chained_lse = chain(False)
    ordered, ordered_lse = chain(True)
    assert torch.equal(chained.view(torch.int16), ordered.view(torch.int16))
    assert torch.equal(chained_lse.view(torch.int32), ordered_lse.view(torch.int32))
    assert a.device_status(clear=True) == 0


def test_chained_forwards_in_a_graph(cuda):
    """A chain of one-wave forwards captured in a CUDA graph (the launches become programmatic
    edges) replays to the bits of the same chain run eagerly with a synchronise after every call."""
    a = api()
    batch, heads, seq, width = 2, 8, 512, 32
    gen = torch.Generator(device="cpu").manual_seed(921)
    q, k, v = (torch.randn(batch, heads, seq, width, generator=gen).to(cuda) for _ in range(3))
    mask = torch.ones(batch, seq, dtype=torch.uint8, device=cuda)
    st = a.strides_of(q)
    buffers = [q.clone(), torch.empty_like(q)]
    lse = torch.empty(batch, heads, seq, 2, device=cuda)

    def chain(stream):
        for i in range(6):
            src, dst = buffers[i % 2], buffers[(i + 1) % 2]
            assert a.attention_fp32_forward_flash(src, k, v, mask, dst, lse, batch, heads, seq, seq, -1, st, st, st, st, stream) == 0

    side = torch.cuda.Stream(cuda)
    with torch.cuda.stream(side):
        chain(side)  # kernel attributes are set outside the capture
        side.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            chain(torch.cuda.current_stream(cuda))
    buffers[0].copy_(q)
    graph.replay()
    torch.cuda.synchronize(cuda)
    replayed, replayed_lse = buffers[0].clone(), lse.clone()
    expected, expected_lse = run_chain(cuda, width, q, k, v, mask, 6, synchronise=True, torch_ops=False)
    assert torch.equal(replayed.view(torch.int32), expected.view(torch.int32))
    assert torch.equal(replayed_lse.view(torch.int32), expected_lse.view(torch.int32))
    del graph
    assert a.device_status(clear=True) == 0
