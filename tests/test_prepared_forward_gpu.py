"""The d = 32 flash forward's prepared-operand path: an operand pre-pass splits every 64-key tile of
K and V once into scratch from the library's stream-ordered pool, then the forward (launched as the
pre-pass's programmatic dependent) bulk-copies those stage images.

The path runs when it pays for its pre-pass: grids beyond one wave of the split-warp kernel, or
windows of at least 24 key tiles. The shapes below are chosen to take it (on a 148-SM B200) in each
CTA form: one Q tile, two Q tiles, and two threads per row.

Checked here, on the GPU:
* results against the oracle at shapes whose key windows do not start on a 64-key tile (radius),
  with padded keys, key counts that are not a multiple of 64, every CTA form;
* capture in a CUDA graph: the pool allocation, both kernels and the release are recorded, and
  replays on new inputs give the eager call's bits;
* two streams running forwards at the same time: each stream's scratch is its own (results equal
  the single-stream ones bit for bit);
* rocmkernels_attention_release_scratch returns the idle pool memory and later calls still work.
"""
from __future__ import annotations

import numpy as np
import pytest

from attention_cases import assert_forward_close, make_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def api():
    from rocmkernels_b200 import attention

    return attention


def device_problem(cuda, batch, heads, queries, keys, seed, mask_fraction=0.0):
    q, k, v, _, mask = make_inputs(batch, heads, queries, keys, 32, seed=seed, dist="normal", mask_fraction=mask_fraction)
    tensors = [torch.from_numpy(x).to(cuda) for x in (q, k, v, mask)]
    return (q, k, v, mask), tensors


def run_forward(cuda, tensors, queries, keys, radius, stream=None):
    dq, dk, dv, dmask = tensors
    batch, heads = dq.shape[0], dq.shape[1]
    out = torch.empty(batch, heads, queries, 32, device=cuda)
    lse = torch.empty(batch, heads, queries, 2, device=cuda)
    a = api()
    qs, ks = a.strides_of(dq), a.strides_of(dk)
    status = a.attention_fp32_forward_flash(dq, dk, dv, dmask, out, lse, batch, heads, queries, keys, radius, qs, ks, ks,
                                            a.strides_of(out), stream)
    return status, out, lse


# (batch, heads, queries, keys, radius, mask fraction): radius windows that start inside a key
# tile, ragged key counts, padded keys. Forms: two threads per row (cases 1, 2, 6), one Q tile
# (cases 3, 4), two Q tiles (case 5).
CASES = [(40, 4, 300, 300, 100, 0.0), (3, 60, 200, 333, 37, 0.2), (3, 4, 129, 2000, -1, 0.3), (2, 2, 777, 1600, 800, 0.1),
         (1, 100, 256, 2000, -1, 0.1), (16, 12, 256, 320, 70, 0.15)]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b{}h{}q{}k{}r{}m{}".format(*c))
def test_prepared_forward_matches_oracle(cuda, case):
    batch, heads, queries, keys, radius, fraction = case
    (q, k, v, mask), tensors = device_problem(cuda, batch, heads, queries, keys, 701 + queries, fraction)
    status, out, lse = run_forward(cuda, tensors, queries, keys, radius)
    assert status == 0
    expected = oracle.attention(q, k, v, mask, None, radius, forward_only=True, threads=oracle.cpu_count())
    assert_forward_close(out.cpu().numpy(), lse.cpu().numpy(), expected, f"prepared {case}")
    assert api().device_status(clear=True) == 0


def test_graph_capture_replays_the_forward(cuda):
    batch, heads, seq = 4, 3, 2048
    (_, _, _, _), tensors = device_problem(cuda, batch, heads, seq, seq, 711)
    stream = torch.cuda.Stream(cuda)
    with torch.cuda.stream(stream):
        status, out, lse = run_forward(cuda, tensors, seq, seq, -1, stream)  # warm the pool and kernel attributes
        assert status == 0
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            captured_status, graph_out, graph_lse = run_forward(cuda, tensors, seq, seq, -1, torch.cuda.current_stream(cuda))
    assert captured_status == 0
    for seed in (712, 713):
        (_, _, _, _), fresh = device_problem(cuda, batch, heads, seq, seq, seed)
        for dst, src in zip(tensors, fresh):
            dst.copy_(src)
        graph.replay()
        torch.cuda.synchronize(cuda)
        status, eager_out, eager_lse = run_forward(cuda, tensors, seq, seq, -1)
        torch.cuda.synchronize(cuda)
        assert status == 0
        assert torch.equal(graph_out.view(torch.int32), eager_out.view(torch.int32))
        assert torch.equal(graph_lse.view(torch.int32), eager_lse.view(torch.int32))
    del graph
    assert api().device_status(clear=True) == 0


def test_two_streams_keep_their_scratch_apart(cuda):
    problems = [device_problem(cuda, 2, 12, 2048, 2048, seed)[1] for seed in (721, 722)]
    expected = []
    for tensors in problems:
        status, out, lse = run_forward(cuda, tensors, 2048, 2048, -1)
        assert status == 0
        expected.append((out, lse))
    torch.cuda.synchronize(cuda)
    streams = [torch.cuda.Stream(cuda) for _ in problems]
    results = [[], []]
    for _ in range(6):  # interleaved launches, no synchronisation between the streams
        for i, (tensors, st) in enumerate(zip(problems, streams)):
            with torch.cuda.stream(st):
                status, out, lse = run_forward(cuda, tensors, 2048, 2048, -1, st)
                assert status == 0
                results[i].append((out, lse))
    torch.cuda.synchronize(cuda)
    for i in range(2):
        for out, lse in results[i]:
            assert torch.equal(out.view(torch.int32), expected[i][0].view(torch.int32))
            assert torch.equal(lse.view(torch.int32), expected[i][1].view(torch.int32))
    assert api().device_status(clear=True) == 0


def test_release_scratch_then_forward(cuda):
    (q, k, v, mask), tensors = device_problem(cuda, 1, 8, 2048, 2048, 731)
    status, _, _ = run_forward(cuda, tensors, 2048, 2048, -1)
    assert status == 0
    torch.cuda.synchronize(cuda)
    assert api().release_scratch() == 0
    status, out, lse = run_forward(cuda, tensors, 2048, 2048, -1)
    assert status == 0
    expected = oracle.attention(q, k, v, mask, None, -1, forward_only=True, threads=oracle.cpu_count())
    assert_forward_close(out.cpu().numpy(), lse.cpu().numpy(), expected, "after release")
    assert np.isfinite(out.cpu().numpy()).all()
