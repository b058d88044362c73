"""attention_fp32_forward_flash_workspace: the d = 32 flash forward with caller scratch. An operand
pre-pass splits every 64-key tile of K and V once into the caller's workspace, then the forward
(launched as the pre-pass's programmatic dependent) bulk-copies those stage images.

The prepared path runs when it pays for its pre-pass: grids beyond one wave of the split-warp
kernel, or windows of at least 24 key tiles; elsewhere the entry runs the plain flash kernel and
leaves the workspace untouched. The shapes below are chosen to take it (on a 148-SM B200) in each
CTA form: one Q tile, two Q tiles, and two threads per row.

Checked here, on the GPU:
* results against the oracle at shapes whose key windows do not start on a 64-key tile (radius),
  with padded keys, key counts that are not a multiple of 64, every CTA form; the kernel-name
  query names the prepared path for each;
* capture in a CUDA graph with a workspace allocated before capture: replays on new inputs give
  the eager call's bits;
* two streams running forwards at the same time, each with its own workspace: results equal the
  single-stream ones bit for bit;
* the workspace size query, the rejection of a null or short workspace, and a workspace that is
  16-byte but not 128-byte aligned (the plain kernel runs);
* the rotary form against rotary_fp32 followed by the workspace forward, bit for bit.
"""
from __future__ import annotations

import pytest

from attention_cases import assert_forward_close, make_inputs
from oracle import oracle
from test_rotary_gpu import put, tables

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

INVALID_VALUE = 1
PREPARED = "tcgen05-f16x2-flash-d32-prepared"


def api():
    from rocmkernels_b200 import attention

    return attention


def device_problem(cuda, batch, heads, queries, keys, seed, mask_fraction=0.0):
    q, k, v, _, mask = make_inputs(batch, heads, queries, keys, 32, seed=seed, dist="normal", mask_fraction=mask_fraction)
    tensors = [torch.from_numpy(x).to(cuda) for x in (q, k, v, mask)]
    return (q, k, v, mask), tensors


def new_workspace(cuda, batch, heads, keys):
    return torch.empty(api().attention_fp32_forward_flash_workspace_size(batch, heads, keys), dtype=torch.uint8, device=cuda)


def run_forward(cuda, tensors, queries, keys, radius, workspace, stream=None, capacity=None):
    dq, dk, dv, dmask = tensors
    batch, heads = dq.shape[0], dq.shape[1]
    out = torch.empty(batch, heads, queries, 32, device=cuda)
    lse = torch.empty(batch, heads, queries, 2, device=cuda)
    a = api()
    qs, ks = a.strides_of(dq), a.strides_of(dk)
    if capacity is not None:  # a raw address with an explicit byte count
        status = a.lib().attention_fp32_forward_flash_workspace(
            a.ptr(dq), a.ptr(dk), a.ptr(dv), a.ptr(dmask), a.ptr(out), a.ptr(lse), batch, heads, queries, keys, radius, qs, ks, ks,
            a.strides_of(out), workspace, capacity, None)
    else:
        status = a.attention_fp32_forward_flash_workspace(dq, dk, dv, dmask, out, lse, batch, heads, queries, keys, radius, qs, ks,
                                                          ks, a.strides_of(out), stream, workspace=workspace)
    return status, out, lse


# (batch, heads, queries, keys, radius, mask fraction): radius windows that start inside a key
# tile, ragged key counts, padded keys. Forms: two threads per row (cases 1, 2, 6), one Q tile
# (cases 3, 4), two Q tiles (case 5).
CASES = [(40, 4, 300, 300, 100, 0.0), (3, 60, 200, 333, 37, 0.2), (3, 4, 129, 2000, -1, 0.3), (2, 2, 777, 1600, 800, 0.1),
         (1, 100, 256, 2000, -1, 0.1), (16, 12, 256, 320, 70, 0.15)]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b{}h{}q{}k{}r{}m{}".format(*c))
def test_prepared_forward_matches_oracle(cuda, case):
    batch, heads, queries, keys, radius, fraction = case
    assert api().flash_workspace_kernel_name(batch, heads, queries, keys) == PREPARED
    (q, k, v, mask), tensors = device_problem(cuda, batch, heads, queries, keys, 701 + queries, fraction)
    status, out, lse = run_forward(cuda, tensors, queries, keys, radius, new_workspace(cuda, batch, heads, keys))
    assert status == 0
    expected = oracle.attention(q, k, v, mask, None, radius, forward_only=True, threads=oracle.cpu_count())
    assert_forward_close(out.cpu().numpy(), lse.cpu().numpy(), expected, f"prepared {case}")
    assert api().device_status(clear=True) == 0


def test_graph_capture_replays_the_forward(cuda):
    batch, heads, seq = 4, 3, 2048
    (_, _, _, _), tensors = device_problem(cuda, batch, heads, seq, seq, 711)
    workspace = new_workspace(cuda, batch, heads, seq)
    stream = torch.cuda.Stream(cuda)
    with torch.cuda.stream(stream):
        status, out, lse = run_forward(cuda, tensors, seq, seq, -1, workspace, stream)  # kernel attributes set outside capture
        assert status == 0
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            captured_status, graph_out, graph_lse = run_forward(cuda, tensors, seq, seq, -1, workspace,
                                                                torch.cuda.current_stream(cuda))
    assert captured_status == 0
    for seed in (712, 713):
        (_, _, _, _), fresh = device_problem(cuda, batch, heads, seq, seq, seed)
        for dst, src in zip(tensors, fresh):
            dst.copy_(src)
        graph.replay()
        torch.cuda.synchronize(cuda)
        status, eager_out, eager_lse = run_forward(cuda, tensors, seq, seq, -1, new_workspace(cuda, batch, heads, seq))
        torch.cuda.synchronize(cuda)
        assert status == 0
        assert torch.equal(graph_out.view(torch.int32), eager_out.view(torch.int32))
        assert torch.equal(graph_lse.view(torch.int32), eager_lse.view(torch.int32))
    del graph
    assert api().device_status(clear=True) == 0


def test_two_streams_with_their_own_workspaces(cuda):
    problems = [device_problem(cuda, 2, 12, 2048, 2048, seed)[1] for seed in (721, 722)]
    workspaces = [new_workspace(cuda, 2, 12, 2048) for _ in problems]
    expected = []
    for tensors, workspace in zip(problems, workspaces):
        status, out, lse = run_forward(cuda, tensors, 2048, 2048, -1, workspace)
        assert status == 0
        expected.append((out, lse))
    torch.cuda.synchronize(cuda)
    streams = [torch.cuda.Stream(cuda) for _ in problems]
    results = [[], []]
    for _ in range(6):  # interleaved launches, no synchronisation between the streams
        for i, (tensors, st) in enumerate(zip(problems, streams)):
            with torch.cuda.stream(st):
                status, out, lse = run_forward(cuda, tensors, 2048, 2048, -1, workspaces[i], st)
                assert status == 0
                results[i].append((out, lse))
    torch.cuda.synchronize(cuda)
    for i in range(2):
        for out, lse in results[i]:
            assert torch.equal(out.view(torch.int32), expected[i][0].view(torch.int32))
            assert torch.equal(lse.view(torch.int32), expected[i][1].view(torch.int32))
    assert api().device_status(clear=True) == 0


def test_workspace_size_and_alignment(cuda):
    batch, heads, seq = 1, 8, 2048
    size = api().attention_fp32_forward_flash_workspace_size(batch, heads, seq)
    assert size == batch * heads * (seq // 64) * 16400
    (q, k, v, mask), tensors = device_problem(cuda, batch, heads, seq, seq, 731)
    buffer = torch.empty(size + 512, dtype=torch.uint8, device=cuda)
    base = (buffer.data_ptr() + 255) // 256 * 256
    for capacity in (size - 1, 0):
        status, _, _ = run_forward(cuda, tensors, seq, seq, -1, base, capacity=capacity)
        assert status == INVALID_VALUE
    status, _, _ = run_forward(cuda, tensors, seq, seq, -1, None, capacity=size)
    assert status == INVALID_VALUE
    expected = oracle.attention(q, k, v, mask, None, -1, forward_only=True, threads=oracle.cpu_count())
    for address in (base, base + 16):  # 128-byte aligned: prepared; 16 bytes off: the plain kernel
        status, out, lse = run_forward(cuda, tensors, seq, seq, -1, address, capacity=size)
        assert status == 0
        torch.cuda.synchronize(cuda)
        assert_forward_close(out.cpu().numpy(), lse.cpu().numpy(), expected, f"workspace at +{address - base}")
    assert api().device_status(clear=True) == 0


def test_rotary_workspace_equals_rotary_then_forward(cuda):
    batch, heads, seq = 2, 8, 2048
    a = api()
    (_, _, _, _), (dq, dk, dv, dmask) = device_problem(cuda, batch, heads, seq, seq, 741)
    cos, sin = (put(cuda, t) for t in tables(batch, seq, 742))
    ts = a.Strides(seq * 32, 0, 32)
    # rotary_fp32 writes its outputs token-major: [batch][length][heads][32].
    rq = torch.empty(batch, seq, heads, 32, device=cuda)
    rk = torch.empty_like(rq)
    token = a.Strides(seq * heads * 32, 32, heads * 32)
    bhsd = a.strides_of(dq)
    assert a.rotary_fp32(dq, dk, cos, sin, rq, rk, batch, heads, seq, 0, bhsd, bhsd, ts, ts) == 0
    out = torch.empty(batch, heads, seq, 32, device=cuda)
    lse = torch.empty(batch, heads, seq, 2, device=cuda)
    assert a.attention_fp32_forward_flash_workspace(rq, rk, dv, dmask, out, lse, batch, heads, seq, seq, -1, token, token, bhsd,
                                                    a.strides_of(out), workspace=new_workspace(cuda, batch, heads, seq)) == 0
    fused_out = torch.empty_like(out)
    fused_lse = torch.empty_like(lse)
    assert a.attention_fp32_forward_flash_rotary_workspace(dq, dk, dv, cos, sin, dmask, fused_out, fused_lse, batch, heads, seq, seq,
                                                           -1, bhsd, bhsd, bhsd, ts, ts, a.strides_of(out),
                                                           workspace=new_workspace(cuda, batch, heads, seq)) == 0
    torch.cuda.synchronize(cuda)
    assert torch.equal(fused_out.view(torch.int32), out.view(torch.int32))
    assert torch.equal(fused_lse.view(torch.int32), lse.view(torch.int32))
    assert a.device_status(clear=True) == 0
