"""The bounded pipeline waits give up, report and leave the context usable.

Every mbarrier wait of the tensor-core kernels is bounded: when it runs out, the kernel records
status 1 in the device status word, drains its own copies and MMAs, writes NaN for the rows it
could not finish, frees TMEM and returns. Here a wait is made to run out on purpose, without any
fault: the wait-test build of the library (librocmkernels_attention_waittest.so, RK_WAIT_TEST)
bounds each wait at ~0.5 ms instead of ~1 s, and CTA 0 of its flash forward can be told never to
issue one key tile's TMA loads, so the barrier that tile would complete is never completed.

Checked, in a child process that loads the wait-test build: the launch returns 0 and the
process does not hang; the status word reads 1; CTA 0's rows are NaN (O and lse) while every
other row matches the oracle; after clearing the status and withholding nothing, the next call
on the same context is clean and matches the oracle everywhere.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parent.parent
WAIT_TEST_LIBRARY = REPO / "rocmkernels_b200" / "librocmkernels_attention_waittest.so"

_CHILD = r"""
import ctypes, json, sys, time
import numpy as np
import torch
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/tests")
from attention_cases import FORWARD_TOL, make_inputs, normwise
from oracle import oracle
from rocmkernels_b200 import attention as api

batch, heads, seq, withheld, cta_rows = (int(x) for x in sys.argv[2:7])
entry = sys.argv[7]
library = api.lib()
withhold = library.rocmkernels_attention_test_withhold_tile
withhold.argtypes, withhold.restype = [ctypes.c_int], ctypes.c_int
cuda = torch.device("cuda:0")
q, k, v, upstream, mask = make_inputs(batch, heads, seq, seq, 32, dist="normal", mask3=False)
expected = oracle.attention(q, k, v, mask, None, -1, threads=8, forward_only=True)
dq, dk, dv, dmask = (torch.from_numpy(x).to(cuda) for x in (q, k, v, mask))
st = api.Strides(heads * seq * 32, seq * 32, 32)
workspace = torch.empty(api.attention_fp32_forward_flash_workspace_size(batch, heads, seq), dtype=torch.uint8, device=cuda)

def run():
    out = torch.full((batch, heads, seq, 32), 7.0, device=cuda)
    lse = torch.full((batch, heads, seq, 2), 7.0, device=cuda)
    start = time.perf_counter()
    if entry == "workspace":
        status = api.attention_fp32_forward_flash_workspace(dq, dk, dv, dmask, out, lse, batch, heads, seq, seq, -1, st, st, st, st,
                                                            workspace=workspace)
    else:
        status = api.attention_fp32_forward_flash(dq, dk, dv, dmask, out, lse, batch, heads, seq, seq, -1, st, st, st, st)
    torch.cuda.synchronize(cuda)
    return status, time.perf_counter() - start, out.cpu().numpy(), lse.cpu().numpy()

name_of = api.flash_workspace_kernel_name if entry == "workspace" else api.flash_kernel_name
report = {"kernel": name_of(batch, heads, seq, seq)}
assert api.device_status(clear=True) == 0
assert withhold(withheld) == 0
status, seconds, out, lse = run()
report.update(failed_status=status, failed_seconds=seconds, device_status=api.device_status(clear=True))
report["cta0_nan"] = bool(np.isnan(out[0, 0, :cta_rows]).all() and np.isnan(lse[0, 0, :cta_rows]).all())
rest = np.ones((batch, heads, seq), bool)
rest[0, 0, :cta_rows] = False
report["rest_finite"] = bool(np.isfinite(out[rest]).all())
report["rest_error"] = max(normwise(out[rest], expected["output"][rest]), normwise(lse[rest], expected["lse"][rest]))
assert withhold(-1) == 0
status, seconds, out, lse = run()
report.update(clean_status=status, clean_device_status=api.device_status(clear=True),
              clean_error=max(normwise(out, expected["output"]), normwise(lse, expected["lse"])))
print("REPORT " + json.dumps(report))
"""


# (batch, heads, seq, withheld key tile, rows of CTA 0, entry), one case per CTA form of the d = 32
# forward on a 148-SM B200: one Q tile per CTA (a grid that fits one wave; tile 5 is loaded after
# the prefetch, when its stage is released), two Q tiles per CTA (200 one-tile CTAs: more than one
# wave, fewer than two per SM; tile 2 is one of the prefetched stages), and, through the workspace
# entry, the prepared kernel with two threads per row (320 one-tile CTAs, two per SM).
@pytest.mark.parametrize("batch,heads,seq,withheld,cta_rows,entry,kernel",
                         [(1, 1, 512, 5, 128, "plain", "tcgen05-f16x2-flash-d32"),
                          (1, 100, 256, 2, 256, "plain", "tcgen05-f16x2-flash-d32"),
                          (1, 160, 256, 2, 128, "workspace", "tcgen05-f16x2-flash-d32-prepared")])
def test_withheld_tile_runs_a_wait_out(cuda, batch, heads, seq, withheld, cta_rows, entry, kernel):
    assert WAIT_TEST_LIBRARY.exists(), "build it with `python -m rocmkernels_b200.build --wait-test`"
    env = dict(os.environ, ROCMKERNELS_ATTENTION_LIBRARY=str(WAIT_TEST_LIBRARY))
    args = [str(REPO), str(batch), str(heads), str(seq), str(withheld), str(cta_rows), entry]
    result = subprocess.run([sys.executable, "-c", _CHILD, *args], capture_output=True, text=True, timeout=300, env=env)
    assert result.returncode == 0, result.stdout[-2000:] + result.stderr[-4000:]
    line = next(l for l in result.stdout.splitlines() if l.startswith("REPORT "))
    report = json.loads(line[len("REPORT "):])
    assert report["kernel"] == kernel
    assert report["failed_status"] == 0            # the launch itself succeeded
    assert report["failed_seconds"] < 30.0         # every wait gave up; nothing hung
    assert report["device_status"] == 1           # kStatusWaitTimeout recorded
    assert report["cta0_nan"]                      # the rows CTA 0 could not finish
    assert report["rest_finite"] and report["rest_error"] <= 1e-5
    assert report["clean_status"] == 0 and report["clean_device_status"] == 0
    assert report["clean_error"] <= 1e-5           # the context is still usable
