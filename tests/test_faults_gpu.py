"""Failure detection without a GPU fault (1 GPU).

  * an allocation that fails (the library's fault-injection hook) is
    reported as MOE_B200_E_NOMEM, for weights and for workspace growth, and
    the next call succeeds with correct results;
  * a bounded device wait that nobody satisfies (the tensor-core kernels'
    own mbarrier helper, 1 ms limit, nothing else in flight) returns
    MOE_B200_E_TIMEOUT with the site in the status word, and the device
    stays usable;
  * expert parallel: a group whose other rank never joins, and a group made
    from a bad id, end in the host watchdog (the communicator is aborted)
    with MOE_B200_E_TIMEOUT or MOE_B200_E_NCCL instead of blocking for good;
    these run in child processes with their own time limit, so that even a
    host-side hang could not stall the suite.
llm.c's own convention for all of these is abort() with a message
(src/transformer.c:28-32); the llm.c drop-ins keep it, the C-ABI returns the
status."""
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import pytest

import moe_b200 as M
import oracle_lib as O

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent


def _problem():
    return O.MoEProblem(200, 256, 8, 2, 384, seed=4)


def _upload(p):
    return M.MoEWeights.upload(p.W_router, [e[0] for e in p.experts], [e[1] for e in p.experts],
                               [e[2] for e in p.experts], p.k)


_ALLOC_CHILD = r"""
import sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
import numpy as np
import moe_b200 as M, oracle_lib as O
M.init(0)
def upload(p):
    return M.MoEWeights.upload(p.W_router, [e[0] for e in p.experts], [e[1] for e in p.experts],
                               [e[2] for e in p.experts], p.k)
def status(fn):
    try:
        fn()
        return 0
    except M.MoEError as e:
        return e.status
p = O.MoEProblem(200, 256, 8, 2, 384, seed=4)
M.debug_fail_alloc(1)                       # the router matrix of the upload
print("UPLOAD", status(lambda: upload(p)))
M.debug_fail_alloc(3)                       # the third allocation of a weight set: W_down
print("SYNTH", status(lambda: M.MoEWeights.synth(1, 0.02, 256, 384, 8, 2)))
w = upload(p)                               # the hook fired once per arming
out, _, ids = M.moe_forward(w, p.x, path=M.PATH_FP32)
want, _, _ = p.oracle_forward(forced_ids=ids)
print("AFTER_WEIGHTS", O.rel_err(out, want))
# a fresh process has no workspace: the next forward of a larger T grows it
q = O.MoEProblem(4096, 256, 8, 2, 384, seed=4)
M.debug_fail_alloc(1)
print("GROW", status(lambda: M.moe_forward(w, q.x, path=M.PATH_FP32)))
out, _, ids = M.moe_forward(w, q.x, path=M.PATH_FP32)
rows = np.arange(0, q.T, 97, dtype=np.int32)
want, _, _ = q.oracle_forward(rows=rows, forced_ids=ids)
print("AFTER_GROW", O.rel_err(out[rows], want))
w.free()
"""


def test_allocation_failure_is_nomem_and_library_recovers():
    """Run in a new process, so the library starts without a workspace and
    the injected failure hits the allocations named in the child."""
    r = subprocess.run([sys.executable, "-c", _ALLOC_CHILD, str(REPO / "llm.c_b200"),
                        str(REPO / "tests")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    got = dict(ln.split(" ", 1) for ln in r.stdout.splitlines() if " " in ln)
    assert int(got["UPLOAD"]) == M.E_NOMEM
    assert int(got["SYNTH"]) == M.E_NOMEM
    assert float(got["AFTER_WEIGHTS"]) < 1e-5
    assert int(got["GROW"]) == M.E_NOMEM
    assert float(got["AFTER_GROW"]) < 1e-5


def test_bounded_device_wait_times_out_and_device_stays_usable(moe):
    M.debug_wait_probe(1000, arrive=True)             # satisfied wait: OK
    t0 = time.perf_counter()
    with pytest.raises(M.MoEError) as e:
        M.debug_wait_probe(1000, arrive=False)         # nobody arrives: 1 ms limit
    assert e.value.status == M.E_TIMEOUT
    assert "site 99" in str(e.value)
    assert time.perf_counter() - t0 < 5.0
    p = _problem()
    w = _upload(p)
    out, _, ids = M.moe_forward(w, p.x, path=M.PATH_TF32)
    want, _, _ = p.oracle_forward(forced_ids=ids)
    assert O.rel_err(out, want) < 2e-3
    w.free()


_EP_CHILD = r"""
import os, sys, time
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
os.environ["NCCL_NVLS_ENABLE"] = "0"
os.environ["MOE_B200_EP_TIMEOUT_MS"] = "1500"
import torch
import moe_b200 as M
M.init(0)
w = M.MoEWeights.synth(2, 0.02, 256, 384, 8, 2)
mode = sys.argv[3]
uid = M.ep_unique_id() if mode == "missing_rank" else bytes(M.EP_ID_BYTES)
rank = 0 if mode == "missing_rank" else 1
t0 = time.time()
try:
    M.EP(uid, rank, 2, 64, w)
    print("RESULT created")
except M.MoEError as e:
    print("RESULT", e.status, round(time.time() - t0, 2), str(e).replace("\n", " "))
# the process and the device stay usable
x = torch.randn(64, 256, device="cuda")
out = torch.empty_like(x)
M.moe_forward_device(w, x.data_ptr(), 64, out.data_ptr())
torch.cuda.synchronize()
print("USABLE", bool(torch.isfinite(out).all()))
"""


@pytest.mark.parametrize("mode", ["missing_rank", "bad_id"])
def test_expert_parallel_watchdog_ends_a_group_that_cannot_form(mode):
    r = subprocess.run([sys.executable, "-c", _EP_CHILD, str(REPO / "llm.c_b200"),
                        str(REPO / "tests"), mode], capture_output=True, text=True, timeout=180)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    res = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT")]
    assert res and res[0] != "RESULT created", r.stdout
    status = int(res[0].split()[1])
    assert status in (M.E_TIMEOUT, M.E_NCCL), res[0]
    assert float(res[0].split()[2]) < 60.0
    assert "USABLE True" in r.stdout
