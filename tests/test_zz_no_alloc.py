"""GPU test of moe_b200_forward_noalloc, the entry point for callers that
cannot allocate device memory while they run (a fixed-budget serving loop,
a program whose device memory belongs to another framework's allocator).
All of its intermediates live in a static 16 MiB array inside the library.

It is checked through the C-ABI against the regular device entry point on
the same FP32 expert path, and against the CPU oracle (the restatement of
the reference's moe_forward), on two calls in a row with different inputs, so
that whatever the first call leaves in the shared array cannot leak into
the second.  The tolerances are the parity tests' own: probabilities within
2e-6 (the regular entry point may sum the router logits in another order),
routing identical except where two experts' logits lie within 1e-6, layer
output within 1e-5.  This file is named to be collected last.
"""
import numpy as np
import pytest

import moe_b200 as M
import oracle_lib as O

pytestmark = pytest.mark.gpu

TOL = 1e-5        # the FP32 path's layer tolerance (max|Δ| / max|ref|)
PROBS_TOL = 2e-6  # router probabilities


def _upload(p):
    return M.MoEWeights.upload(p.W_router, [e[0] for e in p.experts], [e[1] for e in p.experts],
                               [e[2] for e in p.experts], p.k)


def _run_both(w, x_np, bias_np, E, k):
    import torch
    T, d = x_np.shape
    s = torch.cuda.Stream()
    x = torch.from_numpy(x_np).cuda()
    bias = torch.from_numpy(bias_np).cuda() if bias_np is not None else None
    bptr = bias.data_ptr() if bias is not None else None
    outs = []
    for noalloc in (False, True):
        out = torch.full((T, d), float("nan"), device="cuda")
        probs = torch.full((T, E), float("nan"), device="cuda")
        ids = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        if noalloc:
            M.moe_forward_noalloc(w, x.data_ptr(), T, out.data_ptr(), probs.data_ptr(),
                                  ids.data_ptr(), bias_ptr=bptr, stream=s.cuda_stream)
        else:
            M.moe_forward_device(w, x.data_ptr(), T, out.data_ptr(), probs.data_ptr(),
                                 ids.data_ptr(), bias_ptr=bptr, path=M.PATH_FP32,
                                 stream=s.cuda_stream)
        s.synchronize()
        outs.append((out.cpu().numpy(), probs.cpu().numpy(), ids.cpu().numpy()))
    return outs


def test_noalloc_matches_device_entry_point_two_calls(moe):
    p = O.MoEProblem(96, 384, 8, 2, 1536, seed=11)
    w = _upload(p)
    x2 = O.synth(12, O.stream_x(), 33 * 384, 1.0).reshape(33, 384)
    bias2 = O.synth(12, O.stream_bias(), 8, 1.0)
    for x, bias in ((p.x, None), (x2, bias2)):
        (r_out, r_probs, r_ids), (n_out, n_probs, n_ids) = _run_both(w, x, bias, p.E, p.k)
        assert np.isfinite(n_out).all()
        logits = np.empty((x.shape[0], p.E), np.float32)
        O.oracle().oracle_router(O._f(np.ascontiguousarray(x)), x.shape[0], x.shape[1],
                                 O._f(p.W_router), O._f(bias), p.E, p.k, O._f(logits),
                                 None, None, None)
        for t in np.nonzero(np.any(n_ids != r_ids, axis=1))[0]:
            assert O.routing_mismatch_allowed(logits[t], n_ids[t], r_ids[t], p.k)
        assert np.max(np.abs(n_probs - r_probs)) <= PROBS_TOL
        assert O.rel_err(n_out, r_out) < TOL
        # and against the CPU restatement of the reference's moe_forward
        q = O.MoEProblem(x.shape[0], 384, 8, 2, 1536, seed=11, bias=bias)
        q.x = np.ascontiguousarray(x)
        want, _, _ = q.oracle_forward(forced_ids=n_ids)
        assert O.rel_err(n_out, want) < TOL
    w.free()


_FRESH_PROCESS = r"""
import sys, torch
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
import moe_b200 as M, oracle_lib as O
M.init(0)
p = O.MoEProblem(8, 384, 8, 2, 1536, seed=5)
w = M.MoEWeights.upload(p.W_router, [e[0] for e in p.experts], [e[1] for e in p.experts],
                        [e[2] for e in p.experts], p.k)
x = torch.randn(400, 384, device="cuda")
out = torch.empty_like(x)
probs = torch.empty(400, 8, device="cuda")
ids = torch.empty(400, 2, dtype=torch.int32, device="cuda")
M.moe_forward_noalloc(w, x.data_ptr(), 40, out.data_ptr(), probs.data_ptr(), ids.data_ptr())
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
M.moe_forward_noalloc(w, x.data_ptr(), 400, out.data_ptr(), probs.data_ptr(), ids.data_ptr())
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
assert torch.isfinite(out).all()
print("FREE", free0, free1)
"""


def test_noalloc_allocates_nothing_in_a_fresh_process():
    """In a new process the library has no workspace yet, so a call that fell
    back on it would have to allocate: 400 tokens need about 8 MB of
    intermediates, beyond the driver's 2 MB allocation granularity.  After a
    40-token warm-up (which loads the kernels), the device's free memory must
    not move across the 400-token call."""
    import subprocess
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    r = subprocess.run([sys.executable, "-c", _FRESH_PROCESS, str(repo / "llm.c_b200"),
                        str(repo / "tests")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    free0, free1 = (int(v) for v in r.stdout.split("FREE")[1].split())
    assert free0 == free1, f"free device memory moved by {free0 - free1} bytes"


def test_noalloc_rejects_oversized_call(moe):
    import torch
    w = M.MoEWeights.synth(3, 0.02, 1024, 4096, 8, 2)
    T = 4096                       # needs ~200 MB of intermediates
    x = torch.zeros((T, 1024), device="cuda")
    out = torch.empty_like(x)
    with pytest.raises(M.MoEError) as ei:
        M.moe_forward_noalloc(w, x.data_ptr(), T, out.data_ptr())
    assert ei.value.status == M.E_INVALID
    assert "static array" in str(ei.value)
    w.free()
