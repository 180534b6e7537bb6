"""The host-buffer forward (moe_b200_forward) pipelines its copies over token
chunks when the input is large (>= 64 MB) on the TF32 and FP32 paths: H2D of
one chunk and D2H of another overlap the compute of a third.  Each row's
result must not depend on the chunking: the outputs, router probabilities
and expert ids equal the device-buffer call on the whole batch bit for bit,
for token counts that do and do not divide into router tiles."""
import numpy as np
import pytest
import torch

import moe_b200 as M
import oracle_lib as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("path", [M.PATH_TF32, M.PATH_FP32, M.PATH_AUTO], ids=["tf32", "fp32", "auto"])
@pytest.mark.parametrize("T", [17000, 36864])
def test_pipelined_host_forward_equals_device(moe, T, path):
    d, E, k, F = 1024, 16, 2, 512
    w = M.MoEWeights.synth(7, 0.02, d, F, E, k)
    x = O.synth(7, O.stream_x(), T * d, 1.0).reshape(T, d)
    bias = O.synth(7, O.stream_bias(), E, 1.0)
    out_h, probs_h, ids_h = M.moe_forward(w, x, bias=bias, path=path)
    # an explicit chunk count gives the same bits too
    out_4 = np.empty_like(out_h)
    M.moe_forward_host_ptr(w, x.ctypes.data, T, out_4.ctypes.data, None, None,
                           bias.ctypes.data, path=path, host_chunks=4)
    assert np.array_equal(out_4, out_h)
    dev = torch.device("cuda", 0)
    xd = torch.from_numpy(x).to(dev)
    bd = torch.from_numpy(bias).to(dev)
    out = torch.empty_like(xd)
    probs = torch.empty(T, E, device=dev)
    ids = torch.empty(T, k, dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    M.moe_forward_device(w, xd.data_ptr(), T, out.data_ptr(), probs.data_ptr(), ids.data_ptr(),
                         bias_ptr=bd.data_ptr(), path=path, stream=s)
    torch.cuda.synchronize()
    assert np.array_equal(out_h, out.cpu().numpy())
    assert np.array_equal(probs_h, probs.cpu().numpy())
    assert np.array_equal(ids_h, ids.cpu().numpy())
    w.free()


def test_pipelined_block_ffn_equals_device(moe):
    """moe_b200_block_ffn on host buffers (RMSNorm + MoE + residual in place,
    pipelined over chunks) equals the device-buffer call bit for bit."""
    T, d, E, k, F = 20000, 1024, 16, 2, 512
    w = M.MoEWeights.synth(3, 0.02, d, F, E, k)
    x = O.synth(3, O.stream_x(), T * d, 4.0).reshape(T, d)
    rms = (1.0 + O.synth(3, O.stream_rms(), d, 0.1)).astype(np.float32)
    x_h, xn_h, probs_h, ids_h = M.block_ffn(w, x, rms, path=M.PATH_TF32)
    dev = torch.device("cuda", 0)
    xd = torch.from_numpy(x.copy()).to(dev)
    rd = torch.from_numpy(rms).to(dev)
    xn = torch.empty_like(xd)
    probs = torch.empty(T, E, device=dev)
    ids = torch.empty(T, k, dtype=torch.int32, device=dev)
    M.block_ffn_device(w, rd.data_ptr(), 1e-5, xd.data_ptr(), T, xn.data_ptr(), probs.data_ptr(),
                       ids.data_ptr(), path=M.PATH_TF32,
                       stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(x_h, xd.cpu().numpy())
    assert np.array_equal(xn_h, xn.cpu().numpy())
    assert np.array_equal(probs_h, probs.cpu().numpy())
    assert np.array_equal(ids_h, ids.cpu().numpy())
    w.free()
