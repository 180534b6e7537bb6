"""The FFN half of llm.c's block_forward (src/transformer.c:752-767) fused on
the B200: RMSNorm in front of the MoE, residual add in the combine.

  * the device RMSNorm equals the oracle's restatement bit for bit, at
    widths that exercise every phase of the reference's summation order
    and both the vector and the scalar load paths;
  * the fused call equals the unfused one bit for bit: x_out == x +
    moe_forward(x_norm) with the same device kernels;
  * against the reference's golden block fixtures: x_norm within 5e-7
    (the reference's -ffast-math 1/sqrtf is an estimate), the MoE output
    and x_out within the path tolerance of max|ffn_out| plus two ulps of
    the residual stream (the rounding of the sum);
  * the device-buffer call updates x in place and equals the host call,
    and misaligned device buffers are rejected;
  * llm.c's block structs through moe_b200_llmc_block_ffn, MoE and dense
    blocks, against the reference's rms_norm + moe_forward / ffn_forward +
    residual."""
import ctypes as C

import numpy as np
import pytest
import torch

import llmc_model as LM
import moe_b200 as M
import oracle_lib as O
from golden import make_golden as G

pytestmark = pytest.mark.gpu

TOL = {M.PATH_FP32: 1e-5, M.PATH_TF32: 2e-3, M.PATH_TF32X3: 1e-5}
PATHS = [M.PATH_FP32, M.PATH_TF32, M.PATH_TF32X3]
PATH_IDS = ["fp32", "tf32", "tf32x3"]


def upload(p):
    return M.MoEWeights.upload(p.W_router, [e[0] for e in p.experts], [e[1] for e in p.experts],
                               [e[2] for e in p.experts], p.k)


def _close(got, want, rel):
    g, w = got.astype(np.float64), want.astype(np.float64)
    return bool(np.all(np.abs(g - w) <= rel * np.abs(w) + 1e-30))


@pytest.mark.parametrize("d", [8, 13, 16, 44, 256, 384, 4096, 7168])
def test_rmsnorm_bit_exact_vs_oracle(moe, d):
    p = O.BlockProblem(96, d, 2, 1, 16, seed=d)
    p.x *= np.random.default_rng(d).uniform(0.01, 30.0, (96, 1)).astype(np.float32)
    w = upload(p)
    _, xn, _, _ = M.block_ffn(w, p.x, p.rms_w, path=M.PATH_FP32)
    assert np.array_equal(xn, p.oracle_rms())
    w.free()


@pytest.mark.parametrize("path", PATHS, ids=PATH_IDS)
@pytest.mark.parametrize("shape", [(97, 44, 6, 3, 72), (1000, 512, 16, 4, 768), (1, 256, 8, 2, 512)],
                         ids=["odd", "mid", "T1"])
def test_fused_equals_unfused(moe, path, shape):
    T, d, E, k, F = shape
    p = O.BlockProblem(T, d, E, k, F, seed=T + d, bias="normal")
    w = upload(p)
    x_out, xn, probs, ids = M.block_ffn(w, p.x, p.rms_w, bias=p.bias, path=path)
    ffn, probs2, ids2 = M.moe_forward(w, xn, bias=p.bias, path=path)
    assert np.array_equal(x_out, p.x + ffn)
    assert np.array_equal(probs, probs2) and np.array_equal(ids, ids2)
    # and the MoE part against the oracle on the same (bit-identical) x_norm
    assert np.array_equal(xn, p.oracle_rms())
    want, _, want_ids = p.moe_on(xn).oracle_forward()
    if np.array_equal(ids, want_ids):
        assert O.rel_err(ffn, want) < TOL[path]
    w.free()


@pytest.mark.parametrize("path", PATHS, ids=PATH_IDS)
@pytest.mark.parametrize("name", ["block_odd", "block_d13", "block_c1"])
def test_block_golden(moe, name, path):
    z = np.load(G.HERE / f"{name}.npz")
    T, d, E, k, F, seed = (int(z[n]) for n in ("T", "d", "E", "k", "F", "seed"))
    p = O.BlockProblem(T, d, E, k, F, seed=seed, x_std=float(z["x_std"]), eps=float(z["eps"]))
    w = upload(p)
    x_out, xn, probs, ids = M.block_ffn(w, p.x, p.rms_w, eps=float(z["eps"]), path=path)
    rows = z["rows"]
    assert np.array_equal(ids, z["ids"])
    assert np.max(np.abs(probs - z["probs"])) < 2e-6
    assert _close(xn[rows], z["x_norm"], 5e-7)
    ffn = x_out.astype(np.float64) - p.x
    scale = float(np.max(np.abs(z["ffn_out"])))
    # the MoE output within the path tolerance, plus the fp32 rounding of the sum
    lim = TOL[path] * scale + 2 * float(np.spacing(np.float32(np.max(np.abs(z["x_out"])))))
    assert np.max(np.abs(ffn[rows] - z["ffn_out"])) <= lim
    assert np.max(np.abs(x_out[rows].astype(np.float64) - z["x_out"])) <= lim
    w.free()


def test_block_device_in_place(moe):
    p = O.BlockProblem(300, 256, 8, 2, 512, seed=12)
    w = upload(p)
    want_x, want_xn, want_probs, want_ids = M.block_ffn(w, p.x, p.rms_w, path=M.PATH_TF32X3)
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(p.x.copy()).to(dev)
    rw = torch.from_numpy(p.rms_w).to(dev)
    xn = torch.empty_like(x)
    probs = torch.empty(p.T, p.E, device=dev)
    ids = torch.empty(p.T, p.k, dtype=torch.int32, device=dev)
    M.block_ffn_device(w, rw.data_ptr(), 1e-5, x.data_ptr(), p.T, xn.data_ptr(),
                       probs.data_ptr(), ids.data_ptr(), path=M.PATH_TF32X3,
                       stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(x.cpu().numpy(), want_x)
    assert np.array_equal(xn.cpu().numpy(), want_xn)
    assert np.array_equal(probs.cpu().numpy(), want_probs)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    # x_norm may be omitted (library workspace)
    x2 = torch.from_numpy(p.x.copy()).to(dev)
    M.block_ffn_device(w, rw.data_ptr(), 1e-5, x2.data_ptr(), p.T, path=M.PATH_TF32X3,
                       stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(x2.cpu().numpy(), want_x)
    # a device buffer off the 16-byte boundary is rejected, not read
    flat = torch.zeros(p.T * p.d + 1, device=dev)
    for call in (lambda: M.block_ffn_device(w, rw.data_ptr(), 1e-5, flat.data_ptr() + 4, p.T),
                 lambda: M.moe_forward_device(w, flat.data_ptr() + 4, p.T, x.data_ptr())):
        with pytest.raises(M.MoEError) as e:
            call()
        assert e.value.status == M.E_INVALID
    # T = 0 is a no-op
    M.block_ffn_device(w, rw.data_ptr(), 1e-5, x.data_ptr(), 0)
    w.free()


def _llmc_block_ffn():
    L = M.lib()
    L.moe_b200_llmc_block_ffn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    L.moe_b200_llmc_block_ffn.restype = None
    return L.moe_b200_llmc_block_ffn


def _np(mat):
    return np.ctypeslib.as_array(mat.data, shape=(mat.rows, mat.cols))


@pytest.mark.skipif(not O.ref_available(), reason="reference build absent")
@pytest.mark.parametrize("E,k", [(8, 2), (1, 1)], ids=["moe", "dense"])
def test_llmc_block_ffn_matches_reference(moe, E, k):
    R = O.ref()
    T, d, F = 40, 256, 384
    m = R.ref_model_init(512, 64, d, 2, 4, 2, 64, 0, F, E, k, 1e-5, 1e4, 17)
    model = C.cast(m, C.POINTER(LM.Model)).contents
    rng = np.random.default_rng(3)
    for layer in range(2):
        bw = model.weights.blocks[layer]
        rms = np.ctypeslib.as_array(bw.rms_ffn, shape=(d,))
        rms[:] = 1.0 + 0.1 * rng.standard_normal(d).astype(np.float32)   # llm.c inits ones
        x = (4.0 * rng.standard_normal((T, d))).astype(np.float32)
        xn = np.empty_like(x)
        R.ref_rms_norm(O._f(x), T, d, O._f(rms), 1e-5, O._f(xn))
        ffn = np.empty_like(x)
        if bw.use_moe:
            ex = [bw.moe.experts[e] for e in range(E)]
            probs = np.empty((T, E), np.float32)
            ids = np.empty((T, k), np.int32)
            assert R.ref_moe_forward(O._f(xn), T, d, O._f(np.ascontiguousarray(_np(bw.moe.W_router))),
                                     E, k, O._ptr_array([_np(e.W_gate) for e in ex]),
                                     O._ptr_array([_np(e.W_up) for e in ex]),
                                     O._ptr_array([_np(e.W_down) for e in ex]), F, O._f(ffn),
                                     O._f(probs), O._i(ids)) == 0
        else:
            R.ref_ffn_forward(O._f(xn), T, d, O._f(np.ascontiguousarray(_np(bw.ffn.W_gate))),
                              O._f(np.ascontiguousarray(_np(bw.ffn.W_up))),
                              O._f(np.ascontiguousarray(_np(bw.ffn.W_down))), F, O._f(ffn))
        want = x + ffn
        got = x.copy()
        mat = M.LlmcMatrix(O._f(got), None, T, d)
        _llmc_block_ffn()(C.addressof(mat), C.addressof(bw), None, C.addressof(model.cfg))
        lim = 1e-5 * float(np.max(np.abs(ffn))) + 2 * float(np.spacing(np.float32(np.max(np.abs(want)))))
        assert np.max(np.abs(got.astype(np.float64) - want)) <= lim
    O.release_ref_model(m)
