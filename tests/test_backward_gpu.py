"""MoE backward on the B200 (moe_b200_backward*) against float64 torch
autograd of the same forward with the GPU's routing held fixed
(tests/torch_ref.py).

Tolerance: max|Δ| / max|ref| for dx and every weight gradient, 1e-5 on
the FP32 FFMA path (FP32 arithmetic against a float64 reference) and 4e-3
on the TF32 tensor-core path (TF32 operands through two chained GEMMs);
the aux loss within 1e-5 relative on both.  Also: bit-stable repeats,
accumulation across calls, the device entry point equal to the host one,
edge shapes (T = 1, k = 1, E = 1, d not a multiple of 4) and rejected
arguments."""
import ctypes as C

import numpy as np
import pytest
import torch

import moe_b200 as M
import oracle_lib as O
import torch_ref

pytestmark = pytest.mark.gpu

TOL = {M.PATH_FP32: 1e-5, M.PATH_TF32: 4e-3}
PATHS = [M.PATH_FP32, M.PATH_TF32]
PATH_IDS = ["fp32", "tf32"]


def upload(p):
    return M.MoEWeights.upload(p.W_router, [e[0] for e in p.experts], [e[1] for e in p.experts],
                               [e[2] for e in p.experts], p.k)


def _dy(p, seed):
    return (np.random.default_rng(seed).standard_normal((p.T, p.d)) * 0.1).astype(np.float32)


def _check(p, w, dy, aux_coef, path=M.PATH_FP32):
    tol = TOL[path]
    g = M.MoEGrads(w)
    dx, aux = M.moe_backward(w, p.x, dy, g, bias=p.bias, aux_coef=aux_coef, path=path)
    got = g.download()
    _, _, ids = M.moe_forward(w, p.x, bias=p.bias, path=M.PATH_FP32)
    ref = torch_ref.moe_grads(p.x, p.W_router, p.bias, p.experts, ids, dy, aux_coef)
    errs = {"dx": O.rel_err(dx, ref[0]), "router": O.rel_err(got[0], ref[1])}
    if p.bias is not None:
        errs["bias"] = O.rel_err(got[1], ref[2])
    for name, a, b in (("gate", got[2], ref[3]), ("up", got[3], ref[4]), ("down", got[4], ref[5])):
        for e in range(p.E):
            if np.any(ids == e):
                errs[f"{name}[{e}]"] = O.rel_err(a[e], b[e])
            else:
                assert not np.any(a[e]), f"{name}[{e}] of an unused expert"
    worst = max(errs, key=errs.get)
    assert errs[worst] < tol, f"{worst}: {errs[worst]:.3e} (dx {errs['dx']:.3e})"
    assert abs(aux - ref[6]) <= 1e-5 * abs(ref[6])
    g.free()
    return dx, got


@pytest.mark.parametrize("shape,bias,aux", [
    ((97, 44, 6, 3, 72), "normal", 0.01),
    ((512, 256, 8, 2, 512), None, 0.0),
    ((300, 128, 16, 4, 256), "normal", 0.1),
    ((33, 13, 4, 2, 24), "normal", 0.05),       # d not a multiple of 4
    ((1, 64, 8, 2, 128), None, 0.01),           # one token
    ((64, 64, 8, 1, 96), None, 0.01),           # top-1
], ids=["odd", "mid", "k4", "d13", "T1", "k1"])
@pytest.mark.parametrize("path", PATHS, ids=PATH_IDS)
def test_backward_matches_autograd(moe, shape, bias, aux, path):
    T, d, E, k, F = shape
    p = O.MoEProblem(T, d, E, k, F, seed=T + d + E, bias=bias)
    w = upload(p)
    _check(p, w, _dy(p, T), aux, path)
    w.free()


@pytest.mark.parametrize("path", PATHS, ids=PATH_IDS)
def test_backward_larger_layer(moe, path):
    """c3-like proportions, scaled down: several 128-row tiles per expert,
    d_pad and 2·F_pad multiples of 256 (the 256-column tensor-core tiles)."""
    p = O.MoEProblem(2048, 512, 8, 2, 1024, seed=21, bias="normal")
    w = upload(p)
    _check(p, w, _dy(p, 7), 0.01, path)
    w.free()


def test_backward_tf32_close_to_fp32(moe):
    p = O.MoEProblem(1024, 384, 8, 2, 640, seed=13, bias="normal")
    w = upload(p)
    dy = _dy(p, 9)
    g32, g_tc = M.MoEGrads(w), M.MoEGrads(w)
    dx32, a32 = M.moe_backward(w, p.x, dy, g32, bias=p.bias, aux_coef=0.01, path=M.PATH_FP32)
    dxtc, atc = M.moe_backward(w, p.x, dy, g_tc, bias=p.bias, aux_coef=0.01, path=M.PATH_TF32)
    assert M.last_path() == M.PATH_TF32
    assert O.rel_err(dxtc, dx32) < TOL[M.PATH_TF32]
    assert a32 == atc                        # the router and L_aux are FP32 on both paths
    for a, b in zip(g_tc.download(), g32.download()):
        for u, v in zip(a if isinstance(a, list) else [a], b if isinstance(b, list) else [b]):
            assert O.rel_err(u, v) < TOL[M.PATH_TF32]
    g32.free()
    g_tc.free()
    w.free()


def test_backward_single_expert(moe):
    """E = 1: softmax over one logit is 1, so the router gets no gradient."""
    p = O.MoEProblem(50, 64, 1, 1, 96, seed=4)
    w = upload(p)
    dx, got = _check(p, w, _dy(p, 1), 0.5)
    assert not np.any(got[0])
    w.free()


def test_backward_bit_stable_and_accumulates(moe):
    p = O.MoEProblem(256, 128, 8, 2, 256, seed=9, bias="normal")
    w = upload(p)
    dy = _dy(p, 2)
    g1, g2 = M.MoEGrads(w), M.MoEGrads(w)
    dx1, a1 = M.moe_backward(w, p.x, dy, g1, bias=p.bias, aux_coef=0.02)
    dx2, a2 = M.moe_backward(w, p.x, dy, g2, bias=p.bias, aux_coef=0.02)
    assert np.array_equal(dx1, dx2) and a1 == a2
    one = g1.download()
    for a, b in zip(one, g2.download()):
        for u, v in zip(a if isinstance(a, list) else [a], b if isinstance(b, list) else [b]):
            assert np.array_equal(u, v)
    M.moe_backward(w, p.x, dy, g1, bias=p.bias, aux_coef=0.02)     # accumulates: g1 = 2·one
    two = g1.download()
    for a, b in zip(two, one):
        for u, v in zip(a if isinstance(a, list) else [a], b if isinstance(b, list) else [b]):
            assert np.array_equal(u, 2 * v)
    g1.zero()
    assert not np.any(g1.download()[4][0])
    g1.free()
    g2.free()
    w.free()


def test_backward_device_equals_host(moe):
    p = O.MoEProblem(200, 256, 8, 2, 384, seed=5, bias="normal")
    w = upload(p)
    dy = _dy(p, 3)
    gh = M.MoEGrads(w)
    dx_h, aux_h = M.moe_backward(w, p.x, dy, gh, bias=p.bias, aux_coef=0.01)
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(p.x).to(dev)
    tdy = torch.from_numpy(dy).to(dev)
    b = torch.from_numpy(p.bias).to(dev)
    dx = torch.empty_like(x)
    aux = torch.empty(1, device=dev)
    gd = M.MoEGrads(w)
    M.moe_backward_device(w, x.data_ptr(), p.T, tdy.data_ptr(), dx.data_ptr(), gd,
                          bias_ptr=b.data_ptr(), aux_coef=0.01, aux_ptr=aux.data_ptr(),
                          stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(dx.cpu().numpy(), dx_h)
    assert float(aux.item()) == aux_h
    for a, b2 in zip(gh.download(), gd.download()):
        for u, v in zip(a if isinstance(a, list) else [a], b2 if isinstance(b2, list) else [b2]):
            assert np.array_equal(u, v)
    gh.free()
    gd.free()
    w.free()


def test_backward_rejects_bad_arguments(moe):
    p = O.MoEProblem(16, 64, 4, 2, 64, seed=1)
    q = O.MoEProblem(16, 64, 8, 2, 64, seed=1)
    w, wq = upload(p), upload(q)
    g = M.MoEGrads(wq)
    with pytest.raises(M.MoEError) as e:               # gradients of another expert set
        M.moe_backward(w, p.x, _dy(p, 1), g)
    assert e.value.status == M.E_INVALID
    g.free()
    g = M.MoEGrads(w)
    dev = torch.device("cuda", 0)
    flat = torch.zeros(p.T * p.d + 1, device=dev)
    with pytest.raises(M.MoEError) as e:               # misaligned device buffer
        M.moe_backward_device(w, flat.data_ptr() + 4, p.T, flat.data_ptr(), flat.data_ptr(), g)
    assert e.value.status == M.E_INVALID
    dx, aux = M.moe_backward(w, p.x[:0], _dy(p, 1)[:0], g)   # T = 0: nothing to do
    assert dx.shape == (0, p.d) and aux == 0.0
    g.free()
    w.free()
    wq.free()


@pytest.mark.skipif(not O.ref_available(), reason="reference build absent")
def test_dense_backward_matches_reference_ffn_backward(moe):
    """One expert with a zero router is llm.c's dense FFN: the library's
    backward equals the reference's own ffn_backward (src/transformer.c:
    181-264) within the FP32 tolerance."""
    T, d, F = 300, 256, 384
    p = O.MoEProblem(T, d, 1, 1, F, seed=8)
    p.W_router[:] = 0.0
    w = upload(p)
    dy = _dy(p, 4)
    g = M.MoEGrads(w)
    dx, _ = M.moe_backward(w, p.x, dy, g, path=M.PATH_FP32)
    got = g.download()
    Wg, Wu, Wd = p.experts[0]
    dWg, dWu, dWd = np.zeros_like(Wg), np.zeros_like(Wu), np.zeros_like(Wd)
    rdx = np.empty_like(dx)
    O.ref().ref_ffn_backward(O._f(p.x), T, d, O._f(Wg), O._f(Wu), O._f(Wd), F, O._f(dy),
                             O._f(dWg), O._f(dWu), O._f(dWd), O._f(rdx))
    assert O.rel_err(dx, rdx) < TOL[M.PATH_FP32]
    for a, b in ((got[2][0], dWg), (got[3][0], dWu), (got[4][0], dWd)):
        assert O.rel_err(a, b) < TOL[M.PATH_FP32]
    assert not np.any(got[0])
    g.free()
    w.free()


def test_llmc_moe_backward_symbol(moe, monkeypatch):
    """llm.c-struct moe_backward: adds into the .grad matrices (existing
    contents kept), overwrites d_x, and equals the C-ABI backward."""
    monkeypatch.setenv("MOE_B200_AUX_COEF", "0.02")
    p = O.MoEProblem(200, 128, 8, 2, 192, seed=10)
    llmc = M.LlmcMoE(p.W_router, [e[0] for e in p.experts], [e[1] for e in p.experts],
                     [e[2] for e in p.experts], p.k, grads=True)
    for a in llmc.grads:
        a[:] = 1.0                                    # gradients already accumulated
    dy = _dy(p, 6)
    dx = llmc.backward(p.x, dy)
    w = upload(p)
    g = M.MoEGrads(w)
    want_dx, _ = M.moe_backward(w, p.x, dy, g, aux_coef=0.02, path=M.PATH_AUTO)
    wr, _, gg, gu, gd = g.download()
    assert np.array_equal(dx, want_dx)
    E = p.E
    assert np.array_equal(llmc.grads[0], (1.0 + wr).astype(np.float32))
    for e in range(E):
        assert np.array_equal(llmc.grads[1 + e], 1.0 + gg[e])
        assert np.array_equal(llmc.grads[1 + E + e], 1.0 + gu[e])
        assert np.array_equal(llmc.grads[1 + 2 * E + e], 1.0 + gd[e])
    L = M.lib()
    L.moe_b200_invalidate.argtypes = [C.c_void_p]
    assert L.moe_b200_invalidate(C.addressof(llmc.moe)) == 0
    g.free()
    w.free()
