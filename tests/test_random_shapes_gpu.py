"""Randomised shapes on the B200 (fixed seeds, so the round-end run is
deterministic): each layer through the three forward paths against the
oracle (routing identical except at near-ties, outputs within the path's
tolerance on the oracle evaluated with the GPU's ids) and through both
backward paths against float64 autograd."""
import numpy as np
import pytest

import moe_b200 as M
import oracle_lib as O
import torch_ref

pytestmark = pytest.mark.gpu

FWD_TOL = {M.PATH_FP32: 1e-5, M.PATH_TF32: 2e-3, M.PATH_TF32X3: 1e-5}
BWD_TOL = {M.PATH_FP32: 1e-5, M.PATH_TF32: 4e-3}


def _shapes(n=12, seed=2024):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        E = int(rng.integers(1, 33))
        k = int(rng.integers(1, min(E, 8) + 1))
        out.append((int(rng.integers(1, 700)), int(rng.integers(1, 300)), E, k,
                    int(rng.integers(1, 400)), int(rng.integers(0, 2**31 - 1))))
    return out


SHAPES = _shapes()


def _upload(p):
    return M.MoEWeights.upload(p.W_router, [e[0] for e in p.experts], [e[1] for e in p.experts],
                               [e[2] for e in p.experts], p.k)


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "T%d_d%d_E%d_k%d_F%d" % s[:5])
def test_random_layer_all_paths(moe, shape):
    T, d, E, k, F, seed = shape
    p = O.MoEProblem(T, d, E, k, F, seed=seed, bias="normal")
    w = _upload(p)
    lg, oprobs, oids, _ = p.oracle_router()
    for path, tol in FWD_TOL.items():
        out, probs, ids = M.moe_forward(w, p.x, bias=p.bias, path=path)
        bad = [t for t in np.nonzero(np.any(ids != oids, axis=1))[0]
               if not O.routing_mismatch_allowed(lg[t], ids[t], oids[t], k)]
        assert not bad, f"path {path}: routing differs beyond near-ties at {bad[:5]}"
        assert np.max(np.abs(probs - oprobs)) < 2e-6
        want, _, _ = p.oracle_forward(forced_ids=ids)
        assert O.rel_err(out, want) < tol, f"path {path}"
    dy = (np.random.default_rng(seed % 1000).standard_normal((T, d)) * 0.1).astype(np.float32)
    _, _, ids = M.moe_forward(w, p.x, bias=p.bias, path=M.PATH_FP32)
    ref = torch_ref.moe_grads(p.x, p.W_router, p.bias, p.experts, ids, dy, 0.01)
    for path, tol in BWD_TOL.items():
        g = M.MoEGrads(w)
        dx, _ = M.moe_backward(w, p.x, dy, g, bias=p.bias, aux_coef=0.01, path=path)
        wr, b, gg, gu, gd = g.download()
        assert O.rel_err(dx, ref[0]) < tol, f"backward {path}: dx"
        assert O.rel_err(wr, ref[1]) < tol, f"backward {path}: router"
        for e in range(E):
            if np.any(ids == e):
                for name, a, r in (("gate", gg[e], ref[3][e]), ("up", gu[e], ref[4][e]),
                                   ("down", gd[e], ref[5][e])):
                    assert O.rel_err(a, r) < tol, f"backward {path}: {name}[{e}]"
        g.free()
    w.free()
