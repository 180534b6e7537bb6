"""CTA-pair (tcgen05 cta_group::2, 256×256 tiles over two SMs) TF32 grouped
GEMMs against the single-SM kernels and the oracle.

The TF32 path uses the single-SM 128-row kernels by default; opts.cta_pair
= 1 selects the pair kernels (up/gate always, down when d_pad % 256 == 0).
Both compute the same products in the same K order, so their outputs agree
to fp32 rounding; each is checked against the oracle on a row subset
(TF32 tolerance 2e-3).  Shapes cover expert groups smaller than one CTA's
128 rows (the second CTA of the pair has no valid rows), groups straddling
the 128/256-row boundaries, empty experts, and a ragged d (down on the
single-SM kernel, up/gate on the pair)."""
import numpy as np
import pytest

import moe_b200 as M
import oracle_lib as O
from golden import make_golden as G

pytestmark = pytest.mark.gpu

GOLDEN = G.moe_fixtures()


def _upload(p):
    return M.MoEWeights.upload(p.W_router, [e[0] for e in p.experts], [e[1] for e in p.experts],
                               [e[2] for e in p.experts], p.k)


@pytest.mark.parametrize("cta_pair", [True, False], ids=["pair", "single"])
@pytest.mark.parametrize("case", GOLDEN, ids=lambda p: p.stem)
def test_golden_tf32_both_kernels(moe, case, cta_pair):
    z = np.load(case)
    p = O.MoEProblem(int(z["T"]), int(z["d"]), int(z["E"]), int(z["k"]), int(z["F"]),
                     seed=int(z["seed"]), w_std=float(z["w_std"]))
    tw = str(z["tweak"])
    G.apply_tweak(p, None if tw == "None" else tw)
    w = _upload(p)
    out, probs, ids = M.moe_forward(w, p.x, path=M.PATH_TF32, cta_pair=cta_pair)
    w.free()
    rows = z["rows"]
    # rows whose routing differs at a near-tie are recomputed with the GPU's ids
    want, _, _ = p.oracle_forward(rows=rows, forced_ids=ids)
    assert O.rel_err(out[rows], want) < 2e-3


SHAPES = [
    # T,    d,   E,  k,  F,    bias
    (700, 512, 64, 2, 640, None),        # ~22 rows per expert: pair's 2nd CTA idle
    (3000, 512, 12, 3, 700, "normal"),   # skewed loads, ragged F (F_pad 768)
    (4100, 256, 16, 1, 384, None),       # ~256 rows per expert: 256-row boundary
    (1500, 320, 8, 2, 512, "normal"),    # d_pad 384: down on the single-SM kernel
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"T{s[0]}_d{s[1]}_E{s[2]}_k{s[3]}_F{s[4]}")
def test_pair_matches_single_and_oracle(moe, shape):
    T, d, E, k, F, bias = shape
    p = O.MoEProblem(T, d, E, k, F, seed=7, bias=bias)
    w = _upload(p)
    a_out, a_probs, a_ids = M.moe_forward(w, p.x, p.bias, path=M.PATH_TF32, cta_pair=True)
    counts = M.last_counts(w)
    b_out, b_probs, b_ids = M.moe_forward(w, p.x, p.bias, path=M.PATH_TF32, cta_pair=False)
    w.free()
    assert np.array_equal(a_ids, b_ids) and np.array_equal(a_probs, b_probs)
    assert counts.sum() == T * k
    # same products, same K order: agreement to fp32 rounding
    assert O.rel_err(a_out, b_out) < 1e-5
    rows = np.sort(np.random.default_rng(1).choice(T, 64, replace=False)).astype(np.int32)
    want, _, _ = p.oracle_forward(rows=rows, forced_ids=a_ids)
    assert O.rel_err(a_out[rows], want) < 2e-3


def test_pair_deterministic(moe):
    p = O.MoEProblem(3000, 512, 12, 3, 700, seed=3)
    w = _upload(p)
    a = M.moe_forward(w, p.x, path=M.PATH_TF32, cta_pair=True)
    b = M.moe_forward(w, p.x, path=M.PATH_TF32, cta_pair=True)
    w.free()
    for u, v in zip(a, b):
        assert np.array_equal(u, v)


# 3xTF32 decode-sized path on CTA pairs: the same products in the same order
# as the single-CTA kernel, so the outputs agree to fp32 rounding; each is
# checked against the oracle at the FP32-path tolerance.
DEC_SHAPES = [
    # T,   d,    E,  k,  F,    bias
    (256, 512, 16, 4, 640, None),        # d_pad 512: down on pairs too; ~64 rows per expert
    (96, 320, 8, 2, 384, "normal"),      # d_pad 384: down on single CTAs, up/gate on pairs
    (1, 256, 8, 2, 512, None),           # one token
    (700, 256, 64, 1, 256, None),        # ~11 rows per expert, many experts
]


@pytest.mark.parametrize("shape", DEC_SHAPES, ids=lambda s: f"T{s[0]}_d{s[1]}_E{s[2]}_k{s[3]}_F{s[4]}")
def test_decode_pair_matches_single_and_oracle(moe, shape):
    T, d, E, k, F, bias = shape
    p = O.MoEProblem(T, d, E, k, F, seed=11, bias=bias)
    w = _upload(p)
    a_out, a_probs, a_ids = M.moe_forward(w, p.x, p.bias, path=M.PATH_TF32X3, cta_pair=True)
    b_out, b_probs, b_ids = M.moe_forward(w, p.x, p.bias, path=M.PATH_TF32X3, cta_pair=False)
    w.free()
    assert np.array_equal(a_ids, b_ids) and np.array_equal(a_probs, b_probs)
    assert O.rel_err(a_out, b_out) < 1e-6
    rows = np.arange(T, dtype=np.int32) if T <= 64 else \
        np.sort(np.random.default_rng(2).choice(T, 64, replace=False)).astype(np.int32)
    want, _, _ = p.oracle_forward(rows=rows, forced_ids=a_ids)
    assert O.rel_err(a_out[rows], want) < 1e-5


def test_decode_pair_deterministic(moe):
    p = O.MoEProblem(256, 512, 16, 4, 640, seed=5)
    w = _upload(p)
    a = M.moe_forward(w, p.x, path=M.PATH_TF32X3, cta_pair=True)
    b = M.moe_forward(w, p.x, path=M.PATH_TF32X3, cta_pair=True)
    w.free()
    for u, v in zip(a, b):
        assert np.array_equal(u, v)
