"""The FFN half of llm.c's block_forward (src/transformer.c:752-767):
RMSNorm, MoE, residual.  CPU pins of the oracle's restatement.

  * oracle_rms_norm against the reference's own rms_norm
    (src/matrix.c:666-713) for widths that exercise every phase of its
    AVX2 sum (16-lane chunks, the 8-lane chunk, the scalar tail).  The
    reference build's -ffast-math computes 1/sqrtf as a reciprocal-square-
    root estimate plus a Newton step (its bits depend on the host CPU), so
    the pin is 5e-7 relative per element, not bit equality; the sum order
    itself is pinned through the GPU kernel, which must equal the oracle
    bit for bit;
  * oracle_block_ffn against the reference's rms_norm + moe_forward +
    mat_add_inplace, and against the golden block fixtures the reference
    wrote (tests/golden/make_golden.py)."""
from pathlib import Path

import numpy as np
import pytest

import oracle_lib as O

GOLDEN = Path(__file__).resolve().parent / "golden"
BLOCK_CASES = ["block_odd", "block_d13", "block_c1"]

needs_ref = pytest.mark.skipif(not O.ref_available(), reason="reference build absent")


def _close(got, want, rel):
    """|got - want| <= rel * |want| elementwise (plus a denormal floor)."""
    g, w = got.astype(np.float64), want.astype(np.float64)
    return bool(np.all(np.abs(g - w) <= rel * np.abs(w) + 1e-30))


@needs_ref
@pytest.mark.parametrize("d", [1, 7, 8, 13, 16, 24, 44, 256, 384, 4096, 5120])
def test_oracle_rms_norm_matches_reference(d):
    p = O.BlockProblem(64, d, 2, 1, 8, seed=d, with_experts=False)
    p.x *= np.random.default_rng(d).uniform(0.01, 30.0, (64, 1)).astype(np.float32)
    assert _close(p.oracle_rms(), p.ref_rms(), 5e-7)


def test_oracle_rms_norm_definition():
    """Independent of the reference: rows scale to unit RMS, times the weights."""
    p = O.BlockProblem(16, 384, 2, 1, 8, seed=1, with_experts=False)
    xn = p.oracle_rms().astype(np.float64)
    x = p.x.astype(np.float64)
    want = x / np.sqrt((x * x).mean(1, keepdims=True) + 1e-5) * p.rms_w
    assert np.max(np.abs(xn - want) / np.abs(want).max()) < 1e-6


@needs_ref
@pytest.mark.parametrize("shape", [(97, 44, 6, 3, 72), (64, 256, 8, 2, 512)])
def test_oracle_block_matches_reference(shape):
    T, d, E, k, F = shape
    p = O.BlockProblem(T, d, E, k, F, seed=3)
    x_o, xn_o, probs_o, ids_o = p.oracle_block()
    x_r, xn_r, probs_r, ids_r, ffn_r = p.ref_block()
    assert _close(xn_o, xn_r, 5e-7)
    assert np.array_equal(ids_o, ids_r)
    assert np.max(np.abs(probs_o - probs_r)) < 1e-6
    # the MoE output within the layer tolerance; the block adds it to x in fp32
    ffn_o = p.moe_on(xn_o).oracle_forward()[0]
    assert O.rel_err(ffn_o, ffn_r) < 1e-5
    assert np.array_equal(x_o, p.x + ffn_o)
    assert O.rel_err(x_o, x_r) < 1e-6


@pytest.mark.parametrize("name", BLOCK_CASES)
def test_oracle_block_matches_golden(name):
    z = np.load(GOLDEN / f"{name}.npz")
    T, d, E, k, F, seed = (int(z[n]) for n in ("T", "d", "E", "k", "F", "seed"))
    p = O.BlockProblem(T, d, E, k, F, seed=seed, x_std=float(z["x_std"]), eps=float(z["eps"]))
    x_o, xn_o, probs_o, ids_o = p.oracle_block()
    rows = z["rows"]
    assert np.array_equal(ids_o, z["ids"])
    assert np.max(np.abs(probs_o - z["probs"])) < 1e-6
    assert _close(xn_o[rows], z["x_norm"], 5e-7)
    ffn_o = p.moe_on(xn_o).oracle_forward()[0]
    assert O.rel_err(ffn_o[rows], z["ffn_out"]) < 1e-5
    assert O.rel_err(x_o[rows], z["x_out"]) < 1e-6
    assert abs(x_o.astype(np.float64).sum() - float(z["x_out_sum"])) < 1e-6 * np.abs(x_o).sum()
