"""Generate the golden MoE fixtures in this folder by running the
UNMODIFIED reference moe_forward (llm.c src/transformer.c:287-366, built
into oracle/_ref/libllmref.so by oracle/Makefile) on seeded synthetic
inputs.

Inputs are not stored: every case records its generator parameters
(T, d, E, k, F, seed, w_std) and tests/oracle_lib.MoEProblem regenerates
the identical tensors.  Outputs stored per case:
  ids   [T×k] int32   expert ids in rank order (cache->expert_ids)
  probs [T×E] f32     full softmax (cache->router_probs)
  out   [R×d] f32     layer output for rows `rows` (R <= 256)
  out_sum             float64 sum of the full [T×d] output (checksum)

Special cases hand-built on top of the generator:
  ties_dup      expert 2's router column duplicates expert 1's, so every
                token has an exact tie between them (lower index must win)
  ties_zero_row token rows 0..3 are all-zero, so all E logits tie
                (ids must be 0, 1, ..., k-1)

Block cases (block_*.npz): the FFN half of block_forward
(src/transformer.c:752-767) — the reference's rms_norm, moe_forward and
the residual add — on oracle_lib.BlockProblem inputs (x ~ N(0, 4), rms_ffn
weights 1 + N(0, 0.1), eps 1e-5).  Stored per case:
  ids, probs          as above
  x_out [R×d] f32     x after the block for rows `rows`
  x_norm [R×d] f32    the reference's rms_norm output for those rows (its
                      1/sqrtf is a -ffast-math estimate, so these bits are
                      this host's; tests compare them within 5e-7)
  ffn_out [R×d] f32   the MoE output before the residual (cache->ffn_out)
  x_out_sum           float64 sum of the full x after the block

Run:  python tests/golden/make_golden.py   (needs the reference sources
built into oracle/_ref; the committed .npz files are what tests read)
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
import oracle_lib as O  # noqa: E402

CASES = [
    # name, T, d, E, k, F, seed, tweak
    ("kat_small", 64, 8, 4, 2, 16, 0, None),
    ("odd_shapes", 97, 40, 6, 3, 72, 5, None),
    ("k1_e16", 128, 64, 16, 1, 96, 7, None),
    ("k4_e32", 96, 128, 32, 4, 160, 9, None),
    ("ties_dup", 64, 32, 8, 2, 64, 3, "dup"),
    ("ties_zero_row", 32, 16, 8, 3, 32, 4, "zero"),
    ("c1", 2048, 256, 8, 2, 1024, 0, None),
]


BLOCK_CASES = [
    # name, T, d, E, k, F, seed  (d = 44: 16-lane chunks, one 8-lane chunk and a
    # 4-column tail; d = 13: no 16-lane chunk, a 5-column tail, unaligned rows)
    ("block_odd", 97, 44, 6, 3, 72, 5),
    ("block_d13", 33, 13, 4, 2, 24, 8),
    ("block_c1", 2048, 256, 8, 2, 1024, 0),
]


def moe_fixtures():
    """The MoE-layer fixtures (the block_* files hold block cases)."""
    return sorted(p for p in HERE.glob("*.npz") if not p.stem.startswith("block_"))


def build_problem(T, d, E, k, F, seed, tweak):
    p = O.MoEProblem(T, d, E, k, F, seed=seed)
    apply_tweak(p, tweak)
    return p


def apply_tweak(p, tweak):
    if tweak == "dup":
        p.W_router[:, 2] = p.W_router[:, 1]
    elif tweak == "zero":
        p.x[0:4, :] = 0.0


def main():
    if not O.ref_available():
        raise SystemExit("oracle/_ref/libllmref.so missing: run make -C oracle ref")
    for name, T, d, E, k, F, seed, tweak in CASES:
        p = build_problem(T, d, E, k, F, seed, tweak)
        out, probs, ids = p.ref_forward(threads=1)
        rows = np.arange(T, dtype=np.int32)
        if T > 256:
            rows = np.sort(np.random.default_rng(seed).choice(T, 256, replace=False)).astype(np.int32)
        np.savez_compressed(HERE / f"{name}.npz",
                            T=T, d=d, E=E, k=k, F=F, seed=seed,
                            tweak=str(tweak), w_std=np.float32(0.02),
                            ids=ids, probs=probs, rows=rows, out=out[rows],
                            out_sum=np.float64(out.astype(np.float64).sum()))
        print(f"{name}: T={T} d={d} E={E} k={k} F={F} -> {HERE / (name + '.npz')}")
    for name, T, d, E, k, F, seed in BLOCK_CASES:
        p = O.BlockProblem(T, d, E, k, F, seed=seed)
        x_out, x_norm, probs, ids, ffn_out = p.ref_block(threads=1)
        rows = np.arange(T, dtype=np.int32)
        if T > 256:
            rows = np.sort(np.random.default_rng(seed).choice(T, 256, replace=False)).astype(np.int32)
        np.savez_compressed(HERE / f"{name}.npz",
                            T=T, d=d, E=E, k=k, F=F, seed=seed, x_std=np.float32(4.0),
                            eps=np.float32(1e-5), ids=ids, probs=probs, rows=rows,
                            x_out=x_out[rows], x_norm=x_norm[rows], ffn_out=ffn_out[rows],
                            x_out_sum=np.float64(x_out.astype(np.float64).sum()))
        print(f"{name}: T={T} d={d} E={E} k={k} F={F} -> {HERE / (name + '.npz')}")


if __name__ == "__main__":
    main()
