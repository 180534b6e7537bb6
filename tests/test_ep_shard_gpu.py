"""Expert shards on one GPU: a shard's slots hold the experts it was built
with (in the given order), the single-GPU entry points reject a shard, and a
one-rank expert-parallel group over a shard whose slots hold the experts in
another order (plus an empty spare) gives the single-GPU forward's results
bit for bit (the FP32 and TF32 paths), so the slot mapping is right."""
import numpy as np
import pytest

import moe_b200 as M
import oracle_lib as O

pytestmark = pytest.mark.gpu


def test_shard_slots_and_rejection(moe):
    w = M.MoEWeights.synth_shard(3, 0.02, 256, 384, 8, 2, [5, 1, 6], 5)
    assert w.slots().tolist() == [5, 1, 6, -1, -1]
    x = np.zeros((4, 256), np.float32)
    with pytest.raises(M.MoEError) as e:
        M.moe_forward(w, x)
    assert e.value.status == M.E_INVALID
    w.free()
    with pytest.raises(M.MoEError):
        M.MoEWeights.synth_shard(3, 0.02, 256, 384, 8, 2, [5, 5], 3)     # repeated expert
    with pytest.raises(M.MoEError):
        M.MoEWeights.synth_shard(3, 0.02, 256, 384, 8, 2, [0, 1, 2], 2)  # more than the slots


@pytest.mark.parametrize("path", [M.PATH_FP32, M.PATH_TF32])
def test_one_rank_group_over_permuted_shard_matches_single_gpu(moe, path):
    p = O.MoEProblem(512, 256, 8, 2, 384, seed=8, bias="zipf")
    full = M.MoEWeights.upload(p.W_router, [e[0] for e in p.experts], [e[1] for e in p.experts],
                               [e[2] for e in p.experts], p.k)
    order = [7, 2, 0, 5, 3, 6, 1, 4]
    shard = M.MoEWeights.upload_shard(p.W_router, [p.experts[e][0] for e in order],
                                      [p.experts[e][1] for e in order],
                                      [p.experts[e][2] for e in order], p.k, order, 8)
    assert shard.slots().tolist() == order
    ep = M.EP(M.ep_unique_id(), 0, 1, p.T, shard)
    out, probs, ids = ep.forward(p.x, p.bias, path=path)
    r_out, r_probs, r_ids = M.moe_forward(full, p.x, p.bias, path=path)
    assert np.array_equal(ids, r_ids) and np.array_equal(probs, r_probs)
    assert np.array_equal(out, r_out)
    ep.rebalance()                                  # one rank, no spare: nothing to place
    assert np.array_equal(ep.placement()[0], np.argsort(order))
    counts_all, rows = ep.counts()
    assert rows == p.T * p.k and counts_all.sum() == p.T * p.k
    ep.destroy()
    shard.free()
    full.free()
