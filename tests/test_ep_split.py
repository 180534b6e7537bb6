"""CPU tests of expert-parallel row placement (the host copies of what the
device runs every forward, and of the rebalance's placement):

  * ep_split: every source row (rank r, expert e, local position) lands in
    exactly one receive slot of a rank that holds e, inside that rank's
    segment for e; each holder's range is contiguous in the expert's global
    row order and, for replicated experts, starts on a 128-row tile; sharded
    experts with one holder go whole to it;
  * ep_place: replicas go only to spare slots of ranks that do not hold the
    expert yet, never lower the balance, and under c5's Zipf(1.1) popularity
    with 8 ranks (8 base experts, strided, and 4 spares each) bring the
    highest rank cost close to the mean, where the plain 8-per-rank sharding
    leaves the first rank (which holds expert 0) with over twice the mean;
  * both are deterministic, and two gloo ranks that all-gather their counts
    derive the same placement and split."""
import os

import numpy as np
import pytest

import moe_b200 as M


def base_place(E, G, n_slots, replicate_all=False):
    pl = -np.ones((G, E), np.int32)
    for q in range(G):
        ex = list(range(E)) if replicate_all else M.ep_shard_experts(E, G, q)
        for j, e in enumerate(ex):
            pl[q, e] = j
    return pl


def simulate(counts, place, n_slots):
    G, E = counts.shape
    sp = M.ep_split(counts, place, n_slots)
    nh, hold, beg, dst = sp["n_holders"], sp["holders"], sp["row_begin"], sp["recv_offset"]
    tot = counts.sum(axis=0)
    # receive segments of every rank: slot -> (offset, rows)
    seg = {}
    for q in range(G):
        off = 0
        rows_of_slot = {}
        for e in range(E):
            j = place[q, e]
            if j < 0:
                continue
            i = list(hold[e, :nh[e]]).index(q)
            rows_of_slot[j] = (e, int(beg[e, i + 1] - beg[e, i]))
        for j in range(n_slots):
            e, n = rows_of_slot.get(j, (-1, 0))
            seg[(q, j)] = (off, n, e)
            off += n
        assert sp["recv_rows"][q] == off
    seen = set()
    for e in range(E):
        assert nh[e] == int((place[:, e] >= 0).sum())
        assert list(hold[e, :nh[e]]) == sorted(np.nonzero(place[:, e] >= 0)[0].tolist())
        b = beg[e, :nh[e] + 1]
        assert b[0] == 0 and b[-1] == tot[e] and np.all(np.diff(b) >= 0)
        if nh[e] > 1:
            assert all(x % 128 == 0 or x == tot[e] for x in b)
        base = np.concatenate([[0], np.cumsum(counts[:, e])])
        for r in range(G):
            for lr in range(counts[r, e]):
                gp = base[r] + lr
                i = int(np.searchsorted(b, gp, side="right")) - 1
                q = int(hold[e, i])
                p = int(dst[e, i] + gp - b[i])
                off, n, se = seg[(q, place[q, e])]
                assert se == e and off <= p < off + n
                assert (q, p) not in seen
                seen.add((q, p))
    assert len(seen) == counts.sum()
    return sp


def zipf_counts(G, E, per_rank, s=1.1, seed=0):
    p = np.arange(1, E + 1, dtype=np.float64) ** -s
    return np.stack([np.random.default_rng(seed + r).multinomial(per_rank, p / p.sum())
                     for r in range(G)]).astype(np.int32)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_split_random_shards_and_replicas(world):
    rng = np.random.default_rng(world)
    for trial in range(4):
        E = int(rng.integers(world, 24))
        S = int(rng.integers(-(-E // world), E + 1))
        counts = rng.integers(0, 300, size=(world, E)).astype(np.int32)
        place = base_place(E, world, S)
        simulate(counts, place, S)
        full = base_place(E, world, E, replicate_all=True)
        simulate(counts, full, E)
        placed = M.ep_place(counts, place, S)
        simulate(counts, placed, S)


def test_single_holder_takes_the_whole_expert():
    G, E = 4, 8
    counts = np.arange(G * E, dtype=np.int32).reshape(G, E) * 7
    place = base_place(E, G, 2)
    sp = simulate(counts, place, 2)
    for e in range(E):
        assert sp["n_holders"][e] == 1 and sp["row_begin"][e, 1] == counts[:, e].sum()


def test_place_zipf_c5_balance():
    G, E, S = 8, 64, 12
    counts = zipf_counts(G, E, 16384)
    base = base_place(E, G, S)
    cost0 = simulate(counts, base, S)["cost"]
    placed = M.ep_place(counts, base, S)
    cost1 = simulate(counts, placed, S)["cost"]
    assert cost0.max() / cost0.mean() > 2.0        # plain sharding: rank 0 carries expert 0
    assert cost1.max() / cost1.mean() < 1.08
    assert cost1.max() <= cost0.max()
    # replicas only in spare slots, base experts kept in their slots
    for q in range(G):
        for e in M.ep_shard_experts(E, G, q):
            assert placed[q, e] == base[q, e]
        extra = [(e, placed[q, e]) for e in range(E) if placed[q, e] >= 0 and base[q, e] < 0]
        assert all(j >= E // G for _, j in extra)
        used = [j for j in placed[q] if j >= 0]
        assert len(used) == len(set(used)) <= S
    assert np.array_equal(placed, M.ep_place(counts, base, S))    # deterministic


def test_place_without_spares_changes_nothing():
    G, E = 4, 16
    counts = zipf_counts(G, E, 4096)
    base = base_place(E, G, E // G)
    assert np.array_equal(M.ep_place(counts, base, E // G), base)


def test_split_replicated_everywhere_balances():
    # every rank holds every expert (a full set on each rank)
    G, E = 8, 64
    counts = zipf_counts(G, E, 16384, seed=3)
    cost = simulate(counts, base_place(E, G, E, replicate_all=True), E)["cost"]
    assert cost.max() / cost.mean() < 1.05


def test_split_rejects_unheld_expert():
    G, E = 2, 4
    counts = np.ones((G, E), np.int32)
    place = base_place(E, G, 2)
    place[:, 3] = -1
    with pytest.raises(M.MoEError) as e:
        M.ep_split(counts, place, 2)
    assert e.value.status == M.E_INVALID


def test_split_empty():
    simulate(np.zeros((4, 5), np.int32), base_place(5, 4, 2), 2)


def _gloo_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        E, S = 16, 10
        mine = torch.from_numpy(zipf_counts(1, E, 2048, seed=50 + rank)[0])
        allc = [torch.zeros(E, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(allc, mine)
        counts = torch.stack(allc).numpy()
        placed = M.ep_place(counts, base_place(E, world, S), S)
        sp = M.ep_split(counts, placed, S)
        q.put((rank, counts.tolist(), placed.tolist(), sp["row_begin"].tolist(),
               sp["recv_offset"].tolist()))
    finally:
        dist.destroy_process_group()


def test_placement_over_gloo_world2():
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][1:] == res[1][1:]      # same counts, placement and split on both ranks
    counts, placed = np.array(res[0][1], np.int32), np.array(res[0][2], np.int32)
    simulate(counts, placed, 10)
