"""CPU tests of the expert-parallel partition (the host copy of the logic the
device runs every forward): every rank derives the same split of the global
expert-sorted rows into `world` equal slices, and every source row lands in
exactly one slot of the right expert in its slice.  One test runs the
counts exchange over a world_size-2 gloo group."""
import os

import numpy as np
import pytest

import moe_b200 as M


def simulate(counts, capacity=0):
    """Map every (source rank, expert, local rank-in-expert) row to its
    (slice, slot) the way the gather kernel does, and check the result."""
    G, E = counts.shape
    plans = [M.ep_partition(counts, q, capacity) for q in range(G)]
    starts = [p[2] for p in plans] + [plans[-1][2] + plans[-1][3]]
    M_rows = int(counts.sum())
    assert starts[0] == 0 and starts[-1] == M_rows and starts == sorted(starts)
    seen = {}
    for r in range(G):
        _, base_r, _, _ = plans[r]
        for e in range(E):
            for lr in range(counts[r, e]):
                gp = int(base_r[e]) + lr
                q = int(np.searchsorted(starts, gp, side="right")) - 1
                p = gp - starts[q]
                assert 0 <= q < G
                cnt_q = plans[q][0]
                off_q = np.concatenate([[0], np.cumsum(cnt_q)])
                assert off_q[e] <= p < off_q[e] + cnt_q[e], "row lands outside its expert block"
                assert (q, p) not in seen
                seen[(q, p)] = (r, e, lr)
    sizes = [int(p[0].sum()) for p in plans]
    assert sizes == [p[3] for p in plans]
    assert sum(sizes) == M_rows == len(seen)
    if capacity:
        assert max(sizes) <= capacity
    for e in range(E):
        assert sum(int(p[0][e]) for p in plans) == counts[:, e].sum()
    return plans, sizes


def cost(plan):
    """Cost units of a slice: 2 per 128-row tile of each expert, 1 per expert."""
    return sum(2 * ((int(n) + 127) // 128) + 1 for n in plan[0] if n > 0)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_partition_random(world):
    rng = np.random.default_rng(world)
    for trial in range(5):
        E = int(rng.integers(1, 20))
        counts = rng.integers(0, 30, size=(world, E)).astype(np.int32)
        simulate(counts)


def test_partition_skewed_zipf():
    # Zipf(1.1) popularity: a few experts hold most rows, dozens hold a
    # handful; the cost-balanced slices stay within a few percent of each
    # other in cost, where equal-row slices would not
    G, E = 8, 64
    p = np.arange(1, E + 1, dtype=np.float64) ** -1.1
    counts = np.stack([np.random.default_rng(r).multinomial(16384, p / p.sum())
                       for r in range(G)]).astype(np.int32)
    plans, sizes = simulate(counts)
    costs = [cost(pl) for pl in plans]
    assert max(costs) / np.mean(costs) < 1.03
    # a slice boundary inside an expert falls on a 128-row tile boundary
    # of that expert, except at the expert's end
    tot = counts.sum(0)
    goff = np.concatenate([[0], np.cumsum(tot)])
    for pl in plans[1:]:
        s = pl[2]
        e = int(np.searchsorted(goff, s, side="right")) - 1
        if e < E and goff[e] < s < goff[e + 1]:
            assert (s - goff[e]) % 128 == 0


def test_partition_capacity_fallback():
    G, E = 4, 8
    counts = np.zeros((G, E), np.int32)
    counts[:, 0] = 1000                   # one huge expert, tiny others
    counts[:, 1:] = 3
    plans, sizes = simulate(counts, capacity=(counts.sum() + G - 1) // G)
    assert max(sizes) - min(sizes) <= 1   # equal rows when cost slices would not fit


def test_partition_empty():
    simulate(np.zeros((4, 5), np.int32))


def _gloo_worker(rank, world, port, q):
    import torch.distributed as dist
    import torch
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        E = 6
        mine = torch.from_numpy(np.random.default_rng(100 + rank).integers(0, 50, E).astype(np.int32))
        allc = [torch.zeros(E, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(allc, mine)
        counts = torch.stack(allc).numpy()
        cnt, base, lo, rows = M.ep_partition(counts, rank)
        q.put((rank, counts.tolist(), cnt.tolist(), base.tolist(), lo, rows))
    finally:
        dist.destroy_process_group()


def test_partition_over_gloo_world2():
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
    counts = np.array(res[0][1], np.int32)
    assert counts.tolist() == res[1][1]          # both ranks saw the same counts
    simulate(counts)
    for rank, _, cnt, base, lo, rows in res:
        c2, b2, lo2, rows2 = M.ep_partition(counts, rank)
        assert cnt == c2.tolist() and base == b2.tolist() and lo == lo2 and rows == rows2
