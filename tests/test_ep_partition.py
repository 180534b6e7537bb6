"""CPU tests of the expert-parallel partition (the host copy of the logic the
device runs every forward): every rank derives the same split of the global
expert-sorted rows into `world` equal slices, and every source row lands in
exactly one slot of the right expert in its slice.  One test runs the
counts exchange over a world_size-2 gloo group."""
import os

import numpy as np
import pytest

import moe_b200 as M


def simulate(counts):
    """Map every (source rank, expert, local rank-in-expert) row to its
    (slice, slot) the way the gather kernel does, and check the result."""
    G, E = counts.shape
    plans = [M.ep_partition(counts, q) for q in range(G)]
    chunk = plans[0][3]
    M_rows = int(counts.sum())
    assert all(p[3] == chunk for p in plans)
    seen = {}
    for r in range(G):
        _, base_r, _, _ = plans[r]
        for e in range(E):
            for lr in range(counts[r, e]):
                gp = int(base_r[e]) + lr
                q, p = divmod(gp, chunk)
                assert 0 <= q < G
                cnt_q = plans[q][0]
                off_q = np.concatenate([[0], np.cumsum(cnt_q)])
                assert off_q[e] <= p < off_q[e] + cnt_q[e], "row lands outside its expert block"
                assert (q, p) not in seen
                seen[(q, p)] = (r, e, lr)
    sizes = [int(p[0].sum()) for p in plans]
    assert sum(sizes) == M_rows == len(seen)
    assert max(sizes) <= chunk and max(sizes) - min(sizes) <= chunk
    # every slice but the last is full: work is balanced to within one slice
    assert all(s == chunk for s in sizes[:-1]) or M_rows < G
    for e in range(E):
        assert sum(int(p[0][e]) for p in plans) == counts[:, e].sum()
    return sizes


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_partition_random(world):
    rng = np.random.default_rng(world)
    for trial in range(5):
        E = int(rng.integers(1, 20))
        counts = rng.integers(0, 30, size=(world, E)).astype(np.int32)
        simulate(counts)


def test_partition_skewed_zipf():
    # one expert holds most of the rows: it is split across slices
    G, E = 8, 16
    p = np.arange(1, E + 1, dtype=np.float64) ** -1.1
    counts = np.stack([np.random.default_rng(r).multinomial(400, p / p.sum()) for r in range(G)])
    sizes = simulate(counts.astype(np.int32))
    assert max(sizes) - min(sizes) <= 1 or len(set(sizes[:-1])) == 1


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
