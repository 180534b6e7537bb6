"""Multi-GPU test of the expert-parallel forward: 2 (or more) ranks, one
process per GPU, each holding a shard of the experts (its contiguous base
experts plus spare slots) and forwarding its share of the tokens.

Every row's arithmetic is independent of which rank computes it and with
which copy of the expert's weights, so each rank's output must equal a
single-GPU forward of the same tokens over the full expert set, bit for bit,
on every expert path, with one exception: TF32 on decode-sized expert
groups runs the weight-streaming kernel's one-pass mode, whose single-GPU
down GEMM adds two K halves while the expert-parallel one (rows written
straight to their owners) does not split K; there the two agree to the TF32
tolerance.

Checked before and after moe_b200_ep_rebalance (which must place replicas
of the hot experts of the Zipf case in spare slots, the same placement on
every rank), with equal and with unequal token counts per rank (one rank
with none), on AUTO and every explicit path; the host-buffer forward split into token
chunks equals the unsplit one bit for bit.  Skipped when fewer than 2 GPUs
are visible."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [
    # T total, d, E, k, F, seed, bias, spare slots per rank
    (256, 512, 32, 4, 640, 0, None, 2),
    (2048, 256, 16, 2, 512, 1, "zipf", 3),
]


def _n_gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _worker(rank, world, port, q):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "tests"))
    sys.path.insert(0, str(repo / "llm.c_b200"))
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    import moe_b200 as M
    import oracle_lib as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    results = []
    try:
        M.init(rank)
        for (T, d, E, k, F, seed, bias, spare) in CASES:
            p = O.MoEProblem(T, d, E, k, F, seed=seed, bias=bias)
            full = M.MoEWeights.upload(p.W_router, [e[0] for e in p.experts],
                                       [e[1] for e in p.experts], [e[2] for e in p.experts], k)
            mine = M.ep_shard_experts(E, world, rank)
            n_slots = len(mine) + spare
            shard = M.MoEWeights.upload_shard(p.W_router, [p.experts[e][0] for e in mine],
                                              [p.experts[e][1] for e in mine],
                                              [p.experts[e][2] for e in mine], k, mine, n_slots)
            obj = [M.ep_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            Tl = T // world
            ep = M.EP(obj[0], rank, world, Tl, shard)
            xs = np.ascontiguousarray(p.x[rank * Tl:(rank + 1) * Tl])
            # unequal counts: the last rank forwards no tokens, rank 0 half of its share
            uneq = {world - 1: 0, 0: Tl // 2}.get(rank, Tl)
            for phase in ("sharded", "rebalanced"):
                for path in (M.PATH_AUTO, M.PATH_FP32, M.PATH_TF32, M.PATH_TF32X3):
                    for n_tok in (Tl, uneq):
                        out, probs, ids = ep.forward(xs[:n_tok], p.bias, path=path)
                        r_out, r_probs, r_ids = M.moe_forward(full, xs[:n_tok], p.bias, path=path)
                        eff = path
                        if path == M.PATH_AUTO:
                            eff = M.PATH_TF32 if Tl * world * k / E >= 64 else M.PATH_TF32X3
                            r_out, r_probs, r_ids = M.moe_forward(full, xs[:n_tok], p.bias,
                                                                  path=eff)
                        onepass = eff == M.PATH_TF32 and Tl * world * k / E < 64
                        results.append(dict(rank=rank, case=(T, d, E), phase=phase, path=path,
                                            n_tok=n_tok, tol=2e-3 if onepass else 1e-6,
                                            ids_equal=bool(np.array_equal(ids, r_ids)),
                                            probs_equal=bool(np.array_equal(probs, r_probs)),
                                            out_equal=bool(np.array_equal(out, r_out)),
                                            rel_err=O.rel_err(out, r_out) if n_tok else 0.0))
                if phase == "sharded":
                    ep.forward(xs, p.bias)            # the counts the rebalance reads
                    counts_all, _ = ep.counts()
                    ep.rebalance()
                    placement = ep.placement()
                    results.append(dict(rank=rank, case=(T, d, E), placement=placement.tolist(),
                                        slots=shard.slots().tolist(), mine=mine,
                                        counts=counts_all.tolist(), n_slots=n_slots))
            # the host-buffer forward in 3 token chunks (3 collective forwards)
            # gives the 1-chunk results bit for bit
            one = ep.forward(xs, p.bias, path=M.PATH_TF32, host_chunks=1)
            three = ep.forward(xs, p.bias, path=M.PATH_TF32, host_chunks=3)
            results.append(dict(rank=rank, case=(T, d, E), chunks_equal=all(
                bool(np.array_equal(u, v)) for u, v in zip(one, three))))
            ep.forward(xs, p.bias)                # every rank's full share, then the counts
            counts_all, rows = ep.counts()
            results.append(dict(rank=rank, case=(T, d, E), counts_total=int(counts_all.sum()),
                                want_total=T * k, recv_rows=rows))
            dist.barrier()
            ep.destroy()
            shard.free()
            full.free()
        q.put((rank, results, None))
    except Exception as ex:   # report, do not hang the other rank
        q.put((rank, results, repr(ex)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_n_gpus() < 2, reason="needs 2 GPUs")
def test_ep_sharded_matches_single_gpu():
    import multiprocessing as mp
    import moe_b200 as M
    world = min(_n_gpus(), 4)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    errors = [(r, e) for r, _, e in got if e]
    assert not errors, errors
    placements = {}
    for _, res, _ in got:
        for r in res:
            if "counts_total" in r:
                # the last (full) forward: every token's k rows were routed
                assert r["counts_total"] == r["want_total"]
            elif "placement" in r:
                placements.setdefault(r["case"], []).append(r)
            elif "chunks_equal" in r:
                assert r["chunks_equal"], r
            else:
                assert r["ids_equal"] and r["probs_equal"], r
                assert r["out_equal"] or r["rel_err"] < r["tol"], r
    for case, rs in placements.items():
        pl = [np.array(r["placement"]) for r in rs]
        assert all(np.array_equal(pl[0], x) for x in pl[1:])       # one placement everywhere
        P = pl[0]
        for r in rs:                                               # each shard's slots agree
            slots = np.array(r["slots"])
            for e in range(P.shape[1]):
                j = P[r["rank"], e]
                if j >= 0:
                    assert slots[j] == e
            for e in r["mine"]:
                assert slots[list(r["mine"]).index(e)] == e        # base experts kept
        counts = np.array(rs[0]["counts"], np.int32)
        base = -np.ones_like(P)
        for r in rs:
            for j, e in enumerate(r["mine"]):
                base[r["rank"], e] = j
        assert np.array_equal(P, M.ep_place(counts, base, rs[0]["n_slots"]))
        if case[2] == 16:                                          # the Zipf case replicates
            assert (P >= 0).sum() > (base >= 0).sum()
