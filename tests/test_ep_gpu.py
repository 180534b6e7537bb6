"""Multi-GPU test of the expert-parallel forward: 2 (or more) ranks, one
process per GPU, each forwarding its share of the tokens.  Every row's
arithmetic is independent of which rank computes it, so each rank's output
must equal a single-GPU forward of the same tokens, bit for bit, on every
expert path, with one exception: TF32 on decode-sized expert groups runs
the weight-streaming kernel's one-pass mode, whose single-GPU down GEMM
adds two K halves while the expert-parallel one (rows written straight to
their owners) does not split K; there the two agree to the TF32 tolerance.
Skipped when fewer than 2 GPUs are visible."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [
    # T total, d, E, k, F, seed, bias
    (256, 512, 32, 4, 640, 0, None),
    (2048, 256, 16, 2, 512, 1, "zipf"),
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
        for (T, d, E, k, F, seed, bias) in CASES:
            p = O.MoEProblem(T, d, E, k, F, seed=seed, bias=bias)
            w = M.MoEWeights.upload(p.W_router, [e[0] for e in p.experts],
                                    [e[1] for e in p.experts], [e[2] for e in p.experts], k)
            obj = [M.ep_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            Tl = T // world
            ep = M.EP(obj[0], rank, world, Tl, w)
            xs = np.ascontiguousarray(p.x[rank * Tl:(rank + 1) * Tl])
            for path in (M.PATH_FP32, M.PATH_TF32, M.PATH_TF32X3):
                for rep in range(2):
                    out, probs, ids = ep.forward(xs, p.bias, path=path)
                    r_out, r_probs, r_ids = M.moe_forward(w, xs, p.bias, path=path)
                    onepass = path == M.PATH_TF32 and T * k / E < 64
                    results.append(dict(rank=rank, case=(T, d, E), path=path, rep=rep,
                                        tol=2e-3 if onepass else 1e-6,
                                        ids_equal=bool(np.array_equal(ids, r_ids)),
                                        probs_equal=bool(np.array_equal(probs, r_probs)),
                                        out_equal=bool(np.array_equal(out, r_out)),
                                        rel_err=O.rel_err(out, r_out)))
            counts_all, rows = ep.counts()
            results.append(dict(rank=rank, case=(T, d, E), counts_total=int(counts_all.sum()),
                                want_total=T * k, slice_rows=rows))
            dist.barrier()
            ep.destroy()
            w.free()
        q.put((rank, results, None))
    except Exception as ex:   # report, do not hang the other rank
        q.put((rank, results, repr(ex)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_n_gpus() < 2, reason="needs 2 GPUs")
def test_ep_matches_single_gpu():
    import multiprocessing as mp
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
    for _, res, _ in got:
        for r in res:
            if "counts_total" in r:
                assert r["counts_total"] == r["want_total"]
                # cost-balanced slices: within the receive capacity (T·k/world + 25% + 256)
                per = r["want_total"] // world
                assert r["slice_rows"] <= per + per // 4 + 256
            else:
                assert r["ids_equal"] and r["probs_equal"], r
                assert r["out_equal"] or r["rel_err"] < r["tol"], r
