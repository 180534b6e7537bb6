#!/usr/bin/env python
"""MoE-layer tokens/s on B200 (llm.c's moe_forward hot path).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5]
  python bench.py --impl reference ...   # the reference's CPU moe_forward

A step is one forward of the MoE layer over the config's T tokens.  With N
GPUs (torchrun) the layer runs expert-parallel: tokens are split across
ranks; the experts are sharded (E/N base experts per rank plus spare slots
that a load-aware rebalance fills with replicas of hot experts, copied over
NVLink, before the timed region); token rows reach a rank holding their
expert and results return by direct NVLink peer stores, and NCCL carries
the counts and two barriers; `value` is the whole job's tokens/s (T fixed:
strong scaling) and the timing is the max over ranks.  Inputs are seeded
synthetic tensors with the config's shapes and distributions (no dataset is
involved).

The default line (c5) also carries sub-records measured in the same run on
one GPU: the FP32-accuracy path on c5 (`fp32_path`), the decode-sized
configuration c4 on AUTO (3xTF32, FP32 accuracy) and on TF32 (`decode`), and
the c2 single-token decode step (`decode_c2`).

Printed: one JSON line on rank 0 (see the keys in `main`).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "llm.c_b200"))

DECODE_PREFILL = 512        # c2: KV cache prefilled with 512 random tokens

CONFIGS = {
    # name: T, d, E, k, F, seed, bias (c2 is the 6-layer decode step, run_decode)
    "c2": dict(T=1, d=384, E=8, k=2, F=1536, seed=0, bias=None),
    "c1": dict(T=2048, d=256, E=8, k=2, F=1024, seed=0, bias=None),
    "c3": dict(T=16384, d=1024, E=16, k=2, F=4096, seed=1, bias="normal"),
    "c4": dict(T=256, d=2048, E=32, k=4, F=5632, seed=0, bias=None),
    "c5": dict(T=65536, d=4096, E=64, k=2, F=14336, seed=0, bias="zipf"),
}
W_STD = 0.02
ZIPF_S = 1.1
EP_SPARE_SLOTS = 4          # spare expert slots per rank for hot-expert replicas


def flops_per_step(c):
    T, d, E, k, F = c["T"], c["d"], c["E"], c["k"], c["F"]
    return 2.0 * T * d * E + 6.0 * T * k * d * F


def min_bytes_per_step(c, experts_touched):
    T, d, E, k, F = c["T"], c["d"], c["E"], c["k"], c["F"]
    return 4.0 * (d * E + experts_touched * 3 * d * F + 2 * T * d) + 4.0 * T * E + 4.0 * T * k


def zipf_bias(E):
    return (-ZIPF_S * np.log(np.arange(1, E + 1, dtype=np.float64))).astype(np.float32)


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return {"hbm_gbs": j["hbm_gbs"], "bf16": j["bf16_tflops"],
                "bf16_sustained": j.get("bf16_tflops_sustained", j["bf16_tflops"]),
                "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "src": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled during the timed region.

    nvidia-smi takes a few hundred milliseconds to print its first sample, so
    entering the context waits (up to 3 s) until the first sample has arrived:
    the samples then cover the timed region even when it is short (a multi-GPU
    step of ~10 ms), at 50 ms intervals; a region shorter than one interval
    keeps the sample taken right after it."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def _read(self):
        for line in self.proc.stdout:
            if line.strip():
                self.lines.append(line)
                self.first.set()

    def __enter__(self):
        import threading
        self.first = threading.Event()
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            self.first.wait(timeout=3.0)
            self.lines = []              # the first sample precedes the timed region
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            # a region shorter than the sampling interval still gets the
            # sample that follows it (up to 0.2 s later)
            t_end = time.time() + 0.2
            while not self.lines and time.time() < t_end:
                time.sleep(0.005)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.reader.join(timeout=5)

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------
# CPU: the reference's own moe_forward on a bounded sample of the workload
# ----------------------------------------------------------------------------
def reference_sample(c, budget_s, threads):
    """Time llm.c's moe_forward (oracle/_ref, the unmodified reference
    sources) on S tokens of the config, S sized to ~budget_s seconds.

    Every token costs the same k expert FFNs, so tokens/s of a sample is
    the workload's.  For large expert sets only the weights of 8 experts
    are materialised on the host and the sample is drawn from tokens whose
    top-k (by the reference's bias-free router, with a clear logit margin)
    stays inside them; the other experts' weights are never read.
    Returns (tokens_per_s, S, kind, description)."""
    sys.path.insert(0, str(REPO / "tests"))
    import oracle_lib as O

    T, d, E, k, F, seed = c["T"], c["d"], c["E"], c["k"], c["F"], c["seed"]
    kind = "reference" if O.ref_available() else "port"
    R = min(T, 8192)
    x = O.synth(seed, O.stream_x(), R * d, 1.0).reshape(R, d)
    wr = O.synth(seed, O.stream_router(), d * E, W_STD).reshape(d, E)
    logits = np.empty((R, E), np.float32)
    ids = np.empty((R, k), np.int32)
    O.oracle().oracle_router(O._f(x), R, d, O._f(wr), None, E, k, O._f(logits), None,
                             O._i(ids), None)
    weight_bytes = 3 * d * F * 4
    if E * weight_bytes <= 8e9:
        U = list(range(E))
        cand = np.arange(R)
    else:
        U = list(np.argsort(-np.bincount(ids.ravel(), minlength=E), kind="stable")[:8])
        srt = -np.sort(-logits, axis=1)
        margin = srt[:, k - 1] - srt[:, k]
        ok = np.all(np.isin(ids, U), axis=1) & (margin > 1e-3)
        cand = np.nonzero(ok)[0]
    dummy = np.zeros(1, np.float32)
    g, u, dn = [dummy] * E, [dummy] * E, [dummy] * E
    for e in U:
        g[e] = O.synth(seed, O.stream_expert(e, 0), d * F, W_STD).reshape(d, F)
        u[e] = O.synth(seed, O.stream_expert(e, 1), d * F, W_STD).reshape(d, F)
        dn[e] = O.synth(seed, O.stream_expert(e, 2), F * d, W_STD).reshape(F, d)
    gp = O._ptr_array(g)
    up = O._ptr_array(u)
    dp = O._ptr_array(dn)

    keep = (g, u, dn)          # gp/up/dp hold raw pointers into these arrays

    def run(rows):
        assert keep                # run() outlives this function: keep the weights alive
        xs = np.ascontiguousarray(x[rows])
        n = len(rows)
        out = np.empty((n, d), np.float32)
        probs = np.empty((n, E), np.float32)
        idr = np.empty((n, k), np.int32)
        t0 = time.perf_counter()
        if kind == "reference":
            O.ref().ref_moe_forward(O._f(xs), n, d, O._f(wr), E, k, gp, up, dp, F, O._f(out),
                                    O._f(probs), O._i(idr))
        else:
            O.oracle().oracle_moe_forward(O._f(xs), n, d, O._f(wr), None, E, k, gp, up, dp, F,
                                          None, n, None, O._f(out), O._f(probs), O._i(idr),
                                          threads)
        return time.perf_counter() - t0

    if kind == "reference":
        O.ref().ref_set_threads(threads)
    probe = cand[: max(1, min(len(cand), 4))]
    t_probe = run(probe) / len(probe)
    S = int(max(1, min(len(cand), budget_s / max(t_probe, 1e-9))))
    rows = cand[:S]
    dt = run(rows)
    desc = (f"{S} of the config's tokens (first {R} rows, experts {len(U)} of {E} resident"
            f"{'' if len(U) == E else ', tokens routed inside them'}), {threads} threads, "
            f"router without bias (the reference has none; per-token cost is unchanged)")
    return S / dt, S, kind, desc, run, rows


def run_reference_arm(args, c):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = len(os.sched_getaffinity(0))
    tps, S, kind, desc, run, rows = reference_sample(c, budget_s=args.ref_budget, threads=threads)
    for _ in range(args.warmup):
        run(rows)
    times = [run(rows) for _ in range(args.steps)]
    ms = 1000.0 * statistics.mean(times)
    value = S / (ms / 1000.0)
    line = {
        "metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s",
        "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.config, **{kk: c[kk] for kk in ("T", "d", "E", "k", "F")},
                   "sample_tokens": S},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind,
                         "sample": desc},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# c2: the single-token decode step of a 6-layer llm.c model with MoE FFNs
# ----------------------------------------------------------------------------
def reference_decode_ms(dec, steps, threads, prefill=()):
    """The reference's own pieces for one decode step on the same model:
    llm.c's inference_step (which leaves the MoE FFN out, src/inference.c:
    342-343) plus, per MoE layer, llm.c's moe_forward on one token.
    prefill: tokens run through the reference's inference_step first, untimed
    (they fill its KV cache)."""
    sys.path.insert(0, str(REPO / "tests"))
    import oracle_lib as O
    import ctypes as C
    R = O.ref()
    R.ref_set_threads(threads)
    R.ref_inference_step.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    m_ptr, s_ptr = C.addressof(dec.model), C.addressof(dec.state)
    c = dec.c
    for t in prefill:
        R.ref_inference_step(m_ptr, s_ptr, int(t))
    t0 = time.perf_counter()
    for i in range(steps):
        R.ref_inference_step(m_ptr, s_ptr, i % c.vocab)
    step_ms = 1000.0 * (time.perf_counter() - t0) / steps
    x = np.random.default_rng(3).standard_normal((1, c.d)).astype(np.float32)
    moe_ms = 0.0
    for layer, mw in dec.moe_weight_structs():
        E = mw.n_experts
        ex = [mw.experts[e] for e in range(E)]
        g = (O._fp * E)(*[e.W_gate.data for e in ex])
        u = (O._fp * E)(*[e.W_up.data for e in ex])
        dn = (O._fp * E)(*[e.W_down.data for e in ex])
        out = np.empty((1, c.d), np.float32)
        probs = np.empty((1, E), np.float32)
        ids = np.empty((1, mw.top_k), np.int32)
        reps = 20
        t0 = time.perf_counter()
        for _ in range(reps):
            R.ref_moe_forward(O._f(x), 1, c.d, mw.W_router.data, E, mw.top_k, g, u, dn, c.ffn,
                              O._f(out), O._f(probs), O._i(ids))
        moe_ms += 1000.0 * (time.perf_counter() - t0) / reps
    return step_ms, moe_ms


def stage_timeline(M, dec, cfg, prefill, toks):
    """The device decoder's stage timeline (a decoder made with
    MOE_B200_DECODER_STAMPS=1, outside the timed loops): per stage kind, the
    median over layers and steps of its hand-off (its first CTA's return from
    the wait, after the previous stage's last CTA exit), its work (last exit
    after the last wait) and its span (last exit after the previous stage's
    last exit), in microseconds; plus the step's device time."""
    os.environ["MOE_B200_DECODER_STAMPS"] = "1"
    try:
        tdec = M.Decoder(C.addressof(dec.model), cfg.max_seq)
    finally:
        del os.environ["MOE_B200_DECODER_STAMPS"]
    for t in prefill:
        tdec.step(int(t))
    kinds = ["qkv", "attn", "oproj", "upgate", "down"]
    per = {k: {"handoff": [], "work": [], "span": []} for k in kinds + ["lmhead"]}
    total = []
    for t in toks:
        tdec.step(int(t))
        st = tdec.stage_times(cfg.n_layers)
        prev_exit = 0.0
        for i in range(st.shape[0]):
            k = "lmhead" if i == st.shape[0] - 1 else kinds[i % 5]
            entry, w0, w1, ex = st[i]
            if i > 0:
                per[k]["handoff"].append(w0 - prev_exit)
                per[k]["span"].append(ex - prev_exit)
            per[k]["work"].append(ex - w1)
            prev_exit = ex
        total.append(st[-1, 3])
    tdec.free()
    med = lambda v: float(np.median(v)) if v else None
    return {"device_us_per_step": med(total), "steps": len(toks),
            "stages_us": {k: {m: med(v) for m, v in d.items()} for k, d in per.items()},
            "what": "median over layers and steps: handoff = first return from the wait after "
                    "the previous stage's last CTA exit; work = last exit after the last wait; "
                    "span = last exit after the previous stage's last exit (globaltimer stamps)"}


def run_decode(args):
    import torch  # noqa: F401  (CUDA context before the library, as in the other arms)
    import moe_b200 as M
    import llmc_model as LM
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # positions the host decoder state takes: the prefill, warm-up and timed
    # steps, the 5 steps of the MoE stage split, then the 5 steps of the
    # reference's own inference_step (the CPU baseline), which writes its KV
    # cache without a bounds check; plus spare
    cfg = LM.DecodeConfig(max_seq=DECODE_PREFILL + args.warmup + args.steps + 5 + 5 + 8)
    dec = LM.LlmcDecoder(cfg, seed=0)
    rng = np.random.default_rng(1)
    if args.impl == "reference":
        # the reference alone, on the host: its inference_step fills the KV
        # cache (untimed), then the timed steps
        threads = len(os.sched_getaffinity(0))
        step_ms, moe_ms = reference_decode_ms(dec, max(args.steps, 3), threads,
                                              prefill=rng.integers(0, cfg.vocab, DECODE_PREFILL))
        value = 1000.0 / (step_ms + moe_ms)
        line = {"metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s",
                "impl": "reference", "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": step_ms + moe_ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": "c2", "layers": cfg.n_layers, "d_model": cfg.d,
                           "n_experts": cfg.n_experts, "top_k": cfg.top_k, "d_ff": cfg.ffn,
                           "kv_cached_tokens": DECODE_PREFILL},
                "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads,
                                 "kind": "reference",
                                 "sample": f"inference_step {step_ms:.3f} ms (MoE left out by "
                                           f"the reference) + 6 x moe_forward(T=1) {moe_ms:.3f} ms"},
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    M.init(0)
    prefill = rng.integers(0, cfg.vocab, DECODE_PREFILL)
    toks = rng.integers(0, cfg.vocab, args.warmup + args.steps)

    # ---- device-resident decode (moe_b200_decoder_*): the whole step on the
    # B200 as one CUDA graph; per step the token goes up (4 B) and, in the
    # e2e loop, the vocab logits come back
    ddec = M.Decoder(C.addressof(dec.model), cfg.max_seq)
    for t in prefill:
        ddec.step(int(t))
    logits = np.empty(cfg.vocab, np.float32)
    for t in toks[:args.warmup]:
        ddec.step(int(t), logits)
    base = ddec.pos
    with ClockSampler(0) as clk:
        t0 = time.perf_counter()
        for t in toks[args.warmup:]:
            ddec.step(int(t))                      # logits stay on the device
        ms = 1000.0 * (time.perf_counter() - t0) / args.steps
    ddec.set_pos(base)
    t0 = time.perf_counter()
    for t in toks[args.warmup:]:
        ddec.step(int(t), logits)                  # + D2H of the logits
    e2e_ms = 1000.0 * (time.perf_counter() - t0) / args.steps
    launches = ddec.launches
    ddec.free()
    timeline = stage_timeline(M, dec, cfg, prefill, toks[args.warmup:]) if args.stage_times else None
    # the same step as one persistent cooperative kernel (one launch per step)
    sdec = M.Decoder(C.addressof(dec.model), cfg.max_seq, M.Decoder.PERSISTENT)
    for t in prefill:
        sdec.step(int(t))
    for t in toks[:args.warmup]:
        sdec.step(int(t))
    t0 = time.perf_counter()
    for t in toks[args.warmup:]:
        sdec.step(int(t))
    sk_ms = 1000.0 * (time.perf_counter() - t0) / args.steps
    stage_launches = sdec.launches
    sdec.free()

    # ---- the drop-in host inference_step (llm.c's arithmetic on the host,
    # MoE blocks on the B200), for comparison
    for t in prefill:
        dec.step(int(t))
    for t in toks[:args.warmup]:
        dec.step(int(t))
    t0 = time.perf_counter()
    for t in toks[args.warmup:]:
        dec.step(int(t))
    host_ms = 1000.0 * (time.perf_counter() - t0) / args.steps
    # the MoE stage split of the same steps, in a separate pass
    M.profile_enable(True)
    M.profile_read()
    for t in toks[args.warmup:args.warmup + min(args.steps, 5)]:
        dec.step(int(t))
    M.profile_enable(False)
    stage_ms, n_fw = M.profile_read()
    stage_avg = {s: v / max(n_fw, 1) for s, v in stage_ms.items()}

    # algorithmic bytes of one step: every weight it reads once (attention,
    # the k experts of each layer, LM head, the embedding row) and the KV
    # cache of the positions attended (the mean position of the timed steps)
    nq, kv = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    P = DECODE_PREFILL + args.warmup + args.steps / 2.0
    step_bytes = 4.0 * (cfg.n_layers * (cfg.d * (nq + 2 * kv) + nq * cfg.d + 2 * cfg.d
                                        + cfg.top_k * 3 * cfg.d * cfg.ffn
                                        + cfg.d * cfg.n_experts + 2 * P * kv)
                        + cfg.d * cfg.vocab + 2 * cfg.d)
    peaks = measured_peaks()
    step_gbs = step_bytes / (ms / 1000.0) / 1e9
    line = {
        "metric": "moe_layer_tokens_per_s", "value": 1000.0 / ms, "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "c2", "layers": cfg.n_layers, "d_model": cfg.d,
                   "n_heads": cfg.n_heads, "n_kv_heads": cfg.n_kv_heads, "d_ff": cfg.ffn,
                   "n_experts": cfg.n_experts, "top_k": cfg.top_k,
                   "kv_cached_tokens": DECODE_PREFILL, "batch": 1,
                   "parallelism": "single GPU; the whole decode step on the device: 31 stage "
                                  "kernels replayed as one CUDA graph (moe_b200_decoder, the "
                                  "default variant)"},
        "e2e": {"value": 1000.0 / e2e_ms, "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": 4, "d2h_bytes_per_step": cfg.vocab * 4,
                "timing": "host wall clock around synchronous decoder steps (token up, logits "
                          "down)"},
        "roofline": {"bound": "hbm",
                     "kernel": "the decode step's stage kernels (31 launches in one CUDA graph)",
                     "achieved": step_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": step_gbs / peaks["hbm_gbs"], "traffic": None,
                     "peak_src": peaks["src"] + " HBM copy bandwidth",
                     "note": f"{step_bytes / 1e6:.1f} MB read per step; latency-bound: "
                             f"31 dependent stages"},
        "persistent_kernel": {"tokens_per_s": 1000.0 / sk_ms, "ms_per_step": sk_ms,
                          "launches_per_step": stage_launches,
                          "what": "the same device step as one persistent cooperative kernel "
                                  "(stages behind a bounded grid barrier)"},
        "host_dropin": {"tokens_per_s": 1000.0 / host_ms, "ms_per_step": host_ms,
                        "what": "llm.c's inference_step restated on the host with the MoE "
                                "blocks on the B200 (the drop-in symbol)",
                        "moe_device_ms_per_step": cfg.n_layers * sum(stage_avg.values()),
                        "stages_ms": stage_avg},
        "gpu_launches": launches * args.steps,
        "clocks": clk.summary(),
    }
    if timeline is not None:
        line["stage_timeline"] = timeline
    if not args.no_cpu_baseline and (REPO / "oracle" / "_ref" / "libllmref.so").exists():
        threads = len(os.sched_getaffinity(0))
        step_ms, moe_ms = reference_decode_ms(dec, 5, threads)
        line["cpu_baseline"] = {"value": 1000.0 / (step_ms + moe_ms), "unit": "tokens/s",
                                "cores": threads, "kind": "reference",
                                "sample": f"5 steps: inference_step {step_ms:.3f} ms (MoE left "
                                          f"out by the reference) + 6 x moe_forward(T=1) "
                                          f"{moe_ms:.3f} ms"}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# GPU
# ----------------------------------------------------------------------------
def run_backward(args, c):
    """The MoE backward (the forward recomputed inside) on one GPU: tokens/s
    and FLOP rate against the peak of the arithmetic the path runs on (TF32
    tensor cores: the measured bf16 rate / 2; FP32 FFMA: the nominal FFMA
    peak)."""
    import torch
    import moe_b200 as M
    M.init(0)
    T, d, E, k, F, seed = c["T"], c["d"], c["E"], c["k"], c["F"], c["seed"]
    w = M.MoEWeights.synth(seed, W_STD, d, F, E, k)
    g = M.MoEGrads(w)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    x = torch.empty((T, d), device="cuda")
    M.synth_fill(x.data_ptr(), T * d, seed, M.STREAM_X, 1.0, cuda_stream=stream.cuda_stream)
    dy = torch.empty((T, d), device="cuda")
    M.synth_fill(dy.data_ptr(), T * d, seed + 1, M.STREAM_X, 0.1, cuda_stream=stream.cuda_stream)
    dx = torch.empty_like(x)
    aux = torch.empty(1, device="cuda")
    bias = None
    if c["bias"] == "zipf":
        bias = torch.from_numpy(zipf_bias(E)).cuda()
    elif c["bias"] == "normal":
        bias = torch.empty(E, device="cuda")
        M.synth_fill(bias.data_ptr(), E, seed, M.STREAM_BIAS, 1.0, cuda_stream=stream.cuda_stream)
    bptr = bias.data_ptr() if bias is not None else None

    path = {"auto": M.PATH_AUTO, "tf32": M.PATH_TF32, "fp32": M.PATH_FP32,
            "tf32x3": M.PATH_TF32X3}[args.path]

    def step():
        M.moe_backward_device(w, x.data_ptr(), T, dy.data_ptr(), dx.data_ptr(), g, bias_ptr=bptr,
                              aux_coef=0.01, aux_ptr=aux.data_ptr(), stream=stream.cuda_stream,
                              path=path)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    launches = M.last_launches()
    path_used = M.last_path()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    rows = T * k
    flops = 18.0 * rows * d * F + 6.0 * T * d * E      # forward recompute + backward
    props = torch.cuda.get_device_properties(0)
    clocks = clk.summary()
    achieved = flops / (ms / 1000.0) / 1e12
    if path_used == M.PATH_TF32:
        peaks = measured_peaks()
        peak = peaks["bf16_sustained"] / 2.0
        bound, peak_src = "tensor (TF32)", peaks["src"] + " bf16 sustained / 2 (TF32 rate)"
    else:
        mhz = clocks.get("sm_max_mhz") or 1965.0
        peak = props.multi_processor_count * 128 * 2 * mhz * 1e6 / 1e12
        bound, peak_src = "fp32 FFMA", "nominal: SMs x 128 FP32 lanes x 2 x max SM clock"
    line = {
        "metric": "moe_backward_tokens_per_s", "value": T / (ms / 1000.0), "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": args.config + "-backward", "T": T, "d_model": d, "n_experts": E,
                   "top_k": k, "d_ff": F, "router_bias": c["bias"], "aux_coef": 0.01,
                   "path": args.path,
                   "path_run": "tf32 (tcgen05)" if path_used == M.PATH_TF32 else "fp32 (FFMA)"},
        "roofline": {"bound": bound, "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak, "peak_src": peak_src,
                     "flops_per_step": flops},
        "gpu_launches": launches * args.steps,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    g.free()
    w.free()


def block_ffn_measure(args, M, w, x, bptr, host_bias_ptr, path, stream, stage_ms_moe, n_moe,
                      moe_ms, T, d, E, k):
    """Device and end-to-end timing of moe_b200_block_ffn (RMSNorm + MoE +
    residual) on the bench workload, against the MoE-only step just timed."""
    import torch
    peaks = measured_peaks()
    rms = torch.ones(d, device="cuda") + 0.1 * torch.randn(d, device="cuda",
                                                           generator=torch.Generator("cuda").manual_seed(1))
    xb = x.clone()
    xn = torch.empty_like(x)
    probs = torch.empty((T, E), device="cuda")
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")

    def step():
        M.block_ffn_device(w, rms.data_ptr(), 1e-5, xb.data_ptr(), T, xn.data_ptr(),
                           probs.data_ptr(), ids.data_ptr(), bias_ptr=bptr, path=path,
                           stream=stream.cuda_stream, cta_pair=args.cta_pair)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    launches = M.last_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    M.profile_enable(True)                      # stage split: a separate pass
    M.profile_read()
    for _ in range(min(args.steps, 5)):
        step()
    torch.cuda.synchronize()
    M.profile_enable(False)
    st, n = M.profile_read()
    # the RMSNorm runs inside the router stage: its time is the router stage's growth
    norm_ms = st["router"] / max(n, 1) - stage_ms_moe["router"] / max(n_moe, 1)
    norm_bytes = 2.0 * 4 * T * d                 # read x, write x_norm
    # end to end through the host C-ABI: x up, x (and probs, ids) back
    hx = torch.empty((T, d), dtype=torch.float32, pin_memory=True)
    hx.copy_(x.cpu())
    hrms = rms.cpu().contiguous()
    hprobs = torch.empty((T, E), dtype=torch.float32, pin_memory=True)
    hids = torch.empty((T, k), dtype=torch.int32, pin_memory=True)
    hb = host_bias_ptr

    def e2e():
        M.block_ffn_host_ptr(w, hrms.data_ptr(), 1e-5, hx.data_ptr(), T, None, hprobs.data_ptr(),
                             hids.data_ptr(), hb, path=path, cta_pair=args.cta_pair)

    for _ in range(2):
        e2e()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e()
    e2e_ms = 1000.0 * (time.perf_counter() - t0) / args.steps
    return {
        "ms_per_step": ms, "tokens_per_s": T / (ms / 1000.0),
        "overhead_vs_moe_ms": ms - moe_ms,
        "rmsnorm_ms": norm_ms,
        "rmsnorm_gbs": norm_bytes / (norm_ms / 1000.0) / 1e9 if norm_ms > 0 else None,
        "rmsnorm_frac_of_hbm": (norm_bytes / (norm_ms / 1000.0) / 1e9 / peaks["hbm_gbs"]
                                if norm_ms > 0 else None),
        "launches_per_step": launches,
        "e2e": {"value": T / (e2e_ms / 1000.0), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": 4 * T * d + 4 * d + (4 * E if hb is not None else 0),
                "d2h_bytes_per_step": 4 * T * d + 4 * T * E + 4 * T * k},
    }


def rank_experts(split, placement, rank):
    """Experts whose rows `rank` computes under a split (M.ep_split)."""
    n = 0
    for e in range(placement.shape[1]):
        if placement[rank, e] < 0:
            continue
        holders = list(split["holders"][e, :split["n_holders"][e]])
        i = holders.index(rank)
        n += int(split["row_begin"][e, i + 1] > split["row_begin"][e, i])
    return n


def _timed(step, stream, steps, warmup):
    """Mean device ms of `step` over `steps` launches after `warmup`, CUDA
    events on `stream`, synchronised on both sides."""
    import torch
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    return ev0.elapsed_time(ev1) / steps


def fp32_path_record(M, w, x, bptr, stream, c):
    """c5 at FP32 accuracy (tolerance 1e-5), beside the TF32 headline, on
    both expert paths that give it: the FP32 FFMA grouped GEMMs (tokens/s
    and the FFMA rate of the layer) and the 3xTF32 tensor-core kernel
    (`tf32x3`: tokens/s and its FLOP rate against the TF32 peak, of which
    it issues three MMAs per product)."""
    import torch
    T, d, E, k, F = c["T"], c["d"], c["E"], c["k"], c["F"]
    out = torch.empty((T, d), device="cuda")
    props = torch.cuda.get_device_properties(0)
    peaks = measured_peaks()
    recs = {}
    for path in (M.PATH_FP32, M.PATH_TF32X3):
        def step():
            M.moe_forward_device(w, x.data_ptr(), T, out.data_ptr(), bias_ptr=bptr, path=path,
                                 stream=stream.cuda_stream)

        with ClockSampler(0) as clk:
            ms = _timed(step, stream, steps=2, warmup=1)
        clocks = clk.summary()
        tflops = flops_per_step(c) / (ms / 1000.0) / 1e12
        rec = {"tokens_per_s": T / (ms / 1000.0), "ms_per_step": ms, "tolerance": 1e-5,
               "achieved_tflops": tflops, "clocks": clocks}
        if path == M.PATH_FP32:
            mhz = clocks.get("sm_mhz") or 1965.0
            ffma_peak = props.multi_processor_count * 128 * 2 * mhz * 1e6 / 1e12
            rec.update({"dtype": "f32", "path_run": "fp32 (FFMA grouped GEMMs)",
                        "ffma_peak_tflops": ffma_peak, "frac_of_ffma_peak": tflops / ffma_peak,
                        "peak_src": "nominal: SMs x 128 FP32 lanes x 2 x median SM clock under "
                                    "load"})
            recs.update(rec)
        else:
            tf32_peak = peaks["bf16_sustained"] / 2.0
            rec.update({"dtype": "tf32x3", "path_run": "tf32x3 (3xTF32 weight-streaming kernel)",
                        "tf32_peak_tflops": tf32_peak,
                        "frac_of_tf32_peak_x3": 3.0 * tflops / tf32_peak,
                        "peak_src": f"{peaks['src']} bf16 sustained / 2 (TF32 rate); three "
                                    "MMAs per product"})
            recs["tf32x3"] = rec
    return recs


def decode_c4_record(M, stream):
    """Configuration 4 (256 tokens, d 2048, E 32, top-4, d_ff 5632): a
    decode-sized layer, weight-streaming and HBM-bound.  AUTO runs the 3xTF32
    kernel (FP32 accuracy, 1e-5); TF32 its one-pass mode (2e-3).  Roofline:
    the touched experts' gate and up weight bytes over the up/gate kernel's
    device time, against the measured HBM copy bandwidth."""
    import torch
    c = CONFIGS["c4"]
    T, d, E, k, F, seed = c["T"], c["d"], c["E"], c["k"], c["F"], c["seed"]
    w = M.MoEWeights.synth(seed, W_STD, d, F, E, k)
    x = torch.empty((T, d), device="cuda")
    M.synth_fill(x.data_ptr(), T * d, seed, M.STREAM_X, 1.0, cuda_stream=stream.cuda_stream)
    out = torch.empty((T, d), device="cuda")
    peaks = measured_peaks()
    rec = {"workload": "c4", "T": T, "d_model": d, "n_experts": E, "top_k": k, "d_ff": F}
    for name, path, tol in (("auto", M.PATH_AUTO, 1e-5), ("tf32", M.PATH_TF32, 2e-3)):
        def step():
            M.moe_forward_device(w, x.data_ptr(), T, out.data_ptr(), path=path,
                                 stream=stream.cuda_stream)
        with ClockSampler(0) as clk:
            ms = _timed(step, stream, steps=20, warmup=3)
        path_run = M.last_path()
        counts = M.last_counts(w)
        M.profile_enable(True)
        M.profile_read()
        for _ in range(5):
            step()
        torch.cuda.synchronize()
        M.profile_enable(False)
        st, n = M.profile_read()
        up_ms = st["upgate"] / max(n, 1)
        touched = int(np.count_nonzero(counts))
        gbs = 2.0 * d * F * 4 * touched / (up_ms / 1000.0) / 1e9
        rec[name] = {"tokens_per_s": T / (ms / 1000.0), "ms_per_step": ms,
                     "path_run": {M.PATH_TF32: "tf32 (one-pass weight streaming)",
                                  M.PATH_TF32X3: "tf32x3 (FP32 accuracy)"}.get(path_run, "?"),
                     "tolerance": tol,
                     "roofline": {"bound": "hbm", "kernel": "dec_gemm<up/gate>",
                                  "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                  "frac": gbs / peaks["hbm_gbs"],
                                  "peak_src": peaks["src"] + " HBM copy bandwidth"},
                     "stages_ms": {s_: v / max(n, 1) for s_, v in st.items()},
                     "clocks": clk.summary()}
    w.free()
    return rec


def decode_c2_record(M):
    """Configuration 2: one token through the 6-layer MoE model with a
    512-token KV cache, the whole step on the device (31 stage kernels in
    one CUDA graph)."""
    import llmc_model as LM
    steps = 40
    cfg = LM.DecodeConfig(max_seq=DECODE_PREFILL + steps + 8)
    dec = LM.LlmcDecoder(cfg, seed=0)
    rng = np.random.default_rng(1)
    ddec = M.Decoder(C.addressof(dec.model), cfg.max_seq)
    for t in rng.integers(0, cfg.vocab, DECODE_PREFILL):
        ddec.step(int(t))
    toks = rng.integers(0, cfg.vocab, steps)
    with ClockSampler(0) as clk:
        t0 = time.perf_counter()
        for t in toks:
            ddec.step(int(t))
        ms = 1000.0 * (time.perf_counter() - t0) / steps
    launches = ddec.launches
    ddec.free()
    nq, kv = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    P = DECODE_PREFILL + steps / 2.0
    step_bytes = 4.0 * (cfg.n_layers * (cfg.d * (nq + 2 * kv) + nq * cfg.d + 2 * cfg.d
                                        + cfg.top_k * 3 * cfg.d * cfg.ffn
                                        + cfg.d * cfg.n_experts + 2 * P * kv)
                        + cfg.d * cfg.vocab + 2 * cfg.d)
    peaks = measured_peaks()
    gbs = step_bytes / (ms / 1000.0) / 1e9
    return {"workload": "c2", "tokens_per_s": 1000.0 / ms, "ms_per_step": ms,
            "kv_cached_tokens": DECODE_PREFILL, "launches_per_step": launches,
            "timing": "host wall clock around synchronous decoder steps (token up)",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"],
                         "bytes_per_step": step_bytes},
            "clocks": clk.summary()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c5", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--path", default="auto", choices=["auto", "tf32", "fp32", "tf32x3"])
    ap.add_argument("--ref-budget", type=float, default=6.0,
                    help="seconds of CPU work per reference sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true",
                    help="skip the fp32_path / decode / decode_c2 sub-records of the c5 line")
    ap.add_argument("--experts", type=int, default=None,
                    help="override n_experts (small profiling cases of the expert GEMMs)")
    ap.add_argument("--backward", action="store_true",
                    help="time the MoE backward (moe_b200_backward_device) instead of the forward")
    ap.add_argument("--cta-pair", action="store_true",
                    help="TF32 path on the CTA-pair (cta_group::2) GEMM kernels")
    ap.add_argument("--stage-times", action="store_true",
                    help="c2: add the device decoder's stage timeline (a separate decoder with "
                         "globaltimer stamps, outside the timed loops)")
    ap.add_argument("--tokens", type=int, default=None,
                    help="override T (small profiling cases; the JSON config records it)")
    ap.add_argument("--d-ff", type=int, default=None,
                    help="override d_ff (profiling cases for the router, dispatch and combine "
                         "kernels, which do not depend on it)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    c = dict(CONFIGS[args.config])
    if args.tokens:
        c["T"] = args.tokens
    if args.d_ff:
        c["F"] = args.d_ff
    if args.experts:
        c["E"] = args.experts

    if args.config == "c2":
        run_decode(args)
        return
    if args.backward:
        run_backward(args, c)
        return
    if args.impl == "reference":
        run_reference_arm(args, c)
        return

    import torch
    import moe_b200 as M

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        # the group's NCCL traffic is a few counts and barriers: keep it on
        # plain NVLink transport (no NVLS multicast objects)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    M.init(local)
    path = {"auto": M.PATH_AUTO, "tf32": M.PATH_TF32, "fp32": M.PATH_FP32,
            "tf32x3": M.PATH_TF32X3}[args.path]
    T, d, E, k, F, seed = c["T"], c["d"], c["E"], c["k"], c["F"], c["seed"]
    if T % world:
        raise SystemExit(f"T={T} is not divisible by {world} ranks")
    Tl = T // world                      # this rank's tokens (strong scaling: T fixed)
    n_slots = E
    if world > 1:
        # this rank's shard: its E/world base experts plus spare slots for
        # the replicas of hot experts that the rebalance places
        mine = M.ep_shard_experts(E, world, rank)
        n_slots = min(E, len(mine) + EP_SPARE_SLOTS)
        w = M.MoEWeights.synth_shard(seed, W_STD, d, F, E, k, mine, n_slots)
    else:
        w = M.MoEWeights.synth(seed, W_STD, d, F, E, k)
    # a dedicated stream: the legacy default stream's handle is 0, which the
    # library reads as "use the library stream"
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    # rows [rank*Tl, (rank+1)*Tl) of the same global x the 1-GPU run sees
    x = torch.empty((Tl, d), dtype=torch.float32, device="cuda")
    M.synth_fill(x.data_ptr(), Tl * d, seed, M.STREAM_X, 1.0, first=rank * Tl * d,
                 cuda_stream=stream.cuda_stream)
    bias = None
    if c["bias"] == "zipf":
        bias = torch.from_numpy(zipf_bias(E)).cuda()
    elif c["bias"] == "normal":
        bias = torch.empty(E, device="cuda")
        M.synth_fill(bias.data_ptr(), E, seed, M.STREAM_BIAS, 1.0, cuda_stream=stream.cuda_stream)
    out = torch.empty((Tl, d), dtype=torch.float32, device="cuda")
    probs = torch.empty((Tl, E), dtype=torch.float32, device="cuda")
    ids = torch.empty((Tl, k), dtype=torch.int32, device="cuda")
    bptr = bias.data_ptr() if bias is not None else None

    ep = None
    if world > 1:
        obj = [M.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ep = M.EP(obj[0], rank, world, Tl, w)

    def step():
        if ep is None:
            M.moe_forward_device(w, x.data_ptr(), Tl, out.data_ptr(), probs.data_ptr(),
                                 ids.data_ptr(), bias_ptr=bptr, path=path,
                                 stream=stream.cuda_stream, cta_pair=args.cta_pair)
        else:
            ep.forward_device(x.data_ptr(), Tl, out.data_ptr(), probs.data_ptr(), ids.data_ptr(),
                              bias_ptr=bptr, path=path, stream=stream.cuda_stream)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    placement = None
    if ep is not None:
        # load-aware replicas from the first forward's counts (set-up, like
        # the weight upload; not timed)
        step()
        barrier()
        ep.rebalance()
        barrier()
    for _ in range(args.warmup):
        step()
    barrier()
    launches_per_step = M.last_launches()
    path_used = M.last_path()
    if ep is None:
        counts = M.last_counts(w)
        slice_rows = Tl * k
        my_experts = int(np.count_nonzero(counts))
    else:
        counts_all, slice_rows = ep.counts()
        counts = counts_all.sum(axis=0)
        placement = ep.placement()
        my_experts = rank_experts(M.ep_split(counts_all, placement, n_slots), placement, rank)

    # ---- device-resident timed region (CUDA events on the launch stream,
    # barrier + synchronize on both sides, max over ranks)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)
    # the per-stage split comes from a separate pass: the stage events would
    # otherwise sit inside the timed region (every rank runs the same steps)
    M.profile_enable(True)
    M.profile_read()
    for _ in range(min(args.steps, 5)):
        step()
    barrier()
    M.profile_enable(False)
    stage_ms, n_fw = M.profile_read()
    value = T / (ms / 1000.0)

    # ---- end to end through the public host-buffer C-ABI (pinned buffers,
    # H2D of x and D2H of out/probs/ids inside every step)
    hx = torch.empty((Tl, d), dtype=torch.float32, pin_memory=True)
    hx.copy_(x.cpu())
    hout = torch.empty((Tl, d), dtype=torch.float32, pin_memory=True)
    hprobs = torch.empty((Tl, E), dtype=torch.float32, pin_memory=True)
    hids = torch.empty((Tl, k), dtype=torch.int32, pin_memory=True)
    hbias = bias.cpu().contiguous() if bias is not None else None
    hb = hbias.data_ptr() if hbias is not None else None

    def e2e_step():
        if ep is None:
            M.moe_forward_host_ptr(w, hx.data_ptr(), Tl, hout.data_ptr(), hprobs.data_ptr(),
                                   hids.data_ptr(), hb, path=path, cta_pair=args.cta_pair)
        else:
            ep.forward_host_ptr(hx.data_ptr(), Tl, hout.data_ptr(), hprobs.data_ptr(),
                                hids.data_ptr(), hb, path=path)

    for _ in range(2):
        e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(1000.0 * (time.perf_counter() - t0) / args.steps)
    barrier()
    assert torch.equal(hout, out.cpu()), "e2e output differs from the device-resident run"

    # ---- the FFN half of block_forward fused around the same MoE
    # (src/transformer.c:752-767): RMSNorm in front, residual in the combine.
    # x is updated in place step after step on a scratch copy.
    block = None
    if ep is None:
        block = block_ffn_measure(args, M, w, x, bptr, hb, path, stream, stage_ms_moe=stage_ms,
                                  n_moe=n_fw, moe_ms=ms, T=T, d=d, E=E, k=k)

    # ---- roofline of the dominant kernel (expert up/gate GEMM on this rank)
    peaks = measured_peaks()
    tf32_peak = peaks["bf16_sustained"] / 2.0
    stage_avg = {s: v / max(n_fw, 1) for s, v in stage_ms.items()}
    stages_by_rank = None
    if dist is not None:
        stages_by_rank = [None] * world
        dist.all_gather_object(stages_by_rank, {"stages": stage_avg, "slice_rows": slice_rows,
                                                "sm_mhz": clk.summary().get("sm_mhz")})
    up_ms = stage_avg["upgate"]
    touched = int(np.count_nonzero(counts))
    traffic = None
    tfile = REPO / "profiles" / "traffic.json"
    if tfile.exists() and world == 1:
        tj = json.loads(tfile.read_text())
        traffic = tj.get(args.config, {}).get("upgate_bytes_per_launch")
    # gate and up weights of the experts this rank computes rows of (each
    # read once)
    w_bytes = 2.0 * d * F * 4 * my_experts
    up_flops = 4.0 * slice_rows * d * F
    # the TF32 grouped GEMM is tensor-bound when the expert groups are large
    # and weight-streaming (HBM-bound) when they are decode-sized
    tf32_tensor_bound = (up_flops / (tf32_peak * 1e12)) >= (w_bytes / (peaks["hbm_gbs"] * 1e9))
    if path_used == M.PATH_TF32 and tf32_tensor_bound:
        # tensor-bound grouped GEMM: 2 GEMMs (gate, up) of this rank's rows
        achieved = up_flops / (up_ms / 1000.0) / 1e12
        roof = {"bound": "tensor", "kernel": "tc_grouped_gemm<256,swiglu> (expert up/gate)",
                "achieved": achieved, "peak": tf32_peak, "unit": "TFLOP/s",
                "frac": achieved / tf32_peak, "traffic": traffic,
                "peak_src": f"{peaks['src']} bf16 sustained / 2 (TF32 rate)"}
    else:
        # weight-streaming (3xTF32, FP32 FFMA, or TF32 on decode-sized
        # groups): HBM-bound on the gate and up weights
        achieved = w_bytes / (up_ms / 1000.0) / 1e9
        roof = {"bound": "hbm",
                "kernel": {M.PATH_TF32X3: "dec_gemm<up/gate> (3xTF32 weight streaming)",
                           M.PATH_TF32: ("dec_gemm<up/gate, one-pass TF32> (weight streaming)"
                                         if T * k / E < 64 else
                                         "tc_grouped_gemm<256,swiglu> (expert up/gate)"),
                           }.get(path_used, "ffma_grouped<up/gate> (FP32)"),
                "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                "peak_src": peaks["src"] + " HBM copy bandwidth"}
    t_roof = max(flops_per_step(c) / (tf32_peak * 1e12 * world),
                 min_bytes_per_step(c, touched) / (peaks["hbm_gbs"] * 1e9 * world))
    if world > 1:
        # rows crossing NVLink per rank and direction (dispatch, then return)
        a2a = 4.0 * d * (T * k / world) * (world - 1) / world
        t_roof += a2a / 770e9

    dtype = {M.PATH_TF32: "tf32", M.PATH_FP32: "f32", M.PATH_TF32X3: "tf32x3"}.get(path_used, "?")
    line = {
        "metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic",
        "config": {"workload": args.config + ("-profile" if (args.tokens or args.d_ff or
                                                             args.experts) else ""),
                   "T": T, "d_model": d, "n_experts": E, "top_k": k,
                   "d_ff": F, "router_bias": c["bias"], "path": args.path,
                   "path_run": {M.PATH_TF32: "tf32", M.PATH_FP32: "fp32",
                                M.PATH_TF32X3: "tf32x3"}.get(path_used, "?"),
                   "parallelism": f"ep{world}" + (
                       f" (experts sharded {E // world} per rank + up to "
                       f"{n_slots - E // world} hot-expert replicas, rows split by cost)"
                       if world > 1 else ""),
                   "l2": "inputs larger than L2"
                   if 4 * T * d > 126e6 else "inputs smaller than L2 (no flush)"},
        "e2e": {"value": T / (e2e_ms / 1000.0), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": 4 * T * d + (4 * E * world if bias is not None else 0),
                "d2h_bytes_per_step": 4 * T * d + 4 * T * E + 4 * T * k,
                "timing": "host wall clock around synchronous forward calls, max over ranks"},
        "roofline": {**roof, "layer_frac": t_roof / (ms / 1000.0)},
        "stages_ms": stage_avg,
        "stages_ms_by_rank": stages_by_rank,
        "expert_counts_max_over_mean": float(counts.max() / counts.mean()),
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    # time x median SM clock: compares runs at different power-capped clocks
    mhz = [r["sm_mhz"] for r in stages_by_rank if r.get("sm_mhz")] if stages_by_rank else \
        ([line["clocks"]["sm_mhz"]] if line["clocks"].get("sm_mhz") else [])
    if mhz:
        med = float(statistics.median(mhz))
        line["clock_normalized"] = {"sm_mhz_median_over_ranks": med,
                                    "ms_x_sm_ghz": ms * med / 1000.0,
                                    "what": "ms per step x median SM clock (GHz) during the timed "
                                            "region; equal work at equal efficiency gives equal "
                                            "values at any clock"}
    if block is not None:
        line["block_ffn"] = block
    if placement is not None:
        held = (placement >= 0).sum(axis=1)
        line["expert_parallel"] = {
            "slots_per_rank": n_slots, "experts_held_per_rank": held.tolist(),
            "weights_gb_per_rank_max": float(held.max() * 3 * d * F * 4 / 1e9),
            "replicas": int((placement >= 0).sum() - E),
            "recv_rows_by_rank": [r["slice_rows"] for r in stages_by_rank] if stages_by_rank else None}
    subrecords = world == 1 and rank == 0 and args.config == "c5" and not (args.tokens or args.d_ff) \
        and not args.no_sub
    if subrecords:
        line["fp32_path"] = fp32_path_record(M, w, x, bptr, stream, c)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = len(os.sched_getaffinity(0))
        tps, S, kind, desc, _, _ = reference_sample(c, budget_s=12.0, threads=threads)
        line["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": threads, "kind": kind,
                                "sample": desc}
    if ep is not None:
        ep.destroy()
        dist.barrier()
        dist.destroy_process_group()
    w.free()
    if subrecords:
        del x, out, probs, ids
        torch.cuda.empty_cache()
        line["decode"] = decode_c4_record(M, stream)
        line["decode_c2"] = decode_c2_record(M)
    if rank == 0:
        print(json.dumps(line), flush=True)

if __name__ == "__main__":
    main()
