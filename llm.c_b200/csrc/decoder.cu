// decoder.cu — llm.c's single-token KV-cache forward (src/inference.c:231-358,
// with the MoE branch its TODO at :342-343 leaves out) run entirely on the
// device, replayed as one CUDA graph per generated token.
//
// Everything the step touches stays in HBM: embeddings, per-layer norm and
// attention weights, the experts (the library's packed, resident expert
// sets), final norm, LM head, RoPE tables and the KV cache.  Per step the
// host writes the token id (4 bytes) and reads the logits back.
//
// Per layer, six FP32 kernels (a decode step is latency-bound: ~45 MB of
// weights for the configuration-2 model):
//   1 qkv     RMSNorm (:209-215) + x·[W_Q | W_K | W_V] (:174-182), RoPE at
//             the step's position on the q and k columns (:189-203), k and v
//             appended to the KV cache (:279-281)
//   2 attn    per (query head, 64-position chunk): scores q·k·(1/sqrt(hd)),
//             chunk max, exp-sums and exp-weighted V (flash decoding); GQA
//             head mapping kvh = qh / (n_heads / n_kv_heads) (:285-305)
//   3 oproj   combines the chunks of every head into the softmax-weighted
//             head outputs, then x += head_out·W_O (:307-309)
//   4 router  RMSNorm (:311) + logits x_norm·W_router + the reference's
//             softmax / top-k / renormalisation (src/transformer.c:299-337)
//   5 upgate  per selected expert and hidden unit f: gate and up dot
//             products and the reference's silu(gate)·up (:157-165)
//   6 down    per output column: y_r = h_r·W_down[e_r] for each rank r and
//             x += sum_r w_r·y_r in rank order (:355-358)
// and after the last layer one kernel for the final RMSNorm and the LM head
// (:350-356), which also advances the device-side position.  Dense blocks
// (use_moe = 0) run as a one-expert MoE: probability 1, weight p/p = 1
// exactly, so the FFN output is unchanged.
//
// Every reduction has a fixed order, so a step is deterministic.
#include "kernels.cuh"
#include "weights.cuh"
#include "../../include/llmc_moe.h"
#include "../../include/moe_b200.h"

#include <cstdlib>
#include <cstring>
#include <vector>

namespace moe {
namespace decs {

constexpr int kThreads = 256;           // 8 warps
constexpr int CH = 64;                  // attention positions per chunk
constexpr int kMaxD = 8192;             // d_model limit (normalised vector in smem)
constexpr int kUnitsPerWarp = 2;        // up/gate stage: hidden units per warp
constexpr int kUnitsPerCta = kUnitsPerWarp * kThreads / 32;

struct Dims {
    int d, d_pad, nh, nkv, hd, nq, kvd, qkv, vocab, max_seq, nchunk;
    float eps, scale;
};

// per-layer device pointers (an array of these lives in device memory)
struct LayerPtrs {
    const float *rms_attn, *rms_ffn, *w_qkv, *w_o, *router, *ug, *dn;
    int E, k, F, F_pad;
};

// every buffer a step reads or writes
struct StepArgs {
    Dims D;
    int L;
    const LayerPtrs *layers;
    const float *embed, *rms_final, *lm_head, *rope_cos, *rope_sin;
    float *kc, *vc;                    // [L][max_seq][kvd]
    float *x, *q, *part, *h, *logits, *wts;
    int *state, *ids;                  // state = {token, pos}
    unsigned *bar;                     // grid barrier counter (zeroed before each step)
    int *err;                          // barrier timeout flag
    int *err_host;                     // mapped pinned copy, written at the end of every step
    float *trace;                      // [L][2][d]: pre-FFN x_norm and FFN output per layer
    unsigned long long *stamps;        // stage timeline [5 L + 1][4] (%globaltimer ns), or null
    int pdl_early;                     // stage kernels: let the next kernel launch on entry
    int flags;                         // stage kernels hand off through done[] (see stage_wait):
                                       // 1 the next kernel may launch after a CTA's wait, 2 after its work
    int early_mask;                    // flag mode: stage kinds (bit 0 qkv .. 4 down) whose CTAs
                                       // let the next kernel launch on entry
    unsigned *done;                    // [6 L + 1] CTAs finished per stage, then per layer the
                                       // up/gate stage's ids-published count (zeroed before each step)
};

struct Smem {
    float xn[kMaxD];                   // normalised vector / head outputs
    float red[kThreads];
    float qs[128];
    float sc[CH];
    float lg[kMaxExperts];
    int sel[kMaxTopK];
    float w[kMaxTopK];
    int flag;
};

// Values written by other CTAs of the same launch are read through L2
// (ld.global.cg): the persistent kernel has no kernel boundary to drop stale
// L1 lines.  Weights, which no step writes, use the read-only path.
__device__ __forceinline__ float ldcg(const float *p) { return __ldcg(p); }

// Programmatic dependent launch.  The stage kernels are launched so that
// the next kernel's CTAs may start before the current one has finished (as
// its CTAs exit, or, with pdl_early, as soon as they all started: each
// calls pdl_trigger() on entry); a kernel loads what does not depend on the
// previous stage (weight rows, RoPE factors, cached keys of earlier
// positions) and calls stage_wait() before it reads anything the previous
// stage wrote or writes anything.  In the griddepcontrol modes stage_wait()
// returns once the previous kernel has completed and its writes are visible
// (in a kernel launched without the dependency, the step's first kernel,
// it is a no-op).
//
// Flag mode (A.flags): griddepcontrol.wait returns only ~1-3 us after the
// previous grid's last CTA exits (grid completion and memory flush), which
// across 31 stages was a third of the step.  Instead every CTA of stage s
// adds 1 to done[s] once its results are stored (stage_signal: CTA barrier,
// then a device-scope fence and the add by one thread), and a CTA of stage
// s + 1 waits until done[s] counts every CTA of stage s (acquire load,
// bounded by kWaitNs; a timeout sets *A.err, which also releases every other
// waiter).  Each CTA lets the next kernel launch only after its own wait
// (griddepcontrol.launch_dependents), so that kernel's CTAs are placed only
// once every CTA of this one is resident and past its wait: at most two
// stages share the SMs, and the running one never waits on the waiting one.
// Stage ids: 5 l + {0 qkv, 1 attn, 2 oproj, 3 upgate, 4 down}, 5 L the LM
// head; -1 in the persistent kernel, whose grid barriers order the stages.
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__host__ __device__ inline int down_cols(int k);

// CTAs launched for stage s (they match enqueue_step's grids)
__device__ inline unsigned stage_ctas(const StepArgs &A, int s) {
    const Dims &D = A.D;
    if (s == 5 * A.L) return (unsigned)((D.vocab + 31) / 32);
    const int l = s / 5;
    switch (s % 5) {
    case 0: return (unsigned)((D.qkv + 31) / 32);
    case 1: return (unsigned)(D.nh * D.nchunk);
    case 2: return (unsigned)((D.d + 31) / 32);
    case 3: {
        const LayerPtrs &Lp = A.layers[l];
        return (unsigned)(Lp.k * ((Lp.F + kUnitsPerCta - 1) / kUnitsPerCta));
    }
    default: {
        const int c = down_cols(A.layers[l].k);
        return (unsigned)((D.d + c - 1) / c);
    }
    }
}

// n floats from p into L2, one 128-byte line per thread of `nthreads`
// (thread t of them); no registers held, nothing waits for it.
__device__ __forceinline__ void prefetch_l2(const float *p, size_t n, int t, int nthreads) {
    for (size_t l = t; l < (n + 31) / 32; l += nthreads)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(p + l * 32));
}

// Stage timeline (MOE_B200_DECODER_STAMPS=1): per stage, the earliest CTA
// entry, the earliest and latest return from the stage's wait, and the
// latest CTA exit, in %globaltimer nanoseconds (thread 0 of each CTA).
__device__ __forceinline__ void stamp_min(const StepArgs &A, int st, int which) {
    if (A.stamps && st >= 0 && threadIdx.x == 0)
        atomicMin(A.stamps + 4 * st + which, (unsigned long long)globaltimer_ns());
}
__device__ __forceinline__ void stamp_max(const StepArgs &A, int st, int which) {
    if (A.stamps && st >= 0 && threadIdx.x == 0)
        atomicMax(A.stamps + 4 * st + which, (unsigned long long)globaltimer_ns());
}
// the CTA's exit: after every thread's work
__device__ __forceinline__ void stamp_exit(const StepArgs &A, int st) {
    if (A.stamps) {
        __syncthreads();
        stamp_max(A, st, 3);
    }
}

// Flag mode: wait (thread 0, then the CTA) until done[idx] reaches target.
__device__ __forceinline__ void flag_wait(const StepArgs &A, int idx, unsigned target) {
    if (threadIdx.x == 0) {
        const uint64_t t0 = globaltimer_ns();
        while (true) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(A.done + idx)
                         : "memory");
            if (v >= target) break;
            if (*(volatile int *)A.err) break;
            if (globaltimer_ns() - t0 > kWaitNs) { atomicExch(A.err, 1); break; }
            __nanosleep(32);
        }
    }
    __syncthreads();
}

__device__ __forceinline__ void stage_wait(const StepArgs &A, int st) {
    if (st < 0) return;
    if (!A.flags) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        stamp_min(A, st, 1);
        stamp_max(A, st, 2);
        return;
    }
    if (st > 0) flag_wait(A, st - 1, stage_ctas(A, st - 1));
    stamp_min(A, st, 1);
    stamp_max(A, st, 2);
    if (A.flags == 1) pdl_trigger();
}

// Flag mode: this CTA's results of stage st are stored (every thread).
__device__ __forceinline__ void stage_signal(const StepArgs &A, int st) {
    if (!A.flags || st < 0) return;
    if (A.flags == 2) pdl_trigger();
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(A.done + st, 1u);
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// S.xn[i] = x[i] * (1 / sqrt(mean(x²) + eps)) * w[i] for i < d, zero up to
// d_pad (rmsnorm_vec, src/inference.c:209-215); every CTA sums the squares
// in the same fixed order.
__device__ __forceinline__ void rmsnorm_to_smem(const float *x, const float *__restrict__ w,
                                                const Dims &D, Smem &S) {
    constexpr int KEEP = 8;            // values kept in registers (d <= 2048)
    float xv[KEEP], wv[KEEP];
    float ss = 0.0f;
#pragma unroll
    for (int u = 0; u < KEEP; u++) {   // the weights load alongside x, not after the sum
        const int i = threadIdx.x + u * kThreads;
        xv[u] = i < D.d ? ldcg(x + i) : 0.0f;
        wv[u] = i < D.d ? __ldg(w + i) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < KEEP; u++) ss = __fmaf_rn(xv[u], xv[u], ss);
    for (int i = threadIdx.x + KEEP * kThreads; i < D.d; i += kThreads) {
        const float v = ldcg(x + i);
        ss = __fmaf_rn(v, v, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) S.red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int q = 0; q < kThreads / 32; q++) tot += S.red[q];
    const float inv = 1.0f / sqrtf(tot / (float)D.d + D.eps);
#pragma unroll
    for (int u = 0; u < KEEP; u++) {
        const int i = threadIdx.x + u * kThreads;
        if (i < D.d_pad) S.xn[i] = i < D.d ? __fmul_rn(__fmul_rn(xv[u], inv), wv[u]) : 0.0f;
    }
    for (int i = threadIdx.x + KEEP * kThreads; i < D.d_pad; i += kThreads)
        S.xn[i] = i < D.d ? __fmul_rn(__fmul_rn(ldcg(x + i), inv), __ldg(w + i)) : 0.0f;
    __syncthreads();
}

// 32 output columns of v[0..n_in)·W[n_in × ld] (row-major, the reference's
// matvec layout, src/inference.c:174-182): lane = column, warps split the
// rows, partial sums added in warp order.  The value is valid in warp 0.
// The first kPreRows rows of a thread's column do not depend on the input
// vector, so a stage loads them (matvec32_preload) before the vector is
// ready (RMSNorm, attention combine) and matvec32 starts from them; the sum
// still runs over the rows in order, so the result is the same.
constexpr int kPreRows = 48;
struct MatvecPre {
    float w[kPreRows];
};

__device__ __forceinline__ void matvec32_preload(const float *__restrict__ W, int n_in, int ld,
                                                 int col, bool valid, MatvecPre &P) {
    const int warp = threadIdx.x >> 5;
    const int rows = (n_in + 7) / 8, r0 = warp * rows, r1 = min(n_in, r0 + rows);
#pragma unroll
    for (int u = 0; u < kPreRows; u++)
        P.w[u] = (valid && r0 + u < r1) ? __ldg(W + (size_t)(r0 + u) * ld + col) : 0.0f;
}

__device__ __forceinline__ float matvec32(const float *v, const float *__restrict__ W, int n_in,
                                          int ld, int col, bool valid, Smem &S,
                                          const MatvecPre *P = nullptr) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rows = (n_in + 7) / 8, r0 = warp * rows, r1 = min(n_in, r0 + rows);
    float acc = 0.0f;
    if (valid) {
        int first = r0;
        if (P) {
#pragma unroll
            for (int u = 0; u < kPreRows; u++)
                if (r0 + u < r1) acc = __fmaf_rn(v[r0 + u], P->w[u], acc);
            first = r0 + kPreRows;
        }
        // 24 rows' loads in flight before their FMAs (a decode step is
        // memory-latency bound); the sum still runs in row order
        for (int i0 = first; i0 < r1; i0 += 24) {
            float wv[24];
#pragma unroll
            for (int u = 0; u < 24; u++)
                wv[u] = i0 + u < r1 ? __ldg(W + (size_t)(i0 + u) * ld + col) : 0.0f;
#pragma unroll
            for (int u = 0; u < 24; u++)
                if (i0 + u < r1) acc = __fmaf_rn(v[i0 + u], wv[u], acc);
        }
    }
    S.red[warp * 32 + lane] = acc;
    __syncthreads();
    float out = 0.0f;
    if (warp == 0) {
#pragma unroll
        for (int q = 0; q < 8; q++) out += S.red[q * 32 + lane];
    }
    __syncthreads();                   // S.red is reused by the next item
    return out;
}

// ---- the stages; `item` is a unit of a stage's work ----

// 1: RMSNorm, x·[W_Q | W_K | W_V] for 32 columns, RoPE, KV append.  Layer 0
// starts from the token's embedding row; item 0 also stores it as the
// residual stream.
__device__ void qkv_item(const StepArgs &A, const LayerPtrs &Lp, int layer, int token, int pos,
                         int item, Smem &S, int st) {
    const Dims &D = A.D;
    const float *src = layer == 0 ? A.embed + (size_t)token * D.d : A.x;
    const int lane = threadIdx.x & 31, col = item * 32 + lane;
    // weights and RoPE factors first: neither depends on the residual stream
    MatvecPre P;
    matvec32_preload(Lp.w_qkv, D.d, D.qkv, col, col < D.qkv, P);
    const int c = col < D.nq ? col : col - D.nq;
    const int half = D.hd / 2, pi = (c % D.hd) >> 1;
    float cr = 0.0f, sr = 0.0f;
    if (threadIdx.x < 32 && col < D.nq + D.kvd) {
        cr = __ldg(A.rope_cos + (size_t)pos * half + pi);
        sr = __ldg(A.rope_sin + (size_t)pos * half + pi);
    }
    stage_wait(A, st);
    if (layer == 0 && item == 0)
        for (int i = threadIdx.x; i < D.d; i += kThreads) A.x[i] = __ldg(src + i);
    rmsnorm_to_smem(src, Lp.rms_attn, D, S);
    const float v = matvec32(S.xn, Lp.w_qkv, D.d, D.qkv, col, col < D.qkv, S, &P);
    if (threadIdx.x < 32) {
        // RoPE pairs (2i, 2i+1) of a head sit in adjacent lanes
        const float other = __shfl_xor_sync(0xffffffffu, v, 1);
        float *kc = A.kc + (size_t)layer * D.max_seq * D.kvd;
        float *vc = A.vc + (size_t)layer * D.max_seq * D.kvd;
        if (col < D.nq + D.kvd) {
            const bool even = (c & 1) == 0;
            const float v0 = even ? v : other, v1 = even ? other : v;
            const float r = even ? __fsub_rn(__fmul_rn(v0, cr), __fmul_rn(v1, sr))
                                 : __fadd_rn(__fmul_rn(v0, sr), __fmul_rn(v1, cr));
            if (col < D.nq) A.q[col] = r;
            else kc[(size_t)pos * D.kvd + c] = r;
        } else if (col < D.qkv) {
            vc[(size_t)pos * D.kvd + (col - D.nq - D.kvd)] = v;
        }
    }
}

// 2: query head h, positions [chunk*CH, +CH) of 0..pos: chunk max m, sum of
// exp(s - m) and the exp-weighted V sum, written to part[h][chunk] =
// {m, l, o[hd]} (scores q·k / sqrt(hd), GQA kvh = h / (nh / nkv),
// src/inference.c:285-305).
__device__ void attn_item(const StepArgs &A, int layer, int pos, int h, int chunk, Smem &S,
                          int st) {
    const Dims &D = A.D;
    const int j0 = chunk * CH, n = min(CH, pos + 1 - j0);
    const float *kc = A.kc + (size_t)layer * D.max_seq * D.kvd;
    const float *vc = A.vc + (size_t)layer * D.max_seq * D.kvd;
    float *dst = A.part + ((size_t)h * D.nchunk + chunk) * (D.hd + 2);
    const int g = h / (D.nh / D.nkv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int PW = CH / (kThreads / 32);          // positions per warp
    float kv[PW][4];                                  // hd <= 128: 4 values per lane
    // every key and value load in flight first; the cache rows of earlier
    // steps' positions do not depend on this step, only position pos (this
    // step's token) does
#pragma unroll
    for (int t = 0; t < PW; t++) {
        const int jj = warp + t * (kThreads / 32);
        const float *kr = kc + (size_t)(j0 + jj) * D.kvd + g * D.hd;
#pragma unroll
        for (int c = 0; c < 4; c++)
            kv[t][c] = (jj < n && j0 + jj != pos && lane + 32 * c < D.hd) ? ldcg(kr + lane + 32 * c)
                                                                          : 0.0f;
    }
    // the value pass's positions for this thread: groups of hd threads split
    // the chunk (at most CH / (kThreads / hd) = 32 positions each for hd <= 128)
    constexpr int VMAX = 32;
    const int groups = kThreads / D.hd, gi = threadIdx.x / D.hd, i = threadIdx.x - gi * D.hd;
    const int per = (n + groups - 1) / groups;
    const int jlo = gi * per, jhi = min(n, jlo + per);
    const float *vcol = vc + (size_t)j0 * D.kvd + g * D.hd + i;
    float vpre[VMAX];
#pragma unroll
    for (int u = 0; u < VMAX; u++)
        vpre[u] = (gi < groups && jlo + u < jhi && j0 + jlo + u != pos)
                      ? ldcg(vcol + (size_t)(jlo + u) * D.kvd) : 0.0f;
    stage_wait(A, st);
#pragma unroll
    for (int t = 0; t < PW; t++) {
        const int jj = warp + t * (kThreads / 32);
        if (j0 + jj != pos) continue;
        const float *kr = kc + (size_t)(j0 + jj) * D.kvd + g * D.hd;
#pragma unroll
        for (int c = 0; c < 4; c++)
            kv[t][c] = (jj < n && lane + 32 * c < D.hd) ? ldcg(kr + lane + 32 * c) : 0.0f;
    }
    for (int i = threadIdx.x; i < D.hd; i += kThreads) S.qs[i] = ldcg(A.q + h * D.hd + i);
    __syncthreads();
#pragma unroll
    for (int t = 0; t < PW; t++) {
        const int jj = warp + t * (kThreads / 32);
        float p = 0.0f;
#pragma unroll
        for (int c = 0; c < 4; c++)
            if (lane + 32 * c < D.hd) p = __fmaf_rn(S.qs[lane + 32 * c], kv[t][c], p);
        p = warp_sum(p);
        if (lane == 0 && jj < n) S.sc[jj] = __fmul_rn(p, D.scale);
    }
    __syncthreads();
    if (warp == 0) {                   // max, exp and sum over the chunk (CH = 64: 2 per lane)
        const float s0 = lane < n ? S.sc[lane] : -INFINITY;
        const float s1 = lane + 32 < n ? S.sc[lane + 32] : -INFINITY;
        float m = fmaxf(s0, s1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float e0 = lane < n ? expf(__fsub_rn(s0, m)) : 0.0f;
        const float e1 = lane + 32 < n ? expf(__fsub_rn(s1, m)) : 0.0f;
        if (lane < n) S.sc[lane] = e0;
        if (lane + 32 < n) S.sc[lane + 32] = e1;
        const float l = warp_sum(__fadd_rn(e0, e1));
        if (lane == 0) { dst[0] = m; dst[1] = l; }
    }
    __syncthreads();
    // the exp-weighted V sum: the chunk's positions are split over groups of
    // hd threads (every thread of the CTA busy; the values were loaded before
    // the wait, only position pos's after it), the sum in position order, the
    // group partials added in group order
    if (gi < groups) {
        float o = 0.0f;
#pragma unroll
        for (int u = 0; u < VMAX; u++) {
            if (jlo + u >= jhi) break;
            const float v = j0 + jlo + u == pos ? ldcg(vcol + (size_t)(jlo + u) * D.kvd) : vpre[u];
            o = __fmaf_rn(S.sc[jlo + u], v, o);
        }
        S.red[gi * D.hd + i] = o;
    }
    __syncthreads();
    if (threadIdx.x < D.hd) {
        float o = S.red[threadIdx.x];
        for (int q = 1; q < groups; q++) o = __fadd_rn(o, S.red[q * D.hd + threadIdx.x]);
        dst[2 + threadIdx.x] = o;
    }
    __syncthreads();                   // S.qs / S.sc / S.red are reused by the next item
}

// 3: softmax-weighted head outputs from the chunks, then x += head_out·W_O
// for 32 columns (src/inference.c:307-309).
__device__ void oproj_item(const StepArgs &A, const LayerPtrs &Lp, int pos, int item, Smem &S,
                           int st) {
    const Dims &D = A.D;
    const int nch = (pos + 1 + CH - 1) / CH;
    const int lane = threadIdx.x & 31, col = item * 32 + lane;
    MatvecPre P;                       // W_O rows do not wait for the attention output
    matvec32_preload(Lp.w_o, D.nq, D.d, col, col < D.d, P);
    // Flag mode: the residual stream is final once this layer's Q/K/V stage
    // is done (it waited for the previous layer's down stage, or wrote the
    // embedding), which every attention CTA had seen before this kernel was
    // launched; so this wait returns at once and the residual loads now.
    const bool early_x = A.flags == 1 && st > 0;
    float xres = 0.0f;
    if (early_x) {
        flag_wait(A, st - 2, stage_ctas(A, st - 2));
        if (threadIdx.x < 32 && col < D.d) xres = ldcg(A.x + col);
    }
    stage_wait(A, st);
    for (int t = threadIdx.x; t < D.nq; t += kThreads) {
        const int h = t / D.hd, i = t % D.hd;
        const float *ph = A.part + (size_t)h * D.nchunk * (D.hd + 2);
        float M = -INFINITY, L = 0.0f, O = 0.0f;
        for (int c0 = 0; c0 < nch; c0 += 12) {         // 12 chunks' loads in flight
            float mc[12], lc[12], oc[12];
#pragma unroll
            for (int u = 0; u < 12; u++) {
                const float *pc = ph + (size_t)(c0 + u) * (D.hd + 2);
                const bool ok = c0 + u < nch;
                mc[u] = ok ? ldcg(pc) : -INFINITY;
                lc[u] = ok ? ldcg(pc + 1) : 0.0f;
                oc[u] = ok ? ldcg(pc + 2 + i) : 0.0f;
            }
            // the batch's maximum first, so its exponentials are independent
            // of each other; the sums still run chunk by chunk in order
            float Mn = M;
#pragma unroll
            for (int u = 0; u < 12; u++) Mn = fmaxf(Mn, mc[u]);
            const float a = expf(__fsub_rn(M, Mn));
            L = __fmul_rn(L, a);
            O = __fmul_rn(O, a);
#pragma unroll
            for (int u = 0; u < 12; u++) {
                if (c0 + u >= nch) break;
                const float b = expf(__fsub_rn(mc[u], Mn));
                L = __fmaf_rn(lc[u], b, L);
                O = __fmaf_rn(oc[u], b, O);
            }
            M = Mn;
        }
        S.xn[t] = __fdiv_rn(O, L);
    }
    __syncthreads();
    const float v = matvec32(S.xn, Lp.w_o, D.nq, D.d, col, col < D.d, S, &P);
    if (threadIdx.x < 32 && col < D.d) A.x[col] = __fadd_rn(early_x ? xres : ldcg(A.x + col), v);
}

// 4 (once per CTA before its up/gate items): RMSNorm into S.xn, router
// logits and the reference's routing of the token into S.sel / S.w
// (src/inference.c:311; src/transformer.c:299-337).  `publish` also stores
// the ids and weights for the down stage, and the normalised vector into
// the layer's trace row.
__device__ void route_cta(const StepArgs &A, const LayerPtrs &Lp, int layer, bool publish,
                          Smem &S, int st) {
    const Dims &D = A.D;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the first 16 router weights of this lane's first expert, before the
    // residual-stream wait of the RMSNorm
    float w0[16];
#pragma unroll
    for (int u = 0; u < 16; u++) {
        const int i = lane + 32 * u;
        w0[u] = (warp < Lp.E && i < D.d) ? __ldg(Lp.router + (size_t)i * Lp.E + warp) : 0.0f;
    }
    stage_wait(A, st);
    rmsnorm_to_smem(A.x, Lp.rms_ffn, D, S);
    if (publish)
        for (int i = threadIdx.x; i < D.d; i += kThreads) A.trace[(size_t)layer * 2 * D.d + i] = S.xn[i];
    for (int e = warp; e < Lp.E; e += kThreads / 32) {
        float p = 0.0f;
        for (int i0 = lane; i0 < D.d; i0 += 32 * 16) {   // 16 loads in flight per lane
            float wv[16];
#pragma unroll
            for (int u = 0; u < 16; u++) {
                const int i = i0 + 32 * u;
                wv[u] = (e == warp && i0 == lane) ? w0[u]
                        : i < D.d ? __ldg(Lp.router + (size_t)i * Lp.E + e) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 16; u++) {
                const int i = i0 + 32 * u;
                if (i < D.d) p = __fmaf_rn(S.xn[i], wv[u], p);
            }
        }
        p = warp_sum(p);
        if (lane == 0) S.lg[e] = p;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (Lp.E <= 8) route_token8(S.lg, Lp.E, Lp.k, S.sel, S.w);
        else route_token(S.lg, Lp.E, Lp.k, S.sel, S.w);
        if (publish) {
            for (int r = 0; r < Lp.k; r++) { A.ids[r] = S.sel[r]; A.wts[r] = S.w[r]; }
            if (A.flags == 1) {                 // the down stage may load its rows now
                __threadfence();
                atomicAdd(A.done + 5 * A.L + 1 + layer, 1u);
            }
        }
    }
    __syncthreads();
}

// After the routing (S.sel valid): the down rows of the selected experts
// into L2, one 128-byte line per thread of the stage (thread t of nthreads),
// so that the down stage's weight loads hit L2.
__device__ __forceinline__ void prefetch_down(const StepArgs &A, const LayerPtrs &Lp, int t,
                                              int nthreads, const Smem &S) {
    const size_t lines = (size_t)A.D.d_pad * Lp.F_pad / 32;     // per expert
    for (size_t l = t; l < lines * Lp.k; l += nthreads) {
        const int r = (int)(l / lines);
        const float *p = Lp.dn + (size_t)S.sel[r] * A.D.d_pad * Lp.F_pad + (l - r * lines) * 32;
        asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
    }
}

// 5: kUnitsPerCta hidden units of rank r, kUnitsPerWarp consecutive units
// per warp (their loads in flight together): the gate and up rows of expert
// S.sel[r] in the packed layout (128 gate rows, then the matching 128 up
// rows), dot x_norm, the reference's silu(gate)·up into h[r][f].
__device__ void upgate_item(const StepArgs &A, const LayerPtrs &Lp, int item, Smem &S) {
    const Dims &D = A.D;
    const int nfb = (Lp.F + kUnitsPerCta - 1) / kUnitsPerCta;
    const int r = item / nfb, lane = threadIdx.x & 31;
    const int f0 = (item % nfb) * kUnitsPerCta + (threadIdx.x >> 5) * kUnitsPerWarp;
    if (f0 >= Lp.F) return;
    const int e = S.sel[r];
    const float4 *gw[kUnitsPerWarp], *uw[kUnitsPerWarp];
    bool on[kUnitsPerWarp];
#pragma unroll
    for (int v = 0; v < kUnitsPerWarp; v++) {
        const int f = f0 + v;
        on[v] = f < Lp.F;
        const size_t grow = (size_t)e * 2 * Lp.F_pad + (size_t)(f / 128) * 256 + (f % 128);
        gw[v] = reinterpret_cast<const float4 *>(Lp.ug + grow * D.d_pad);
        uw[v] = reinterpret_cast<const float4 *>(Lp.ug + (grow + 128) * D.d_pad);
    }
    const float4 *x4 = reinterpret_cast<const float4 *>(S.xn);
    float g[kUnitsPerWarp], u[kUnitsPerWarp];
#pragma unroll
    for (int v = 0; v < kUnitsPerWarp; v++) g[v] = u[v] = 0.0f;
    const int n4 = D.d_pad / 4;
    for (int i0 = lane; i0 < n4; i0 += 32 * 4) {        // 4 gate/up float4 pairs per unit in flight
        float4 a[kUnitsPerWarp][4], b[kUnitsPerWarp][4];
#pragma unroll
        for (int v = 0; v < kUnitsPerWarp; v++)
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int i = i0 + 32 * q;
                const bool ok = on[v] && i < n4;
                a[v][q] = ok ? __ldg(gw[v] + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                b[v][q] = ok ? __ldg(uw[v] + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
        for (int v = 0; v < kUnitsPerWarp; v++)
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int i = i0 + 32 * q;
                if (i >= n4) break;
                const float4 xv = x4[i];
                g[v] = __fmaf_rn(xv.x, a[v][q].x, g[v]); g[v] = __fmaf_rn(xv.y, a[v][q].y, g[v]);
                g[v] = __fmaf_rn(xv.z, a[v][q].z, g[v]); g[v] = __fmaf_rn(xv.w, a[v][q].w, g[v]);
                u[v] = __fmaf_rn(xv.x, b[v][q].x, u[v]); u[v] = __fmaf_rn(xv.y, b[v][q].y, u[v]);
                u[v] = __fmaf_rn(xv.z, b[v][q].z, u[v]); u[v] = __fmaf_rn(xv.w, b[v][q].w, u[v]);
            }
    }
#pragma unroll
    for (int v = 0; v < kUnitsPerWarp; v++) {
        const float gs = warp_sum(g[v]), us = warp_sum(u[v]);
        if (lane == 0 && on[v]) A.h[(size_t)r * Lp.F_pad + f0 + v] = swiglu_ref(gs, us);
    }
}

// 6: one warp per (output column, rank): y_r = h_r·W_down[ids[r]] row j
// (packed [d_pad × F_pad]), then x[j] += w_0·y_0 + w_1·y_1 + ... in rank
// order (src/transformer.c:355-358).  A CTA's 8 warps cover down_cols(k)
// columns, so the k rows of a column load in parallel.  The sum runs over
// the row in batches of 8 float4 per lane (padding lanes add 0·0).
__host__ __device__ inline int down_cols(int k) { return k >= kThreads / 32 ? 1 : (kThreads / 32) / k; }

__device__ void down_item(const StepArgs &A, const LayerPtrs &Lp, int layer, int item, Smem &S,
                          int st) {
    const Dims &D = A.D;
    const int cols = down_cols(Lp.k);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cw = warp / Lp.k, r = warp - cw * Lp.k;
    const int j = item * cols + cw;
    float y = 0.0f;
    stage_wait(A, st);
    if (cw < cols && j < D.d) {
        const int e = __ldcg(A.ids + r);
        const float4 *wr = reinterpret_cast<const float4 *>(Lp.dn + ((size_t)e * D.d_pad + j) * Lp.F_pad);
        const float4 *hr = reinterpret_cast<const float4 *>(A.h + (size_t)r * Lp.F_pad);
        for (int i0 = lane; i0 < Lp.F_pad / 4; i0 += 32 * 8) {   // 8 float4 pairs in flight
            float4 a[8], hb[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = i0 + 32 * u;
                const bool ok = i < Lp.F_pad / 4;
                a[u] = ok ? __ldg(wr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                hb[u] = ok ? __ldcg(hr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                y = __fmaf_rn(hb[u].x, a[u].x, y); y = __fmaf_rn(hb[u].y, a[u].y, y);
                y = __fmaf_rn(hb[u].z, a[u].z, y); y = __fmaf_rn(hb[u].w, a[u].w, y);
            }
        }
        y = warp_sum(y);
    }
    if (lane == 0) S.red[warp] = y;
    __syncthreads();
    if (threadIdx.x < cols) {
        const int jj = item * cols + threadIdx.x;
        if (jj < D.d) {
            float out = 0.0f;
            for (int rr = 0; rr < Lp.k; rr++)
                out = __fmaf_rn(ldcg(A.wts + rr), S.red[threadIdx.x * Lp.k + rr], out);
            A.trace[((size_t)layer * 2 + 1) * D.d + jj] = out;
            A.x[jj] = __fadd_rn(ldcg(A.x + jj), out);
        }
    }
    __syncthreads();                   // S.red is reused by the next item
}

// Flag mode, the same arithmetic as down_item with the expert rows loaded
// before the up/gate stage finishes: the up/gate stage's first CTA publishes
// the layer's ids and weights right after it routes the token (done counter
// ids_ready(layer)), so a CTA here waits for that, loads the first kDownPre
// float4 of each lane's weight row (and the residual of its columns, final
// since the W_O stage), and only then waits for h.  h (k × F_pad floats) is
// staged in shared memory by the whole CTA.  Used when the rows fit
// (F_pad ≤ 4 · 32 · kDownPre, k · F_pad ≤ kMaxD).
constexpr int kDownPre = 16;            // two batches of 8
__device__ __forceinline__ int ids_ready(const StepArgs &A, int layer) { return 5 * A.L + 1 + layer; }
__device__ __forceinline__ bool down_flag_fits(const LayerPtrs &Lp) {
    return Lp.F_pad / 4 <= 32 * kDownPre && Lp.k * Lp.F_pad <= kMaxD;
}

__device__ void down_item_flag(const StepArgs &A, const LayerPtrs &Lp, int layer, int item,
                               Smem &S, int st) {
    const Dims &D = A.D;
    const int cols = down_cols(Lp.k);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cw = warp / Lp.k, r = warp - cw * Lp.k;
    const int j = item * cols + cw;
    const bool active = cw < cols && j < D.d;
    const int n4 = Lp.F_pad / 4;
    // the next stage's weights into L2 while this layer's up/gate runs: its
    // CTAs then preload them from L2 instead of HBM
    {
        const int t = blockIdx.x * kThreads + threadIdx.x, nt = gridDim.x * kThreads;
        if (layer + 1 < A.L) prefetch_l2(A.layers[layer + 1].w_qkv, (size_t)D.d * D.qkv, t, nt);
        else prefetch_l2(A.lm_head, (size_t)D.d * D.vocab, t, nt);
    }
    flag_wait(A, ids_ready(A, layer), 1u);
    if (threadIdx.x < Lp.k) {
        S.sel[threadIdx.x] = __ldcg(A.ids + threadIdx.x);
        S.w[threadIdx.x] = ldcg(A.wts + threadIdx.x);
    }
    __syncthreads();
    float4 wp[kDownPre];
    if (active) {
        const float4 *wr =
            reinterpret_cast<const float4 *>(Lp.dn + ((size_t)S.sel[r] * D.d_pad + j) * Lp.F_pad);
#pragma unroll
        for (int u = 0; u < kDownPre; u++) {
            const int i = lane + 32 * u;
            wp[u] = i < n4 ? __ldg(wr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    const int jj = item * cols + threadIdx.x;
    const float xres = (threadIdx.x < cols && jj < D.d) ? ldcg(A.x + jj) : 0.0f;
    stage_wait(A, st);
    {
        const float4 *h4 = reinterpret_cast<const float4 *>(A.h);
        float4 *s4 = reinterpret_cast<float4 *>(S.xn);
        for (int i = threadIdx.x; i < Lp.k * n4; i += kThreads) s4[i] = __ldcg(h4 + i);
    }
    __syncthreads();
    float y = 0.0f;
    if (active) {
        const float4 *hr = reinterpret_cast<const float4 *>(S.xn) + (size_t)r * n4;
        // batches of 8 as in down_item, each run only where its loop would run it
#pragma unroll
        for (int u = 0; u < kDownPre; u++) {
            if (lane + 32 * 8 * (u / 8) >= n4) break;
            const int i = lane + 32 * u;
            const float4 hb = i < n4 ? hr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            y = __fmaf_rn(hb.x, wp[u].x, y); y = __fmaf_rn(hb.y, wp[u].y, y);
            y = __fmaf_rn(hb.z, wp[u].z, y); y = __fmaf_rn(hb.w, wp[u].w, y);
        }
        y = warp_sum(y);
    }
    if (lane == 0) S.red[warp] = y;
    __syncthreads();
    if (threadIdx.x < cols && jj < D.d) {
        float out = 0.0f;
        for (int rr = 0; rr < Lp.k; rr++)
            out = __fmaf_rn(S.w[rr], S.red[threadIdx.x * Lp.k + rr], out);
        A.trace[((size_t)layer * 2 + 1) * D.d + jj] = out;
        A.x[jj] = __fadd_rn(xres, out);
    }
    __syncthreads();
}

// 7: final RMSNorm and 32 columns of the LM head (x_norm·lm_head, [d × vocab]).
__device__ void lmhead_item(const StepArgs &A, int item, bool normed, Smem &S, int st) {
    const Dims &D = A.D;
    const int lane = threadIdx.x & 31, col = item * 32 + lane;
    MatvecPre P;
    matvec32_preload(A.lm_head, D.d, D.vocab, col, col < D.vocab, P);
    stage_wait(A, st);
    if (!normed) rmsnorm_to_smem(A.x, A.rms_final, D, S);
    const float v = matvec32(S.xn, A.lm_head, D.d, D.vocab, col, col < D.vocab, S, &P);
    if (threadIdx.x < 32 && col < D.vocab) A.logits[col] = v;
}

// ---- one kernel per stage (the graph path) ----

__global__ void __launch_bounds__(kThreads) qkv_kernel(StepArgs A, int layer) {
    __shared__ Smem S;
    stamp_min(A, 5 * layer, 0);
    if (A.pdl_early) pdl_trigger();
    if (A.flags == 1 && (A.early_mask >> 0 & 1)) pdl_trigger();
    const LayerPtrs Lp = A.layers[layer];
    const int st = 5 * layer;
    qkv_item(A, Lp, layer, A.state[0], A.state[1], blockIdx.x, S, st);
    stamp_exit(A, st);
    stage_signal(A, st);
}
__global__ void __launch_bounds__(kThreads) attn_kernel(StepArgs A, int layer) {
    __shared__ Smem S;
    stamp_min(A, 5 * layer + 1, 0);
    if (A.pdl_early) pdl_trigger();
    if (A.flags == 1 && (A.early_mask >> 1 & 1)) pdl_trigger();
    const int pos = A.state[1], st = 5 * layer + 1;
    // chunks past the step's position have no work (they still count as done)
    if ((int)blockIdx.y * CH <= pos) attn_item(A, layer, pos, blockIdx.x, blockIdx.y, S, st);
    stamp_exit(A, st);
    stage_signal(A, st);
}
__global__ void __launch_bounds__(kThreads, 1) oproj_kernel(StepArgs A, int layer) {
    __shared__ Smem S;
    stamp_min(A, 5 * layer + 2, 0);
    if (A.pdl_early) pdl_trigger();
    if (A.flags == 1 && (A.early_mask >> 2 & 1)) pdl_trigger();
    const int st = 5 * layer + 2;
    oproj_item(A, A.layers[layer], A.state[1], blockIdx.x, S, st);
    stamp_exit(A, st);
    stage_signal(A, st);
}
__global__ void __launch_bounds__(kThreads) upgate_kernel(StepArgs A, int layer) {
    __shared__ Smem S;
    stamp_min(A, 5 * layer + 3, 0);
    if (A.pdl_early) pdl_trigger();
    if (A.flags == 1 && (A.early_mask >> 3 & 1)) pdl_trigger();
    const LayerPtrs Lp = A.layers[layer];
    const int st = 5 * layer + 3;
    route_cta(A, Lp, layer, blockIdx.x == 0, S, st);
    // in flag mode the down stage loads its rows itself once the ids are out
    if (A.flags != 1 || !down_flag_fits(Lp))
        prefetch_down(A, Lp, blockIdx.x * kThreads + threadIdx.x, gridDim.x * kThreads, S);
    upgate_item(A, Lp, blockIdx.x, S);
    stamp_exit(A, st);
    stage_signal(A, st);
}
__global__ void __launch_bounds__(kThreads, 1) down_kernel(StepArgs A, int layer) {
    __shared__ Smem S;
    stamp_min(A, 5 * layer + 4, 0);
    if (A.pdl_early) pdl_trigger();
    if (A.flags == 1 && (A.early_mask >> 4 & 1)) pdl_trigger();
    const int st = 5 * layer + 4;
    const LayerPtrs Lp = A.layers[layer];
    if (A.flags == 1 && down_flag_fits(Lp)) down_item_flag(A, Lp, layer, blockIdx.x, S, st);
    else down_item(A, Lp, layer, blockIdx.x, S, st);
    stamp_exit(A, st);
    stage_signal(A, st);
}
__global__ void __launch_bounds__(kThreads) lmhead_kernel(StepArgs A) {
    __shared__ Smem S;
    stamp_min(A, 5 * A.L, 0);
    if (A.pdl_early) pdl_trigger();
    lmhead_item(A, blockIdx.x, false, S, 5 * A.L);
    stamp_exit(A, 5 * A.L);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        A.state[1] += 1;
        *(volatile int *)A.err_host = *(volatile int *)A.err;   // read by the host after the step
    }
}

// the stage timeline back to "no stamp": minima to ~0, maxima to 0
__global__ void stamps_reset_kernel(unsigned long long *stamps, int n) {
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        stamps[i] = (i % 4 < 2) ? ~0ull : 0ull;
}

// ---- the whole step as one persistent cooperative kernel ----

// Grid-wide barrier: every CTA arrives on one counter and waits, bounded by
// kWaitNs of %globaltimer, until all gridDim.x CTAs of this phase arrived.
// Returns false (and sets *err) if the wait ran out or another CTA gave up.
__device__ __forceinline__ bool grid_barrier(const StepArgs &A, unsigned target, Smem &S) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(A.bar, 1u);
        int good = 1;
        const uint64_t t0 = globaltimer_ns();
        while (true) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(A.bar) : "memory");
            if (v >= target) break;
            if (*(volatile int *)A.err) { good = 0; break; }
            if (globaltimer_ns() - t0 > kWaitNs) { atomicExch(A.err, 1); good = 0; break; }
        }
        __threadfence();
        S.flag = good;
    }
    __syncthreads();
    return S.flag != 0;
}

__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(StepArgs A) {
    __shared__ Smem S;
    const Dims &D = A.D;
    const int token = A.state[0], pos = A.state[1];
    const int G = gridDim.x, b = blockIdx.x;
    unsigned phase = 0;
    const int n_qkv = (D.qkv + 31) / 32, n_col = (D.d + 31) / 32;
    const int nch = (pos + 1 + CH - 1) / CH;
    for (int l = 0; l < A.L; l++) {
        const LayerPtrs Lp = A.layers[l];
        for (int it = b; it < n_qkv; it += G) qkv_item(A, Lp, l, token, pos, it, S, -1);
        if (!grid_barrier(A, ++phase * G, S)) return;
        for (int it = b; it < D.nh * nch; it += G) attn_item(A, l, pos, it / nch, it % nch, S, -1);
        if (!grid_barrier(A, ++phase * G, S)) return;
        for (int it = b; it < n_col; it += G) oproj_item(A, Lp, pos, it, S, -1);
        if (!grid_barrier(A, ++phase * G, S)) return;
        const int n_ug = Lp.k * ((Lp.F + kUnitsPerCta - 1) / kUnitsPerCta);
        if (b < n_ug) {
            route_cta(A, Lp, l, b == 0, S, -1);
            prefetch_down(A, Lp, b * kThreads + threadIdx.x, min(G, n_ug) * kThreads, S);
            for (int it = b; it < n_ug; it += G) upgate_item(A, Lp, it, S);
        }
        if (!grid_barrier(A, ++phase * G, S)) return;
        const int n_down = (D.d + down_cols(Lp.k) - 1) / down_cols(Lp.k);
        for (int it = b; it < n_down; it += G) down_item(A, Lp, l, it, S, -1);
        if (!grid_barrier(A, ++phase * G, S)) return;
    }
    const int n_lm = (D.vocab + 31) / 32;
    bool normed = false;
    for (int it = b; it < n_lm; it += G) {
        lmhead_item(A, it, normed, S, -1);
        normed = true;                  // S.xn keeps the normalised vector across items
    }
    if (b == 0 && threadIdx.x == 0) {
        A.state[1] = pos + 1;
        *(volatile int *)A.err_host = *(volatile int *)A.err;
    }
}

}  // namespace decs
}  // namespace moe

using namespace moe;
using namespace moe::decs;

struct DecLayer {
    float *rms_attn = nullptr, *rms_ffn = nullptr, *w_qkv = nullptr, *w_o = nullptr;
    moe_b200_weights *ffn = nullptr;
};

struct moe_b200_decoder {
    int device = 0;
    Dims D{};
    int L = 0, pos = 0, flags = 0, grid = 0;
    float *embed = nullptr, *rms_final = nullptr, *lm_head = nullptr, *rope_cos = nullptr,
          *rope_sin = nullptr;
    std::vector<DecLayer> layers;
    LayerPtrs *d_layers = nullptr;
    float *kc = nullptr, *vc = nullptr;          // [L][max_seq][kvd]
    float *x = nullptr, *q = nullptr, *part = nullptr, *h = nullptr, *logits = nullptr,
          *wts = nullptr;
    int *state = nullptr, *ids = nullptr;        // state = {token, pos}
    unsigned *bar = nullptr;
    unsigned *done = nullptr;                    // [6 L + 1], StepArgs::done
    int *err = nullptr;
    int *h_err = nullptr;                        // mapped pinned copy of err (StepArgs::err_host)
    int *d_err_host = nullptr;                   // its device address
    float *trace = nullptr;                      // [L][2][d], see StepArgs::trace
    unsigned long long *stamps = nullptr;        // StepArgs::stamps (MOE_B200_DECODER_STAMPS=1)
    int *h_token = nullptr;                      // pinned
    int maxF_pad = 0;
    cudaStream_t stream = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int launches = 0;
    // programmatic dependent launch of the stage kernels: 0 off, 1 each kernel
    // lets the next one launch on entry, 2 the next one launches as the
    // current one's CTAs exit, 3 flag mode (see stage_wait)
    int pdl = 3;
    // flag mode: stage kinds whose CTAs trigger the next launch on entry;
    // the down stage by default (c2 0.1466 -> 0.1461 ms; every stage: 0.168)
    int early_mask = 16;
};

namespace {

int dfail(int code, const char *msg) { return moe::set_last_error(code, msg); }

#define DCK(call)                                                                          \
    do {                                                                                   \
        cudaError_t e_ = (call);                                                           \
        if (e_ != cudaSuccess) return dfail(MOE_B200_E_CUDA, cudaGetErrorString(e_));       \
    } while (0)

int upload(float **dst, const float *src, size_t n) {
    DCK(cudaMalloc(dst, n * sizeof(float)));
    DCK(cudaMemcpy(*dst, src, n * sizeof(float), cudaMemcpyHostToDevice));
    return MOE_B200_OK;
}

void free_all(moe_b200_decoder *m) {
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    for (DecLayer &l : m->layers) {
        cudaFree(l.rms_attn); cudaFree(l.rms_ffn); cudaFree(l.w_qkv); cudaFree(l.w_o);
        if (l.ffn) moe_b200_weights_free(l.ffn);
    }
    cudaFree(m->d_layers);
    cudaFree(m->embed); cudaFree(m->rms_final); cudaFree(m->lm_head);
    cudaFree(m->rope_cos); cudaFree(m->rope_sin); cudaFree(m->kc); cudaFree(m->vc);
    cudaFree(m->x); cudaFree(m->q); cudaFree(m->part); cudaFree(m->h);
    cudaFree(m->logits); cudaFree(m->wts); cudaFree(m->state); cudaFree(m->ids);
    cudaFree(m->bar); cudaFree(m->done); cudaFree(m->stamps); cudaFree(m->err); cudaFree(m->trace);
    if (m->h_token) cudaFreeHost(m->h_token);
    if (m->h_err) cudaFreeHost(m->h_err);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

StepArgs step_args(const moe_b200_decoder *m) {
    StepArgs A{};
    A.D = m->D;
    A.L = m->L;
    A.layers = m->d_layers;
    A.embed = m->embed; A.rms_final = m->rms_final; A.lm_head = m->lm_head;
    A.rope_cos = m->rope_cos; A.rope_sin = m->rope_sin;
    A.kc = m->kc; A.vc = m->vc;
    A.x = m->x; A.q = m->q; A.part = m->part; A.h = m->h; A.logits = m->logits; A.wts = m->wts;
    A.state = m->state; A.ids = m->ids; A.bar = m->bar; A.err = m->err;
    A.trace = m->trace;
    A.stamps = (m->flags & MOE_B200_DECODER_PERSISTENT) ? nullptr : m->stamps;
    A.err_host = m->d_err_host;
    A.pdl_early = m->pdl == 1;
    A.flags = (m->flags & MOE_B200_DECODER_PERSISTENT) ? 0 : m->pdl == 3 ? 1 : m->pdl == 4 ? 2 : 0;
    A.done = m->done;
    A.early_mask = m->early_mask;
    return A;
}

// The persistent single-kernel step when asked for; otherwise (the default,
// the faster one measured) one kernel per stage.
static bool persistent(int flags) { return (flags & MOE_B200_DECODER_PERSISTENT) != 0; }

// the step's device work, in order, on m->stream
int enqueue_step(moe_b200_decoder *m) {
    const Dims &D = m->D;
    cudaStream_t s = m->stream;
    StepArgs A = step_args(m);
    if (persistent(m->flags)) {
        DCK(cudaMemsetAsync(m->bar, 0, sizeof(unsigned), s));
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.gridDim = dim3(m->grid, 1, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.stream = s;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        DCK(cudaLaunchKernelEx(&cfg, decode_step_kernel, A));
        m->launches = 1;
        return MOE_B200_OK;
    }
    // every kernel but the step's first may start while its predecessor
    // runs (programmatic dependent launch; the kernels order their reads and
    // writes with griddepcontrol or, in flag mode, the done[] counters,
    // zeroed here: see stage_wait)
    if (m->pdl >= 3) DCK(cudaMemsetAsync(m->done, 0, (size_t)(6 * m->L + 1) * sizeof(unsigned), s));
    if (m->stamps) {
        stamps_reset_kernel<<<1, 256, 0, s>>>(m->stamps, 4 * (5 * m->L + 1));
        DCK(cudaGetLastError());
    }
    int n = 0;
    auto launch = [&](auto kernel, dim3 grid, auto... args) -> cudaError_t {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.gridDim = grid;
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.stream = s;
        cfg.attrs = attr;
        cfg.numAttrs = (m->pdl != 0 && n > 0) ? 1 : 0;
        n++;
        return cudaLaunchKernelEx(&cfg, kernel, args...);
    };
    for (int l = 0; l < m->L; l++) {
        const moe_b200_weights *w = m->layers[l].ffn;
        DCK(launch(qkv_kernel, dim3(ceil_div(D.qkv, 32)), A, l));
        DCK(launch(attn_kernel, dim3(D.nh, D.nchunk), A, l));
        DCK(launch(oproj_kernel, dim3(ceil_div(D.d, 32)), A, l));
        DCK(launch(upgate_kernel, dim3(w->k * ceil_div(w->F, kUnitsPerCta)), A, l));
        DCK(launch(down_kernel, dim3(ceil_div(D.d, down_cols(w->k))), A, l));
    }
    DCK(launch(lmhead_kernel, dim3(ceil_div(D.vocab, 32)), A));
    DCK(cudaGetLastError());
    m->launches = n;
    return MOE_B200_OK;
}

}  // namespace

// Build a decoder from host tensors in llm.c's layouts and the blocks' FFNs
// already on the device (ownership of every src.blocks[l].ffn passes to the
// decoder, also on failure).
int moe::decoder_build(const DecSrc &src, int max_seq, int flags, moe_b200_decoder **out) {
    *out = nullptr;
    auto drop_ffns = [&]() {
        for (const DecBlockSrc &b : src.blocks)
            if (b.ffn) moe_b200_weights_free(b.ffn);
    };
    const llmc_ModelConfig &c = src.cfg;
    const int d = c.d_model, nh = c.n_heads, nkv = c.n_kv_heads, hd = c.head_dim;
    const int L = (int)src.blocks.size();
    if (d <= 0 || d > kMaxD || nh <= 0 || nkv <= 0 || nh % nkv || hd <= 0 || hd > 128 ||
        hd % 32 || nh * hd > kMaxD || c.vocab_size <= 0 || L <= 0) {
        drop_ffns();
        return dfail(MOE_B200_E_INVALID, "unsupported model shape for the device decoder");
    }
    if ((flags & ~(MOE_B200_DECODER_STAGE_KERNELS | MOE_B200_DECODER_PERSISTENT)) ||
        ((flags & MOE_B200_DECODER_STAGE_KERNELS) && persistent(flags))) {
        drop_ffns();
        return dfail(MOE_B200_E_INVALID, "unknown or conflicting decoder flags");
    }
    if (max_seq <= 0 || max_seq > src.rope_len) {
        drop_ffns();
        return dfail(MOE_B200_E_INVALID, "max_seq exceeds the model's RoPE table");
    }
    moe_b200_decoder *m = new moe_b200_decoder();
    cudaGetDevice(&m->device);
    m->flags = flags;
    if (const char *p = std::getenv("MOE_B200_DECODER_PDL")) m->pdl = std::atoi(p);
    if (const char *p = std::getenv("MOE_B200_DECODER_EARLY")) m->early_mask = std::atoi(p);
    const char *stp = std::getenv("MOE_B200_DECODER_STAMPS");
    const bool want_stamps = stp && std::atoi(stp) != 0 && !persistent(flags);
    Dims &D = m->D;
    D.d = d; D.d_pad = round_up(d, 128); D.nh = nh; D.nkv = nkv; D.hd = hd; D.nq = nh * hd;
    D.kvd = nkv * hd; D.qkv = D.nq + 2 * D.kvd; D.vocab = c.vocab_size; D.max_seq = max_seq;
    D.nchunk = ceil_div(max_seq, CH); D.eps = c.rms_norm_eps; D.scale = 1.0f / sqrtf((float)hd);
    m->L = L;
    m->layers.resize(L);
    for (int l = 0; l < L; l++) m->layers[l].ffn = src.blocks[l].ffn;   // freed with m from here
    auto bail = [&](int r) { free_all(m); return r; };
#define DTRY(x)                      \
    do {                             \
        int r_ = (x);                \
        if (r_) return bail(r_);     \
    } while (0)
    DTRY(upload(&m->embed, src.embed, (size_t)D.vocab * d));
    DTRY(upload(&m->rms_final, src.rms_final, d));
    DTRY(upload(&m->lm_head, src.lm_head, (size_t)d * D.vocab));
    DTRY(upload(&m->rope_cos, src.rope_cos, (size_t)max_seq * (hd / 2)));
    DTRY(upload(&m->rope_sin, src.rope_sin, (size_t)max_seq * (hd / 2)));
    std::vector<LayerPtrs> lp(L);
    std::vector<float> qkv((size_t)d * D.qkv);
    for (int l = 0; l < L; l++) {
        const DecBlockSrc &b = src.blocks[l];
        DecLayer &ly = m->layers[l];
        if (!ly.ffn || ly.ffn->d != d) return bail(dfail(MOE_B200_E_INVALID, "block FFN shape"));
        DTRY(upload(&ly.rms_attn, b.rms_attn, d));
        DTRY(upload(&ly.rms_ffn, b.rms_ffn, d));
        for (int i = 0; i < d; i++) {           // [W_Q | W_K | W_V] columns per row
            float *row = qkv.data() + (size_t)i * D.qkv;
            std::memcpy(row, b.W_Q + (size_t)i * D.nq, D.nq * sizeof(float));
            std::memcpy(row + D.nq, b.W_K + (size_t)i * D.kvd, D.kvd * sizeof(float));
            std::memcpy(row + D.nq + D.kvd, b.W_V + (size_t)i * D.kvd, D.kvd * sizeof(float));
        }
        DTRY(upload(&ly.w_qkv, qkv.data(), qkv.size()));
        DTRY(upload(&ly.w_o, b.W_O, (size_t)D.nq * d));
        const moe_b200_weights *w = ly.ffn;
        if (w->k > kMaxTopK) return bail(dfail(MOE_B200_E_INVALID, "top_k too large"));
        lp[l] = LayerPtrs{ly.rms_attn, ly.rms_ffn, ly.w_qkv, ly.w_o, w->router, w->ug, w->dn,
                          w->E, w->k, w->F, w->F_pad};
        m->maxF_pad = m->maxF_pad > w->F_pad ? m->maxF_pad : w->F_pad;
    }
    const size_t cache = (size_t)m->L * max_seq * D.kvd;
    if (cudaMalloc(&m->d_layers, lp.size() * sizeof(LayerPtrs)) != cudaSuccess ||
        cudaMalloc(&m->kc, cache * 4) != cudaSuccess || cudaMalloc(&m->vc, cache * 4) != cudaSuccess ||
        cudaMalloc(&m->x, (size_t)d * 4) != cudaSuccess ||
        cudaMalloc(&m->q, (size_t)D.nq * 4) != cudaSuccess ||
        cudaMalloc(&m->part, (size_t)nh * D.nchunk * (hd + 2) * 4) != cudaSuccess ||
        cudaMalloc(&m->h, (size_t)kMaxTopK * m->maxF_pad * 4) != cudaSuccess ||
        cudaMalloc(&m->logits, (size_t)D.vocab * 4) != cudaSuccess ||
        cudaMalloc(&m->wts, kMaxTopK * 4) != cudaSuccess ||
        cudaMalloc(&m->ids, kMaxTopK * 4) != cudaSuccess ||
        cudaMalloc(&m->state, 2 * 4) != cudaSuccess ||
        cudaMalloc(&m->bar, 4) != cudaSuccess || cudaMalloc(&m->err, 4) != cudaSuccess ||
        cudaMalloc(&m->done, (size_t)(6 * L + 1) * sizeof(unsigned)) != cudaSuccess ||
        cudaMalloc(&m->trace, (size_t)m->L * 2 * d * 4) != cudaSuccess ||
        (want_stamps &&
         cudaMalloc(&m->stamps, (size_t)4 * (5 * L + 1) * sizeof(unsigned long long)) != cudaSuccess) ||
        cudaMallocHost(&m->h_token, 4) != cudaSuccess ||
        cudaHostAlloc(&m->h_err, 4, cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer((void **)&m->d_err_host, m->h_err, 0) != cudaSuccess) {
        cudaGetLastError();
        return bail(dfail(MOE_B200_E_NOMEM, "decoder buffers do not fit"));
    }
    *(volatile int *)m->h_err = 0;
    // h is zeroed once: the up/gate stage writes units [0, F), and the
    // padding units [F, F_pad) meet zero weight columns in the down stage
    if (cudaMemcpy(m->d_layers, lp.data(), lp.size() * sizeof(LayerPtrs),
                   cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(m->state, 0, 8) != cudaSuccess || cudaMemset(m->err, 0, 4) != cudaSuccess ||
        cudaMemset(m->h, 0, (size_t)kMaxTopK * m->maxF_pad * 4) != cudaSuccess ||
        cudaMemset(m->kc, 0, cache * 4) != cudaSuccess || cudaMemset(m->vc, 0, cache * 4) != cudaSuccess ||
        cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(dfail(MOE_B200_E_CUDA, "decoder set-up"));
    if (persistent(flags)) {
        // one CTA per SM, all co-resident (cooperative launch)
        int per_sm = 0, sms = moe::device_sms(m->device);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel, kThreads, 0) !=
                cudaSuccess || per_sm < 1 || sms < 1)
            return bail(dfail(MOE_B200_E_CUDA, "cooperative decode kernel cannot be resident"));
        m->grid = sms;
    }
    // the step as one graph
    if (cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
        return bail(dfail(MOE_B200_E_CUDA, "stream capture"));
    const int rc = enqueue_step(m);
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(m->stream, &g);
    if (rc) { if (g) cudaGraphDestroy(g); return bail(rc); }
    if (ce != cudaSuccess) return bail(dfail(MOE_B200_E_CUDA, cudaGetErrorString(ce)));
    m->graph = g;
    if (cudaGraphInstantiate(&m->exec, g, 0) != cudaSuccess)
        return bail(dfail(MOE_B200_E_CUDA, "graph instantiate"));
    *out = m;
    return MOE_B200_OK;
#undef DTRY
}

extern "C" int moe_b200_decoder_create(const void *model, int max_seq, int flags,
                                       moe_b200_decoder **out) {
    if (!model || !out) return dfail(MOE_B200_E_INVALID, "null argument");
    *out = nullptr;
    const llmc_Model *mp = static_cast<const llmc_Model *>(model);
    const llmc_ModelConfig &c = mp->cfg;
    if (mp->weights.n_layers <= 0 || mp->rope.head_dim != c.head_dim)
        return dfail(MOE_B200_E_INVALID, "unsupported model for the device decoder");
    int rc = moe_b200_init(-1);
    if (rc) return rc;
    const llmc_ModelWeights &W = mp->weights;
    DecSrc src;
    src.cfg = c;
    src.embed = W.embed.data;
    src.rms_final = W.rms_final;
    src.lm_head = W.lm_head.data;
    src.rope_cos = mp->rope.cos_table;
    src.rope_sin = mp->rope.sin_table;
    src.rope_len = mp->rope.max_seq_len;
    src.blocks.resize(W.n_layers);
    const int d = c.d_model, F = c.ffn_hidden;
    for (int l = 0; l < W.n_layers; l++) {
        const llmc_BlockWeights &b = W.blocks[l];
        DecBlockSrc &o = src.blocks[l];
        o.rms_attn = b.rms_attn; o.rms_ffn = b.rms_ffn;
        o.W_Q = b.attn.W_Q.data; o.W_K = b.attn.W_K.data; o.W_V = b.attn.W_V.data;
        o.W_O = b.attn.W_O.data;
        if (b.use_moe) {
            const llmc_MoEWeights &mw = b.moe;
            std::vector<const float *> g(mw.n_experts), u(mw.n_experts), dn(mw.n_experts);
            for (int e = 0; e < mw.n_experts; e++) {
                g[e] = mw.experts[e].W_gate.data;
                u[e] = mw.experts[e].W_up.data;
                dn[e] = mw.experts[e].W_down.data;
            }
            rc = moe_b200_weights_upload(mw.W_router.data, g.data(), u.data(), dn.data(), d, F,
                                         mw.n_experts, mw.top_k, &o.ffn);
        } else {                                   // dense FFN = one expert, weight 1
            std::vector<float> zr(d, 0.0f);
            const float *g = b.ffn.W_gate.data, *u = b.ffn.W_up.data, *dn = b.ffn.W_down.data;
            rc = moe_b200_weights_upload(zr.data(), &g, &u, &dn, d, F, 1, 1, &o.ffn);
        }
        if (rc) {
            for (int q = 0; q < l; q++) moe_b200_weights_free(src.blocks[q].ffn);
            return rc;
        }
    }
    return moe::decoder_build(src, max_seq, flags, out);
}

extern "C" int moe_b200_decoder_step(moe_b200_decoder *m, int token, float *logits) {
    if (!m) return dfail(MOE_B200_E_INVALID, "null decoder");
    if (token < 0 || token >= m->D.vocab) return dfail(MOE_B200_E_INVALID, "token out of range");
    if (m->pos >= m->D.max_seq) return dfail(MOE_B200_E_INVALID, "KV cache full");
    DCK(cudaSetDevice(m->device));
    *m->h_token = token;
    DCK(cudaMemcpyAsync(m->state, m->h_token, 4, cudaMemcpyHostToDevice, m->stream));
    DCK(cudaGraphLaunch(m->exec, m->stream));
    if (logits)
        DCK(cudaMemcpyAsync(logits, m->logits, (size_t)m->D.vocab * 4, cudaMemcpyDeviceToHost,
                            m->stream));
    DCK(cudaStreamSynchronize(m->stream));
    // the grid barrier's timeout flag comes back through mapped host memory,
    // written by the step's last kernel (no copy, no second synchronisation)
    if (*(volatile int *)m->h_err)
        return dfail(MOE_B200_E_TIMEOUT, "decode step: grid barrier wait ran out");
    m->pos++;
    return MOE_B200_OK;
}

extern "C" int moe_b200_decoder_set_pos(moe_b200_decoder *m, int pos) {
    if (!m) return dfail(MOE_B200_E_INVALID, "null decoder");
    if (pos < 0 || pos > m->pos) return dfail(MOE_B200_E_INVALID, "position beyond the cache");
    DCK(cudaSetDevice(m->device));
    DCK(cudaStreamSynchronize(m->stream));
    DCK(cudaMemcpy(m->state + 1, &pos, 4, cudaMemcpyHostToDevice));
    m->pos = pos;
    return MOE_B200_OK;
}

extern "C" int moe_b200_decoder_pos(const moe_b200_decoder *m) { return m ? m->pos : -1; }

extern "C" int moe_b200_decoder_launches(const moe_b200_decoder *m) { return m ? m->launches : 0; }

extern "C" int moe_b200_decoder_stage_times(moe_b200_decoder *m, double *out, int n) {
    if (!m || !out) return dfail(MOE_B200_E_INVALID, "null argument");
    if (!m->stamps) return dfail(MOE_B200_E_STATE, "stage timeline off (MOE_B200_DECODER_STAMPS=1)");
    const int ns = 5 * m->L + 1;
    if (n < 4 * ns) return dfail(MOE_B200_E_INVALID, "out holds fewer than 4 * (5 L + 1) values");
    if (m->pos == 0) return dfail(MOE_B200_E_STATE, "no step taken yet");
    DCK(cudaSetDevice(m->device));
    DCK(cudaStreamSynchronize(m->stream));
    std::vector<unsigned long long> h((size_t)4 * ns);
    DCK(cudaMemcpy(h.data(), m->stamps, h.size() * sizeof(unsigned long long),
                   cudaMemcpyDeviceToHost));
    const unsigned long long t0 = h[0];
    for (size_t i = 0; i < h.size(); i++) {
        const bool unset = (i % 4 < 2) ? h[i] == ~0ull : h[i] == 0ull;
        out[i] = unset ? -1.0 : (double)(long long)(h[i] - t0) * 1e-3;
    }
    return ns;
}

extern "C" int moe_b200_decoder_trace(moe_b200_decoder *m, int layer, float *x_norm,
                                      float *ffn_out) {
    if (!m) return dfail(MOE_B200_E_INVALID, "null decoder");
    if (layer < 0 || layer >= m->L) return dfail(MOE_B200_E_INVALID, "layer out of range");
    if (m->pos == 0) return dfail(MOE_B200_E_STATE, "no step taken yet");
    DCK(cudaSetDevice(m->device));
    DCK(cudaStreamSynchronize(m->stream));
    const size_t d = (size_t)m->D.d;
    if (x_norm)
        DCK(cudaMemcpy(x_norm, m->trace + (size_t)layer * 2 * d, d * 4, cudaMemcpyDeviceToHost));
    if (ffn_out)
        DCK(cudaMemcpy(ffn_out, m->trace + ((size_t)layer * 2 + 1) * d, d * 4,
                       cudaMemcpyDeviceToHost));
    return MOE_B200_OK;
}

extern "C" int moe_b200_decoder_destroy(moe_b200_decoder *m) {
    if (!m) return MOE_B200_OK;
    cudaSetDevice(m->device);
    cudaStreamSynchronize(m->stream);
    free_all(m);
    return MOE_B200_OK;
}
