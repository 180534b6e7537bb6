// expert_decode.cu — weight-streaming expert GEMMs for decode-sized expert
// groups (a few to ~64 tokens per expert), at FP32 accuracy on tcgen05
// tensor cores (3xTF32).
//
// Reference arithmetic: llm.c src/transformer.c:157-165 (gate = x·W_gate,
// up = x·W_up, h = silu(gate)⊙up, y = h·W_down) per selected expert.
//
// Shape.  With few tokens per expert the GEMMs are weight-streaming: every
// weight byte is read once and used by a handful of tokens, so the kernel
// is HBM-bound if the tensor cores can keep FP32 accuracy.  Operands are
// swapped so the weights fill the 128-row MMA dimension (M) and the
// tokens the N dimension (64 per tile): D[weight rows × tokens] =
// W[rows × K] · X[tokens × K]^T, with no padding waste on the weight side.
//
// FP32 accuracy (tolerance 1e-5) from TF32 tensor cores: each operand is
// split into big = tf32(v) (the tensor core reads only the TF32 bits of an
// fp32 operand, i.e. truncates) and small = v - trunc_tf32(v) (exact in
// fp32), and D += W·X_big + W·X_small + W_small·X_big (the "3xTF32" split
// of Ootomo & Yokota 2022; the dropped W_small·X_small term is ~2^-20
// relative).  Token operands arrive with their small part precomputed in
// global memory (split kernel after the gather; the up/gate epilogue writes
// H's small part); weight tiles get theirs from a converter warpgroup as
// they land, written straight into tensor memory (one thread per weight
// row, tcgen05.st), where the MMA takes it as its A operand.  X_big and
// X_small sit back to back in shared memory, so one N=128 MMA computes
// W·[X_big | X_small] and a second (N=64, A from TMEM) adds W_small·X_big
// into the first half: 2 MMAs per 8-wide K slice.
//
// Pipelining.  Every tcgen05 instruction and every mbarrier wait costs the
// waiting thread tens of cycles, and the single MMA-issuing thread is the
// long pole: so it does one wait, the 8 MMAs and ONE commit per K step, in
// a loop unrolled over the ring period so that every ring position and
// descriptor offset is a constant.
//   * One commit per step arrives on done[step % R]; every consumer of
//     "the MMAs of step m have finished" (ring-slot reuse by the producers
//     and the converter, partial ready for the epilogue) waits on that
//     barrier at its own lag.  R is at least every ring depth, so no waiter
//     can fall a whole phase behind (no parity aliasing).
//   * The converter warps wait for everything else the step needs — the
//     weight tile, the token tile, a free TMEM partial slot, a free W_small
//     slot — convert, and signal ready[step % NS] once.
// Loads have long latencies under load (~2 us from HBM for the weights,
// ~0.7 us from L2 for the token rows), so the shared-memory rings are as
// deep as fits: weights W 8 × 16 KB (own producer warp, up to 8 steps
// ahead) and tokens X_big|X_small 4 × 16 KB (own producer warp); 10 weight
// and 2 token stages measured 1.6× slower (the token ring starves).  W_small
// lives in TMEM (8 slots of 32 columns), not in shared memory.
// Warp roles (11 warps): 0 weight producer, 10 token producer, 1 TMEM
// allocator + MMA issuer, 2-5 converter, 6-9 epilogue.  The tensor core's
// own accumulation truncates, and over a long K that alone costs ~1e-5, so
// every SPP K steps (SPP × 32 of K, 128 by default) are multiplied into a
// FRESH 128×128 TMEM partial (a 2-slot ring) and the epilogue warps add the
// partials in registers with IEEE round-to-nearest — the long sum over K is
// ordinary fp32 arithmetic, as on the FFMA path.  Up/gate tiles hold 64 gate rows and the 64
// matching up rows, so the SwiGLU runs in the epilogue: the warps holding
// the up half hand their values to the gate-half warps through shared
// memory, under an mbarrier pair.  Every wait is bounded; a timeout aborts
// the CTA cleanly.
#include "tc_common.cuh"

#include <cstdlib>

namespace moe {
namespace dec {

using namespace tc;

constexpr int MW = 128;                 // weight rows per tile (MMA M)
constexpr int NTOK = 64;                // tokens per tile (MMA N)
constexpr int BK = 32;                  // K per step (128 bytes of fp32)
constexpr int NW = 8;                   // weight ring stages
constexpr int NX = 4;                   // token-operand ring stages
constexpr int NS = 8;                   // W_small ring slots (TMEM, 32 columns each)
constexpr int NSLOT = 2;                // TMEM ring of per-step partial products
constexpr int R = 8;                    // done[] ring: >= NW, NX, NS, NSLOT
static_assert(R >= NW && R >= NX && R >= NS && R >= NSLOT, "done ring too short");
// the MMA loop is unrolled over R steps with every ring position a constant
static_assert(NW == R && NS == R && R % NX == 0 && R % NSLOT == 0, "ring sizes");
constexpr int A_BYTES = MW * BK * 4;    // 16 KB
constexpr int B_BYTES = NTOK * BK * 4;  // 8 KB
constexpr int X_BYTES = 2 * B_BYTES;    // X_big | X_small
constexpr int kThreads = 352;
// TMEM columns: partial slot s at s*128 ([W·X_big + W_small·X_big |
// W·X_small]), then the W_small operand slots
constexpr int SLOT_COLS = 2 * NTOK;
constexpr uint32_t WS_COL0 = NSLOT * SLOT_COLS;
constexpr uint32_t TMEM_COLS = 512;
static_assert(WS_COL0 + NS * BK <= TMEM_COLS, "TMEM columns");
constexpr int UPS_LD = NTOK + 1;        // padded row of the up hand-off buffer
constexpr int RING_BYTES = NW * A_BYTES + NX * X_BYTES;
constexpr int SMEM_BYTES = RING_BYTES + 64 * UPS_LD * 4 + 1024 + 512;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");

struct DecArgs {
    const int *plan;        // cnt | off | mt128 | mt64 | mt256 (token tiles of 64 use mt64)
    int E;
    int num_kb;             // K steps of 32 per tile (K / 32 / ksplit)
    int ksplit;             // down only: K halves per weight block (1 or 2), into y and y2
    int NB;                 // weight blocks per expert (F_pad/64 or d_pad/128)
    int w_rows_per_expert;  // 2*F_pad (up/gate) or d_pad (down)
    float *h_big, *h_small; // up/gate outputs [rows × F_pad]
    int ldh;
    float *y;               // down output [rows × d_pad] (local)
    float *y2;              // down output of the second K half (ksplit = 2)
    int ldy;
    float *const *y_ptrs;   // expert parallel: per-rank output bases
    const int2 *ret;        // expert parallel: (rank, row) of each slice row
    DeviceStatus *status;
};

struct DecTile {
    int e, tt, nb, row0, ntok;
};

__device__ __forceinline__ DecTile dec_decode(int tile, const int *plan, int E, int NB) {
    const int *cnt = plan, *off = plan + E, *mt64 = off + 2 * (E + 1);
    int lo = 0, hi = E;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(mt64 + mid) * NB <= tile) lo = mid; else hi = mid - 1;
    }
    DecTile t;
    t.e = lo;
    const int m0 = __ldg(mt64 + lo), mcount = __ldg(mt64 + lo + 1) - m0;
    const int l = tile - m0 * NB;
    t.nb = l / mcount;          // weight block outer: concurrent CTAs share it in L2
    t.tt = l - t.nb * mcount;
    t.row0 = __ldg(off + lo) + t.tt * NTOK;
    t.ntok = min(NTOK, __ldg(cnt + lo) - t.tt * NTOK);
    return t;
}

// Position in a ring of N entries: index and the parity of its current use
// (incremental: the hot loops do no division).
template <int N>
struct Ring {
    int i = 0;
    uint32_t ph = 0;
    __device__ __forceinline__ void next() {
        if (++i == N) { i = 0; ph ^= 1; }
    }
};

// Wait until the MMAs of step m have finished (done[m % R], its (m / R)-th
// phase).
__device__ __forceinline__ bool wait_done(uint64_t *done, int m, volatile int *abort_flag) {
    return mbar_wait(&done[m % R], (uint32_t)((m / R) & 1), abort_flag);
}

// PAIR: a 2-CTA cluster computes a 256-row weight block (128 rows per CTA)
// with tcgen05 cta_group::2 MMAs (M=256) issued by the rank-0 CTA, so each
// MMA instruction carries twice the weight bytes.  Each CTA streams its own
// weight rows and writes its own W_small into its own TMEM; the token
// operand B is split by columns between the CTAs (MMA1's N=128 =
// [X_big | X_small]: X_big in rank 0, X_small in rank 1; MMA2's N=64 =
// X_big: tokens 0..31 in rank 0, 32..63 in rank 1).  Both CTAs' converter
// warps arrive on rank 0's ready barrier (cluster-scope release); rank 0's
// single commit per step arrives on both CTAs' done rings (multicast
// commit, not a load).
// ONEPASS: plain TF32 (tolerance 2e-3, the prefill tensor-core path's
// numerics) instead of 3xTF32.  One N=64 MMA per 8-wide K slice (W·X with X
// rounded to nearest TF32 by the dispatch), accumulated in TMEM over the
// whole tile (two per-tile accumulators of 64 columns, alternating, so the
// epilogue of one tile overlaps the MMAs of the next); no W_small, no
// per-step partials.  The converter warps only gate the ring (weight tile,
// token tile, free accumulator) and the epilogue waits once per tile on
// accfull[tile % 2].  H is stored rounded to nearest TF32.
template <bool UPGATE, bool PAIR, bool ONEPASS, int SPP>
__global__ void __launch_bounds__(kThreads, 1)
dec_gemm(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmXb,
         const __grid_constant__ CUtensorMap tmXs, const __grid_constant__ CUtensorMap tmXb32,
         DecArgs a)
{
    static_assert(!(PAIR && ONEPASS), "ONEPASS runs on single CTAs");
    static_assert(R % (SPP * NSLOT) == 0, "a partial's steps sit in one unrolled ring period");
    constexpr int MM = PAIR ? 2 * MW : MW;                  // MMA M (weight rows per block)
    constexpr uint32_t IDESC_N128 = idesc_tf32(MM, 2 * NTOK);
    constexpr uint32_t IDESC_N64 = idesc_tf32(MM, NTOK);
    // token stage: single [X_big 8 KB | X_small 8 KB]; pair [MMA1 half 8 KB | MMA2 half 4 KB]
    constexpr int XB = PAIR ? B_BYTES + B_BYTES / 2 : X_BYTES;
    constexpr int XB2 = PAIR ? B_BYTES : 0;                 // offset of MMA2's B in a stage
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~static_cast<uintptr_t>(1023));
    uint8_t *sW = smem;                                  // [NW][16 KB]
    uint8_t *sX = sW + NW * A_BYTES;                     // [NX][XB]
    float *ups = reinterpret_cast<float *>(smem + RING_BYTES);   // [64][UPS_LD]
    uint64_t *bars = reinterpret_cast<uint64_t *>(ups + 64 * UPS_LD);
    uint64_t *wfull = bars, *xfull = wfull + NW, *ready = xfull + NX, *done = ready + NS;
    uint64_t *pempty = done + R;
    uint64_t *ups_ready = pempty + NSLOT, *ups_free = ups_ready + 1, *fin = ups_free + 1;
    uint64_t *accfull = fin + 1;                         // ONEPASS: [NSLOT] tile accumulators
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accfull + NSLOT);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_rank() : 0;
    const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;     // CTA or CTA pair
    const int nunits = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NW; s++) mbar_init(&wfull[s], 1);
        for (int s = 0; s < NX; s++) mbar_init(&xfull[s], 1);
        for (int s = 0; s < NS; s++) mbar_init(&ready[s], PAIR ? 256 : 128);
        for (int s = 0; s < R; s++) mbar_init(&done[s], 1);
        for (int s = 0; s < NSLOT; s++) mbar_init(&pempty[s], 128);
        for (int s = 0; s < NSLOT; s++) mbar_init(&accfull[s], 1);
        mbar_init(ups_ready, 64);
        mbar_init(ups_free, 64);
        mbar_init(fin, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmXb)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmXs)) : "memory");
        if (PAIR)
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmXb32))
                         : "memory");
    }
    __syncwarp();
    if (warp == 1) {
        if (PAIR) tmem_alloc_pair(tmem_slot, TMEM_COLS);
        else tmem_alloc(tmem_slot, TMEM_COLS);
    }
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync();            // the peer's barriers exist before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // mt64[E] * NB weight-block × token tiles, each split in ksplit K ranges
    const int total = __ldg(a.plan + a.E + 2 * (a.E + 1) + a.E) * a.NB * a.ksplit;
    // this unit's tiles are unit, unit + nunits, ...; K steps are numbered
    // across them
    const int my_tiles = unit < total ? (total - 1 - unit) / nunits + 1 : 0;
    const int nsteps = my_tiles * a.num_kb;

    auto set_abort = [&](int site) {
        if (!*abort_flag) {
            *abort_flag = 1;
            atomicExch(&a.status->timeout, site);
        }
    };

    if (warp == 0 || warp == 10) {
        // ---------------- TMA producers: weights (warp 0), tokens (warp 10) ----------------
        if (lane == 0) {
            const bool weights = warp == 0;
            const int depth = weights ? NW : NX;
            uint64_t *full = weights ? wfull : xfull;
            int n = 0;                                   // K step
            bool ok = true;
            for (int tile = unit; tile < total && ok; tile += nunits) {
                const DecTile t = dec_decode(tile / a.ksplit, a.plan, a.E, a.NB);
                const int kb0 = (tile % a.ksplit) * a.num_kb;
                int wrow, wrow2 = 0;
                if (UPGATE) {
                    // this CTA's 64 gate rows f0.. (and, 128 rows on, the matching up rows)
                    const int f0 = t.nb * (PAIR ? 128 : 64) + (int)rank * 64;
                    wrow = t.e * a.w_rows_per_expert + (f0 / 128) * 256 + (f0 % 128);
                    wrow2 = wrow + 128;
                } else {
                    wrow = t.e * a.w_rows_per_expert + t.nb * MM + (int)rank * MW;
                }
                for (int kb = 0; kb < a.num_kb; kb++, n++) {
                    // the stage's previous contents (step n - depth) are consumed
                    if (n >= depth && !wait_done(done, n - depth, abort_flag)) { ok = false; break; }
                    const int st = n % depth;
                    if (weights) {
                        uint8_t *dst = sW + st * A_BYTES;
                        mbar_expect_tx(&full[st], A_BYTES);
                        if (UPGATE) {
                            tma_load_2d(dst, &tmW, (kb0 + kb) * BK, wrow, &full[st]);
                            tma_load_2d(dst + A_BYTES / 2, &tmW, (kb0 + kb) * BK, wrow2, &full[st]);
                        } else {
                            tma_load_2d(dst, &tmW, (kb0 + kb) * BK, wrow, &full[st]);
                        }
                    } else if (ONEPASS) {
                        uint8_t *dst = sX + st * XB;
                        mbar_expect_tx(&full[st], B_BYTES);
                        tma_load_2d(dst, &tmXb, (kb0 + kb) * BK, t.row0, &full[st]);
                    } else if (!PAIR) {
                        uint8_t *dst = sX + st * XB;
                        mbar_expect_tx(&full[st], XB);
                        tma_load_2d(dst, &tmXb, (kb0 + kb) * BK, t.row0, &full[st]);
                        tma_load_2d(dst + B_BYTES, &tmXs, (kb0 + kb) * BK, t.row0, &full[st]);
                    } else {
                        // this CTA's column halves of the two B operands
                        uint8_t *dst = sX + st * XB;
                        mbar_expect_tx(&full[st], XB);
                        tma_load_2d(dst, rank ? &tmXs : &tmXb, (kb0 + kb) * BK, t.row0, &full[st]);
                        tma_load_2d(dst + XB2, &tmXb32, (kb0 + kb) * BK, t.row0 + (int)rank * 32, &full[st]);
                    }
                }
            }
            if (!ok) set_abort(weights ? 11 : 17);
            if (*abort_flag) {
                // loads still in flight (the last `depth` steps issued) land
                // before the CTA winds down
                for (int m = n - 1; m >= 0 && m >= n - depth; m--)
                    mbar_wait(&full[m % depth], (uint32_t)((m / depth) & 1), nullptr);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: one wait, 8 MMAs, one commit per step ----------------
        if (lane == 0 && rank == 0) {
            // descriptors of ring entry 0; entry j is +j*(bytes >> 4) in the
            // start-address field, and +2 there is the next 8-wide K slice
            const uint64_t dw0 = sw128_desc(smem_u32(sW));
            const uint64_t dx0 = sw128_desc(smem_u32(sX));   // single: X_small follows X_big
            const uint32_t ts0 = tmem_base + WS_COL0;
            bool ok = true;
            uint32_t ph = 0;                      // parity of ready[] in this round of R steps
            int kb = 0, tl = 0;                   // ONEPASS: K step in the tile, tile count
            for (int n0 = 0; n0 < nsteps && ok; n0 += R, ph ^= 1) {
#pragma unroll
                for (int j = 0; j < R; j++) {
                    if (n0 + j >= nsteps) break;
                    // ready: W_small written, and (checked by the converter)
                    // the weight and token tiles landed, the TMEM slot free.
                    if (!(PAIR ? mbar_wait_cluster(&ready[j], ph, abort_flag)
                               : mbar_wait(&ready[j], ph, abort_flag))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(((j / SPP) % NSLOT) * SLOT_COLS);
                    const uint64_t dw = dw0 + (uint64_t)(j * (A_BYTES >> 4));
                    const uint64_t dx = dx0 + (uint64_t)((j % NX) * (XB >> 4));
                    const uint64_t dx2 = dx + (uint64_t)(XB2 >> 4);      // MMA2's B
                    const uint32_t ts = ts0 + (uint32_t)(j * BK);
                    if constexpr (ONEPASS) {
                        const uint32_t dacc = tmem_base + (uint32_t)((tl & 1) * NTOK);
#pragma unroll
                        for (int kk = 0; kk < BK / 8; kk++)
                            mma_tf32(dacc, dw + 2 * kk, dx + 2 * kk, IDESC_N64, (kb | kk) ? 1u : 0u);
                        mma_commit(&done[j]);
                        if (++kb == a.num_kb) {           // the tile's accumulator is complete
                            mma_commit(&accfull[tl & 1]);
                            kb = 0;
                            tl++;
                        }
                    } else {
#pragma unroll
                        for (int kk = 0; kk < BK / 8; kk++) {
                            // cols 0..63: W·X_big, cols 64..127: W·X_small (X_big|X_small as one
                            // 128-row B), then cols 0..63 += W_small·X_big (A: 8 columns of
                            // W_small in TMEM)
                            const uint32_t acc = (kk || (j % SPP)) ? 1u : 0u;
                            if (PAIR) {
                                mma_tf32_pair(d, dw + 2 * kk, dx + 2 * kk, IDESC_N128, acc);
                                mma_tf32_ts_pair(d, ts + 8 * kk, dx2 + 2 * kk, IDESC_N64, 1u);
                            } else {
                                mma_tf32(d, dw + 2 * kk, dx + 2 * kk, IDESC_N128, acc);
                                mma_tf32_ts(d, ts + 8 * kk, dx2 + 2 * kk, IDESC_N64, 1u);
                            }
                        }
                        if (PAIR) mma_commit_pair(&done[j]);
                        else mma_commit(&done[j]);
                    }
                }
            }
            if (!ok) set_abort(12);
            if (PAIR) mma_commit_pair_local(fin);
            else mma_commit(fin);
            mbar_wait(fin, 0, nullptr);
        }
    } else if (warp < 6) {
        // ---------------- converter (warps 2..5) ----------------
        // waits for what the step needs, W stage -> W_small slot, one
        // arrive on ready.  Every warp needs the weight tile and the
        // W_small slot; the token tile and the TMEM slot, which only the
        // MMA needs, are vouched for by one warp each (their arrives on
        // ready carry the acquire on to the MMA thread).
        const int cw = warp - 2;                  // converter warp 0..3
        const int crow = (warp & 3) * 32 + lane;  // weight row = TMEM lane this thread writes
        const uint32_t ws_lane = tmem_base + ((uint32_t)((warp & 3) * 32) << 16);
        Ring<NW> rw;
        Ring<NS> rs;
        Ring<NX> rx;
        Ring<NSLOT> rp;
        Ring<R> rlag;                             // step n - NS of the done ring
        bool ok = true;
        if constexpr (ONEPASS) {
            // gate only: every warp waits for the weight tile (which bounds
            // how far ahead of the MMAs it runs), warp 2 for the token tile,
            // warp 3 at a tile's first step for its free accumulator
            int kb = 0;
            for (int n = 0; n < nsteps; n++) {
                if (!mbar_wait(&wfull[rw.i], rw.ph, abort_flag) ||
                    (cw == 2 && !mbar_wait(&xfull[rx.i], rx.ph, abort_flag)) ||
                    (cw == 3 && kb == 0 && !mbar_wait(&pempty[rp.i], rp.ph ^ 1, abort_flag))) {
                    ok = false;
                    break;
                }
                mbar_arrive(&ready[rs.i]);
                rw.next(); rs.next(); rx.next();
                if (++kb == a.num_kb) { kb = 0; rp.next(); }
            }
            if (!ok) set_abort(13);
        } else {
            for (int n = 0; n < nsteps; n++) {
                if (!mbar_wait(&wfull[rw.i], rw.ph, abort_flag) ||
                    (cw == 2 && !mbar_wait(&xfull[rx.i], rx.ph, abort_flag)) ||
                    (cw == 3 && n % SPP == 0 && !mbar_wait(&pempty[rp.i], rp.ph ^ 1, abort_flag))) {
                    ok = false;
                    break;
                }
                if (n >= NS) {                        // the W_small slot's last reader finished
                    if (!mbar_wait(&done[rlag.i], rlag.ph, abort_flag)) { ok = false; break; }
                    rlag.next();
                }
                // this thread's weight row: its 128 bytes, 16-byte chunks
                // permuted by the 128-byte swizzle (chunk c sits at c ^ (row % 8))
                const uint8_t *wrow = sW + rw.i * A_BYTES + crow * 128;
                float ws[BK];
    #pragma unroll
                for (int c = 0; c < BK / 4; c++) {
                    const float4 v = *reinterpret_cast<const float4 *>(wrow + ((c ^ (crow & 7)) << 4));
                    ws[4 * c + 0] = tf32_residual(v.x);
                    ws[4 * c + 1] = tf32_residual(v.y);
                    ws[4 * c + 2] = tf32_residual(v.z);
                    ws[4 * c + 3] = tf32_residual(v.w);
                }
                tmem_st32(ws_lane + WS_COL0 + (uint32_t)(rs.i * BK), ws);
                tc_fence_before();
                if (PAIR) mbar_arrive_cluster(mapa(smem_u32(&ready[rs.i]), 0));
                else mbar_arrive(&ready[rs.i]);
                rw.next(); rs.next(); rx.next();
                if (n % SPP == SPP - 1) rp.next();
            }
            if (!ok) set_abort(13);
        }
    } else {
        // ---------------- epilogue (warps 6..9) ----------------
        const int q = warp & 3;                   // TMEM lane quarter
        uint32_t ups_phase = 0;
        bool ok = true;
        int n = 0;
        const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
        for (int tile = unit; tile < total && ok; tile += nunits) {
            const DecTile t = dec_decode(tile / a.ksplit, a.plan, a.E, a.NB);
            float *ydst = (tile % a.ksplit) ? a.y2 : a.y;
            float v[NTOK];
#pragma unroll
            for (int j = 0; j < NTOK; j++) v[j] = 0.0f;
            if constexpr (ONEPASS) {
                const int slot = n & 1;           // n counts this CTA's tiles here
                if (!mbar_wait(&accfull[slot], (uint32_t)((n >> 1) & 1), abort_flag)) {
                    set_abort(14);
                    break;
                }
                tc_fence_after();
                tmem_ld64(lane_base + (uint32_t)(slot * NTOK), v);
                tc_fence_before();
                mbar_arrive(&pempty[slot]);
                n++;
            } else {
                for (int kb = 0; kb < a.num_kb; kb += SPP, n += SPP) {
                    // the partial of steps n .. n+SPP-1 is complete once the
                    // last of them has finished
                    if (!wait_done(done, n + SPP - 1, abort_flag)) { set_abort(14); ok = false; break; }
                    tc_fence_after();
                    const uint32_t slot = (uint32_t)((n / SPP) % NSLOT);
                    const uint32_t taddr = lane_base + slot * SLOT_COLS;
#pragma unroll
                    for (int c = 0; c < NTOK; c += 32) {
                        float pb[32], ps[32];
                        // W·X_big + W_small·X_big, and W·X_small
                        tmem_ld32x2(taddr + c, taddr + NTOK + c, pb, ps);
#pragma unroll
                        for (int j = 0; j < 32; j++) v[c + j] = __fadd_rn(v[c + j], __fadd_rn(pb[j], ps[j]));
                    }
                    tc_fence_before();
                    mbar_arrive(&pempty[slot]);
                }
            }
            if (!ok) break;
            if (UPGATE) {
                if (q >= 2) {                      // up rows: hand them to the gate warps
                    const int f = (q - 2) * 32 + lane;
                    if (!mbar_wait(ups_free, ups_phase ^ 1, abort_flag)) { set_abort(15); break; }
#pragma unroll
                    for (int j = 0; j < NTOK; j++) ups[f * UPS_LD + j] = v[j];
                    mbar_arrive(ups_ready);
                } else {                           // gate rows: SwiGLU and store h split
                    const int f = q * 32 + lane;
                    if (!mbar_wait(ups_ready, ups_phase, abort_flag)) { set_abort(16); break; }
                    const size_t col = (size_t)t.nb * (PAIR ? 128 : 64) + rank * 64 + f;
#pragma unroll
                    for (int j = 0; j < NTOK; j++) {
                        if (j >= t.ntok) break;
                        const float h = swiglu_ref(v[j], ups[f * UPS_LD + j]);
                        const size_t o = (size_t)(t.row0 + j) * a.ldh + col;
                        if (ONEPASS) {
                            a.h_big[o] = round_tf32(h);
                        } else {
                            a.h_big[o] = h;
                            a.h_small[o] = tf32_residual(h);
                        }
                    }
                    mbar_arrive(ups_free);
                }
                ups_phase ^= 1;
            } else {
                const int jcol = t.nb * MM + (int)rank * MW + q * 32 + lane;   // output column of y
#pragma unroll
                for (int j = 0; j < NTOK; j++) {
                    if (j >= t.ntok) break;
                    const int row = t.row0 + j;
                    float *dst;
                    if (a.ret != nullptr) {
                        const int2 rr = a.ret[row];
                        dst = a.y_ptrs[rr.x] + (size_t)rr.y * a.ldy;
                    } else {
                        dst = ydst + (size_t)row * a.ldy;
                    }
                    dst[jcol] = v[j];
                }
            }
        }
        if (!UPGATE && a.ret != nullptr) __threadfence_system();
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync();            // neither CTA leaves while the pair still works
    tc_fence_after();
    if (warp == 1) {
        if (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
        else tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// small = v - trunc_tf32(v) beside the unchanged v (the big part is v
// itself: the tensor core reads only its TF32 bits)
__global__ void split_tf32_kernel(const float4 *__restrict__ big, float4 *__restrict__ small,
                                  size_t n4)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
         i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = big[i];
        small[i] = make_float4(tf32_residual(v.x), tf32_residual(v.y), tf32_residual(v.z),
                               tf32_residual(v.w));
    }
}

}  // namespace dec

cudaError_t dec_set_attributes() {
    const void *fns[14] = {(const void *)dec::dec_gemm<true, false, false, 1>,
                           (const void *)dec::dec_gemm<false, false, false, 1>,
                           (const void *)dec::dec_gemm<true, false, false, 2>,
                           (const void *)dec::dec_gemm<false, false, false, 2>,
                           (const void *)dec::dec_gemm<true, false, false, 4>,
                           (const void *)dec::dec_gemm<false, false, false, 4>,
                           (const void *)dec::dec_gemm<true, true, false, 1>,
                           (const void *)dec::dec_gemm<false, true, false, 1>,
                           (const void *)dec::dec_gemm<true, true, false, 2>,
                           (const void *)dec::dec_gemm<false, true, false, 2>,
                           (const void *)dec::dec_gemm<true, true, false, 4>,
                           (const void *)dec::dec_gemm<false, true, false, 4>,
                           (const void *)dec::dec_gemm<true, false, true, 1>,
                           (const void *)dec::dec_gemm<false, false, true, 1>};
    for (const void *f : fns) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             dec::SMEM_BYTES);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// CTA pairs of the decode kernel that can be resident at once (0 if none)
int dec_max_pairs(int num_sms) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (num_sms / 2), 1, 1);
    cfg.blockDim = dim3(dec::kThreads, 1, 1);
    cfg.dynamicSmemBytes = dec::SMEM_BYTES;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, dec::dec_gemm<true, true, false, 1>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n < num_sms / 2 ? n : num_sms / 2;
}

cudaError_t launch_split_tf32(float *big, float *small, size_t n, cudaStream_t s) {
    const size_t n4 = n / 4;
    const int blocks = (int)(ceil_div<size_t>(n4, 256) < 148 * 16 ? ceil_div<size_t>(n4, 256) : 148 * 16);
    dec::split_tf32_kernel<<<blocks > 0 ? blocks : 1, 256, 0, s>>>(
        reinterpret_cast<float4 *>(big), reinterpret_cast<float4 *>(small), n4);
    return cudaGetLastError();
}

// persistent units (CTAs, or CTA pairs) for a grid of (token tiles × NB) tiles
static int dec_units(int rows_bound, int E, int NB, int cap) {
    const int bound = (ceil_div(rows_bound, dec::NTOK) + E) * NB;
    return bound < cap ? (bound > 0 ? bound : 1) : cap;
}

// K steps (of 32) per TMEM partial on the 3xTF32 path: 1, 2 or 4, the
// largest that divides the tile's steps and does not exceed
// MOE_B200_DEC_SPP (default 4).  Measured at c4 (one B200, 1965 MHz):
// up/gate 0.732 / 0.695 / 0.680 ms for 1 / 2 / 4 steps per partial, layer
// error against the oracle 1.4e-6 / 1.9e-6 / 2.7e-6 (3.1e-6 with d = 4096,
// d_ff = 14336): fewer partials cut the epilogue's tensor-memory reads, and
// each partial's in-tensor-core accumulation adds its truncation error.
static int dec_spp(int num_kb) {
    static const int want = [] {
        const char *p = std::getenv("MOE_B200_DEC_SPP");
        const int v = p ? std::atoi(p) : 4;
        return v >= 4 ? 4 : (v >= 2 ? 2 : 1);
    }();
    int spp = want;
    while (spp > 1 && num_kb % spp != 0) spp /= 2;
    return spp;
}

template <bool UPGATE>
static cudaError_t dec_launch(const DecMaps &m, const dec::DecArgs &a, int units, bool pair,
                              bool onepass, cudaStream_t s) {
    if (onepass) {
        dec::dec_gemm<UPGATE, false, true, 1><<<units, dec::kThreads, dec::SMEM_BYTES, s>>>(
            m.tmW, m.tmXb, m.tmXb, m.tmXb, a);
        return cudaGetLastError();
    }
    if (!pair) {
        switch (dec_spp(a.num_kb)) {
        case 4:
            dec::dec_gemm<UPGATE, false, false, 4><<<units, dec::kThreads, dec::SMEM_BYTES, s>>>(
                m.tmW, m.tmXb, m.tmXs, m.tmXb, a);
            break;
        case 2:
            dec::dec_gemm<UPGATE, false, false, 2><<<units, dec::kThreads, dec::SMEM_BYTES, s>>>(
                m.tmW, m.tmXb, m.tmXs, m.tmXb, a);
            break;
        default:
            dec::dec_gemm<UPGATE, false, false, 1><<<units, dec::kThreads, dec::SMEM_BYTES, s>>>(
                m.tmW, m.tmXb, m.tmXs, m.tmXb, a);
        }
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * units, 1, 1);
    cfg.blockDim = dim3(dec::kThreads, 1, 1);
    cfg.dynamicSmemBytes = dec::SMEM_BYTES;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (dec_spp(a.num_kb)) {
    case 4:
        return cudaLaunchKernelEx(&cfg, dec::dec_gemm<UPGATE, true, false, 4>, m.tmW, m.tmXb,
                                  m.tmXs, m.tmXb32, a);
    case 2:
        return cudaLaunchKernelEx(&cfg, dec::dec_gemm<UPGATE, true, false, 2>, m.tmW, m.tmXb,
                                  m.tmXs, m.tmXb32, a);
    default:
        return cudaLaunchKernelEx(&cfg, dec::dec_gemm<UPGATE, true, false, 1>, m.tmW, m.tmXb,
                                  m.tmXs, m.tmXb32, a);
    }
}

cudaError_t launch_dec_upgate(const DecMaps &m, int d_pad, int F_pad, float *h_big, float *h_small,
                              const int *plan, int E, int rows_bound, int num_sms, int max_pairs,
                              DeviceStatus *status, cudaStream_t s, bool onepass)
{
    const bool pair = max_pairs > 0 && !onepass;
    dec::DecArgs a{};
    a.plan = plan; a.E = E; a.num_kb = d_pad / dec::BK; a.ksplit = 1; a.NB = F_pad / (pair ? 128 : 64);
    a.w_rows_per_expert = 2 * F_pad; a.h_big = h_big; a.h_small = h_small; a.ldh = F_pad;
    a.status = status;
    return dec_launch<true>(m, a, dec_units(rows_bound, E, a.NB, pair ? max_pairs : num_sms), pair,
                            onepass, s);
}

// K halves for the down GEMM (1 or 2): halves when its weight blocks would
// fill the SMs in few, unevenly filled waves (and K splits evenly).
int dec_down_ksplit(int F_pad, int d_pad, int rows_bound, int E, int num_sms) {
    const int kb = F_pad / dec::BK;
    const int bound = (ceil_div(rows_bound, dec::NTOK) + E) * (d_pad / dec::MW);
    return (kb % 2 == 0 && bound < 8 * num_sms) ? 2 : 1;
}

cudaError_t launch_dec_down(const DecMaps &m, int F_pad, int d_pad, float *y, const int *plan,
                            int E, int rows_bound, int num_sms, int max_pairs, DeviceStatus *status,
                            cudaStream_t s, float *const *y_ptrs, const int2 *ret, float *y2,
                            bool onepass)
{
    const bool pair = max_pairs > 0 && d_pad % (2 * dec::MW) == 0 && !onepass;
    const int kb = F_pad / dec::BK;
    if (y2 != nullptr && (kb % 2 != 0 || ret != nullptr)) return cudaErrorInvalidValue;
    dec::DecArgs a{};
    a.plan = plan; a.E = E; a.NB = d_pad / (pair ? 2 * dec::MW : dec::MW);
    a.ksplit = y2 != nullptr ? 2 : 1;       // second K half written to y2
    a.num_kb = kb / a.ksplit;
    a.w_rows_per_expert = d_pad; a.y = y; a.y2 = y2; a.ldy = d_pad; a.y_ptrs = y_ptrs; a.ret = ret;
    a.status = status;
    return dec_launch<false>(m, a,
                             dec_units(rows_bound, E, a.NB * a.ksplit, pair ? max_pairs : num_sms),
                             pair, onepass, s);
}

}  // namespace moe
