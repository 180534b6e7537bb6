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
// they land.  X_big and X_small sit back to back in shared memory, so one
// N=128 MMA computes W·[X_big | X_small] and a second (N=64) adds
// W_small·X_big into the first half: 2 MMAs per K step.
//
// Warp roles (10 warps): 0 TMA producer, 1 TMEM allocator + MMA issuer,
// 2-5 converter (weight tile -> big in place + small beside it, then a
// proxy fence), 6-9 epilogue.  4-stage ring of 48 KB (W, W_small, X_big,
// X_small).  The tensor core's own accumulation truncates, and over a long
// K that alone costs ~1e-5, so each 32-wide K stage is multiplied into a
// FRESH 128×64 TMEM partial (an 8-slot ring) and the epilogue warps add the
// partials in registers with IEEE round-to-nearest — the long sum over K is
// ordinary fp32 arithmetic, as on the FFMA path.  Up/gate
// tiles hold 64 gate rows and the 64 matching up rows, so the SwiGLU runs
// in the epilogue: the warps holding the up half hand their values to the
// gate-half warps through shared memory, under an mbarrier pair.  Every
// wait is bounded; a timeout aborts the CTA cleanly.
#include "tc_common.cuh"

namespace moe {
namespace dec {

using namespace tc;

constexpr int MW = 128;                 // weight rows per tile (MMA M)
constexpr int NTOK = 64;                // tokens per tile (MMA N)
constexpr int BK = 32;                  // K per stage (128 bytes of fp32)
constexpr int STAGES = 4;
constexpr int A_BYTES = MW * BK * 4;    // 16 KB
constexpr int B_BYTES = NTOK * BK * 4;  // 8 KB
constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;   // W, W_small, X_big, X_small
constexpr int kThreads = 320;
constexpr int NSLOT = 4;                // TMEM ring of per-stage partial products
constexpr int SLOT_COLS = 2 * NTOK;     // [W·X_big + W_small·X_big | W·X_small]
constexpr uint32_t TMEM_COLS = NSLOT * SLOT_COLS;   // 512
constexpr int UPS_LD = NTOK + 1;        // padded row of the up hand-off buffer
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 64 * UPS_LD * 4 + 1024 + 512;

struct DecArgs {
    const int *plan;        // cnt | off | mt128 | mt64 (token tiles of 64 use mt64)
    int E;
    int num_kb;             // K / 32
    int NB;                 // weight blocks per expert (F_pad/64 or d_pad/128)
    int w_rows_per_expert;  // 2*F_pad (up/gate) or d_pad (down)
    float *h_big, *h_small; // up/gate outputs [rows × F_pad]
    int ldh;
    float *y;               // down output [rows × d_pad] (local)
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

template <bool UPGATE>
__global__ void __launch_bounds__(kThreads, 1)
dec_gemm(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmXb,
         const __grid_constant__ CUtensorMap tmXs, DecArgs a)
{
    constexpr uint32_t IDESC_N128 = idesc_tf32(MW, 2 * NTOK);
    constexpr uint32_t IDESC_N64 = idesc_tf32(MW, NTOK);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~static_cast<uintptr_t>(1023));
    float *ups = reinterpret_cast<float *>(smem + STAGES * STAGE_BYTES);   // [64][UPS_LD]
    uint64_t *bars = reinterpret_cast<uint64_t *>(ups + 64 * UPS_LD);
    uint64_t *full = bars, *conv = bars + STAGES, *empty = bars + 2 * STAGES;
    uint64_t *pfull = bars + 3 * STAGES, *pempty = pfull + NSLOT;
    uint64_t *ups_ready = pempty + NSLOT, *ups_free = ups_ready + 1, *fin = ups_free + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], 128);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < NSLOT; i++) {
            mbar_init(&pfull[i], 1);
            mbar_init(&pempty[i], 128);
        }
        mbar_init(ups_ready, 64);
        mbar_init(ups_free, 64);
        mbar_init(fin, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmXb)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmXs)) : "memory");
    }
    __syncwarp();
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int total = __ldg(a.plan + a.E + 2 * (a.E + 1) + a.E) * a.NB;   // mt64[E] * NB

    auto stage_ptr = [&](int s) { return smem + s * STAGE_BYTES; };
    auto set_abort = [&](int site) {
        if (!*abort_flag) {
            *abort_flag = 1;
            atomicExch(&a.status->timeout, site);
        }
    };

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int issued[STAGES];
            uint32_t issued_phase[STAGES];
            for (int s = 0; s < STAGES; s++) issued[s] = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                const DecTile t = dec_decode(tile, a.plan, a.E, a.NB);
                int wrow, wrow2 = 0;
                if (UPGATE) {
                    const int f0 = t.nb * 64;
                    wrow = t.e * a.w_rows_per_expert + (f0 / 128) * 256 + (f0 % 128);
                    wrow2 = wrow + 128;                   // the matching up rows
                } else {
                    wrow = t.e * a.w_rows_per_expert + t.nb * MW;
                }
                for (int kb = 0; kb < a.num_kb; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) { ok = false; break; }
                    uint8_t *sp = stage_ptr(stage);
                    mbar_expect_tx(&full[stage], A_BYTES + 2 * B_BYTES);
                    if (UPGATE) {
                        tma_load_2d(sp, &tmW, kb * BK, wrow, &full[stage]);
                        tma_load_2d(sp + A_BYTES / 2, &tmW, kb * BK, wrow2, &full[stage]);
                    } else {
                        tma_load_2d(sp, &tmW, kb * BK, wrow, &full[stage]);
                    }
                    tma_load_2d(sp + 2 * A_BYTES, &tmXb, kb * BK, t.row0, &full[stage]);
                    tma_load_2d(sp + 2 * A_BYTES + B_BYTES, &tmXs, kb * BK, t.row0, &full[stage]);
                    issued[stage] = 1;
                    issued_phase[stage] = phase;
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
            }
            if (!ok) set_abort(11);
            if (*abort_flag)
                for (int s = 0; s < STAGES; s++)
                    if (issued[s]) mbar_wait(&full[s], issued_phase[s], nullptr);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int stage = 0, slot = 0;
            uint32_t phase = 0, sphase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                for (int kb = 0; kb < a.num_kb; kb++) {
                    if (!mbar_wait(&conv[stage], phase, abort_flag)) { ok = false; break; }
                    if (!mbar_wait(&pempty[slot], sphase ^ 1, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(slot * SLOT_COLS);
                    const uint32_t w = smem_u32(stage_ptr(stage));
                    const uint32_t ws = w + A_BYTES, xb = w + 2 * A_BYTES;   // X_small follows X_big
#pragma unroll
                    for (int kk = 0; kk < BK / 8; kk++) {
                        const uint32_t o = kk * 32;
                        // cols 0..63: W·X_big, cols 64..127: W·X_small (X_big|X_small as one 128-row B)
                        mma_tf32(d, sw128_desc(w + o), sw128_desc(xb + o), IDESC_N128, kk ? 1u : 0u);
                        // cols 0..63 += W_small·X_big
                        mma_tf32(d, sw128_desc(ws + o), sw128_desc(xb + o), IDESC_N64, 1u);
                    }
                    mma_commit(&empty[stage]);     // smem stage free once these finish
                    mma_commit(&pfull[slot]);      // partial ready for the epilogue
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                    if (++slot == NSLOT) { slot = 0; sphase ^= 1; }
                }
            }
            if (!ok) set_abort(12);
            mma_commit(fin);
            mbar_wait(fin, 0, nullptr);
        }
    } else if (warp < 6) {
        // ---------------- converter (warps 2..5) ----------------
        const int ct = threadIdx.x - 64;          // 0..127
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
            for (int kb = 0; kb < a.num_kb; kb++) {
                if (!mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
                const float4 *w4 = reinterpret_cast<const float4 *>(stage_ptr(stage));
                float4 *s4 = reinterpret_cast<float4 *>(stage_ptr(stage) + A_BYTES);
#pragma unroll 4
                for (int i = ct; i < A_BYTES / 16; i += 128) {
                    const float4 v = w4[i];
                    s4[i] = make_float4(tf32_residual(v.x), tf32_residual(v.y),
                                        tf32_residual(v.z), tf32_residual(v.w));
                }
                fence_proxy_async_smem();   // st.shared -> visible to tcgen05.mma
                mbar_arrive(&conv[stage]);
                if (++stage == STAGES) { stage = 0; phase ^= 1; }
            }
        }
        if (!ok) set_abort(13);
    } else {
        // ---------------- epilogue (warps 6..9) ----------------
        const int q = warp & 3;                   // TMEM lane quarter
        int slot = 0;
        uint32_t sphase = 0, ups_phase = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
            const DecTile t = dec_decode(tile, a.plan, a.E, a.NB);
            float v[NTOK];
#pragma unroll
            for (int j = 0; j < NTOK; j++) v[j] = 0.0f;
            for (int kb = 0; kb < a.num_kb; kb++) {
                if (!mbar_wait(&pfull[slot], sphase, abort_flag)) { set_abort(14); ok = false; break; }
                tc_fence_after();
                const uint32_t taddr =
                    tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(slot * SLOT_COLS);
#pragma unroll
                for (int c = 0; c < NTOK; c += 32) {
                    float pb[32], ps[32];
                    tmem_ld32(taddr + c, pb);             // W·X_big + W_small·X_big
                    tmem_ld32(taddr + NTOK + c, ps);      // W·X_small
#pragma unroll
                    for (int j = 0; j < 32; j++) v[c + j] = __fadd_rn(v[c + j], __fadd_rn(pb[j], ps[j]));
                }
                tc_fence_before();
                mbar_arrive(&pempty[slot]);
                if (++slot == NSLOT) { slot = 0; sphase ^= 1; }
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
                    const size_t col = (size_t)t.nb * 64 + f;
#pragma unroll
                    for (int j = 0; j < NTOK; j++) {
                        if (j >= t.ntok) break;
                        const float h = swiglu_ref(v[j], ups[f * UPS_LD + j]);
                        const size_t o = (size_t)(t.row0 + j) * a.ldh + col;
                        a.h_big[o] = h;
                        a.h_small[o] = tf32_residual(h);
                    }
                    mbar_arrive(ups_free);
                }
                ups_phase ^= 1;
            } else {
                const int jcol = t.nb * MW + q * 32 + lane;   // output column of y
#pragma unroll
                for (int j = 0; j < NTOK; j++) {
                    if (j >= t.ntok) break;
                    const int row = t.row0 + j;
                    float *dst;
                    if (a.ret != nullptr) {
                        const int2 rr = a.ret[row];
                        dst = a.y_ptrs[rr.x] + (size_t)rr.y * a.ldy;
                    } else {
                        dst = a.y + (size_t)row * a.ldy;
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
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
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
    cudaError_t e = cudaFuncSetAttribute(dec::dec_gemm<true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         dec::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(dec::dec_gemm<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                dec::SMEM_BYTES);
}

cudaError_t launch_split_tf32(float *big, float *small, size_t n, cudaStream_t s) {
    const size_t n4 = n / 4;
    const int blocks = (int)(ceil_div<size_t>(n4, 256) < 148 * 16 ? ceil_div<size_t>(n4, 256) : 148 * 16);
    dec::split_tf32_kernel<<<blocks > 0 ? blocks : 1, 256, 0, s>>>(
        reinterpret_cast<float4 *>(big), reinterpret_cast<float4 *>(small), n4);
    return cudaGetLastError();
}

static int dec_grid(int rows_bound, int E, int NB, int num_sms) {
    const int bound = (ceil_div(rows_bound, dec::NTOK) + E) * NB;
    return bound < num_sms ? (bound > 0 ? bound : 1) : num_sms;
}

cudaError_t launch_dec_upgate(const DecMaps &m, int d_pad, int F_pad, float *h_big, float *h_small,
                              const int *plan, int E, int rows_bound, int num_sms,
                              DeviceStatus *status, cudaStream_t s)
{
    dec::DecArgs a{};
    a.plan = plan; a.E = E; a.num_kb = d_pad / dec::BK; a.NB = F_pad / 64;
    a.w_rows_per_expert = 2 * F_pad; a.h_big = h_big; a.h_small = h_small; a.ldh = F_pad;
    a.status = status;
    dec::dec_gemm<true><<<dec_grid(rows_bound, E, a.NB, num_sms), dec::kThreads, dec::SMEM_BYTES, s>>>(
        m.tmW, m.tmXb, m.tmXs, a);
    return cudaGetLastError();
}

cudaError_t launch_dec_down(const DecMaps &m, int F_pad, int d_pad, float *y, const int *plan,
                            int E, int rows_bound, int num_sms, DeviceStatus *status,
                            cudaStream_t s, float *const *y_ptrs, const int2 *ret)
{
    dec::DecArgs a{};
    a.plan = plan; a.E = E; a.num_kb = F_pad / dec::BK; a.NB = d_pad / dec::MW;
    a.w_rows_per_expert = d_pad; a.y = y; a.ldy = d_pad; a.y_ptrs = y_ptrs; a.ret = ret;
    a.status = status;
    dec::dec_gemm<false><<<dec_grid(rows_bound, E, a.NB, num_sms), dec::kThreads, dec::SMEM_BYTES, s>>>(
        m.tmW, m.tmXb, m.tmXs, a);
    return cudaGetLastError();
}

}  // namespace moe
