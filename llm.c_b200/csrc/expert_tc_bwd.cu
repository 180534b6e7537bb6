// expert_tc_bwd.cu — tcgen05 TF32 GEMMs of the MoE backward (the gradient of
// llm.c's expert FFN, src/transformer.c:157-165, batched per expert).
//
// Four products, all read in place from the forward's buffers and the
// packed expert weights (no transposed copies):
//   DH         dH[rows×F]  = dO[rows×d] · Wdᵀ      A K-major, B = dn[e][j][f]   MN-major
//              epilogue: SwiGLU backward, dG / dU written in the weights'
//              gate/up column order
//   DX         dX[rows×d]  = dGU[rows×2F] · Wguᵀ   A K-major, B = ug[e][c][j]   MN-major
//   WG_DOWN    dWd_e[F×d] += H_eᵀ · dO_e            A = H (MN-major), B = dO (MN-major)
//   WG_UPGATE  dWgu_e[d×2F] += X_eᵀ · dGU_e         A = X_perm, B = dGU (both MN-major)
// The weight-gradient products run K over expert e's rows, which start at a
// multiple of 32 in the backward's dispatch and are zero-padded to the next
// multiple, so every TMA box of a K block lies inside the expert.
//
// MN-major operands are loaded as 32-float (128-byte) chunks along M/N, each
// a box of 32 K rows: chunk c at c·4 KB of the stage.  For 32-bit (tf32)
// MN-major operands the tensor cores take only the 128-byte swizzle with
// 32-byte atoms (descriptor layout SWIZZLE_128B_BASE32B, TMA
// CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B): 4-row atoms of 512 bytes, so the
// descriptor's leading byte offset is the chunk stride and its stride byte
// offset the 512-byte atom stride, and the K=8 step of each MMA advances
// the start address by 8 rows = 1 KB.  (The 16-byte-atom SW128 layout of
// the K-major operands, read as MN-major, leaves the accumulator at zero.)
//
// Same warp roles, ring, double-buffered TMEM accumulators and bounded waits
// as the forward kernel (expert_tc.cu), with eight epilogue warps instead of
// four: the backward epilogues (SwiGLU backward, gradient read-modify-write)
// are heavier than the forward's and would otherwise bound the short-K tiles.
// The weight-gradient epilogue adds into the gradient buffers; each element
// belongs to one tile, so there are no atomics.
#include "tc_common.cuh"

namespace moe {
namespace tcb {

using namespace tc;   // TMEM, MMA, mbarrier and TMA helpers

constexpr int BM = 128;
constexpr int BK = 32;
constexpr int STAGES = 4;
constexpr int GM = 8;
constexpr int kThreads = 320;   // producer, MMA issuer, 8 epilogue warps
constexpr int A_BYTES = BM * BK * 4;
constexpr int CHUNK_BYTES = 32 * BK * 4;        // one 32-float MN chunk of 32 K rows
constexpr int EPI_FLOATS = 32 * 33;

enum Mode { DH = 0, DX = 1, WG_DOWN = 2, WG_UPGATE = 3 };

// MN-major, 128-byte swizzle with 32-byte atoms: 32-float chunks `lbo` bytes
// apart, 4-row atoms 512 bytes apart, descriptor version 1.
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t saddr, uint32_t lbo) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) |
           ((uint64_t)(512 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)1 << 61);
}

__host__ __device__ constexpr uint32_t idesc_majors(int M, int N, bool a_mn, bool b_mn) {
    return idesc_tf32(M, N) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16);
}

struct Args {
    const int *plan;
    int E;
    int num_kb;          // DH / DX: K blocks
    int b_k_rows;        // DH / DX: B rows per expert along K (d_pad or 2·F_pad)
    int NT, MT;          // n-tiles; m-tiles per expert (weight gradients)
    float *out;          // DH: dGU, DX: dX_perm
    int ldo;
    const float *gu;     // DH: the gate / up pre-activations [rows × 2·F_pad]
    float *g0, *g1;      // WG_DOWN: g0 = dW_down; WG_UPGATE: g0 = dW_gate, g1 = dW_up
    int d, F;
    DeviceStatus *status;
};

struct Tile {
    int e, mi, ni;
    int a_row;           // DH / DX: first activation row; WG: first K row
    int nkb;             // K blocks of this tile (0: nothing to do)
    int nvalid;          // DH / DX: valid rows from a_row
};

__device__ __forceinline__ int gate_col(int f) { return (f >> 7) * 256 + (f & 127); }

template <int MODE>
__device__ __forceinline__ Tile decode(int tile, const Args &a) {
    Tile t;
    const int E = a.E;
    const int *cnt = a.plan, *off = a.plan + E;
    if (MODE == DH || MODE == DX) {
        const int *mt = off + E + 1;
        const int NT = a.NT;
        int lo = 0, hi = E;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (__ldg(mt + mid) * NT <= tile) lo = mid; else hi = mid - 1;
        }
        t.e = lo;
        const int m0 = __ldg(mt + lo);
        const int mcount = __ldg(mt + lo + 1) - m0;
        const int l = tile - m0 * NT;
        const int g = l / (GM * NT);
        const int rem = l - g * GM * NT;
        const int gcount = min(GM, mcount - g * GM);
        t.ni = rem / gcount;
        t.mi = g * GM + (rem - t.ni * gcount);
        t.a_row = __ldg(off + t.e) + t.mi * BM;
        t.nvalid = __ldg(cnt + t.e) - t.mi * BM;
        t.nkb = a.num_kb;
    } else {
        // inside an expert the index of the smaller operand runs fastest, so
        // the CTAs running together share the tiles of the larger one:
        // WG_UPGATE's A (X_perm, d columns) is smaller than its B (dGU, 2F),
        // WG_DOWN's B (dO, d columns) smaller than its A (H, F)
        const int per = a.MT * a.NT;
        t.e = tile / per;
        const int rem = tile - t.e * per;
        if (MODE == WG_UPGATE) {
            t.ni = rem / a.MT;
            t.mi = rem - t.ni * a.MT;
        } else {
            t.mi = rem / a.NT;
            t.ni = rem - t.mi * a.NT;
        }
        t.a_row = __ldg(off + t.e);
        t.nkb = (__ldg(cnt + t.e) + BK - 1) / BK;
        t.nvalid = 0;
    }
    return t;
}

template <int MODE>
__device__ __forceinline__ int total_tiles(const Args &a) {
    if (MODE == DH || MODE == DX) return __ldg(a.plan + 2 * a.E + 1 + a.E) * a.NT;
    return a.E * a.MT * a.NT;
}

template <int BN, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
tc_bwd_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const Args a)
{
    constexpr bool A_MN = (MODE == WG_DOWN || MODE == WG_UPGATE);
    constexpr int B_BYTES = BN * BK * 4;
    constexpr int B_CHUNKS = BN / 32;
    constexpr uint32_t TMEM_COLS = 2 * BN;
    constexpr uint32_t IDESC = idesc_majors(BM, BN, A_MN, true);

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~static_cast<uintptr_t>(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_BYTES;
    float *sEpi = reinterpret_cast<float *>(sB + STAGES * B_BYTES);
    uint64_t *bars = reinterpret_cast<uint64_t *>(sEpi + 8 * EPI_FLOATS);
    uint64_t *full = bars;
    uint64_t *empty = bars + STAGES;
    uint64_t *tfull = bars + 2 * STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *fin = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 256);
        }
        mbar_init(fin, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    }
    __syncwarp();
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total = total_tiles<MODE>(a);

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0, issued_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                const Tile t = decode<MODE>(tile, a);
                for (int kb = 0; kb < t.nkb; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) { ok = false; break; }
                    mbar_expect_tx(&full[stage], A_BYTES + B_BYTES);
                    uint8_t *da = sA + stage * A_BYTES;
                    uint8_t *db = sB + stage * B_BYTES;
                    if (A_MN) {
#pragma unroll
                        for (int c = 0; c < BM / 32; c++)
                            tma_load_2d(da + c * CHUNK_BYTES, &tmA, t.mi * BM + c * 32,
                                        t.a_row + kb * BK, &full[stage]);
                    } else {
                        tma_load_2d(da, &tmA, kb * BK, t.a_row, &full[stage]);
                    }
                    const int b_k = (A_MN ? t.a_row : t.e * a.b_k_rows) + kb * BK;
#pragma unroll
                    for (int c = 0; c < B_CHUNKS; c++)
                        tma_load_2d(db + c * CHUNK_BYTES, &tmB, t.ni * BN + c * 32, b_k,
                                    &full[stage]);
                    issued |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
            }
            if (!ok || *abort_flag) {
                if (!*abort_flag) { *abort_flag = 1; atomicExch(&a.status->timeout, 11); }
                for (int s = 0; s < STAGES; s++)
                    if ((issued >> s) & 1u) mbar_wait(&full[s], (issued_phase >> s) & 1u, nullptr);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                const Tile t = decode<MODE>(tile, a);
                if (t.nkb == 0) continue;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < t.nkb; kb++) {
                    if (!mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 8; kk++) {
                        const uint64_t ad = A_MN ? sw128_mn_desc(a0 + kk * 1024, CHUNK_BYTES)
                                                 : sw128_desc(a0 + kk * 32);
                        mma_tf32(d_tmem, ad, sw128_mn_desc(b0 + kk * 1024, CHUNK_BYTES), IDESC,
                                 (kb | kk) ? 1u : 0u);
                    }
                    mma_commit(&empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
                mma_commit(&tfull[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            if (!ok && !*abort_flag) { *abort_flag = 1; atomicExch(&a.status->timeout, 12); }
            mma_commit(fin);
            mbar_wait(fin, 0, nullptr);
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        // two warps per TMEM lane quarter (a warp reaches lanes 32·(warp % 4)
        // and up), each taking half of the tile's columns
        const int ew = warp - 2;
        const int q = warp & 3;
        const int col_lo = (ew >> 2) * (BN / 2);
        int acc = 0;
        uint32_t acc_phase = 0;
        float *stage = sEpi + ew * EPI_FLOATS;
        const int sub = lane >> 3, c4 = (lane & 7) * 4;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
            const Tile t = decode<MODE>(tile, a);
            if (t.nkb == 0) continue;
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) {
                if (!*abort_flag) { *abort_flag = 1; atomicExch(&a.status->timeout, 13); }
                break;
            }
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
            const int mrow0 = q * 32;                 // this warp's first tile row
#pragma unroll 1
            for (int col = col_lo; col < col_lo + BN / 2; col += 32) {
                float v[32];
                tmem_ld32(taddr + col, v);
#pragma unroll
                for (int j = 0; j < 32; j++) stage[lane * 33 + j] = v[j];
                __syncwarp();
                if constexpr (MODE == DH) {
                    // all gate / up loads of the chunk first, then the math: the
                    // loads overlap instead of waiting behind each pass's stores
                    float4 g4[8], u4[8];
                    size_t base[8];
#pragma unroll
                    for (int pass = 0; pass < 8; pass++) {
                        const int r = pass * 4 + sub;
                        base[pass] = (size_t)(t.a_row + mrow0 + r) * a.ldo +
                                     gate_col(t.ni * BN + col + c4);
                        if (mrow0 + r < t.nvalid) {
                            g4[pass] = __ldg(reinterpret_cast<const float4 *>(a.gu + base[pass]));
                            u4[pass] = __ldg(reinterpret_cast<const float4 *>(a.gu + base[pass] + 128));
                        }
                    }
#pragma unroll
                    for (int pass = 0; pass < 8; pass++) {
                        const int r = pass * 4 + sub;
                        if (mrow0 + r >= t.nvalid) continue;
                        // h = silu(g)·u:  dU = dH·silu(g),  dG = dH·u·silu'(g)
                        const float *sr = stage + r * 33 + c4;
                        const float dh[4] = {sr[0], sr[1], sr[2], sr[3]};
                        const float gv[4] = {g4[pass].x, g4[pass].y, g4[pass].z, g4[pass].w};
                        const float uv[4] = {u4[pass].x, u4[pass].y, u4[pass].z, u4[pass].w};
                        float dg[4], du[4];
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_ref(-gv[j])));
                            const float silu = __fmul_rn(gv[j], sig);
                            const float ds = __fmul_rn(
                                sig, __fadd_rn(1.0f, __fmul_rn(gv[j], __fsub_rn(1.0f, sig))));
                            du[j] = round_tf32(__fmul_rn(dh[j], silu));
                            dg[j] = round_tf32(__fmul_rn(__fmul_rn(dh[j], uv[j]), ds));
                        }
                        *reinterpret_cast<float4 *>(a.out + base[pass]) =
                            make_float4(dg[0], dg[1], dg[2], dg[3]);
                        *reinterpret_cast<float4 *>(a.out + base[pass] + 128) =
                            make_float4(du[0], du[1], du[2], du[3]);
                    }
                } else if constexpr (MODE == DX) {
#pragma unroll
                    for (int pass = 0; pass < 8; pass++) {
                        const int r = pass * 4 + sub;       // row within this warp's 32
                        if (mrow0 + r >= t.nvalid) continue;
                        const float *sr = stage + r * 33 + c4;
                        const size_t row = (size_t)(t.a_row + mrow0 + r);
                        *reinterpret_cast<float4 *>(a.out + row * a.ldo + t.ni * BN + col + c4) =
                            make_float4(sr[0], sr[1], sr[2], sr[3]);
                    }
                } else {
                    // weight gradients: read-modify-write of 4 consecutive elements
                    // per lane and pass; all reads of the chunk are issued first
                    //   WG_DOWN    dW_down[e][f = m][j = n]          rows of d
                    //   WG_UPGATE  dW_gate / dW_up[e][j = m][f]      rows of F, n in the
                    //              weights' gate/up column order
                    const int rowlen = MODE == WG_DOWN ? a.d : a.F;
                    const int mlim = MODE == WG_DOWN ? a.F : a.d;
                    const int n = t.ni * BN + col + c4;
                    const int within = n & 255;
                    float *gbase = (MODE == WG_UPGATE && within >= 128) ? a.g1 : a.g0;
                    const int c0 = MODE == WG_DOWN ? n : (n >> 8) * 128 + (within & 127);
                    const int nv = max(0, min(4, rowlen - c0));        // valid columns
                    const bool vec = nv == 4 && (rowlen & 3) == 0;
                    float *dst[8];
                    float cur[8][4];
#pragma unroll
                    for (int pass = 0; pass < 8; pass++) {
                        const int m = t.mi * BM + mrow0 + pass * 4 + sub;   // gradient row
                        dst[pass] = (m < mlim && nv > 0)
                                        ? gbase + ((size_t)t.e * mlim + m) * rowlen + c0
                                        : nullptr;
                        if (dst[pass] != nullptr) {
                            if (vec) {
                                const float4 v = *reinterpret_cast<const float4 *>(dst[pass]);
                                cur[pass][0] = v.x; cur[pass][1] = v.y;
                                cur[pass][2] = v.z; cur[pass][3] = v.w;
                            } else {
#pragma unroll
                                for (int j = 0; j < 4; j++) cur[pass][j] = j < nv ? dst[pass][j] : 0.f;
                            }
                        }
                    }
#pragma unroll
                    for (int pass = 0; pass < 8; pass++) {
                        if (dst[pass] == nullptr) continue;
                        const float *sr = stage + (pass * 4 + sub) * 33 + c4;
                        float o[4];
#pragma unroll
                        for (int j = 0; j < 4; j++) o[j] = __fadd_rn(cur[pass][j], sr[j]);
                        if (vec) {
                            *reinterpret_cast<float4 *>(dst[pass]) = make_float4(o[0], o[1], o[2], o[3]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 4; j++)
                                if (j < nv) dst[pass][j] = o[j];
                        }
                    }
                }
                __syncwarp();
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(TMEM_COLS)
                     : "memory");
    }
}

template <int BN>
constexpr int smem_bytes() {
    return STAGES * (A_BYTES + BN * BK * 4) + 8 * EPI_FLOATS * 4 + 1024 + 256;
}
static_assert(smem_bytes<256>() <= 227 * 1024, "stage ring + epilogue staging exceed 227 KB");

template <int BN, int MODE>
static cudaError_t launch(const CUtensorMap &tmA, const CUtensorMap &tmB, const Args &a, int tiles,
                          int num_sms, cudaStream_t s) {
    // the attribute belongs to the current device: set it on every launch
    cudaError_t e = cudaFuncSetAttribute(tc_bwd_gemm<BN, MODE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem_bytes<BN>());
    if (e != cudaSuccess) return e;
    const int grid = max(1, min(num_sms, tiles));
    tc_bwd_gemm<BN, MODE><<<grid, kThreads, smem_bytes<BN>(), s>>>(tmA, tmB, a);
    return cudaGetLastError();
}

}  // namespace tcb

static int bwd_bn(int n) { return n % 256 == 0 ? 256 : 128; }

cudaError_t launch_tc_bwd(const TcBwd &g, cudaStream_t s) {
    using namespace tcb;
    Args a{};
    a.plan = g.plan;
    a.E = g.E;
    a.d = g.d;
    a.F = g.F;
    a.status = g.status;
    const int mtiles = ceil_div(g.rows_bound, BM) + g.E;
    cudaError_t e;
    // dH = dO·Wdᵀ (N = F_pad), SwiGLU backward into dGU
    {
        const int bn = bwd_bn(g.F_pad);
        a.num_kb = g.d_pad / BK;
        a.b_k_rows = g.d_pad;
        a.NT = g.F_pad / bn;
        a.out = g.dgu;
        a.ldo = 2 * g.F_pad;
        a.gu = g.gu;
        e = bn == 256 ? launch<256, DH>(g.tm_dO_k, g.tm_dn_mn, a, mtiles * a.NT, g.num_sms, s)
                      : launch<128, DH>(g.tm_dO_k, g.tm_dn_mn, a, mtiles * a.NT, g.num_sms, s);
        if (e != cudaSuccess) return e;
    }
    // the alignment rows of dGU are read by the weight-gradient GEMM
    if ((e = launch_zero_pad_rows(g.dgu, 2 * g.F_pad, g.plan, g.E, s)) != cudaSuccess) return e;
    // dW_down[e] += H_eᵀ·dO_e  (M = F_pad, N = d_pad)
    {
        const int bn = bwd_bn(g.d_pad);
        a.MT = g.F_pad / BM;
        a.NT = g.d_pad / bn;
        a.g0 = g.g_down;
        a.g1 = nullptr;
        const int tiles = g.E * a.MT * a.NT;
        e = bn == 256 ? launch<256, WG_DOWN>(g.tm_h_mn, g.tm_dO_mn, a, tiles, g.num_sms, s)
                      : launch<128, WG_DOWN>(g.tm_h_mn, g.tm_dO_mn, a, tiles, g.num_sms, s);
        if (e != cudaSuccess) return e;
    }
    // dW_gate / dW_up[e] += X_eᵀ·dGU_e  (M = d_pad, N = 2·F_pad)
    {
        a.MT = g.d_pad / BM;
        a.NT = 2 * g.F_pad / 256;
        a.g0 = g.g_gate;
        a.g1 = g.g_up;
        e = launch<256, WG_UPGATE>(g.tm_x_mn, g.tm_dgu_mn, a, g.E * a.MT * a.NT, g.num_sms, s);
        if (e != cudaSuccess) return e;
    }
    // dX_perm = dGU·Wguᵀ  (N = d_pad)
    {
        const int bn = bwd_bn(g.d_pad);
        a.num_kb = 2 * g.F_pad / BK;
        a.b_k_rows = 2 * g.F_pad;
        a.NT = g.d_pad / bn;
        a.out = g.dxp;
        a.ldo = g.d_pad;
        a.gu = nullptr;
        e = bn == 256 ? launch<256, DX>(g.tm_dgu_k, g.tm_ug_mn, a, mtiles * a.NT, g.num_sms, s)
                      : launch<128, DX>(g.tm_dgu_k, g.tm_ug_mn, a, mtiles * a.NT, g.num_sms, s);
    }
    return e;
}

}  // namespace moe
