// expert_tc.cu — tcgen05 TF32 grouped expert GEMMs for prefill-sized
// expert groups (llm.c src/transformer.c:157-165, batched over all tokens
// routed to each expert).
//
// One persistent CTA per SM walks a static round-robin list of output
// tiles (expert, 128-row m-tile, BN-column n-tile).  Warp roles:
//   warp 0      TMA producer: 128B-swizzled K-major tiles of activations
//               (128×32 fp32) and weights (BN×32 fp32) into a 4-stage
//               shared-memory ring (plain per-CTA loads)
//   warp 1      TMEM allocator and MMA issuer: tcgen05.mma kind::tf32,
//               M=128, N=BN, K=8, four per stage, accumulating in TMEM;
//               tcgen05.commit frees the smem stage / publishes the tile
//   warps 2..9  epilogue: tcgen05.ld 32x32b rows out of TMEM (two
//               accumulator buffers, so the epilogue of tile i overlaps
//               the main loop of tile i+1), fused SwiGLU for up/gate,
//               row-masked stores.  Two warps per TMEM lane quarter, each
//               on half of the tile's columns: the SwiGLU's dependent
//               chains (exponential, IEEE division) are latency-bound, and
//               with K short (d = 256..1024) the epilogue, not the MMAs,
//               sets the pace, so two warps per scheduler halve it.
// Tile order inside an expert is grouped by GM m-tiles so that the CTAs
// running together share a few weight tiles and a few activation row
// blocks in L2.
//
// Every mbarrier wait is bounded (kWaitNs of %globaltimer); a timeout
// sets an abort flag that all roles observe, records the site in the
// device status word, and the CTA drains its in-flight MMAs and TMA loads
// before it frees TMEM and exits.
#include "tc_common.cuh"

#include <cstdlib>

namespace moe {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 32;          // fp32 elements per K step = 128 bytes
constexpr int STAGES = 4;
// m-tiles per raster group (defaults; MOE_B200_TC_GROUP_M_UPGATE / _DOWN).
// Up/gate (K = d): a group's activation rows are small (16 × 128 rows × d),
// so 16 m-tiles halve the weight passes of the large experts against 8
// (c5: 114 passes of the gate/up weights per launch instead of 175, ~35 %
// less DRAM traffic, ~1 % faster, measured).  Down (K = F, rows 3.5× wider)
// keeps 8, so a group's rows stay well inside L2.
constexpr int GM = 8;
constexpr int GM_UPGATE = 16;
constexpr int EPI_WARPS = 8;   // two per TMEM lane quarter, each on half the columns
constexpr int kThreads = 64 + 32 * EPI_WARPS;
constexpr int A_BYTES = BM * BK * 4;
constexpr int EPI_FLOATS = 32 * 33;   // per epilogue warp: 32×32 chunk, padded rows

struct TileCoord {
    int e, ml, ni;
};

// tile -> (expert, m-tile within expert, n-tile); tiles of expert e are
// [mt128[e]*NT, mt128[e+1]*NT), grouped by gm m-tiles, n-tiles inside.
// Each group reads all of the expert's weight tiles once, so an expert of
// mt m-tiles streams its weights ceil(mt / gm) times.
__device__ __forceinline__ TileCoord decode_tile(int tile, const int *mt, int E, int NT, int gm) {
    int lo = 0, hi = E;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(mt + mid) * NT <= tile) lo = mid; else hi = mid - 1;
    }
    TileCoord c;
    c.e = lo;
    const int m0 = __ldg(mt + lo);
    const int mcount = __ldg(mt + lo + 1) - m0;
    const int l = tile - m0 * NT;
    const int g = l / (gm * NT);
    const int rem = l - g * gm * NT;
    const int gcount = min(gm, mcount - g * gm);
    c.ni = rem / gcount;
    c.ml = g * gm + (rem - c.ni * gcount);
    return c;
}

template <int BN, bool SWIGLU>
__global__ void __launch_bounds__(kThreads, 1)
tc_grouped_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const int *__restrict__ plan, int E, int num_kb, int b_rows_per_expert,
                int NT, float *__restrict__ out, int ldo, DeviceStatus *status,
                float *const *__restrict__ out_ptrs, const int2 *__restrict__ ret,
                float *__restrict__ gu_save, int gm)
{
    // gu_save (SWIGLU, optional): the gate and up pre-activations [rows × 2·ldo]
    // in the weights' row order (per 128 columns: 128 gate, then 128 up), for
    // the backward
    constexpr int B_BYTES = BN * BK * 4;
    constexpr uint32_t TMEM_COLS = 2 * BN;        // two accumulator buffers
    constexpr uint32_t IDESC = idesc_tf32(BM, BN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~static_cast<uintptr_t>(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_BYTES;
    float *sEpi = reinterpret_cast<float *>(sB + STAGES * B_BYTES);   // [EPI_WARPS][32][33]
    uint64_t *bars = reinterpret_cast<uint64_t *>(sEpi + EPI_WARPS * EPI_FLOATS);
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
        for (int a = 0; a < 2; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 32 * EPI_WARPS);
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

    const int *cnt = plan;
    const int *off = plan + E;
    const int *mt = off + E + 1;
    const int total = __ldg(mt + E) * NT;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0, issued_phase = 0;    // bit s: stage s loaded / its phase
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                const TileCoord c = decode_tile(tile, mt, E, NT, gm);
                const int a_row = __ldg(off + c.e) + c.ml * BM;
                const int b_row = c.e * b_rows_per_expert + c.ni * BN;
                for (int kb = 0; kb < num_kb; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) { ok = false; break; }
                    mbar_expect_tx(&full[stage], A_BYTES + B_BYTES);
                    tma_load_2d(sA + stage * A_BYTES, &tmA, kb * BK, a_row, &full[stage]);
                    tma_load_2d(sB + stage * B_BYTES, &tmB, kb * BK, b_row, &full[stage]);
                    issued |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
            }
            if (!ok || *abort_flag) {
                if (!*abort_flag) { *abort_flag = 1; atomicExch(&status->timeout, 1); }
                // drain TMA loads still in flight into this CTA's smem
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
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < num_kb; kb++) {
                    if (!mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 8; kk++)
                        mma_tf32(d_tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), IDESC,
                                 (kb | kk) ? 1u : 0u);
                    mma_commit(&empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
                mma_commit(&tfull[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            if (!ok && !*abort_flag) { *abort_flag = 1; atomicExch(&status->timeout, 2); }
            // all MMAs issued by this CTA complete before TMEM is released
            mma_commit(fin);
            mbar_wait(fin, 0, nullptr);
        }
    } else {
        // ---------------- epilogue (warps 2..9) ----------------
        const int q = warp & 3;                 // TMEM lane quarter of this warp
        const int ew = warp - 2;                // epilogue warp 0..7
        const int half = ew >> 2;               // which half of the columns
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
            const TileCoord c = decode_tile(tile, mt, E, NT, gm);
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) {
                if (!*abort_flag) { *abort_flag = 1; atomicExch(&status->timeout, 3); }
                break;
            }
            tc_fence_after();
            const int nvalid = __ldg(cnt + c.e) - c.ml * BM;
            const int row0 = __ldg(off + c.e) + c.ml * BM + q * 32;   // this warp's first row
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
            constexpr int NCOLS = SWIGLU ? BN / 2 : BN;
            const size_t ncol0 = (size_t)c.ni * NCOLS;
            // Stores go out row-contiguous: each 32×32 chunk is transposed
            // through shared memory so that 8 lanes write one row's 128
            // bytes and a warp instruction covers 4 whole row segments
            // (full sectors locally, full-size packets over NVLink).
            float *stage = sEpi + ew * EPI_FLOATS;
            const int sub = lane >> 3, c4 = (lane & 7) * 4;
            float *rowdst[8];
#pragma unroll
            for (int pass = 0; pass < 8; pass++) {
                const int r = pass * 4 + sub;
                rowdst[pass] = nullptr;
                if (q * 32 + r < nvalid) {
                    const size_t grow = (size_t)(row0 + r);
                    if (!SWIGLU && ret != nullptr) {
                        // expert-parallel: the row goes back to the rank that
                        // owns its token (peer memory over NVLink)
                        const int2 rr = ret[grow];
                        rowdst[pass] = out_ptrs[rr.x] + (size_t)rr.y * ldo + ncol0;
                    } else {
                        rowdst[pass] = out + grow * ldo + ncol0;
                    }
                }
            }
#pragma unroll 1
            for (int col = half * (NCOLS / 2); col < (half + 1) * (NCOLS / 2); col += 32) {
                float v[32];
                if (SWIGLU) {
                    float u[32];
                    tmem_ld32(taddr + col, v);
                    tmem_ld32(taddr + BN / 2 + col, u);
                    if (gu_save != nullptr && q * 32 + lane < nvalid) {
                        // this lane's row, 32 consecutive gate then up columns,
                        // stored straight from registers
                        float *gp = gu_save + (size_t)(row0 + lane) * 2 * ldo + (size_t)c.ni * 256 + col;
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            *reinterpret_cast<float4 *>(gp + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                            *reinterpret_cast<float4 *>(gp + 128 + j) =
                                make_float4(u[j], u[j + 1], u[j + 2], u[j + 3]);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 32; j++)   // h feeds the TF32 down GEMM: rounded
                        v[j] = round_tf32(swiglu_ref(v[j], u[j]));
                } else {
                    tmem_ld32(taddr + col, v);
                }
#pragma unroll
                for (int j = 0; j < 32; j++) stage[lane * 33 + j] = v[j];
                __syncwarp();
#pragma unroll
                for (int pass = 0; pass < 8; pass++) {
                    const int r = pass * 4 + sub;
                    if (rowdst[pass] != nullptr) {
                        const float *sr = stage + r * 33 + c4;
                        *reinterpret_cast<float4 *>(rowdst[pass] + col + c4) =
                            make_float4(sr[0], sr[1], sr[2], sr[3]);
                    }
                }
                __syncwarp();
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
        // peer stores must be visible before the rank-wide barrier that
        // follows this kernel on the stream
        if (ret != nullptr) __threadfence_system();
    }

    __syncwarp();          // lanes 1..31 of warps 0/1 wait for their lane 0
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
    return STAGES * (A_BYTES + BN * BK * 4) + EPI_WARPS * EPI_FLOATS * 4 + 1024 /*align slack*/ +
           256 /*barriers*/;
}

static_assert(smem_bytes<256>() <= 227 * 1024, "shared memory per CTA");

}  // namespace tc

cudaError_t tc_set_attributes() {
    cudaError_t e;
    e = cudaFuncSetAttribute(tc::tc_grouped_gemm<256, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, tc::smem_bytes<256>());
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(tc::tc_grouped_gemm<256, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, tc::smem_bytes<256>());
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(tc::tc_grouped_gemm<128, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, tc::smem_bytes<128>());
    return e;
}

static int tile_bound(int rows_bound, int E) { return ceil_div(rows_bound, tc::BM) + E; }

// m-tiles per raster group of the up/gate and of the down GEMM: the
// environment variables MOE_B200_TC_GROUP_M_UPGATE / _DOWN (1..64) when set,
// else tc::GM_UPGATE / tc::GM
static int group_m(bool upgate) {
    static const int gm[2] = {[] {
        const char *p = std::getenv("MOE_B200_TC_GROUP_M_DOWN");
        const int v = p ? std::atoi(p) : 0;
        return v >= 1 && v <= 64 ? v : tc::GM;
    }(), [] {
        const char *p = std::getenv("MOE_B200_TC_GROUP_M_UPGATE");
        const int v = p ? std::atoi(p) : 0;
        return v >= 1 && v <= 64 ? v : tc::GM_UPGATE;
    }()};
    return gm[upgate ? 1 : 0];
}

cudaError_t launch_tc_upgate(const TcGemm &g, int d_pad, int F_pad, float *h, const int *plan,
                             int E, int rows_bound, int num_sms, DeviceStatus *status,
                             cudaStream_t s, float *gu_save)
{
    const int NT = F_pad / 128;               // 256 weight rows (128 gate + 128 up) per tile
    const int bound = tile_bound(rows_bound, E) * NT;
    const int grid = max(1, min(num_sms, bound));
    tc::tc_grouped_gemm<256, true><<<grid, tc::kThreads, tc::smem_bytes<256>(), s>>>(
        g.tmA, g.tmB, plan, E, d_pad / tc::BK, 2 * F_pad, NT, h, F_pad, status, nullptr, nullptr,
        gu_save, group_m(true));
    return cudaGetLastError();
}

cudaError_t launch_tc_down(const TcGemm &g, int F_pad, int d_pad, int bn, float *y,
                           const int *plan, int E, int rows_bound, int num_sms,
                           DeviceStatus *status, cudaStream_t s, float *const *y_ptrs,
                           const int2 *ret)
{
    const int NT = d_pad / bn;
    const int bound = tile_bound(rows_bound, E) * NT;
    const int grid = max(1, min(num_sms, bound));
    if (bn == 256)
        tc::tc_grouped_gemm<256, false><<<grid, tc::kThreads, tc::smem_bytes<256>(), s>>>(
            g.tmA, g.tmB, plan, E, F_pad / tc::BK, d_pad, NT, y, d_pad, status, y_ptrs, ret,
            nullptr, group_m(false));
    else
        tc::tc_grouped_gemm<128, false><<<grid, tc::kThreads, tc::smem_bytes<128>(), s>>>(
            g.tmA, g.tmB, plan, E, F_pad / tc::BK, d_pad, NT, y, d_pad, status, y_ptrs, ret,
            nullptr, group_m(false));
    return cudaGetLastError();
}

}  // namespace moe
