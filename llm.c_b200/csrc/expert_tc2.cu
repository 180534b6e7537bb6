// expert_tc2.cu — 2-SM (cta_group::2) variant of the TF32 grouped expert
// GEMMs: a cluster of two CTAs on two SMs computes a 256×256 output tile.
//
// Why: at one SM per 128×256 tile the shared-memory port carries the TMA
// writes (48 KB per 32-wide K step) plus the MMA reads of the same bytes,
// about 1.5× what it can move while the tensor pipe runs flat out.  With a
// CTA pair, each SM stores and feeds only its own 128 rows of A and half of
// B (32 KB per K step) for the same MMA work per SM.
//
// Roles per CTA (192 threads): warp 0 TMA producer, warp 1 MMA issuer (the
// cluster's rank-0 CTA only) + TMEM allocator, warps 2-5 epilogue.
//   * Each CTA TMA-loads its own 128 A rows and its 128 B rows into its own
//     shared memory (plain per-CTA loads, no multicast); the loads' byte
//     counts complete on the rank-0 CTA's `full` barrier (cta_group::2
//     form), whose producer posts the expected bytes of both CTAs.
//   * The rank-0 CTA issues tcgen05.mma.cta_group::2 (M=256, N=256, K=8);
//     the hardware reads each CTA's half of A and B from that CTA's shared
//     memory and writes each CTA's 128 output rows into that CTA's TMEM.
//     tcgen05.commit with a two-CTA mask frees the stage in both CTAs and
//     publishes the accumulator to both epilogues.
//   * Each CTA's epilogue reads its own TMEM rows (SwiGLU on up/gate:
//     columns 0..127 are the gate half of B, 128..255 the up half) and
//     arrives on the rank-0 CTA's `tempty` barrier through its cluster
//     address.
// Every wait is bounded; both CTAs always reach the closing cluster barrier
// so neither leaves while the other (or the MMA) still uses its memory.
#include "tc_common.cuh"

namespace moe {
namespace tc2 {

using namespace tc;

constexpr int BM = 256;                  // output rows per pair tile (128 per CTA)
constexpr int BN = 256;                  // output columns per tile
constexpr int BK = 32;
constexpr int STAGES = 6;
constexpr int HALF_BYTES = 128 * BK * 4; // 16 KB: this CTA's A rows, or its B rows
constexpr int STAGE_BYTES = 2 * HALF_BYTES;
constexpr int GM = 4;                    // 256-row m-tiles per raster group
constexpr int kThreads = 192;
constexpr int EPI_FLOATS = 32 * 33;
constexpr uint32_t TMEM_COLS = 2 * BN;   // two accumulator buffers
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 4 * EPI_FLOATS * 4 + 1024 + 256;

// Load into this CTA's shared memory; the byte count completes on the
// barrier at `mbar_cluster` (the rank-0 CTA's).
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, int x, int y,
                                                 uint32_t mbar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar_cluster)
        : "memory");
}

struct PairTile {
    int e, ml, ni;
};

__device__ __forceinline__ PairTile decode_pair_tile(int tile, const int *mt, int E, int NT) {
    int lo = 0, hi = E;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(mt + mid) * NT <= tile) lo = mid; else hi = mid - 1;
    }
    PairTile c;
    c.e = lo;
    const int m0 = __ldg(mt + lo), mcount = __ldg(mt + lo + 1) - m0;
    const int l = tile - m0 * NT;
    const int g = l / (GM * NT);
    const int rem = l - g * GM * NT;
    const int gcount = min(GM, mcount - g * GM);
    c.ni = rem / gcount;
    c.ml = g * GM + (rem - c.ni * gcount);
    return c;
}

template <bool SWIGLU>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
tc_grouped_gemm_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const int *__restrict__ plan, int E, int num_kb, int b_rows_per_expert,
                     int NT, float *__restrict__ out, int ldo, DeviceStatus *status,
                     float *const *__restrict__ out_ptrs, const int2 *__restrict__ ret)
{
    constexpr uint32_t IDESC = idesc_tf32(BM, BN);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~static_cast<uintptr_t>(1023));
    float *sEpi = reinterpret_cast<float *>(smem + STAGES * STAGE_BYTES);
    uint64_t *bars = reinterpret_cast<uint64_t *>(sEpi + 4 * EPI_FLOATS);
    uint64_t *full = bars, *empty = bars + STAGES;
    uint64_t *tfull = bars + 2 * STAGES, *tempty = tfull + 2, *fin = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);      // rank 0's expect_tx arrive (+ both CTAs' bytes)
            mbar_init(&empty[s], 1);     // one multicast commit per use
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 256);  // both CTAs' epilogue threads (rank 0's barrier)
        }
        mbar_init(fin, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    }
    __syncwarp();
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();                      // peer barriers initialised before any remote use
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int *cnt = plan, *off = plan + E;
    const int *mt = off + 3 * (E + 1);   // mt256
    const int total = __ldg(mt + E) * NT;
    auto set_abort = [&](int site) {
        if (!*abort_flag) {
            *abort_flag = 1;
            atomicExch(&status->timeout, site);
        }
    };

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = pair; tile < total && ok; tile += npairs) {
                const PairTile c = decode_pair_tile(tile, mt, E, NT);
                const int a_row = __ldg(off + c.e) + c.ml * BM + (int)rank * 128;
                const int b_row = c.e * b_rows_per_expert + c.ni * BN + (int)rank * 128;
                for (int kb = 0; kb < num_kb; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) { ok = false; break; }
                    uint8_t *sp = smem + stage * STAGE_BYTES;
                    const uint32_t full0 = mapa(smem_u32(&full[stage]), 0);
                    if (rank == 0) mbar_expect_tx(&full[stage], 2 * STAGE_BYTES);
                    tma_load_2d_pair(sp, &tmA, kb * BK, a_row, full0);
                    tma_load_2d_pair(sp + HALF_BYTES, &tmB, kb * BK, b_row, full0);
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
            }
            if (!ok) set_abort(21);
            if (*abort_flag) {
                // loads in flight complete on the rank-0 barrier: give them
                // time to land before the CTA pair winds down
                const uint64_t t0 = globaltimer_ns();
                while (globaltimer_ns() - t0 < 2000000ULL) { }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (rank 0 only) ----------------
        if (lane == 0 && rank == 0) {
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = true;
            for (int tile = pair; tile < total && ok; tile += npairs) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < num_kb; kb++) {
                    if (!mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(smem + stage * STAGE_BYTES);
                    const uint32_t b0 = a0 + HALF_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 8; kk++)
                        mma_tf32_pair(d, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), IDESC,
                                      (kb | kk) ? 1u : 0u);
                    mma_commit_pair(&empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
                mma_commit_pair(&tfull[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            if (!ok) set_abort(22);
            mma_commit_pair_local(fin);
            mbar_wait(fin, 0, nullptr);
        }
    } else {
        // ---------------- epilogue (warps 2..5, both CTAs) ----------------
        const int q = warp & 3;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = pair; tile < total; tile += npairs) {
            const PairTile c = decode_pair_tile(tile, mt, E, NT);
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) { set_abort(23); break; }
            tc_fence_after();
            const int nvalid = __ldg(cnt + c.e) - c.ml * BM - (int)rank * 128;
            const int row0 = __ldg(off + c.e) + c.ml * BM + (int)rank * 128 + q * 32;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
            constexpr int NCOLS = SWIGLU ? BN / 2 : BN;
            const size_t ncol0 = (size_t)c.ni * NCOLS;
            float *stage = sEpi + q * EPI_FLOATS;
            const int sub = lane >> 3, c4 = (lane & 7) * 4;
            float *rowdst[8];
#pragma unroll
            for (int pass = 0; pass < 8; pass++) {
                const int r = pass * 4 + sub;
                rowdst[pass] = nullptr;
                if (q * 32 + r < nvalid) {
                    const size_t grow = (size_t)(row0 + r);
                    if (!SWIGLU && ret != nullptr) {
                        const int2 rr = ret[grow];
                        rowdst[pass] = out_ptrs[rr.x] + (size_t)rr.y * ldo + ncol0;
                    } else {
                        rowdst[pass] = out + grow * ldo + ncol0;
                    }
                }
            }
#pragma unroll 1
            for (int col = 0; col < NCOLS; col += 32) {
                float v[32];
                if (SWIGLU) {
                    float u[32];
                    tmem_ld32(taddr + col, v);
                    tmem_ld32(taddr + BN / 2 + col, u);
#pragma unroll
                    for (int j = 0; j < 32; j++) v[j] = round_tf32(swiglu_ref(v[j], u[j]));
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
            mbar_arrive_cluster(mapa(smem_u32(&tempty[acc]), 0));
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
        if (ret != nullptr) __threadfence_system();
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    cluster_sync();                      // neither CTA leaves while the pair still works
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(TMEM_COLS)
                     : "memory");
    }
}

}  // namespace tc2

cudaError_t tc2_set_attributes() {
    cudaError_t e = cudaFuncSetAttribute(tc2::tc_grouped_gemm_pair<true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         tc2::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(tc2::tc_grouped_gemm_pair<false>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, tc2::SMEM_BYTES);
}

// Pairs that can be resident at once (cluster placement can leave SMs
// unpaired); queried once per device.
int tc2_max_pairs(int num_sms) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (num_sms / 2), 1, 1);
    cfg.blockDim = dim3(tc2::kThreads, 1, 1);
    cfg.dynamicSmemBytes = tc2::SMEM_BYTES;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, tc2::tc_grouped_gemm_pair<true>, &cfg) != cudaSuccess ||
        n <= 0) {
        cudaGetLastError();
        return num_sms / 2;
    }
    return min(n, num_sms / 2);
}

static int pair_grid(int rows_bound, int E, int NT, int max_pairs) {
    const int tiles = (ceil_div(rows_bound, tc2::BM) + E) * NT;
    return 2 * max(1, min(max_pairs, tiles));
}

cudaError_t launch_tc2_upgate(const TcGemm &g, int d_pad, int F_pad, float *h, const int *plan,
                              int E, int rows_bound, int max_pairs, DeviceStatus *status,
                              cudaStream_t s)
{
    const int NT = F_pad / 128;               // 256 weight rows (128 gate + 128 up) per tile
    tc2::tc_grouped_gemm_pair<true><<<pair_grid(rows_bound, E, NT, max_pairs), tc2::kThreads,
                                       tc2::SMEM_BYTES, s>>>(
        g.tmA, g.tmB, plan, E, d_pad / tc2::BK, 2 * F_pad, NT, h, F_pad, status, nullptr, nullptr);
    return cudaGetLastError();
}

cudaError_t launch_tc2_down(const TcGemm &g, int F_pad, int d_pad, float *y, const int *plan,
                            int E, int rows_bound, int max_pairs, DeviceStatus *status,
                            cudaStream_t s, float *const *y_ptrs, const int2 *ret)
{
    const int NT = d_pad / tc2::BN;
    tc2::tc_grouped_gemm_pair<false><<<pair_grid(rows_bound, E, NT, max_pairs), tc2::kThreads,
                                        tc2::SMEM_BYTES, s>>>(
        g.tmA, g.tmB, plan, E, F_pad / tc2::BK, d_pad, NT, y, d_pad, status, y_ptrs, ret);
    return cudaGetLastError();
}

}  // namespace moe
