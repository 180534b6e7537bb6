// expert_ffma.cu — FP32 (FFMA) grouped expert GEMMs.
//
// The exact-arithmetic path of the expert FFN (llm.c src/transformer.c:
// 157-165: gate = x·W_gate, up = x·W_up, h = silu(gate)⊙up, y = h·W_down),
// used when the caller asks for FP32 accuracy (MOE_B200_PATH_FP32, 1e-5)
// and for expert groups too small for a 128-row tensor-core tile.
//
// Tiles: 64 permuted rows × 64 output columns, K in steps of 16; one CTA of
// 256 threads, each thread a 4×4 register block (×2 for gate and up).
// Expert e's rows are the contiguous slice [off[e], off[e]+cnt[e]) of the
// permuted activations; blockIdx.x walks the 64-row m-tiles of all experts
// (plan mt64 prefix), blockIdx.y the output columns.
#include "kernels.cuh"

namespace moe {

namespace {

constexpr int BM = 64, BN = 64, BK = 16;

__device__ __forceinline__ bool decode_mtile(const int *plan, int E, int bx, int &e,
                                             int &row0, int &nrows) {
    const int *cnt = plan, *off = plan + E, *mt64 = off + 2 * (E + 1);
    if (bx >= mt64[E]) return false;
    int lo = 0, hi = E;
    while (lo < hi) {                       // last e with mt64[e] <= bx
        const int mid = (lo + hi + 1) >> 1;
        if (mt64[mid] <= bx) lo = mid; else hi = mid - 1;
    }
    e = lo;
    const int mt = bx - mt64[e];
    row0 = off[e] + mt * BM;
    nrows = min(BM, cnt[e] - mt * BM);
    return true;
}

// Load a BM×BK (or BN×BK) K-major tile as [BK][64] (transposed) into smem.
__device__ __forceinline__ void load_tile_t(float (*dst)[BM + 4], const float *src, int ld,
                                            int row0, int nrows, int k0) {
    const int tid = threadIdx.x;
    const int r = tid >> 2, kq = (tid & 3) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < nrows) v = __ldg(reinterpret_cast<const float4 *>(src + (size_t)(row0 + r) * ld + k0 + kq));
    dst[kq + 0][r] = v.x;
    dst[kq + 1][r] = v.y;
    dst[kq + 2][r] = v.z;
    dst[kq + 3][r] = v.w;
}

}  // namespace

template <bool SWIGLU>
__global__ void __launch_bounds__(256)
ffma_grouped_kernel(const float *__restrict__ A, int K,
                    const float *__restrict__ B, int b_rows_per_expert,
                    float *__restrict__ C, int ldc, const int *__restrict__ plan, int E,
                    float *const *__restrict__ out_ptrs, const int2 *__restrict__ ret,
                    float *__restrict__ gu_save)
{
    // gu_save (SWIGLU, optional): the gate and up pre-activations [rows × 2·ldc]
    // in the weights' row order (per 128 columns: 128 gate, then 128 up), for
    // the backward
    __shared__ __align__(16) float As[BK][BM + 4];
    __shared__ __align__(16) float Bs[BK][BN + 4];
    __shared__ __align__(16) float Us[BK][BN + 4];

    int e, row0, nrows;
    if (!decode_mtile(plan, E, blockIdx.x, e, row0, nrows)) return;
    const int n0 = blockIdx.y * BN;                      // output column base
    int brow, urow = 0;
    if (SWIGLU) {
        // gate rows of f-block (n0/128) then the matching up rows 128 below
        brow = e * b_rows_per_expert + (n0 / 128) * 256 + (n0 % 128);
        urow = brow + 128;
    } else {
        brow = e * b_rows_per_expert + n0;
    }

    const int tid = threadIdx.x;
    const int ty = tid >> 4, tx = tid & 15;
    float acc[4][4], accu[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) { acc[i][j] = 0.f; accu[i][j] = 0.f; }

    for (int k0 = 0; k0 < K; k0 += BK) {
        load_tile_t(As, A, K, row0, nrows, k0);
        load_tile_t(Bs, B, K, brow, BN, k0);
        if (SWIGLU) load_tile_t(Us, B, K, urow, BN, k0);
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            const float4 a = *reinterpret_cast<const float4 *>(&As[kk][ty * 4]);
            const float4 b = *reinterpret_cast<const float4 *>(&Bs[kk][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w};
            const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
            if (SWIGLU) {
                const float4 u = *reinterpret_cast<const float4 *>(&Us[kk][tx * 4]);
                const float uv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) accu[i][j] = __fmaf_rn(av[i], uv[j], accu[i][j]);
            }
        }
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = ty * 4 + i;
        if (r >= nrows) continue;
        float4 o;
        if (SWIGLU) {
            o.x = swiglu_ref(acc[i][0], accu[i][0]);
            o.y = swiglu_ref(acc[i][1], accu[i][1]);
            o.z = swiglu_ref(acc[i][2], accu[i][2]);
            o.w = swiglu_ref(acc[i][3], accu[i][3]);
        } else {
            o = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
        }
        if (SWIGLU && gu_save != nullptr) {
            float *g = gu_save + (size_t)(row0 + r) * 2 * ldc + (n0 / 128) * 256 + (n0 % 128) + tx * 4;
            *reinterpret_cast<float4 *>(g) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
            *reinterpret_cast<float4 *>(g + 128) =
                make_float4(accu[i][0], accu[i][1], accu[i][2], accu[i][3]);
        }
        float *dst = C + (size_t)(row0 + r) * ldc;
        if (!SWIGLU && ret != nullptr) {          // expert-parallel return to the owner
            const int2 rr = ret[row0 + r];
            dst = out_ptrs[rr.x] + (size_t)rr.y * ldc;
        }
        *reinterpret_cast<float4 *>(dst + n0 + tx * 4) = o;
    }
    if (!SWIGLU && ret != nullptr) __threadfence_system();
}

static int mtile_bound(int rows_bound, int E, int bm) { return ceil_div(rows_bound, bm) + E; }

cudaError_t launch_ffma_upgate(const float *x_perm, int d_pad, const float *w_ug, int F_pad,
                               float *h, const int *plan, int E, int rows_bound, cudaStream_t s,
                               float *gu_save)
{
    dim3 grid(mtile_bound(rows_bound, E, BM), F_pad / BN);
    ffma_grouped_kernel<true><<<grid, 256, 0, s>>>(x_perm, d_pad, w_ug, 2 * F_pad, h, F_pad, plan, E,
                                                   nullptr, nullptr, gu_save);
    return cudaGetLastError();
}

cudaError_t launch_ffma_down(const float *h, int F_pad, const float *w_d, int d_pad,
                             float *y, const int *plan, int E, int rows_bound, cudaStream_t s,
                             float *const *y_ptrs, const int2 *ret)
{
    dim3 grid(mtile_bound(rows_bound, E, BM), d_pad / BN);
    ffma_grouped_kernel<false><<<grid, 256, 0, s>>>(h, F_pad, w_d, d_pad, y, d_pad, plan, E,
                                                    y_ptrs, ret, nullptr);
    return cudaGetLastError();
}

}  // namespace moe
