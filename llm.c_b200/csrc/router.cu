// router.cu — K1-K3 of the MoE block: router logits x·W_router (+bias),
// row softmax, top-k selection and renormalisation, plus the per-tile
// expert histogram that starts the dispatch.
//
// Reference: llm.c src/transformer.c:299-337 (router, softmax, top-k,
// renormalisation) and src/matrix.c:529-586 (softmax_rows).
//
// One CTA owns kRouterTile = 64 tokens.  The logits are a skinny FP32 GEMM
// ([64 × d]·[d × E], E <= 128): FFMA with a TPT×EPT register tile per
// thread, K in chunks of 32 staged through shared memory, the next chunk
// prefetched into registers while the current one is multiplied.  FP32
// (not TF32) because routing must match the reference's fp32 logits to
// ~1e-6.  Then one thread per token runs the reference's softmax and
// selection arithmetic, so identical logits give bit-identical
// probabilities and identical ids, and one thread per expert counts the
// tile's tokens that chose it, recording each (token, rank)'s stable rank
// among them.
#include "kernels.cuh"

namespace moe {

namespace {

constexpr int TT = kRouterTile;   // 64 tokens per CTA
constexpr int DC = 32;            // K chunk
constexpr int XS = DC + 4;        // x tile row stride (floats), 16B aligned

template <int EB> struct RouterShape;
template <> struct RouterShape<8>   { static constexpr int TPT = 1, EPT = 2; };
template <> struct RouterShape<16>  { static constexpr int TPT = 1, EPT = 4; };
template <> struct RouterShape<32>  { static constexpr int TPT = 2, EPT = 4; };
template <> struct RouterShape<64>  { static constexpr int TPT = 4, EPT = 4; };
template <> struct RouterShape<128> { static constexpr int TPT = 4, EPT = 8; };

}  // namespace

template <int EB>
__global__ void __launch_bounds__(256)
router_topk_kernel(const float *__restrict__ x, int T, int d,
                   const float *__restrict__ w_router,   // [d×E]
                   const float *__restrict__ bias,       // [E] or null
                   int E, int k,
                   float *__restrict__ probs,            // [T×E]
                   int *__restrict__ ids,                // [T×k]
                   float *__restrict__ wts,              // [T×k]
                   int *__restrict__ loc,                // [T×k]
                   int *__restrict__ tile_cnt)           // [tiles×E]
{
    constexpr int TPT = RouterShape<EB>::TPT, EPT = RouterShape<EB>::EPT;
    constexpr int NTX = EB / EPT;                 // threads along experts
    static_assert((TT / TPT) * NTX == 256, "thread tile must cover 256 threads");
    constexpr int MAIN_FLOATS = TT * XS + DC * EB;
    constexpr int LG_FLOATS = TT * (EB + 1);
    __shared__ __align__(16) float smem[MAIN_FLOATS > LG_FLOATS ? MAIN_FLOATS : LG_FLOATS];
    __shared__ int sid[TT][kMaxTopK];
    __shared__ float swt[TT][kMaxTopK];
    float *xs = smem;                 // [TT][XS]
    float *ws = smem + TT * XS;       // [DC][EB]
    float *lg = smem;                 // [TT][EB+1] (after the main loop)

    const int tile = blockIdx.x;
    const int t0 = tile * TT;
    const int tid = threadIdx.x;
    const int tx = tid % NTX, ty = tid / NTX;
    const bool vec_x = (d & 3) == 0;

    float acc[TPT][EPT];
#pragma unroll
    for (int i = 0; i < TPT; i++)
#pragma unroll
        for (int j = 0; j < EPT; j++) acc[i][j] = 0.0f;

    // register staging of one chunk: x as float4 (2 per thread), W scalar
    constexpr int XV = TT * DC / 4 / 256;        // float4 of x per thread = 2
    constexpr int WN = DC * EB / 256;            // W floats per thread
    float4 xr[XV];
    float wr[WN];

    auto load_chunk = [&](int i0) {
#pragma unroll
        for (int q = 0; q < XV; q++) {
            const int idx = tid + q * 256;
            const int r = idx / (DC / 4), c4 = idx % (DC / 4);
            const int t = t0 + r, i = i0 + c4 * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t < T) {
                const float *p = x + (size_t)t * d + i;
                if (vec_x && i + 3 < d) {
                    v = __ldg(reinterpret_cast<const float4 *>(p));
                } else {
                    if (i + 0 < d) v.x = __ldg(p + 0);
                    if (i + 1 < d) v.y = __ldg(p + 1);
                    if (i + 2 < d) v.z = __ldg(p + 2);
                    if (i + 3 < d) v.w = __ldg(p + 3);
                }
            }
            xr[q] = v;
        }
#pragma unroll
        for (int q = 0; q < WN; q++) {
            const int idx = tid + q * 256;
            const int r = idx / EB, c = idx % EB;
            const int i = i0 + r;
            wr[q] = (i < d && c < E) ? __ldg(w_router + (size_t)i * E + c) : 0.0f;
        }
    };
    auto store_chunk = [&]() {
#pragma unroll
        for (int q = 0; q < XV; q++) {
            const int idx = tid + q * 256;
            const int r = idx / (DC / 4), c4 = idx % (DC / 4);
            *reinterpret_cast<float4 *>(xs + r * XS + c4 * 4) = xr[q];
        }
#pragma unroll
        for (int q = 0; q < WN; q++) ws[tid + q * 256] = wr[q];
    };

    load_chunk(0);
    for (int i0 = 0; i0 < d; i0 += DC) {
        __syncthreads();                 // previous chunk fully consumed
        store_chunk();
        __syncthreads();
        if (i0 + DC < d) load_chunk(i0 + DC);   // overlaps the FMAs below
#pragma unroll 8
        for (int c = 0; c < DC; c++) {
            float xv[TPT], wv[EPT];
#pragma unroll
            for (int i = 0; i < TPT; i++) xv[i] = xs[(ty * TPT + i) * XS + c];
            if constexpr (EPT % 4 == 0) {
#pragma unroll
                for (int j = 0; j < EPT; j += 4) {   // 16-byte aligned: EPT % 4 == 0
                    const float4 w4 = *reinterpret_cast<const float4 *>(ws + c * EB + tx * EPT + j);
                    wv[j] = w4.x; wv[j + 1] = w4.y; wv[j + 2] = w4.z; wv[j + 3] = w4.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < EPT; j += 2) {   // 8-byte aligned: EPT == 2
                    const float2 w2 = *reinterpret_cast<const float2 *>(ws + c * EB + tx * EPT + j);
                    wv[j] = w2.x; wv[j + 1] = w2.y;
                }
            }
#pragma unroll
            for (int i = 0; i < TPT; i++)
#pragma unroll
                for (int j = 0; j < EPT; j++) acc[i][j] = __fmaf_rn(xv[i], wv[j], acc[i][j]);
        }
    }
    __syncthreads();                     // xs/ws are reused as lg below
#pragma unroll
    for (int i = 0; i < TPT; i++)
#pragma unroll
        for (int j = 0; j < EPT; j++) {
            const int e = tx * EPT + j;
            if (e < E)
                lg[(ty * TPT + i) * (EB + 1) + e] =
                    bias ? __fadd_rn(acc[i][j], __ldg(bias + e)) : acc[i][j];
        }
    __syncthreads();

    if (tid < TT && t0 + tid < T) {
        float *row = lg + tid * (EB + 1);
        // softmax_rows, AVX2+FMA branch: 8-wide part then scalar tail.
        const int nv = E - E % 8;
        float mx = -1e38f;
        for (int e = 0; e < E; e++) mx = fmaxf(mx, row[e]);
        float lane[8];
#pragma unroll
        for (int l = 0; l < 8; l++) lane[l] = 0.0f;
        for (int e = 0; e < nv; e++) {
            const float ex = exp_ref(__fsub_rn(row[e], mx));
            row[e] = ex;
            lane[e & 7] = __fadd_rn(lane[e & 7], ex);
        }
        const float a0 = __fadd_rn(lane[0], lane[4]), a1 = __fadd_rn(lane[1], lane[5]);
        const float a2 = __fadd_rn(lane[2], lane[6]), a3 = __fadd_rn(lane[3], lane[7]);
        float sum = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
        for (int e = nv; e < E; e++) {
            row[e] = expf(__fsub_rn(row[e], mx));
            sum = __fadd_rn(sum, row[e]);
        }
        const float inv = __fdiv_rn(1.0f, sum);
        for (int e = 0; e < nv; e++) row[e] = __fmul_rn(row[e], inv);
        for (int e = nv; e < E; e++) row[e] = __fdiv_rn(row[e], sum);

        // top-k (src/transformer.c:318-332): k passes, strict '>', best = -1,
        // best_e = 0, e ascending, already-chosen experts skipped.
        int sel[kMaxTopK];
        for (int r = 0; r < k; r++) {
            float best = -1.0f;
            int best_e = 0;
            for (int e = 0; e < E; e++) {
                bool taken = false;
                for (int q = 0; q < r; q++) taken |= (sel[q] == e);
                if (!taken && row[e] > best) { best = row[e]; best_e = e; }
            }
            sel[r] = best_e;
        }
        // renormalisation (src/transformer.c:334-337,350)
        float s = 0.0f;
        for (int r = 0; r < k; r++) s = __fadd_rn(s, row[sel[r]]);
        const float winv = (s > 1e-9f) ? __fdiv_rn(1.0f, s) : 0.0f;
        for (int r = 0; r < k; r++) {
            sid[tid][r] = sel[r];
            swt[tid][r] = __fmul_rn(row[sel[r]], winv);
        }
    }
    __syncthreads();

    // coalesced tile writes (rows of the tile are contiguous in memory)
    const int nt = min(TT, T - t0);
    for (int q = tid; q < nt * E; q += 256) {
        const int r = q / E, c = q % E;
        probs[(size_t)t0 * E + q] = lg[r * (EB + 1) + c];
    }
    for (int q = tid; q < nt * k; q += 256) {
        const int r = q / k, c = q % k;
        ids[(size_t)t0 * k + q] = sid[r][c];
        wts[(size_t)t0 * k + q] = swt[r][c];
    }
    // per-expert tile histogram and stable local ranks (token order)
    for (int e = tid; e < E; e += 256) {
        int c = 0;
        for (int r = 0; r < nt; r++)
            for (int q = 0; q < k; q++)
                if (sid[r][q] == e) loc[(size_t)(t0 + r) * k + q] = c++;
        tile_cnt[(size_t)tile * E + e] = c;
    }
}

cudaError_t launch_router(const float *x, int T, int d, const float *w_router,
                          const float *bias, int E, int k, float *probs, int *ids,
                          float *wts, int *loc, int *tile_cnt, cudaStream_t s)
{
    const int tiles = ceil_div(T, TT);
    if (E <= 8)
        router_topk_kernel<8><<<tiles, 256, 0, s>>>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt);
    else if (E <= 16)
        router_topk_kernel<16><<<tiles, 256, 0, s>>>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt);
    else if (E <= 32)
        router_topk_kernel<32><<<tiles, 256, 0, s>>>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt);
    else if (E <= 64)
        router_topk_kernel<64><<<tiles, 256, 0, s>>>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt);
    else
        router_topk_kernel<128><<<tiles, 256, 0, s>>>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt);
    return cudaGetLastError();
}

}  // namespace moe
