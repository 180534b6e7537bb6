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

// FFMA dot products of this CTA's 64 tokens with W_router over K range
// [d0, d1): acc[i][j] += x[t0 + ty*TPT + i][k] * W[k][tx*EPT + j].
template <int EB>
__device__ __forceinline__ void router_dot(const float *__restrict__ x, int T, int d,
                                           const float *__restrict__ w_router, int E, int t0,
                                           int d0, int d1, float *smem,
                                           float (&acc)[RouterShape<EB>::TPT][RouterShape<EB>::EPT])
{
    constexpr int TPT = RouterShape<EB>::TPT, EPT = RouterShape<EB>::EPT;
    constexpr int NTX = EB / EPT;
    float *xs = smem;                 // [TT][XS]
    float *ws = smem + TT * XS;       // [DC][EB]
    const int tid = threadIdx.x;
    const int tx = tid % NTX, ty = tid / NTX;
    const bool vec_x = (d & 3) == 0;
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
                if (vec_x && i + 3 < d1) {
                    v = __ldg(reinterpret_cast<const float4 *>(p));
                } else {
                    if (i + 0 < d1) v.x = __ldg(p + 0);
                    if (i + 1 < d1) v.y = __ldg(p + 1);
                    if (i + 2 < d1) v.z = __ldg(p + 2);
                    if (i + 3 < d1) v.w = __ldg(p + 3);
                }
            }
            xr[q] = v;
        }
#pragma unroll
        for (int q = 0; q < WN; q++) {
            const int idx = tid + q * 256;
            const int r = idx / EB, c = idx % EB;
            const int i = i0 + r;
            wr[q] = (i < d1 && c < E) ? __ldg(w_router + (size_t)i * E + c) : 0.0f;
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

    load_chunk(d0);
    for (int i0 = d0; i0 < d1; i0 += DC) {
        __syncthreads();                 // previous chunk fully consumed
        store_chunk();
        __syncthreads();
        if (i0 + DC < d1) load_chunk(i0 + DC);   // overlaps the FMAs below
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
    __syncthreads();                     // smem is reused by the caller
}

// Softmax, top-k, renormalisation, tile writes and the tile histogram for
// the logits in lg [TT][EB+1] (bias already added).
template <int EB>
__device__ __forceinline__ void router_tail(float *lg, int T, int E, int k, int tile,
                                            float *__restrict__ probs, int *__restrict__ ids,
                                            float *__restrict__ wts, int *__restrict__ loc,
                                            int *__restrict__ tile_cnt,
                                            int (*sid)[kMaxTopK], float (*swt)[kMaxTopK])
{
    const int tid = threadIdx.x;
    const int t0 = tile * TT;
    if (tid < TT && t0 + tid < T) {
        int sel[kMaxTopK];
        float wsel[kMaxTopK];
        route_token(lg + tid * (EB + 1), E, k, sel, wsel);
#pragma unroll
        for (int r = 0; r < kMaxTopK; r++) {
            if (r < k) {
                sid[tid][r] = sel[r];
                swt[tid][r] = wsel[r];
            }
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
    // per-expert tile histogram and stable local ranks (slot order: token,
    // then rank): a warp per expert, 32 slots per ballot, ranks by prefix
    // popcount
    const int warp = tid >> 5, lane = tid & 31;
    const int nslot = nt * k;
    for (int e = warp; e < E; e += 8) {
        int c = 0;
        for (int s0 = 0; s0 < nslot; s0 += 32) {
            const int sl = s0 + lane;
            const bool hit = sl < nslot && sid[sl / k][sl % k] == e;
            const unsigned m = __ballot_sync(0xffffffffu, hit);
            if (hit) loc[(size_t)t0 * k + sl] = c + __popc(m & ((1u << lane) - 1u));
            c += __popc(m);
        }
        if (lane == 0) tile_cnt[(size_t)tile * E + e] = c;
    }
}

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
    constexpr int NTX = EB / EPT;
    static_assert((TT / TPT) * NTX == 256, "thread tile must cover 256 threads");
    constexpr int MAIN_FLOATS = TT * XS + DC * EB;
    constexpr int LG_FLOATS = TT * (EB + 1);
    __shared__ __align__(16) float smem[MAIN_FLOATS > LG_FLOATS ? MAIN_FLOATS : LG_FLOATS];
    __shared__ int sid[TT][kMaxTopK];
    __shared__ float swt[TT][kMaxTopK];

    const int tile = blockIdx.x;
    const int tx = threadIdx.x % NTX, ty = threadIdx.x / NTX;
    float acc[TPT][EPT];
#pragma unroll
    for (int i = 0; i < TPT; i++)
#pragma unroll
        for (int j = 0; j < EPT; j++) acc[i][j] = 0.0f;
    router_dot<EB>(x, T, d, w_router, E, tile * TT, 0, d, smem, acc);
    float *lg = smem;                 // [TT][EB+1]
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
    router_tail<EB>(lg, T, E, k, tile, probs, ids, wts, loc, tile_cnt, sid, swt);
}

// Small T: the K range is split over blockIdx.y so that enough CTAs run;
// each writes its partial logits, and router_reduce_topk_kernel sums the
// splits in a fixed order (deterministic) before the same tail.
template <int EB>
__global__ void __launch_bounds__(256)
router_partial_kernel(const float *__restrict__ x, int T, int d,
                      const float *__restrict__ w_router, int E, int dsplit,
                      float *__restrict__ part)             // [nsplit][T][E]
{
    constexpr int TPT = RouterShape<EB>::TPT, EPT = RouterShape<EB>::EPT;
    constexpr int NTX = EB / EPT;
    __shared__ __align__(16) float smem[TT * XS + DC * EB];
    const int tile = blockIdx.x, split = blockIdx.y;
    const int d0 = split * dsplit, d1 = min(d, d0 + dsplit);
    const int tx = threadIdx.x % NTX, ty = threadIdx.x / NTX;
    float acc[TPT][EPT];
#pragma unroll
    for (int i = 0; i < TPT; i++)
#pragma unroll
        for (int j = 0; j < EPT; j++) acc[i][j] = 0.0f;
    router_dot<EB>(x, T, d, w_router, E, tile * TT, d0, d1, smem, acc);
    float *dst = part + (size_t)split * T * E;
#pragma unroll
    for (int i = 0; i < TPT; i++) {
        const int t = tile * TT + ty * TPT + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < EPT; j++) {
            const int e = tx * EPT + j;
            if (e < E) dst[(size_t)t * E + e] = acc[i][j];
        }
    }
}

template <int EB>
__global__ void __launch_bounds__(256)
router_reduce_topk_kernel(const float *__restrict__ part, int nsplit, int T,
                          const float *__restrict__ bias, int E, int k,
                          float *__restrict__ probs, int *__restrict__ ids,
                          float *__restrict__ wts, int *__restrict__ loc,
                          int *__restrict__ tile_cnt)
{
    __shared__ __align__(16) float lg[TT * (EB + 1)];
    __shared__ int sid[TT][kMaxTopK];
    __shared__ float swt[TT][kMaxTopK];
    const int tile = blockIdx.x, t0 = tile * TT;
    // Each thread owns VPT logits (q = tid + 256 i) and sums their splits in
    // ascending order.  The loads of SB splits of all VPT logits are issued
    // together (about 64 in flight per thread), so the L2 round trips
    // overlap instead of running one logit after another.
    constexpr int VPT = (TT * EB + 255) / 256;
    constexpr int SB = VPT >= 32 ? 2 : (VPT >= 16 ? 4 : 8);
    const size_t stride = (size_t)T * E;
    int off[VPT];                                // logit index t·E + e, -1 if none
    float v[VPT];
#pragma unroll
    for (int i = 0; i < VPT; i++) {
        const int q = threadIdx.x + 256 * i, r = q / E, e = q % E;
        off[i] = (q < TT * E && t0 + r < T) ? (t0 + r) * E + e : -1;
        v[i] = 0.0f;
    }
    for (int sp = 0; sp < nsplit; sp += SB) {
        float a[VPT][SB];
#pragma unroll
        for (int i = 0; i < VPT; i++)
#pragma unroll
            for (int j = 0; j < SB; j++)
                a[i][j] = (off[i] >= 0 && sp + j < nsplit)
                              ? __ldg(part + (size_t)(sp + j) * stride + off[i]) : 0.0f;
#pragma unroll
        for (int i = 0; i < VPT; i++)
#pragma unroll
            for (int j = 0; j < SB; j++)
                if (sp + j < nsplit) v[i] = __fadd_rn(v[i], a[i][j]);
    }
#pragma unroll
    for (int i = 0; i < VPT; i++) {
        if (off[i] < 0) continue;
        const int q = threadIdx.x + 256 * i, r = q / E, e = q % E;
        lg[r * (EB + 1) + e] = bias ? __fadd_rn(v[i], __ldg(bias + e)) : v[i];
    }
    __syncthreads();
    router_tail<EB>(lg, T, E, k, tile, probs, ids, wts, loc, tile_cnt, sid, swt);
}

int router_splits(int T, int d) {
    const int tiles = ceil_div(T, TT);
    if (tiles >= 64 || d < 256) return 1;
    int ns = ceil_div(256, tiles);
    ns = min(ns, d / 128);
    return max(ns, 1);
}

template <int EB>
static void launch_router_eb(const float *x, int T, int d, const float *w_router, const float *bias,
                             int E, int k, float *probs, int *ids, float *wts, int *loc,
                             int *tile_cnt, float *part, int nsplit, cudaStream_t s)
{
    const int tiles = ceil_div(T, TT);
    if (nsplit <= 1 || part == nullptr) {
        router_topk_kernel<EB><<<tiles, 256, 0, s>>>(x, T, d, w_router, bias, E, k, probs, ids, wts,
                                                     loc, tile_cnt);
        return;
    }
    const int dsplit = round_up(ceil_div(d, nsplit), DC);
    nsplit = ceil_div(d, dsplit);
    router_partial_kernel<EB><<<dim3(tiles, nsplit), 256, 0, s>>>(x, T, d, w_router, E, dsplit, part);
    router_reduce_topk_kernel<EB><<<tiles, 256, 0, s>>>(part, nsplit, T, bias, E, k, probs, ids, wts,
                                                        loc, tile_cnt);
}

cudaError_t launch_router(const float *x, int T, int d, const float *w_router,
                          const float *bias, int E, int k, float *probs, int *ids,
                          float *wts, int *loc, int *tile_cnt, cudaStream_t s,
                          float *part, int nsplit)
{
    if (E <= 8)
        launch_router_eb<8>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt, part, nsplit, s);
    else if (E <= 16)
        launch_router_eb<16>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt, part, nsplit, s);
    else if (E <= 32)
        launch_router_eb<32>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt, part, nsplit, s);
    else if (E <= 64)
        launch_router_eb<64>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt, part, nsplit, s);
    else
        launch_router_eb<128>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt, part, nsplit, s);
    return cudaGetLastError();
}

}  // namespace moe
