// router_dispatch.cu — router (logits, softmax, top-k, renormalisation) and
// dispatch (histogram, scan, stable permutation, row gather) of the MoE
// feed-forward block.
//
// Reference: llm.c src/transformer.c:299-345 (router, top-k, per-token
// view) and src/matrix.c:529-586 (softmax_rows).
#include "kernels.cuh"

namespace moe {

// ---------------------------------------------------------------------
// K1-K3  router_topk
//
// One CTA owns a tile of kRouterTile tokens.  Logits x·W_router are FP32
// FFMA dot products (E <= 128 is far too narrow for a tensor-core tile),
// sequential over d per output.  The softmax, the top-k selection and the
// renormalisation then run one thread per token, mirroring the
// reference's arithmetic (src/matrix.c:529-586, src/transformer.c:
// 312-337) so that identical logits give bit-identical probabilities and
// identical ids.  Finally one thread per expert counts the tile's tokens
// that chose it and records each (token, rank)'s stable position among
// them — the first half of the dispatch.
// ---------------------------------------------------------------------
template <int EPT>
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
    constexpr int TT = kRouterTile;
    constexpr int DC = EPT >= 16 ? 32 : 64;   // keeps static smem < 48 KB
    constexpr int EP = 8 * EPT;
    __shared__ float xs[TT][DC + 1];
    __shared__ float ws[DC][EP];
    __shared__ float lg[TT][EP + 1];
    __shared__ int sid[TT][kMaxTopK];
    __shared__ float swt[TT][kMaxTopK];

    const int tile = blockIdx.x;
    const int t0 = tile * TT;
    const int tid = threadIdx.x;
    const int tl = tid >> 3;     // token within tile (0..31)
    const int eo = tid & 7;      // expert residue

    float acc[EPT];
#pragma unroll
    for (int j = 0; j < EPT; j++) acc[j] = 0.0f;

    for (int i0 = 0; i0 < d; i0 += DC) {
        for (int q = tid; q < TT * DC; q += 256) {
            const int r = q / DC, c = q % DC;
            const int t = t0 + r, i = i0 + c;
            xs[r][c] = (t < T && i < d) ? __ldg(x + (size_t)t * d + i) : 0.0f;
        }
        for (int q = tid; q < DC * EP; q += 256) {
            const int r = q / EP, c = q % EP;
            const int i = i0 + r;
            ws[r][c] = (i < d && c < E) ? __ldg(w_router + (size_t)i * E + c) : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int c = 0; c < DC; c++) {
            const float xv = xs[tl][c];
#pragma unroll
            for (int j = 0; j < EPT; j++) acc[j] = __fmaf_rn(xv, ws[c][eo + 8 * j], acc[j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < EPT; j++) {
        const int e = eo + 8 * j;
        if (e < E) lg[tl][e] = bias ? __fadd_rn(acc[j], __ldg(bias + e)) : acc[j];
    }
    __syncthreads();

    if (tid < TT && t0 + tid < T) {
        float *row = lg[tid];
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

        // top-k: k passes, strict '>', best = -1, best_e = 0, e ascending.
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
        probs[(size_t)t0 * E + q] = lg[r][c];
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

// ---------------------------------------------------------------------
// K4a  dispatch_scan — one CTA.  For every expert: exclusive prefix of
// the tile histograms (tile_pref), total count, expert row offset in the
// permuted buffer, and the m-tile prefixes the grouped GEMMs schedule on.
// Plan layout (ints): cnt[E] | off[E+1] | mt128[E+1] | mt64[E+1]
// ---------------------------------------------------------------------
__global__ void __launch_bounds__(1024)
dispatch_scan_kernel(const int *__restrict__ tile_cnt, int n_tiles, int E,
                     int *__restrict__ tile_pref, int *__restrict__ plan)
{
    __shared__ int cnt_s[kMaxExperts];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = blockDim.x >> 5;
    for (int e = warp; e < E; e += nwarps) {
        int running = 0;
        for (int base = 0; base < n_tiles; base += 32) {
            const int t = base + lane;
            const int v = (t < n_tiles) ? tile_cnt[(size_t)t * E + e] : 0;
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += n;
            }
            if (t < n_tiles) tile_pref[(size_t)t * E + e] = running + incl - v;
            running += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) cnt_s[e] = running;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int *cnt = plan, *off = plan + E, *mt128 = off + E + 1, *mt64 = mt128 + E + 1;
        int o = 0, m1 = 0, m2 = 0;
        for (int e = 0; e < E; e++) {
            cnt[e] = cnt_s[e];
            off[e] = o; mt128[e] = m1; mt64[e] = m2;
            o += cnt_s[e];
            m1 += (cnt_s[e] + 127) / 128;
            m2 += (cnt_s[e] + 63) / 64;
        }
        off[E] = o; mt128[E] = m1; mt64[E] = m2;
    }
}

// ---------------------------------------------------------------------
// K4b  dispatch_gather — one warp per (token, rank) entry: its slot in
// the expert-sorted order (stable: token order within an expert), and a
// float4 copy of the token's row into the permuted activation buffer,
// zero-padded from d to d_pad.
// ---------------------------------------------------------------------
__global__ void __launch_bounds__(256)
dispatch_gather_kernel(const float *__restrict__ x, int T, int d, int d_pad,
                       int k, int E,
                       const int *__restrict__ ids, const int *__restrict__ loc,
                       const int *__restrict__ tile_pref,
                       const int *__restrict__ plan,
                       int *__restrict__ pos_of, float *__restrict__ x_perm,
                       int round_to_tf32, DeviceStatus *status)
{
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= T * k) return;
    const int t = warp / k;
    const int e = ids[warp];
    const int *off = plan + E;
    const int rows = off[E];
    int pos = off[e] + tile_pref[(size_t)(t / kRouterTile) * E + e] + loc[warp];
    if (pos < 0 || pos >= rows || e < 0 || e >= E) {   // never expected
        if (lane == 0) atomicExch(&status->bad_index, 1);
        return;
    }
    if (lane == 0) pos_of[warp] = pos;
    const float *src = x + (size_t)t * d;
    float *dst = x_perm + (size_t)pos * d_pad;
    if ((d & 3) == 0) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *d4 = reinterpret_cast<float4 *>(dst);
        const int n4 = d >> 2, p4 = d_pad >> 2;
        for (int c = lane; c < p4; c += 32) {
            float4 v = (c < n4) ? __ldg(s4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            if (round_to_tf32) {
                v.x = round_tf32(v.x); v.y = round_tf32(v.y);
                v.z = round_tf32(v.z); v.w = round_tf32(v.w);
            }
            d4[c] = v;
        }
    } else {
        for (int c = lane; c < d_pad; c += 32) {
            const float v = (c < d) ? __ldg(src + c) : 0.0f;
            dst[c] = round_to_tf32 ? round_tf32(v) : v;
        }
    }
}

// ---------------------------------------------------------------------
// K7  combine — out[t] = Σ_r w_{t,r} · y[pos(t,r)] for r = 0..k-1 in rank
// order, starting from zero with one fused multiply-add per term, as the
// reference accumulates (src/transformer.c:296,355-358).  No atomics: the
// result is bit-stable run to run.
// ---------------------------------------------------------------------
__global__ void __launch_bounds__(256)
combine_kernel(const float *__restrict__ y, int d, int d_pad, int T, int k,
               const int *__restrict__ pos_of, const float *__restrict__ wts,
               float *__restrict__ out)
{
    const int t = blockIdx.x;
    if (t >= T) return;
    int pos[kMaxTopK];
    float w[kMaxTopK];
#pragma unroll
    for (int r = 0; r < kMaxTopK; r++) {
        if (r < k) { pos[r] = pos_of[(size_t)t * k + r]; w[r] = wts[(size_t)t * k + r]; }
    }
    float *o = out + (size_t)t * d;
    if ((d & 3) == 0) {
        for (int c = threadIdx.x; c < (d >> 2); c += blockDim.x) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int r = 0; r < kMaxTopK; r++) {
                if (r < k) {
                    const float4 v = __ldg(reinterpret_cast<const float4 *>(y + (size_t)pos[r] * d_pad) + c);
                    acc.x = __fmaf_rn(w[r], v.x, acc.x);
                    acc.y = __fmaf_rn(w[r], v.y, acc.y);
                    acc.z = __fmaf_rn(w[r], v.z, acc.z);
                    acc.w = __fmaf_rn(w[r], v.w, acc.w);
                }
            }
            reinterpret_cast<float4 *>(o)[c] = acc;
        }
    } else {
        for (int c = threadIdx.x; c < d; c += blockDim.x) {
            float acc = 0.0f;
            for (int r = 0; r < k; r++) acc = __fmaf_rn(w[r], __ldg(y + (size_t)pos[r] * d_pad + c), acc);
            o[c] = acc;
        }
    }
}

// ---------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------
cudaError_t launch_router(const float *x, int T, int d, const float *w_router,
                          const float *bias, int E, int k, float *probs, int *ids,
                          float *wts, int *loc, int *tile_cnt, cudaStream_t s)
{
    const int tiles = ceil_div(T, kRouterTile);
    if (E <= 8)        router_topk_kernel<1><<<tiles, 256, 0, s>>>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt);
    else if (E <= 16)  router_topk_kernel<2><<<tiles, 256, 0, s>>>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt);
    else if (E <= 32)  router_topk_kernel<4><<<tiles, 256, 0, s>>>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt);
    else if (E <= 64)  router_topk_kernel<8><<<tiles, 256, 0, s>>>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt);
    else               router_topk_kernel<16><<<tiles, 256, 0, s>>>(x, T, d, w_router, bias, E, k, probs, ids, wts, loc, tile_cnt);
    return cudaGetLastError();
}

cudaError_t launch_dispatch(const float *x, int T, int d, int d_pad, int E, int k,
                            const int *ids, const int *loc, const int *tile_cnt,
                            int *tile_pref, int *plan, int *pos_of, float *x_perm,
                            int round_to_tf32, DeviceStatus *status, cudaStream_t s)
{
    const int tiles = ceil_div(T, kRouterTile);
    dispatch_scan_kernel<<<1, 1024, 0, s>>>(tile_cnt, tiles, E, tile_pref, plan);
    const int warps = T * k;
    dispatch_gather_kernel<<<ceil_div(warps, 8), 256, 0, s>>>(x, T, d, d_pad, k, E, ids, loc,
                                                               tile_pref, plan, pos_of, x_perm, round_to_tf32, status);
    return cudaGetLastError();
}

cudaError_t launch_combine(const float *y, int d, int d_pad, int T, int k,
                           const int *pos_of, const float *wts, float *out, cudaStream_t s)
{
    int threads = 256;
    const int work = (d & 3) == 0 ? d / 4 : d;
    if (work < 256) threads = max(32, round_up(work, 32));
    combine_kernel<<<T, threads, 0, s>>>(y, d, d_pad, T, k, pos_of, wts, out);
    return cudaGetLastError();
}

}  // namespace moe
