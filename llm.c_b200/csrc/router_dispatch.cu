// router_dispatch.cu — dispatch (scan, stable permutation, row gather) and
// combine of the MoE feed-forward block; the router is in router.cu.
//
// Reference: llm.c src/transformer.c:299-345 (router, top-k, per-token
// view) and src/matrix.c:529-586 (softmax_rows).
#include "kernels.cuh"

namespace moe {

// ---------------------------------------------------------------------
// K4a  dispatch_scan — one CTA.  For every expert: exclusive prefix of
// the tile histograms (tile_pref), total count, expert row offset in the
// permuted buffer, and the m-tile prefixes the grouped GEMMs schedule on.
// Plan layout (ints): cnt[E] | off[E+1] | mt128[E+1] | mt64[E+1] | mt256[E+1]
// With align > 1 every expert's rows start at a multiple of align (the
// backward's weight-gradient GEMMs run K over an expert's rows with TMA).
// ---------------------------------------------------------------------
__global__ void __launch_bounds__(1024)
dispatch_scan_kernel(const int *__restrict__ tile_cnt, int n_tiles, int E,
                     int *__restrict__ tile_pref, int *__restrict__ plan, int align)
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
        int *mt256 = mt64 + E + 1;
        int o = 0, m1 = 0, m2 = 0, m3 = 0;
        for (int e = 0; e < E; e++) {
            cnt[e] = cnt_s[e];
            off[e] = o; mt128[e] = m1; mt64[e] = m2; mt256[e] = m3;
            o += (cnt_s[e] + align - 1) / align * align;
            m1 += (cnt_s[e] + 127) / 128;
            m2 += (cnt_s[e] + 63) / 64;
            m3 += (cnt_s[e] + 255) / 256;
        }
        off[E] = o; mt128[E] = m1; mt64[E] = m2; mt256[E] = m3;
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

// K7, rows of 4-float multiples with k <= KT: the same arithmetic, with U
// float4 columns per thread loaded together (U·KT row loads in flight, 8 or
// 16 with the second K half) before any is used, so a thread's loads overlap
// instead of waiting one round trip per column.
template <int KT, int U>
__global__ void __launch_bounds__(256)
combine4_kernel(const float *__restrict__ y, int d, int d_pad, int T, int k,
                const int *__restrict__ pos_of, const float *__restrict__ wts,
                float *out, const float *__restrict__ y2, const float *resid)
{
    const int t = blockIdx.x;
    if (t >= T) return;
    const float4 *yr[KT], *y2r[KT];
    float w[KT];
#pragma unroll
    for (int r = 0; r < KT; r++) {
        const int p = r < k ? pos_of[(size_t)t * k + r] : 0;
        w[r] = r < k ? wts[(size_t)t * k + r] : 0.0f;
        yr[r] = reinterpret_cast<const float4 *>(y + (size_t)p * d_pad);
        y2r[r] = y2 ? reinterpret_cast<const float4 *>(y2 + (size_t)p * d_pad) : nullptr;
    }
    const int n4 = d >> 2;
    float4 *o = reinterpret_cast<float4 *>(out + (size_t)t * d);
    const float4 *xr = resid ? reinterpret_cast<const float4 *>(resid + (size_t)t * d) : nullptr;
    for (int c0 = threadIdx.x; c0 < n4; c0 += U * blockDim.x) {
        float4 v[U][KT];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = c0 + u * blockDim.x;
#pragma unroll
            for (int r = 0; r < KT; r++)
                v[u][r] = (r < k && c < n4) ? __ldg(yr[r] + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (y2) {
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int c = c0 + u * blockDim.x;
#pragma unroll
                for (int r = 0; r < KT; r++) {
                    if (r < k && c < n4) {
                        const float4 v2 = __ldg(y2r[r] + c);
                        v[u][r].x = __fadd_rn(v[u][r].x, v2.x); v[u][r].y = __fadd_rn(v[u][r].y, v2.y);
                        v[u][r].z = __fadd_rn(v[u][r].z, v2.z); v[u][r].w = __fadd_rn(v[u][r].w, v2.w);
                    }
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = c0 + u * blockDim.x;
            if (c >= n4) break;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int r = 0; r < KT; r++) {
                if (r < k) {
                    acc.x = __fmaf_rn(w[r], v[u][r].x, acc.x);
                    acc.y = __fmaf_rn(w[r], v[u][r].y, acc.y);
                    acc.z = __fmaf_rn(w[r], v[u][r].z, acc.z);
                    acc.w = __fmaf_rn(w[r], v[u][r].w, acc.w);
                }
            }
            if (xr) {
                const float4 x = xr[c];
                acc.x = __fadd_rn(x.x, acc.x); acc.y = __fadd_rn(x.y, acc.y);
                acc.z = __fadd_rn(x.z, acc.z); acc.w = __fadd_rn(x.w, acc.w);
            }
            o[c] = acc;
        }
    }
}

// ---------------------------------------------------------------------
// K7  combine — out[t] = Σ_r w_{t,r} · y[pos(t,r)] for r = 0..k-1 in rank
// order, starting from zero with one fused multiply-add per term, as the
// reference accumulates (src/transformer.c:296,355-358).  No atomics: the
// result is bit-stable run to run.  With `resid` (block_forward's residual,
// src/transformer.c:767) the finished sum is added to it, as
// mat_add_inplace does (src/matrix.c:491-500); resid may be out itself.
// ---------------------------------------------------------------------
__global__ void __launch_bounds__(256)
combine_kernel(const float *__restrict__ y, int d, int d_pad, int T, int k,
               const int *__restrict__ pos_of, const float *__restrict__ wts,
               float *out, const float *__restrict__ y2, const float *resid)
{
    // y2 (optional): the second K half of the down GEMM, added to y first
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
                    float4 v = __ldg(reinterpret_cast<const float4 *>(y + (size_t)pos[r] * d_pad) + c);
                    if (y2) {
                        const float4 v2 = __ldg(reinterpret_cast<const float4 *>(y2 + (size_t)pos[r] * d_pad) + c);
                        v.x = __fadd_rn(v.x, v2.x); v.y = __fadd_rn(v.y, v2.y);
                        v.z = __fadd_rn(v.z, v2.z); v.w = __fadd_rn(v.w, v2.w);
                    }
                    acc.x = __fmaf_rn(w[r], v.x, acc.x);
                    acc.y = __fmaf_rn(w[r], v.y, acc.y);
                    acc.z = __fmaf_rn(w[r], v.z, acc.z);
                    acc.w = __fmaf_rn(w[r], v.w, acc.w);
                }
            }
            if (resid) {
                const float4 x = reinterpret_cast<const float4 *>(resid + (size_t)t * d)[c];
                acc.x = __fadd_rn(x.x, acc.x); acc.y = __fadd_rn(x.y, acc.y);
                acc.z = __fadd_rn(x.z, acc.z); acc.w = __fadd_rn(x.w, acc.w);
            }
            reinterpret_cast<float4 *>(o)[c] = acc;
        }
    } else {
        for (int c = threadIdx.x; c < d; c += blockDim.x) {
            float acc = 0.0f;
            for (int r = 0; r < k; r++) {
                float v = __ldg(y + (size_t)pos[r] * d_pad + c);
                if (y2) v = __fadd_rn(v, __ldg(y2 + (size_t)pos[r] * d_pad + c));
                acc = __fmaf_rn(w[r], v, acc);
            }
            if (resid) acc = __fadd_rn(resid[(size_t)t * d + c], acc);
            o[c] = acc;
        }
    }
}

// ---------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------
cudaError_t launch_dispatch(const float *x, int T, int d, int d_pad, int E, int k,
                            const int *ids, const int *loc, const int *tile_cnt,
                            int *tile_pref, int *plan, int *pos_of, float *x_perm,
                            int round_to_tf32, DeviceStatus *status, cudaStream_t s, int align)
{
    const int tiles = ceil_div(T, kRouterTile);
    dispatch_scan_kernel<<<1, 1024, 0, s>>>(tile_cnt, tiles, E, tile_pref, plan, align);
    const int warps = T * k;
    dispatch_gather_kernel<<<ceil_div(warps, 8), 256, 0, s>>>(x, T, d, d_pad, k, E, ids, loc,
                                                               tile_pref, plan, pos_of, x_perm, round_to_tf32, status);
    return cudaGetLastError();
}

cudaError_t launch_combine(const float *y, int d, int d_pad, int T, int k,
                           const int *pos_of, const float *wts, float *out, cudaStream_t s,
                           const float *y2, const float *resid)
{
    int threads = 256;
    const int work = (d & 3) == 0 ? d / 4 : d;
    if (work < 256) threads = max(32, round_up(work, 32));
    if ((d & 3) == 0 && k <= 2)
        combine4_kernel<2, 4><<<T, threads, 0, s>>>(y, d, d_pad, T, k, pos_of, wts, out, y2, resid);
    else if ((d & 3) == 0 && k <= 4)
        combine4_kernel<4, 2><<<T, threads, 0, s>>>(y, d, d_pad, T, k, pos_of, wts, out, y2, resid);
    else
        combine_kernel<<<T, threads, 0, s>>>(y, d, d_pad, T, k, pos_of, wts, out, y2, resid);
    return cudaGetLastError();
}

}  // namespace moe

namespace moe {
cudaError_t launch_dispatch_scan(const int *tile_cnt, int T, int E, int *tile_pref, int *plan,
                                 cudaStream_t s)
{
    dispatch_scan_kernel<<<1, 1024, 0, s>>>(tile_cnt, ceil_div(T, kRouterTile), E, tile_pref, plan, 1);
    return cudaGetLastError();
}
}  // namespace moe

namespace moe {
// Zero the alignment rows of every expert segment, [off[e] + cnt[e],
// off[e + 1]), of a [rows × ld] expert-sorted buffer.
__global__ void __launch_bounds__(256)
zero_pad_rows_kernel(float *__restrict__ buf, int ld, const int *__restrict__ plan, int E)
{
    const int e = blockIdx.x;
    const int *cnt = plan, *off = plan + E;
    const size_t r0 = (size_t)off[e] + cnt[e], r1 = (size_t)off[e + 1];
    for (size_t i = r0 * ld + threadIdx.x; i < r1 * ld; i += blockDim.x) buf[i] = 0.0f;
}

cudaError_t launch_zero_pad_rows(float *buf, int ld, const int *plan, int E, cudaStream_t s)
{
    zero_pad_rows_kernel<<<E, 256, 0, s>>>(buf, ld, plan, E);
    return cudaGetLastError();
}
}  // namespace moe
