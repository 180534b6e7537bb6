// moe_backward.cu — backward of the MoE feed-forward block.
//
// llm.c has no MoE backward: model_backward (src/transformer.c:981-1013)
// stops at the RMSNorms and attention, and moe_forward's comment
// (src/transformer.c:280-282) leaves the Switch load-balancing loss to the
// training loop.  This is the gradient of the forward the library computes
// (src/transformer.c:287-366), with the top-k choice held fixed:
//   p = softmax(x·W_r + b),  S = top-k(p),  w_r = p_{S_r} / Σ_s p_{S_s},
//   y = Σ_r w_r · FFN_{S_r}(x),  FFN_e(x) = (silu(x·Wg_e) ⊙ x·Wu_e)·Wd_e,
// plus aux_coef · L_aux, the Switch Transformer load-balancing loss
//   L_aux = E · Σ_e f_e · P_e,  f_e = n_e / (T·k) (the expert's share of the
//   T·k assignments, a constant),  P_e = mean over tokens of p_{t,e}.
// Given dy = ∂L/∂y it writes dx and adds the weight gradients into gradient
// buffers in llm.c's layouts (W_router [d×E], W_gate / W_up [d×F],
// W_down [F×d]) and the router bias gradient [E].
//
// FP32 FFMA throughout.  Every sum runs in a fixed order and every output
// element belongs to one thread (no atomics), so results are bit-stable run
// to run.  The GEMMs share one 64×64-tile FFMA core whose operands may be
// contiguous along K or along M/N; the weight-gradient GEMMs run K over an
// expert's rows of the forward's expert-sorted buffers.
#include "kernels.cuh"

namespace moe {

namespace {

constexpr int BM = 64, BN = 64, BK = 16, LDS = BM + 4;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// The m-tile of the forward's plan (64-row tiles of each expert's rows).
__device__ __forceinline__ bool decode_mtile(const int *plan, int E, int bx, int &e, int &row0,
                                             int &nrows) {
    const int *cnt = plan, *off = plan + E, *mt64 = off + 2 * (E + 1);
    if (bx >= mt64[E]) return false;
    int lo = 0, hi = E;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (mt64[mid] <= bx) lo = mid; else hi = mid - 1;
    }
    e = lo;
    const int mt = bx - mt64[e];
    row0 = off[e] + mt * BM;
    nrows = min(BM, cnt[e] - mt * BM);
    return true;
}

// A [BK × 64] slab into shared memory as s[k][i]: element (i, k) lives at
// p[i·ld + k] (KC, contiguous along k) or p[k·ld + i]; i >= iend or
// k >= kend read as zero.  `vec`: 16-byte loads are legal (ld % 4 == 0, p
// aligned, and for KC slabs k0 % 4 == 0).
template <bool KC>
__device__ __forceinline__ void load_slab(float (*s)[LDS], const float *__restrict__ p, int ld,
                                          int i0, int iend, int k0, int kend, bool vec) {
    const int tid = threadIdx.x;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (KC) {
        const int i = tid >> 2, kq = (tid & 3) * 4;
        const int gi = i0 + i, gk = k0 + kq;
        if (gi < iend) {
            const float *q = p + (size_t)gi * ld + gk;
            if (vec && gk + 3 < kend) {
                const float4 t = __ldg(reinterpret_cast<const float4 *>(q));
                v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
            } else {
#pragma unroll
                for (int c = 0; c < 4; c++)
                    if (gk + c < kend) v[c] = __ldg(q + c);
            }
        }
#pragma unroll
        for (int c = 0; c < 4; c++) s[kq + c][i] = v[c];
    } else {
        const int k = tid >> 4, iq = (tid & 15) * 4;
        const int gk = k0 + k, gi = i0 + iq;
        if (gk < kend) {
            const float *q = p + (size_t)gk * ld + gi;
            if (vec && gi + 3 < iend) {
                const float4 t = __ldg(reinterpret_cast<const float4 *>(q));
                v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
            } else {
#pragma unroll
                for (int c = 0; c < 4; c++)
                    if (gi + c < iend) v[c] = __ldg(q + c);
            }
        }
        *reinterpret_cast<float4 *>(&s[k][iq]) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

// acc[i][j] = Σ_{k in [kbeg, kend)} A(m0 + ty·4 + i, k) · B(n0 + tx·4 + j, k), k ascending.
template <bool A_KC, bool B_KC>
__device__ __forceinline__ void gemm_tile(const float *__restrict__ A, int lda, int m0, int mend,
                                          bool avec, const float *__restrict__ B, int ldb, int n0,
                                          int nend, bool bvec, int kbeg, int kend,
                                          float (&acc)[4][4]) {
    __shared__ __align__(16) float As[BK][LDS];
    __shared__ __align__(16) float Bs[BK][LDS];
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.f;
    for (int k0 = kbeg; k0 < kend; k0 += BK) {
        load_slab<A_KC>(As, A, lda, m0, mend, k0, kend, avec);
        load_slab<B_KC>(Bs, B, ldb, n0, nend, k0, kend, bvec);
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
        }
        __syncthreads();
    }
}

// column of the gate pre-activation of output f in the weights' row order
// (per 128 columns: 128 gate rows, then the 128 matching up rows)
__device__ __forceinline__ int gate_col(int f) { return (f >> 7) * 256 + (f & 127); }

}  // namespace

// ---- combine backward: dw_{t,r} = dy_t · y_{t,r};  dO_{t,r} = w_{t,r} · dy_t
__global__ void __launch_bounds__(256)
bwd_combine_kernel(const float *__restrict__ dy, const float *__restrict__ y,
                   const int *__restrict__ pos_of, const float *__restrict__ wts, int d, int d_pad,
                   int k, float *__restrict__ dw, float *__restrict__ dO, int round) {
    // round: dO feeds TF32 tensor-core GEMMs, so it is rounded to nearest TF32
    __shared__ float red[8];
    const int t = blockIdx.x;
    const float *g = dy + (size_t)t * d;
    for (int r = 0; r < k; r++) {
        const int p = pos_of[(size_t)t * k + r];
        const float w = wts[(size_t)t * k + r];
        const float *yr = y + (size_t)p * d_pad;
        float *o = dO + (size_t)p * d_pad;
        float part = 0.f;
        for (int j = threadIdx.x; j < d_pad; j += 256) {
            const float gj = j < d ? __ldg(g + j) : 0.f;
            if (j < d) part = __fmaf_rn(gj, __ldg(yr + j), part);
            const float v = __fmul_rn(w, gj);
            o[j] = round ? round_tf32(v) : v;
        }
        part = warp_sum(part);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
        __syncthreads();
        if (threadIdx.x == 0) {
            float sum = 0.f;
            for (int i = 0; i < 8; i++) sum = __fadd_rn(sum, red[i]);
            dw[(size_t)t * k + r] = sum;
        }
        __syncthreads();
    }
}

// ---- router backward, one warp per token: the renormalisation, the aux
// loss term, then the softmax
__global__ void __launch_bounds__(256)
bwd_router_kernel(const float *__restrict__ probs, const int *__restrict__ ids,
                  const float *__restrict__ wts, const float *__restrict__ dw,
                  const int *__restrict__ cnt, int T, int E, int k, float aux_scale,
                  float *__restrict__ dlogit) {
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= T) return;
    const float *p = probs + (size_t)t * E;
    const int *id = ids + (size_t)t * k;
    // w_r = p_{S_r} · (1 / s), s summed in rank order as the forward does
    float s = 0.f, q = 0.f;
    for (int r = 0; r < k; r++) s = __fadd_rn(s, p[id[r]]);
    for (int r = 0; r < k; r++) q = __fmaf_rn(dw[(size_t)t * k + r], wts[(size_t)t * k + r], q);
    const bool live = s > 1e-9f;
    auto dp_of = [&](int e) {
        float v = __fmul_rn(aux_scale, (float)cnt[e]);
        if (live)
            for (int r = 0; r < k; r++)
                if (id[r] == e) v = __fadd_rn(v, __fdiv_rn(__fsub_rn(dw[(size_t)t * k + r], q), s));
        return v;
    };
    float dot = 0.f;
    for (int e = lane; e < E; e += 32) dot = __fmaf_rn(p[e], dp_of(e), dot);
    dot = warp_sum(dot);
    for (int e = lane; e < E; e += 32)
        dlogit[(size_t)t * E + e] = __fmul_rn(p[e], __fsub_rn(dp_of(e), dot));
}

// ---- per expert column: P_e = mean_t p_{t,e}; bias gradient Σ_t dlogit_{t,e}
__global__ void __launch_bounds__(256)
bwd_colsum_kernel(const float *__restrict__ probs, const float *__restrict__ dlogit, int T, int E,
                  float *__restrict__ pmean, float *__restrict__ g_bias) {
    __shared__ float rp[8], rd[8];
    const int e = blockIdx.x;
    float sp = 0.f, sd = 0.f;
    for (int t = threadIdx.x; t < T; t += 256) {
        sp = __fadd_rn(sp, probs[(size_t)t * E + e]);
        sd = __fadd_rn(sd, dlogit[(size_t)t * E + e]);
    }
    sp = warp_sum(sp);
    sd = warp_sum(sd);
    if ((threadIdx.x & 31) == 0) { rp[threadIdx.x >> 5] = sp; rd[threadIdx.x >> 5] = sd; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.f, b = 0.f;
        for (int i = 0; i < 8; i++) { a = __fadd_rn(a, rp[i]); b = __fadd_rn(b, rd[i]); }
        pmean[e] = __fdiv_rn(a, (float)T);
        if (g_bias) g_bias[e] = __fadd_rn(g_bias[e], b);
    }
}

// ---- L_aux = E · Σ_e (n_e / (T·k)) · P_e
__global__ void bwd_aux_kernel(const float *__restrict__ pmean, const int *__restrict__ cnt,
                               int T, int E, int k, float *__restrict__ aux_loss) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const float inv = __fdiv_rn(1.0f, __fmul_rn((float)T, (float)k));
    float sum = 0.f;
    for (int e = 0; e < E; e++) sum = __fmaf_rn(__fmul_rn((float)cnt[e], inv), pmean[e], sum);
    *aux_loss = __fmul_rn((float)E, sum);
}

// ---- dH = dO · Wd_eᵀ, then the SwiGLU backward into dG, dU
// (h = silu(g) ⊙ u:  dU = dH ⊙ silu(g),  dG = dH ⊙ u ⊙ silu'(g))
__global__ void __launch_bounds__(256)
bwd_dh_kernel(const float *__restrict__ dO, int d_pad, const float *__restrict__ dn, int F_pad,
              const float *__restrict__ gu, float *__restrict__ dgu, const int *__restrict__ plan,
              int E) {
    int e, row0, nrows;
    if (!decode_mtile(plan, E, blockIdx.x, e, row0, nrows)) return;
    const int n0 = blockIdx.y * BN;
    float acc[4][4];
    // B(f, j) = Wd_e[f][j] = dn[e][j][f]
    gemm_tile<true, false>(dO, d_pad, row0, row0 + nrows, true, dn + (size_t)e * d_pad * F_pad,
                           F_pad, n0, F_pad, true, 0, d_pad, acc);
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    const int c = gate_col(n0 + tx * 4);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = ty * 4 + i;
        if (r >= nrows) continue;
        const size_t base = (size_t)(row0 + r) * 2 * F_pad + c;
        const float4 g4 = *reinterpret_cast<const float4 *>(gu + base);
        const float4 u4 = *reinterpret_cast<const float4 *>(gu + base + 128);
        const float gv[4] = {g4.x, g4.y, g4.z, g4.w}, uv[4] = {u4.x, u4.y, u4.z, u4.w};
        float dg[4], du[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_ref(-gv[j])));
            const float silu = __fmul_rn(gv[j], sig);
            const float dsilu = __fmul_rn(sig, __fadd_rn(1.0f, __fmul_rn(gv[j], __fsub_rn(1.0f, sig))));
            du[j] = __fmul_rn(acc[i][j], silu);
            dg[j] = __fmul_rn(__fmul_rn(acc[i][j], uv[j]), dsilu);
        }
        *reinterpret_cast<float4 *>(dgu + base) = make_float4(dg[0], dg[1], dg[2], dg[3]);
        *reinterpret_cast<float4 *>(dgu + base + 128) = make_float4(du[0], du[1], du[2], du[3]);
    }
}

// ---- dX_perm = [dG | dU] · [Wg_e | Wu_e]ᵀ  (K over the weights' row order)
__global__ void __launch_bounds__(256)
bwd_dxp_kernel(const float *__restrict__ dgu, int F_pad, const float *__restrict__ ug, int d_pad,
               float *__restrict__ dxp, const int *__restrict__ plan, int E) {
    int e, row0, nrows;
    if (!decode_mtile(plan, E, blockIdx.x, e, row0, nrows)) return;
    const int n0 = blockIdx.y * BN;
    float acc[4][4];
    // B(j, c) = ug[e][c][j]
    gemm_tile<true, false>(dgu, 2 * F_pad, row0, row0 + nrows, true,
                           ug + (size_t)e * 2 * F_pad * d_pad, d_pad, n0, d_pad, true, 0,
                           2 * F_pad, acc);
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = ty * 4 + i;
        if (r >= nrows) continue;
        *reinterpret_cast<float4 *>(dxp + (size_t)(row0 + r) * d_pad + n0 + tx * 4) =
            make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    }
}

// ---- dWd_e[f][j] += Σ_{rows of e} H[row][f] · dO[row][j]
__global__ void __launch_bounds__(256)
bwd_wgrad_down_kernel(const float *__restrict__ h, int F_pad, const float *__restrict__ dO,
                      int d_pad, int F, int d, const int *__restrict__ plan, int E,
                      float *__restrict__ g_down) {
    const int e = blockIdx.z;
    const int cnt = plan[e], off = plan[E + e];
    if (cnt == 0) return;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    float acc[4][4];
    gemm_tile<false, false>(h, F_pad, m0, F_pad, true, dO, d_pad, n0, d_pad, true, off, off + cnt,
                            acc);
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    float *g = g_down + (size_t)e * F * d;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int f = m0 + ty * 4 + i;
        if (f >= F) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int col = n0 + tx * 4 + j;
            if (col < d) g[(size_t)f * d + col] = __fadd_rn(g[(size_t)f * d + col], acc[i][j]);
        }
    }
}

// ---- dWg_e[j][f] += Σ X[row][j] · dG[row][f];  dWu_e likewise with dU
__global__ void __launch_bounds__(256)
bwd_wgrad_upgate_kernel(const float *__restrict__ x_perm, int d_pad, const float *__restrict__ dgu,
                        int F_pad, int d, int F, const int *__restrict__ plan, int E,
                        float *__restrict__ g_gate, float *__restrict__ g_up) {
    const int e = blockIdx.z;
    const int cnt = plan[e], off = plan[E + e];
    if (cnt == 0) return;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    float acc[4][4];
    gemm_tile<false, false>(x_perm, d_pad, m0, d_pad, true, dgu, 2 * F_pad, n0, 2 * F_pad, true,
                            off, off + cnt, acc);
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    // a 64-column tile lies inside one gate or up half of a 256-column block
    const int blk = n0 >> 8, within = n0 & 255;
    float *g = (within >= 128 ? g_up : g_gate) + (size_t)e * d * F;
    const int f0 = blk * 128 + (within & 127) + tx * 4;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int j = m0 + ty * 4 + i;
        if (j >= d) continue;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int f = f0 + c;
            if (f < F) g[(size_t)j * F + f] = __fadd_rn(g[(size_t)j * F + f], acc[i][c]);
        }
    }
}

// ---- router part of dx: dx[t][j] = Σ_e dlogit[t][e] · W_r[j][e]  (overwrites dx)
__global__ void __launch_bounds__(256)
bwd_router_dx_kernel(const float *__restrict__ dlogit, const float *__restrict__ router, int T,
                     int d, int E, int vec, float *__restrict__ dx) {
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    float acc[4][4];
    gemm_tile<true, true>(dlogit, E, m0, T, vec, router, E, n0, d, vec, 0, E, acc);
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int t = m0 + ty * 4 + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int col = n0 + tx * 4 + j;
            if (col < d) dx[(size_t)t * d + col] = acc[i][j];
        }
    }
}

// ---- W_r gradient: g_router[j][e] += Σ_t x[t][j] · dlogit[t][e].  The
// token range is split over blockIdx.z (fixed split points); each split
// writes its partial sums, and bwd_router_wgrad_reduce adds them in split
// order.
__global__ void __launch_bounds__(256)
bwd_router_wgrad_kernel(const float *__restrict__ x, const float *__restrict__ dlogit, int T, int d,
                        int E, int xvec, int evec, int chunk, float *__restrict__ part) {
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const int t0 = blockIdx.z * chunk, t1 = min(T, t0 + chunk);
    float acc[4][4];
    gemm_tile<false, false>(x, d, m0, d, xvec, dlogit, E, n0, E, evec, t0, t1, acc);
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    float *p = part + (size_t)blockIdx.z * d * E;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int j = m0 + ty * 4 + i;
        if (j >= d) continue;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int e = n0 + tx * 4 + c;
            if (e < E) p[(size_t)j * E + e] = acc[i][c];
        }
    }
}

__global__ void __launch_bounds__(256)
bwd_router_wgrad_reduce(const float *__restrict__ part, int splits, size_t n,
                        float *__restrict__ g_router) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        float s = part[i];
        for (int z = 1; z < splits; z++) s = __fadd_rn(s, part[(size_t)z * n + i]);
        g_router[i] = __fadd_rn(g_router[i], s);
    }
}

// splits of the router weight gradient's token range (at most kRouterSplits)
int router_wgrad_splits(int T, int d, int E) {
    const int tiles = ceil_div(d, BM) * ceil_div(E, BN);
    int s = ceil_div(2 * 148, tiles);
    s = min(s, kRouterWgradSplits);
    s = min(s, max(1, T / 256));
    return max(1, s);
}

// ---- dx[t] = (Σ_r dX_perm[pos(t, r)], rank order) + the router part already in dx
__global__ void __launch_bounds__(256)
bwd_dx_gather_kernel(const float *__restrict__ dxp, const int *__restrict__ pos_of, int d, int d_pad,
                     int k, float *__restrict__ dx) {
    const int t = blockIdx.x;
    int pos[kMaxTopK];
#pragma unroll
    for (int r = 0; r < kMaxTopK; r++)
        if (r < k) pos[r] = pos_of[(size_t)t * k + r];
    float *o = dx + (size_t)t * d;
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        float acc = __ldg(dxp + (size_t)pos[0] * d_pad + j);
#pragma unroll
        for (int r = 1; r < kMaxTopK; r++)
            if (r < k) acc = __fadd_rn(acc, __ldg(dxp + (size_t)pos[r] * d_pad + j));
        o[j] = __fadd_rn(acc, o[j]);
    }
}

static bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

// combine, renormalisation / aux / softmax backward, column sums, L_aux
cudaError_t launch_bwd_head(const BwdArgs &a, cudaStream_t s, int *n) {
    const int T = a.T, E = a.E, k = a.k;
    bwd_combine_kernel<<<T, 256, 0, s>>>(a.dy, a.y, a.pos_of, a.wts, a.d, a.d_pad, k, a.dw, a.dO,
                                         a.round_tf32);
    const float aux_scale = a.aux_coef * (float)E / ((float)T * (float)T * (float)k);
    const int *cnt = a.plan;
    bwd_router_kernel<<<ceil_div(T, 8), 256, 0, s>>>(a.probs, a.ids, a.wts, a.dw, cnt, T, E, k,
                                                     aux_scale, a.dlogit);
    bwd_colsum_kernel<<<E, 256, 0, s>>>(a.probs, a.dlogit, T, E, a.pmean, a.g_bias);
    *n += 3;
    if (a.aux_loss) {
        bwd_aux_kernel<<<1, 32, 0, s>>>(a.pmean, cnt, T, E, k, a.aux_loss);
        *n += 1;
    }
    return cudaGetLastError();
}

// the expert GEMMs on FP32 FFMA: dH + SwiGLU backward, dWd, dWg / dWu, dX_perm
cudaError_t launch_bwd_ffma_gemms(const BwdArgs &a, cudaStream_t s, int *n) {
    const int E = a.E;
    const int mt = ceil_div(a.rows_bound, BM) + E;
    bwd_dh_kernel<<<dim3(mt, a.F_pad / BN), 256, 0, s>>>(a.dO, a.d_pad, a.dn, a.F_pad, a.gu, a.dgu,
                                                         a.plan, E);
    bwd_wgrad_down_kernel<<<dim3(a.F_pad / BM, a.d_pad / BN, E), 256, 0, s>>>(
        a.h, a.F_pad, a.dO, a.d_pad, a.F, a.d, a.plan, E, a.g_down);
    bwd_wgrad_upgate_kernel<<<dim3(a.d_pad / BM, 2 * a.F_pad / BN, E), 256, 0, s>>>(
        a.x_perm, a.d_pad, a.dgu, a.F_pad, a.d, a.F, a.plan, E, a.g_gate, a.g_up);
    bwd_dxp_kernel<<<dim3(mt, a.d_pad / BN), 256, 0, s>>>(a.dgu, a.F_pad, a.ug, a.d_pad, a.dxp,
                                                          a.plan, E);
    *n += 4;
    return cudaGetLastError();
}

// the router's dx and dW_router, then dx gathered over the ranks
cudaError_t launch_bwd_tail(const BwdArgs &a, cudaStream_t s, int *n) {
    const int T = a.T, E = a.E, k = a.k;
    const int evec = (E % 4 == 0) && aligned16(a.dlogit) && aligned16(a.router);
    bwd_router_dx_kernel<<<dim3(ceil_div(T, BM), ceil_div(a.d, BN)), 256, 0, s>>>(
        a.dlogit, a.router, T, a.d, E, evec, a.dx);
    const int xvec = (a.d % 4 == 0) && aligned16(a.x);
    const int dvec = (E % 4 == 0) && aligned16(a.dlogit);
    const int splits = router_wgrad_splits(T, a.d, E);
    const int chunk = round_up(ceil_div(T, splits), BK);
    const int zs = ceil_div(T, chunk);
    bwd_router_wgrad_kernel<<<dim3(ceil_div(a.d, BM), ceil_div(E, BN), zs), 256, 0, s>>>(
        a.x, a.dlogit, T, a.d, E, xvec, dvec, chunk, a.wr_part);
    const size_t nre = (size_t)a.d * E;
    const int rblocks = (int)((nre + 255) / 256 < 1024 ? (nre + 255) / 256 : 1024);
    bwd_router_wgrad_reduce<<<rblocks, 256, 0, s>>>(a.wr_part, zs, nre, a.g_router);
    *n += 1;
    int threads = 256;
    if (a.d < 256) threads = max(32, round_up(a.d, 32));
    bwd_dx_gather_kernel<<<T, threads, 0, s>>>(a.dxp, a.pos_of, a.d, a.d_pad, k, a.dx);
    *n += 3;
    return cudaGetLastError();
}

cudaError_t launch_moe_backward(const BwdArgs &a, cudaStream_t s, int *launches) {
    int n = 0;
    cudaError_t e = cudaSuccess;
    if (a.T > 0) {
        e = launch_bwd_head(a, s, &n);
        if (e == cudaSuccess) e = launch_bwd_ffma_gemms(a, s, &n);
        if (e == cudaSuccess) e = launch_bwd_tail(a, s, &n);
    }
    if (launches) *launches = n;
    return e;
}

}  // namespace moe
