/*
 * moe_oracle.c — CPU restatement of llm.c's MoE feed-forward forward pass.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Compiled with IEEE semantics
 * (-ffp-contract=off, no fast-math); every fused multiply-add below is an
 * explicit fmaf() where the reference's AVX2+FMA code issues one.
 *
 * Reference functions restated, by file:line of llm.c:
 *   exp_avx2 / sigmoid_avx2 / silu_avx2   src/matrix.c:82-127
 *   softmax_rows                          src/matrix.c:529-586
 *   swiglu                                src/matrix.c:618-655
 *   ffn_forward                           src/transformer.c:157-165
 *   moe_forward                           src/transformer.c:287-366
 *   mat_mul_add (bias broadcast)          src/matrix.c:418-439
 *   rms_norm                              src/matrix.c:666-713
 *   hsum256                               include/simd.h:110-121
 *   block_forward, FFN half               src/transformer.c:752-767
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <stdio.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ========================================================================
 * Synthetic generator (independent restatement of the product's)
 * ===================================================================== */

static inline uint64_t sm64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

static inline uint64_t stream_key(uint64_t seed, uint64_t stream) {
    return sm64(sm64(seed) ^ (stream * 0xD6E8FEB86659FD93ULL));
}

static inline float synth_one(uint64_t key, uint64_t idx, float std) {
    uint32_t s = 0;
    for (int j = 0; j < 3; j++) {
        uint64_t h = sm64(key + 3ULL * idx + (uint64_t)j);
        s += (uint32_t)(h & 0xFFFF) + (uint32_t)((h >> 16) & 0xFFFF) +
             (uint32_t)((h >> 32) & 0xFFFF) + (uint32_t)(h >> 48);
    }
    /* sum of 12 uniforms (u+0.5)/65536 minus 6 == (s - 393210) / 65536,
     * exact in fp32 because |s - 393210| < 2^19. */
    float z = (float)((int32_t)s - 393210) * (1.0f / 65536.0f);
    return z * std;
}

void oracle_synth_normal(uint64_t seed, uint64_t stream, uint64_t first,
                         size_t n, float std, float *dst) {
    uint64_t key = stream_key(seed, stream);
    #pragma omp parallel for schedule(static) if (n > 65536)
    for (size_t i = 0; i < n; i++) dst[i] = synth_one(key, first + i, std);
}

uint64_t oracle_stream_x(void)      { return 1; }
uint64_t oracle_stream_router(void) { return 2; }
uint64_t oracle_stream_bias(void)   { return 3; }
uint64_t oracle_stream_expert(int e, int which) {
    return 0x100ULL + 4ULL * (uint64_t)e + (uint64_t)which;
}

/* ========================================================================
 * exp / sigmoid / silu as the reference computes them
 * ===================================================================== */

/* Coefficients of the degree-6 polynomial for 2^f on [0,1): the
 * reference's table (src/matrix.c:86-92).  They are the Taylor
 * coefficients (ln 2)^i / i! written to ten decimals; the i = 4 entry is one
 * float ulp above the exact Taylor value, so the table is kept as written
 * for bit-exact router probabilities. */
static const float c_exp[7] = {
    1.0000000000f, 0.6931471806f, 0.2402265069f, 0.0555041086f,
    0.0096181292f, 0.0013333558f, 0.0001540353f,
};
static inline void exp_init(void) {}

/* src/matrix.c:82-116 — one lane of exp_avx2. */
float oracle_exp_ref(float v) {
    exp_init();
    const float log2e = 1.4426950408f;
    if (v < -88.0f) v = -88.0f;   /* _mm256_max_ps(v, -88) */
    if (v >  88.0f) v =  88.0f;   /* _mm256_min_ps(.., 88) */
    float z  = v * log2e;
    float n  = floorf(z);
    float f  = z - n;
    float p  = c_exp[6];
    for (int i = 5; i >= 0; i--) p = fmaf(p, f, c_exp[i]);
    int32_t ni = (int32_t)lrintf(n);
    uint32_t bits = (uint32_t)(ni + 127) << 23;
    float scale;
    memcpy(&scale, &bits, sizeof scale);
    return p * scale;
}

/* sigmoid_avx2 / silu_avx2 (src/matrix.c:118-127). */
static inline float sigmoid_ref(float v) {
    return 1.0f / (1.0f + oracle_exp_ref(-v));
}
static inline float silu_ref(float v) { return v * sigmoid_ref(v); }

/* ========================================================================
 * softmax_rows (src/matrix.c:529-586, the SIMD_AVX2FMA branch)
 * ===================================================================== */

static void softmax_row(float *row, int cols) {
    int nv = cols - cols % 8;          /* columns handled 8-wide */
    /* step 1: max (order-independent) */
    float row_max = -1e38f;
    for (int j = 0; j < nv; j++) if (row[j] > row_max) row_max = row[j];
    if (nv == 0) row_max = -1e38f;
    for (int j = nv; j < cols; j++) if (row[j] > row_max) row_max = row[j];

    /* step 2: exp and lane-wise partial sums */
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < nv; j++) {
        float ex = oracle_exp_ref(row[j] - row_max);
        row[j] = ex;
        lane[j % 8] = lane[j % 8] + ex;
    }
    /* hsum256: (l0+l4 + l1+l5) + (l2+l6 + l3+l7) */
    float a0 = lane[0] + lane[4], a1 = lane[1] + lane[5];
    float a2 = lane[2] + lane[6], a3 = lane[3] + lane[7];
    float sum = (a0 + a1) + (a2 + a3);
    for (int j = nv; j < cols; j++) {
        row[j] = expf(row[j] - row_max);
        sum += row[j];
    }

    /* step 3: normalise — vector part by reciprocal, tail by division */
    float inv = 1.0f / sum;
    for (int j = 0; j < nv; j++) row[j] = row[j] * inv;
    for (int j = nv; j < cols; j++) row[j] = row[j] / sum;
}

void oracle_softmax_rows(float *m, int rows, int cols) {
    for (int i = 0; i < rows; i++) softmax_row(m + (size_t)i * cols, cols);
}

/* swiglu (src/matrix.c:618-655): vector part silu_avx2(g)*u, scalar tail
 * g/(1+expf(-g))*u. */
void oracle_swiglu(const float *g, const float *u, float *h, int n) {
    int nv = n - n % 8;
    for (int i = 0; i < nv; i++) h[i] = silu_ref(g[i]) * u[i];
    for (int i = nv; i < n; i++) h[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
}

/* ========================================================================
 * Router: logits, softmax, top-k, renormalisation
 * ===================================================================== */

/* Top-k selection (src/transformer.c:318-332): k passes, strict '>', the
 * scan starts at best = -1, best_e = 0 and runs e ascending, skipping ids
 * already taken — so ties go to the lower expert index. */
static void topk_select(const float *probs, int E, int k, int *ids) {
    for (int ki = 0; ki < k; ki++) {
        float best = -1.0f;
        int best_e = 0;
        for (int e = 0; e < E; e++) {
            int already = 0;
            for (int kj = 0; kj < ki; kj++)
                if (ids[kj] == e) { already = 1; break; }
            if (!already && probs[e] > best) { best = probs[e]; best_e = e; }
        }
        ids[ki] = best_e;
    }
}

/* Renormalised weights (src/transformer.c:334-337,350). */
static void renorm(const float *probs, const int *ids, int k, float *w) {
    float s = 0.0f;
    for (int r = 0; r < k; r++) s += probs[ids[r]];
    float inv = (s > 1e-9f) ? 1.0f / s : 0.0f;
    for (int r = 0; r < k; r++) w[r] = probs[ids[r]] * inv;
}

void oracle_router(const float *x, int T, int d,
                   const float *W_router, const float *bias, int E, int k,
                   float *logits_out, float *probs, int *ids, float *wts) {
    exp_init();
    #pragma omp parallel for schedule(static)
    for (int t = 0; t < T; t++) {
        double acc[256];
        float row[256];
        const float *xt = x + (size_t)t * d;
        for (int e = 0; e < E; e++) acc[e] = 0.0;
        for (int i = 0; i < d; i++) {
            double xi = (double)xt[i];
            const float *wr = W_router + (size_t)i * E;
            for (int e = 0; e < E; e++) acc[e] += xi * (double)wr[e];
        }
        for (int e = 0; e < E; e++) {
            row[e] = (float)acc[e];
            if (bias) row[e] = row[e] + bias[e];
        }
        if (logits_out) memcpy(logits_out + (size_t)t * E, row, E * sizeof(float));
        softmax_row(row, E);
        if (probs) memcpy(probs + (size_t)t * E, row, E * sizeof(float));
        int tid[64];
        float tw[64];
        topk_select(row, E, k, tid);
        renorm(row, tid, k, tw);
        if (ids) memcpy(ids + (size_t)t * k, tid, k * sizeof(int));
        if (wts) memcpy(wts + (size_t)t * k, tw, k * sizeof(float));
    }
}

/* ========================================================================
 * Expert FFN
 * ===================================================================== */

/* One token through one expert: y = (silu(x·Wg) ⊙ (x·Wu)) · Wd, with fp64
 * accumulation rounded to fp32 where the reference stores fp32 matrices
 * (gate_buf, up_buf, h, expert_out). */
static void ffn_token(const float *xt, int d, const float *Wg, const float *Wu,
                      const float *Wd, int F, float *y,
                      double *dg, double *du, float *g, float *u, float *h,
                      double *dy) {
    for (int f = 0; f < F; f++) { dg[f] = 0.0; du[f] = 0.0; }
    for (int i = 0; i < d; i++) {
        double xi = (double)xt[i];
        const float *wg = Wg + (size_t)i * F;
        const float *wu = Wu + (size_t)i * F;
        for (int f = 0; f < F; f++) {
            dg[f] += xi * (double)wg[f];
            du[f] += xi * (double)wu[f];
        }
    }
    for (int f = 0; f < F; f++) { g[f] = (float)dg[f]; u[f] = (float)du[f]; }
    oracle_swiglu(g, u, h, F);
    for (int j = 0; j < d; j++) dy[j] = 0.0;
    for (int f = 0; f < F; f++) {
        double hf = (double)h[f];
        const float *wd = Wd + (size_t)f * d;
        for (int j = 0; j < d; j++) dy[j] += hf * (double)wd[j];
    }
    for (int j = 0; j < d; j++) y[j] = (float)dy[j];
}

typedef struct {
    double *dg, *du, *dy;
    float *g, *u, *h;
} ffn_scratch;

static ffn_scratch scratch_alloc(int d, int F) {
    ffn_scratch s;
    s.dg = (double *)malloc((size_t)F * sizeof(double));
    s.du = (double *)malloc((size_t)F * sizeof(double));
    s.dy = (double *)malloc((size_t)d * sizeof(double));
    s.g  = (float *)malloc((size_t)F * sizeof(float));
    s.u  = (float *)malloc((size_t)F * sizeof(float));
    s.h  = (float *)malloc((size_t)F * sizeof(float));
    if (!s.dg || !s.du || !s.dy || !s.g || !s.u || !s.h) {
        fprintf(stderr, "[oracle] OOM\n");
        abort();
    }
    return s;
}

static void scratch_free(ffn_scratch *s) {
    free(s->dg); free(s->du); free(s->dy); free(s->g); free(s->u); free(s->h);
}

void oracle_ffn_forward(const float *x, int n, int d,
                        const float *W_gate, const float *W_up,
                        const float *W_down, int F, float *out) {
    exp_init();
    #pragma omp parallel
    {
        ffn_scratch s = scratch_alloc(d, F);
        #pragma omp for schedule(static)
        for (int t = 0; t < n; t++)
            ffn_token(x + (size_t)t * d, d, W_gate, W_up, W_down, F,
                      out + (size_t)t * d, s.dg, s.du, s.g, s.u, s.h, s.dy);
        scratch_free(&s);
    }
}

/* Combine (src/transformer.c:296,355-358): out starts at zero and adds
 * w_r * y_r for r = 0..k-1 in rank order with one fused multiply-add. */
static void combine_row(const float *y /*[k×d]*/, const float *w, int k, int d,
                        float *out) {
    for (int j = 0; j < d; j++) out[j] = 0.0f;
    for (int r = 0; r < k; r++)
        for (int j = 0; j < d; j++)
            out[j] = fmaf(w[r], y[(size_t)r * d + j], out[j]);
}

/* Shared driver: route all T tokens, then evaluate the selected rows with
 * an expert-weight provider. */
typedef void (*expert_provider)(void *ctx, int e, const float **wg,
                                const float **wu, const float **wd);

static void moe_forward_common(const float *x, int T, int d,
                               const float *W_router, const float *bias,
                               int E, int k, int F,
                               expert_provider prov, void *prov_ctx,
                               void (*prov_release)(void *ctx, int e),
                               const int *rows, int n_rows,
                               const int *forced_ids,
                               float *out, float *probs, int *ids,
                               int threads) {
    exp_init();
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    float *p_all = (float *)malloc((size_t)T * E * sizeof(float));
    int *id_all  = (int *)malloc((size_t)T * k * sizeof(int));
    if (!p_all || !id_all) { fprintf(stderr, "[oracle] OOM\n"); abort(); }
    oracle_router(x, T, d, W_router, bias, E, k, NULL, p_all, id_all, NULL);
    if (probs) memcpy(probs, p_all, (size_t)T * E * sizeof(float));
    if (ids) memcpy(ids, id_all, (size_t)T * k * sizeof(int));

    int nr = rows ? n_rows : T;
    const int *use_ids = forced_ids ? forced_ids : id_all;
    float *ysel = (float *)malloc((size_t)nr * k * d * sizeof(float));
    float *wsel = (float *)malloc((size_t)nr * k * sizeof(float));
    if (!ysel || !wsel) { fprintf(stderr, "[oracle] OOM\n"); abort(); }
    for (int i = 0; i < nr; i++) {
        int t = rows ? rows[i] : i;
        renorm(p_all + (size_t)t * E, use_ids + (size_t)t * k, k,
               wsel + (size_t)i * k);
    }
    /* expert by expert, so a provider may materialise one expert at a time */
    for (int e = 0; e < E; e++) {
        int any = 0;
        for (int i = 0; i < nr && !any; i++) {
            int t = rows ? rows[i] : i;
            for (int r = 0; r < k; r++)
                if (use_ids[(size_t)t * k + r] == e) { any = 1; break; }
        }
        if (!any) continue;
        const float *wg, *wu, *wd;
        prov(prov_ctx, e, &wg, &wu, &wd);
        #pragma omp parallel
        {
            ffn_scratch s = scratch_alloc(d, F);
            #pragma omp for schedule(dynamic, 1)
            for (int i = 0; i < nr; i++) {
                int t = rows ? rows[i] : i;
                for (int r = 0; r < k; r++) {
                    if (use_ids[(size_t)t * k + r] != e) continue;
                    ffn_token(x + (size_t)t * d, d, wg, wu, wd, F,
                              ysel + ((size_t)i * k + r) * d,
                              s.dg, s.du, s.g, s.u, s.h, s.dy);
                }
            }
            scratch_free(&s);
        }
        if (prov_release) prov_release(prov_ctx, e);
    }
    for (int i = 0; i < nr; i++)
        combine_row(ysel + (size_t)i * k * d, wsel + (size_t)i * k, k, d,
                    out + (size_t)i * d);
    free(ysel); free(wsel); free(p_all); free(id_all);
}

typedef struct {
    const float *const *wg, *const *wu, *const *wd;
} host_ctx;

static void host_provider(void *c, int e, const float **wg, const float **wu,
                          const float **wd) {
    host_ctx *h = (host_ctx *)c;
    *wg = h->wg[e]; *wu = h->wu[e]; *wd = h->wd[e];
}

void oracle_moe_forward(const float *x, int T, int d,
                        const float *W_router, const float *bias,
                        int E, int k,
                        const float *const *W_gate,
                        const float *const *W_up,
                        const float *const *W_down, int F,
                        const int *rows, int n_rows,
                        const int *forced_ids,
                        float *out, float *probs, int *ids, int threads) {
    host_ctx h = { W_gate, W_up, W_down };
    moe_forward_common(x, T, d, W_router, bias, E, k, F, host_provider, &h,
                       NULL, rows, n_rows, forced_ids, out, probs, ids,
                       threads);
}

typedef struct {
    uint64_t seed;
    float std;
    int d, F;
    float *wg, *wu, *wd;
} synth_ctx;

static void synth_provider(void *c, int e, const float **wg, const float **wu,
                           const float **wd) {
    synth_ctx *s = (synth_ctx *)c;
    size_t n = (size_t)s->d * s->F;
    oracle_synth_normal(s->seed, oracle_stream_expert(e, 0), 0, n, s->std, s->wg);
    oracle_synth_normal(s->seed, oracle_stream_expert(e, 1), 0, n, s->std, s->wu);
    oracle_synth_normal(s->seed, oracle_stream_expert(e, 2), 0, n, s->std, s->wd);
    *wg = s->wg; *wu = s->wu; *wd = s->wd;
}

void oracle_moe_forward_synth(const float *x, int T, int d,
                              const float *W_router, const float *bias,
                              int E, int k, int F,
                              uint64_t seed, float w_std,
                              const int *rows, int n_rows,
                              const int *forced_ids,
                              float *out, float *probs, int *ids, int threads) {
    synth_ctx s;
    size_t n = (size_t)d * F;
    s.seed = seed; s.std = w_std; s.d = d; s.F = F;
    s.wg = (float *)malloc(n * sizeof(float));
    s.wu = (float *)malloc(n * sizeof(float));
    s.wd = (float *)malloc(n * sizeof(float));
    if (!s.wg || !s.wu || !s.wd) { fprintf(stderr, "[oracle] OOM\n"); abort(); }
    moe_forward_common(x, T, d, W_router, bias, E, k, F, synth_provider, &s,
                       NULL, rows, n_rows, forced_ids, out, probs, ids,
                       threads);
    free(s.wg); free(s.wu); free(s.wd);
}

/* ========================================================================
 * RMSNorm and the FFN half of block_forward
 * ===================================================================== */

/* hsum256 (include/simd.h:110-121): upper half added to lower half, then
 * (s0 + s1) + (s2 + s3). */
static float hsum8(const float *l) {
    const float s0 = l[0] + l[4], s1 = l[1] + l[5], s2 = l[2] + l[6], s3 = l[3] + l[7];
    return (s0 + s1) + (s2 + s3);
}

void oracle_rms_norm(const float *x, int rows, int cols, const float *weight, float eps,
                     float *out) {
    for (int i = 0; i < rows; i++) {
        const float *xr = x + (size_t)i * cols;
        float *yr = out + (size_t)i * cols;
        float a[16] = {0};
        int j = 0;
        for (; j <= cols - 16; j += 16)
            for (int l = 0; l < 16; l++) a[l] = fmaf(xr[j + l], xr[j + l], a[l]);
        float b[8];
        for (int l = 0; l < 8; l++) b[l] = a[l] + a[l + 8];
        for (; j <= cols - 8; j += 8)
            for (int l = 0; l < 8; l++) b[l] = fmaf(xr[j + l], xr[j + l], b[l]);
        float ss = hsum8(b);
        for (; j < cols; j++) ss += xr[j] * xr[j];
        const float inv = 1.0f / sqrtf(ss / (float)cols + eps);
        for (int c = 0; c < cols; c++) yr[c] = xr[c] * inv * weight[c];
    }
}

void oracle_block_ffn(float *x, int T, int d, const float *rms_weight, float eps,
                      const float *W_router, const float *bias, int E, int k, int F,
                      const float *const *W_gate, const float *const *W_up,
                      const float *const *W_down, float *xn, float *probs, int *ids,
                      int threads) {
    const size_t n = (size_t)T * d;
    float *norm = xn ? xn : (float *)malloc(n * sizeof(float));
    float *ffn = (float *)malloc(n * sizeof(float));
    if (!norm || !ffn) { fprintf(stderr, "[oracle] OOM\n"); abort(); }
    oracle_rms_norm(x, T, d, rms_weight, eps, norm);
    oracle_moe_forward(norm, T, d, W_router, bias, E, k, W_gate, W_up, W_down, F, NULL, T, NULL,
                       ffn, probs, ids, threads);
    for (size_t i = 0; i < n; i++) x[i] = x[i] + ffn[i];
    free(ffn);
    if (!xn) free(norm);
}
