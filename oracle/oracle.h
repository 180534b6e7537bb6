/*
 * oracle.h — CPU test oracle for the MoE feed-forward hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this code: only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg use it, and only as the checker.
 *
 * Two independent pieces live here:
 *   1. A restatement of the reference's MoE forward
 *      (llm.c src/transformer.c:287-366) in plain C, with IEEE arithmetic,
 *      fp64 accumulation for the products, and the reference's own softmax,
 *      top-k selection, renormalisation, SwiGLU and combine order.  It adds
 *      an optional router bias (logits += b before the softmax), as
 *      mat_mul_add (src/matrix.c:418-439) would apply it.
 *   2. The seeded synthetic input generator (counter-based, bit-identical
 *      on host and device), restated independently of the product's CUDA
 *      copy so the two can be checked against each other.
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- synthetic inputs -------------------------------------------------- */

/* Fill dst[0..n) with approx-N(0, std) values of stream `stream` under
 * `seed`, starting at element index `first`.  Element i is a pure
 * function of (seed, stream, first + i): Irwin–Hall sum of twelve 16-bit
 * uniforms drawn from three splitmix64 hashes, scaled exactly by 2^-16,
 * then one fp32 multiply by std. */
void oracle_synth_normal(uint64_t seed, uint64_t stream, uint64_t first,
                         size_t n, float std, float *dst);

/* Stream ids shared with the product generator. */
uint64_t oracle_stream_x(void);
uint64_t oracle_stream_router(void);
uint64_t oracle_stream_bias(void);
uint64_t oracle_stream_expert(int expert, int which /*0 gate,1 up,2 down*/);

/* ---- reference restatement --------------------------------------------- */

/* exp as the reference's softmax/silu compute it (src/matrix.c:82-116):
 * clamp to [-88, 88], 2^n * P6(f) with P6 the degree-6 Taylor polynomial
 * of 2^f, Horner with fused multiply-adds. */
float oracle_exp_ref(float v);

/* softmax_rows restated (src/matrix.c:529-586, AVX2+FMA build): lane-wise
 * 8-way partial sums over the first 8*floor(cols/8) columns, hsum tree,
 * scalar libm tail, multiply by 1/sum on the vector part and divide on
 * the tail. In place on m[rows × cols]. */
void oracle_softmax_rows(float *m, int rows, int cols);

/* rms_norm restated (src/matrix.c:666-713, AVX2+FMA build), per row of
 * x[rows × cols]: sum of squares in 16 fused-multiply-add lanes over
 * 16-column chunks, lanes j and j+8 added, further 8-column chunks fused
 * into those 8 lanes, hsum tree, scalar tail (multiply, then add);
 * inv = 1 / sqrt(ss / cols + eps); out = (x * inv) * weight. */
void oracle_rms_norm(const float *x, int rows, int cols, const float *weight, float eps,
                     float *out);

/* The FFN half of block_forward (src/transformer.c:752-767) for a MoE
 * block: xn = rms_norm(x, rms_weight); x += moe_forward(xn), the add
 * being mat_add_inplace's (src/matrix.c:491-500).  x is updated in place;
 * xn (T×d, may be NULL), probs and ids as oracle_moe_forward. */
void oracle_block_ffn(float *x, int T, int d, const float *rms_weight, float eps,
                      const float *W_router, const float *bias, int E, int k, int F,
                      const float *const *W_gate, const float *const *W_up,
                      const float *const *W_down, float *xn, float *probs, int *ids,
                      int threads);

/* swiglu restated (src/matrix.c:618-655): h = silu(g) * u elementwise. */
void oracle_swiglu(const float *g, const float *u, float *h, int n);

/* Router only: logits (+bias), softmax, top-k ids (rank order) and the
 * renormalised weights (src/transformer.c:299-337,350).
 * probs [T×E], ids [T×k], wts [T×k] (any may be NULL except ids/wts when
 * needed by the caller). logits_out [T×E] optional (pre-softmax). */
void oracle_router(const float *x, int T, int d,
                   const float *W_router, const float *bias, int E, int k,
                   float *logits_out, float *probs, int *ids, float *wts);

/* Full MoE forward for a subset of rows.
 *   x        [T×d] row-major
 *   W_router [d×E]; bias [E] or NULL
 *   W_gate[e], W_up[e] [d×F]; W_down[e] [F×d]  (reference host layout)
 *   rows     token indices to evaluate (NULL = all T, n_rows ignored)
 *   forced_ids [T×k] or NULL: use these expert ids instead of the
 *              oracle's own top-k (to check the expert math on a token
 *              whose routing legitimately differs at a near-tie)
 *   out      [n_rows×d] (or [T×d] when rows == NULL)
 *   probs    [T×E] or NULL; ids [T×k] or NULL (full T always)
 *   threads  OpenMP threads (<=0: runtime default)
 */
void oracle_moe_forward(const float *x, int T, int d,
                        const float *W_router, const float *bias,
                        int E, int k,
                        const float *const *W_gate,
                        const float *const *W_up,
                        const float *const *W_down, int F,
                        const int *rows, int n_rows,
                        const int *forced_ids,
                        float *out, float *probs, int *ids, int threads);

/* Same as oracle_moe_forward but the expert weights are regenerated on the
 * fly from the synthetic generator (seed, oracle_stream_expert(e, ·), std),
 * one expert at a time, so configurations whose weights do not fit in host
 * memory can still be checked on a row subset.  x, W_router and bias are
 * passed in. */
void oracle_moe_forward_synth(const float *x, int T, int d,
                              const float *W_router, const float *bias,
                              int E, int k, int F,
                              uint64_t seed, float w_std,
                              const int *rows, int n_rows,
                              const int *forced_ids,
                              float *out, float *probs, int *ids, int threads);

/* Single-expert dense SwiGLU FFN on n rows (src/transformer.c:157-165). */
void oracle_ffn_forward(const float *x, int n, int d,
                        const float *W_gate, const float *W_up,
                        const float *W_down, int F, float *out);

#ifdef __cplusplus
}
#endif
#endif
