/*
 * ref_driver.c — flat C entry points into the UNMODIFIED reference
 * sources (llm.c src/matrix.c, src/attention.c, src/transformer.c),
 * compiled together into oracle/_ref/libllmref.so by oracle/Makefile.
 *
 * TEST INFRASTRUCTURE ONLY.  The functions only build the reference's own
 * structs (include/matrix.h:33-38, include/transformer.h:35-58,121-123,
 * include/config.h:23-48) around caller buffers and call the reference:
 *   ref_moe_forward   -> moe_forward      (src/transformer.c:287-366)
 *   ref_softmax_rows  -> softmax_rows     (src/matrix.c:529-586)
 *   ref_swiglu        -> swiglu           (src/matrix.c:618-655)
 *   ref_ffn_forward   -> ffn_forward      (src/transformer.c:157-165)
 *   ref_ffn_backward  -> ffn_backward     (src/transformer.c:181-264)
 *   ref_model_*       -> model_init / model_forward / model_free
 *                        (src/transformer.c:475-802), with srand(seed)
 *   ref_inference_*   -> inference_init / inference_step (src/inference.c)
 */
#include <stdlib.h>
#include <string.h>
#include "transformer.h"
#ifdef _OPENMP
#include <omp.h>
#endif

void scipy_openblas_set_num_threads64_(int n);

void ref_set_threads(int n) {
#ifdef _OPENMP
    omp_set_num_threads(n);
#endif
    scipy_openblas_set_num_threads64_(n);
}

int ref_moe_forward(const float *x, int T, int d, const float *W_router,
                    int E, int k, const float *const *W_gate,
                    const float *const *W_up, const float *const *W_down,
                    int F, float *out, float *probs, int *ids) {
    FFNWeights *ex = (FFNWeights *)calloc((size_t)E, sizeof(FFNWeights));
    if (!ex) return -1;
    for (int e = 0; e < E; e++) {
        ex[e].W_gate = (Matrix){ (float *)W_gate[e], NULL, d, F };
        ex[e].W_up   = (Matrix){ (float *)W_up[e],   NULL, d, F };
        ex[e].W_down = (Matrix){ (float *)W_down[e], NULL, F, d };
    }
    MoEWeights mw;
    mw.experts   = ex;
    mw.W_router  = (Matrix){ (float *)W_router, NULL, d, E };
    mw.n_experts = E;
    mw.top_k     = k;
    ModelConfig cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.d_model = d;
    cfg.ffn_hidden = F;
    cfg.n_experts = E;
    cfg.top_k_experts = k;
    ForwardCache cache;
    memset(&cache, 0, sizeof cache);
    cache.router_probs = probs;
    cache.expert_ids = ids;
    Matrix xm = { (float *)x, NULL, T, d };
    Matrix om = { out, NULL, T, d };
    moe_forward(&xm, &mw, &cfg, &cache, &om);
    free(ex);
    return 0;
}

void ref_softmax_rows(float *m, int rows, int cols) {
    Matrix mm = { m, NULL, rows, cols };
    softmax_rows(&mm);
}

void ref_swiglu(const float *g, const float *u, float *h, int n) {
    Matrix gm = { (float *)g, NULL, 1, n };
    Matrix um = { (float *)u, NULL, 1, n };
    Matrix hm = { h, NULL, 1, n };
    swiglu(&gm, &um, &hm);
}

/* the reference's dense SwiGLU backward (ffn_backward, src/transformer.c:
 * 181-264) at x: the saved gate/up pre-activations and h are made with the
 * reference's own mat_mul and swiglu; weight gradients accumulate into dWg,
 * dWu, dWd (llm.c's convention), d_x is overwritten */
void ref_ffn_backward(const float *x, int n, int d, const float *Wg, const float *Wu,
                      const float *Wd, int F, const float *d_out, float *dWg, float *dWu,
                      float *dWd, float *d_x) {
    FFNWeights w;
    w.W_gate = (Matrix){ (float *)Wg, dWg, d, F };
    w.W_up   = (Matrix){ (float *)Wu, dWu, d, F };
    w.W_down = (Matrix){ (float *)Wd, dWd, F, d };
    Matrix xm = { (float *)x, NULL, n, d };
    Matrix gp = mat_alloc(n, F, 0), up = mat_alloc(n, F, 0), h = mat_alloc(n, F, 0);
    mat_mul(&xm, &w.W_gate, &gp);
    mat_mul(&xm, &w.W_up, &up);
    swiglu(&gp, &up, &h);
    Matrix dom = { (float *)d_out, NULL, n, d };
    Matrix dxm = { d_x, NULL, n, d };
    ffn_backward(&xm, &w, &gp, &up, &h, &dom, &dxm);
    mat_free(&gp);
    mat_free(&up);
    mat_free(&h);
}

void ref_ffn_forward(const float *x, int n, int d, const float *Wg,
                     const float *Wu, const float *Wd, int F, float *out) {
    FFNWeights w;
    w.W_gate = (Matrix){ (float *)Wg, NULL, d, F };
    w.W_up   = (Matrix){ (float *)Wu, NULL, d, F };
    w.W_down = (Matrix){ (float *)Wd, NULL, F, d };
    ModelConfig cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.d_model = d;
    cfg.ffn_hidden = F;
    Matrix gb = mat_alloc(n, F, 0), ub = mat_alloc(n, F, 0);
    Matrix xm = { (float *)x, NULL, n, d };
    Matrix om = { out, NULL, n, d };
    ffn_forward(&xm, &w, &cfg, &gb, &ub, &om);
    mat_free(&gb);
    mat_free(&ub);
}

/* ---- whole-model entry points for the decode (config 2) oracle --------- */
#include "inference.h"

void *ref_model_init(int vocab, int max_seq, int d, int n_layers, int n_heads, int n_kv,
                     int head_dim, int window, int ffn, int n_experts, int top_k, float eps,
                     float theta, unsigned seed) {
    ModelConfig cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.vocab_size = vocab; cfg.max_seq_len = max_seq; cfg.d_model = d;
    cfg.n_layers = n_layers; cfg.n_heads = n_heads; cfg.n_kv_heads = n_kv;
    cfg.head_dim = head_dim; cfg.window_size = window; cfg.ffn_hidden = ffn;
    cfg.n_experts = n_experts; cfg.top_k_experts = top_k; cfg.rms_norm_eps = eps;
    cfg.rope_theta = theta;
    srand(seed);
    return model_init(&cfg);
}

void ref_model_free(void *m) { model_free((Model *)m); }

/* logits of the last position of model_forward over tokens[0..n) */
void ref_model_forward_last(void *mp, const int *tokens, int n, float *logits_last) {
    Model *m = (Model *)mp;
    int V = m->cfg.vocab_size;
    Matrix lg = mat_alloc(n, V, 0);
    model_forward(m, tokens, n, &lg);
    memcpy(logits_last, lg.data + (size_t)(n - 1) * V, (size_t)V * sizeof(float));
    mat_free(&lg);
}

void *ref_inference_init(void *m) { return inference_init((const Model *)m); }
void ref_inference_free(void *s) { inference_free((InferenceState *)s); }
void ref_inference_step(void *m, void *s, int token) {
    inference_step((const Model *)m, (InferenceState *)s, token);
}
float *ref_inference_logits(void *s) { return ((InferenceState *)s)->logits; }
int ref_inference_pos(void *s) { return ((InferenceState *)s)->seq_pos; }

/* llm.c's own checkpoint format (model_save / model_load, src/transformer.c:573-697) */
int ref_model_save(void *m, const char *path) { return model_save((const Model *)m, path); }
void *ref_model_load(const char *path) { return model_load(path); }

/* the reference's rms_norm (src/matrix.c:666-713) over plain arrays */
void ref_rms_norm(const float *x, int rows, int cols, const float *weight, float eps,
                  float *out) {
    Matrix in = {(float *)x, NULL, rows, cols};
    Matrix o = {out, NULL, rows, cols};
    rms_norm(&in, weight, eps, &o);
}

/* logits of positions [first, n) of model_forward over tokens[0..n)
 * (rows = n - first, row-major into `out`) */
void ref_model_forward_rows(void *mp, const int *tokens, int n, int first, float *out) {
    Model *m = (Model *)mp;
    int V = m->cfg.vocab_size;
    Matrix lg = mat_alloc(n, V, 0);
    model_forward(m, tokens, n, &lg);
    memcpy(out, lg.data + (size_t)first * V, (size_t)(n - first) * V * sizeof(float));
    mat_free(&lg);
}

/* the reference's moe_forward with block `layer`'s own MoE weights of a
 * Model (src/transformer.c:287-366) on x [T×d]; probs / ids may be NULL */
int ref_model_moe_forward(void *mp, int layer, const float *x, int T, float *out, float *probs,
                          int *ids) {
    Model *m = (Model *)mp;
    if (layer < 0 || layer >= m->cfg.n_layers || !m->weights.blocks[layer].use_moe) return -1;
    const MoEWeights *mw = &m->weights.blocks[layer].moe;
    const int d = m->cfg.d_model, E = mw->n_experts, k = mw->top_k;
    float *pb = probs ? probs : (float *)malloc((size_t)T * E * sizeof(float));
    int *ib = ids ? ids : (int *)malloc((size_t)T * k * sizeof(int));
    if (!pb || !ib) return -1;
    ForwardCache cache;
    memset(&cache, 0, sizeof cache);
    cache.router_probs = pb;
    cache.expert_ids = ib;
    Matrix xm = { (float *)x, NULL, T, d };
    Matrix om = { out, NULL, T, d };
    moe_forward(&xm, mw, &m->cfg, &cache, &om);
    if (!probs) free(pb);
    if (!ids) free(ib);
    return 0;
}
