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
