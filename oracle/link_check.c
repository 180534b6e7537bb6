/*
 * link_check.c — a minimal llm.c program, linked two ways by oracle/Makefile
 * (TEST INFRASTRUCTURE ONLY):
 *
 *   _ref/link_ref    against the UNMODIFIED reference library alone
 *                    (oracle/_ref/libllmref.so: src/matrix.c, attention.c,
 *                    inference.c, tokenizer.c, transformer.c built -fPIC);
 *   _ref/link_b200   against libmoe_b200.so FIRST and then the same
 *                    reference library: the binding a maintainer adds.  The
 *                    reference objects are position-independent, so
 *                    block_forward's call to moe_forward (src/transformer.c:
 *                    761-764) goes through the PLT and binds to the first
 *                    definition in load order, libmoe_b200.so's; so does this
 *                    program's call to inference_step (include/inference.h:137).
 *
 * It builds a MoE model with the reference's model_init (srand seed), runs
 * the reference's model_forward over a fixed token sequence and, on a fresh
 * InferenceState, inference_step over the same tokens, and writes
 *   int32 T, int32 V, float logits[T][V] (model_forward),
 *   float logits[V] (after the last inference_step)
 * to the output file.  With -DWITH_B200 it also prints how many kernels the
 * library launched in its last call, which is non-zero only if the
 * interposed moe_forward ran.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "inference.h"
#include "transformer.h"

#ifdef WITH_B200
int moe_b200_last_launches(void);
int moe_b200_last_path(void);
#endif

int main(int argc, char **argv) {
    if (argc != 2) {
        fprintf(stderr, "usage: %s out.bin\n", argv[0]);
        return 2;
    }
    ModelConfig cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.vocab_size = 512; cfg.max_seq_len = 64; cfg.d_model = 256; cfg.n_layers = 2;
    cfg.n_heads = 4; cfg.n_kv_heads = 2; cfg.head_dim = 64; cfg.window_size = 0;
    cfg.ffn_hidden = 512; cfg.n_experts = 8; cfg.top_k_experts = 2;
    cfg.rms_norm_eps = 1e-5f; cfg.rope_theta = 1e4f;
    srand(7);
    Model *m = model_init(&cfg);
    const int T = 48, V = cfg.vocab_size;
    int tokens[48];
    unsigned s = 12345u;
    for (int i = 0; i < T; i++) {
        s = s * 1664525u + 1013904223u;
        tokens[i] = (int)((s >> 8) % (unsigned)V);
    }
    Matrix lg = mat_alloc(T, V, 0);
    model_forward(m, tokens, T, &lg);
#ifdef WITH_B200
    printf("model_forward: b200_launches=%d b200_path=%d\n", moe_b200_last_launches(),
           moe_b200_last_path());
#endif
    InferenceState *st = inference_init(m);
    for (int i = 0; i < T; i++) inference_step(m, st, tokens[i]);
#ifdef WITH_B200
    printf("inference_step: b200_launches=%d b200_path=%d\n", moe_b200_last_launches(),
           moe_b200_last_path());
#endif
    FILE *f = fopen(argv[1], "wb");
    if (!f) return 1;
    const int hdr[2] = {T, V};
    int ok = fwrite(hdr, sizeof hdr, 1, f) == 1 &&
             fwrite(lg.data, sizeof(float), (size_t)T * V, f) == (size_t)T * V &&
             fwrite(st->logits, sizeof(float), (size_t)V, f) == (size_t)V;
    fclose(f);
    inference_free(st);
    mat_free(&lg);
    model_free(m);
    return ok ? 0 : 1;
}
