/*
 * llmc_moe.h — llm.c's own MoE entry point, exported by libmoe_b200.so as
 * a drop-in replacement.
 *
 * The structs below restate llm.c's types field for field (same order,
 * same C types), so a pointer to llm.c's own struct can be passed where
 * these are expected.  The layouts have to be identical for the drop-in to
 * work; the names carry an llmc_ prefix so this header can be included
 * next to llm.c's headers.
 *   llmc_Matrix        == Matrix        include/matrix.h:33-38
 *   llmc_FFNWeights    == FFNWeights    include/transformer.h:35-39
 *   llmc_MoEWeights    == MoEWeights    include/transformer.h:53-58
 *   llmc_ModelConfig   == ModelConfig   include/config.h:23-48
 *   llmc_ForwardCache  == ForwardCache  include/transformer.h:107-124
 */
#ifndef LLMC_MOE_H
#define LLMC_MOE_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    float *data;
    float *grad;
    int rows;
    int cols;
} llmc_Matrix;

typedef struct {
    llmc_Matrix W_gate;
    llmc_Matrix W_up;
    llmc_Matrix W_down;
} llmc_FFNWeights;

typedef struct {
    llmc_FFNWeights *experts;
    llmc_Matrix W_router;
    int n_experts;
    int top_k;
} llmc_MoEWeights;

typedef struct {
    int vocab_size;
    int max_seq_len;
    int d_model;
    int n_layers;
    int n_heads;
    int n_kv_heads;
    int head_dim;
    int window_size;
    int ffn_hidden;
    int n_experts;
    int top_k_experts;
    float rms_norm_eps;
    float rope_theta;
} llmc_ModelConfig;

typedef struct {
    llmc_Matrix x_norm_attn;
    llmc_Matrix x_norm_ffn;
    llmc_Matrix attn_out;
    llmc_Matrix ffn_out;
    llmc_Matrix Q, K, V;
    llmc_Matrix attn_scores;
    llmc_Matrix attn_weighted;
    llmc_Matrix gate_buf;
    llmc_Matrix up_buf;
    float *router_probs;
    int *expert_ids;
} llmc_ForwardCache;

/*
 * moe_forward — replaces llm.c's moe_forward (src/transformer.c:287-366,
 * declared at include/transformer.h:270-272) with the same signature and
 * semantics: reads x [rows × cols] and the host MoE weights, overwrites
 * out [rows × cols], writes cache->router_probs [rows × n_experts] and
 * cache->expert_ids [rows × top_k] (rank order).  The expert set is
 * uploaded to the device the first time a given MoEWeights pointer is seen
 * and stays resident; call moe_b200_invalidate after changing its weights
 * (llm.c's training step mutates them in src/train.c:211-229).  On failure
 * it prints the reason and calls abort(), as llm.c's allocator does
 * (src/transformer.c:28-32).  The expert arithmetic follows the
 * environment variable MOE_B200_PATH = auto | tf32 | fp32 (default auto).
 */
void moe_forward(const llmc_Matrix *x, const llmc_MoEWeights *w,
                 const llmc_ModelConfig *cfg, llmc_ForwardCache *cache,
                 llmc_Matrix *out);

/* Drop the device copy of an expert set uploaded by moe_forward (no-op if
 * none).  Returns MOE_B200_OK or a negative status. */
int moe_b200_invalidate(const void *moe_weights);

#ifdef __cplusplus
}
#endif
#endif /* LLMC_MOE_H */
