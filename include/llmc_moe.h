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
 *   llmc_ForwardCache  == ForwardCache  include/transformer.h:108-124
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

/* Decode-side types (for the drop-in inference_step below):
 *   llmc_AttentionWeights == AttentionWeights  include/attention.h:40-45
 *   llmc_RoPEBuffer       == RoPEBuffer        include/attention.h:75-80
 *   llmc_BlockWeights     == BlockWeights      include/transformer.h:64-80
 *   llmc_ModelWeights     == ModelWeights      include/transformer.h:86-98
 *   llmc_Model            == Model             include/transformer.h:130-136
 *   llmc_LayerKVCache     == LayerKVCache      include/inference.h:45-48
 *   llmc_InferenceState   == InferenceState    include/inference.h:53-76 */
typedef struct {
    llmc_Matrix W_Q, W_K, W_V, W_O;
} llmc_AttentionWeights;

typedef struct {
    float *cos_table;
    float *sin_table;
    int max_seq_len;
    int head_dim;
} llmc_RoPEBuffer;

typedef struct {
    float *rms_attn;
    llmc_AttentionWeights attn;
    float *rms_ffn;
    int use_moe;
    union {
        llmc_FFNWeights ffn;
        llmc_MoEWeights moe;
    };
} llmc_BlockWeights;

typedef struct {
    llmc_Matrix embed;
    llmc_BlockWeights *blocks;
    int n_layers;
    float *rms_final;
    llmc_Matrix lm_head;
} llmc_ModelWeights;

typedef struct {
    llmc_ModelConfig cfg;
    llmc_ModelWeights weights;
    llmc_ForwardCache *caches;
    llmc_RoPEBuffer rope;
    void *train_scratch;
} llmc_Model;

typedef struct {
    float *K;
    float *V;
} llmc_LayerKVCache;

typedef struct {
    llmc_LayerKVCache *kv_cache;
    int n_layers;
    int seq_pos;
    int n_kv_heads;
    int head_dim;
    int kv_dim;
    int max_seq_len;
    float *x, *x_norm, *q, *k, *v, *attn_buf, *head_out, *logits;
} llmc_InferenceState;

/*
 * inference_step — replaces llm.c's inference_step (src/inference.c:231-358,
 * declared at include/inference.h:137) with the same signature and the same
 * single-token KV-cache forward, and fills in the MoE branch that llm.c
 * leaves as a TODO (src/inference.c:342-343): for a MoE block the pre-FFN
 * normalised vector goes through the B200 MoE forward (T = 1) and is added
 * to the residual, exactly as the dense branch adds its FFN output.  The
 * non-MoE arithmetic (RMSNorm, Q/K/V/O projections, RoPE, KV-cache append,
 * GQA attention over all cached positions, LM head) is a CPU restatement of
 * the reference's.  Aborts on a device failure, like moe_forward.
 * With the environment variable MOE_B200_DECODE=device the whole step runs
 * on the B200 instead (moe_b200_decoder_* in moe_b200.h; one decoder per
 * Model, created on first use): logits and seq_pos are updated as usual,
 * but the KV cache lives on the device and s->kv_cache is not written.  A
 * smaller seq_pos than the device's rewinds it; call moe_b200_invalidate(m)
 * after changing the model's weights.
 */
void inference_step(const llmc_Model *m, llmc_InferenceState *s, int token);

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

/*
 * moe_b200_llmc_block_ffn — the FFN half of llm.c's block_forward
 * (src/transformer.c:752-767) as one call, for a maintainer to put in place
 * of those lines:
 *     x_norm = rms_norm(x, bw->rms_ffn, eps); x += FFN_or_MoE(x_norm)
 * x [rows × d_model] is updated in place.  MoE blocks write
 * cache->router_probs and cache->expert_ids as moe_forward does; dense
 * blocks run their FFN as one expert.  cache->x_norm_ffn and cache->ffn_out
 * are not written: nothing in llm.c reads them after block_forward
 * (model_backward recomputes the norms from its saved block inputs,
 * src/transformer.c:986-996).  Weights stay resident as for moe_forward
 * (moe_b200_invalidate with &bw->moe or &bw->ffn).  Aborts on failure.
 */
void moe_b200_llmc_block_ffn(llmc_Matrix *x, const llmc_BlockWeights *bw,
                             llmc_ForwardCache *cache, const llmc_ModelConfig *cfg);

/*
 * moe_backward — the MoE block's backward, which llm.c's model_backward
 * (src/transformer.c:981-1013) lacks, with ffn_backward's conventions
 * (src/transformer.c:181-264): given the block input x and d_out = dL/d(out),
 * the weight gradients are ADDED into w->W_router.grad and each expert's
 * W_gate / W_up / W_down .grad (NULL ones are skipped) and d_x is
 * overwritten.  The top-k choice is held fixed; with MOE_B200_AUX_COEF = c
 * (default 0) the Switch load-balancing loss c · E · Σ_e f_e · P_e is
 * included.  The forward is recomputed (MOE_B200_PATH as for moe_forward:
 * tf32 tensor cores, fp32 FFMA, auto picks by group size).  Aborts on
 * failure.
 */
void moe_backward(const llmc_Matrix *x, const llmc_MoEWeights *w, const llmc_ModelConfig *cfg,
                  const llmc_ForwardCache *cache, const llmc_Matrix *d_out, llmc_Matrix *d_x);

/* Debug trace of the host inference_step above (not its device mode):
 * while enabled, every step records each layer's pre-FFN normalised vector
 * x_norm [d_model] and its FFN/MoE output [d_model] before the residual
 * add; moe_b200_llmc_trace_read returns those of `layer` from the last step
 * (MOE_B200_E_STATE before any).  Enabling clears the record.  No
 * counterpart in llm.c: it exists so that each layer's MoE can be checked
 * against the reference's moe_forward (src/transformer.c:287-366) on the
 * same x_norm. */
int moe_b200_llmc_trace_enable(int enable);
int moe_b200_llmc_trace_read(int layer, float *x_norm, float *ffn_out);

/* Drop the device copy of an expert set uploaded by moe_forward, given its
 * MoEWeights pointer, or the device decoder of inference_step's device mode,
 * given its Model pointer (no-op if none).  Returns MOE_B200_OK or a
 * negative status. */
int moe_b200_invalidate(const void *weights_or_model);

#ifdef __cplusplus
}
#endif
#endif /* LLMC_MOE_H */
