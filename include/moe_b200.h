/*
 * moe_b200.h — C-ABI of the B200-native Mixture-of-Experts feed-forward
 * hot path of llm.c.
 *
 * Every entry point is plain C: host or device pointers, sizes and status
 * codes.  No CUDA or PyTorch type appears in a signature (streams are
 * passed as `void *` holding a cudaStream_t, NULL = the library's stream).
 *
 * The computation is the reference's moe_forward (llm.c
 * src/transformer.c:287-366): router logits x·W_router (+ optional bias),
 * row softmax, per-token top-k by probability with ties to the lower
 * expert index, weights renormalised over the selected k, SwiGLU experts
 * y = (silu(x·W_gate) ⊙ (x·W_up))·W_down, and the weighted combine in
 * rank order.  Outputs are overwritten, never accumulated into.
 *
 * All calls return MOE_B200_OK (0) or a negative status; there is no CPU
 * fallback: without a usable sm_100 device every compute call fails with
 * MOE_B200_E_NODEV.
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define MOE_B200_OK          0
#define MOE_B200_E_INVALID  (-1)  /* bad argument or unsupported shape      */
#define MOE_B200_E_CUDA     (-2)  /* a CUDA runtime call failed             */
#define MOE_B200_E_NOMEM    (-3)  /* device or pinned allocation failed      */
#define MOE_B200_E_NCCL     (-4)  /* NCCL failure (expert parallel)          */
#define MOE_B200_E_TIMEOUT  (-5)  /* a bounded device wait ran out           */
#define MOE_B200_E_NODEV    (-6)  /* no usable sm_100 device                 */
#define MOE_B200_E_STATE    (-7)  /* call made in the wrong state            */

/* ---- expert arithmetic path ------------------------------------------- */
#define MOE_B200_PATH_AUTO   0  /* TF32 for prefill-sized expert groups (on
                                    average >= 64 rows per expert), 3xTF32
                                    weight streaming for decode-sized ones  */
#define MOE_B200_PATH_TF32   1  /* tcgen05 TF32 (tol 2e-3): grouped GEMMs
                                    for prefill-sized groups, one-pass TF32
                                    weight streaming for decode-sized ones  */
#define MOE_B200_PATH_FP32   2  /* FP32 FFMA grouped GEMMs (tol 1e-5)       */
#define MOE_B200_PATH_TF32X3 3  /* tcgen05 3xTF32 weight-streaming GEMMs,
                                    FP32 accuracy (tol 1e-5)                */

typedef struct {
    int path;            /* MOE_B200_PATH_*                                   */
    int cta_pair;        /* tensor-core paths: 0 = single-SM kernels (the
                            fastest measured), 1 = CTA-pair kernels (tcgen05
                            cta_group::2, M=256 over two SMs; down only when
                            d is padded to a multiple of 256)               */
    int host_chunks;     /* moe_b200_forward (host buffers): token chunks whose
                            copies overlap the compute of the others; 0 = auto,
                            1 = none.  Applied on the TF32 / FP32 paths to
                            inputs of 64 MB and up, with chunks of at least
                            4352 tokens, so results equal the one-chunk call
                            bit for bit.  moe_b200_ep_forward: the same, each
                            chunk one collective forward (0 = 2 chunks when
                            max_tokens_per_rank·d·4 >= 64 MB); every rank
                            must pass the same value                        */
    int reserved[5];     /* zero                                              */
} moe_b200_opts;

/* Opaque device-resident expert set (router + E SwiGLU experts). */
typedef struct moe_b200_weights moe_b200_weights;

/* ---- library ----------------------------------------------------------- */

/* Version string of the library build. */
const char *moe_b200_version(void);

/* Human-readable name of a status code. */
const char *moe_b200_strerror(int status);

/* Detail text of the last failure on this host thread ("" if none). */
const char *moe_b200_last_error(void);

/* Select and initialise a CUDA device for this host thread (creates the
 * library stream and workspace lazily).  device < 0 keeps the current one. */
int moe_b200_init(int device);

/* Release every device resource the library holds on all devices. */
void moe_b200_shutdown(void);

/* ---- weights ----------------------------------------------------------- */

/* Upload an expert set from the reference's host layout (row-major fp32):
 *   W_router [d×E]; W_gate[e], W_up[e] [d×F]; W_down[e] [F×d].
 * Replaces llm.c's implicit use of host MoEWeights (include/transformer.h
 * :53-58).  The library repacks the experts once on the device into its
 * K-major, gate/up-interleaved layout; the host arrays are not retained. */
int moe_b200_weights_upload(const float *W_router,
                            const float *const *W_gate,
                            const float *const *W_up,
                            const float *const *W_down,
                            int d, int F, int E, int top_k,
                            moe_b200_weights **out);

/* Build an expert set directly on the device from the seeded synthetic
 * generator (every weight ~N(0, w_std), streams as in
 * moe_b200_synth_fill), for benchmarks whose weights would not fit in
 * host memory.  Equivalent to generating the host arrays and calling
 * moe_b200_weights_upload. */
int moe_b200_weights_synth(uint64_t seed, float w_std, int d, int F, int E,
                           int top_k, moe_b200_weights **out);

/* Expert-parallel shards (no counterpart in llm.c, whose MoEWeights always
 * hold every expert, include/transformer.h:53-58): a set with n_slots packed
 * expert slots of which the first n_local hold the experts listed in
 * experts[0..n_local) (global ids, distinct); the remaining slots are spares
 * that moe_b200_ep_rebalance may fill with replicas of hot experts.  The
 * router always covers all E experts (every rank routes its own tokens).
 * Only the moe_b200_ep_* calls run a shard; the single-GPU entry points
 * reject it with MOE_B200_E_INVALID.
 *   _synth_shard: the experts from the seeded generator (the same values
 *                 moe_b200_weights_synth gives those experts);
 *   _upload_shard: W_gate[i], W_up[i], W_down[i] are local expert i's host
 *                 matrices (llm.c's layouts), i < n_local. */
int moe_b200_weights_synth_shard(uint64_t seed, float w_std, int d, int F, int E, int top_k,
                                 int n_local, const int *experts, int n_slots,
                                 moe_b200_weights **out);
int moe_b200_weights_upload_shard(const float *W_router, const float *const *W_gate,
                                  const float *const *W_up, const float *const *W_down,
                                  int d, int F, int E, int top_k, int n_local,
                                  const int *experts, int n_slots, moe_b200_weights **out);
/* Slot count of a set and the global expert id in each slot (-1 = empty
 * spare); slot_expert has room for n_slots ints (either may be NULL). */
int moe_b200_weights_slots(const moe_b200_weights *w, int *n_slots, int *slot_expert);

/* Free a weight set (synchronises the device). */
int moe_b200_weights_free(moe_b200_weights *w);

/* Shape of a weight set. */
int moe_b200_weights_shape(const moe_b200_weights *w, int *d, int *F, int *E,
                           int *top_k);

/* Copy the device weights back into the reference host layout (for
 * checkpoint round trips and tests).  Any output pointer may be NULL. */
int moe_b200_weights_download(const moe_b200_weights *w, float *W_router,
                              float *const *W_gate, float *const *W_up,
                              float *const *W_down);

/* ---- forward ----------------------------------------------------------- */

/* MoE forward on HOST buffers; synchronous, like llm.c's moe_forward.
 *   x            [T×d] input rows (cache->x_norm_ffn in llm.c)
 *   router_bias  [E] added to the logits before the softmax, or NULL
 *                (NULL is the reference's behaviour)
 *   out          [T×d] overwritten
 *   router_probs [T×E] full softmax, or NULL   (cache->router_probs)
 *   expert_ids   [T×k] rank-ordered ids, or NULL (cache->expert_ids)
 * T = 0 is a no-op.  opts may be NULL (MOE_B200_PATH_AUTO). */
int moe_b200_forward(const moe_b200_weights *w, const float *router_bias,
                     const float *x, int T, float *out, float *router_probs,
                     int *expert_ids, const moe_b200_opts *opts);

/* Same computation on DEVICE buffers, asynchronous on `stream`
 * (a cudaStream_t, or NULL for the library stream).  No host
 * synchronisation and no allocation once the workspace has grown to T, so
 * the call can be captured in a CUDA graph after one warm-up call at the
 * largest T.  d_x and d_out must be 16-byte aligned. */
int moe_b200_forward_device(const moe_b200_weights *w, const float *d_bias,
                            const float *d_x, int T, float *d_out,
                            float *d_router_probs, int *d_expert_ids,
                            const moe_b200_opts *opts, void *stream);

/* The FFN half of llm.c's block_forward for a MoE block
 * (src/transformer.c:752-767) in one call:
 *   x_norm = rms_norm(x, rms_weight, eps)      (src/matrix.c:666-713)
 *   x     += moe_forward(x_norm)               (mat_add_inplace)
 * The RMSNorm runs on the device in front of the router, and the residual
 * add is fused into the combine, so x goes up once and comes back once.
 *   rms_weight [d]    block's rms_ffn
 *   x [T×d]           residual stream, updated in place
 *   x_norm [T×d]      receives the normalised rows (cache->x_norm_ffn), or
 *                     NULL
 *   router_bias, router_probs, expert_ids, opts as moe_b200_forward.
 * The RMSNorm follows the reference's summation order with correctly rounded
 * division and square root. */
int moe_b200_block_ffn(const moe_b200_weights *w, const float *rms_weight, float eps,
                       const float *router_bias, float *x, int T, float *x_norm,
                       float *router_probs, int *expert_ids, const moe_b200_opts *opts);

/* Same on DEVICE buffers, asynchronous on `stream` (NULL = library stream);
 * d_x and d_x_norm 16-byte aligned. */
int moe_b200_block_ffn_device(const moe_b200_weights *w, const float *d_rms_weight, float eps,
                              const float *d_bias, float *d_x, int T, float *d_x_norm,
                              float *d_router_probs, int *d_expert_ids,
                              const moe_b200_opts *opts, void *stream);

/* ---- backward (training) --------------------------------------------------
 * llm.c has no MoE backward (model_backward, src/transformer.c:981-1013,
 * stops at the norms and attention) and leaves the Switch load-balancing loss
 * to the training loop (src/transformer.c:280-282).  This is the gradient of
 * the forward above with the top-k choice held fixed, plus aux_coef · L_aux:
 *   L_aux = n_experts · Σ_e f_e · P_e,  f_e = tokens routed to e / (T·top_k),
 *   P_e = mean router probability of e.
 * Gradients accumulate (+=) in a moe_b200_grads object, in llm.c's layouts:
 * W_router [d×E], router bias [E], W_gate / W_up [d×F], W_down [F×d] per
 * expert.  The forward is recomputed inside the call.  Arithmetic by
 * opts->path: MOE_B200_PATH_FP32 (or TF32X3) FP32 FFMA, tolerance 1e-5;
 * MOE_B200_PATH_TF32 tcgen05 tensor cores, tolerance 2e-3; AUTO picks TF32
 * when the average expert group fills half a 128-row tile (the forward's
 * rule).  Every sum runs in a fixed order: bit-stable run to run. */
typedef struct moe_b200_grads moe_b200_grads;

int moe_b200_grads_create(const moe_b200_weights *w, moe_b200_grads **g);   /* zeroed */
int moe_b200_grads_zero(moe_b200_grads *g);
/* Any pointer may be NULL (that part is skipped). */
int moe_b200_grads_download(const moe_b200_grads *g, float *dW_router, float *d_bias,
                            float *const *dW_gate, float *const *dW_up, float *const *dW_down);
int moe_b200_grads_free(moe_b200_grads *g);

/* Host buffers, synchronous.  x [T×d] the forward's input, dy [T×d] the
 * gradient of the loss with respect to the forward's output; writes
 * dx [T×d] and, when aux_loss is not NULL, L_aux of this batch (its gradient
 * enters with weight aux_coef whether or not the value is requested). */
int moe_b200_backward(const moe_b200_weights *w, const float *router_bias, const float *x,
                      int T, const float *dy, float aux_coef, float *dx, moe_b200_grads *g,
                      float *aux_loss, const moe_b200_opts *opts);

/* Same on device buffers (16-byte aligned), asynchronous on `stream`. */
int moe_b200_backward_device(const moe_b200_weights *w, const float *d_bias, const float *d_x,
                             int T, const float *d_dy, float aux_coef, float *d_dx,
                             moe_b200_grads *g, float *d_aux_loss, const moe_b200_opts *opts,
                             void *stream);

/* Size of the static device array behind moe_b200_forward_noalloc. */
#define MOE_B200_NOALLOC_SCRATCH_BYTES (16u << 20)

/* MoE forward that allocates nothing: the same computation as
 * moe_b200_forward_device on the FP32 FFMA expert path (tolerance 1e-5),
 * with every intermediate buffer carved out of one fixed-size array that
 * is compiled into the library (MOE_B200_NOALLOC_SCRATCH_BYTES, 16 MiB, held
 * on every GPU that loads the library until the process exits).  This
 * entry point has no counterpart in llm.c.
 *
 * It is for callers that cannot call cudaMalloc while they run: a serving
 * or decode loop with a device-memory budget fixed at start-up, a program
 * whose device memory is owned by another framework's caching allocator,
 * or latency-critical code that must stay out of the CUDA allocator.  Such
 * a caller creates the weights once beforehand (moe_b200_weights_upload
 * allocates) and then passes only its own device buffers:
 *   d_x [T×d] in; d_out [T×d] out (overwritten); d_router_probs [T×E] and
 *   d_expert_ids [T×k] out, or NULL; d_bias [E] or NULL; `stream` a
 *   cudaStream_t (NULL = the legacy default stream).
 * The call is synchronous: it returns after the results are in d_out.
 * Shapes whose intermediates do not fit the array (roughly T·k·(2·d + F)·4
 * bytes plus router buffers) are rejected with MOE_B200_E_INVALID and a
 * message from moe_b200_last_error(); split such a call into smaller T.
 * The first call on a device looks up the array's device address; make that
 * first call before any stream capture.  Every call shares the one array,
 * so calls that overlap on the GPU (two streams or two host threads on the
 * same device) race; serialise them. */
int moe_b200_forward_noalloc(const moe_b200_weights *w, const float *d_bias,
                             const float *d_x, int T, float *d_out,
                             float *d_router_probs, int *d_expert_ids, void *stream);

/* Per-expert token counts of the last forward on this device (host array
 * of E ints); synchronises the library stream. */
int moe_b200_last_counts(const moe_b200_weights *w, int *counts);

/* Number of kernel launches the last forward issued on this device. */
int moe_b200_last_launches(void);

/* Expert arithmetic path (MOE_B200_PATH_TF32, _FP32 or _TF32X3) the last
 * forward on this device ran, after AUTO was resolved; 0 before any. */
int moe_b200_last_path(void);

/* SM count of `device` (-1 = current) and the number of CTA pairs (two-SM
 * clusters) of the TF32 pair GEMM that can be resident at once; either
 * output may be NULL.  No counterpart in llm.c (a diagnostic of this
 * library's launch sizing). */
int moe_b200_device_info(int device, int *num_sms, int *cta_pairs);

/* ---- device-resident decode (llm.c's inference_step on the B200) ------- */
/* Replaces llm.c's single-token KV-cache forward (src/inference.c:231-358,
 * declared at include/inference.h:137) with a device-resident one, MoE
 * blocks included (llm.c leaves them as a TODO at src/inference.c:342-343).
 * `model` is an llm.c Model (include/llmc_moe.h, llmc_Model); every weight
 * it holds, the RoPE tables and a KV cache of `max_seq` positions
 * (max_seq <= the model's RoPE table length) are copied to the current
 * device once.  Dense blocks (use_moe = 0) are supported.  The caller's
 * Model is only read during create; later changes to it need a new decoder.
 * A step appends `token` at the current position and writes the vocab
 * logits to host memory (if `logits` is not NULL); the position advances
 * like InferenceState.seq_pos.  Steps run as one CUDA graph.  Returns
 * MOE_B200_E_TIMEOUT if a bounded device wait ran out.  No counterpart in
 * llm.c beyond inference_step itself. */
typedef struct moe_b200_decoder moe_b200_decoder;
/* flags: 0 or MOE_B200_DECODER_STAGE_KERNELS = one kernel per stage (31
 * for six layers, the faster variant measured, the default; the stages hand
 * off through per-stage completion counters; the environment variable
 * MOE_B200_DECODER_PDL=2 selects griddepcontrol.wait hand-offs instead, and
 * MOE_B200_DECODER_EARLY is a bit mask of stage kinds whose CTAs let the
 * next kernel be placed on entry, default 16 = the down stage);
 * MOE_B200_DECODER_PERSISTENT = the whole step as ONE persistent cooperative
 * kernel (one CTA per SM, stages separated by a bounded grid-wide barrier).
 * Both run the same arithmetic and give the same bits; asking for both is
 * rejected. */
#define MOE_B200_DECODER_STAGE_KERNELS 1
#define MOE_B200_DECODER_PERSISTENT 2
int moe_b200_decoder_create(const void *model, int max_seq, int flags, moe_b200_decoder **dec);
int moe_b200_decoder_step(moe_b200_decoder *dec, int token, float *logits);
/* Rewind to position `pos` (<= the current one); later steps overwrite the
 * cache from there. */
int moe_b200_decoder_set_pos(moe_b200_decoder *dec, int pos);
int moe_b200_decoder_pos(const moe_b200_decoder *dec);
/* Kernels in one step (the graph's launches). */
int moe_b200_decoder_launches(const moe_b200_decoder *dec);
/* Debug read-back of the last step's FFN half of `layer`: the pre-FFN
 * normalised vector x_norm [d] (what the router and the experts read,
 * src/inference.c:311) and the FFN/MoE branch output [d] before the
 * residual add; either pointer may be NULL.  Synchronises the decoder.  For
 * per-layer parity against the reference's moe_forward with T=1 on the same
 * x_norm (src/transformer.c:287-366). */
int moe_b200_decoder_trace(moe_b200_decoder *dec, int layer, float *x_norm, float *ffn_out);
/* Stage timeline of the last step (stage kernels created with the
 * environment variable MOE_B200_DECODER_STAMPS=1): for each of the 5 L + 1
 * stages (5 l + {0 Q/K/V, 1 attention, 2 W_O, 3 up/gate, 4 down}, then the
 * LM head) four times in microseconds from the step's first CTA entry: the
 * earliest CTA entry, the earliest and the latest return from the stage's
 * wait for its predecessor, the latest CTA exit (-1 when not recorded).
 * out holds at least 4 * (5 L + 1) doubles; returns the stage count or a
 * negative status.  Profiling aid, no counterpart in llm.c. */
int moe_b200_decoder_stage_times(moe_b200_decoder *dec, double *out, int n);
int moe_b200_decoder_destroy(moe_b200_decoder *dec);

/* ---- llm.c checkpoints straight to the device ----------------------------
 * Files written by llm.c's model_save (src/transformer.c:573-617): the magic
 * "CLLM", the ModelConfig, then every tensor as fp32 in a fixed order.
 * Experts are streamed through double-buffered pinned staging, one expert
 * at a time, so a checkpoint far larger than host memory loads; no llm.c
 * Model is built on the host. */
/* The checkpoint's ModelConfig (llmc_ModelConfig, include/llmc_moe.h). */
int moe_b200_checkpoint_config(const char *path, void *cfg);
/* The MoE block of `layer` (or its dense FFN, as one expert) as a device
 * expert set, the same as moe_b200_weights_upload from the loaded Model. */
int moe_b200_checkpoint_load_experts(const char *path, int layer, moe_b200_weights **w);
/* A device decoder (moe_b200_decoder_create) straight from a checkpoint;
 * the RoPE tables are built as llm.c's rope_buffer_init builds them. */
int moe_b200_decoder_load(const char *path, int max_seq, int flags, moe_b200_decoder **dec);

/* ---- expert parallel (one process per GPU, NVLink) --------------------- */
/* llm.c has no multi-GPU path (README.md:379 lists it as a roadmap item);
 * these entry points extend moe_forward to G GPUs of one node.
 *
 * Experts are sharded: each rank passes its shard (moe_b200_weights_*_shard:
 * its base experts plus spare slots; a full set also works and then every
 * rank holds every expert).  Every rank routes its own tokens.  The rows of
 * an expert, over all source ranks, are split among the ranks that hold it
 * so that the estimated GEMM cost per rank is as even as the placement
 * allows; moe_b200_ep_rebalance adds replicas of hot experts in spare slots
 * from the last forward's per-expert counts.  Token rows and result rows
 * move by direct peer stores over NVLink (CUDA IPC); NCCL carries only
 * per-expert counts and two barriers.  All calls except
 * moe_b200_ep_unique_id, moe_b200_ep_split and moe_b200_ep_place are
 * collective: every rank makes them, in the same order. */
#define MOE_B200_EP_ID_BYTES 128
typedef struct moe_b200_ep moe_b200_ep;

/* Create the NCCL id on one rank (id: MOE_B200_EP_ID_BYTES bytes); the
 * caller broadcasts it to the other ranks by any host means. */
int moe_b200_ep_unique_id(void *id);

/* Join the group: rank in [0, world), at most max_tokens_per_rank tokens per
 * forward on each rank (the same value on every rank), this rank's expert
 * set `w` (a shard or a full set; every rank the same slot count, and every
 * expert held by some rank).  The group fills w's spare slots on rebalance.
 * Receive buffers are sized for world·max_tokens_per_rank·top_k rows, so no
 * routing can overflow them.  The environment variable
 * MOE_B200_EP_TIMEOUT_MS sets the host watchdog (moe_b200_ep_set_timeout). */
int moe_b200_ep_create(const void *id, int rank, int world, int max_tokens_per_rank,
                       moe_b200_weights *w, moe_b200_ep **out);

/* Leave the group and free its buffers (collective). */
int moe_b200_ep_destroy(moe_b200_ep *ep);

/* Forward of this rank's T tokens (device buffers, asynchronous on
 * `stream`, NULL = the group's stream); same outputs as
 * moe_b200_forward_device for these tokens.  AUTO resolves the arithmetic
 * path from the group's capacity (max_tokens_per_rank · world), the same on
 * every rank. */
int moe_b200_ep_forward_device(moe_b200_ep *ep, const float *d_bias, const float *d_x, int T,
                               float *d_out, float *d_router_probs, int *d_expert_ids,
                               const moe_b200_opts *opts, void *stream);

/* Same with host buffers, synchronous (H2D of x, D2H of the outputs, in
 * token chunks whose copies overlap the other chunks' forwards, see
 * moe_b200_opts.host_chunks; results do not depend on the chunking).  With
 * a watchdog set, a step that does not finish in time (a rank that stopped
 * joining the collectives) aborts the communicator and returns
 * MOE_B200_E_TIMEOUT; the group must then be destroyed. */
int moe_b200_ep_forward(moe_b200_ep *ep, const float *router_bias, const float *x, int T,
                        float *out, float *router_probs, int *expert_ids,
                        const moe_b200_opts *opts);

/* Per-rank, per-expert counts of the last collective forward ([world × E];
 * after a chunked host-buffer call, its last chunk's) and the number of rows
 * this rank received; synchronises the device. */
int moe_b200_ep_counts(moe_b200_ep *ep, int *counts_all, int *recv_rows);

/* The current placement [world × E]: slot of expert e on rank q, or -1. */
int moe_b200_ep_placement(const moe_b200_ep *ep, int *place);

/* Collective: from the last forward's counts, every rank computes the same
 * load-aware placement (moe_b200_ep_place from the base experts) and copies
 * the weights of its new replicas from the expert's base holder over NVLink
 * into its spare slots.  Call between forwards, not during one. */
int moe_b200_ep_rebalance(moe_b200_ep *ep);

/* Host watchdog of the host-buffer forward and of rebalance, in ms (0 = wait
 * without limit, the default unless MOE_B200_EP_TIMEOUT_MS is set). */
int moe_b200_ep_set_timeout(moe_b200_ep *ep, int timeout_ms);

/* The split every rank derives each forward from counts_all [world × E] and
 * place [world × E] (slot of e on rank q, -1 = not held; slots < n_slots):
 * single-holder experts go whole to their holder; replicated experts, most
 * rows first, are cut into 128-row tiles, each to the holder whose estimated
 * cost after taking it is lowest (2 units per tile, 1 more for the first
 * tile of a segment), and every holder takes its tiles as one contiguous
 * range in ascending rank order.  Outputs: n_holders[E], holders[E × world]
 * (ranks, ascending), row_begin[E × (world+1)] (holder i's first row in
 * the expert's global order: source rank, then local order),
 * recv_offset[E × world] (where holder i's range starts in its receive
 * buffer, slots in slot order), and, if not NULL, recv_rows[world] and
 * cost[world].  Host computation. */
int moe_b200_ep_split(const int *counts_all, int world, int E, const int *place, int n_slots,
                      int *n_holders, int *holders, int *row_begin, int *recv_offset,
                      long long *recv_rows, long long *cost);

/* The placement moe_b200_ep_rebalance adopts: from base_place (every rank's
 * base experts), repeatedly take the rank with the highest estimated cost
 * and its experts by the rows it carries, and place a replica on the least
 * loaded rank with a free slot that does not hold that expert yet, keeping
 * the first such move that lowers the highest cost; stop when none does.
 * Host computation, deterministic. */
int moe_b200_ep_place(const int *counts_all, int world, int E, const int *base_place,
                      int n_slots, int *place);

/* ---- stage timing ------------------------------------------------------ */

/* Stages of one forward, in launch order. */
#define MOE_B200_STAGE_ROUTER    0   /* logits, softmax, top-k, tile histogram */
#define MOE_B200_STAGE_DISPATCH  1   /* scan + permutation/gather              */
#define MOE_B200_STAGE_UPGATE    2   /* expert x·[W_gate|W_up] + SwiGLU        */
#define MOE_B200_STAGE_DOWN      3   /* expert h·W_down                        */
#define MOE_B200_STAGE_COMBINE   4   /* weighted rank-order combine            */
#define MOE_B200_NUM_STAGES      5

/* Enable (1) or disable (0) per-stage CUDA-event timing of every forward
 * on this device.  Events are recorded on the stream the kernels run on. */
int moe_b200_profile_enable(int enable);

/* Sum of each stage's device time in ms (stage_ms[MOE_B200_NUM_STAGES])
 * and the number of forwards timed since the last read; resets both.
 * Synchronises the timed streams. */
int moe_b200_profile_read(double *stage_ms, int *n_forwards);

/* ---- failure detection without a GPU fault ------------------------------
 * Test hooks; no counterpart in llm.c, which aborts on any failure
 * (src/transformer.c:28-32).  Neither faults, traps or hangs the GPU. */

/* Make the n-th device allocation the library makes from now on (weights,
 * workspace growth, expert-parallel buffers) fail as if the device were out
 * of memory; the call reports MOE_B200_E_NOMEM and the library stays
 * usable.  n = 0 turns the hook off. */
int moe_b200_debug_fail_alloc(int n);

/* One CTA waits on an mbarrier with the library's bounded-wait helper (the
 * one every tensor-core kernel uses) for at most limit_us microseconds
 * (<= 2 s), with nothing else in flight.  arrive = 1: the CTA arrives
 * first, the wait succeeds, MOE_B200_OK.  arrive = 0: nobody arrives, the
 * wait gives up, the kernel records its site in the status word and
 * returns, and the call reports MOE_B200_E_TIMEOUT; the device stays
 * usable. */
int moe_b200_debug_wait_probe(int limit_us, int arrive);

/* ---- synthetic inputs (benchmark plumbing) ----------------------------- */

/* Fill d_dst[0..n) on the device with the seeded approximately-N(0,std)
 * generator: element i is the Irwin–Hall sum of twelve 16-bit uniforms
 * from three splitmix64 hashes of (seed, stream, first + i), minus 6,
 * times std — bit-identical to the host generator of the test oracle. */
int moe_b200_synth_fill(float *d_dst, size_t n, uint64_t seed,
                        uint64_t stream, uint64_t first, float std,
                        void *cuda_stream);

/* Stream ids used by moe_b200_weights_synth and the benchmarks. */
#define MOE_B200_STREAM_X       1ULL
#define MOE_B200_STREAM_ROUTER  2ULL
#define MOE_B200_STREAM_BIAS    3ULL
#define MOE_B200_STREAM_EXPERT(e, which) (0x100ULL + 4ULL * (uint64_t)(e) + (uint64_t)(which))

#ifdef __cplusplus
}
#endif
#endif /* MOE_B200_H */
