// kernels.cuh — kernel launchers of the MoE hot path (internal).
#pragma once
#include "common.cuh"
#include <cuda.h>

namespace moe {

constexpr int kRouterTile = 64;   // tokens per router CTA (dispatch tile granularity)

// Plan (ints, device): cnt[E] | off[E+1] | mt128[E+1] | mt64[E+1] | mt256[E+1]
// (mtN = prefix over experts of ceil(cnt/N): the N-row m-tiles the grouped
// GEMMs schedule on)
__host__ __device__ inline int plan_ints(int E) { return E + 4 * (E + 1); }

// part/nsplit: optional [nsplit × T × E] buffer for the split-K variant used
// when T is too small to fill the GPU (router_splits gives nsplit)
cudaError_t launch_router(const float *x, int T, int d, const float *w_router,
                          const float *bias, int E, int k, float *probs, int *ids,
                          float *wts, int *loc, int *tile_cnt, cudaStream_t s,
                          float *part = nullptr, int nsplit = 1);
int router_splits(int T, int d);

cudaError_t launch_dispatch(const float *x, int T, int d, int d_pad, int E, int k,
                            const int *ids, const int *loc, const int *tile_cnt,
                            int *tile_pref, int *plan, int *pos_of, float *x_perm,
                            int round_to_tf32, DeviceStatus *status, cudaStream_t s,
                            int align = 1);
// zero rows [off[e] + cnt[e], off[e + 1]) of every expert segment of buf [rows × ld]
cudaError_t launch_zero_pad_rows(float *buf, int ld, const int *plan, int E, cudaStream_t s);

// scan only (the expert-parallel path does its own gather)
cudaError_t launch_dispatch_scan(const int *tile_cnt, int T, int E, int *tile_pref, int *plan,
                                 cudaStream_t s);

cudaError_t launch_combine(const float *y, int d, int d_pad, int T, int k,
                           const int *pos_of, const float *wts, float *out, cudaStream_t s,
                           const float *y2 = nullptr, const float *resid = nullptr);
// MoE backward (moe_backward.cu); rows are the expert-sorted (token, rank)
// slots of the forward's plan.
struct BwdArgs {
    int T, d, E, k, F, d_pad, F_pad, rows_bound;
    const int *plan, *pos_of, *ids;
    const float *x, *x_perm, *gu, *h, *y, *probs, *wts;   // forward state
    const float *router, *ug, *dn;                          // device weights
    const float *dy;                                        // [T × d]
    float aux_coef;
    float *dw, *dO, *dgu, *dxp, *dlogit, *pmean;            // workspace (dxp may be y)
    float *wr_part;                                         // [router_wgrad_splits × d × E]
    float *dx;                                              // [T × d]
    float *g_router, *g_bias, *g_gate, *g_up, *g_down;      // accumulated gradients
    float *aux_loss;                                        // device scalar or null
    int round_tf32;                                         // dO feeds TF32 GEMMs
};
// the whole backward on FP32 FFMA, or its three parts (the tensor-core
// backward replaces the middle one)
constexpr int kRouterWgradSplits = 64;
int router_wgrad_splits(int T, int d, int E);
cudaError_t launch_moe_backward(const BwdArgs &a, cudaStream_t s, int *launches);
cudaError_t launch_bwd_head(const BwdArgs &a, cudaStream_t s, int *n);
cudaError_t launch_bwd_ffma_gemms(const BwdArgs &a, cudaStream_t s, int *n);
cudaError_t launch_bwd_tail(const BwdArgs &a, cudaStream_t s, int *n);

// tcgen05 TF32 backward GEMMs (expert_tc_bwd.cu): dH + SwiGLU backward,
// dW_down, dW_gate / dW_up, dX_perm.  Expert segments of the plan start at
// multiples of 32 rows with zeroed alignment rows in h, dO and x_perm.  The
// *_mn maps use the 128-byte swizzle with 32-byte atoms, the *_k maps the
// plain 128-byte swizzle.
struct TcBwd {
    CUtensorMap tm_dO_k;    // dO    [rows × d_pad], box 128 rows (K-major A)
    CUtensorMap tm_dn_mn;   // dn    [E·d_pad × F_pad], box 32 rows (MN-major B)
    CUtensorMap tm_h_mn;    // h     [rows × F_pad], box 32 rows
    CUtensorMap tm_dO_mn;   // dO    [rows × d_pad], box 32 rows
    CUtensorMap tm_x_mn;    // x_perm [rows × d_pad], box 32 rows
    CUtensorMap tm_dgu_mn;  // dGU   [rows × 2·F_pad], box 32 rows
    CUtensorMap tm_dgu_k;   // dGU   [rows × 2·F_pad], box 128 rows (K-major A)
    CUtensorMap tm_ug_mn;   // ug    [E·2·F_pad × d_pad], box 32 rows
    const int *plan;
    int E, d, F, d_pad, F_pad, rows_bound, num_sms;
    const float *gu;        // saved gate / up pre-activations
    float *dgu, *dxp;
    float *g_down, *g_gate, *g_up;
    DeviceStatus *status;
};
cudaError_t launch_tc_bwd(const TcBwd &g, cudaStream_t s);

// block_forward's pre-FFN RMSNorm over rows of x[T × d] (block_ffn.cu)
cudaError_t launch_rmsnorm(const float *x, int T, int d, const float *weight, float eps,
                           float *out, cudaStream_t s);
int rmsnorm_max_d();

// FP32 FFMA grouped expert GEMMs (64-row tiles scheduled on mt64).
//   upgate: H[rows×F_pad] = swiglu(X_perm·Wg^T, X_perm·Wu^T)
//   down:   Y[rows×d_pad] = H·Wd^T
cudaError_t launch_ffma_upgate(const float *x_perm, int d_pad, const float *w_ug, int F_pad,
                               float *h, const int *plan, int E, int rows_bound, cudaStream_t s,
                               float *gu_save = nullptr);
cudaError_t launch_ffma_down(const float *h, int F_pad, const float *w_d, int d_pad,
                             float *y, const int *plan, int E, int rows_bound, cudaStream_t s,
                             float *const *y_ptrs = nullptr, const int2 *ret = nullptr);

// tcgen05 TF32 grouped GEMMs (128-row tiles scheduled on mt128), persistent.
struct TcGemm {
    CUtensorMap tmA;   // activations [rows × K_pad], box {32, 128}, SW128
    CUtensorMap tmB;   // weights [E*NB × K_pad], box {32, BN}, SW128
};
cudaError_t launch_tc_upgate(const TcGemm &g, int d_pad, int F_pad, float *h, const int *plan,
                             int E, int rows_bound, int num_sms, DeviceStatus *status, cudaStream_t s,
                             float *gu_save = nullptr);
// y_ptrs/ret (expert parallel): output row i goes to y_ptrs[ret[i].x] + ret[i].y * d_pad
cudaError_t launch_tc_down(const TcGemm &g, int F_pad, int d_pad, int bn, float *y, const int *plan,
                           int E, int rows_bound, int num_sms, DeviceStatus *status, cudaStream_t s,
                           float *const *y_ptrs = nullptr, const int2 *ret = nullptr);
cudaError_t tc_set_attributes();
// The same GEMMs on CTA pairs (tcgen05 cta_group::2): 256×256 output tiles
// scheduled on mt256; tmB has box {32, 128} (each CTA loads half of the
// weight tile).  Down needs d_pad % 256 == 0.
cudaError_t launch_tc2_upgate(const TcGemm &g, int d_pad, int F_pad, float *h, const int *plan,
                              int E, int rows_bound, int max_pairs, DeviceStatus *status,
                              cudaStream_t s);
cudaError_t launch_tc2_down(const TcGemm &g, int F_pad, int d_pad, float *y, const int *plan,
                            int E, int rows_bound, int max_pairs, DeviceStatus *status,
                            cudaStream_t s, float *const *y_ptrs = nullptr,
                            const int2 *ret = nullptr);
cudaError_t tc2_set_attributes();
int tc2_max_pairs(int num_sms);

// 3xTF32 weight-streaming GEMMs for decode-sized expert groups
struct DecMaps {
    CUtensorMap tmW;    // weights, box {32, 64} (up/gate) or {32, 128} (down)
    CUtensorMap tmXb;   // token operand big part  [rows × K], box {32, 64}
    CUtensorMap tmXs;   // token operand small part [rows × K], box {32, 64}
    CUtensorMap tmXb32; // big part again, box {32, 32} (CTA-pair kernels)
};
cudaError_t dec_set_attributes();
// max_pairs > 0: run on CTA pairs (M=256 per MMA), at most max_pairs of them
// (down only when d_pad % 256 == 0); 0: single CTAs
int dec_max_pairs(int num_sms);
cudaError_t launch_split_tf32(float *big, float *small, size_t n, cudaStream_t s);
cudaError_t launch_dec_upgate(const DecMaps &m, int d_pad, int F_pad, float *h_big, float *h_small,
                              const int *plan, int E, int rows_bound, int num_sms, int max_pairs,
                              DeviceStatus *status, cudaStream_t s, bool onepass = false);
cudaError_t launch_dec_down(const DecMaps &m, int F_pad, int d_pad, float *y, const int *plan,
                            int E, int rows_bound, int num_sms, int max_pairs, DeviceStatus *status,
                            cudaStream_t s, float *const *y_ptrs = nullptr,
                            const int2 *ret = nullptr, float *y2 = nullptr,
                            bool onepass = false);
// 2 when the down GEMM should run in two K halves (into y and a second
// buffer y2, summed by the combine), else 1
int dec_down_ksplit(int F_pad, int d_pad, int rows_bound, int E, int num_sms);

// weight repack: src row-major [R × C] (one expert matrix) -> dst rows of
// the K-major layout, see moe_b200.cu.
cudaError_t launch_repack_upgate(const float *wg, const float *wu, int d, int F, int d_pad,
                                 int F_pad, float *dst, cudaStream_t s);
cudaError_t launch_repack_down(const float *wd, int d, int F, int d_pad, int F_pad, float *dst,
                               cudaStream_t s);
cudaError_t launch_unpack_upgate(const float *src, int d, int F, int d_pad, int F_pad,
                                 float *wg, float *wu, cudaStream_t s);
cudaError_t launch_unpack_down(const float *src, int d, int F, int d_pad, int F_pad, float *wd,
                               cudaStream_t s);
cudaError_t launch_synth(float *dst, size_t n, uint64_t seed, uint64_t stream, uint64_t first,
                         float std, cudaStream_t s);
cudaError_t launch_synth_pack_expert(float *ug, float *dn, int d, int F, int d_pad, int F_pad,
                                     uint64_t seed, uint64_t stream_g, uint64_t stream_u,
                                     uint64_t stream_d, float std, cudaStream_t s);

}  // namespace moe
