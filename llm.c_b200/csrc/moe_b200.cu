// moe_b200.cu — host side of the C-ABI (include/moe_b200.h): device
// contexts, workspace, weight residency, and the forward orchestration
//   router -> scan -> gather -> expert up/gate(+SwiGLU) -> expert down -> combine
// all on one stream with no host synchronisation in between (every grid
// that depends on routing reads its tile counts from the device plan).
#include "../../include/moe_b200.h"
#include "kernels.cuh"
#include "weights.cuh"

#include <cuda.h>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>

using namespace moe;

// ---------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------
static thread_local char g_err[512] = "";

static int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

int moe::set_last_error(int code, const char *detail) { return fail(code, "%s", detail); }

#define CK(call)                                                                              \
    do {                                                                                      \
        cudaError_t _e = (call);                                                              \
        if (_e != cudaSuccess)                                                                \
            return fail(_e == cudaErrorMemoryAllocation ? MOE_B200_E_NOMEM : MOE_B200_E_CUDA, \
                        "%s failed: %s (%s:%d)", #call, cudaGetErrorString(_e), __FILE__,     \
                        __LINE__);                                                            \
    } while (0)

// ---------------------------------------------------------------------
// tensor maps (driver entry point fetched through the runtime, so the
// library does not link libcuda directly)
// ---------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D fp32 row-major [rows × cols] tensor, box {32, box_rows}, 128B swizzle.
static int make_tmap(CUtensorMap *m, const float *ptr, int64_t rows, int64_t cols, int box_rows,
                     bool mn_major = false) {
    // mn_major: operand read MN-major by tcgen05 kind::tf32, which takes only
    // the 128-byte swizzle with 32-byte atoms
    EncodeTiledFn enc = get_encode();
    if (!enc) return fail(MOE_B200_E_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
    cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(ptr), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MOE_B200_E_CUDA, "cuTensorMapEncodeTiled error %d", (int)r);
    return MOE_B200_OK;
}

// ---------------------------------------------------------------------
// per-device context and workspace
// ---------------------------------------------------------------------
namespace {

struct Buf {
    void *p = nullptr;
    size_t cap = 0;
};

static int grow(Buf &b, size_t bytes) {
    if (bytes <= b.cap) return MOE_B200_OK;
    if (b.p) CK(cudaFree(b.p));
    b.p = nullptr;
    b.cap = 0;
    size_t want = bytes + bytes / 8 + 256;
    CK(dev_alloc(&b.p, want));
    b.cap = want;
    return MOE_B200_OK;
}

struct Ctx {
    int device = -1;
    int num_sms = 0;
    int tc2_pairs = 0;                   // co-resident CTA pairs of the 2-SM GEMM
    int dec_pairs = 0;                   // co-resident CTA pairs of the 2-SM decode kernel
    int cc_major = 0, cc_minor = 0;
    cudaStream_t stream = nullptr;
    // host-buffer forward pipeline: copies in and out on their own streams,
    // ordered against the compute on `stream` by per-chunk events
    static constexpr int kMaxChunks = 4;
    cudaStream_t s_in = nullptr, s_out = nullptr;
    cudaEvent_t ev_in[kMaxChunks] = {}, ev_done[kMaxChunks] = {};
    DeviceStatus *status = nullptr;      // device
    DeviceStatus *h_status = nullptr;    // pinned host copy, read back with each host call's results
    bool attrs_set = false;
    // workspace
    Buf probs, ids, wts, loc, tile_cnt, tile_pref, plan, pos_of, x_perm, h, y;
    Buf xs, hs;                          // small parts of the 3xTF32 split
    Buf y2;                              // second K half of a split down GEMM
    Buf rpart;                           // split-K router partial logits (small T)
    Buf io_x, io_out, io_bias;
    Buf xn, io_rms;                      // block FFN: RMSNorm output, host-call norm weights
    Buf gu, dO, dgu, dw, dlogit, pmean;  // backward: saved pre-activations and gradients
    Buf io_dy, io_dx, io_aux, wr_part;
    int last_E = 0;
    int last_launches = 0;
    int last_path = 0;
    // stage timing: ring of event sets, folded into the sums when read or
    // when the ring wraps
    bool prof = false;
    static constexpr int kSlots = 64;
    cudaEvent_t ev[kSlots][MOE_B200_NUM_STAGES + 1] = {};
    bool pending[kSlots] = {};
    int next_slot = 0;
    double stage_ms[MOE_B200_NUM_STAGES] = {};
    int n_timed = 0;
};

std::mutex g_mu;
Ctx *g_ctx[64] = {nullptr};

}  // namespace


static int get_ctx(int device, Ctx **out) {
    if (device < 0) CK(cudaGetDevice(&device));
    if (device >= 64) return fail(MOE_B200_E_INVALID, "device %d out of range", device);
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx *c = g_ctx[device];
    if (!c) {
        int n = 0;
        cudaError_t e = cudaGetDeviceCount(&n);
        if (e != cudaSuccess || n == 0)
            return fail(MOE_B200_E_NODEV, "no CUDA device: %s", cudaGetErrorString(e));
        if (device >= n) return fail(MOE_B200_E_NODEV, "device %d not present (%d)", device, n);
        CK(cudaSetDevice(device));
        cudaDeviceProp prop;
        CK(cudaGetDeviceProperties(&prop, device));
        if (prop.major != 10)
            return fail(MOE_B200_E_NODEV, "device %d is sm_%d%d; this build needs sm_100",
                        device, prop.major, prop.minor);
        c = new Ctx();
        c->device = device;
        c->num_sms = prop.multiProcessorCount;
        c->cc_major = prop.major;
        c->cc_minor = prop.minor;
        CK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
        CK(cudaMalloc(&c->status, sizeof(DeviceStatus)));
        CK(cudaMemset(c->status, 0, sizeof(DeviceStatus)));
        CK(cudaHostAlloc(&c->h_status, sizeof(DeviceStatus), cudaHostAllocDefault));
        CK(tc_set_attributes());
        CK(dec_set_attributes());
        CK(tc2_set_attributes());
        c->tc2_pairs = tc2_max_pairs(c->num_sms);
        c->dec_pairs = dec_max_pairs(c->num_sms);
        c->attrs_set = true;
        g_ctx[device] = c;
    }
    CK(cudaSetDevice(device));
    *out = c;
    return MOE_B200_OK;
}

// ---------------------------------------------------------------------
// library
// ---------------------------------------------------------------------
extern "C" const char *moe_b200_version(void) { return "moe_b200 0.1 (sm_100a)"; }

extern "C" const char *moe_b200_strerror(int s) {
    switch (s) {
    case MOE_B200_OK: return "ok";
    case MOE_B200_E_INVALID: return "invalid argument";
    case MOE_B200_E_CUDA: return "CUDA error";
    case MOE_B200_E_NOMEM: return "out of memory";
    case MOE_B200_E_NCCL: return "NCCL error";
    case MOE_B200_E_TIMEOUT: return "device wait timed out";
    case MOE_B200_E_NODEV: return "no usable sm_100 device";
    case MOE_B200_E_STATE: return "bad state";
    default: return "unknown status";
    }
}

extern "C" const char *moe_b200_last_error(void) { return g_err; }

extern "C" int moe_b200_init(int device) {
    Ctx *c;
    return get_ctx(device, &c);
}

static void free_buf(Buf &b) {
    if (b.p) cudaFree(b.p);
    b.p = nullptr;
    b.cap = 0;
}

extern "C" void moe_b200_shutdown(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    for (int i = 0; i < 64; i++) {
        Ctx *c = g_ctx[i];
        if (!c) continue;
        cudaSetDevice(i);
        cudaStreamSynchronize(c->stream);
        Buf *bufs[] = {&c->probs, &c->ids, &c->wts, &c->loc, &c->tile_cnt, &c->tile_pref,
                       &c->plan, &c->pos_of, &c->x_perm, &c->h, &c->y, &c->xs, &c->hs,
                       &c->rpart, &c->y2, &c->io_x, &c->io_out, &c->io_bias,
                       &c->xn, &c->io_rms, &c->gu, &c->dO, &c->dgu, &c->dw, &c->dlogit,
                       &c->pmean, &c->io_dy, &c->io_dx, &c->io_aux, &c->wr_part};
        for (Buf *b : bufs) free_buf(*b);
        cudaFree(c->status);
        if (c->h_status) cudaFreeHost(c->h_status);
        if (c->s_in) cudaStreamSynchronize(c->s_in), cudaStreamDestroy(c->s_in);
        if (c->s_out) cudaStreamSynchronize(c->s_out), cudaStreamDestroy(c->s_out);
        for (int k = 0; k < Ctx::kMaxChunks; k++) {
            if (c->ev_in[k]) cudaEventDestroy(c->ev_in[k]);
            if (c->ev_done[k]) cudaEventDestroy(c->ev_done[k]);
        }
        cudaStreamDestroy(c->stream);
        delete c;
        g_ctx[i] = nullptr;
    }
}

// ---------------------------------------------------------------------
// weights
// ---------------------------------------------------------------------
static int check_shape(int d, int F, int E, int k) {
    if (d <= 0 || F <= 0) return fail(MOE_B200_E_INVALID, "d=%d F=%d must be positive", d, F);
    if (E < 1 || E > kMaxExperts)
        return fail(MOE_B200_E_INVALID, "n_experts=%d outside [1, %d]", E, kMaxExperts);
    if (k < 1 || k > E || k > kMaxTopK)
        return fail(MOE_B200_E_INVALID, "top_k=%d outside [1, min(E, %d)]", k, kMaxTopK);
    if ((int64_t)d * F > (int64_t)1 << 31)
        return fail(MOE_B200_E_INVALID, "d*F too large");
    return MOE_B200_OK;
}

// A set of n_slots packed expert slots (n_slots = E: a full set, slot e =
// expert e) with a router over all E experts.
static int weights_alloc(Ctx *c, int d, int F, int E, int k, moe_b200_weights **out,
                         int n_slots = -1) {
    moe_b200_weights *w = new moe_b200_weights();
    w->device = c->device;
    w->d = d; w->F = F; w->E = E; w->k = k;
    w->d_pad = round_up(d, 128);
    w->F_pad = round_up(F, 128);
    w->down_bn = (w->d_pad % 256 == 0) ? 256 : 128;
    const int S = n_slots < 0 ? E : n_slots;
    w->n_slots = S;
    w->slot_expert.resize(S);
    for (int j = 0; j < S; j++) w->slot_expert[j] = n_slots < 0 ? j : -1;
    const size_t ug = (size_t)S * 2 * w->F_pad * w->d_pad, dn = (size_t)S * w->d_pad * w->F_pad;
    cudaError_t e1 = dev_alloc((void **)&w->router, (size_t)d * E * 4);
    cudaError_t e2 = e1 == cudaSuccess ? dev_alloc((void **)&w->ug, ug * 4) : e1;
    cudaError_t e3 = e2 == cudaSuccess ? dev_alloc((void **)&w->dn, dn * 4) : e2;
    if (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess) {
        cudaFree(w->router); cudaFree(w->ug); cudaFree(w->dn);
        delete w;
        cudaGetLastError();
        return fail(MOE_B200_E_NOMEM, "weights (%.2f GB) do not fit on device %d",
                    (double)(ug + dn) * 4 / 1e9, c->device);
    }
    int rc = make_tmap(&w->tm_ug, w->ug, (int64_t)S * 2 * w->F_pad, w->d_pad, 256);
    if (rc == 0) rc = make_tmap(&w->tm_dn, w->dn, (int64_t)S * w->d_pad, w->F_pad, w->down_bn);
    if (rc == 0) rc = make_tmap(&w->tm_ug64, w->ug, (int64_t)S * 2 * w->F_pad, w->d_pad, 64);
    if (rc == 0) rc = make_tmap(&w->tm_dn128, w->dn, (int64_t)S * w->d_pad, w->F_pad, 128);
    if (rc == 0) rc = make_tmap(&w->tm_ug128, w->ug, (int64_t)S * 2 * w->F_pad, w->d_pad, 128);
    if (rc) {
        cudaFree(w->router); cudaFree(w->ug); cudaFree(w->dn);
        delete w;
        return rc;
    }
    *out = w;
    return MOE_B200_OK;
}

int moe::weights_create(int d, int F, int E, int k, moe_b200_weights **out) {
    int rc = check_shape(d, F, E, k);
    if (rc) return rc;
    Ctx *c;
    if ((rc = get_ctx(-1, &c))) return rc;
    return weights_alloc(c, d, F, E, k, out);
}

int moe::weights_put_expert(moe_b200_weights *w, int ex, const float *d_stage, cudaStream_t s) {
    const size_t dF = (size_t)w->d * w->F;
    float *ug = w->ug + (size_t)ex * 2 * w->F_pad * w->d_pad;
    float *dn = w->dn + (size_t)ex * w->d_pad * w->F_pad;
    if (launch_repack_upgate(d_stage, d_stage + dF, w->d, w->F, w->d_pad, w->F_pad, ug, s) ||
        launch_repack_down(d_stage + 2 * dF, w->d, w->F, w->d_pad, w->F_pad, dn, s))
        return fail(MOE_B200_E_CUDA, "repack launch failed");
    return MOE_B200_OK;
}

cudaStream_t moe::current_stream() {
    Ctx *c;
    return get_ctx(-1, &c) ? nullptr : c->stream;
}

extern "C" int moe_b200_weights_upload(const float *W_router, const float *const *W_gate,
                                       const float *const *W_up, const float *const *W_down,
                                       int d, int F, int E, int top_k, moe_b200_weights **out) {
    if (!out || !W_router || !W_gate || !W_up || !W_down)
        return fail(MOE_B200_E_INVALID, "null argument");
    moe_b200_weights *w;
    int rc = moe::weights_create(d, F, E, top_k, &w);
    if (rc) return rc;
    Ctx *c;
    if ((rc = get_ctx(-1, &c))) { moe_b200_weights_free(w); return rc; }
    float *stage = nullptr;
    const size_t dF = (size_t)d * F;
    cudaError_t e = cudaMalloc(&stage, 3 * dF * 4);
    if (e != cudaSuccess) {
        moe_b200_weights_free(w);
        return fail(MOE_B200_E_NOMEM, "upload staging: %s", cudaGetErrorString(e));
    }
    rc = MOE_B200_OK;
    do {
        if (cudaMemcpy(w->router, W_router, (size_t)d * E * 4, cudaMemcpyHostToDevice)) {
            rc = fail(MOE_B200_E_CUDA, "router upload failed");
            break;
        }
        for (int ex = 0; ex < E && !rc; ex++) {
            if (!W_gate[ex] || !W_up[ex] || !W_down[ex]) {
                rc = fail(MOE_B200_E_INVALID, "expert %d has a null matrix", ex);
                break;
            }
            if (cudaMemcpyAsync(stage, W_gate[ex], dF * 4, cudaMemcpyHostToDevice, c->stream) ||
                cudaMemcpyAsync(stage + dF, W_up[ex], dF * 4, cudaMemcpyHostToDevice, c->stream) ||
                cudaMemcpyAsync(stage + 2 * dF, W_down[ex], dF * 4, cudaMemcpyHostToDevice,
                                c->stream)) {
                rc = fail(MOE_B200_E_CUDA, "expert %d upload failed", ex);
                break;
            }
            if ((rc = moe::weights_put_expert(w, ex, stage, c->stream))) break;
            // staging is reused by the next expert
            if (cudaStreamSynchronize(c->stream)) {
                rc = fail(MOE_B200_E_CUDA, "repack failed: %s", cudaGetErrorString(cudaGetLastError()));
                break;
            }
        }
    } while (0);
    cudaFree(stage);
    if (rc) {
        moe_b200_weights_free(w);
        return rc;
    }
    *out = w;
    return MOE_B200_OK;
}

extern "C" int moe_b200_weights_synth(uint64_t seed, float w_std, int d, int F, int E,
                                      int top_k, moe_b200_weights **out) {
    if (!out) return fail(MOE_B200_E_INVALID, "null argument");
    int rc = check_shape(d, F, E, top_k);
    if (rc) return rc;
    Ctx *c;
    if ((rc = get_ctx(-1, &c))) return rc;
    moe_b200_weights *w;
    if ((rc = weights_alloc(c, d, F, E, top_k, &w))) return rc;
    CK(launch_synth(w->router, (size_t)d * E, seed, MOE_B200_STREAM_ROUTER, 0, w_std, c->stream));
    for (int ex = 0; ex < E; ex++) {
        float *ug = w->ug + (size_t)ex * 2 * w->F_pad * w->d_pad;
        float *dn = w->dn + (size_t)ex * w->d_pad * w->F_pad;
        CK(launch_synth_pack_expert(ug, dn, d, F, w->d_pad, w->F_pad, seed,
                                    MOE_B200_STREAM_EXPERT(ex, 0), MOE_B200_STREAM_EXPERT(ex, 1),
                                    MOE_B200_STREAM_EXPERT(ex, 2), w_std, c->stream));
    }
    CK(cudaStreamSynchronize(c->stream));
    *out = w;
    return MOE_B200_OK;
}

// ---- expert-parallel shards ----
static int check_shard(int E, int n_local, const int *experts, int n_slots) {
    if (n_local < 0 || n_slots < 1 || n_local > n_slots || n_slots > E || (n_local > 0 && !experts))
        return fail(MOE_B200_E_INVALID, "shard: need 0 <= n_local <= n_slots <= E (%d, %d, %d)",
                    n_local, n_slots, E);
    std::vector<char> seen(E, 0);
    for (int i = 0; i < n_local; i++) {
        if (experts[i] < 0 || experts[i] >= E || seen[experts[i]])
            return fail(MOE_B200_E_INVALID, "shard: expert id %d out of range or repeated",
                        experts[i]);
        seen[experts[i]] = 1;
    }
    return MOE_B200_OK;
}

extern "C" int moe_b200_weights_synth_shard(uint64_t seed, float w_std, int d, int F, int E,
                                            int top_k, int n_local, const int *experts,
                                            int n_slots, moe_b200_weights **out) {
    if (!out) return fail(MOE_B200_E_INVALID, "null argument");
    int rc = check_shape(d, F, E, top_k);
    if (!rc) rc = check_shard(E, n_local, experts, n_slots);
    if (rc) return rc;
    Ctx *c;
    if ((rc = get_ctx(-1, &c))) return rc;
    moe_b200_weights *w;
    if ((rc = weights_alloc(c, d, F, E, top_k, &w, n_slots))) return rc;
    w->shard = 1;
    CK(launch_synth(w->router, (size_t)d * E, seed, MOE_B200_STREAM_ROUTER, 0, w_std, c->stream));
    for (int j = 0; j < n_local; j++) {
        const int ex = experts[j];
        float *ug = w->ug + (size_t)j * 2 * w->F_pad * w->d_pad;
        float *dn = w->dn + (size_t)j * w->d_pad * w->F_pad;
        CK(launch_synth_pack_expert(ug, dn, d, F, w->d_pad, w->F_pad, seed,
                                    MOE_B200_STREAM_EXPERT(ex, 0), MOE_B200_STREAM_EXPERT(ex, 1),
                                    MOE_B200_STREAM_EXPERT(ex, 2), w_std, c->stream));
        w->slot_expert[j] = ex;
    }
    CK(cudaStreamSynchronize(c->stream));
    *out = w;
    return MOE_B200_OK;
}

extern "C" int moe_b200_weights_upload_shard(const float *W_router, const float *const *W_gate,
                                             const float *const *W_up, const float *const *W_down,
                                             int d, int F, int E, int top_k, int n_local,
                                             const int *experts, int n_slots,
                                             moe_b200_weights **out) {
    if (!out || !W_router || (n_local > 0 && (!W_gate || !W_up || !W_down)))
        return fail(MOE_B200_E_INVALID, "null argument");
    int rc = check_shape(d, F, E, top_k);
    if (!rc) rc = check_shard(E, n_local, experts, n_slots);
    if (rc) return rc;
    Ctx *c;
    if ((rc = get_ctx(-1, &c))) return rc;
    moe_b200_weights *w;
    if ((rc = weights_alloc(c, d, F, E, top_k, &w, n_slots))) return rc;
    w->shard = 1;
    float *stage = nullptr;
    const size_t dF = (size_t)d * F;
    if (n_local > 0 && cudaMalloc(&stage, 3 * dF * 4) != cudaSuccess) {
        cudaGetLastError();
        moe_b200_weights_free(w);
        return fail(MOE_B200_E_NOMEM, "upload staging does not fit");
    }
    rc = MOE_B200_OK;
    if (cudaMemcpy(w->router, W_router, (size_t)d * E * 4, cudaMemcpyHostToDevice))
        rc = fail(MOE_B200_E_CUDA, "router upload failed");
    for (int j = 0; j < n_local && !rc; j++) {
        if (!W_gate[j] || !W_up[j] || !W_down[j]) {
            rc = fail(MOE_B200_E_INVALID, "local expert %d has a null matrix", j);
            break;
        }
        if (cudaMemcpyAsync(stage, W_gate[j], dF * 4, cudaMemcpyHostToDevice, c->stream) ||
            cudaMemcpyAsync(stage + dF, W_up[j], dF * 4, cudaMemcpyHostToDevice, c->stream) ||
            cudaMemcpyAsync(stage + 2 * dF, W_down[j], dF * 4, cudaMemcpyHostToDevice, c->stream)) {
            rc = fail(MOE_B200_E_CUDA, "local expert %d upload failed", j);
            break;
        }
        if ((rc = moe::weights_put_expert(w, j, stage, c->stream))) break;
        if (cudaStreamSynchronize(c->stream)) {
            rc = fail(MOE_B200_E_CUDA, "repack failed: %s", cudaGetErrorString(cudaGetLastError()));
            break;
        }
        w->slot_expert[j] = experts[j];
    }
    if (stage) cudaFree(stage);
    if (rc) {
        moe_b200_weights_free(w);
        return rc;
    }
    *out = w;
    return MOE_B200_OK;
}

extern "C" int moe_b200_weights_slots(const moe_b200_weights *w, int *n_slots, int *slot_expert) {
    if (!w) return fail(MOE_B200_E_INVALID, "null weights");
    if (n_slots) *n_slots = w->n_slots;
    if (slot_expert)
        for (int j = 0; j < w->n_slots; j++) slot_expert[j] = w->slot_expert[j];
    return MOE_B200_OK;
}

int moe::weights_full(const moe_b200_weights *w) {
    if (w && w->shard)
        return fail(MOE_B200_E_INVALID,
                    "an expert-parallel shard holds only some experts: use moe_b200_ep_*");
    return MOE_B200_OK;
}

extern "C" int moe_b200_weights_free(moe_b200_weights *w) {
    if (!w) return MOE_B200_OK;
    cudaSetDevice(w->device);
    cudaDeviceSynchronize();
    cudaFree(w->router);
    cudaFree(w->ug);
    cudaFree(w->dn);
    delete w;
    return MOE_B200_OK;
}

extern "C" int moe_b200_weights_shape(const moe_b200_weights *w, int *d, int *F, int *E,
                                      int *top_k) {
    if (!w) return fail(MOE_B200_E_INVALID, "null weights");
    if (d) *d = w->d;
    if (F) *F = w->F;
    if (E) *E = w->E;
    if (top_k) *top_k = w->k;
    return MOE_B200_OK;
}

extern "C" int moe_b200_weights_download(const moe_b200_weights *w, float *W_router,
                                         float *const *W_gate, float *const *W_up,
                                         float *const *W_down) {
    if (!w) return fail(MOE_B200_E_INVALID, "null weights");
    Ctx *c;
    int rc = get_ctx(w->device, &c);
    if (rc) return rc;
    const int d = w->d, F = w->F;
    const size_t dF = (size_t)d * F;
    if (W_router) CK(cudaMemcpy(W_router, w->router, (size_t)d * w->E * 4, cudaMemcpyDeviceToHost));
    if (!W_gate && !W_up && !W_down) return MOE_B200_OK;
    if ((rc = weights_full(w))) return rc;
    float *stage = nullptr;
    CK(cudaMalloc(&stage, 3 * dF * 4));
    for (int ex = 0; ex < w->E; ex++) {
        const float *ug = w->ug + (size_t)ex * 2 * w->F_pad * w->d_pad;
        const float *dn = w->dn + (size_t)ex * w->d_pad * w->F_pad;
        CK(launch_unpack_upgate(ug, d, F, w->d_pad, w->F_pad, stage, stage + dF, c->stream));
        CK(launch_unpack_down(dn, d, F, w->d_pad, w->F_pad, stage + 2 * dF, c->stream));
        CK(cudaStreamSynchronize(c->stream));
        if (W_gate && W_gate[ex]) CK(cudaMemcpy(W_gate[ex], stage, dF * 4, cudaMemcpyDeviceToHost));
        if (W_up && W_up[ex]) CK(cudaMemcpy(W_up[ex], stage + dF, dF * 4, cudaMemcpyDeviceToHost));
        if (W_down && W_down[ex])
            CK(cudaMemcpy(W_down[ex], stage + 2 * dF, dF * 4, cudaMemcpyDeviceToHost));
    }
    cudaFree(stage);
    return MOE_B200_OK;
}

// ---------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------
static bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

// Decode-sized expert groups (average below half a 128-row tile): the
// expert GEMMs stream weights (dec_gemm) rather than fill token tiles.
static bool decode_sized(const moe_b200_weights *w, int T) {
    return (double)T * w->k / w->E < 64.0;
}

// Column width of the TF32 down GEMM's tiles: 256 where the tiles fill the
// SMs, else 128 (twice the tiles, so that small layers spread over more
// SMs).  Sets the weight tensor map to match.  The width does not change
// any output element's arithmetic, only which CTA computes it.
static int down_tile_width(const Ctx *c, const moe_b200_weights *w, int rows, TcGemm *dn) {
    const int tiles256 = (int)((ceil_div(rows, 128) + w->E) * (w->d_pad / 256));
    if (w->down_bn == 256 && tiles256 < c->num_sms) {
        dn->tmB = w->tm_dn128;
        return 128;
    }
    dn->tmB = w->tm_dn;
    return w->down_bn;
}

static int pick_path(const moe_b200_weights *w, int T, const moe_b200_opts *opts) {
    int path = opts ? opts->path : MOE_B200_PATH_AUTO;
    if (path == MOE_B200_PATH_AUTO) {
        // tensor-core tiles are 128 rows: use them once the average expert
        // group fills half a tile; smaller (decode-sized) groups stream the
        // weights through the 3xTF32 tensor-core kernel (FP32 accuracy).
        path = decode_sized(w, T) ? MOE_B200_PATH_TF32X3 : MOE_B200_PATH_TF32;
    }
    return path;
}

static int ensure_workspace(Ctx *c, const moe_b200_weights *w, int T) {
    const size_t Tk = (size_t)T * w->k, tiles = ceil_div(T, kRouterTile);
    int rc;
    if ((rc = grow(c->probs, (size_t)T * w->E * 4))) return rc;
    if ((rc = grow(c->ids, Tk * 4))) return rc;
    if ((rc = grow(c->wts, Tk * 4))) return rc;
    if ((rc = grow(c->loc, Tk * 4))) return rc;
    if ((rc = grow(c->tile_cnt, tiles * w->E * 4))) return rc;
    if ((rc = grow(c->tile_pref, tiles * w->E * 4))) return rc;
    if ((rc = grow(c->plan, (size_t)plan_ints(w->E) * 4))) return rc;
    if ((rc = grow(c->pos_of, Tk * 4))) return rc;
    if ((rc = grow(c->x_perm, Tk * w->d_pad * 4))) return rc;
    if ((rc = grow(c->h, Tk * w->F_pad * 4))) return rc;
    if ((rc = grow(c->y, Tk * w->d_pad * 4))) return rc;
    return MOE_B200_OK;
}

static int fold_slot(Ctx *c, int slot) {
    if (!c->pending[slot]) return MOE_B200_OK;
    CK(cudaEventSynchronize(c->ev[slot][MOE_B200_NUM_STAGES]));
    for (int i = 0; i < MOE_B200_NUM_STAGES; i++) {
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, c->ev[slot][i], c->ev[slot][i + 1]));
        c->stage_ms[i] += ms;
    }
    c->n_timed++;
    c->pending[slot] = false;
    return MOE_B200_OK;
}

// returns the event set to record into for this forward, or nullptr
static cudaEvent_t *prof_slot(Ctx *c) {
    if (!c->prof) return nullptr;
    const int slot = c->next_slot;
    if (fold_slot(c, slot)) return nullptr;
    if (!c->ev[slot][0])
        for (int i = 0; i <= MOE_B200_NUM_STAGES; i++)
            if (cudaEventCreate(&c->ev[slot][i]) != cudaSuccess) return nullptr;
    c->pending[slot] = true;
    c->next_slot = (slot + 1) % Ctx::kSlots;
    return c->ev[slot];
}

// block_forward's FFN half around the MoE forward (src/transformer.c:752-767):
// the input is the residual stream x, RMSNorm writes x_norm for the router
// and the dispatch, and the combine adds the MoE output back onto x.
struct BlockNorm {
    const float *weight;   // device [d]
    float eps;
    float *x_norm;         // device [T × d]
};

static int forward_on(Ctx *c, const moe_b200_weights *w, const float *d_bias, const float *d_x,
                      int T, float *d_out, float *d_probs, int *d_ids,
                      const moe_b200_opts *opts, cudaStream_t s,
                      const BlockNorm *bn = nullptr) {
    int rc = weights_full(w);
    if (rc) return rc;
    if ((rc = ensure_workspace(c, w, T))) return rc;
    const int E = w->E, k = w->k, d = w->d;
    const int rows = T * k;
    float *probs = d_probs ? d_probs : (float *)c->probs.p;
    int *ids = d_ids ? d_ids : (int *)c->ids.p;
    float *wts = (float *)c->wts.p;
    int *loc = (int *)c->loc.p, *tile_cnt = (int *)c->tile_cnt.p, *tile_pref = (int *)c->tile_pref.p;
    int *plan = (int *)c->plan.p, *pos_of = (int *)c->pos_of.p;
    float *x_perm = (float *)c->x_perm.p, *h = (float *)c->h.p, *y = (float *)c->y.p;
    int launches = 0;
    float *y2 = nullptr;                 // second K half of the down GEMM, when split
    cudaEvent_t *ev = prof_slot(c);
#define MARK(i) \
    if (ev) CK(cudaEventRecord(ev[i], s))

    MARK(0);
    const float *resid = nullptr;
    if (bn) {
        CK(launch_rmsnorm(d_x, T, d, bn->weight, bn->eps, bn->x_norm, s));
        launches += 1;
        resid = d_x;
        d_x = bn->x_norm;
    }
    const int nsplit = router_splits(T, d);
    if (nsplit > 1 && (rc = grow(c->rpart, (size_t)nsplit * T * E * 4))) return rc;
    CK(launch_router(d_x, T, d, w->router, d_bias, E, k, probs, ids, wts, loc, tile_cnt, s,
                     (float *)c->rpart.p, nsplit));
    launches += nsplit > 1 ? 2 : 1;
    MARK(1);
    const int path = pick_path(w, T, opts);
    CK(launch_dispatch(d_x, T, d, w->d_pad, E, k, ids, loc, tile_cnt, tile_pref, plan, pos_of,
                       x_perm, path == MOE_B200_PATH_TF32, c->status, s));
    launches += 2;
    MARK(2);
    // TF32 on decode-sized groups: the weight-streaming kernel in its
    // one-pass TF32 mode (same tolerance as the grouped GEMM)
    const bool onepass = path == MOE_B200_PATH_TF32 && decode_sized(w, T);
    if (path == MOE_B200_PATH_TF32 && !onepass) {
        TcGemm up, dn;
        const bool pair = opts && opts->cta_pair && c->tc2_pairs > 0;
        if ((rc = make_tmap(&up.tmA, x_perm, rows, w->d_pad, 128))) return rc;
        if ((rc = make_tmap(&dn.tmA, h, rows, w->F_pad, 128))) return rc;
        if (pair) {
            up.tmB = w->tm_ug128;
            CK(launch_tc2_upgate(up, w->d_pad, w->F_pad, h, plan, E, rows, c->tc2_pairs,
                                 c->status, s));
        } else {
            up.tmB = w->tm_ug;
            CK(launch_tc_upgate(up, w->d_pad, w->F_pad, h, plan, E, rows, c->num_sms, c->status,
                                s));
        }
        MARK(3);
        if (pair && w->d_pad % 256 == 0) {
            dn.tmB = w->tm_dn128;
            CK(launch_tc2_down(dn, w->F_pad, w->d_pad, y, plan, E, rows, c->tc2_pairs, c->status,
                               s));
        } else {
            const int bn = down_tile_width(c, w, rows, &dn);
            CK(launch_tc_down(dn, w->F_pad, w->d_pad, bn, y, plan, E, rows, c->num_sms,
                              c->status, s));
        }
    } else if (path == MOE_B200_PATH_TF32X3 || onepass) {
        float *xs = nullptr, *hs = nullptr;
        if (!onepass) {
            if ((rc = grow(c->xs, (size_t)rows * w->d_pad * 4))) return rc;
            if ((rc = grow(c->hs, (size_t)rows * w->F_pad * 4))) return rc;
            xs = (float *)c->xs.p;
            hs = (float *)c->hs.p;
        }
        DecMaps up, dn;
        up.tmW = w->tm_ug64;
        if ((rc = make_tmap(&up.tmXb, x_perm, rows, w->d_pad, 64))) return rc;
        dn.tmW = w->tm_dn128;
        if ((rc = make_tmap(&dn.tmXb, h, rows, w->F_pad, 64))) return rc;
        if (onepass) {
            up.tmXs = up.tmXb32 = up.tmXb;
            dn.tmXs = dn.tmXb32 = dn.tmXb;
        } else {
            if ((rc = make_tmap(&up.tmXs, xs, rows, w->d_pad, 64))) return rc;
            if ((rc = make_tmap(&up.tmXb32, x_perm, rows, w->d_pad, 32))) return rc;
            if ((rc = make_tmap(&dn.tmXs, hs, rows, w->F_pad, 64))) return rc;
            if ((rc = make_tmap(&dn.tmXb32, h, rows, w->F_pad, 32))) return rc;
        }
        const int dpairs = (opts && opts->cta_pair && !onepass) ? c->dec_pairs : 0;
        if (!dpairs && dec_down_ksplit(w->F_pad, w->d_pad, rows, E, c->num_sms) == 2) {
            if ((rc = grow(c->y2, (size_t)rows * w->d_pad * 4))) return rc;
            y2 = (float *)c->y2.p;
        }
        if (!onepass) {
            CK(launch_split_tf32(x_perm, xs, (size_t)rows * w->d_pad, s));
            launches += 1;
        }
        CK(launch_dec_upgate(up, w->d_pad, w->F_pad, h, hs, plan, E, rows, c->num_sms, dpairs,
                             c->status, s, onepass));
        MARK(3);
        CK(launch_dec_down(dn, w->F_pad, w->d_pad, y, plan, E, rows, c->num_sms, dpairs,
                           c->status, s, nullptr, nullptr, y2, onepass));
    } else if (path == MOE_B200_PATH_FP32) {
        CK(launch_ffma_upgate(x_perm, w->d_pad, w->ug, w->F_pad, h, plan, E, rows, s));
        MARK(3);
        CK(launch_ffma_down(h, w->F_pad, w->dn, w->d_pad, y, plan, E, rows, s));
    } else {
        return fail(MOE_B200_E_INVALID, "unknown path %d", path);
    }
    launches += 2;
    MARK(4);
    CK(launch_combine(y, d, w->d_pad, T, k, pos_of, wts, d_out, s, y2, resid));
    launches += 1;
    MARK(5);
#undef MARK
    c->last_E = E;
    c->last_launches = launches;
    c->last_path = path;
    return MOE_B200_OK;
}

extern "C" int moe_b200_forward_device(const moe_b200_weights *w, const float *d_bias,
                                       const float *d_x, int T, float *d_out,
                                       float *d_router_probs, int *d_expert_ids,
                                       const moe_b200_opts *opts, void *stream) {
    if (!w) return fail(MOE_B200_E_INVALID, "null weights");
    if (T < 0) return fail(MOE_B200_E_INVALID, "T=%d", T);
    if (T == 0) return MOE_B200_OK;
    if (!d_x || !d_out) return fail(MOE_B200_E_INVALID, "null x/out");
    if (!aligned16(d_x) || !aligned16(d_out))
        return fail(MOE_B200_E_INVALID, "device x/out must be 16-byte aligned");
    if ((int64_t)T * w->k > (int64_t)1 << 30) return fail(MOE_B200_E_INVALID, "T too large");
    Ctx *c;
    int rc = get_ctx(w->device, &c);
    if (rc) return rc;
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    return forward_on(c, w, d_bias, d_x, T, d_out, d_router_probs, d_expert_ids, opts, s);
}

static int block_args_check(const moe_b200_weights *w, const void *rms_weight, const void *x,
                            int T) {
    if (!w) return fail(MOE_B200_E_INVALID, "null weights");
    if (T < 0) return fail(MOE_B200_E_INVALID, "T=%d", T);
    if (T > 0 && (!x || !rms_weight)) return fail(MOE_B200_E_INVALID, "null x/rms_weight");
    if ((int64_t)T * w->k > (int64_t)1 << 30) return fail(MOE_B200_E_INVALID, "T too large");
    if (w->d > rmsnorm_max_d()) return fail(MOE_B200_E_INVALID, "d=%d above the RMSNorm limit", w->d);
    return MOE_B200_OK;
}

extern "C" int moe_b200_block_ffn_device(const moe_b200_weights *w, const float *d_rms_weight,
                                         float eps, const float *d_bias, float *d_x, int T,
                                         float *d_x_norm, float *d_router_probs,
                                         int *d_expert_ids, const moe_b200_opts *opts,
                                         void *stream) {
    int rc = block_args_check(w, d_rms_weight, d_x, T);
    if (rc || T == 0) return rc;
    if (!aligned16(d_x) || (d_x_norm && !aligned16(d_x_norm)))
        return fail(MOE_B200_E_INVALID, "device x/x_norm must be 16-byte aligned");
    Ctx *c;
    if ((rc = get_ctx(w->device, &c))) return rc;
    if (!d_x_norm) {
        if ((rc = grow(c->xn, (size_t)T * w->d * 4))) return rc;
        d_x_norm = (float *)c->xn.p;
    }
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    const BlockNorm bn{d_rms_weight, eps, d_x_norm};
    return forward_on(c, w, d_bias, d_x, T, d_x, d_router_probs, d_expert_ids, opts, s, &bn);
}

// End of a synchronous host call on stream s: the status word comes back
// on the stream with the results (one pinned async copy), so one stream
// synchronisation covers both.
static int sync_and_check(Ctx *c, cudaStream_t s) {
    CK(cudaMemcpyAsync(c->h_status, c->status, sizeof(DeviceStatus), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    const DeviceStatus st = *c->h_status;
    if (st.timeout || st.bad_index) {
        CK(cudaMemset(c->status, 0, sizeof st));
        if (st.timeout)
            return fail(MOE_B200_E_TIMEOUT, "device wait timed out (site %d)", st.timeout);
        return fail(MOE_B200_E_CUDA, "device bounds check rejected an index");
    }
    return MOE_B200_OK;
}

// Chunks of the host-buffer forward.  Copies overlap compute only when a
// chunk's rows give the same bits as the whole call: the TF32 and FP32
// expert paths compute every row independently of the others, and the
// router sums its logits in one pass once a call has 64 router tiles (4033
// tokens).  Chunks are rounded up to whole router tiles, which can shorten
// the last one by up to 64 tokens per chunk, hence the 4096 + 64·kMaxChunks
// floor.  1 = no pipeline.
// The automatic count weighs the copies against the compute each extra chunk
// adds: smaller expert groups fill tensor-core tiles less well, which costs
// most when the expert weights dwarf the activations.  Measured end to end
// (pinned buffers): configuration 3 (weights 13x the activations) 4.07 ms
// in one chunk, 2.99 / 2.80 / 2.81 ms in 2 / 3 / 4; configuration 5 (45x)
// 112.9 ms in one, 100.6 / 103.0 / 104.6 ms in 2 / 3 / 4.
// tokens per chunk of a pipelined host call (the last chunk takes the rest)
static int chunk_tokens(int T, int chunks) {
    return (int)round_up(ceil_div(T, chunks), kRouterTile);
}

static int forward_chunks(const moe_b200_weights *w, int path, int T, size_t x_bytes, int want) {
    if (path != MOE_B200_PATH_TF32 && path != MOE_B200_PATH_FP32) return 1;
    if (x_bytes < ((size_t)64 << 20) || want == 1) return 1;
    const int most = std::min(Ctx::kMaxChunks, T / (4096 + 64 * Ctx::kMaxChunks));
    if (want <= 0) {
        const double weight_bytes = 3.0 * w->d * w->F * w->E * 4.0;
        want = weight_bytes > 24.0 * (double)x_bytes ? 2 : 3;
    }
    int n = std::max(1, std::min(want, most));
    // TF32 runs a different kernel on decode-sized groups: every chunk (the
    // last is the smallest) must fall on the same side as the whole call,
    // so that the result is bit-identical to one device call
    if (path == MOE_B200_PATH_TF32)
        while (n > 1 && decode_sized(w, T - (n - 1) * chunk_tokens(T, n)) != decode_sized(w, T))
            n--;
    return n;
}

static int ensure_pipeline(Ctx *c) {
    if (c->s_in) return MOE_B200_OK;
    CK(cudaStreamCreateWithFlags(&c->s_in, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&c->s_out, cudaStreamNonBlocking));
    for (int k = 0; k < Ctx::kMaxChunks; k++) {
        CK(cudaEventCreateWithFlags(&c->ev_in[k], cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&c->ev_done[k], cudaEventDisableTiming));
    }
    return MOE_B200_OK;
}

// The pipelined host-buffer forward: every chunk's H2D on s_in, its forward
// on the library stream once its rows have landed, its D2H on s_out once
// its forward is done.  With pinned host buffers the copies of one chunk
// overlap the compute of the others.
// block (optional): block_forward's FFN half; the result is x itself, updated
// in place in io_x, and x_norm (host, optional) receives the RMSNorm rows
// from the workspace xn.
struct HostBlock {
    const float *d_rms;
    float eps;
    float *x_norm;
};

static int forward_pipelined(Ctx *c, const moe_b200_weights *w, const float *d_bias,
                             const float *x, int T, float *out, float *router_probs,
                             int *expert_ids, const moe_b200_opts *opts, int chunks,
                             const HostBlock *block = nullptr) {
    int rc = ensure_pipeline(c);
    if (rc) return rc;
    const int d = w->d, E = w->E, k = w->k;
    const int Tc = chunk_tokens(T, chunks);
    float *io_x = (float *)c->io_x.p;
    float *io_out = block ? io_x : (float *)c->io_out.p;
    float *xn = block ? (float *)c->xn.p : nullptr;
    float *probs = (float *)c->probs.p;
    int *ids = (int *)c->ids.p;
    cudaStream_t s = c->stream;
    int n = 0;
    for (int t0 = 0; t0 < T; t0 += Tc, n++) {
        const size_t tn = (size_t)std::min(Tc, T - t0);
        // the previous call's D2H of this chunk must be done before its rows are reused
        CK(cudaStreamWaitEvent(c->s_in, c->ev_done[n], 0));
        CK(cudaMemcpyAsync(io_x + (size_t)t0 * d, x + (size_t)t0 * d, tn * d * 4,
                           cudaMemcpyHostToDevice, c->s_in));
        CK(cudaEventRecord(c->ev_in[n], c->s_in));
    }
    int launches = 0;
    n = 0;
    for (int t0 = 0; t0 < T; t0 += Tc, n++) {
        const int tn = std::min(Tc, T - t0);
        CK(cudaStreamWaitEvent(s, c->ev_in[n], 0));
        BlockNorm bn{};
        if (block) bn = BlockNorm{block->d_rms, block->eps, xn + (size_t)t0 * d};
        rc = forward_on(c, w, d_bias, io_x + (size_t)t0 * d, tn, io_out + (size_t)t0 * d,
                        probs + (size_t)t0 * E, ids + (size_t)t0 * k, opts, s,
                        block ? &bn : nullptr);
        if (rc) return rc;
        launches += c->last_launches;
        CK(cudaEventRecord(c->ev_done[n], s));
        CK(cudaStreamWaitEvent(c->s_out, c->ev_done[n], 0));
        CK(cudaMemcpyAsync(out + (size_t)t0 * d, io_out + (size_t)t0 * d, (size_t)tn * d * 4,
                           cudaMemcpyDeviceToHost, c->s_out));
        if (block && block->x_norm)
            CK(cudaMemcpyAsync(block->x_norm + (size_t)t0 * d, xn + (size_t)t0 * d,
                               (size_t)tn * d * 4, cudaMemcpyDeviceToHost, c->s_out));
        if (router_probs)
            CK(cudaMemcpyAsync(router_probs + (size_t)t0 * E, probs + (size_t)t0 * E,
                               (size_t)tn * E * 4, cudaMemcpyDeviceToHost, c->s_out));
        if (expert_ids)
            CK(cudaMemcpyAsync(expert_ids + (size_t)t0 * k, ids + (size_t)t0 * k,
                               (size_t)tn * k * 4, cudaMemcpyDeviceToHost, c->s_out));
    }
    c->last_launches = launches;
    CK(cudaStreamSynchronize(c->s_out));
    return sync_and_check(c, s);
}

extern "C" int moe_b200_forward(const moe_b200_weights *w, const float *router_bias,
                                const float *x, int T, float *out, float *router_probs,
                                int *expert_ids, const moe_b200_opts *opts) {
    if (!w) return fail(MOE_B200_E_INVALID, "null weights");
    if (T < 0) return fail(MOE_B200_E_INVALID, "T=%d", T);
    if (T == 0) return MOE_B200_OK;
    if (!x || !out) return fail(MOE_B200_E_INVALID, "null x/out");
    if ((int64_t)T * w->k > (int64_t)1 << 30) return fail(MOE_B200_E_INVALID, "T too large");
    Ctx *c;
    int rc = get_ctx(w->device, &c);
    if (rc) return rc;
    const size_t xb = (size_t)T * w->d * 4;
    if ((rc = grow(c->io_x, xb))) return rc;
    if ((rc = grow(c->io_out, xb))) return rc;
    if ((rc = grow(c->io_bias, (size_t)w->E * 4))) return rc;
    if ((rc = ensure_workspace(c, w, T))) return rc;
    cudaStream_t s = c->stream;
    const float *d_bias = nullptr;
    if (router_bias) {
        CK(cudaMemcpyAsync(c->io_bias.p, router_bias, (size_t)w->E * 4, cudaMemcpyHostToDevice, s));
        d_bias = (const float *)c->io_bias.p;
    }
    // the path is resolved once for the whole call, so every chunk runs the same one
    moe_b200_opts o;
    std::memset(&o, 0, sizeof o);
    if (opts) o = *opts;
    o.path = pick_path(w, T, opts);
    const int chunks = forward_chunks(w, o.path, T, xb, o.host_chunks);
    if (chunks > 1)
        return forward_pipelined(c, w, d_bias, x, T, out, router_probs, expert_ids, &o, chunks);
    CK(cudaMemcpyAsync(c->io_x.p, x, xb, cudaMemcpyHostToDevice, s));
    rc = forward_on(c, w, d_bias, (const float *)c->io_x.p, T, (float *)c->io_out.p,
                    (float *)c->probs.p, (int *)c->ids.p, &o, s);
    if (rc) return rc;
    CK(cudaMemcpyAsync(out, c->io_out.p, xb, cudaMemcpyDeviceToHost, s));
    if (router_probs)
        CK(cudaMemcpyAsync(router_probs, c->probs.p, (size_t)T * w->E * 4, cudaMemcpyDeviceToHost, s));
    if (expert_ids)
        CK(cudaMemcpyAsync(expert_ids, c->ids.p, (size_t)T * w->k * 4, cudaMemcpyDeviceToHost, s));
    return sync_and_check(c, s);
}

extern "C" int moe_b200_block_ffn(const moe_b200_weights *w, const float *rms_weight, float eps,
                                  const float *router_bias, float *x, int T, float *x_norm,
                                  float *router_probs, int *expert_ids,
                                  const moe_b200_opts *opts) {
    int rc = block_args_check(w, rms_weight, x, T);
    if (rc || T == 0) return rc;
    Ctx *c;
    if ((rc = get_ctx(w->device, &c))) return rc;
    const size_t xb = (size_t)T * w->d * 4;
    if ((rc = grow(c->io_x, xb))) return rc;
    if ((rc = grow(c->xn, xb))) return rc;
    if ((rc = grow(c->io_rms, (size_t)w->d * 4))) return rc;
    if ((rc = grow(c->io_bias, (size_t)w->E * 4))) return rc;
    if ((rc = ensure_workspace(c, w, T))) return rc;
    cudaStream_t s = c->stream;
    CK(cudaMemcpyAsync(c->io_rms.p, rms_weight, (size_t)w->d * 4, cudaMemcpyHostToDevice, s));
    const float *d_bias = nullptr;
    if (router_bias) {
        CK(cudaMemcpyAsync(c->io_bias.p, router_bias, (size_t)w->E * 4, cudaMemcpyHostToDevice, s));
        d_bias = (const float *)c->io_bias.p;
    }
    moe_b200_opts o;
    std::memset(&o, 0, sizeof o);
    if (opts) o = *opts;
    o.path = pick_path(w, T, opts);
    const int chunks = forward_chunks(w, o.path, T, xb, o.host_chunks);
    if (chunks > 1) {
        const HostBlock hb{(const float *)c->io_rms.p, eps, x_norm};
        return forward_pipelined(c, w, d_bias, x, T, x, router_probs, expert_ids, &o, chunks, &hb);
    }
    CK(cudaMemcpyAsync(c->io_x.p, x, xb, cudaMemcpyHostToDevice, s));
    const BlockNorm bn{(const float *)c->io_rms.p, eps, (float *)c->xn.p};
    rc = forward_on(c, w, d_bias, (const float *)c->io_x.p, T, (float *)c->io_x.p,
                    (float *)c->probs.p, (int *)c->ids.p, &o, s, &bn);
    if (rc) return rc;
    CK(cudaMemcpyAsync(x, c->io_x.p, xb, cudaMemcpyDeviceToHost, s));
    if (x_norm) CK(cudaMemcpyAsync(x_norm, c->xn.p, xb, cudaMemcpyDeviceToHost, s));
    if (router_probs)
        CK(cudaMemcpyAsync(router_probs, c->probs.p, (size_t)T * w->E * 4, cudaMemcpyDeviceToHost, s));
    if (expert_ids)
        CK(cudaMemcpyAsync(expert_ids, c->ids.p, (size_t)T * w->k * 4, cudaMemcpyDeviceToHost, s));
    return sync_and_check(c, s);
}

// ---------------------------------------------------------------------
// backward (moe_backward.cu): gradient buffers in llm.c's layouts
// ---------------------------------------------------------------------
struct moe_b200_grads {
    int device = -1;
    int d = 0, F = 0, E = 0;
    float *router = nullptr, *bias = nullptr, *gate = nullptr, *up = nullptr, *down = nullptr;
};

static void grads_release(moe_b200_grads *g) {
    for (float *p : {g->router, g->bias, g->gate, g->up, g->down})
        if (p) cudaFree(p);
    delete g;
}

extern "C" int moe_b200_grads_create(const moe_b200_weights *w, moe_b200_grads **out) {
    if (!w || !out) return fail(MOE_B200_E_INVALID, "null argument");
    *out = nullptr;
    Ctx *c;
    int rc = weights_full(w);
    if (rc) return rc;
    if ((rc = get_ctx(w->device, &c))) return rc;
    auto *g = new moe_b200_grads();
    g->device = w->device;
    g->d = w->d; g->F = w->F; g->E = w->E;
    const size_t dE = (size_t)w->d * w->E, dFE = (size_t)w->d * w->F * w->E;
    const struct { float **p; size_t n; } parts[] = {
        {&g->router, dE}, {&g->bias, (size_t)w->E}, {&g->gate, dFE}, {&g->up, dFE}, {&g->down, dFE}};
    for (const auto &pt : parts) {
        if (cudaMalloc(pt.p, pt.n * 4) != cudaSuccess || cudaMemset(*pt.p, 0, pt.n * 4) != cudaSuccess) {
            cudaGetLastError();
            grads_release(g);
            return fail(MOE_B200_E_NOMEM, "gradient buffers");
        }
    }
    *out = g;
    return MOE_B200_OK;
}

extern "C" int moe_b200_grads_zero(moe_b200_grads *g) {
    if (!g) return fail(MOE_B200_E_INVALID, "null gradients");
    const size_t dE = (size_t)g->d * g->E, dFE = (size_t)g->d * g->F * g->E;
    CK(cudaMemset(g->router, 0, dE * 4));
    CK(cudaMemset(g->bias, 0, (size_t)g->E * 4));
    CK(cudaMemset(g->gate, 0, dFE * 4));
    CK(cudaMemset(g->up, 0, dFE * 4));
    CK(cudaMemset(g->down, 0, dFE * 4));
    return MOE_B200_OK;
}

extern "C" int moe_b200_grads_download(const moe_b200_grads *g, float *dW_router, float *d_bias,
                                       float *const *dW_gate, float *const *dW_up,
                                       float *const *dW_down) {
    if (!g) return fail(MOE_B200_E_INVALID, "null gradients");
    CK(cudaDeviceSynchronize());
    const size_t dF = (size_t)g->d * g->F;
    if (dW_router) CK(cudaMemcpy(dW_router, g->router, (size_t)g->d * g->E * 4, cudaMemcpyDeviceToHost));
    if (d_bias) CK(cudaMemcpy(d_bias, g->bias, (size_t)g->E * 4, cudaMemcpyDeviceToHost));
    for (int e = 0; e < g->E; e++) {
        if (dW_gate && dW_gate[e])
            CK(cudaMemcpy(dW_gate[e], g->gate + e * dF, dF * 4, cudaMemcpyDeviceToHost));
        if (dW_up && dW_up[e])
            CK(cudaMemcpy(dW_up[e], g->up + e * dF, dF * 4, cudaMemcpyDeviceToHost));
        if (dW_down && dW_down[e])
            CK(cudaMemcpy(dW_down[e], g->down + e * dF, dF * 4, cudaMemcpyDeviceToHost));
    }
    return MOE_B200_OK;
}

extern "C" int moe_b200_grads_free(moe_b200_grads *g) {
    if (!g) return MOE_B200_OK;
    cudaDeviceSynchronize();
    grads_release(g);
    return MOE_B200_OK;
}

// The forward again (saving the gate/up pre-activations), then the backward
// kernels, all on stream s.  FP32: FFMA GEMMs, every expert segment packed.
// TF32: tcgen05 GEMMs; expert segments start at multiples of 32 rows with
// zeroed alignment rows, because the weight-gradient GEMMs run K over them.
static int backward_on(Ctx *c, const moe_b200_weights *w, const float *d_bias, const float *d_x,
                       int T, const float *d_dy, float aux_coef, float *d_dx, moe_b200_grads *g,
                       float *d_aux, const moe_b200_opts *opts, cudaStream_t s) {
    int rc = weights_full(w);
    if (rc) return rc;
    if ((rc = ensure_workspace(c, w, T))) return rc;
    const int E = w->E, k = w->k, d = w->d;
    int path = pick_path(w, T, opts);
    if (path != MOE_B200_PATH_TF32) path = MOE_B200_PATH_FP32;
    const bool tc = path == MOE_B200_PATH_TF32;
    const size_t rows = (size_t)T * k;
    const size_t rows_buf = tc ? rows + (size_t)31 * E : rows;      // with alignment rows
    if ((rc = grow(c->x_perm, rows_buf * w->d_pad * 4)) || (rc = grow(c->h, rows_buf * w->F_pad * 4)) ||
        (rc = grow(c->y, rows_buf * w->d_pad * 4)) || (rc = grow(c->gu, rows_buf * 2 * w->F_pad * 4)) ||
        (rc = grow(c->dO, rows_buf * w->d_pad * 4)) || (rc = grow(c->dgu, rows_buf * 2 * w->F_pad * 4)) ||
        (rc = grow(c->dw, rows * 4)) || (rc = grow(c->dlogit, (size_t)T * E * 4)) ||
        (rc = grow(c->pmean, (size_t)E * 4)) ||
        (rc = grow(c->wr_part, (size_t)router_wgrad_splits(T, d, E) * d * E * 4)))
        return rc;
    float *probs = (float *)c->probs.p, *wts = (float *)c->wts.p;
    int *ids = (int *)c->ids.p, *plan = (int *)c->plan.p, *pos_of = (int *)c->pos_of.p;
    float *x_perm = (float *)c->x_perm.p, *h = (float *)c->h.p, *y = (float *)c->y.p;
    float *gu = (float *)c->gu.p, *dO = (float *)c->dO.p, *dgu = (float *)c->dgu.p;
    const int nsplit = router_splits(T, d);
    if (nsplit > 1 && (rc = grow(c->rpart, (size_t)nsplit * T * E * 4))) return rc;
    CK(launch_router(d_x, T, d, w->router, d_bias, E, k, probs, ids, wts, (int *)c->loc.p,
                     (int *)c->tile_cnt.p, s, (float *)c->rpart.p, nsplit));
    CK(launch_dispatch(d_x, T, d, w->d_pad, E, k, ids, (int *)c->loc.p, (int *)c->tile_cnt.p,
                       (int *)c->tile_pref.p, plan, pos_of, x_perm, tc ? 1 : 0, c->status, s,
                       tc ? 32 : 1));
    int fwd_launches = (nsplit > 1 ? 2 : 1) + 2;
    if (tc) {
        CK(launch_zero_pad_rows(x_perm, w->d_pad, plan, E, s));
        TcGemm up, dn;
        if ((rc = make_tmap(&up.tmA, x_perm, (int64_t)rows_buf, w->d_pad, 128))) return rc;
        if ((rc = make_tmap(&dn.tmA, h, (int64_t)rows_buf, w->F_pad, 128))) return rc;
        up.tmB = w->tm_ug;
        const int bn = down_tile_width(c, w, (int)rows, &dn);
        CK(launch_tc_upgate(up, w->d_pad, w->F_pad, h, plan, E, (int)rows, c->num_sms, c->status,
                            s, gu));
        CK(launch_zero_pad_rows(h, w->F_pad, plan, E, s));
        CK(launch_tc_down(dn, w->F_pad, w->d_pad, bn, y, plan, E, (int)rows, c->num_sms,
                          c->status, s, nullptr, nullptr));
        fwd_launches += 4;
    } else {
        CK(launch_ffma_upgate(x_perm, w->d_pad, w->ug, w->F_pad, h, plan, E, (int)rows, s, gu));
        CK(launch_ffma_down(h, w->F_pad, w->dn, w->d_pad, y, plan, E, (int)rows, s));
        fwd_launches += 2;
    }
    BwdArgs a{};
    a.T = T; a.d = d; a.E = E; a.k = k; a.F = w->F; a.d_pad = w->d_pad; a.F_pad = w->F_pad;
    a.rows_bound = (int)rows;
    a.plan = plan; a.pos_of = pos_of; a.ids = ids;
    a.x = d_x; a.x_perm = x_perm; a.gu = (const float *)c->gu.p; a.h = h; a.y = y;
    a.probs = probs; a.wts = wts;
    a.router = w->router; a.ug = w->ug; a.dn = w->dn;
    a.dy = d_dy; a.aux_coef = aux_coef;
    a.dw = (float *)c->dw.p; a.dO = (float *)c->dO.p; a.dgu = (float *)c->dgu.p;
    a.dxp = y;                                // y is last read by the combine backward
    a.dlogit = (float *)c->dlogit.p; a.pmean = (float *)c->pmean.p;
    a.wr_part = (float *)c->wr_part.p;
    a.dx = d_dx;
    a.g_router = g->router; a.g_bias = g->bias; a.g_gate = g->gate; a.g_up = g->up;
    a.g_down = g->down;
    a.aux_loss = d_aux;
    a.round_tf32 = tc ? 1 : 0;
    int n = 0;
    if (!tc) {
        CK(launch_moe_backward(a, s, &n));
    } else {
        CK(launch_bwd_head(a, s, &n));
        CK(launch_zero_pad_rows(dO, w->d_pad, plan, E, s));
        TcBwd b{};
        const int64_t rb = (int64_t)rows_buf;
        if ((rc = make_tmap(&b.tm_dO_k, dO, rb, w->d_pad, 128)) ||
            (rc = make_tmap(&b.tm_dn_mn, w->dn, (int64_t)E * w->d_pad, w->F_pad, 32, true)) ||
            (rc = make_tmap(&b.tm_h_mn, h, rb, w->F_pad, 32, true)) ||
            (rc = make_tmap(&b.tm_dO_mn, dO, rb, w->d_pad, 32, true)) ||
            (rc = make_tmap(&b.tm_x_mn, x_perm, rb, w->d_pad, 32, true)) ||
            (rc = make_tmap(&b.tm_dgu_mn, dgu, rb, 2 * w->F_pad, 32, true)) ||
            (rc = make_tmap(&b.tm_dgu_k, dgu, rb, 2 * w->F_pad, 128)) ||
            (rc = make_tmap(&b.tm_ug_mn, w->ug, (int64_t)E * 2 * w->F_pad, w->d_pad, 32, true)))
            return rc;
        b.plan = plan;
        b.E = E; b.d = d; b.F = w->F; b.d_pad = w->d_pad; b.F_pad = w->F_pad;
        b.rows_bound = (int)rows; b.num_sms = c->num_sms;
        b.gu = gu; b.dgu = dgu; b.dxp = y;
        b.g_down = g->down; b.g_gate = g->gate; b.g_up = g->up;
        b.status = c->status;
        CK(launch_tc_bwd(b, s));
        CK(launch_bwd_tail(a, s, &n));
        n += 1 + 5;         // dO alignment rows; dH, dGU alignment rows, dWd, dWgu, dX
    }
    c->last_E = E;
    c->last_launches = fwd_launches + n;
    c->last_path = path;
    return MOE_B200_OK;
}

static int backward_args_check(const moe_b200_weights *w, const moe_b200_grads *g, int T) {
    if (!w || !g) return fail(MOE_B200_E_INVALID, "null weights or gradients");
    if (g->d != w->d || g->F != w->F || g->E != w->E || g->device != w->device)
        return fail(MOE_B200_E_INVALID, "gradients were made for another expert set");
    if (T < 0) return fail(MOE_B200_E_INVALID, "T=%d", T);
    if ((int64_t)T * w->k > (int64_t)1 << 30) return fail(MOE_B200_E_INVALID, "T too large");
    return MOE_B200_OK;
}

extern "C" int moe_b200_backward_device(const moe_b200_weights *w, const float *d_bias,
                                        const float *d_x, int T, const float *d_dy,
                                        float aux_coef, float *d_dx, moe_b200_grads *g,
                                        float *d_aux_loss, const moe_b200_opts *opts,
                                        void *stream) {
    int rc = backward_args_check(w, g, T);
    if (rc || T == 0) return rc;
    if (!d_x || !d_dy || !d_dx) return fail(MOE_B200_E_INVALID, "null x, dy or dx");
    if (!aligned16(d_x) || !aligned16(d_dy) || !aligned16(d_dx))
        return fail(MOE_B200_E_INVALID, "device x, dy and dx must be 16-byte aligned");
    Ctx *c;
    if ((rc = get_ctx(w->device, &c))) return rc;
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    return backward_on(c, w, d_bias, d_x, T, d_dy, aux_coef, d_dx, g, d_aux_loss, opts, s);
}

extern "C" int moe_b200_backward(const moe_b200_weights *w, const float *router_bias,
                                 const float *x, int T, const float *dy, float aux_coef, float *dx,
                                 moe_b200_grads *g, float *aux_loss, const moe_b200_opts *opts) {
    int rc = backward_args_check(w, g, T);
    if (rc) return rc;
    if (T == 0) {
        if (aux_loss) *aux_loss = 0.0f;
        return MOE_B200_OK;
    }
    if (!x || !dy || !dx) return fail(MOE_B200_E_INVALID, "null x, dy or dx");
    Ctx *c;
    if ((rc = get_ctx(w->device, &c))) return rc;
    const size_t xb = (size_t)T * w->d * 4;
    if ((rc = grow(c->io_x, xb)) || (rc = grow(c->io_dy, xb)) || (rc = grow(c->io_dx, xb)) ||
        (rc = grow(c->io_bias, (size_t)w->E * 4)) || (rc = grow(c->io_aux, 4)))
        return rc;
    cudaStream_t s = c->stream;
    CK(cudaMemcpyAsync(c->io_x.p, x, xb, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(c->io_dy.p, dy, xb, cudaMemcpyHostToDevice, s));
    const float *d_bias = nullptr;
    if (router_bias) {
        CK(cudaMemcpyAsync(c->io_bias.p, router_bias, (size_t)w->E * 4, cudaMemcpyHostToDevice, s));
        d_bias = (const float *)c->io_bias.p;
    }
    rc = backward_on(c, w, d_bias, (const float *)c->io_x.p, T, (const float *)c->io_dy.p,
                     aux_coef, (float *)c->io_dx.p, g, aux_loss ? (float *)c->io_aux.p : nullptr,
                     opts, s);
    if (rc) return rc;
    CK(cudaMemcpyAsync(dx, c->io_dx.p, xb, cudaMemcpyDeviceToHost, s));
    if (aux_loss) CK(cudaMemcpyAsync(aux_loss, c->io_aux.p, 4, cudaMemcpyDeviceToHost, s));
    return sync_and_check(c, s);
}

extern "C" int moe_b200_last_counts(const moe_b200_weights *w, int *counts) {
    if (!w || !counts) return fail(MOE_B200_E_INVALID, "null argument");
    Ctx *c;
    int rc = get_ctx(w->device, &c);
    if (rc) return rc;
    if (!c->plan.p || c->last_E != w->E) return fail(MOE_B200_E_STATE, "no forward on record");
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaMemcpy(counts, c->plan.p, (size_t)w->E * 4, cudaMemcpyDeviceToHost));
    return MOE_B200_OK;
}

extern "C" int moe_b200_last_path(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64 || !g_ctx[dev]) return 0;
    return g_ctx[dev]->last_path;
}

extern "C" int moe_b200_last_launches(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64 || !g_ctx[dev]) return 0;
    return g_ctx[dev]->last_launches;
}

// hooks for the expert-parallel forward (ep.cu): the same stage timing and
// launch count as a single-GPU forward on this device
cudaEvent_t *moe::profile_events(int device) {
    Ctx *c;
    if (get_ctx(device, &c)) return nullptr;
    return prof_slot(c);
}

void moe::note_forward(int device, int E, int launches, int path) {
    Ctx *c;
    if (get_ctx(device, &c)) return;
    c->last_E = E;
    c->last_launches = launches;
    c->last_path = path;
}

extern "C" int moe_b200_device_info(int device, int *num_sms, int *cta_pairs) {
    Ctx *c;
    int rc = get_ctx(device, &c);
    if (rc) return rc;
    if (num_sms) *num_sms = c->num_sms;
    if (cta_pairs) *cta_pairs = c->tc2_pairs;
    return MOE_B200_OK;
}

int moe::device_sms(int device) {
    Ctx *c;
    if (get_ctx(device, &c)) return 0;
    return c->num_sms;
}

extern "C" int moe_b200_synth_fill(float *d_dst, size_t n, uint64_t seed, uint64_t stream,
                                   uint64_t first, float std, void *cuda_stream) {
    if (!d_dst && n) return fail(MOE_B200_E_INVALID, "null destination");
    Ctx *c;
    int rc = get_ctx(-1, &c);
    if (rc) return rc;
    cudaStream_t s = cuda_stream ? (cudaStream_t)cuda_stream : c->stream;
    CK(launch_synth(d_dst, n, seed, stream, first, std, s));
    if (!cuda_stream) CK(cudaStreamSynchronize(s));
    return MOE_B200_OK;
}

extern "C" int moe_b200_profile_enable(int enable) {
    Ctx *c;
    int rc = get_ctx(-1, &c);
    if (rc) return rc;
    c->prof = enable != 0;
    return MOE_B200_OK;
}

extern "C" int moe_b200_profile_read(double *stage_ms, int *n_forwards) {
    Ctx *c;
    int rc = get_ctx(-1, &c);
    if (rc) return rc;
    for (int i = 0; i < Ctx::kSlots; i++)
        if ((rc = fold_slot(c, i))) return rc;
    if (stage_ms)
        for (int i = 0; i < MOE_B200_NUM_STAGES; i++) stage_ms[i] = c->stage_ms[i];
    if (n_forwards) *n_forwards = c->n_timed;
    for (int i = 0; i < MOE_B200_NUM_STAGES; i++) c->stage_ms[i] = 0.0;
    c->n_timed = 0;
    return MOE_B200_OK;
}
