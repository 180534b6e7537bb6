// noalloc.cu — moe_b200_forward_noalloc: the MoE forward on the FP32 expert
// path with all of its scratch in one fixed, statically allocated device
// array instead of the library's cudaMalloc-grown workspace.
//
// Who needs it: callers that must not allocate device memory while they
// run.  Examples are a serving or decode loop that lives inside a memory
// budget fixed at start-up, a host program whose device memory belongs to
// another framework's caching allocator (a raw cudaMalloc/cudaFree would
// fragment or synchronise it), and latency-critical code that may not call
// into the CUDA allocator.  Such a caller builds its weights once at set-up
// (moe_b200_weights_upload does allocate) and afterwards passes only its
// own device buffers for inputs and outputs.
//
// The array is part of the library image: every GPU that loads the library
// holds MOE_B200_NOALLOC_SCRATCH_BYTES of device memory for it until the
// process exits.
#include "../../include/moe_b200.h"
#include "kernels.cuh"
#include "weights.cuh"

#include <cstdio>
#include <mutex>

using namespace moe;

// One scratch array, shared by every call on a device.  It keeps the last
// call's contents; calls that overlap on the GPU (two streams, or two host
// threads on the same device) race on it.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MOE_B200_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_na_mu;
unsigned char *g_na_ptr[kMaxDevices] = {nullptr};   // device address of the array, per device

// Set-up, once per device, with that device current.  On the host the
// array's name is only a stand-in for the device symbol, so its device
// address has to be fetched before any kernel can be given it.  The cached
// address belongs to the device's current context: it does not survive a
// cudaDeviceReset of that device (the library has to be reloaded then).
int na_setup(int dev, unsigned char **ptr) {
    if (dev < 0 || dev >= kMaxDevices)
        return set_last_error(MOE_B200_E_INVALID,
                              "moe_b200_forward_noalloc: device ordinal beyond 63");
    std::lock_guard<std::mutex> lk(g_na_mu);
    if (!g_na_ptr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            char msg[200];
            std::snprintf(msg, sizeof msg, "cudaGetSymbolAddress(scratch) failed: %s",
                          cudaGetErrorString(e));
            return set_last_error(MOE_B200_E_CUDA, msg);
        }
        g_na_ptr[dev] = static_cast<unsigned char *>(p);
    }
    *ptr = g_na_ptr[dev];
    return MOE_B200_OK;
}

// Bump carving of 256-byte aligned regions out of the array (or, with a
// null base, a dry run that only sums the sizes).
struct Carve {
    unsigned char *base;
    size_t used;
    template <typename T>
    T *take(size_t count) {
        T *p = base ? reinterpret_cast<T *>(base + used) : nullptr;
        used += (count * sizeof(T) + 255) & ~static_cast<size_t>(255);
        return p;
    }
};

struct Scratch {
    DeviceStatus *status;
    float *probs, *wts, *x_perm, *h, *y;
    int *ids, *loc, *pos_of, *tile_cnt, *tile_pref, *plan;
};

size_t carve(const moe_b200_weights *w, int T, unsigned char *base, Scratch *s) {
    const size_t Tk = (size_t)T * w->k, tiles = ceil_div(T, kRouterTile);
    Carve c{base, 0};
    s->status = c.take<DeviceStatus>(1);
    s->probs = c.take<float>((size_t)T * w->E);   // used when the caller passes none
    s->ids = c.take<int>(Tk);                      // used when the caller passes none
    s->wts = c.take<float>(Tk);
    s->loc = c.take<int>(Tk);
    s->pos_of = c.take<int>(Tk);
    s->tile_cnt = c.take<int>(tiles * w->E);
    s->tile_pref = c.take<int>(tiles * w->E);
    s->plan = c.take<int>(plan_ints(w->E));
    s->x_perm = c.take<float>(Tk * w->d_pad);
    s->h = c.take<float>(Tk * w->F_pad);
    s->y = c.take<float>(Tk * w->d_pad);
    return c.used;
}

int na_cuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return MOE_B200_OK;
    char msg[200];
    std::snprintf(msg, sizeof msg, "%s failed: %s", what, cudaGetErrorString(e));
    return set_last_error(MOE_B200_E_CUDA, msg);
}

}  // namespace

extern "C" int moe_b200_forward_noalloc(const moe_b200_weights *w, const float *d_bias,
                                        const float *d_x, int T, float *d_out,
                                        float *d_router_probs, int *d_expert_ids,
                                        void *stream) {
    if (!w || !d_x || !d_out)
        return set_last_error(MOE_B200_E_INVALID, "moe_b200_forward_noalloc: null weights, x or out");
    if (T < 0) return set_last_error(MOE_B200_E_INVALID, "moe_b200_forward_noalloc: T < 0");
    if (((uintptr_t)d_x | (uintptr_t)d_out) & 15)
        return set_last_error(MOE_B200_E_INVALID,
                              "moe_b200_forward_noalloc: x and out must be 16-byte aligned");
    if (T == 0) return MOE_B200_OK;
    if (int rcf = weights_full(w)) return rcf;
    Scratch sc;
    const size_t need = carve(w, T, nullptr, &sc);
    if ((int64_t)T * w->k > (int64_t)1 << 30 || need > (size_t)MOE_B200_NOALLOC_SCRATCH_BYTES) {
        char msg[256];
        std::snprintf(msg, sizeof msg,
                      "moe_b200_forward_noalloc: T=%d needs %zu bytes of scratch, more than the "
                      "%zu-byte static array; split the call into smaller T",
                      T, need, (size_t)MOE_B200_NOALLOC_SCRATCH_BYTES);
        return set_last_error(MOE_B200_E_INVALID, msg);
    }
    int dev = -1;
    int rc = na_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc) return rc;
    if (dev != w->device)
        return set_last_error(MOE_B200_E_INVALID,
                              "moe_b200_forward_noalloc: the weights live on another device");
    unsigned char *base = nullptr;
    if ((rc = na_setup(dev, &base))) return rc;
    carve(w, T, base, &sc);
    float *probs = d_router_probs ? d_router_probs : sc.probs;
    int *ids = d_expert_ids ? d_expert_ids : sc.ids;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int rows = T * w->k;

    // Only the status word must start at zero; every other region is fully
    // written by the kernel that produces it before any kernel reads it.
    if ((rc = na_cuda(cudaMemsetAsync(sc.status, 0, sizeof(DeviceStatus), s), "cudaMemsetAsync")))
        return rc;
    if ((rc = na_cuda(launch_router(d_x, T, w->d, w->router, d_bias, w->E, w->k, probs, ids,
                                    sc.wts, sc.loc, sc.tile_cnt, s), "router launch")))
        return rc;
    if ((rc = na_cuda(launch_dispatch(d_x, T, w->d, w->d_pad, w->E, w->k, ids, sc.loc,
                                      sc.tile_cnt, sc.tile_pref, sc.plan, sc.pos_of, sc.x_perm,
                                      0, sc.status, s), "dispatch launch")))
        return rc;
    if ((rc = na_cuda(launch_ffma_upgate(sc.x_perm, w->d_pad, w->ug, w->F_pad, sc.h, sc.plan,
                                         w->E, rows, s), "expert up/gate launch")))
        return rc;
    if ((rc = na_cuda(launch_ffma_down(sc.h, w->F_pad, w->dn, w->d_pad, sc.y, sc.plan, w->E,
                                       rows, s), "expert down launch")))
        return rc;
    if ((rc = na_cuda(launch_combine(sc.y, w->d, w->d_pad, T, w->k, sc.pos_of, sc.wts, d_out, s),
                      "combine launch")))
        return rc;
    // the status word comes back on the caller's stream, then one wait
    DeviceStatus st;
    if ((rc = na_cuda(cudaMemcpyAsync(&st, sc.status, sizeof st, cudaMemcpyDeviceToHost, s),
                      "cudaMemcpyAsync")))
        return rc;
    if ((rc = na_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize"))) return rc;
    if (st.bad_index)
        return set_last_error(MOE_B200_E_CUDA, "device bounds check rejected an index");
    if (st.timeout) return set_last_error(MOE_B200_E_TIMEOUT, "device wait timed out");
    return MOE_B200_OK;
}
