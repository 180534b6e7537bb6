// ep.cu — expert-parallel MoE forward over NVLink (one process per GPU).
//
// Load balance by work, not by expert: every rank holds the full expert
// set (replicated weights; c5's 45 GB fits a B200), routes its own tokens,
// and all ranks derive the same partition of the GLOBAL expert-sorted row
// order into G equal contiguous slices.  Rank q computes the expert GEMMs of
// slice q.  The global order is expert-major, then source rank, then the
// source's stable local order, so:
//   * the rows a rank sends to one slice owner form one contiguous run of
//     its local expert-sorted order;
//   * the owner's slice is already grouped by expert, with the same plan
//     format the single-GPU grouped GEMMs read.
//
// Data movement is fused into the kernels and uses no NCCL data
// collectives.  The dispatch gather stores each token row straight into
// the slice owner's receive buffer (CUDA IPC peer mapping, NVLink stores),
// with a return address (source rank, source row).  The down GEMM's
// epilogue stores each result row straight back into the token owner's
// output buffer.  NCCL carries only the per-expert counts (E ints per rank)
// and two stream-ordered barriers, so a forward never waits on the host.
// No TMA ever reads peer memory; every CTA loads only its own tiles.
//
// Stream order per forward on rank r (every rank issues the same NCCL
// calls in the same order):
//   router -> scan -> allgather(counts) -> partition -> gather(peer stores)
//   -> barrier -> up/gate -> down(peer stores) -> barrier -> combine
#include "../../include/moe_b200.h"
#include "kernels.cuh"
#include "weights.cuh"

#include "nccl_dyn.cuh"

#include <cstdio>
#include <cstring>
#include <vector>

using namespace moe;

// ---------------------------------------------------------------------
// partition (host copy: tests and diagnostics; device copy: the forward)
//
// Slices are balanced on estimated cost, not on rows: the grouped GEMMs
// spend per 128-row m-tile, and each expert segment of a slice adds about
// half an m-tile more (its partially filled last tile and its own pass over
// the expert's weights).  So an expert with n rows costs 2·ceil(n/128) + 1
// units, and slice boundaries fall on m-tile boundaries inside experts.  A
// slice may then hold somewhat more rows than T·k/G; if any slice would
// exceed the receive capacity, the partition falls back to equal rows.
// Integer arithmetic throughout, so every rank (and the host copy) derives
// the same boundaries.
// ---------------------------------------------------------------------
__host__ __device__ inline void ep_slices(const int *C, int G, int E, long long capacity,
                                          long long *S /* G+1 */) {
    long long M = 0, U = 0;
    for (int e = 0; e < E; e++) {
        long long tot = 0;
        for (int r = 0; r < G; r++) tot += C[r * E + e];
        M += tot;
        U += 2 * ((tot + 127) / 128) + (tot > 0 ? 1 : 0);
    }
    S[0] = 0;
    int q = 1;
    long long cum = 0, goff = 0;
    for (int e = 0; e < E && q < G; e++) {
        long long tot = 0;
        for (int r = 0; r < G; r++) tot += C[r * E + e];
        const long long tiles = (tot + 127) / 128;
        const long long units = 2 * tiles + (tot > 0 ? 1 : 0);
        // boundary q sits at cost q·U/G; place it inside this expert when the
        // expert's cost range reaches it
        while (q < G && (long long)q * U <= (long long)G * (cum + units)) {
            const long long num = (long long)q * U - (long long)G * (cum + 1);   // 2t·G ≈ num
            long long t = num <= 0 ? 0 : (num + G) / (2LL * G);
            if (t > tiles) t = tiles;
            const long long rows = 128 * t < tot ? 128 * t : tot;
            S[q] = goff + rows;
            q++;
        }
        cum += units;
        goff += tot;
    }
    for (; q < G; q++) S[q] = M;
    S[G] = M;
    bool fits = true;
    for (q = 1; q <= G; q++) {
        if (S[q] < S[q - 1]) S[q] = S[q - 1];
        if (capacity > 0 && S[q] - S[q - 1] > capacity) fits = false;
    }
    if (!fits) {                               // equal rows always fit
        const long long chunk = M > 0 ? (M + G - 1) / G : 1;
        for (q = 0; q <= G; q++) S[q] = (long long)q * chunk < M ? (long long)q * chunk : M;
    }
}

__host__ __device__ inline void ep_partition(const int *C, int G, int E, int rank,
                                             long long capacity, int *cnt_q, int *base_r,
                                             long long *S /* G+1 */) {
    ep_slices(C, G, E, capacity, S);
    const long long lo = S[rank], hi = S[rank + 1];
    long long goff = 0;
    for (int e = 0; e < E; e++) {
        long long tot = 0, before = 0;
        for (int r = 0; r < G; r++) {
            if (r < rank) before += C[r * E + e];
            tot += C[r * E + e];
        }
        const long long a = goff > lo ? goff : lo;
        const long long b = goff + tot < hi ? goff + tot : hi;
        if (cnt_q) cnt_q[e] = b > a ? (int)(b - a) : 0;
        if (base_r) base_r[e] = (int)(goff + before);
        goff += tot;
    }
}

// One thread: this rank's slice plan (cnt | off | mt128 | mt64 | mt256), the global
// base of this rank's rows per expert, and the slice boundaries.
__global__ void ep_plan_kernel(const int *__restrict__ counts_all, int G, int E, int rank,
                               long long capacity, int *__restrict__ plan,
                               int *__restrict__ base_r, int *__restrict__ slices)
{
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int *cnt = plan, *off = plan + E, *mt128 = off + E + 1, *mt64 = mt128 + E + 1;
    int *mt256 = mt64 + E + 1;
    long long S[65];
    ep_partition(counts_all, G, E, rank, capacity, cnt, base_r, S);
    int o = 0, m1 = 0, m2 = 0, m3 = 0;
    for (int e = 0; e < E; e++) {
        off[e] = o; mt128[e] = m1; mt64[e] = m2; mt256[e] = m3;
        o += cnt[e];
        m1 += (cnt[e] + 127) / 128;
        m2 += (cnt[e] + 63) / 64;
        m3 += (cnt[e] + 255) / 256;
    }
    off[E] = o; mt128[E] = m1; mt64[E] = m2; mt256[E] = m3;
    for (int q = 0; q <= G; q++) slices[q] = (int)S[q];
}

// One warp per local (token, rank) entry: its local expert-sorted slot (for
// the combine), its global slot, and a float4 copy of the token row into the
// slice owner's receive buffer with the return address beside it.
__global__ void __launch_bounds__(256)
ep_gather_kernel(const float *__restrict__ x, int T, int d, int d_pad, int k, int E, int rank,
                 int G, int max_rows, const int *__restrict__ ids, const int *__restrict__ loc,
                 const int *__restrict__ tile_pref, const int *__restrict__ plan_local,
                 const int *__restrict__ base_r, const int *__restrict__ slices,
                 float *const *__restrict__ recv_ptrs, int2 *const *__restrict__ ret_ptrs,
                 int *__restrict__ pos_of, int round_to_tf32, DeviceStatus *status)
{
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp < T * k) {
        const int t = warp / k;
        const int e = ids[warp];
        const int lr = tile_pref[(size_t)(t / kRouterTile) * E + e] + loc[warp];
        const int pos_local = plan_local[E + e] + lr;
        const int gp = base_r[e] + lr;
        int lo = 0, hi = G - 1;                 // slice q with slices[q] <= gp < slices[q+1]
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (slices[mid] <= gp) lo = mid; else hi = mid - 1;
        }
        const int q = lo, p = gp - slices[q];
        if (e < 0 || e >= E || q < 0 || q >= G || p < 0 || p >= max_rows || pos_local < 0 ||
            pos_local >= T * k) {
            if (lane == 0) atomicExch(&status->bad_index, 1);
        } else {
            if (lane == 0) {
                pos_of[warp] = pos_local;
                ret_ptrs[q][p] = make_int2(rank, pos_local);
            }
            const float *src = x + (size_t)t * d;
            float *dst = recv_ptrs[q] + (size_t)p * d_pad;
            if ((d & 3) == 0) {
                const float4 *s4 = reinterpret_cast<const float4 *>(src);
                float4 *d4 = reinterpret_cast<float4 *>(dst);
                for (int c = lane; c < (d_pad >> 2); c += 32) {
                    float4 v = (c < (d >> 2)) ? __ldg(s4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                    if (round_to_tf32) {
                        v.x = round_tf32(v.x); v.y = round_tf32(v.y);
                        v.z = round_tf32(v.z); v.w = round_tf32(v.w);
                    }
                    d4[c] = v;
                }
            } else {
                for (int c = lane; c < d_pad; c += 32) {
                    const float v = (c < d) ? __ldg(src + c) : 0.0f;
                    dst[c] = round_to_tf32 ? round_tf32(v) : v;
                }
            }
        }
    }
    __threadfence_system();   // peer stores visible before the barrier that follows
}

// ---------------------------------------------------------------------
// state
// ---------------------------------------------------------------------
struct moe_b200_ep {
    int rank = 0, world = 1, device = 0, max_T = 0, max_rows = 0, recv_rows = 0;
    const moe_b200_weights *w = nullptr;
    ncclComm_t comm = nullptr;
    cudaStream_t stream = nullptr;      // library stream for the host-buffer entry
    DeviceStatus *status = nullptr;
    // IPC-shared buffers (this rank's) and the peer tables
    float *recv_x = nullptr;            // [recv_rows × d_pad]
    int2 *ret = nullptr;                // [recv_rows]
    float *y = nullptr;                 // [max_rows × d_pad] written by slice owners
    float **d_recv_ptrs = nullptr, **d_y_ptrs = nullptr;
    int2 **d_ret_ptrs = nullptr;
    std::vector<void *> opened;         // peer mappings to close
    // local work buffers
    float *h = nullptr;                 // [recv_rows × F_pad]
    float *xs = nullptr, *hs = nullptr; // 3xTF32 small parts of recv_x and h
    float *rpart = nullptr;             // split-K router partial logits (small T)
    int rsplit = 1;
    float *probs = nullptr, *wts = nullptr;
    int *ids = nullptr, *loc = nullptr, *tile_cnt = nullptr, *tile_pref = nullptr;
    int *plan_local = nullptr, *plan_q = nullptr, *pos_of = nullptr;
    int *counts_all = nullptr, *base_r = nullptr, *slices = nullptr, *bar = nullptr;
    float *io_x = nullptr, *io_out = nullptr, *io_bias = nullptr;
    TcGemm up{}, dn{};
    DecMaps dup{}, ddn{};
};

namespace {

int ep_fail(int code, const char *fmt, const char *a = "", const char *b = "") {
    char msg[300];
    std::snprintf(msg, sizeof msg, fmt, a, b);
    return set_last_error(code, msg);
}

#define EP_CK(call)                                                                         \
    do {                                                                                    \
        cudaError_t _e = (call);                                                            \
        if (_e != cudaSuccess)                                                              \
            return ep_fail(_e == cudaErrorMemoryAllocation ? MOE_B200_E_NOMEM : MOE_B200_E_CUDA, \
                           "%s: %s", #call, cudaGetErrorString(_e));                        \
    } while (0)

#define EP_NC(call)                                                                         \
    do {                                                                                    \
        ncclResult_t _r = (call);                                                           \
        if (_r != ncclSuccess)                                                              \
            return ep_fail(MOE_B200_E_NCCL, "%s: %s", #call, nccl().GetErrorString(_r));       \
    } while (0)

// encode a 2-D fp32 tensor map (same layout as the single-GPU path)
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int ep_tmap(CUtensorMap *m, const float *ptr, int64_t rows, int64_t cols, int box_rows) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess || q != cudaDriverEntryPointSuccess)
        return ep_fail(MOE_B200_E_CUDA, "cuTensorMapEncodeTiled unavailable%s%s");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
    cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = reinterpret_cast<EncodeTiledFn>(p)(
        m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(ptr), dims, strides, box, estr,
        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return ep_fail(MOE_B200_E_CUDA, "cuTensorMapEncodeTiled failed%s%s");
    return MOE_B200_OK;
}

void ep_release(moe_b200_ep *ep) {
    if (!ep) return;
    cudaSetDevice(ep->device);
    cudaDeviceSynchronize();
    for (void *p : ep->opened) cudaIpcCloseMemHandle(p);
    if (ep->comm) nccl().CommDestroy(ep->comm);
    void *bufs[] = {ep->recv_x, ep->ret, ep->y, ep->d_recv_ptrs, ep->d_y_ptrs, ep->d_ret_ptrs,
                    ep->h, ep->xs, ep->hs, ep->rpart, ep->probs, ep->wts, ep->ids, ep->loc, ep->tile_cnt, ep->tile_pref,
                    ep->plan_local, ep->plan_q, ep->pos_of, ep->counts_all, ep->base_r,
                    ep->slices, ep->bar, ep->io_x, ep->io_out, ep->io_bias, ep->status};
    for (void *b : bufs)
        if (b) cudaFree(b);
    if (ep->stream) cudaStreamDestroy(ep->stream);
    delete ep;
}

}  // namespace

// ---------------------------------------------------------------------
// C-ABI
// ---------------------------------------------------------------------
extern "C" int moe_b200_ep_unique_id(void *id_out) {
    if (!id_out) return ep_fail(MOE_B200_E_INVALID, "null id buffer%s%s");
    static_assert(sizeof(ncclUniqueId) <= MOE_B200_EP_ID_BYTES, "NCCL id does not fit");
    if (!nccl().ok) return ep_fail(MOE_B200_E_NCCL, "libnccl.so.2 not found%s%s");
    ncclUniqueId id;
    EP_NC(nccl().GetUniqueId(&id));
    std::memset(id_out, 0, MOE_B200_EP_ID_BYTES);
    std::memcpy(id_out, &id, sizeof id);
    return MOE_B200_OK;
}

extern "C" int moe_b200_ep_partition(const int *counts_all, int world, int E, int rank,
                                     long long capacity, int *cnt_rank, int *base_rank,
                                     long long *slice_start, long long *slice_rows) {
    if (!counts_all || world < 1 || world > 64 || E < 1 || rank < 0 || rank >= world)
        return ep_fail(MOE_B200_E_INVALID, "bad partition arguments%s%s");
    long long S[65];
    ep_partition(counts_all, world, E, rank, capacity, cnt_rank, base_rank, S);
    if (slice_start) *slice_start = S[rank];
    if (slice_rows) *slice_rows = S[rank + 1] - S[rank];
    return MOE_B200_OK;
}

extern "C" int moe_b200_ep_create(const void *unique_id, int rank, int world,
                                  int max_tokens_per_rank, const moe_b200_weights *w,
                                  moe_b200_ep **out) {
    if (!unique_id || !w || !out || world < 1 || world > 64 || rank < 0 || rank >= world ||
        max_tokens_per_rank < 1)
        return ep_fail(MOE_B200_E_INVALID, "bad arguments to moe_b200_ep_create%s%s");
    if ((int64_t)max_tokens_per_rank * w->k > (int64_t)1 << 30)
        return ep_fail(MOE_B200_E_INVALID, "max_tokens_per_rank too large%s%s");
    if (!nccl().ok) return ep_fail(MOE_B200_E_NCCL, "libnccl.so.2 not found%s%s");
    EP_CK(cudaSetDevice(w->device));
    if (device_sms(w->device) == 0) return ep_fail(MOE_B200_E_NODEV, "device unusable%s%s");
    moe_b200_ep *ep = new moe_b200_ep();
    ep->rank = rank;
    ep->world = world;
    ep->device = w->device;
    ep->w = w;
    ep->max_T = max_tokens_per_rank;
    ep->max_rows = max_tokens_per_rank * w->k;
    // cost-balanced slices may hold more rows than T·k: 25% headroom, beyond
    // which the partition falls back to equal rows
    ep->recv_rows = ep->max_rows + ep->max_rows / 4 + 256;
    int rc = MOE_B200_OK;
#define TRY(x)                      \
    do {                            \
        if ((rc = (x))) {           \
            ep_release(ep);         \
            return rc;              \
        }                           \
    } while (0)
    auto alloc = [&](void **p, size_t bytes) -> int {
        cudaError_t e = cudaMalloc(p, bytes);
        if (e != cudaSuccess)
            return ep_fail(MOE_B200_E_NOMEM, "expert-parallel buffers: %s%s", cudaGetErrorString(e));
        return MOE_B200_OK;
    };
    const size_t R = ep->max_rows, RR = ep->recv_rows, T = ep->max_T, E = w->E, G = world;
    const size_t tiles = ceil_div<size_t>(T, kRouterTile);
    TRY(alloc((void **)&ep->recv_x, RR * w->d_pad * 4));
    TRY(alloc((void **)&ep->ret, RR * sizeof(int2)));
    TRY(alloc((void **)&ep->y, R * w->d_pad * 4));
    TRY(alloc((void **)&ep->h, RR * w->F_pad * 4));
    TRY(alloc((void **)&ep->xs, RR * w->d_pad * 4));
    ep->rsplit = router_splits((int)T, w->d);
    if (ep->rsplit > 1) TRY(alloc((void **)&ep->rpart, (size_t)ep->rsplit * T * E * 4));
    TRY(alloc((void **)&ep->hs, RR * w->F_pad * 4));
    TRY(alloc((void **)&ep->probs, T * E * 4));
    TRY(alloc((void **)&ep->wts, R * 4));
    TRY(alloc((void **)&ep->ids, R * 4));
    TRY(alloc((void **)&ep->loc, R * 4));
    TRY(alloc((void **)&ep->pos_of, R * 4));
    TRY(alloc((void **)&ep->tile_cnt, tiles * E * 4));
    TRY(alloc((void **)&ep->tile_pref, tiles * E * 4));
    TRY(alloc((void **)&ep->plan_local, plan_ints(E) * 4));
    TRY(alloc((void **)&ep->plan_q, plan_ints(E) * 4));
    TRY(alloc((void **)&ep->counts_all, G * E * 4));
    TRY(alloc((void **)&ep->base_r, E * 4));
    TRY(alloc((void **)&ep->slices, (G + 1) * 4));
    TRY(alloc((void **)&ep->bar, 4));
    TRY(alloc((void **)&ep->io_x, T * w->d * 4));
    TRY(alloc((void **)&ep->io_out, T * w->d * 4));
    TRY(alloc((void **)&ep->io_bias, E * 4));
    TRY(alloc((void **)&ep->status, sizeof(DeviceStatus)));
    TRY(alloc((void **)&ep->d_recv_ptrs, G * sizeof(float *)));
    TRY(alloc((void **)&ep->d_y_ptrs, G * sizeof(float *)));
    TRY(alloc((void **)&ep->d_ret_ptrs, G * sizeof(int2 *)));
    if (cudaMemset(ep->status, 0, sizeof(DeviceStatus)) != cudaSuccess ||
        cudaMemset(ep->bar, 0, 4) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ep->stream, cudaStreamNonBlocking) != cudaSuccess)
        TRY(ep_fail(MOE_B200_E_CUDA, "expert-parallel set-up failed%s%s"));
    TRY(ep_tmap(&ep->up.tmA, ep->recv_x, RR, w->d_pad, 128));
    ep->up.tmB = w->tm_ug;
    TRY(ep_tmap(&ep->dn.tmA, ep->h, RR, w->F_pad, 128));
    ep->dn.tmB = w->tm_dn;
    ep->dup.tmW = w->tm_ug64;
    TRY(ep_tmap(&ep->dup.tmXb, ep->recv_x, RR, w->d_pad, 64));
    TRY(ep_tmap(&ep->dup.tmXs, ep->xs, RR, w->d_pad, 64));
    ep->dup.tmXb32 = ep->dup.tmXb;       // CTA-pair map, unused by the single-CTA kernels
    ep->ddn.tmW = w->tm_dn128;
    TRY(ep_tmap(&ep->ddn.tmXb, ep->h, RR, w->F_pad, 64));
    TRY(ep_tmap(&ep->ddn.tmXs, ep->hs, RR, w->F_pad, 64));
    ep->ddn.tmXb32 = ep->ddn.tmXb;

    // communicator
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof id);
    {
        ncclResult_t r = nccl().CommInitRank(&ep->comm, world, id, rank);
        if (r != ncclSuccess) {
            ep->comm = nullptr;
            TRY(ep_fail(MOE_B200_E_NCCL, "ncclCommInitRank: %s%s", nccl().GetErrorString(r)));
        }
    }
    // exchange IPC handles of the three shared buffers (NCCL all-gather)
    std::vector<float *> recv_ptrs(G), y_ptrs(G);
    std::vector<int2 *> ret_ptrs(G);
    recv_ptrs[rank] = ep->recv_x;
    y_ptrs[rank] = ep->y;
    ret_ptrs[rank] = ep->ret;
    if (world > 1) {
        // three IPC handles and this rank's max_tokens_per_rank (every rank
        // must use the same capacity, or their partitions would differ)
        constexpr size_t HB = 3 * sizeof(cudaIpcMemHandle_t) + 64;
        struct {
            cudaIpcMemHandle_t h[3];
            long long max_t;
            char pad[56];
        } mine_blob;
        static_assert(sizeof(mine_blob) == HB, "handle blob layout");
        std::memset(&mine_blob, 0, sizeof mine_blob);
        mine_blob.max_t = max_tokens_per_rank;
        cudaIpcMemHandle_t *mine = mine_blob.h;
        if (cudaIpcGetMemHandle(&mine[0], ep->recv_x) != cudaSuccess ||
            cudaIpcGetMemHandle(&mine[1], ep->ret) != cudaSuccess ||
            cudaIpcGetMemHandle(&mine[2], ep->y) != cudaSuccess)
            TRY(ep_fail(MOE_B200_E_CUDA, "cudaIpcGetMemHandle failed%s%s"));
        unsigned char *dh = nullptr;
        TRY(alloc((void **)&dh, HB * G));
        std::vector<unsigned char> all(HB * G);
        int step = MOE_B200_OK;
        if (cudaMemcpy(dh + HB * rank, &mine_blob, HB, cudaMemcpyHostToDevice) != cudaSuccess)
            step = ep_fail(MOE_B200_E_CUDA, "handle upload failed%s%s");
        if (!step) {
            ncclResult_t r = nccl().AllGather(dh + HB * rank, dh, HB, ncclChar, ep->comm, ep->stream);
            if (r != ncclSuccess)
                step = ep_fail(MOE_B200_E_NCCL, "nccl().AllGather(handles): %s%s", nccl().GetErrorString(r));
        }
        if (!step && (cudaStreamSynchronize(ep->stream) != cudaSuccess ||
                      cudaMemcpy(all.data(), dh, HB * G, cudaMemcpyDeviceToHost) != cudaSuccess))
            step = ep_fail(MOE_B200_E_CUDA, "handle exchange failed%s%s");
        cudaFree(dh);
        TRY(step);
        for (int q = 0; q < world; q++) {
            long long their_t = 0;
            std::memcpy(&their_t, all.data() + HB * q + 3 * sizeof(cudaIpcMemHandle_t), 8);
            if (their_t != max_tokens_per_rank)
                TRY(ep_fail(MOE_B200_E_INVALID,
                            "max_tokens_per_rank differs between ranks%s%s"));
        }
        for (int q = 0; q < world; q++) {
            if (q == rank) continue;
            cudaIpcMemHandle_t hq[3];
            std::memcpy(hq, all.data() + HB * q, 3 * sizeof(cudaIpcMemHandle_t));
            void *p[3] = {nullptr, nullptr, nullptr};
            for (int i = 0; i < 3; i++) {
                cudaError_t e = cudaIpcOpenMemHandle(&p[i], hq[i], cudaIpcMemLazyEnablePeerAccess);
                if (e != cudaSuccess)
                    TRY(ep_fail(MOE_B200_E_CUDA, "cudaIpcOpenMemHandle: %s%s", cudaGetErrorString(e)));
                ep->opened.push_back(p[i]);
            }
            recv_ptrs[q] = (float *)p[0];
            ret_ptrs[q] = (int2 *)p[1];
            y_ptrs[q] = (float *)p[2];
        }
    }
    if (cudaMemcpy(ep->d_recv_ptrs, recv_ptrs.data(), G * sizeof(float *), cudaMemcpyHostToDevice) ||
        cudaMemcpy(ep->d_y_ptrs, y_ptrs.data(), G * sizeof(float *), cudaMemcpyHostToDevice) ||
        cudaMemcpy(ep->d_ret_ptrs, ret_ptrs.data(), G * sizeof(int2 *), cudaMemcpyHostToDevice))
        TRY(ep_fail(MOE_B200_E_CUDA, "peer table upload failed%s%s"));
#undef TRY
    *out = ep;
    return MOE_B200_OK;
}

extern "C" int moe_b200_ep_destroy(moe_b200_ep *ep) {
    ep_release(ep);
    return MOE_B200_OK;
}

extern "C" int moe_b200_ep_forward_device(moe_b200_ep *ep, const float *d_bias, const float *d_x,
                                          int T, float *d_out, float *d_router_probs,
                                          int *d_expert_ids, const moe_b200_opts *opts,
                                          void *stream) {
    if (!ep || !d_x || !d_out) return ep_fail(MOE_B200_E_INVALID, "null argument%s%s");
    if (((uintptr_t)d_x | (uintptr_t)d_out) & 15)
        return ep_fail(MOE_B200_E_INVALID, "x and out must be 16-byte aligned%s%s");
    if (T < 0 || T > ep->max_T)
        return ep_fail(MOE_B200_E_INVALID, "T outside [0, max_tokens_per_rank]%s%s");
    const moe_b200_weights *w = ep->w;
    EP_CK(cudaSetDevice(ep->device));
    ncclResult_t async_err = ncclSuccess;
    EP_NC(nccl().CommGetAsyncError(ep->comm, &async_err));
    if (async_err != ncclSuccess)
        return ep_fail(MOE_B200_E_NCCL, "communicator error: %s%s", nccl().GetErrorString(async_err));
    cudaStream_t s = stream ? (cudaStream_t)stream : ep->stream;
    const int E = w->E, k = w->k, G = ep->world;
    float *probs = d_router_probs ? d_router_probs : ep->probs;
    int *ids = d_expert_ids ? d_expert_ids : ep->ids;
    int path = opts ? opts->path : MOE_B200_PATH_AUTO;
    if (path == MOE_B200_PATH_AUTO)
        path = ((double)T * G * k / E >= 64.0) ? MOE_B200_PATH_TF32 : MOE_B200_PATH_TF32X3;
    cudaEvent_t *ev = profile_events(ep->device);
#define MARK(i) \
    if (ev) EP_CK(cudaEventRecord(ev[i], s))

    MARK(0);
    if (T > 0) {
        // the split-K router only when its buffer (sized for max_tokens) covers T
        const int ns = router_splits(T, w->d);
        const bool split = ns > 1 && ns <= ep->rsplit && ep->rpart != nullptr;
        EP_CK(launch_router(d_x, T, w->d, w->router, d_bias, E, k, probs, ids, ep->wts, ep->loc,
                            ep->tile_cnt, s, split ? ep->rpart : nullptr, split ? ns : 1));
        EP_CK(launch_dispatch_scan(ep->tile_cnt, T, E, ep->tile_pref, ep->plan_local, s));
    } else {
        EP_CK(cudaMemsetAsync(ep->plan_local, 0, E * sizeof(int), s));
    }
    MARK(1);
    EP_NC(nccl().AllGather(ep->plan_local, ep->counts_all, E, ncclInt32, ep->comm, s));
    ep_plan_kernel<<<1, 32, 0, s>>>(ep->counts_all, G, E, ep->rank, ep->recv_rows, ep->plan_q,
                                    ep->base_r, ep->slices);
    EP_CK(cudaGetLastError());
    if (T > 0) {
        ep_gather_kernel<<<ceil_div(T * k, 8), 256, 0, s>>>(
            d_x, T, w->d, w->d_pad, k, E, ep->rank, G, ep->recv_rows, ids, ep->loc,
            ep->tile_pref, ep->plan_local, ep->base_r, ep->slices, ep->d_recv_ptrs,
            ep->d_ret_ptrs, ep->pos_of, path == MOE_B200_PATH_TF32, ep->status);
        EP_CK(cudaGetLastError());
    }
    EP_NC(nccl().AllReduce(ep->bar, ep->bar, 1, ncclInt32, ncclSum, ep->comm, s));
    MARK(2);
    const int rows = ep->recv_rows;
    // TF32 on decode-sized groups (the single-GPU rule, on the whole job's
    // rows per expert): the weight-streaming kernel's one-pass TF32 mode.
    // The down GEMM does not split K here (its rows go straight to their
    // owners), unlike the single-GPU call, so the two agree to the TF32
    // tolerance rather than bit for bit on this path.
    const bool onepass = path == MOE_B200_PATH_TF32 && (double)T * G * k / E < 64.0;
    if (path == MOE_B200_PATH_TF32 && !onepass) {
        const int sms = device_sms(ep->device);
        EP_CK(launch_tc_upgate(ep->up, w->d_pad, w->F_pad, ep->h, ep->plan_q, E, rows, sms,
                               ep->status, s));
        MARK(3);
        EP_CK(launch_tc_down(ep->dn, w->F_pad, w->d_pad, w->down_bn, ep->y, ep->plan_q, E, rows,
                             sms, ep->status, s, ep->d_y_ptrs, ep->ret));
    } else if (path == MOE_B200_PATH_TF32X3 || onepass) {
        const int sms = device_sms(ep->device);
        if (!onepass) EP_CK(launch_split_tf32(ep->recv_x, ep->xs, (size_t)rows * w->d_pad, s));
        EP_CK(launch_dec_upgate(ep->dup, w->d_pad, w->F_pad, ep->h, ep->hs, ep->plan_q, E, rows,
                                sms, 0, ep->status, s, onepass));
        MARK(3);
        EP_CK(launch_dec_down(ep->ddn, w->F_pad, w->d_pad, ep->y, ep->plan_q, E, rows, sms, 0,
                              ep->status, s, ep->d_y_ptrs, ep->ret, nullptr, onepass));
    } else {
        EP_CK(launch_ffma_upgate(ep->recv_x, w->d_pad, w->ug, w->F_pad, ep->h, ep->plan_q, E, rows,
                                 s));
        MARK(3);
        EP_CK(launch_ffma_down(ep->h, w->F_pad, w->dn, w->d_pad, ep->y, ep->plan_q, E, rows, s,
                               ep->d_y_ptrs, ep->ret));
    }
    MARK(4);   // the wait for the other ranks counts under the combine stage
    EP_NC(nccl().AllReduce(ep->bar, ep->bar, 1, ncclInt32, ncclSum, ep->comm, s));
    if (T > 0) EP_CK(launch_combine(ep->y, w->d, w->d_pad, T, k, ep->pos_of, ep->wts, d_out, s));
    MARK(5);
#undef MARK
    note_forward(ep->device, E,
                 T > 0 ? 7 + (path == MOE_B200_PATH_TF32X3) + (router_splits(T, w->d) > 1) : 3,
                 path);
    return MOE_B200_OK;
}

extern "C" int moe_b200_ep_forward(moe_b200_ep *ep, const float *router_bias, const float *x,
                                   int T, float *out, float *router_probs, int *expert_ids,
                                   const moe_b200_opts *opts) {
    if (!ep || (T > 0 && (!x || !out))) return ep_fail(MOE_B200_E_INVALID, "null argument%s%s");
    if (T < 0 || T > ep->max_T)
        return ep_fail(MOE_B200_E_INVALID, "T outside [0, max_tokens_per_rank]%s%s");
    const moe_b200_weights *w = ep->w;
    EP_CK(cudaSetDevice(ep->device));
    cudaStream_t s = ep->stream;
    const size_t xb = (size_t)T * w->d * 4;
    if (T > 0) EP_CK(cudaMemcpyAsync(ep->io_x, x, xb, cudaMemcpyHostToDevice, s));
    const float *d_bias = nullptr;
    if (router_bias) {
        EP_CK(cudaMemcpyAsync(ep->io_bias, router_bias, (size_t)w->E * 4, cudaMemcpyHostToDevice, s));
        d_bias = ep->io_bias;
    }
    int rc = moe_b200_ep_forward_device(ep, d_bias, ep->io_x, T, ep->io_out, ep->probs, ep->ids,
                                        opts, s);
    if (rc) return rc;
    if (T > 0) {
        EP_CK(cudaMemcpyAsync(out, ep->io_out, xb, cudaMemcpyDeviceToHost, s));
        if (router_probs)
            EP_CK(cudaMemcpyAsync(router_probs, ep->probs, (size_t)T * w->E * 4,
                                  cudaMemcpyDeviceToHost, s));
        if (expert_ids)
            EP_CK(cudaMemcpyAsync(expert_ids, ep->ids, (size_t)T * w->k * 4,
                                  cudaMemcpyDeviceToHost, s));
    }
    EP_CK(cudaStreamSynchronize(s));
    DeviceStatus st;
    EP_CK(cudaMemcpy(&st, ep->status, sizeof st, cudaMemcpyDeviceToHost));
    if (st.bad_index || st.timeout) {
        EP_CK(cudaMemset(ep->status, 0, sizeof st));
        return st.timeout ? ep_fail(MOE_B200_E_TIMEOUT, "device wait timed out%s%s")
                          : ep_fail(MOE_B200_E_CUDA, "device bounds check rejected an index%s%s");
    }
    return MOE_B200_OK;
}

extern "C" int moe_b200_ep_counts(moe_b200_ep *ep, int *counts_all, int *slice_rows) {
    if (!ep) return ep_fail(MOE_B200_E_INVALID, "null ep%s%s");
    EP_CK(cudaSetDevice(ep->device));
    EP_CK(cudaDeviceSynchronize());
    if (counts_all)
        EP_CK(cudaMemcpy(counts_all, ep->counts_all, (size_t)ep->world * ep->w->E * 4,
                         cudaMemcpyDeviceToHost));
    if (slice_rows)
        EP_CK(cudaMemcpy(slice_rows, ep->plan_q + 2 * ep->w->E, sizeof(int),
                         cudaMemcpyDeviceToHost));   // off[E] == rows of this slice
    return MOE_B200_OK;
}
