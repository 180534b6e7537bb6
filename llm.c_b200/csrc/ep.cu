// ep.cu — expert-parallel MoE forward over NVLink (one process per GPU).
//
// Experts are sharded: each rank holds a shard of the expert set (for c5,
// 8 of 64 experts per GPU at 8 GPUs) in n_slots packed slots, the first of
// them its base experts, the rest spares.  Under skewed popularity (c5's
// Zipf(1.1) sends ~30 % of all rows to one expert) no static sharding can
// balance the work, so moe_b200_ep_rebalance places replicas of hot experts
// in spare slots, load-aware, from the per-expert counts of the last forward
// (every rank computes the same placement), and copies their weights from
// the base holder's memory over NVLink.  Every forward then splits each
// replicated expert's rows among its holders so the estimated GEMM cost per
// rank is as even as the placement allows.  Every rank routes its own
// tokens (the router covers all experts).
//
// Row order.  The rows of expert e, over all source ranks, are numbered in
// the global order (source rank, then the source's stable local order).
// Holder i of e (holders in ascending rank order) receives the contiguous
// range [beg_e[i], beg_e[i+1]) of that order, so
//   * the rows a source sends to one holder of e are one contiguous run of
//     its local expert-sorted order;
//   * a holder's receive buffer is grouped by slot with the same plan format
//     (cnt | off | mt128 | mt64 | mt256 over slots) the single-GPU grouped
//     GEMMs read, with the shard's packed slots as their weights.
//
// Data movement is fused into the kernels; NCCL carries no rows.  The
// dispatch gather stores each token row straight into the holder's receive
// buffer (CUDA IPC peer mapping, NVLink stores), with a return address
// (source rank, source row).  The down GEMM's epilogue stores each result
// row straight back into the token owner's output buffer.  NCCL carries the
// per-expert counts (E ints per rank) and two stream-ordered barriers, so a
// forward never waits on the host.  No TMA ever reads peer memory; the
// replica copy of the rebalance is a plain-load kernel.
//
// Stream order per forward on rank r (every rank issues the same NCCL
// calls in the same order):
//   router -> scan -> allgather(counts) -> plan -> gather(peer stores)
//   -> barrier -> up/gate -> down(peer stores) -> barrier -> combine
#include "../../include/moe_b200.h"
#include "kernels.cuh"
#include "weights.cuh"

#include "nccl_dyn.cuh"

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

using namespace moe;

namespace {
constexpr int kMaxWorld = 64;
constexpr int kTileRows = 128;

// Estimated GEMM cost of an expert segment of t 128-row m-tiles on one
// rank, in half-m-tiles of tensor-core time: 2 per m-tile, but at least 2
// m-tiles' worth, plus 2.  A segment streams the expert's weights at least
// once, and on B200 that takes ~1.6 m-tiles of TF32 tensor time whatever
// the shape (3·d·F·4 bytes at the HBM rate against 128 rows · 6·d·F flops
// at the TF32 rate); a 2-GPU c5 run measured a segment of one partial tile
// at ~3.3 m-tiles, so the floor is 2 m-tiles and the constant 2 more.
__host__ __device__ inline long long seg_cost_tiles(long long t) {
    return t > 0 ? 2 * (t > 2 ? t : 2) + 2 : 0;
}
__host__ __device__ inline long long seg_cost(long long n) {
    return seg_cost_tiles((n + kTileRows - 1) / kTileRows);
}
}  // namespace

// ---------------------------------------------------------------------
// The split of every expert's rows among its holders (host copy: tests,
// placement; device copy: every forward).  Integer arithmetic only, so
// every rank and the host derive the same result.
//
//   C[q*ldc + e]    rows of expert e on source rank q (all-gathered counts)
//   place[q*E + e]  slot of expert e on rank q, or -1
// Outputs (caller arrays):
//   nh[e]                 number of holders of e
//   hold[e*G + i]         rank of holder i (ascending)
//   beg[e*(G+1) + i]      first row (in e's global order) of holder i;
//                         beg[e*(G+1) + nh[e]] = rows of e
//   dst[e*G + i]          offset of that range in holder i's receive buffer
//   rows_q[q], load[q]    receive rows and estimated cost per rank (or null)
// Single-holder experts go whole to their holder.  Replicated experts, the
// most rows first, are cut into 128-row tiles, each given to the holder
// whose cost after taking it (seg_cost_tiles of its new tile count) is
// lowest (ties: lower rank), then every holder takes its count of tiles as
// one contiguous range in holder order.
// Returns 1 if an expert with rows has no holder, else 0.
// ---------------------------------------------------------------------
__host__ __device__ inline int ep_split(const int *C, int ldc, int G, int E, const int *place,
                                        int S, int *nh, int *hold, int *beg, int *dst,
                                        long long *rows_q, long long *load_out) {
    int tot[kMaxExperts];
    long long load[kMaxWorld];
    int tiles_of[kMaxWorld];
    int bad = 0;
    for (int q = 0; q < G; q++) load[q] = 0;
    for (int e = 0; e < E; e++) {
        int t = 0, n = 0;
        for (int q = 0; q < G; q++) {
            t += C[q * ldc + e];
            if (place[q * E + e] >= 0) hold[e * G + n++] = q;
        }
        tot[e] = t;
        nh[e] = n;
        for (int i = 0; i <= G; i++) beg[e * (G + 1) + i] = t;
        beg[e * (G + 1)] = 0;
        if (n == 0 && t > 0) bad = 1;
        if (n == 1) load[hold[e * G]] += seg_cost(t);
    }
    // replicated experts, the most rows first (ties: lower expert id)
    unsigned char done[kMaxExperts];
    for (int e = 0; e < E; e++) done[e] = (unsigned char)(nh[e] <= 1);
    while (true) {
        int e = -1;
        for (int c = 0; c < E; c++)
            if (!done[c] && (e < 0 || tot[c] > tot[e])) e = c;
        if (e < 0) break;
        done[e] = 1;
        const int n = nh[e];
        for (int i = 0; i < n; i++) tiles_of[i] = 0;
        const int tiles = (tot[e] + kTileRows - 1) / kTileRows;
        for (int t = 0; t < tiles; t++) {
            int best = 0;
            long long best_c = 0;
            for (int i = 0; i < n; i++) {
                const long long c = load[hold[e * G + i]] + seg_cost_tiles(tiles_of[i] + 1) -
                                    seg_cost_tiles(tiles_of[i]);
                if (i == 0 || c < best_c) { best = i; best_c = c; }
            }
            load[hold[e * G + best]] = best_c;
            tiles_of[best]++;
        }
        int b = 0;
        for (int i = 0; i < n; i++) {
            beg[e * (G + 1) + i] = b;
            const long long nb = (long long)b + (long long)kTileRows * tiles_of[i];
            b = nb < tot[e] ? (int)nb : tot[e];
        }
        for (int i = n; i <= G; i++) beg[e * (G + 1) + i] = tot[e];
    }
    // receive layout of every rank: its slots in slot order
    int slot_rows[kMaxExperts];
    for (int q = 0; q < G; q++) {
        for (int j = 0; j < S; j++) slot_rows[j] = 0;
        for (int e = 0; e < E; e++) {
            const int j = place[q * E + e];
            if (j < 0) continue;
            int i = 0;
            while (hold[e * G + i] != q) i++;
            slot_rows[j] = beg[e * (G + 1) + i + 1] - beg[e * (G + 1) + i];
        }
        long long off = 0;
        for (int j = 0; j < S; j++) {
            const long long r = slot_rows[j];
            slot_rows[j] = (int)off;            // now the slot's offset
            off += r;
        }
        if (rows_q) rows_q[q] = off;
        for (int e = 0; e < E; e++) {
            const int j = place[q * E + e];
            if (j < 0) continue;
            int i = 0;
            while (hold[e * G + i] != q) i++;
            dst[e * G + i] = slot_rows[j];
        }
    }
    if (load_out)
        for (int q = 0; q < G; q++) load_out[q] = load[q];
    return bad;
}

// Load-aware placement (host): starting from every rank's base experts,
// add replicas in spare slots while that lowers the highest estimated rank
// cost under ep_split: take the most loaded rank, its experts by the rows it
// carries of them, and place a replica on the least loaded rank with a free
// slot that does not hold the expert yet; keep the first such move that
// lowers the maximum.  Deterministic.
static void ep_place_greedy(const int *C, int G, int E, int S, const int *base, int *place) {
    std::memcpy(place, base, sizeof(int) * (size_t)G * E);
    std::vector<int> nh(E), hold((size_t)E * G), beg((size_t)E * (G + 1)), dst((size_t)E * G);
    std::vector<long long> load(G);
    auto eval = [&]() -> long long {
        ep_split(C, E, G, E, place, S, nh.data(), hold.data(), beg.data(), dst.data(), nullptr,
                 load.data());
        return *std::max_element(load.begin(), load.end());
    };
    auto free_slot = [&](int q) -> int {
        std::vector<char> used(S, 0);
        for (int e = 0; e < E; e++)
            if (place[q * E + e] >= 0) used[place[q * E + e]] = 1;
        for (int j = 0; j < S; j++)
            if (!used[j]) return j;
        return -1;
    };
    long long cur = eval();
    for (int iter = 0; iter < G * S; iter++) {
        const std::vector<long long> ld = load;
        int hot = 0;
        for (int q = 1; q < G; q++)
            if (ld[q] > ld[hot]) hot = q;
        // the hot rank's experts by the rows it carries of them
        std::vector<std::pair<int, int>> cand;
        for (int e = 0; e < E; e++) {
            if (place[hot * E + e] < 0) continue;
            int i = 0;
            while (hold[(size_t)e * G + i] != hot) i++;
            const int rows = beg[(size_t)e * (G + 1) + i + 1] - beg[(size_t)e * (G + 1) + i];
            if (rows > 0) cand.push_back({-rows, e});
        }
        std::sort(cand.begin(), cand.end());
        std::vector<int> targets(G);
        for (int q = 0; q < G; q++) targets[q] = q;
        std::stable_sort(targets.begin(), targets.end(),
                         [&](int a, int b) { return ld[a] < ld[b]; });
        bool moved = false;
        for (const auto &ce : cand) {
            const int e = ce.second;
            for (int q : targets) {
                if (q == hot || place[q * E + e] >= 0) continue;
                const int j = free_slot(q);
                if (j < 0) continue;
                place[q * E + e] = j;
                const long long m = eval();
                if (m < cur) {
                    cur = m;
                    moved = true;
                    break;
                }
                place[q * E + e] = -1;
            }
            if (moved) break;
        }
        if (!moved) break;
        eval();                       // refresh hold/beg/load for the next pass
    }
}

// One thread: the split, this rank's receive plan over its S slots
// (cnt | off | mt128 | mt64 | mt256), and the global position of this rank's
// first row of every expert.
//
// Every rank's all-gathered record is {generation, counts[E]}; each forward
// advances this rank's generation (stamp[0]) once.  If any record carries
// another generation than this rank's, the exchange did not happen (a rank
// stopped joining and the communicator was aborted, leaving the previous
// step's records): the kernel then flags it, marks the step `dead`, and
// gives this rank an empty plan and empty splits, so that no kernel of the
// step stores into another rank's memory.
__global__ void ep_plan_kernel(const int *__restrict__ recs, int G, int E, int S, int rank,
                               const int *__restrict__ place, int *__restrict__ stamp,
                               int *__restrict__ plan, int *__restrict__ base_r,
                               int *__restrict__ nh, int *__restrict__ hold,
                               int *__restrict__ beg, int *__restrict__ dst,
                               int *__restrict__ dead, DeviceStatus *status)
{
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const int gen = stamp[0];
    bool ok = true;
    for (int q = 0; q < G; q++) ok = ok && recs[q * (E + 1)] == gen;
    stamp[0] = gen + 1;
    *dead = ok ? 0 : 1;
    if (!ok) atomicExch(&status->bad_index, 2);
    if (!ok || ep_split(recs + 1, E + 1, G, E, place, S, nh, hold, beg, dst, nullptr, nullptr)) {
        if (ok) atomicExch(&status->bad_index, 1);
        *dead = 1;
        for (int e = 0; e < E; e++) nh[e] = 0;
        for (int i = 0; i < plan_ints(S); i++) plan[i] = 0;
        return;
    }
    int *cnt = plan, *off = plan + S, *mt128 = off + S + 1, *mt64 = mt128 + S + 1;
    int *mt256 = mt64 + S + 1;
    for (int j = 0; j < S; j++) cnt[j] = 0;
    for (int e = 0; e < E; e++) {
        const int j = place[rank * E + e];
        if (j < 0 || j >= S) continue;
        int i = 0;
        while (hold[e * G + i] != rank) i++;
        cnt[j] = beg[e * (G + 1) + i + 1] - beg[e * (G + 1) + i];
    }
    int o = 0, m1 = 0, m2 = 0, m3 = 0;
    for (int j = 0; j < S; j++) {
        off[j] = o; mt128[j] = m1; mt64[j] = m2; mt256[j] = m3;
        o += cnt[j];
        m1 += (cnt[j] + 127) / 128;
        m2 += (cnt[j] + 63) / 64;
        m3 += (cnt[j] + 255) / 256;
    }
    off[S] = o; mt128[S] = m1; mt64[S] = m2; mt256[S] = m3;
    for (int e = 0; e < E; e++) {
        int b = 0;
        for (int r = 0; r < rank; r++) b += recs[r * (E + 1) + 1 + e];
        base_r[e] = b;
    }
}

// One warp per local (token, rank) entry: its local expert-sorted slot (for
// the combine), its place in the expert's global row order, the holder whose
// range contains it, and a float4 copy of the token row into that holder's
// receive buffer with the return address beside it.
__global__ void __launch_bounds__(256)
ep_gather_kernel(const float *__restrict__ x, int T, int d, int d_pad, int k, int E, int rank,
                 int G, int recv_rows, const int *__restrict__ ids, const int *__restrict__ loc,
                 const int *__restrict__ tile_pref, const int *__restrict__ plan_local,
                 const int *__restrict__ base_r, const int *__restrict__ nh,
                 const int *__restrict__ hold, const int *__restrict__ beg,
                 const int *__restrict__ dst, float *const *__restrict__ recv_ptrs,
                 int2 *const *__restrict__ ret_ptrs, int *__restrict__ pos_of, int round_to_tf32,
                 const int *__restrict__ dead, DeviceStatus *status)
{
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp < T * k && !*dead) {
        const int t = warp / k;
        const int e = ids[warp];
        bool ok = e >= 0 && e < E;
        int q = -1, p = -1, pos_local = -1;
        if (ok) {
            const int lr = tile_pref[(size_t)(t / kRouterTile) * E + e] + loc[warp];
            pos_local = plan_local[E + e] + lr;
            const int gp = base_r[e] + lr;
            const int n = nh[e];
            int i = 0;
            while (i + 1 < n && beg[e * (G + 1) + i + 1] <= gp) i++;
            ok = n > 0 && gp >= beg[e * (G + 1) + i] && gp < beg[e * (G + 1) + i + 1];
            if (ok) {
                q = hold[e * G + i];
                p = dst[e * G + i] + gp - beg[e * (G + 1) + i];
            }
        }
        if (!ok || q < 0 || q >= G || p < 0 || p >= recv_rows || pos_local < 0 ||
            pos_local >= T * k) {
            if (lane == 0) atomicExch(&status->bad_index, 1);
        } else {
            if (lane == 0) {
                pos_of[warp] = pos_local;
                ret_ptrs[q][p] = make_int2(rank, pos_local);
            }
            const float *src = x + (size_t)t * d;
            float *dstp = recv_ptrs[q] + (size_t)p * d_pad;
            if ((d & 3) == 0) {
                const float4 *s4 = reinterpret_cast<const float4 *>(src);
                float4 *d4 = reinterpret_cast<float4 *>(dstp);
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
                    dstp[c] = round_to_tf32 ? round_tf32(v) : v;
                }
            }
        }
    }
    __threadfence_system();   // peer stores visible before the barrier that follows
}

// Plain-load copy of one packed expert slot from a peer's shard (IPC
// mapping, NVLink loads) into a local slot.
__global__ void __launch_bounds__(256)
ep_slot_copy_kernel(const float4 *__restrict__ src, float4 *__restrict__ dst, size_t n4)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (size_t)gridDim.x * blockDim.x)
        dst[i] = src[i];
}

// ---------------------------------------------------------------------
// state
// ---------------------------------------------------------------------
struct moe_b200_ep {
    int rank = 0, world = 1, device = 0, max_T = 0, max_rows = 0, recv_rows = 0, S = 0, E = 0;
    moe_b200_weights *w = nullptr;      // this rank's shard (spare slots filled by rebalance)
    ncclComm_t comm = nullptr;
    cudaStream_t stream = nullptr;      // library stream for the host-buffer entry
    DeviceStatus *status = nullptr;
    // placement: slot of expert e on rank q (-1: not held); base = at creation
    std::vector<int> place, base;
    int *d_place = nullptr;
    // IPC-shared buffers (this rank's) and the peer tables
    float *recv_x = nullptr;            // [recv_rows × d_pad]
    int2 *ret = nullptr;                // [recv_rows]
    float *y = nullptr;                 // [max_rows × d_pad] written by the holders
    float **d_recv_ptrs = nullptr, **d_y_ptrs = nullptr;
    int2 **d_ret_ptrs = nullptr;
    std::vector<const float *> peer_ug, peer_dn;   // every rank's packed slots
    std::vector<void *> opened;         // peer mappings to close
    // local work buffers
    float *h = nullptr;                 // [recv_rows × F_pad]
    float *xs = nullptr, *hs = nullptr; // 3xTF32 small parts of recv_x and h (on first use)
    float *rpart = nullptr;             // split-K router partial logits (small T)
    int rsplit = 1;
    float *probs = nullptr, *wts = nullptr;
    int *ids = nullptr, *loc = nullptr, *tile_cnt = nullptr, *tile_pref = nullptr;
    // local record {generation, cnt[E] | off | ...}: the scan writes the plan
    // at local + 1, the all-gather sends local[0 .. E] (generation, counts)
    int *local = nullptr, *plan_local = nullptr, *plan_q = nullptr, *pos_of = nullptr;
    int *recs = nullptr, *base_r = nullptr, *bar = nullptr, *dead = nullptr;
    int *nh = nullptr, *hold = nullptr, *beg = nullptr, *dst = nullptr;
    float *io_x = nullptr, *io_out = nullptr, *io_bias = nullptr;
    int timeout_ms = 0;                 // host watchdog on the group's barriers (0 = none)
    // host-buffer forward: chunk copies in and out on their own streams
    static constexpr int kMaxChunks = 4;
    cudaStream_t s_in = nullptr, s_out = nullptr;
    cudaEvent_t ev_in[kMaxChunks] = {}, ev_done[kMaxChunks] = {};
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
    if (ep->comm) {
        // the communicator is non-blocking: finalize, wait (bounded) until it
        // is quiescent, then free it; abort if it does not settle
        const ncclResult_t f = nccl().CommFinalize(ep->comm);   // usually ncclInProgress
        bool settled = f == ncclSuccess || f == ncclInProgress;
        const auto t0 = std::chrono::steady_clock::now();
        const int limit_ms = ep->timeout_ms > 0 ? ep->timeout_ms : 30000;
        while (settled) {
            ncclResult_t a = ncclInProgress;
            if (nccl().CommGetAsyncError(ep->comm, &a) != ncclSuccess ||
                (a != ncclSuccess && a != ncclInProgress)) {
                settled = false;
                break;
            }
            if (a == ncclSuccess) break;
            if (std::chrono::duration_cast<std::chrono::milliseconds>(
                    std::chrono::steady_clock::now() - t0).count() > limit_ms) {
                settled = false;
                break;
            }
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
        if (settled) nccl().CommDestroy(ep->comm);
        else nccl().CommAbort(ep->comm);
    }
    void *bufs[] = {ep->recv_x, ep->ret, ep->y, ep->d_recv_ptrs, ep->d_y_ptrs, ep->d_ret_ptrs,
                    ep->h, ep->xs, ep->hs, ep->rpart, ep->probs, ep->wts, ep->ids, ep->loc,
                    ep->tile_cnt, ep->tile_pref, ep->local, ep->plan_q, ep->pos_of,
                    ep->recs, ep->base_r, ep->bar, ep->dead, ep->nh, ep->hold, ep->beg, ep->dst,
                    ep->d_place, ep->io_x, ep->io_out, ep->io_bias, ep->status};
    for (void *b : bufs)
        if (b) cudaFree(b);
    if (ep->stream) cudaStreamDestroy(ep->stream);
    if (ep->s_in) cudaStreamDestroy(ep->s_in);
    if (ep->s_out) cudaStreamDestroy(ep->s_out);
    for (int c = 0; c < moe_b200_ep::kMaxChunks; c++) {
        if (ep->ev_in[c]) cudaEventDestroy(ep->ev_in[c]);
        if (ep->ev_done[c]) cudaEventDestroy(ep->ev_done[c]);
    }
    delete ep;
}

// Wait for `s` on the host, but for at most timeout_ms (0 = no limit).  A
// rank that never reaches a collective leaves the others' NCCL kernels
// spinning; past the limit the communicator is aborted, which ends those
// kernels, and the call returns MOE_B200_E_TIMEOUT.  The group is unusable
// afterwards (destroy it).
int ep_wait(moe_b200_ep *ep, cudaStream_t s) {
    if (ep->timeout_ms <= 0) {
        EP_CK(cudaStreamSynchronize(s));
        return MOE_B200_OK;
    }
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        const cudaError_t q = cudaStreamQuery(s);
        if (q == cudaSuccess) return MOE_B200_OK;
        if (q != cudaErrorNotReady)
            return ep_fail(MOE_B200_E_CUDA, "stream: %s%s", cudaGetErrorString(q));
        ncclResult_t async_err = ncclSuccess;
        if (ep->comm && nccl().CommGetAsyncError(ep->comm, &async_err) == ncclSuccess &&
            async_err != ncclSuccess && async_err != ncclInProgress) {
            nccl().CommAbort(ep->comm);
            ep->comm = nullptr;
            return ep_fail(MOE_B200_E_NCCL, "communicator error: %s%s",
                           nccl().GetErrorString(async_err));
        }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0).count();
        if (ms > ep->timeout_ms) {
            if (ep->comm) nccl().CommAbort(ep->comm);
            ep->comm = nullptr;
            return ep_fail(MOE_B200_E_TIMEOUT,
                           "expert-parallel step did not finish within the watchdog limit; "
                           "communicator aborted%s%s");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// Settle an NCCL call on the group's non-blocking communicator: success,
// or ncclInProgress waited out (bounded by the watchdog, after which the
// communicator is aborted and MOE_B200_E_TIMEOUT returned).
int ep_nccl(moe_b200_ep *ep, ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return MOE_B200_OK;
    if (r != ncclInProgress || !ep->comm) {
        if (ep->comm) nccl().CommAbort(ep->comm);
        ep->comm = nullptr;
        return ep_fail(MOE_B200_E_NCCL, "%s: %s", what, nccl().GetErrorString(r));
    }
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        ncclResult_t a = ncclInProgress;
        const ncclResult_t q = nccl().CommGetAsyncError(ep->comm, &a);
        if (q == ncclSuccess && a == ncclSuccess) return MOE_B200_OK;
        if (q != ncclSuccess || a != ncclInProgress) {
            nccl().CommAbort(ep->comm);
            ep->comm = nullptr;
            return ep_fail(MOE_B200_E_NCCL, "%s: %s", what,
                           nccl().GetErrorString(q != ncclSuccess ? q : a));
        }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0).count();
        if (ep->timeout_ms > 0 && ms > ep->timeout_ms) {
            nccl().CommAbort(ep->comm);
            ep->comm = nullptr;
            return ep_fail(MOE_B200_E_TIMEOUT, "%s did not complete within the watchdog limit; "
                                               "communicator aborted%s", what);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

int upload_place(moe_b200_ep *ep) {
    EP_CK(cudaMemcpy(ep->d_place, ep->place.data(), ep->place.size() * sizeof(int),
                     cudaMemcpyHostToDevice));
    return MOE_B200_OK;
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

static int split_args_ok(const int *counts_all, int world, int E, const int *place, int n_slots) {
    return counts_all && place && world >= 1 && world <= kMaxWorld && E >= 1 &&
           E <= kMaxExperts && n_slots >= 1 && n_slots <= E;
}

extern "C" int moe_b200_ep_split(const int *counts_all, int world, int E, const int *place,
                                 int n_slots, int *n_holders, int *holders, int *row_begin,
                                 int *recv_offset, long long *recv_rows, long long *cost) {
    if (!split_args_ok(counts_all, world, E, place, n_slots) || !n_holders || !holders ||
        !row_begin || !recv_offset)
        return ep_fail(MOE_B200_E_INVALID, "bad split arguments%s%s");
    for (int i = 0; i < world * E; i++)
        if (place[i] >= n_slots || place[i] < -1)
            return ep_fail(MOE_B200_E_INVALID, "placement slot out of range%s%s");
    if (ep_split(counts_all, E, world, E, place, n_slots, n_holders, holders, row_begin,
                 recv_offset, recv_rows, cost))
        return ep_fail(MOE_B200_E_INVALID, "an expert with rows has no holder%s%s");
    return MOE_B200_OK;
}

extern "C" int moe_b200_ep_place(const int *counts_all, int world, int E, const int *base_place,
                                 int n_slots, int *place) {
    if (!split_args_ok(counts_all, world, E, base_place, n_slots) || !place)
        return ep_fail(MOE_B200_E_INVALID, "bad placement arguments%s%s");
    for (int e = 0; e < E; e++) {
        int n = 0;
        for (int q = 0; q < world; q++) n += base_place[q * E + e] >= 0;
        if (n == 0) return ep_fail(MOE_B200_E_INVALID, "an expert has no base holder%s%s");
    }
    ep_place_greedy(counts_all, world, E, n_slots, base_place, place);
    return MOE_B200_OK;
}

extern "C" int moe_b200_ep_create(const void *unique_id, int rank, int world,
                                  int max_tokens_per_rank, moe_b200_weights *w,
                                  moe_b200_ep **out) {
    if (!unique_id || !w || !out || world < 1 || world > kMaxWorld || rank < 0 || rank >= world ||
        max_tokens_per_rank < 1)
        return ep_fail(MOE_B200_E_INVALID, "bad arguments to moe_b200_ep_create%s%s");
    if ((int64_t)max_tokens_per_rank * w->k * world > (int64_t)1 << 30)
        return ep_fail(MOE_B200_E_INVALID, "max_tokens_per_rank too large%s%s");
    if (!nccl().ok) return ep_fail(MOE_B200_E_NCCL, "libnccl.so.2 not found%s%s");
    EP_CK(cudaSetDevice(w->device));
    if (device_sms(w->device) == 0) return ep_fail(MOE_B200_E_NODEV, "device unusable%s%s");
    moe_b200_ep *ep = new moe_b200_ep();
    ep->rank = rank;
    ep->world = world;
    ep->device = w->device;
    ep->w = w;
    ep->E = w->E;
    ep->S = w->n_slots;
    ep->max_T = max_tokens_per_rank;
    ep->max_rows = max_tokens_per_rank * w->k;
    // every token of every rank may route to experts this rank holds
    ep->recv_rows = world * ep->max_rows;
    if (const char *p = std::getenv("MOE_B200_EP_TIMEOUT_MS")) ep->timeout_ms = std::atoi(p);
    int rc = MOE_B200_OK;
#define TRY(x)                      \
    do {                            \
        if ((rc = (x))) {           \
            ep_release(ep);         \
            return rc;              \
        }                           \
    } while (0)
    auto alloc = [&](void **p, size_t bytes) -> int {
        cudaError_t e = dev_alloc(p, bytes);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return ep_fail(MOE_B200_E_NOMEM, "expert-parallel buffers: %s%s", cudaGetErrorString(e));
        }
        return MOE_B200_OK;
    };
    const size_t R = ep->max_rows, RR = ep->recv_rows, T = ep->max_T, E = w->E, G = world;
    const size_t S = ep->S;
    const size_t tiles = ceil_div<size_t>(T, kRouterTile);
    TRY(alloc((void **)&ep->recv_x, RR * w->d_pad * 4));
    TRY(alloc((void **)&ep->ret, RR * sizeof(int2)));
    TRY(alloc((void **)&ep->y, R * w->d_pad * 4));
    TRY(alloc((void **)&ep->h, RR * w->F_pad * 4));
    ep->rsplit = router_splits((int)T, w->d);
    if (ep->rsplit > 1) TRY(alloc((void **)&ep->rpart, (size_t)ep->rsplit * T * E * 4));
    TRY(alloc((void **)&ep->probs, T * E * 4));
    TRY(alloc((void **)&ep->wts, R * 4));
    TRY(alloc((void **)&ep->ids, R * 4));
    TRY(alloc((void **)&ep->loc, R * 4));
    TRY(alloc((void **)&ep->pos_of, R * 4));
    TRY(alloc((void **)&ep->tile_cnt, tiles * E * 4));
    TRY(alloc((void **)&ep->tile_pref, tiles * E * 4));
    TRY(alloc((void **)&ep->local, (1 + plan_ints((int)E)) * 4));
    ep->plan_local = ep->local + 1;
    TRY(alloc((void **)&ep->plan_q, plan_ints((int)S) * 4));
    TRY(alloc((void **)&ep->recs, G * (E + 1) * 4));
    TRY(alloc((void **)&ep->dead, 4));
    TRY(alloc((void **)&ep->base_r, E * 4));
    TRY(alloc((void **)&ep->nh, E * 4));
    TRY(alloc((void **)&ep->hold, E * G * 4));
    TRY(alloc((void **)&ep->beg, E * (G + 1) * 4));
    TRY(alloc((void **)&ep->dst, E * G * 4));
    TRY(alloc((void **)&ep->d_place, G * E * 4));
    TRY(alloc((void **)&ep->bar, 4));
    TRY(alloc((void **)&ep->io_x, T * w->d * 4));
    TRY(alloc((void **)&ep->io_out, T * w->d * 4));
    TRY(alloc((void **)&ep->io_bias, E * 4));
    TRY(alloc((void **)&ep->status, sizeof(DeviceStatus)));
    TRY(alloc((void **)&ep->d_recv_ptrs, G * sizeof(float *)));
    TRY(alloc((void **)&ep->d_y_ptrs, G * sizeof(float *)));
    TRY(alloc((void **)&ep->d_ret_ptrs, G * sizeof(int2 *)));
    if (cudaMemset(ep->status, 0, sizeof(DeviceStatus)) != cudaSuccess ||
        cudaMemset(ep->bar, 0, 4) != cudaSuccess || cudaMemset(ep->local, 0, 4) != cudaSuccess ||
        cudaMemset(ep->recs, 0xff, G * (E + 1) * 4) != cudaSuccess ||
        cudaMemset(ep->dead, 0, 4) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ep->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ep->s_in, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ep->s_out, cudaStreamNonBlocking) != cudaSuccess)
        TRY(ep_fail(MOE_B200_E_CUDA, "expert-parallel set-up failed%s%s"));
    for (int c = 0; c < moe_b200_ep::kMaxChunks; c++)
        if (cudaEventCreateWithFlags(&ep->ev_in[c], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&ep->ev_done[c], cudaEventDisableTiming) != cudaSuccess)
            TRY(ep_fail(MOE_B200_E_CUDA, "expert-parallel events%s%s"));
    TRY(ep_tmap(&ep->up.tmA, ep->recv_x, RR, w->d_pad, 128));
    ep->up.tmB = w->tm_ug;
    TRY(ep_tmap(&ep->dn.tmA, ep->h, RR, w->F_pad, 128));
    ep->dn.tmB = w->tm_dn;
    ep->dup.tmW = w->tm_ug64;
    TRY(ep_tmap(&ep->dup.tmXb, ep->recv_x, RR, w->d_pad, 64));
    ep->dup.tmXb32 = ep->dup.tmXb;       // CTA-pair map, unused by the single-CTA kernels
    ep->ddn.tmW = w->tm_dn128;
    TRY(ep_tmap(&ep->ddn.tmXb, ep->h, RR, w->F_pad, 64));
    ep->ddn.tmXb32 = ep->ddn.tmXb;

    // communicator: non-blocking, so that a rank that never joins (or a bad
    // id) ends in the watchdog's abort instead of a host thread blocked for
    // good inside the bootstrap
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof id);
    {
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;
        ep->comm = nullptr;
        const ncclResult_t r = nccl().CommInitRankConfig(&ep->comm, world, id, rank, &cfg);
        TRY(ep_nccl(ep, r, "ncclCommInitRankConfig"));
    }
    // exchange, over NCCL: IPC handles of the three shared buffers and of the
    // shard's packed weights, the group's shape parameters (which must agree)
    // and every rank's base experts
    struct Blob {
        cudaIpcMemHandle_t h[5];
        long long max_t;
        int n_slots, E, d, F;
        int slot_expert[kMaxExperts];
    };
    Blob mine;
    std::memset(&mine, 0, sizeof mine);
    mine.max_t = max_tokens_per_rank;
    mine.n_slots = w->n_slots;
    mine.E = w->E; mine.d = w->d; mine.F = w->F;
    for (int j = 0; j < w->n_slots; j++) mine.slot_expert[j] = w->slot_expert[j];
    if (world > 1 && (cudaIpcGetMemHandle(&mine.h[0], ep->recv_x) != cudaSuccess ||
                      cudaIpcGetMemHandle(&mine.h[1], ep->ret) != cudaSuccess ||
                      cudaIpcGetMemHandle(&mine.h[2], ep->y) != cudaSuccess ||
                      cudaIpcGetMemHandle(&mine.h[3], w->ug) != cudaSuccess ||
                      cudaIpcGetMemHandle(&mine.h[4], w->dn) != cudaSuccess))
        TRY(ep_fail(MOE_B200_E_CUDA, "cudaIpcGetMemHandle failed%s%s"));
    const size_t HB = sizeof(Blob);
    std::vector<Blob> all(G);
    {
        unsigned char *dh = nullptr;
        TRY(alloc((void **)&dh, HB * G));
        int step = MOE_B200_OK;
        if (cudaMemcpy(dh + HB * rank, &mine, HB, cudaMemcpyHostToDevice) != cudaSuccess)
            step = ep_fail(MOE_B200_E_CUDA, "handle upload failed%s%s");
        if (!step)
            step = ep_nccl(ep, nccl().AllGather(dh + HB * rank, dh, HB, ncclChar, ep->comm,
                                                ep->stream), "ncclAllGather(handles)");
        if (!step) step = ep_wait(ep, ep->stream);
        if (!step && cudaMemcpy(all.data(), dh, HB * G, cudaMemcpyDeviceToHost) != cudaSuccess)
            step = ep_fail(MOE_B200_E_CUDA, "handle exchange failed%s%s");
        cudaFree(dh);
        TRY(step);
    }
    ep->place.assign(G * E, -1);
    for (int q = 0; q < world; q++) {
        const Blob &b = all[q];
        if (b.max_t != max_tokens_per_rank || b.n_slots != w->n_slots || b.E != w->E ||
            b.d != w->d || b.F != w->F)
            TRY(ep_fail(MOE_B200_E_INVALID, "ranks disagree on max_tokens_per_rank, the expert "
                                            "shape or the slot count%s%s"));
        for (int j = 0; j < b.n_slots; j++)
            if (b.slot_expert[j] >= 0) ep->place[(size_t)q * E + b.slot_expert[j]] = j;
    }
    for (size_t e = 0; e < E; e++) {
        int n = 0;
        for (size_t q = 0; q < G; q++) n += ep->place[q * E + e] >= 0;
        if (n == 0) TRY(ep_fail(MOE_B200_E_INVALID, "an expert is held by no rank%s%s"));
    }
    ep->base = ep->place;
    TRY(upload_place(ep));
    // peer mappings
    std::vector<float *> recv_ptrs(G), y_ptrs(G);
    std::vector<int2 *> ret_ptrs(G);
    ep->peer_ug.assign(G, nullptr);
    ep->peer_dn.assign(G, nullptr);
    recv_ptrs[rank] = ep->recv_x;
    y_ptrs[rank] = ep->y;
    ret_ptrs[rank] = ep->ret;
    ep->peer_ug[rank] = w->ug;
    ep->peer_dn[rank] = w->dn;
    for (int q = 0; q < world; q++) {
        if (q == rank) continue;
        void *p[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
        for (int i = 0; i < 5; i++) {
            cudaError_t e = cudaIpcOpenMemHandle(&p[i], all[q].h[i], cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess)
                TRY(ep_fail(MOE_B200_E_CUDA, "cudaIpcOpenMemHandle: %s%s", cudaGetErrorString(e)));
            ep->opened.push_back(p[i]);
        }
        recv_ptrs[q] = (float *)p[0];
        ret_ptrs[q] = (int2 *)p[1];
        y_ptrs[q] = (float *)p[2];
        ep->peer_ug[q] = (const float *)p[3];
        ep->peer_dn[q] = (const float *)p[4];
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
    if (!ep->comm) return ep_fail(MOE_B200_E_STATE, "the group was aborted; destroy it%s%s");
    const moe_b200_weights *w = ep->w;
    EP_CK(cudaSetDevice(ep->device));
    ncclResult_t async_err = ncclSuccess;
    EP_NC(nccl().CommGetAsyncError(ep->comm, &async_err));
    if (async_err != ncclSuccess && async_err != ncclInProgress)
        return ep_fail(MOE_B200_E_NCCL, "communicator error: %s%s", nccl().GetErrorString(async_err));
    cudaStream_t s = stream ? (cudaStream_t)stream : ep->stream;
    const int E = w->E, k = w->k, G = ep->world, S = ep->S;
    float *probs = d_router_probs ? d_router_probs : ep->probs;
    int *ids = d_expert_ids ? d_expert_ids : ep->ids;
    // The path is decided from values every rank shares (the group's token
    // capacity), never from this rank's own T: rows of one rank are computed
    // on others, and all of them must run the same arithmetic.
    const double avg_group = (double)ep->max_T * G * k / E;
    int path = opts ? opts->path : MOE_B200_PATH_AUTO;
    if (path == MOE_B200_PATH_AUTO)
        path = avg_group >= 64.0 ? MOE_B200_PATH_TF32 : MOE_B200_PATH_TF32X3;
    const bool onepass = path == MOE_B200_PATH_TF32 && avg_group < 64.0;
    if (path == MOE_B200_PATH_TF32X3 && !ep->xs) {
        EP_CK(cudaMalloc(&ep->xs, (size_t)ep->recv_rows * w->d_pad * 4));
        EP_CK(cudaMalloc(&ep->hs, (size_t)ep->recv_rows * w->F_pad * 4));
        int rc = ep_tmap(&ep->dup.tmXs, ep->xs, ep->recv_rows, w->d_pad, 64);
        if (!rc) rc = ep_tmap(&ep->ddn.tmXs, ep->hs, ep->recv_rows, w->F_pad, 64);
        if (rc) return rc;
    }
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
    int rc = ep_nccl(ep, nccl().AllGather(ep->local, ep->recs, E + 1, ncclInt32, ep->comm, s),
                     "ncclAllGather(counts)");
    if (rc) return rc;
    ep_plan_kernel<<<1, 32, 0, s>>>(ep->recs, G, E, S, ep->rank, ep->d_place, ep->local,
                                    ep->plan_q, ep->base_r, ep->nh, ep->hold, ep->beg, ep->dst,
                                    ep->dead, ep->status);
    EP_CK(cudaGetLastError());
    if (T > 0) {
        ep_gather_kernel<<<ceil_div(T * k, 8), 256, 0, s>>>(
            d_x, T, w->d, w->d_pad, k, E, ep->rank, G, ep->recv_rows, ids, ep->loc,
            ep->tile_pref, ep->plan_local, ep->base_r, ep->nh, ep->hold, ep->beg, ep->dst,
            ep->d_recv_ptrs, ep->d_ret_ptrs, ep->pos_of, path == MOE_B200_PATH_TF32, ep->dead,
            ep->status);
        EP_CK(cudaGetLastError());
    }
    if ((rc = ep_nccl(ep, nccl().AllReduce(ep->bar, ep->bar, 1, ncclInt32, ncclSum, ep->comm, s),
                      "ncclAllReduce(barrier)")))
        return rc;
    MARK(2);
    const int rows = ep->recv_rows;
    // TF32 on decode-sized groups runs the weight-streaming kernel's one-pass
    // mode.  Its down GEMM does not split K here (rows go straight to their
    // owners), unlike the single-GPU call, so the two agree to the TF32
    // tolerance rather than bit for bit on this path.
    if (path == MOE_B200_PATH_TF32 && !onepass) {
        const int sms = device_sms(ep->device);
        EP_CK(launch_tc_upgate(ep->up, w->d_pad, w->F_pad, ep->h, ep->plan_q, S, rows, sms,
                               ep->status, s));
        MARK(3);
        EP_CK(launch_tc_down(ep->dn, w->F_pad, w->d_pad, w->down_bn, ep->y, ep->plan_q, S, rows,
                             sms, ep->status, s, ep->d_y_ptrs, ep->ret));
    } else if (path == MOE_B200_PATH_TF32X3 || onepass) {
        const int sms = device_sms(ep->device);
        if (!onepass) EP_CK(launch_split_tf32(ep->recv_x, ep->xs, (size_t)rows * w->d_pad, s));
        EP_CK(launch_dec_upgate(ep->dup, w->d_pad, w->F_pad, ep->h, ep->hs, ep->plan_q, S, rows,
                                sms, 0, ep->status, s, onepass));
        MARK(3);
        EP_CK(launch_dec_down(ep->ddn, w->F_pad, w->d_pad, ep->y, ep->plan_q, S, rows, sms, 0,
                              ep->status, s, ep->d_y_ptrs, ep->ret, nullptr, onepass));
    } else {
        EP_CK(launch_ffma_upgate(ep->recv_x, w->d_pad, w->ug, w->F_pad, ep->h, ep->plan_q, S, rows,
                                 s));
        MARK(3);
        EP_CK(launch_ffma_down(ep->h, w->F_pad, w->dn, w->d_pad, ep->y, ep->plan_q, S, rows, s,
                               ep->d_y_ptrs, ep->ret));
    }
    MARK(4);   // the wait for the other ranks counts under the combine stage
    if ((rc = ep_nccl(ep, nccl().AllReduce(ep->bar, ep->bar, 1, ncclInt32, ncclSum, ep->comm, s),
                      "ncclAllReduce(barrier)")))
        return rc;
    if (T > 0) EP_CK(launch_combine(ep->y, w->d, w->d_pad, T, k, ep->pos_of, ep->wts, d_out, s));
    MARK(5);
#undef MARK
    note_forward(ep->device, E,
                 T > 0 ? 7 + (path == MOE_B200_PATH_TF32X3) + (router_splits(T, w->d) > 1) : 3,
                 path);
    return MOE_B200_OK;
}

// Chunks of the host-buffer forward: opts->host_chunks when set, else 2 for
// inputs of 64 MB and up (per rank, at the group's capacity) and 1 below.
// Taken from values every rank shares, because every chunk is a collective
// forward; rows are independent of the chunking, so results are not.
static int ep_host_chunks(const moe_b200_ep *ep, const moe_b200_opts *opts) {
    const moe_b200_weights *w = ep->w;
    if (w->d % 4) return 1;                 // chunk starts must stay 16-byte aligned
    int n = opts && opts->host_chunks > 0
                ? opts->host_chunks
                : ((size_t)ep->max_T * w->d * 4 >= ((size_t)64 << 20) ? 2 : 1);
    if (n > moe_b200_ep::kMaxChunks) n = moe_b200_ep::kMaxChunks;
    if (n > ep->max_T) n = ep->max_T;
    return n < 1 ? 1 : n;
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
    const int d = w->d, E = w->E, k = w->k;
    const float *d_bias = nullptr;
    if (router_bias) {
        EP_CK(cudaMemcpyAsync(ep->io_bias, router_bias, (size_t)E * 4, cudaMemcpyHostToDevice, s));
        d_bias = ep->io_bias;
    }
    // chunk c's rows go up on s_in, its forward runs on s once they landed,
    // its results come back on s_out once it finished: the copies of one
    // chunk overlap the forwards of the others (pinned host buffers)
    const int nch = ep_host_chunks(ep, opts);
    const int chunk = (ep->max_T + nch - 1) / nch;
    for (int c = 0; c < nch; c++) {
        const int t0 = c * chunk;
        const int tc = T - t0 < 0 ? 0 : (T - t0 < chunk ? T - t0 : chunk);
        if (tc > 0)
            EP_CK(cudaMemcpyAsync(ep->io_x + (size_t)t0 * d, x + (size_t)t0 * d,
                                  (size_t)tc * d * 4, cudaMemcpyHostToDevice, ep->s_in));
        EP_CK(cudaEventRecord(ep->ev_in[c], ep->s_in));
        EP_CK(cudaStreamWaitEvent(s, ep->ev_in[c], 0));
        int rc = moe_b200_ep_forward_device(ep, d_bias, ep->io_x + (size_t)t0 * d, tc,
                                            ep->io_out + (size_t)t0 * d,
                                            ep->probs + (size_t)t0 * E, ep->ids + (size_t)t0 * k,
                                            opts, s);
        if (rc) return rc;
        EP_CK(cudaEventRecord(ep->ev_done[c], s));
        EP_CK(cudaStreamWaitEvent(ep->s_out, ep->ev_done[c], 0));
        if (tc > 0) {
            EP_CK(cudaMemcpyAsync(out + (size_t)t0 * d, ep->io_out + (size_t)t0 * d,
                                  (size_t)tc * d * 4, cudaMemcpyDeviceToHost, ep->s_out));
            if (router_probs)
                EP_CK(cudaMemcpyAsync(router_probs + (size_t)t0 * E, ep->probs + (size_t)t0 * E,
                                      (size_t)tc * E * 4, cudaMemcpyDeviceToHost, ep->s_out));
            if (expert_ids)
                EP_CK(cudaMemcpyAsync(expert_ids + (size_t)t0 * k, ep->ids + (size_t)t0 * k,
                                      (size_t)tc * k * 4, cudaMemcpyDeviceToHost, ep->s_out));
        }
    }
    int rc = ep_wait(ep, s);
    if (!rc) rc = ep_wait(ep, ep->s_out);
    if (rc) return rc;
    DeviceStatus st;
    EP_CK(cudaMemcpy(&st, ep->status, sizeof st, cudaMemcpyDeviceToHost));
    if (st.bad_index || st.timeout) {
        EP_CK(cudaMemset(ep->status, 0, sizeof st));
        if (st.timeout) return ep_fail(MOE_B200_E_TIMEOUT, "device wait timed out%s%s");
        if (st.bad_index == 2)
            return ep_fail(MOE_B200_E_NCCL, "a rank's count record is from another step: the "
                                            "exchange did not happen%s%s");
        return ep_fail(MOE_B200_E_CUDA, "device bounds check rejected an index%s%s");
    }
    return MOE_B200_OK;
}

extern "C" int moe_b200_ep_counts(moe_b200_ep *ep, int *counts_all, int *recv_rows) {
    if (!ep) return ep_fail(MOE_B200_E_INVALID, "null ep%s%s");
    EP_CK(cudaSetDevice(ep->device));
    EP_CK(cudaDeviceSynchronize());
    if (counts_all) {
        std::vector<int> r((size_t)ep->world * (ep->E + 1));
        EP_CK(cudaMemcpy(r.data(), ep->recs, r.size() * 4, cudaMemcpyDeviceToHost));
        for (int q = 0; q < ep->world; q++)
            std::memcpy(counts_all + (size_t)q * ep->E, r.data() + (size_t)q * (ep->E + 1) + 1,
                        (size_t)ep->E * 4);
    }
    if (recv_rows)
        EP_CK(cudaMemcpy(recv_rows, ep->plan_q + 2 * ep->S, sizeof(int),
                         cudaMemcpyDeviceToHost));   // off[S] == rows this rank received
    return MOE_B200_OK;
}

extern "C" int moe_b200_ep_placement(const moe_b200_ep *ep, int *place) {
    if (!ep || !place) return ep_fail(MOE_B200_E_INVALID, "null argument%s%s");
    std::memcpy(place, ep->place.data(), ep->place.size() * sizeof(int));
    return MOE_B200_OK;
}

extern "C" int moe_b200_ep_rebalance(moe_b200_ep *ep) {
    if (!ep) return ep_fail(MOE_B200_E_INVALID, "null ep%s%s");
    if (!ep->comm) return ep_fail(MOE_B200_E_STATE, "the group was aborted; destroy it%s%s");
    EP_CK(cudaSetDevice(ep->device));
    EP_CK(cudaDeviceSynchronize());
    const int G = ep->world, E = ep->E, S = ep->S;
    std::vector<int> counts((size_t)G * E), place((size_t)G * E);
    int rc = moe_b200_ep_counts(ep, counts.data(), nullptr);
    if (rc) return rc;
    ep_place_greedy(counts.data(), G, E, S, ep->base.data(), place.data());
    // fill this rank's newly assigned slots from the expert's first base
    // holder, over NVLink with plain loads; base slots never change, so the
    // sources stay valid while the other ranks copy too
    moe_b200_weights *w = ep->w;
    const size_t ug_slot = (size_t)2 * w->F_pad * w->d_pad, dn_slot = (size_t)w->d_pad * w->F_pad;
    const int sms = device_sms(ep->device);
    for (int e = 0; e < E; e++) {
        const int j = place[(size_t)ep->rank * E + e];
        if (j < 0 || j == ep->place[(size_t)ep->rank * E + e]) continue;
        int src = -1;
        for (int q = 0; q < G && src < 0; q++)
            if (ep->base[(size_t)q * E + e] >= 0) src = q;
        const int sj = ep->base[(size_t)src * E + e];
        ep_slot_copy_kernel<<<sms * 4, 256, 0, ep->stream>>>(
            reinterpret_cast<const float4 *>(ep->peer_ug[src] + sj * ug_slot),
            reinterpret_cast<float4 *>(w->ug + j * ug_slot), ug_slot / 4);
        ep_slot_copy_kernel<<<sms * 4, 256, 0, ep->stream>>>(
            reinterpret_cast<const float4 *>(ep->peer_dn[src] + sj * dn_slot),
            reinterpret_cast<float4 *>(w->dn + j * dn_slot), dn_slot / 4);
        EP_CK(cudaGetLastError());
    }
    // slots this rank gives up hold nothing from now on
    for (int e = 0; e < E; e++) {
        const int was = ep->place[(size_t)ep->rank * E + e];
        if (was >= 0 && place[(size_t)ep->rank * E + e] != was) w->slot_expert[was] = -1;
    }
    for (int e = 0; e < E; e++) {
        const int j = place[(size_t)ep->rank * E + e];
        if (j >= 0) w->slot_expert[j] = e;
    }
    ep->place = place;
    if ((rc = upload_place(ep))) return rc;
    // every rank has its replicas before anyone forwards with the new placement
    if ((rc = ep_nccl(ep, nccl().AllReduce(ep->bar, ep->bar, 1, ncclInt32, ncclSum, ep->comm,
                                           ep->stream), "ncclAllReduce(barrier)")))
        return rc;
    return ep_wait(ep, ep->stream);
}

extern "C" int moe_b200_ep_set_timeout(moe_b200_ep *ep, int timeout_ms) {
    if (!ep || timeout_ms < 0) return ep_fail(MOE_B200_E_INVALID, "bad arguments%s%s");
    ep->timeout_ms = timeout_ms;
    return MOE_B200_OK;
}
