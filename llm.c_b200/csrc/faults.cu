// faults.cu — failure-detection hooks that fault nothing:
//
//   * moe_b200_debug_fail_alloc(n): the n-th device allocation the library
//     makes from now on (weights, workspace, expert-parallel buffers) fails
//     as if the device were out of memory, so the MOE_B200_E_NOMEM paths can
//     be tested on a healthy GPU.  llm.c's convention for the same event is
//     abort() with a message (src/transformer.c:28-32); the C-ABI returns
//     the status and the llm.c drop-ins print it and abort.
//   * moe_b200_debug_wait_probe(limit_us, arrive): one CTA waits on an
//     mbarrier with the library's bounded-wait helper (the one every
//     tensor-core kernel uses), nothing else in flight.  With arrive = 0
//     nobody arrives, the wait gives up after limit_us, the kernel records
//     the site in the status word and returns; the host reports
//     MOE_B200_E_TIMEOUT and the context stays usable.
#include "../../include/moe_b200.h"
#include "tc_common.cuh"
#include "weights.cuh"

#include <atomic>
#include <cstdio>

namespace moe {

namespace {
std::atomic<int> g_fail_countdown{0};
}

cudaError_t dev_alloc(void **p, size_t bytes) {
    int n = g_fail_countdown.load();
    while (n > 0) {
        if (g_fail_countdown.compare_exchange_weak(n, n - 1)) {
            if (n == 1) {
                *p = nullptr;
                return cudaErrorMemoryAllocation;
            }
            break;
        }
    }
    return cudaMalloc(p, bytes);
}

namespace {
constexpr int kProbeSite = 99;

__global__ void wait_probe_kernel(DeviceStatus *st, unsigned long long limit_ns, int arrive) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        tc::mbar_init(&bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (arrive) tc::mbar_arrive(&bar);
        if (!tc::mbar_wait(&bar, 0, nullptr, limit_ns)) atomicExch(&st->timeout, kProbeSite);
    }
}
}  // namespace

}  // namespace moe

using namespace moe;

extern "C" int moe_b200_debug_fail_alloc(int n) {
    if (n < 0) return set_last_error(MOE_B200_E_INVALID, "moe_b200_debug_fail_alloc: n < 0");
    g_fail_countdown.store(n);
    return MOE_B200_OK;
}

extern "C" int moe_b200_debug_wait_probe(int limit_us, int arrive) {
    if (limit_us <= 0 || limit_us > 2000000)
        return set_last_error(MOE_B200_E_INVALID, "wait probe: limit_us outside (0, 2e6]");
    int rc = moe_b200_init(-1);
    if (rc) return rc;
    DeviceStatus *st = nullptr;
    cudaError_t e = cudaMalloc(&st, sizeof(DeviceStatus));
    if (e == cudaSuccess) e = cudaMemset(st, 0, sizeof(DeviceStatus));
    if (e == cudaSuccess) {
        wait_probe_kernel<<<1, 32>>>(st, (unsigned long long)limit_us * 1000ULL, arrive);
        e = cudaGetLastError();
    }
    DeviceStatus h{};
    if (e == cudaSuccess) e = cudaMemcpy(&h, st, sizeof h, cudaMemcpyDeviceToHost);
    cudaFree(st);
    if (e != cudaSuccess) {
        char msg[200];
        std::snprintf(msg, sizeof msg, "wait probe: %s", cudaGetErrorString(e));
        return set_last_error(MOE_B200_E_CUDA, msg);
    }
    if (h.timeout) {
        char msg[200];
        std::snprintf(msg, sizeof msg, "device wait timed out (site %d) after %d us", h.timeout,
                      limit_us);
        return set_last_error(MOE_B200_E_TIMEOUT, msg);
    }
    return MOE_B200_OK;
}
