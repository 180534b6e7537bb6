// common.cuh — shared device helpers of the MoE hot path.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define MOE_DEV __device__ __forceinline__

namespace moe {

constexpr int kMaxExperts = 128;   // router/dispatch limit (configs use <= 64)
constexpr int kMaxTopK = 8;

template <typename T>
__host__ __device__ __forceinline__ T ceil_div(T a, T b) { return (a + b - 1) / b; }

template <typename T>
__host__ __device__ __forceinline__ T round_up(T a, T b) { return ceil_div(a, b) * b; }

// ---------------------------------------------------------------------
// exp as llm.c's softmax and SwiGLU compute it (src/matrix.c:82-116):
// clamp to [-88, 88], split v*log2(e) = n + f with n = floor, evaluate
// 2^f with the reference's degree-6 polynomial table in Horner form with
// fused multiply-adds, and scale by 2^n built in the exponent field.
// Using the same table keeps router probabilities bit-identical to the
// reference's for identical logits.
// ---------------------------------------------------------------------
MOE_DEV float exp_ref(float v) {
    v = fminf(fmaxf(v, -88.0f), 88.0f);
    const float z = __fmul_rn(v, 1.4426950408f);
    const float n = floorf(z);
    const float f = __fsub_rn(z, n);
    float p = 0.0001540353f;
    p = __fmaf_rn(p, f, 0.0013333558f);
    p = __fmaf_rn(p, f, 0.0096181292f);
    p = __fmaf_rn(p, f, 0.0555041086f);
    p = __fmaf_rn(p, f, 0.2402265069f);
    p = __fmaf_rn(p, f, 0.6931471806f);
    p = __fmaf_rn(p, f, 1.0000000000f);
    const int ni = __float2int_rn(n);
    const float scale = __int_as_float((ni + 127) << 23);
    return __fmul_rn(p, scale);
}

// silu(g) * u as llm.c's swiglu computes it (src/matrix.c:618-655):
// sigmoid = 1 / (1 + exp(-g)), silu = g * sigmoid, h = silu * u.
MOE_DEV float swiglu_ref(float g, float u) {
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_ref(-g)));
    return __fmul_rn(__fmul_rn(g, sig), u);
}

// One token's routing, in place on its logits row[0..E) (bias already
// added): the reference's softmax (softmax_rows, src/matrix.c:529-586, AVX2
// branch: 8-lane partial sums, hsum tree, scalar tail), its top-k
// (src/transformer.c:312-332: k passes, strict '>', best = -1, best_e = 0,
// e ascending, chosen experts skipped) and renormalisation (:334-337,350).
// Leaves the probabilities in row and writes sel[k] (rank order) and w[k].
MOE_DEV void route_token(float *row, int E, int k, int *sel, float *w) {
    // (every small array below is indexed with compile-time indices only, so
    // it stays in registers; the arithmetic and its order are the reference's)
    const int nv = E - E % 8;
    float mx = -1e38f;
    for (int e = 0; e < E; e++) mx = fmaxf(mx, row[e]);
    float lane[8];
#pragma unroll
    for (int l = 0; l < 8; l++) lane[l] = 0.0f;
    for (int e0 = 0; e0 < nv; e0 += 8) {
#pragma unroll
        for (int l = 0; l < 8; l++) {
            const float ex = exp_ref(__fsub_rn(row[e0 + l], mx));
            row[e0 + l] = ex;
            lane[l] = __fadd_rn(lane[l], ex);
        }
    }
    const float a0 = __fadd_rn(lane[0], lane[4]), a1 = __fadd_rn(lane[1], lane[5]);
    const float a2 = __fadd_rn(lane[2], lane[6]), a3 = __fadd_rn(lane[3], lane[7]);
    float sum = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
    for (int e = nv; e < E; e++) {
        row[e] = expf(__fsub_rn(row[e], mx));
        sum = __fadd_rn(sum, row[e]);
    }
    const float inv = __fdiv_rn(1.0f, sum);
    for (int e = 0; e < nv; e++) row[e] = __fmul_rn(row[e], inv);
    for (int e = nv; e < E; e++) row[e] = __fdiv_rn(row[e], sum);
    int pick[kMaxTopK];
#pragma unroll
    for (int r = 0; r < kMaxTopK; r++) pick[r] = -1;
#pragma unroll
    for (int r = 0; r < kMaxTopK; r++) {
        if (r >= k) break;
        float best = -1.0f;
        int best_e = 0;
        for (int e = 0; e < E; e++) {
            bool taken = false;
#pragma unroll
            for (int q = 0; q < kMaxTopK; q++) taken |= (pick[q] == e);
            if (!taken && row[e] > best) { best = row[e]; best_e = e; }
        }
        pick[r] = best_e;
    }
    float s = 0.0f;
#pragma unroll
    for (int r = 0; r < kMaxTopK; r++)
        if (r < k) s = __fadd_rn(s, row[pick[r]]);
    const float winv = (s > 1e-9f) ? __fdiv_rn(1.0f, s) : 0.0f;
#pragma unroll
    for (int r = 0; r < kMaxTopK; r++) {
        if (r < k) {
            sel[r] = pick[r];
            w[r] = __fmul_rn(row[pick[r]], winv);
        }
    }
}

// route_token for E <= 8 with the row in registers: the same arithmetic in
// the same order (E = 8: one 8-lane chunk, hsum tree; E < 8: the scalar
// tail only), every array indexed by compile-time constants.  For a single
// thread on the latency path (the device decode step), where route_token's
// dependent shared-memory accesses cost microseconds.
MOE_DEV void route_token8(float *row_io, int E, int k, int *sel, float *w) {
    float row[8];
#pragma unroll
    for (int e = 0; e < 8; e++) row[e] = e < E ? row_io[e] : 0.0f;
    float mx = -1e38f;
#pragma unroll
    for (int e = 0; e < 8; e++)
        if (e < E) mx = fmaxf(mx, row[e]);
    if (E == 8) {
        float lane[8];
#pragma unroll
        for (int l = 0; l < 8; l++) {
            row[l] = exp_ref(__fsub_rn(row[l], mx));
            lane[l] = __fadd_rn(0.0f, row[l]);
        }
        const float a0 = __fadd_rn(lane[0], lane[4]), a1 = __fadd_rn(lane[1], lane[5]);
        const float a2 = __fadd_rn(lane[2], lane[6]), a3 = __fadd_rn(lane[3], lane[7]);
        const float sum = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
        const float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
        for (int l = 0; l < 8; l++) row[l] = __fmul_rn(row[l], inv);
    } else {
        // no full 8-lane chunk: the zero lanes sum to 0, then the scalar tail
        float sum = __fadd_rn(__fadd_rn(0.0f, 0.0f), __fadd_rn(0.0f, 0.0f));
#pragma unroll
        for (int e = 0; e < 8; e++)
            if (e < E) {
                row[e] = expf(__fsub_rn(row[e], mx));
                sum = __fadd_rn(sum, row[e]);
            }
#pragma unroll
        for (int e = 0; e < 8; e++)
            if (e < E) row[e] = __fdiv_rn(row[e], sum);
    }
    int pick[kMaxTopK];
    float pv[kMaxTopK];
#pragma unroll
    for (int r = 0; r < kMaxTopK; r++) { pick[r] = -1; pv[r] = 0.0f; }
#pragma unroll
    for (int r = 0; r < kMaxTopK; r++) {
        if (r >= k) break;
        float best = -1.0f;
        int best_e = 0;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            if (e >= E) break;
            bool taken = false;
#pragma unroll
            for (int q = 0; q < kMaxTopK; q++) taken |= (pick[q] == e);
            if (!taken && row[e] > best) { best = row[e]; best_e = e; }
        }
        pick[r] = best_e;
        float v = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; e++)
            if (e == best_e) v = row[e];
        pv[r] = v;
    }
    float s = 0.0f;
#pragma unroll
    for (int r = 0; r < kMaxTopK; r++)
        if (r < k) s = __fadd_rn(s, pv[r]);
    const float winv = (s > 1e-9f) ? __fdiv_rn(1.0f, s) : 0.0f;
#pragma unroll
    for (int r = 0; r < kMaxTopK; r++) {
        if (r < k) {
            sel[r] = pick[r];
            w[r] = __fmul_rn(pv[r], winv);
        }
    }
#pragma unroll
    for (int e = 0; e < 8; e++)
        if (e < E) row_io[e] = row[e];
}

// Round an fp32 value to the nearest TF32 (10-bit mantissa, ties away
// from zero), returned as fp32 bits with the low 13 mantissa bits zero.
// tcgen05 kind::tf32 reads only the TF32 bits of its fp32 operands, i.e.
// truncates; rounding the activations first removes that one-sided bias.
MOE_DEV float round_tf32(float v) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return __uint_as_float(r);
}

// v minus its TF32 truncation (the low 13 mantissa bits, as an fp32 value;
// exact): what a tcgen05 kind::tf32 MMA drops when it reads v.
MOE_DEV float tf32_residual(float v) {
    return __fsub_rn(v, __uint_as_float(__float_as_uint(v) & 0xFFFFE000u));
}

// ---------------------------------------------------------------------
// Seeded synthetic generator (bit-identical to the oracle's host copy).
// ---------------------------------------------------------------------
__host__ __device__ __forceinline__ uint64_t sm64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint64_t synth_key(uint64_t seed, uint64_t stream) {
    return sm64(sm64(seed) ^ (stream * 0xD6E8FEB86659FD93ULL));
}

__host__ __device__ __forceinline__ float synth_value(uint64_t key, uint64_t idx, float std) {
    uint32_t s = 0;
#pragma unroll
    for (int j = 0; j < 3; j++) {
        const uint64_t h = sm64(key + 3ULL * idx + (uint64_t)j);
        s += (uint32_t)(h & 0xFFFF) + (uint32_t)((h >> 16) & 0xFFFF) +
             (uint32_t)((h >> 32) & 0xFFFF) + (uint32_t)(h >> 48);
    }
#ifdef __CUDA_ARCH__
    const float z = __fmul_rn((float)((int32_t)s - 393210), 1.0f / 65536.0f);
    return __fmul_rn(z, std);
#else
    const float z = (float)((int32_t)s - 393210) * (1.0f / 65536.0f);
    return z * std;
#endif
}

// ---------------------------------------------------------------------
// Bounded waits: every spin in this library gives up after kWaitNs
// nanoseconds of %globaltimer, records a timeout and lets the kernel
// leave cleanly instead of hanging the GPU.
// ---------------------------------------------------------------------
constexpr uint64_t kWaitNs = 2000000000ULL;   // 2 s

MOE_DEV uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Error word written by kernels (device-global, read by the host).
struct DeviceStatus {
    int timeout;       // nonzero: a bounded wait ran out (code = site id)
    int bad_index;     // nonzero: a bounds check rejected an index
};

}  // namespace moe
