// block_ffn.cu — the pre-FFN RMSNorm of llm.c's block_forward
// (src/transformer.c:753, rms_norm at src/matrix.c:666-713), fused in front
// of the MoE forward; the residual add (src/transformer.c:767) is fused into
// the combine (router_dispatch.cu).
//
// One CTA per row.  The row is staged once in shared memory with coalesced
// 16-byte loads, so HBM sees one read and one write of [T × d].  The sum of
// squares then follows the reference's AVX2+FMA order exactly: 16 lanes of
// fused multiply-adds over 16-column chunks (one thread per lane, reading
// shared memory), lanes j and j+8 added, remaining 8-column chunks fused
// into those 8 lanes, the hsum256 tree (include/simd.h:110-121), and a
// scalar multiply-then-add tail; inv = 1 / sqrt(ss / d + eps) correctly
// rounded; y = (x · inv) · w.  Identical inputs give the CPU restatement's
// bits.  (The reference's own -ffast-math build turns 1/sqrtf into a
// reciprocal-square-root estimate plus a Newton step, which depends on the
// host CPU and differs from the correctly rounded value by a few ulp.)
#include "kernels.cuh"

namespace moe {

namespace {
constexpr int kNormThreads = 128;
}

__global__ void __launch_bounds__(kNormThreads)
rmsnorm_rows_kernel(const float *__restrict__ x, int T, int d, const float *__restrict__ weight,
                    float eps, float *__restrict__ out, int vec)
{
    // vec: d % 4 == 0 and x, weight, out 16-byte aligned (checked on the host)
    extern __shared__ float4 norm_smem4[];
    float *row = reinterpret_cast<float *>(norm_smem4);
    __shared__ float s_inv;
    const int t = blockIdx.x;
    if (t >= T) return;
    const float *xr = x + (size_t)t * d;
    float *yr = out + (size_t)t * d;
    if (vec) {
        for (int c = threadIdx.x; c < (d >> 2); c += kNormThreads)
            norm_smem4[c] = __ldg(reinterpret_cast<const float4 *>(xr) + c);
    } else {
        for (int c = threadIdx.x; c < d; c += kNormThreads) row[c] = __ldg(xr + c);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int l = threadIdx.x;
        const int n16 = d / 16;
        float a = 0.0f;
        if (l < 16) {
#pragma unroll 8
            for (int c = 0; c < n16; c++) {
                const float v = row[c * 16 + l];
                a = __fmaf_rn(v, v, a);
            }
        }
        // vss0 + vss1: lane l (< 8) adds lane l + 8
        float b = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 8));
        int j = n16 * 16;
        for (; j + 8 <= d; j += 8) {
            if (l < 8) {
                const float v = row[j + l];
                b = __fmaf_rn(v, v, b);
            }
        }
        // hsum256: s_i = b_i + b_{i+4}; (s0 + s1) + (s2 + s3)
        const float s = __fadd_rn(b, __shfl_down_sync(0xffffffffu, b, 4));
        const float p = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, 1));
        float ss = __fadd_rn(p, __shfl_down_sync(0xffffffffu, p, 2));
        if (l == 0) {
            for (; j < d; j++) ss = __fadd_rn(ss, __fmul_rn(row[j], row[j]));
            s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)d), eps)));
        }
    }
    __syncthreads();
    const float inv = s_inv;
    if (vec) {
        for (int c = threadIdx.x; c < (d >> 2); c += kNormThreads) {
            const float4 v = norm_smem4[c];
            const float4 g = __ldg(reinterpret_cast<const float4 *>(weight) + c);
            float4 o;
            o.x = __fmul_rn(__fmul_rn(v.x, inv), g.x);
            o.y = __fmul_rn(__fmul_rn(v.y, inv), g.y);
            o.z = __fmul_rn(__fmul_rn(v.z, inv), g.z);
            o.w = __fmul_rn(__fmul_rn(v.w, inv), g.w);
            reinterpret_cast<float4 *>(yr)[c] = o;
        }
    } else {
        for (int c = threadIdx.x; c < d; c += kNormThreads)
            yr[c] = __fmul_rn(__fmul_rn(row[c], inv), __ldg(weight + c));
    }
}

int rmsnorm_max_d() { return 56 * 1024; }   // the staged row fits 224 KB of shared memory

cudaError_t launch_rmsnorm(const float *x, int T, int d, const float *weight, float eps,
                           float *out, cudaStream_t s)
{
    if (T <= 0) return cudaSuccess;
    const size_t smem = (size_t)round_up(d, 4) * 4;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(rmsnorm_rows_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    const auto aligned = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
    const int vec = (d & 3) == 0 && aligned(x) && aligned(weight) && aligned(out);
    rmsnorm_rows_kernel<<<T, kNormThreads, smem, s>>>(x, T, d, weight, eps, out, vec);
    return cudaGetLastError();
}

}  // namespace moe
