// weights.cu — device weight layout of the expert set, and the seeded
// synthetic generator.
//
// Host layout (llm.c include/transformer.h:35-39, row-major fp32):
//   W_gate, W_up [d × F]   W_down [F × d]
// Device layout (K-major, zero-padded to d_pad = roundup(d,128),
// F_pad = roundup(F,128)), one contiguous block per expert:
//   W_ug [2*F_pad × d_pad]: 256-row groups, rows 0..127 of group b are
//        gate columns f = 128b .. 128b+127, rows 128..255 the up columns of
//        the same f — so one 256-wide GEMM tile holds matching gate and up
//        accumulators and SwiGLU runs in its epilogue.
//   W_dn [d_pad × F_pad]: row j = output column j of W_down.
// Padding rows/columns are zero, so padded K contributes nothing and padded
// outputs are never stored.
#include "kernels.cuh"

namespace moe {

// dst row of column c of a [R × C] source matrix, for each layout mode
__device__ __forceinline__ int packed_row(int c, int mode) {
    if (mode == 0) return c;                                  // plain transpose
    const int b = c >> 7, w = c & 127;
    return b * 256 + w + (mode == 2 ? 128 : 0);               // 1 = gate, 2 = up
}

// Transpose src [R × C] (row-major, ld C) into dst rows packed_row(c) of
// length ld_dst, for c < C_pad, r < R_pad; zero outside [R × C].
__global__ void __launch_bounds__(256)
pack_transpose_kernel(const float *__restrict__ src, int R, int C, float *__restrict__ dst,
                      int ld_dst, int R_pad, int C_pad, int mode)
{
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 × 8
    for (int i = ty; i < 32; i += 8) {
        const int r = r0 + i, c = c0 + tx;
        tile[i][tx] = (r < R && c < C) ? src[(size_t)r * C + c] : 0.0f;
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int c = c0 + i, r = r0 + tx;
        if (c < C_pad && r < R_pad) dst[(size_t)packed_row(c, mode) * ld_dst + r] = tile[tx][i];
    }
}

// Inverse of pack_transpose_kernel: dst [R × C] row-major.
__global__ void __launch_bounds__(256)
unpack_transpose_kernel(const float *__restrict__ src, int ld_src, int R, int C,
                        float *__restrict__ dst, int mode)
{
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int i = ty; i < 32; i += 8) {
        const int c = c0 + i, r = r0 + tx;
        tile[i][tx] = (c < C && r < R) ? src[(size_t)packed_row(c, mode) * ld_src + r] : 0.0f;
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int r = r0 + i, c = c0 + tx;
        if (r < R && c < C) dst[(size_t)r * C + c] = tile[tx][i];
    }
}

__global__ void synth_kernel(float *__restrict__ dst, size_t n, uint64_t key, uint64_t first,
                             float std)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        dst[i] = synth_value(key, first + i, std);
}

// Generate one expert's packed weights directly from the synthetic
// streams: element (i, f) of W_gate[e] is value i*F + f of stream
// (e, 0), of W_up[e] stream (e, 1); element (f, j) of W_down[e] is value
// f*d + j of stream (e, 2).
__global__ void synth_pack_upgate_kernel(float *__restrict__ dst, int d, int F, int d_pad,
                                         int F_pad, uint64_t key_g, uint64_t key_u, float std)
{
    const size_t n = (size_t)2 * F_pad * d_pad;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n;
         idx += (size_t)gridDim.x * blockDim.x) {
        const int row = (int)(idx / d_pad), i = (int)(idx % d_pad);
        const int b = row >> 8, w = row & 255;
        const bool up = w >= 128;
        const int f = b * 128 + (w & 127);
        float v = 0.0f;
        if (f < F && i < d) v = synth_value(up ? key_u : key_g, (uint64_t)i * F + f, std);
        dst[idx] = v;
    }
}

__global__ void synth_pack_down_kernel(float *__restrict__ dst, int d, int F, int d_pad,
                                       int F_pad, uint64_t key_d, float std)
{
    const size_t n = (size_t)d_pad * F_pad;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n;
         idx += (size_t)gridDim.x * blockDim.x) {
        const int j = (int)(idx / F_pad), f = (int)(idx % F_pad);
        float v = 0.0f;
        if (j < d && f < F) v = synth_value(key_d, (uint64_t)f * d + j, std);
        dst[idx] = v;
    }
}

cudaError_t launch_repack_upgate(const float *wg, const float *wu, int d, int F, int d_pad,
                                 int F_pad, float *dst, cudaStream_t s)
{
    dim3 grid(F_pad / 32, d_pad / 32);
    pack_transpose_kernel<<<grid, 256, 0, s>>>(wg, d, F, dst, d_pad, d_pad, F_pad, 1);
    pack_transpose_kernel<<<grid, 256, 0, s>>>(wu, d, F, dst, d_pad, d_pad, F_pad, 2);
    return cudaGetLastError();
}

cudaError_t launch_repack_down(const float *wd, int d, int F, int d_pad, int F_pad, float *dst,
                               cudaStream_t s)
{
    dim3 grid(d_pad / 32, F_pad / 32);
    pack_transpose_kernel<<<grid, 256, 0, s>>>(wd, F, d, dst, F_pad, F_pad, d_pad, 0);
    return cudaGetLastError();
}

cudaError_t launch_unpack_upgate(const float *src, int d, int F, int d_pad, int F_pad, float *wg,
                                 float *wu, cudaStream_t s)
{
    (void)F_pad;
    dim3 grid(ceil_div(F, 32), ceil_div(d, 32));
    if (wg) unpack_transpose_kernel<<<grid, 256, 0, s>>>(src, d_pad, d, F, wg, 1);
    if (wu) unpack_transpose_kernel<<<grid, 256, 0, s>>>(src, d_pad, d, F, wu, 2);
    return cudaGetLastError();
}

cudaError_t launch_unpack_down(const float *src, int d, int F, int d_pad, int F_pad, float *wd,
                               cudaStream_t s)
{
    (void)d_pad;
    dim3 grid(ceil_div(d, 32), ceil_div(F, 32));
    unpack_transpose_kernel<<<grid, 256, 0, s>>>(src, F_pad, F, d, wd, 0);
    return cudaGetLastError();
}

cudaError_t launch_synth(float *dst, size_t n, uint64_t seed, uint64_t stream, uint64_t first,
                         float std, cudaStream_t s)
{
    if (n == 0) return cudaSuccess;
    const size_t want = ceil_div<size_t>(n, 256);
    const int blocks = (int)(want < (size_t)148 * 64 ? want : (size_t)148 * 64);
    synth_kernel<<<blocks, 256, 0, s>>>(dst, n, synth_key(seed, stream), first, std);
    return cudaGetLastError();
}

cudaError_t launch_synth_pack_expert(float *ug, float *dn, int d, int F, int d_pad, int F_pad,
                                     uint64_t seed, uint64_t stream_g, uint64_t stream_u,
                                     uint64_t stream_d, float std, cudaStream_t s)
{
    synth_pack_upgate_kernel<<<148 * 32, 256, 0, s>>>(ug, d, F, d_pad, F_pad,
                                                      synth_key(seed, stream_g),
                                                      synth_key(seed, stream_u), std);
    synth_pack_down_kernel<<<148 * 32, 256, 0, s>>>(dn, d, F, d_pad, F_pad,
                                                    synth_key(seed, stream_d), std);
    return cudaGetLastError();
}

}  // namespace moe
