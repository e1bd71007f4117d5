// elementwise.cu - the glue of the layer stack: residual add and RMSNorm between MoE blocks.
//
// Rule (host reference rms_ref, metal/src/elementwise_parity.cpp:84-100, mean form with weight): per row,
// ss = sum of v^2 in fp64, den = sqrt(ss / cols + eps) in fp64, out = (float)((v / den) * w).  The kernel
// keeps every operation in fp64 as the host does; only the order of the ss additions differs (a fixed tree),
// which moves den by a few fp64 ulps and the f32 output essentially never.
#include "common.cuh"
#include "kernels.cuh"

namespace smoe {

constexpr int kNormThreads = 256;

// One CTA per row.  residual may be null (plain rms_norm_weighted), w may be null (unit weight).
__global__ void __launch_bounds__(kNormThreads) add_rms_norm_kernel(float* __restrict__ x,
                                                                    const float* __restrict__ residual,
                                                                    const float* __restrict__ w, int64_t cols,
                                                                    float eps) {
    __shared__ double s_part[kNormThreads / 32];
    __shared__ double s_den;
    const int64_t row = blockIdx.x;
    float* xr = x + row * cols;
    const float* rr = residual ? residual + row * cols : nullptr;
    double ss = 0.0;
    for (int64_t c = threadIdx.x; c < cols; c += kNormThreads) {
        const float v = rr ? __fadd_rn(xr[c], rr[c]) : xr[c];
        if (rr) xr[c] = v;  // the residual sum, read back below by the same thread
        ss = fma((double) v, (double) v, ss);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) s_part[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int i = 0; i < kNormThreads / 32; i++) t += s_part[i];
        s_den = sqrt(t / (double) cols + (double) eps);
    }
    __syncthreads();
    const double den = s_den;
    for (int64_t c = threadIdx.x; c < cols; c += kNormThreads) {
        const double v = (double) xr[c];
        xr[c] = (float) ((v / den) * (w ? (double) w[c] : 1.0));
    }
}

cudaError_t launch_add_rms_norm(float* x, const float* residual, const float* w, int64_t rows, int64_t cols,
                                float eps, cudaStream_t s) {
    add_rms_norm_kernel<<<(unsigned) rows, kNormThreads, 0, s>>>(x, residual, w, cols, eps);
    return cudaGetLastError();
}

}  // namespace smoe
