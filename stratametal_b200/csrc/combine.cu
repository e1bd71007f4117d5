// combine.cu - the weighted combine (row a10) and the shared expert's sigmoid gate (row a9).
//
// out[t][j] = sum_i w[t][i] * parts[slot(t, i)][j] + shared[t][j], the sum taken in fp64 in router order and
// rounded once (pack_parity.cpp:8607-8616, moe_combine_parity.cpp:55-71).  Each product of two floats is
// exact in fp64, so this is the host reference's arithmetic.  The shared term is the shared expert's down
// output times sigmoid(g), g the bf16 gate dot, in f32 (layer_exec.cpp:522-528, pack_parity.cpp:8604-8613);
// it is added plain, not router weighted (shared_expert.hpp:88-92), and the weights are not normalised again
// (shared_expert.hpp:93-96).
#include "common.cuh"
#include "kernels.cuh"

namespace smoe {

__global__ void combine_kernel(const float* __restrict__ parts, const int32_t* __restrict__ slot,
                               const float* __restrict__ w, const float* __restrict__ shared,
                               const float* __restrict__ shared_logit, float* __restrict__ out,
                               float* __restrict__ shared_out, int64_t H, int k, int64_t shared_stride) {
    const int t = blockIdx.y;
    const int64_t j = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= H) return;
    double acc = 0.0;
    for (int i = 0; i < k; i++) {
        const int64_t pi = (int64_t) t * k + i;
        const int64_t s = slot ? (int64_t) slot[pi] : pi;
        if (s < 0) continue;  // an id outside the pool (recorded by the dispatch) contributes nothing
        acc += (double) w[pi] * (double) parts[s * H + j];
    }
    if (shared) {
        float sh = shared[(int64_t) t * shared_stride + j];
        if (shared_logit) {
            const float e = (float) exp(-(double) shared_logit[t]);
            const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
            sh = __fmul_rn(sh, sig);
        }
        if (shared_out) shared_out[(int64_t) t * H + j] = sh;
        acc += (double) sh;
    }
    out[(int64_t) t * H + j] = (float) acc;
}

// The same sum, four outputs per thread with 16-byte loads (H a multiple of 4, 16-byte aligned rows); the token's
// slots and weights are read once per CTA.
__global__ void combine4_kernel(const float* __restrict__ parts, const int32_t* __restrict__ slot,
                                const float* __restrict__ w, const float* __restrict__ shared,
                                const float* __restrict__ shared_logit, float* __restrict__ out,
                                float* __restrict__ shared_out, int64_t H, int k, int64_t shared_stride) {
    __shared__ int64_t s_row[kMaxK];
    __shared__ double s_w[kMaxK];
    const int t = blockIdx.y;
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        const int64_t pi = (int64_t) t * k + i;
        const int64_t sl = slot ? (int64_t) slot[pi] : pi;
        s_row[i] = sl;  // an id outside the pool (slot -1, recorded by the dispatch) contributes nothing
        s_w[i] = (double) w[pi];
    }
    __syncthreads();
    const int64_t j = 4 * ((int64_t) blockIdx.x * blockDim.x + threadIdx.x);
    if (j >= H) return;
    double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
    for (int i = 0; i < k; i++) {
        const int64_t sl = s_row[i];
        if (sl < 0) continue;
        const float4 p = __ldg(reinterpret_cast<const float4*>(parts + sl * H + j));
        const double wi = s_w[i];
        a0 += wi * (double) p.x;
        a1 += wi * (double) p.y;
        a2 += wi * (double) p.z;
        a3 += wi * (double) p.w;
    }
    if (shared) {
        float4 sh = *reinterpret_cast<const float4*>(shared + (int64_t) t * shared_stride + j);
        if (shared_logit) {
            const float e = (float) exp(-(double) shared_logit[t]);
            const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
            sh.x = __fmul_rn(sh.x, sig);
            sh.y = __fmul_rn(sh.y, sig);
            sh.z = __fmul_rn(sh.z, sig);
            sh.w = __fmul_rn(sh.w, sig);
        }
        if (shared_out) *reinterpret_cast<float4*>(shared_out + (int64_t) t * H + j) = sh;
        a0 += (double) sh.x;
        a1 += (double) sh.y;
        a2 += (double) sh.z;
        a3 += (double) sh.w;
    }
    *reinterpret_cast<float4*>(out + (int64_t) t * H + j) = make_float4((float) a0, (float) a1, (float) a2, (float) a3);
}

__global__ void gather_parts_kernel(const float* __restrict__ parts, const int32_t* __restrict__ slot,
                                    float* __restrict__ dst, int64_t H, int k) {
    const int ti = blockIdx.y;  // t * k + i
    const int64_t j = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= H) return;
    const int s = slot[ti];
    dst[(int64_t) ti * H + j] = s < 0 ? 0.f : parts[(int64_t) s * H + j];
}

cudaError_t launch_combine(const float* parts, const int32_t* slot, const float* w, const float* shared,
                           const float* shared_logit, float* out, float* shared_out, int64_t H, int k, int T,
                           int64_t shared_stride, cudaStream_t s) {
    const bool vec = T >= 128 && H % 4 == 0 && shared_stride % 4 == 0 && k <= kMaxK &&
                     (reinterpret_cast<uintptr_t>(parts) | reinterpret_cast<uintptr_t>(out) |
                      reinterpret_cast<uintptr_t>(shared) | reinterpret_cast<uintptr_t>(shared_out)) % 16 == 0;
    if (vec) {
        const dim3 grid((unsigned) ((H / 4 + 255) / 256), (unsigned) T);
        combine4_kernel<<<grid, 256, 0, s>>>(parts, slot, w, shared, shared_logit, out, shared_out, H, k,
                                             shared_stride);
        return cudaGetLastError();
    }
    const dim3 grid((unsigned) ((H + 255) / 256), (unsigned) T);
    combine_kernel<<<grid, 256, 0, s>>>(parts, slot, w, shared, shared_logit, out, shared_out, H, k, shared_stride);
    return cudaGetLastError();
}

cudaError_t launch_gather_parts(const float* parts, const int32_t* slot, float* dst, int64_t H, int k, int T,
                                cudaStream_t s) {
    const dim3 grid((unsigned) ((H + 255) / 256), (unsigned) (T * k));
    gather_parts_kernel<<<grid, 256, 0, s>>>(parts, slot, dst, H, k);
    return cudaGetLastError();
}

}  // namespace smoe
