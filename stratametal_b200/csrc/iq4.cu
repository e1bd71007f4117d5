// iq4.cu - the IQ4_NL and IQ4_XS row dots of the stage entry point smoe_iq_mmvq (the reference's next expert
// formats, iq.metal:516-547; host transcription iq_parity.cpp:106-115, 196-222, geometry :256-263).  The layer
// path does not take these formats yet; this kernel serves the stage-level contract only.
//
// A row against a q8_1 column is the reference's row_dot (iq_parity.cpp:275-292): partial k of the row goes to
// lane k & 31, each lane adds its partials in k order starting from 0, and the 32 lane sums meet in an xor
// butterfly 16, 8, 4, 2, 1.  A partial is (f32(d_w) * f32(d_x)) * (float) sumi with sumi an exact int32:
//   IQ4_NL (18 B / 32 values: fp16 d, qs[16]; byte i holds value i in its low nibble, value i + 16 in its high):
//           two partials per block, partial p over qs bytes 8p .. 8p + 7;
//   IQ4_XS (136 B / 256 values: fp16 d, scales_h u16, scales_l[4], qs[128]): eight 32-value partials ib, qs bytes
//           16 ib .. 16 ib + 15 as above, sumi times (ls - 32) with ls = 4 bits of scales_l | 2 of scales_h << 4.
// Codes index the format's 16-entry non-linear table.  One warp per (row, column).
#include "common.cuh"
#include "kernels.cuh"

namespace smoe {

__constant__ int8_t c_iq4_values[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

__device__ __forceinline__ float iq4_f16(const uint8_t* p) {
    return __half2float(__ushort_as_half((unsigned short) (p[0] | (p[1] << 8))));
}

// sumi of 16 code bytes against the 32 q of one q8_1 block (low nibble -> q[i], high nibble -> q[i + 16]).
__device__ __forceinline__ int iq4_sumi(const uint8_t* qs, const int8_t* q, int i0, int n) {
    int s = 0;
    for (int i = i0; i < i0 + n; i++) {
        s += (int) c_iq4_values[qs[i - i0] & 15] * (int) q[i];
        s += (int) c_iq4_values[qs[i - i0] >> 4] * (int) q[i + 16];
    }
    return s;
}

template <int TYPE>
__global__ void __launch_bounds__(256) iq4_mmvq_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ x,
                                                       int n_in, int n_out, float* __restrict__ y, int c0) {
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), c = c0 + (int) blockIdx.y;
    if (r >= n_out) return;
    const size_t rb = TYPE == kIQ4_NL ? (size_t) (n_in / 32) * 18 : (size_t) (n_in / 256) * 136;
    const uint8_t* row = w + (size_t) r * rb;
    const uint8_t* col = x + (size_t) c * (size_t) (n_in / 32) * 36;
    const int npart = TYPE == kIQ4_NL ? n_in / 16 : n_in / 32;
    float acc = 0.f;
    for (int k = lane; k < npart; k += 32) {
        float d;
        int sumi;
        if (TYPE == kIQ4_NL) {
            const uint8_t* blk = row + (size_t) (k / 2) * 18;
            const uint8_t* xb = col + (size_t) (k / 2) * 36;
            const int p = k % 2;
            sumi = iq4_sumi(blk + 2 + 8 * p, reinterpret_cast<const int8_t*>(xb + 4), 8 * p, 8);
            d = __fmul_rn(iq4_f16(blk), iq4_f16(xb));
        } else {
            const uint8_t* blk = row + (size_t) (k / 8) * 136;
            const uint8_t* xb = col + (size_t) k * 36;
            const int ib = k % 8;
            sumi = iq4_sumi(blk + 8 + 16 * ib, reinterpret_cast<const int8_t*>(xb + 4), 0, 16);
            const int sh = blk[2] | (blk[3] << 8);
            const int ls = ((blk[4 + ib / 2] >> (4 * (ib % 2))) & 15) | (((sh >> (2 * ib)) & 3) << 4);
            sumi *= ls - 32;
            d = __fmul_rn(iq4_f16(blk), iq4_f16(xb));
        }
        acc = __fadd_rn(acc, __fmul_rn(d, (float) sumi));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    if (lane == 0) y[(size_t) c * n_out + r] = acc;
}

cudaError_t launch_iq4_mmvq(int type, const uint8_t* w, const uint8_t* x, int n_in, int n_out, int n_col,
                            float* y, cudaStream_t s) {
    if (type != kIQ4_NL && type != kIQ4_XS) return cudaErrorInvalidValue;
    // columns in launches of at most 65535 (the grid's y limit)
    for (int c0 = 0; c0 < n_col; c0 += 65535) {
        const dim3 grid((unsigned) ((n_out + 7) / 8), (unsigned) min(65535, n_col - c0));
        if (type == kIQ4_NL) iq4_mmvq_kernel<kIQ4_NL><<<grid, 256, 0, s>>>(w, x, n_in, n_out, y, c0);
        else iq4_mmvq_kernel<kIQ4_XS><<<grid, 256, 0, s>>>(w, x, n_in, n_out, y, c0);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace smoe
