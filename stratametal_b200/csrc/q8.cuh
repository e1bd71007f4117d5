// q8.cuh - the q8_1 activation rule and SwiGLU, shared by the router and the expert kernels.
#pragma once

#include "common.cuh"

namespace smoe {

// ------------------------------------------------------------------------------------------------
// q8_1 of one 32-value block by one warp (iq.metal:597-627; host quant_host_block iq_parity.cpp:350-382):
// the amax and the float sum meet in an xor butterfly (offsets 16..1) in the host reference's order.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void quant_q8_1_warp(float xi, uint8_t* __restrict__ yb, int lane) {
    float amax = fabsf(xi), sum = xi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    }
    float d = __fdiv_rn(amax, 127.f);
    if (fabsf(d) > 65504.f) d = copysignf(65504.f, d);
    int q = 0;
    if (amax != 0.f) {
        float r = roundf(__fdiv_rn(xi, d));
        r = fminf(fmaxf(r, -127.f), 127.f);
        q = (int) r;
    }
    yb[4 + lane] = (uint8_t) (int8_t) q;
    if (lane == 0) {
        const float sc = fabsf(sum) > 65504.f ? copysignf(65504.f, sum) : sum;
        const uint16_t dh = f16_bits(d), sh = f16_bits(sc);
        yb[0] = (uint8_t) dh;
        yb[1] = (uint8_t) (dh >> 8);
        yb[2] = (uint8_t) sh;
        yb[3] = (uint8_t) (sh >> 8);
    }
}

// The same q8_1 rule, written in the expert kernels' layout (KAct): 8 words (permuted for Q2_0 weights:
// byte b of word j of half h = value 16h + 4b + j; natural order otherwise), the stored scale read back as the
// dot reads it (f32 of the fp16 d) and 0x4B400000 - (the sum of the 32 q): the bits of 1.5 * 2^23 - sum q, the
// seed of the exact integer-to-float step of the Q2_0 dot (see expert.cu).
__device__ __forceinline__ void quant_ka_warp(float xi, uint8_t* __restrict__ blk48, int lane, bool q2_layout) {
    float amax = fabsf(xi);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float d = __fdiv_rn(amax, 127.f);
    if (fabsf(d) > 65504.f) d = copysignf(65504.f, d);
    int q = 0;
    if (amax != 0.f) {
        float r = roundf(__fdiv_rn(xi, d));
        r = fminf(fmaxf(r, -127.f), 127.f);
        q = (int) r;
    }
    int qs = q;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
    const int L = lane & 7;
    const int src0 = q2_layout ? 16 * (L >> 2) + (L & 3) : 4 * L;
    const int stride = q2_layout ? 4 : 1;
    uint32_t word = 0;
#pragma unroll
    for (int b = 0; b < 4; b++) {
        const int qb = __shfl_sync(0xffffffffu, q, src0 + b * stride);
        word |= ((uint32_t) qb & 0xFFu) << (8 * b);
    }
    if (lane < 8) reinterpret_cast<uint32_t*>(blk48)[lane] = word;
    if (lane == 8) reinterpret_cast<float*>(blk48)[8] = f16_to_f32(f16_bits(d));
    if (lane == 9) reinterpret_cast<int*>(blk48)[9] = 0x4B400000 - qs;
}

// quant_ka_warp for N blocks at once (blocks whose bit in `valid` is clear are skipped): the same arithmetic per
// block, with the N dependency chains interleaved so their shuffle and division latencies overlap.
template <int N>
__device__ __forceinline__ void quant_ka_warp_n(const float (&xi)[N], uint8_t* const (&blk)[N], unsigned valid, int lane,
                                                bool q2_layout) {
    float amax[N], d[N];
    int q[N], qs[N];
#pragma unroll
    for (int i = 0; i < N; i++) amax[i] = fabsf(xi[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < N; i++) amax[i] = fmaxf(amax[i], __shfl_xor_sync(0xffffffffu, amax[i], o));
#pragma unroll
    for (int i = 0; i < N; i++) {
        d[i] = __fdiv_rn(amax[i], 127.f);
        if (fabsf(d[i]) > 65504.f) d[i] = copysignf(65504.f, d[i]);
        q[i] = 0;
        if (amax[i] != 0.f) {
            float r = roundf(__fdiv_rn(xi[i], d[i]));
            r = fminf(fmaxf(r, -127.f), 127.f);
            q[i] = (int) r;
        }
        qs[i] = q[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < N; i++) qs[i] += __shfl_xor_sync(0xffffffffu, qs[i], o);
    const int L = lane & 7;
    const int src0 = q2_layout ? 16 * (L >> 2) + (L & 3) : 4 * L;
    const int stride = q2_layout ? 4 : 1;
#pragma unroll
    for (int i = 0; i < N; i++) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const int qb = __shfl_sync(0xffffffffu, q[i], src0 + b * stride);
            word |= ((uint32_t) qb & 0xFFu) << (8 * b);
        }
        if (!((valid >> i) & 1u)) continue;
        if (lane < 8) reinterpret_cast<uint32_t*>(blk[i])[lane] = word;
        if (lane == 8) reinterpret_cast<float*>(blk[i])[8] = f16_to_f32(f16_bits(d[i]));
        if (lane == 9) reinterpret_cast<int*>(blk[i])[9] = 0x4B400000 - qs[i];
    }
}

// silu(g) * u (iq.metal:630-663).  exp is taken in fp64 and rounded to f32: that is the correctly rounded
// expf, which the host reference's libm expf returns on all but a vanishing fraction of inputs.
__device__ __forceinline__ float silu_mul(float g, float u) {
    const float e = (float) exp(-(double) g);
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, e)), u);
}

}  // namespace smoe
