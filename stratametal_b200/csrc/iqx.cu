// iqx.cu - expert rows in every block format the reference's MMVQ family takes (iq.metal:516-549, host dots
// iq_parity.cpp:125-252): Q2_0 (42), IQ2_S (22), IQ4_NL (20), IQ4_XS (23), IQ3_XXS (18), IQ3_S (21).
//
// Two users:
//   * the stage entry point smoe_iq_mmvq for the IQ4 / IQ3 formats (warp per (row, column));
//   * the "any-format" layer path of smoe_moe_forward, taken by layers with a routed or shared matrix outside
//     Q2_0 / IQ2_S (the reference's other expert packs, e.g. IQ3_S gate/up with IQ4_NL down, iq_parity.cpp:504):
//     grouped gate/up rows (gx_kernel MODE 0) -> SwiGLU + q8_1 of h (gx_swiglu_kernel) -> grouped down rows
//     (MODE 1), over the same work list and combine as the SIMT path.  Activations are the reference's q8_1
//     blocks (36 B: fp16 d, fp16 sum, 32 int8).
//
// A row against a q8_1 column is the reference's row_dot (iq_parity.cpp:275-292): partial k (32 values; IQ4_NL
// 16) goes to lane k & 31, each lane adds its partials in k order starting from 0, and the 32 lane sums meet in
// an xor butterfly 16, 8, 4, 2, 1.  A partial is (f32(d_w) * f32(d_x)) * (float) sumi with sumi an exact int32;
// the formats differ only in how the weights of a partial are decoded and how sumi is scaled (gx_decode and gx_partial below).
// Here a partial's weights are decoded once into eight int8x4 words in the activation's value order and reused
// for every token of the work entry (dp4a against each token's q words).
#include "common.cuh"
#include "kernels.cuh"
#include "q8.cuh"

namespace smoe {

__constant__ int8_t c_iq4_values[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
__device__ const uint32_t k_iq3xxs_grid_dev[256] = {
#include "iq3xxs_grid.inc"
};
__device__ const uint32_t k_iq3s_grid_dev[512] = {
#include "iq3s_grid.inc"
};

SMOE_HD int gx_block_values(int t) {
    return t == kQ2_0 ? 64 : t == kIQ4_NL ? 32 : (t == kIQ2_S || t == kIQ4_XS || t == kIQ3_XXS || t == kIQ3_S) ? 256 : 0;
}
SMOE_HD int gx_block_bytes(int t) {
    return t == kQ2_0 ? 18 : t == kIQ2_S ? 82 : t == kIQ4_NL ? 18 : t == kIQ4_XS ? 136 : t == kIQ3_XXS ? 98
         : t == kIQ3_S ? 110 : 0;
}
// partials per row of n_in values (32 values each; IQ4_NL 16)
SMOE_HD int gx_parts(int t, int n_in) { return t == kIQ4_NL ? n_in / 16 : n_in / 32; }

// The decoded weights of one partial: w[i] holds the int8 weights of the activation values 4i .. 4i + 3 of the
// partial's q8_1 block (IQ4_NL: w[0..1] values 8p .. 8p + 7, w[2..3] values 16 + 8p .. 16 + 8p + 7), the block's
// scale and the integers that scale sumi.
struct GxPart {
    uint32_t w[8];
    float d;
    int a, b;
};

__device__ __forceinline__ uint32_t gx_u16(const uint8_t* p) { return (uint32_t) p[0] | ((uint32_t) p[1] << 8); }

// 4 two-bit codes of one byte (LSB first) -> 4 bytes
__device__ __forceinline__ uint32_t gx_spread2(uint32_t b) {
    uint32_t x = (b | (b << 12)) & 0x000F000Fu;
    return (x | (x << 6)) & 0x03030303u;
}
// negate the bytes of v whose bit in the low 4 bits of `neg` is set
__device__ __forceinline__ uint32_t gx_signed(uint32_t v, uint32_t neg) {
    const uint32_t m = (((neg & 15u) * 0x00204081u) & 0x01010101u) * 0xFFu;
    return __vsub4(v ^ m, m);
}
// 4 IQ4 codes (the low or high nibbles of 4 bytes) -> their table values
__device__ __forceinline__ uint32_t gx_iq4(uint32_t q4, int shift) {
    uint32_t o = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) o |= ((uint32_t) (uint8_t) c_iq4_values[(q4 >> (8 * j + shift)) & 15u]) << (8 * j);
    return o;
}

template <int TYPE>
__device__ __forceinline__ void gx_decode(const uint8_t* __restrict__ row, int k, const uint64_t* g2,
                                          const uint32_t* g3, GxPart& P) {
    if (TYPE == kQ2_0) {  // 32 codes of half k & 1 of block k / 2; sumi = sum code q - sum q
        const uint8_t* blk = row + (size_t) (k >> 1) * 18;
        P.d = f16_to_f32((uint16_t) gx_u16(blk));
        const uint8_t* qs = blk + 2 + 8 * (k & 1);
#pragma unroll
        for (int i = 0; i < 8; i++) P.w[i] = gx_spread2(qs[i]);
    } else if (TYPE == kIQ2_S) {  // group g of block k / 8 (iq_parity.cpp:125-151)
        const uint8_t* blk = row + (size_t) (k >> 3) * 82;
        const int g = k & 7;
        P.d = f16_to_f32((uint16_t) gx_u16(blk));
        const uint32_t qh = blk[66 + g], sc = blk[74 + g];
        P.a = (int) (sc & 15u);
        P.b = (int) (sc >> 4);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t idx = (uint32_t) blk[2 + 4 * g + j] | (((qh >> (2 * j)) & 3u) << 8);
            const uint64_t e = g2[idx];
            const uint32_t sb = blk[34 + 4 * g + j];
            P.w[2 * j] = gx_signed((uint32_t) e, sb);
            P.w[2 * j + 1] = gx_signed((uint32_t) (e >> 32), sb >> 4);
        }
    } else if (TYPE == kIQ4_NL) {  // half p = k & 1 of block k / 2 (iq_parity.cpp:196-206)
        const uint8_t* blk = row + (size_t) (k >> 1) * 18;
        P.d = f16_to_f32((uint16_t) gx_u16(blk));
        const uint8_t* qs = blk + 2 + 8 * (k & 1);
        const uint32_t q0 = (uint32_t) qs[0] | ((uint32_t) qs[1] << 8) | ((uint32_t) qs[2] << 16) | ((uint32_t) qs[3] << 24);
        const uint32_t q1 = (uint32_t) qs[4] | ((uint32_t) qs[5] << 8) | ((uint32_t) qs[6] << 16) | ((uint32_t) qs[7] << 24);
        P.w[0] = gx_iq4(q0, 0);
        P.w[1] = gx_iq4(q1, 0);
        P.w[2] = gx_iq4(q0, 4);
        P.w[3] = gx_iq4(q1, 4);
    } else if (TYPE == kIQ4_XS) {  // group ib of block k / 8 (iq_parity.cpp:208-222)
        const uint8_t* blk = row + (size_t) (k >> 3) * 136;
        const int ib = k & 7;
        P.d = f16_to_f32((uint16_t) gx_u16(blk));
        const uint8_t* qs = blk + 8 + 16 * ib;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t q = (uint32_t) qs[4 * j] | ((uint32_t) qs[4 * j + 1] << 8) | ((uint32_t) qs[4 * j + 2] << 16) |
                               ((uint32_t) qs[4 * j + 3] << 24);
            P.w[j] = gx_iq4(q, 0);
            P.w[4 + j] = gx_iq4(q, 4);
        }
        const uint32_t sh = gx_u16(blk + 2);
        P.a = (int) (((blk[4 + ib / 2] >> (4 * (ib & 1))) & 15u) | (((sh >> (2 * ib)) & 3u) << 4)) - 32;
    } else if (TYPE == kIQ3_XXS) {  // group g of block k / 8 (iq_parity.cpp:153-173)
        const uint8_t* blk = row + (size_t) (k >> 3) * 98;
        const int g = k & 7;
        P.d = f16_to_f32((uint16_t) gx_u16(blk));
        const uint8_t* qs = blk + 2;
        const uint32_t w = (uint32_t) qs[64 + 4 * g] | ((uint32_t) qs[65 + 4 * g] << 8) |
                           ((uint32_t) qs[66 + 4 * g] << 16) | ((uint32_t) qs[67 + 4 * g] << 24);
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint32_t s7 = (w >> (7 * c)) & 127u;
            const uint32_t sg = s7 | ((uint32_t) (__popc(s7) & 1) << 7);  // the eighth sign bit is the parity
            P.w[2 * c] = gx_signed(g3[qs[8 * g + 2 * c]], sg);
            P.w[2 * c + 1] = gx_signed(g3[qs[8 * g + 2 * c + 1]], sg >> 4);
        }
        P.a = (int) (w >> 28);
    } else {  // IQ3_S: group g of block k / 8 (iq_parity.cpp:175-194)
        const uint8_t* blk = row + (size_t) (k >> 3) * 110;
        const int g = k & 7;
        P.d = f16_to_f32((uint16_t) gx_u16(blk));
        const uint8_t* qs = blk + 2;
        const uint32_t qh = blk[66 + g];
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint32_t i0 = qs[8 * g + 2 * c] | (((qh >> (2 * c)) & 1u) << 8);
            const uint32_t i1 = qs[8 * g + 2 * c + 1] | (((qh >> (2 * c + 1)) & 1u) << 8);
            const uint32_t sb = blk[74 + 4 * g + c];
            P.w[2 * c] = gx_signed(g3[i0], sb);
            P.w[2 * c + 1] = gx_signed(g3[i1], sb >> 4);
        }
        P.a = 1 + 2 * (int) ((blk[106 + g / 2] >> (4 * (g & 1))) & 15u);
    }
}

// The partial of decoded weights P against one q8_1 block (q: its 8 words of int8 values, dx its scale).
template <int TYPE>
__device__ __forceinline__ float gx_partial(const GxPart& P, const uint32_t (&q)[8], float dx, int k) {
    int sumi;
    if (TYPE == kQ2_0) {
        int cq = 0, sq = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            cq = __dp4a((int) P.w[i], (int) q[i], cq);
            sq = __dp4a(0x01010101, (int) q[i], sq);
        }
        sumi = cq - sq;
    } else if (TYPE == kIQ2_S) {
        int s0 = 0, s1 = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) s0 = __dp4a((int) P.w[i], (int) q[i], s0);
#pragma unroll
        for (int i = 4; i < 8; i++) s1 = __dp4a((int) P.w[i], (int) q[i], s1);
        sumi = (s0 * P.a + s1 * P.b + (s0 + s1) / 2) / 4;
    } else if (TYPE == kIQ4_NL) {
        const int p = k & 1;
        sumi = __dp4a((int) P.w[0], (int) q[2 * p], 0);
        sumi = __dp4a((int) P.w[1], (int) q[2 * p + 1], sumi);
        sumi = __dp4a((int) P.w[2], (int) q[4 + 2 * p], sumi);
        sumi = __dp4a((int) P.w[3], (int) q[5 + 2 * p], sumi);
    } else {
        sumi = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) sumi = __dp4a((int) P.w[i], (int) q[i], sumi);
        if (TYPE == kIQ4_XS || TYPE == kIQ3_S) sumi *= P.a;
        else sumi = (P.a * sumi + sumi / 2) / 2;  // IQ3_XXS
    }
    return __fmul_rn(__fmul_rn(P.d, dx), (float) sumi);
}

// q words and scale of one q8_1 block (36 B, 4-byte aligned)
__device__ __forceinline__ float gx_load_q(const uint8_t* blk, uint32_t (&q)[8]) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(blk);
#pragma unroll
    for (int i = 0; i < 8; i++) q[i] = p[1 + i];
    return f16_to_f32((uint16_t) (p[0] & 0xFFFFu));
}

// the codebooks a format reads, copied into shared memory by the whole CTA
template <int TYPE>
__device__ __forceinline__ void gx_stage_grids(uint64_t* g2, uint32_t* g3) {
    if (TYPE == kIQ2_S)
        for (int i = threadIdx.x; i < 1024; i += blockDim.x) g2[i] = k_iq2s_grid_dev[i];
    if (TYPE == kIQ3_XXS)
        for (int i = threadIdx.x; i < 256; i += blockDim.x) g3[i] = k_iq3xxs_grid_dev[i];
    if (TYPE == kIQ3_S)
        for (int i = threadIdx.x; i < 512; i += blockDim.x) g3[i] = k_iq3s_grid_dev[i];
}

// ---- the stage entry point: warp per (row, column) -------------------------------------------------------------
template <int TYPE>
__global__ void __launch_bounds__(256) gx_mmvq_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ x,
                                                      int n_in, int n_out, float* __restrict__ y, int c0) {
    __shared__ uint64_t g2[TYPE == kIQ2_S ? 1024 : 1];
    __shared__ uint32_t g3[TYPE == kIQ3_S ? 512 : TYPE == kIQ3_XXS ? 256 : 1];
    gx_stage_grids<TYPE>(g2, g3);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), c = c0 + (int) blockIdx.y;
    if (r >= n_out) return;
    const uint8_t* row = w + (size_t) r * ((size_t) (n_in / gx_block_values(TYPE)) * gx_block_bytes(TYPE));
    const uint8_t* col = x + (size_t) c * (size_t) (n_in / 32) * 36;
    const int np = gx_parts(TYPE, n_in), ppb = TYPE == kIQ4_NL ? 2 : 1;
    float acc = 0.f;
    for (int k = lane; k < np; k += 32) {
        GxPart P;
        gx_decode<TYPE>(row, k, g2, g3, P);
        uint32_t q[8];
        const float dx = gx_load_q(col + (size_t) (k / ppb) * 36, q);
        acc = __fadd_rn(acc, gx_partial<TYPE>(P, q, dx, k));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    if (lane == 0) y[(size_t) c * n_out + r] = acc;
}

bool gx_type_ok(int type) { return gx_block_values(type) != 0; }
size_t gx_row_bytes(int type, int64_t n) {
    const int v = gx_block_values(type);
    if (v == 0 || n <= 0 || n % v) return 0;
    return (size_t) (n / v) * (size_t) gx_block_bytes(type);
}

cudaError_t launch_gx_mmvq(int type, const uint8_t* w, const uint8_t* x, int n_in, int n_out, int n_col, float* y,
                           cudaStream_t s) {
    // columns in launches of at most 65535 (the grid's y limit)
    for (int c0 = 0; c0 < n_col; c0 += 65535) {
        const dim3 grid((unsigned) ((n_out + 7) / 8), (unsigned) std::min(65535, n_col - c0));
        switch (type) {
            case kQ2_0: gx_mmvq_kernel<kQ2_0><<<grid, 256, 0, s>>>(w, x, n_in, n_out, y, c0); break;
            case kIQ2_S: gx_mmvq_kernel<kIQ2_S><<<grid, 256, 0, s>>>(w, x, n_in, n_out, y, c0); break;
            case kIQ4_NL: gx_mmvq_kernel<kIQ4_NL><<<grid, 256, 0, s>>>(w, x, n_in, n_out, y, c0); break;
            case kIQ4_XS: gx_mmvq_kernel<kIQ4_XS><<<grid, 256, 0, s>>>(w, x, n_in, n_out, y, c0); break;
            case kIQ3_XXS: gx_mmvq_kernel<kIQ3_XXS><<<grid, 256, 0, s>>>(w, x, n_in, n_out, y, c0); break;
            case kIQ3_S: gx_mmvq_kernel<kIQ3_S><<<grid, 256, 0, s>>>(w, x, n_in, n_out, y, c0); break;
            default: return cudaErrorInvalidValue;
        }
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// ---- the any-format layer path ------------------------------------------------------------------------------
constexpr int kGxRows = 64;       // rows of one matrix per item
constexpr int kGxThreads = 256;   // 8 warps, each 8 rows of the item

struct GxArgs {
    Matrix m0, m1;          // gate and up (MODE 0), down (MODE 1, m1 unused)
    Work w;
    const uint8_t* act;     // q8_1 rows: tokens of x (MODE 0) or slots of h (MODE 1), n_in / 32 blocks each
    float* y;               // MODE 0: gu[slot][gate n_rows | up n_rows]; MODE 1: parts[slot][n_rows]
    int n_in, n_rows;
    int shared_only;        // 1: the shared expert's slots (its own matrices), 0: the routed work list
};

template <int TYPE, int MODE>
__global__ void __launch_bounds__(kGxThreads) gx_kernel(GxArgs a) {
    extern __shared__ __align__(16) uint8_t gx_sm[];
    uint64_t* g2 = reinterpret_cast<uint64_t*>(gx_sm);                                   // [1024] (IQ2_S)
    uint32_t* g3 = reinterpret_cast<uint32_t*>(gx_sm + (TYPE == kIQ2_S ? 8192 : 0));    // [512] (IQ3)
    uint8_t* sx = gx_sm + (TYPE == kIQ2_S ? 8192 : 0) + (TYPE == kIQ3_S || TYPE == kIQ3_XXS ? 2048 : 0);
    gx_stage_grids<TYPE>(g2, g3);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = a.n_in / 32, np = gx_parts(TYPE, a.n_in), ppb = TYPE == kIQ4_NL ? 2 : 1;
    const Work& w = a.w;
    const int n_entries = a.shared_only ? (w.shared_slots + kChunk - 1) / kChunk : w.sched.count[0];
    const int tiles = (a.n_rows + kGxRows - 1) / kGxRows;
    const size_t rb = (size_t) (a.n_in / gx_block_values(TYPE)) * gx_block_bytes(TYPE);
    for (int item = blockIdx.x; item < n_entries * tiles; item += gridDim.x) {
        const int c = item / tiles, tile = item % tiles;
        int e, beg, n;
        if (a.shared_only) {
            e = 0;
            beg = w.shared_base + c * kChunk;
            n = min(kChunk, w.shared_slots - c * kChunk);
        } else {
            e = w.sched.e[c];
            beg = w.sched.beg[c];
            n = w.sched.n[c];
        }
        // the entry's activation rows into shared memory: [t][nb][36]
        __syncthreads();
        const int words = 9 * nb;
        for (int i = threadIdx.x; i < n * words; i += kGxThreads) {
            const int t = i / words, o = i % words;
            const int slot = beg + t;
            const int src = MODE == 1 ? slot : a.shared_only ? slot - w.shared_base : w.slot_token[slot];
            reinterpret_cast<uint32_t*>(sx)[i] = reinterpret_cast<const uint32_t*>(a.act + (size_t) src * nb * 36)[o];
        }
        __syncthreads();
        for (int rr = warp; rr < kGxRows; rr += kGxThreads / 32) {
            const int r = tile * kGxRows + rr;
            if (r >= a.n_rows) break;
#pragma unroll
            for (int mat = 0; mat < (MODE == 0 ? 2 : 1); mat++) {
                const Matrix& m = mat ? a.m1 : a.m0;
                const uint8_t* row = m.base + (int64_t) e * m.expert_stride + (size_t) r * rb;
                float acc[kChunk];
#pragma unroll
                for (int t = 0; t < kChunk; t++) acc[t] = 0.f;
                for (int k = lane; k < np; k += 32) {
                    GxPart P;
                    gx_decode<TYPE>(row, k, g2, g3, P);
#pragma unroll
                    for (int t = 0; t < kChunk; t++) {
                        if (t >= n) break;  // uniform across the warp
                        uint32_t q[8];
                        const float dx = gx_load_q(sx + ((size_t) t * nb + k / ppb) * 36, q);
                        acc[t] = __fadd_rn(acc[t], gx_partial<TYPE>(P, q, dx, k));
                    }
                }
#pragma unroll
                for (int t = 0; t < kChunk; t++) {
                    if (t >= n) break;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) acc[t] = __fadd_rn(acc[t], __shfl_xor_sync(0xffffffffu, acc[t], o));
                }
                if (lane < n) {
                    float v = acc[0];
#pragma unroll
                    for (int t = 1; t < kChunk; t++)
                        if (lane == t) v = acc[t];
                    const int slot = beg + lane;
                    if (MODE == 0) a.y[(size_t) slot * 2 * a.n_rows + (size_t) mat * a.n_rows + r] = v;
                    else a.y[(size_t) slot * a.n_rows + r] = v;
                }
            }
        }
    }
}

// h[slot] = q8_1(silu(gate) * up) per 32-value block (iq_swiglu_q8, iq.mm:201-210), gu rows [gate F | up F].
__global__ void __launch_bounds__(256) gx_swiglu_kernel(const float* __restrict__ gu, uint8_t* __restrict__ h,
                                                        int64_t rows, int F) {
    const int lane = threadIdx.x & 31;
    const int64_t nbk = (int64_t) F / 32, total = rows * nbk;
    for (int64_t b = (int64_t) blockIdx.x * 8 + (threadIdx.x >> 5); b < total; b += (int64_t) gridDim.x * 8) {
        const int64_t r = b / nbk, j = b % nbk;
        const float* g = gu + r * 2 * F + j * 32;
        quant_q8_1_warp(silu_mul(g[lane], g[F + lane]), h + b * 36, lane);
    }
}

template <int MODE>
static cudaError_t gx_launch(int type, const GxArgs& a, cudaStream_t s) {
    const size_t smem = (type == kIQ2_S ? 8192 : 0) + (type == kIQ3_S || type == kIQ3_XXS ? 2048 : 0) +
                        (size_t) kChunk * (a.n_in / 32) * 36;
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const int grid = nsm * 4;
#define SMOE_GX(T)                                                                                              \
    case T: {                                                                                                   \
        cudaError_t e = cudaFuncSetAttribute(gx_kernel<T, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                             (int) smem);                                                      \
        if (e != cudaSuccess) return e;                                                                         \
        gx_kernel<T, MODE><<<grid, kGxThreads, smem, s>>>(a);                                                   \
        break;                                                                                                  \
    }
    switch (type) {
        SMOE_GX(kQ2_0)
        SMOE_GX(kIQ2_S)
        SMOE_GX(kIQ4_NL)
        SMOE_GX(kIQ4_XS)
        SMOE_GX(kIQ3_XXS)
        SMOE_GX(kIQ3_S)
        default: return cudaErrorInvalidValue;
    }
#undef SMOE_GX
    return cudaGetLastError();
}

cudaError_t launch_gx_gate_up(Matrix gate, Matrix up, Work w, int shared_only, const uint8_t* xq, float* gu,
                              int n_embd, int n_ff, cudaStream_t s) {
    GxArgs a{};
    a.m0 = gate;
    a.m1 = up;
    a.w = w;
    a.act = xq;
    a.y = gu;
    a.n_in = n_embd;
    a.n_rows = n_ff;
    a.shared_only = shared_only;
    return gx_launch<0>(gate.type, a, s);
}

cudaError_t launch_gx_down(Matrix down, Work w, int shared_only, const uint8_t* hq, float* y, int n_ff, int n_embd,
                           cudaStream_t s) {
    GxArgs a{};
    a.m0 = a.m1 = down;
    a.w = w;
    a.act = hq;
    a.y = y;
    a.n_in = n_ff;
    a.n_rows = n_embd;
    a.shared_only = shared_only;
    return gx_launch<1>(down.type, a, s);
}

cudaError_t launch_gx_swiglu(const float* gu, uint8_t* h, int64_t rows, int n_ff, cudaStream_t s) {
    const int64_t blocks = (rows * (n_ff / 32) + 7) / 8;
    gx_swiglu_kernel<<<(unsigned) std::min<int64_t>(blocks, 148 * 16), 256, 0, s>>>(gu, h, rows, n_ff);
    return cudaGetLastError();
}

}  // namespace smoe
