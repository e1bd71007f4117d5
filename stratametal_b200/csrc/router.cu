// router.cu - the MoE router on sm_100a: bf16 GEMV with fp64 accumulation, then softmax / top-k /
// renormalise, fused with the q8_1 quantization of the token (rows a1-a4 of the block).
//
// Numerics (what makes the expert ids exact against the host reference):
//   * the activation is rounded to bf16 with round-to-nearest-even (bf16_bits.hpp:37-47);
//   * each product bf16 x bf16 is exact in fp64 and the 2048-term sum is accumulated in fp64, then rounded
//     once to f32 - the host oracle's bf16_dot (pack_parity.cpp:3795-3799).  The sums of these products span
//     far fewer than 53 bits on this data, so the order of the fp64 additions does not change the result;
//   * the softmax is computed in fp64 (route_ref, pack_parity.cpp:5144-5165), ranked by probability with
//     the lower index on a tie; the weights are (float) p, then (float)((double) w / max(sum, 2^-14)) with
//     the sum taken in rank order.
#include "common.cuh"
#include "kernels.cuh"
#include "q8.cuh"

#include <algorithm>
#include <cfloat>

namespace smoe {

// ------------------------------------------------------------------------------------------------
// a1 + a2: logits.  A CTA owns RPW rows per warp (8 warps) and TT tokens staged in shared memory as bf16
// bits.  Per 256-value chunk a lane converts its 8 weights of each row to fp64 once and applies them to every
// staged token, so each DFMA needs one converted activation and the weight stream is read once per CTA.
// Rows [0, n_out) come from `w`; when `extra` is set, row n_out is that vector (the shared-expert gate
// ffn_gate_inp_shexp) and its result goes to y_extra[t].
// ------------------------------------------------------------------------------------------------
template <bool kF32In, int RPW>
__global__ void __launch_bounds__(256) bf16_gemv_kernel(const void* __restrict__ xin, const uint16_t* __restrict__ w,
                                                        const uint16_t* __restrict__ extra, float* __restrict__ y,
                                                        float* __restrict__ y_extra, int T, int H, int n_out) {
    constexpr int TT = kRouterTokTile;
    extern __shared__ __align__(16) uint16_t xs[];  // [TT][H]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int o0 = (blockIdx.x * 8 + warp) * RPW;
    const int t0 = blockIdx.y * TT;
    const int nt = min(TT, T - t0);
    // stage: 4 floats (or 8 bf16) per load, several loads in flight per thread
    if (kF32In) {
        const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(xin) + (size_t) t0 * H);
        const int n4 = nt * H / 4;
        for (int i = threadIdx.x; i < n4; i += 4 * blockDim.x) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (i + u * blockDim.x < n4) v[u] = __ldg(src + i + u * blockDim.x);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int j = i + u * blockDim.x;
                if (j < n4) {
                    uint2 b;
                    b.x = (uint32_t) bf16_bits(v[u].x) | ((uint32_t) bf16_bits(v[u].y) << 16);
                    b.y = (uint32_t) bf16_bits(v[u].z) | ((uint32_t) bf16_bits(v[u].w) << 16);
                    reinterpret_cast<uint2*>(xs)[j] = b;
                }
            }
        }
    } else {
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(xin) + (size_t) t0 * H);
        for (int i = threadIdx.x; i < nt * H / 8; i += blockDim.x) reinterpret_cast<uint4*>(xs)[i] = __ldg(src + i);
    }
    __syncthreads();
    const int n_rows = n_out + (extra ? 1 : 0);
    if (o0 >= n_rows) return;
    const uint16_t* rowp[RPW];
#pragma unroll
    for (int r = 0; r < RPW; r++) {
        const int o = min(o0 + r, n_rows - 1);
        rowp[r] = o < n_out ? w + (size_t) o * H : extra;
    }
    double acc[RPW][TT];
#pragma unroll
    for (int r = 0; r < RPW; r++)
#pragma unroll
        for (int t = 0; t < TT; t++) acc[r][t] = 0.0;
    for (int c = lane * 8; c < H; c += 256) {
        double wd[RPW][8];
#pragma unroll
        for (int r = 0; r < RPW; r++) {
            const uint4 wv = __ldg(reinterpret_cast<const uint4*>(rowp[r] + c));
            const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int q = 0; q < 4; q++) {
                wd[r][2 * q] = (double) __uint_as_float(wu[q] << 16);
                wd[r][2 * q + 1] = (double) __uint_as_float(wu[q] & 0xFFFF0000u);
            }
        }
#pragma unroll
        for (int t = 0; t < TT; t++) {
            if (t < nt) {
                const uint4 xv = *reinterpret_cast<const uint4*>(xs + t * H + c);
                const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w};
                double xd[8];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    xd[2 * q] = (double) __uint_as_float(xu[q] << 16);
                    xd[2 * q + 1] = (double) __uint_as_float(xu[q] & 0xFFFF0000u);
                }
#pragma unroll
                for (int r = 0; r < RPW; r++)
#pragma unroll
                    for (int q = 0; q < 8; q++) acc[r][t] = fma(xd[q], wd[r][q], acc[r][t]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < RPW; r++) {
        const int o = o0 + r;
#pragma unroll
        for (int t = 0; t < TT; t++) {
            if (t < nt) {
                double v = acc[r][t];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                if (lane == 0 && o < n_rows) {
                    if (o < n_out) y[(size_t) (t0 + t) * n_out + o] = (float) v;
                    else y_extra[t0 + t] = (float) v;
                }
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------
// a1 + a2 for many tokens: the same products as tiles of a GEMM on the fp64 tensor path
// (mma.sync.m8n8k4.f64: exact products, fp64 sums, like the DFMA form).  A CTA computes 64 rows x 128 tokens
// over K chunks of 32, staged once in shared memory already converted to fp64 (weights bf16 -> f64,
// activations f32 -> bf16 RNE -> f64); each of the 8 warps owns a 32-row x 32-token tile, 4 x 4 MMA tiles of
// 8 x 8.  The rows of the staged tiles are padded by 8 doubles so a fragment load touches both bank halves.
// The next chunk is loaded into registers while the current one is multiplied.
// ------------------------------------------------------------------------------------------------
constexpr int kRgRows = 64, kRgToks = 128, kRgK = 32, kRgPad = 8;

__device__ __forceinline__ void dmma_8x8x4(double (&d)[2], double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(d[0]), "+d"(d[1])
                 : "d"(a), "d"(b));
}

// Split-K (few tokens): blockIdx.z takes K range [z H / S, (z + 1) H / S) and writes its fp64 partial sums to
// part[z][t][o]; router_reduce_kernel adds the S partials in z order.  The fp64 sums are exact on this data, so
// the split changes nothing in the result.
__global__ void __launch_bounds__(256) router_gemm_kernel(const float* __restrict__ x, const uint16_t* __restrict__ w,
                                                          const uint16_t* __restrict__ extra, float* __restrict__ y,
                                                          float* __restrict__ y_extra, int T, int H, int n_out,
                                                          double* __restrict__ part) {
    extern __shared__ __align__(16) double rg_smem[];
    double (*ws)[kRgRows + kRgPad] = reinterpret_cast<double (*)[kRgRows + kRgPad]>(rg_smem);
    double (*xs)[kRgToks + kRgPad] = reinterpret_cast<double (*)[kRgToks + kRgPad]>(rg_smem + kRgK * (kRgRows + kRgPad));
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int o0 = blockIdx.x * kRgRows, t0 = blockIdx.y * kRgToks;
    const int n_rows = n_out + (extra ? 1 : 0);
    // loaders: weights, thread -> row tid % 64, k segment (tid / 64) * 8; activations, thread -> token tid % 128,
    // k segment (tid / 128) * 16
    const int wr = tid & 63, wk = (tid >> 6) * 8;
    const int wo = min(o0 + wr, n_rows - 1);
    const uint16_t* wrow = (wo < n_out ? w + (size_t) wo * H : extra) + wk;
    const int xr = tid & 127, xk = (tid >> 7) * 16;
    const float* xrow = x + (size_t) min(t0 + xr, T - 1) * H + xk;
    const int S = gridDim.z;
    const int k_len = H / S, k_beg = (int) blockIdx.z * k_len;
    uint4 wreg;
    float4 xreg[4];
    auto load = [&](int kc) {
        wreg = __ldg(reinterpret_cast<const uint4*>(wrow + kc));
#pragma unroll
        for (int q = 0; q < 4; q++) xreg[q] = __ldg(reinterpret_cast<const float4*>(xrow + kc) + q);
    };
    auto stage = [&]() {
        const uint32_t wu[4] = {wreg.x, wreg.y, wreg.z, wreg.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            ws[wk + 2 * q][wr] = (double) __uint_as_float(wu[q] << 16);
            ws[wk + 2 * q + 1][wr] = (double) __uint_as_float(wu[q] & 0xFFFF0000u);
        }
#pragma unroll
        for (int q = 0; q < 4; q++) {
            xs[xk + 4 * q + 0][xr] = (double) bf16_round(xreg[q].x);
            xs[xk + 4 * q + 1][xr] = (double) bf16_round(xreg[q].y);
            xs[xk + 4 * q + 2][xr] = (double) bf16_round(xreg[q].z);
            xs[xk + 4 * q + 3][xr] = (double) bf16_round(xreg[q].w);
        }
    };
    // warp tile: rows 32 (warp & 1) .., tokens 32 (warp >> 1) ..; fragment roles gid = lane / 4, tig = lane % 4
    const int wro = 32 * (warp & 1), wto = 32 * (warp >> 1);
    const int gid = lane >> 2, tig = lane & 3;
    double acc[4][4][2];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j][0] = acc[i][j][1] = 0.0;
    const bool active = t0 + wto < T;  // warps whose tokens are all padding skip the products
    load(k_beg);
    for (int kc = k_beg; kc < k_beg + k_len; kc += kRgK) {
        __syncthreads();  // the previous chunk is consumed
        stage();
        __syncthreads();
        if (kc + kRgK < k_beg + k_len) load(kc + kRgK);
        if (!active) continue;
#pragma unroll
        for (int k = 0; k < kRgK; k += 4) {
            double a[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = ws[k + tig][wro + 8 * i + gid];   // A[row gid][k tig]
#pragma unroll
            for (int j = 0; j < 4; j++) bv[j] = xs[k + tig][wto + 8 * j + gid];  // B[k tig][token gid]
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) dmma_8x8x4(acc[i][j], a[i], bv[j]);
        }
    }
    // D[row gid][token 2 tig + c]
    if (S == 1) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int o = o0 + wro + 8 * i + gid;
            if (o >= n_rows) continue;
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const int t = t0 + wto + 8 * j + 2 * tig + c;
                    if (t >= T) continue;
                    if (o < n_out) y[(size_t) t * n_out + o] = (float) acc[i][j][c];
                    else y_extra[t] = (float) acc[i][j][c];
                }
        }
        return;
    }
    double* my = part + (size_t) blockIdx.z * T * n_rows;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int o = o0 + wro + 8 * i + gid;
        if (o >= n_rows) continue;
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int c = 0; c < 2; c++) {
                const int t = t0 + wto + 8 * j + 2 * tig + c;
                if (t < T) my[(size_t) t * n_rows + o] = acc[i][j][c];
            }
    }
}

// y[t][o] = (float) sum_z part[z][t][o], z in order (independent loads, then the adds).
__global__ void __launch_bounds__(256) router_reduce_kernel(const double* __restrict__ part, int S, int T, int n_rows,
                                                            int n_out, float* __restrict__ y,
                                                            float* __restrict__ y_extra) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * n_rows) return;
    double v[32];
#pragma unroll
    for (int z = 0; z < 32; z++)
        if (z < S) v[z] = __ldg(part + (size_t) z * T * n_rows + i);
    double acc = 0.0;
#pragma unroll
    for (int z = 0; z < 32; z++)
        if (z < S) acc += v[z];
    const int t = i / n_rows, o = i % n_rows;
    if (o < n_out) y[(size_t) t * n_out + o] = (float) acc;
    else y_extra[t] = (float) acc;
}

// K splits of the few-token router GEMM: enough CTAs for the SMs, K a multiple of the 32-wide chunk.
int router_splits(int T, int n_rows, int H) {
    if (T < 2 || T > kRouterGemmMinTokens || H % kRgK) return 1;
    const int tiles = ((n_rows + kRgRows - 1) / kRgRows) * ((T + kRgToks - 1) / kRgToks);
    int S = 1;
    while (S < 32 && 2 * S * tiles <= 160 && (H / kRgK) % (2 * S) == 0) S *= 2;
    return S;
}

size_t router_split_bytes(int T, int n_rows, int H) {
    const int S = router_splits(T, n_rows, H);
    if (S == 1) return 0;
    return ((size_t) S * T * n_rows * 8 + 255) & ~(size_t) 255;
}

constexpr size_t kRgSmem = (size_t) kRgK * (kRgRows + kRgPad + kRgToks + kRgPad) * sizeof(double);

__global__ void quant_q8_1_kernel(const float* __restrict__ x, uint8_t* __restrict__ y, int64_t n_blocks) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t b = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n_blocks; b += warps)
        quant_q8_1_warp(x[b * 32 + lane], y + b * kQ8Block, lane);
}

__global__ void swiglu_q8_kernel(const float* __restrict__ g, const float* __restrict__ u, uint8_t* __restrict__ y,
                                 int64_t n_blocks) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t b = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n_blocks; b += warps)
        quant_q8_1_warp(silu_mul(g[b * 32 + lane], u[b * 32 + lane]), y + b * kQ8Block, lane);
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ x, uint16_t* __restrict__ y, int64_t n) {
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x)
        y[i] = bf16_bits(x[i]);
}

// ------------------------------------------------------------------------------------------------
// a3 (+ a4): one warp per token, 1 to 8 tokens per CTA (few tokens: one per CTA, so that each warp's fp64 exps and
// selection rounds have an SM's pipes to themselves).  Lane l holds experts l, l + 32, ... (E <= 1024).
// p_e = exp(l_e - max) in fp64; the ranking is by p_e descending with the lower index on a tie (the order of
// the normalised probabilities: one positive divisor for all); the k chosen are then normalised exactly as
// route_ref does: w = (float)(p / sum), chosen = sum of those quotients in rank order, clamped at 2^-14,
// final (float)((double) w / chosen).  The CTAs past the routing ones write the q8_1 image of x.
// ------------------------------------------------------------------------------------------------

constexpr int kTopkWarps = 8;

__host__ __device__ constexpr int topk_tokens_per_cta(int T) { return T <= 148 ? 1 : T <= 592 ? 4 : kTopkWarps; }

// The routing of one token by one warp (route_ref, pack_parity.cpp:5144-5165): ids[0..k) and the renormalised
// weights wout[0..k) (global or shared memory).  p_e = exp(l_e - max) in fp64 and its sum (per-lane partial sums,
// then the xor butterfly).  The ranking by p descending with the lower index on a tie is the ranking by the f32
// logit descending with the same tie rule: exp is increasing, equal logits give equal p, and distinct f32
// logits (at least one f32 ulp apart) give distinct fp64 p in the same order.  So the selection rounds compare
// floats; p is evaluated again, by the same expression, for the k chosen.  Then w = (float)(p / sum), chosen =
// the sum of those quotients in rank order, clamped at 2^-14, and the final weight (float)((double) w / chosen).
//
// The selection orders by an unsigned key that sorts as the float does (-0 and +0 equal: the key of v + 0); a NaN
// logit gets key 0 and is never chosen, nor is an expert past E.  Each round is two warp reductions: the largest
// key, then the lowest index among the lanes that hold it; the lane that gave the winner offers its next best.
__device__ __forceinline__ uint32_t route_key(float v) {
    const uint32_t b = __float_as_uint(v + 0.0f);
    return v != v ? 0u : (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

template <int PER_LANE>
__device__ __forceinline__ void route_warp(const float* __restrict__ l, int E, int k, int32_t* ids, float* wout,
                                           int lane) {
    float lv[PER_LANE];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < PER_LANE; j++) {
        const int e = lane + 32 * j;
        lv[j] = e < E ? l[e] : -INFINITY;
        mx = fmaxf(mx, lv[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    double part = 0.0;
#pragma unroll
    for (int j = 0; j < PER_LANE; j++)
        if (lane + 32 * j < E) part += exp((double) lv[j] - (double) mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    const double sum = part;
    // selection: each lane offers its best untaken key (lowest index first among equal keys); k rounds
    uint32_t kv[PER_LANE];
#pragma unroll
    for (int j = 0; j < PER_LANE; j++) kv[j] = lane + 32 * j < E ? route_key(lv[j]) : 0u;
    uint32_t taken = 0, bk = 0;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < PER_LANE; j++)
        if (kv[j] > bk) { bk = kv[j]; bi = lane + 32 * j; }
    int id0 = 0, id1 = 0;  // ranks lane and 32 + lane (k <= 64)
    for (int i = 0; i < k; i++) {
        const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
        const int ix = __reduce_min_sync(0xffffffffu, bk == mk && bk != 0u ? bi : 0x7fffffff);
        if (lane == (i & 31)) {
            if (i < 32) id0 = ix;
            else id1 = ix;
        }
        if (ix != 0x7fffffff && (ix & 31) == lane) {
            taken |= 1u << (ix >> 5);
            bk = 0;
            bi = 0x7fffffff;
#pragma unroll
            for (int j = 0; j < PER_LANE; j++)
                if (!((taken >> j) & 1u) && kv[j] > bk) { bk = kv[j]; bi = lane + 32 * j; }
        }
    }
    // weights of the chosen, the chosen sum in rank order
    const double pn0 = lane < k ? exp((double) l[id0] - (double) mx) / sum : 0.0;
    const double pn1 = 32 + lane < k ? exp((double) l[id1] - (double) mx) / sum : 0.0;
    double chosen = 0.0;
    for (int i = 0; i < k; i++) chosen += __shfl_sync(0xffffffffu, i < 32 ? pn0 : pn1, i & 31);
    chosen = fmax(chosen, 6.103515625e-05);
    if (lane < k) {
        ids[lane] = id0;
        wout[lane] = (float) ((double) (float) pn0 / chosen);
    }
    if (32 + lane < k) {
        ids[32 + lane] = id1;
        wout[32 + lane] = (float) ((double) (float) pn1 / chosen);
    }
}

template <int PER_LANE>
__global__ void __launch_bounds__(kTopkWarps * 32) router_topk_kernel(const float* __restrict__ logits, int T, int E,
                                                                      int k, int32_t* __restrict__ ids,
                                                                      float* __restrict__ wout,
                                                                      const float* __restrict__ x,
                                                                      uint8_t* __restrict__ xq, int H, KAct xa,
                                                                      int xa_q2, RouterSplit rs) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int tpc = topk_tokens_per_cta(T);
    const int route_blocks = (T + tpc - 1) / tpc;
    if ((int) blockIdx.x >= route_blocks) {
        // the remaining CTAs write the q8_1 image of x: one 32-value block per warp, grid-stride
        const int64_t nq = (int64_t) T * (H / 32);
        const int64_t stride = (int64_t) (gridDim.x - route_blocks) * kTopkWarps;
        for (int64_t q = (int64_t) (blockIdx.x - route_blocks) * kTopkWarps + warp; q < nq; q += stride) {
            const float xi = x[q * 32 + lane];
            if (xq) quant_q8_1_warp(xi, xq + q * kQ8Block, lane);
            if (xa.base) quant_ka_warp(xi, xa.base + q * kKaBlock, lane, xa_q2 != 0);
        }
        return;
    }
    const int t = blockIdx.x * tpc + warp;
    const float* l = logits + (size_t) t * E;
    if (rs.part) {
        // the CTA's tokens' logits from the split-K partials, added in split order (router_reduce_kernel's sum), by
        // all of its threads into shared memory (the routing warps read them there) and out to the logits and gate
        // buffers
        extern __shared__ float s_rl[];  // [tokens per CTA][E]
        const int n_rows = E + (rs.y_extra ? 1 : 0);
        const int t0 = blockIdx.x * tpc, nt = min(tpc, T - t0);
        for (int i = threadIdx.x; i < nt * n_rows; i += kTopkWarps * 32) {
            const int tt = t0 + i / n_rows, o = i % n_rows;
            double v[32];
#pragma unroll
            for (int z = 0; z < 32; z++)
                if (z < rs.S) v[z] = __ldg(rs.part + ((size_t) z * T + tt) * n_rows + o);
            double acc = 0.0;
#pragma unroll
            for (int z = 0; z < 32; z++)
                if (z < rs.S) acc += v[z];
            const float f = (float) acc;
            if (o < E) {
                s_rl[(size_t) (i / n_rows) * E + o] = f;
                rs.lout[(size_t) tt * E + o] = f;
            } else {
                rs.y_extra[tt] = f;
            }
        }
        __syncthreads();
        l = s_rl + (size_t) warp * E;
    }
    if (warp >= tpc || t >= T) return;
    route_warp<PER_LANE>(l, E, k, ids + (size_t) t * k, wout + (size_t) t * k, lane);
}

// ------------------------------------------------------------------------------------------------
// launchers
// ------------------------------------------------------------------------------------------------

cudaError_t launch_bf16_gemv(const void* x, bool f32_in, const uint16_t* w, const uint16_t* extra, float* y,
                             float* y_extra, int T, int H, int n_out, cudaStream_t s, void* split_scratch,
                             int* defer) {
    const int n_rows = n_out + (extra ? 1 : 0);
    const int S = split_scratch ? router_splits(T, n_rows, H) : 1;
    if (defer) *defer = 0;
    if (f32_in && H % kRgK == 0 && (T > kRouterGemmMinTokens || S > 1)) {
        const dim3 grid((n_rows + kRgRows - 1) / kRgRows, (T + kRgToks - 1) / kRgToks, S);
        cudaError_t err = cudaFuncSetAttribute(router_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int) kRgSmem);
        if (err != cudaSuccess) return err;
        double* part = S > 1 ? static_cast<double*>(split_scratch) : nullptr;
        router_gemm_kernel<<<grid, 256, kRgSmem, s>>>(static_cast<const float*>(x), w, extra, y, y_extra, T, H,
                                                      n_out, part);
        if (S > 1 && defer) *defer = S;
        else if (S > 1) router_reduce_kernel<<<(T * n_rows + 255) / 256, 256, 0, s>>>(part, S, T, n_rows, n_out, y, y_extra);
        return cudaGetLastError();
    }
    const size_t smem = (size_t) kRouterTokTile * H * 2;
    // few tokens: one row per warp spreads the weight stream over more SMs; many tokens: two rows per warp
    // reuse each staged token twice while 8 warps per CTA keep the fp64 pipe fed
    const int rpw = T <= 4 ? 1 : 2;
    const dim3 grid((n_rows + 8 * rpw - 1) / (8 * rpw), (T + kRouterTokTile - 1) / kRouterTokTile);
    cudaError_t err = cudaSuccess;
#define SMOE_GEMV(F_, R_)                                                                                     \
    do {                                                                                                      \
        err = cudaFuncSetAttribute(bf16_gemv_kernel<F_, R_>, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                   (int) smem);                                                               \
        if (err != cudaSuccess) return err;                                                                   \
        bf16_gemv_kernel<F_, R_><<<grid, 256, smem, s>>>(x, w, extra, y, y_extra, T, H, n_out);              \
    } while (0)
    if (f32_in) {
        if (rpw == 1) SMOE_GEMV(true, 1);
        else SMOE_GEMV(true, 2);
    } else {
        if (rpw == 1) SMOE_GEMV(false, 1);
        else SMOE_GEMV(false, 2);
    }
#undef SMOE_GEMV
    return cudaGetLastError();
}

cudaError_t launch_router_topk(const float* logits, int T, int E, int k, int32_t* ids, float* w, const float* x,
                               uint8_t* xq, int H, cudaStream_t s, const KAct* xa, int xa_q2, const RouterSplit* split) {
    int blocks = (T + topk_tokens_per_cta(T) - 1) / topk_tokens_per_cta(T);
    if (xq || xa) blocks += (int) std::min<int64_t>(((int64_t) T * (H / 32) + kTopkWarps - 1) / kTopkWarps, 148 * 8);
    const KAct a = xa ? *xa : KAct{};
    const RouterSplit rs = split && split->S > 1 ? *split : RouterSplit{};
    if (rs.part && rs.S > 32) return cudaErrorInvalidValue;
    const size_t smem = rs.part ? (size_t) topk_tokens_per_cta(T) * E * sizeof(float) : 0;
    if (E <= 256) router_topk_kernel<8><<<blocks, kTopkWarps * 32, smem, s>>>(logits, T, E, k, ids, w, x, xq, H, a, xa_q2, rs);
    else if (E <= 512) router_topk_kernel<16><<<blocks, kTopkWarps * 32, smem, s>>>(logits, T, E, k, ids, w, x, xq, H, a, xa_q2, rs);
    else router_topk_kernel<32><<<blocks, kTopkWarps * 32, smem, s>>>(logits, T, E, k, ids, w, x, xq, H, a, xa_q2, rs);
    return cudaGetLastError();
}

static int grid_for(int64_t warps_needed) {
    const int64_t blocks = (warps_needed + 7) / 8;
    return (int) (blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

cudaError_t launch_quant_q8_1(const float* x, int64_t n, uint8_t* y, cudaStream_t s) {
    quant_q8_1_kernel<<<grid_for(n / 32), 256, 0, s>>>(x, y, n / 32);
    return cudaGetLastError();
}

cudaError_t launch_swiglu_q8(const float* g, const float* u, int64_t n, uint8_t* y, cudaStream_t s) {
    swiglu_q8_kernel<<<grid_for(n / 32), 256, 0, s>>>(g, u, y, n / 32);
    return cudaGetLastError();
}

__global__ void quant_ka_kernel(const float* __restrict__ x, int64_t n_blocks, KAct xa, int q2) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t b = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n_blocks; b += warps)
        quant_ka_warp(x[b * 32 + lane], xa.base + b * kKaBlock, lane, q2 != 0);
}

cudaError_t launch_quant_ka(const float* x, int64_t rows, int H, const KAct& xa, int q2, cudaStream_t s) {
    const int64_t nb = rows * (H / 32);
    quant_ka_kernel<<<grid_for(nb), 256, 0, s>>>(x, nb, xa, q2);
    return cudaGetLastError();
}

cudaError_t launch_f32_to_bf16(const float* x, uint16_t* y, int64_t n, cudaStream_t s) {
    const int64_t blocks = (n + 255) / 256;
    f32_to_bf16_kernel<<<(int) (blocks < 148 * 8 ? blocks : 148 * 8), 256, 0, s>>>(x, y, n);
    return cudaGetLastError();
}

}  // namespace smoe
