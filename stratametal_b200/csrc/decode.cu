// decode.cu - one token through one MoE layer in a single cooperative launch (batch-1 decode, configs[0] and the
// configs[3] stack at batch 1).  At one token every stage of the block is a few microseconds of latency and a
// few megabytes of bytes, so the seven launches of the general path cost more than their work; here the whole
// block is three phases of one persistent kernel separated by two grid barriers:
//
//   phase 0  router logits (warp per expert row, fp64 accumulation); every CTA writes the activation's q8_1
//            image into its shared memory; the CTAs past the router rows take the shared expert's
//            (32-row block) items, which need no routing: 32 gate and 32 up row dots, SwiGLU and the q8_1 rule
//            of that block of h
//   phase 1  every CTA ranks the logits itself (route_cta), starts its phase-2 down rows towards L2, then CTAs
//            take the routed (expert slot, 32-row block) items
//   phase 2  CTAs take ranges of output rows: for each row the down dot of every slot (one per half-warp: at
//            n_ff <= 512 the partials fill lanes 0..15, so the xor-16 level of the reference's butterfly adds
//            zeros and the 16-lane butterfly gives the same bits), then the combine of the row in router order
//            (fp64) plus the gated shared expert
//
// Every dot follows the reference's order (partial k of 32 values to lane k & 31, in-lane sums in k order, xor
// butterfly 16..1), the activations use the q8_1 rule and the combine the host's fp64 router-order sum, so the
// output equals the general path's bit for bit.  The grid barriers share an arrival counter in the caller's
// scratch, zeroed by the host before the launch; every wait is bounded (kWaitLimitNs) and a timeout records
// kDevTimeout and ends the CTA.  The launch is cooperative, so every CTA is resident.
#include "common.cuh"
#include "kernels.cuh"
#include "q8.cuh"

namespace smoe {

constexpr int kDecThreads = 512;  // 16 warps
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecMaxRows = 32;   // output rows per CTA in phase 2 (n_embd <= 4096 over >= 128 CTAs)
constexpr int kDecMaxBlocks = 128;  // q8_1 blocks of the activation (n_embd <= 4096)

struct DecodeArgs {
    const float* x;
    float* out;
    const uint16_t* router;
    const uint16_t* ginp;  // shared-expert gate vector (null without a shared expert)
    Matrix gate, up, down, sgate, sup, sdown;
    int H, F, E, k, has_shared;
    float* logits;       // [E]
    float* sh_logit;     // [1]
    int32_t* ids;        // [k]
    float* w;            // [k]
    uint8_t* ha;         // (k + 1) x F / 32 blocks of h
    uint8_t* xq;         // optional q8_1 image of x (trace)
    float* parts;        // optional [k][H] routed outputs in router order (trace)
    float* shared_out;   // optional [H] gated shared expert (trace)
    unsigned* bar;       // [2] arrival count, generation: zero before the launch
};

// All CTAs meet; false when the wait ran out (the caller then ends the CTA).  bar[0] counts arrivals over the
// whole launch (zeroed by the host before it): barrier number n of the launch completes when it reaches
// n * gridDim.x.  One release add per CTA, acquire loads while waiting.
__device__ __forceinline__ bool grid_barrier(unsigned* bar, unsigned n) {
    __syncthreads();
    int ok = 1;
    if (threadIdx.x == 0) {
        const unsigned target = n * gridDim.x;
        unsigned v;
        asm volatile("atom.add.release.gpu.u32 %0, [%1], 1;" : "=r"(v) : "l"(bar) : "memory");
        v += 1;
        if (v < target) {
            const uint64_t t0 = global_timer_ns();
            do {
                asm volatile("ld.acquire.gpu.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
                if (v >= target) break;
                if (global_timer_ns() - t0 > kWaitLimitNs) {
                    ok = 0;
                    atomicOr(&g_smoe_status, kDevTimeout);
                    break;
                }
            } while (true);
        }
    }
    return __syncthreads_and(ok) != 0;
}

// decode_q2 for a row in global memory: the code words come from 2-byte loads inside the 18-byte block (the
// shared-memory version reads whole aligned words, which can reach 4 bytes past the last row of a plane).
__device__ __forceinline__ void decode_q2_global(const uint8_t* __restrict__ row, int k, Dec& w) {
    const uint8_t* blk = row + (k >> 1) * 18;
    w.d = f16_to_f32(*reinterpret_cast<const uint16_t*>(blk));
    const uint16_t* q = reinterpret_cast<const uint16_t*>(blk + 2 + 8 * (k & 1));
    const uint32_t w0 = (uint32_t) q[0] | ((uint32_t) q[1] << 16);
    const uint32_t w1 = (uint32_t) q[2] | ((uint32_t) q[3] << 16);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        w.c[j] = (w0 >> (2 * j)) & 0x03030303u;
        w.c[4 + j] = (w1 >> (2 * j)) & 0x03030303u;
    }
    w.ls = 0;
}

// Four row dots of n_in values against the same n_in / 32 activation blocks, in the reference's order (partial
// kk on lane kk & 31, in-lane sums in kk order, xor butterfly 16..1; every lane returns the sums).  All loads of
// a partial position are issued before its math, so a warp keeps more of them in flight.
__device__ __forceinline__ void row_dot4_warp(const uint8_t* const (&rows)[4], const uint8_t* __restrict__ act,
                                              int n_in, int lane, float (&v)[4]) {
#pragma unroll
    for (int q = 0; q < 4; q++) v[q] = 0.f;
    for (int kk = lane; kk < n_in / 32; kk += 32) {
        Dec d[4];
#pragma unroll
        for (int q = 0; q < 4; q++) decode_q2_global(rows[q], kk, d[q]);
        const ActRegs ar = load_act(act + (size_t) kk * kKaBlock);
#pragma unroll
        for (int q = 0; q < 4; q++) v[q] = __fadd_rn(v[q], partial_layer<kQ2_0>(d[q], ar));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int q = 0; q < 4; q++) v[q] = __fadd_rn(v[q], __shfl_xor_sync(0xffffffffu, v[q], o));
}

// route_warp's result computed by a whole CTA of kDecThreads threads (E <= kDecThreads): thread t holds logit t.
// The order (logit descending, lower index first) comes from a bitonic sort of (logit, index) - partners closer
// than 32 exchange by shuffle, farther ones through shared memory.  p = exp(l - max) in fp64 is evaluated once per
// expert; its sum is taken in route_warp's order (lane l adds p[l], p[l + 32], ... in turn, then the xor
// butterfly), and the weights of the chosen as route_warp forms them, so the two give the same bits.
__device__ __forceinline__ bool rank_before(float va, int ia, float vb, int ib) {
    return va > vb || (va == vb && ia < ib);
}

__device__ __forceinline__ void route_cta(const float* __restrict__ l, int E, int k, int32_t* s_ids, float* s_w) {
    __shared__ float sv[kDecThreads];
    __shared__ int si[kDecThreads];
    __shared__ double sp[kDecThreads];
    __shared__ float s_red[kDecWarps];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float v = t < E ? l[t] : -INFINITY;
    int ix = t;
    float m = v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_red[warp] = m;
    __syncthreads();
    float mx = s_red[0];
#pragma unroll
    for (int i = 1; i < kDecWarps; i++) mx = fmaxf(mx, s_red[i]);
    if (t < E) sp[t] = exp((double) v - (double) mx);
    // bitonic sort of (v, ix), final order: rank_before
    for (int kk = 2; kk <= kDecThreads; kk <<= 1) {
        for (int j = kk >> 1; j > 0; j >>= 1) {
            float pv;
            int pi;
            if (j >= 32) {
                __syncthreads();
                sv[t] = v;
                si[t] = ix;
                __syncthreads();
                pv = sv[t ^ j];
                pi = si[t ^ j];
            } else {
                pv = __shfl_xor_sync(0xffffffffu, v, j);
                pi = __shfl_xor_sync(0xffffffffu, ix, j);
            }
            const bool first = ((t & j) == 0) == ((t & kk) == 0);  // this position keeps the earlier of the two
            const bool mine_first = rank_before(v, ix, pv, pi);
            if (first != mine_first) {
                v = pv;
                ix = pi;
            }
        }
    }
    __syncthreads();
    sv[t] = v;
    si[t] = ix;
    __syncthreads();
    if (warp == 0) {
        double part = 0.0;
        for (int e = lane; e < E; e += 32) part += sp[e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        const double sum = part;
        const double pn0 = lane < k ? sp[si[lane]] / sum : 0.0;
        const double pn1 = 32 + lane < k ? sp[si[32 + lane]] / sum : 0.0;
        double chosen = 0.0;
        for (int i = 0; i < k; i++) chosen += __shfl_sync(0xffffffffu, i < 32 ? pn0 : pn1, i & 31);
        chosen = fmax(chosen, 6.103515625e-05);
        if (lane < k) {
            s_ids[lane] = si[lane];
            s_w[lane] = (float) ((double) (float) pn0 / chosen);
        }
        if (32 + lane < k) {
            s_ids[32 + lane] = si[32 + lane];
            s_w[32 + lane] = (float) ((double) (float) pn1 / chosen);
        }
    }
}

__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

__global__ void __launch_bounds__(kDecThreads, 1) decode_layer_kernel(DecodeArgs a) {
    __shared__ int32_t s_ids[kMaxK];
    __shared__ float s_w[kMaxK];
    __shared__ float s_g[32], s_u[32];
    __shared__ float s_parts[kDecMaxRows][kMaxK + 1];
    __shared__ __align__(16) uint8_t s_xa[kDecMaxBlocks * kKaBlock];  // this CTA's copy of the activation image
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gw = blockIdx.x * kDecWarps + warp, nw = gridDim.x * kDecWarps;
    const int H = a.H, F = a.F, E = a.E, K = a.k;
    const int nslot = K + (a.has_shared ? 1 : 0);
    const int nb = F / 32;
    const int rbg = (H / 64) * 18;

    // gate and up rows of one 32-row block of slot s, SwiGLU, the q8_1 block of h (warp w: rows 2w, 2w + 1)
    auto gate_up_item = [&](int s, int b, const uint8_t* gb, const uint8_t* ub) {
        const uint8_t* rows[4];
#pragma unroll
        for (int q = 0; q < 4; q++) rows[q] = (q < 2 ? gb : ub) + (size_t) (b * 32 + 2 * warp + (q & 1)) * rbg;
        float v[4];
        row_dot4_warp(rows, s_xa, H, lane, v);
        if (lane == 0) {
            s_g[2 * warp] = v[0];
            s_g[2 * warp + 1] = v[1];
            s_u[2 * warp] = v[2];
            s_u[2 * warp + 1] = v[3];
        }
        __syncthreads();
        if (warp == 0)
            quant_ka_warp(silu_mul(s_g[lane], s_u[lane]), a.ha + ((size_t) s * nb + b) * kKaBlock, lane, true);
        __syncthreads();
    };

    // ---- phase 0: the activation image (every CTA, in shared memory), router logits (fp64), and the shared
    // expert's gate/up, which does not depend on the routing ----
    const int router_rows = E + (a.has_shared ? 1 : 0);
    for (int r = gw; r < router_rows; r += nw) {
        const uint16_t* wr = r < E ? a.router + (size_t) r * H : a.ginp;
        double acc = 0.0;
#pragma unroll 8
        for (int c = lane * 8; c < H; c += 256) {
            const uint4 wv = __ldg(reinterpret_cast<const uint4*>(wr + c));
            const float4 x0 = __ldg(reinterpret_cast<const float4*>(a.x + c));
            const float4 x1 = __ldg(reinterpret_cast<const float4*>(a.x + c + 4));
            const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int q = 0; q < 4; q++) {
                acc = fma((double) bf16_round(xv[2 * q]), (double) __uint_as_float(wu[q] << 16), acc);
                acc = fma((double) bf16_round(xv[2 * q + 1]), (double) __uint_as_float(wu[q] & 0xFFFF0000u), acc);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
            if (r < E) a.logits[r] = (float) acc;
            else a.sh_logit[0] = (float) acc;
        }
    }
    // the activation image of this CTA (x is read from L2 by every CTA: all loads first)
    {
        float xi[kDecMaxBlocks / kDecWarps];
#pragma unroll
        for (int i = 0; i < kDecMaxBlocks / kDecWarps; i++) {
            const int b = warp + kDecWarps * i;
            xi[i] = b < H / 32 ? a.x[b * 32 + lane] : 0.f;
        }
#pragma unroll
        for (int i = 0; i < kDecMaxBlocks / kDecWarps; i++) {
            const int b = warp + kDecWarps * i;
            if (b < H / 32) {
                quant_ka_warp(xi[i], s_xa + (size_t) b * kKaBlock, lane, true);
                if (a.xq && blockIdx.x == 0) quant_q8_1_warp(xi[i], a.xq + (size_t) b * kQ8Block, lane);
            }
        }
    }
    __syncthreads();
    // CTAs past the router rows take the shared expert's blocks (if there are enough CTAs; else phase 1 does)
    const int r0 = (router_rows + kDecWarps - 1) / kDecWarps;
    const bool shared_early = a.has_shared && (int) gridDim.x > r0;
    if (shared_early)
        for (int it = (int) blockIdx.x - r0; it >= 0 && it < nb; it += (int) gridDim.x - r0)
            gate_up_item(K, it, a.sgate.base, a.sup.base);
    if (!grid_barrier(a.bar, 1)) return;

    // ---- phase 1: routing (every CTA), routed gate/up + SwiGLU + q8_1 per (slot, 32-row block) ----
    route_cta(a.logits, E, K, s_ids, s_w);
    __syncthreads();
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < K; i += blockDim.x) {
            a.ids[i] = s_ids[i];
            a.w[i] = s_w[i];
        }
    // start this CTA's phase-2 down rows on their way to L2
    const int rows_per = (H + gridDim.x - 1) / gridDim.x;
    const int j0 = blockIdx.x * rows_per, nj = max(0, min(rows_per, H - j0));
    const int rbd = (F / 64) * 18;
    for (int u = threadIdx.x; u < nslot * nj; u += blockDim.x) {
        const int s = u % nslot, jl = u / nslot;
        const uint8_t* row = (s >= K ? a.sdown.base : a.down.base + (int64_t) s_ids[s] * a.down.expert_stride) +
                             (size_t) (j0 + jl) * rbd;
        for (int off = 0; off < rbd; off += 128) prefetch_l2(row + off);
    }
    const int n_items = (shared_early ? K : nslot) * nb;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int s = item / nb, b = item % nb;
        const bool sh = s >= K;
        gate_up_item(s, b, sh ? a.sgate.base : a.gate.base + (int64_t) s_ids[s] * a.gate.expert_stride,
                     sh ? a.sup.base : a.up.base + (int64_t) s_ids[s] * a.up.expert_stride);
    }
    if (!grid_barrier(a.bar, 2)) return;

    // ---- phase 2: down dots by output row range, then the combine of each row ----
    const int hl = lane & 15, half = lane >> 4;
    const int n_dots = nj * nslot;
    constexpr int kBatch = 3;  // dots per half-warp with their loads in flight together
    for (int u2 = warp; 2 * u2 < n_dots; u2 += kDecWarps * kBatch) {  // warp-uniform trip count
        Dec d[kBatch];
        ActRegs ar[kBatch];
        bool act[kBatch];
        int jl[kBatch], sl[kBatch];
#pragma unroll
        for (int i = 0; i < kBatch; i++) {
            const int u = 2 * (u2 + i * kDecWarps) + half;
            const bool valid = u < n_dots;
            jl[i] = valid ? u / nslot : 0;
            sl[i] = valid ? u % nslot : 0;
            act[i] = valid && hl < F / 32;  // partial hl of this dot (lanes past the partials hold zero)
            if (act[i]) {
                const uint8_t* row = (sl[i] >= K ? a.sdown.base
                                                 : a.down.base + (int64_t) s_ids[sl[i]] * a.down.expert_stride) +
                                     (size_t) (j0 + jl[i]) * rbd;
                decode_q2_global(row, hl, d[i]);
                ar[i] = load_act(a.ha + ((size_t) sl[i] * nb + hl) * kKaBlock);
            }
        }
#pragma unroll
        for (int i = 0; i < kBatch; i++) {
            float v = act[i] ? partial_layer<kQ2_0>(d[i], ar[i]) : 0.f;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
            const int u = 2 * (u2 + i * kDecWarps) + half;
            if (u < n_dots && hl == 0) s_parts[jl[i]][sl[i]] = v;
        }
    }
    __syncthreads();
    if ((int) threadIdx.x < nj) {
        const int jl = threadIdx.x, j = j0 + jl;
        double acc = 0.0;
        for (int i = 0; i < K; i++) {
            acc += (double) s_w[i] * (double) s_parts[jl][i];
            if (a.parts) a.parts[(size_t) i * H + j] = s_parts[jl][i];
        }
        if (a.has_shared) {
            const float e = (float) exp(-(double) a.sh_logit[0]);
            const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
            const float shv = __fmul_rn(s_parts[jl][K], sig);
            if (a.shared_out) a.shared_out[j] = shv;
            acc += (double) shv;
        }
        a.out[j] = (float) acc;
    }
}

// The fused path needs every matrix in Q2_0, n_embd a multiple of 256 (the router's 8-value lanes), at most 512
// intermediate values (one half-warp per down dot) and at most 512 experts (one per thread in the routing).
bool decode_qualifies(int H, int F, int E, int k, int gu_type, int d_type, int has_shared, int sg, int su, int sd) {
    const bool q2 = gu_type == kQ2_0 && d_type == kQ2_0 &&
                    (!has_shared || (sg == kQ2_0 && su == kQ2_0 && sd == kQ2_0));
    return q2 && H % 256 == 0 && F % 32 == 0 && F <= 512 && E <= kDecThreads && k <= kMaxK && k <= E;
}

cudaError_t launch_decode_layer(const DecodeArgs& a, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(a.bar, 0, 2 * sizeof(unsigned), s);
    if (e != cudaSuccess) return e;
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    if ((a.H + nsm - 1) / nsm > kDecMaxRows) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) nsm);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_layer_kernel, a);
}

}  // namespace smoe
