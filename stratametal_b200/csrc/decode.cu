// decode.cu - one token through one MoE layer, or through a stack of layers (x = rms_norm(MoE_l(x) + x) per layer),
// in a single persistent cooperative launch: batch-1 decode (configs[0] and the configs[3] stack at batch 1).
//
// At one token every stage of the block is microseconds of latency over a few megabytes, so the block is laid out
// as three phases per layer with grid barriers between them, one CTA per SM (G CTAs):
//
//   A  (x known)        every CTA holds x in shared memory; CTA c computes router rows [c R / G, (c + 1) R / G)
//                       (R = n_expert + 1 with the shared gate row, fp64 sums) from rows it copied into shared memory
//                       during the previous layer, and quantizes its share of x's q8_1 blocks into a global table.
//   B  (logits known)   every CTA ranks the logits itself (sixteen warp-local top-k, then one merge), copies its work
//                       items - whole 32-row blocks of h: 32 gate and 32 up rows of one slot's expert - and its down
//                       rows (output rows [c H / G, (c + 1) H / G) of every slot) into shared memory, forms the routing
//                       weights while they arrive, computes h = silu(g) * u of its items and writes each block's q8_1
//                       image once (the shared expert's items were copied during the previous layer).
//   C  (h known)        every CTA copies the q8_1 images of h, computes its down rows for every slot and combines them
//                       per output row in router order (fp64) with the gated shared expert; in a stack it writes
//                       v = y + x, meets the others once more, and every CTA forms the next x = rms_norm(v) over the
//                       whole row itself (the RMSNorm kernel's exact reduction tree).
//
// Data other CTAs wrote (logits, the q8_1 images of x and h, v) is copied into shared memory with one cp.async.cg each (through L2, every
// load in flight at once): the same addresses are rewritten every layer, and a line kept in this SM's L1 from the
// previous layer would be stale.
//
// Every dot is the reference's order (partial k of 32 values on lane k & 31, in-lane sums in k order, xor
// butterfly 16..1), the activations follow the q8_1 rule, the routing route_warp's arithmetic and the combine
// the host's fp64 router-order sum, so the results equal the general path's (and the oracle's) bit for bit.
//
// Grid barrier: an arrival count in the caller's scratch, zeroed on the stream before each launch; barrier n of the
// launch completes when the count reaches n x the grid (bounded waits: kWaitLimitNs, after which the CTA records
// kDevTimeout and leaves).
#include "common.cuh"
#include "kernels.cuh"
#include "q8.cuh"

#include <algorithm>

namespace smoe {

constexpr int kDecThreads = 512;  // 16 warps
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecMaxDownRows = 32;    // output rows per CTA
constexpr int kDecMaxSlots = kMaxK + 1;
constexpr int kDecMaxExperts = 512;  // sixteen routing keys per lane of the ranking warp

struct DecLayer {
    const uint16_t* router;  // [E][H] bf16
    const uint16_t* ginp;    // [H] bf16 shared gate row (null without a shared expert)
    const uint8_t *gate, *up, *down;
    const uint8_t *sgate, *sup, *sdown;
    const float* norm_w;     // [H] RMSNorm weight after this layer (null: unit)
    int bulk;  // bit 0: gate/up rows by bulk copies (16-byte aligned planes), bit 1: down rows (and 16-byte rows)
};

struct DecodeArgs {
    DecLayer layers[kDecodeMaxLayers];
    int n_layers;
    int H, F, E, k, has_shared;
    int norm;       // 1: x = rms_norm(MoE(x) + x) after every layer; 0: out = MoE(x) (one layer)
    float eps;
    const float* x;
    float* out;
    float* logits;  // [E + 1]
    uint8_t* xa;    // [H / 32][48] q8_1 image of x
    uint8_t* hq;    // [(k + 1) F / 32][48] q8_1 images of h
    float* vbuf;    // [H]
    unsigned* bar;  // [1]: arrivals over the launch (zero at launch)
    // single-layer trace (null otherwise)
    int32_t* ids;
    float* w;
    float* sh_logit;
    uint8_t* xq;
    float* parts;
    float* shared_out;
};

// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// All CTAs meet at barrier number n (1, 2, ... within the launch); false when this CTA's wait ran out (recorded in
// the status word).  bar[0] counts arrivals over the whole launch (zeroed before it): barrier n completes when it
// reaches n * gridDim.x.  One release add per CTA, acquire loads with a short back-off while waiting.
__device__ __forceinline__ bool dec_grid_sync(unsigned* bar, unsigned n) {
    __syncthreads();
    int ok = 1;
    if (threadIdx.x == 0) {
        const unsigned target = n * gridDim.x;
        unsigned v;
        asm volatile("atom.add.release.gpu.u32 %0, [%1], 1;" : "=r"(v) : "l"(bar) : "memory");
        if (v + 1 < target) {
            const uint64_t t0 = global_timer_ns();
            while (ld_acquire(bar) < target) {
                if (global_timer_ns() - t0 > kWaitLimitNs) {
                    ok = 0;
                    atomicOr(&g_smoe_status, kDevTimeout);
                    break;
                }
                __nanosleep(20);
            }
        }
    }
    return __syncthreads_and(ok) != 0;
}

// Global -> shared memory copy of `bytes` by the whole CTA: cp.async of 16-byte pieces when both ends and the size
// allow them, of 4-byte pieces when they allow those, else plain byte copies (complete on return).  The caller
// commits the group and waits for it.
__device__ __forceinline__ void dec_stage(uint8_t* dst, const uint8_t* src, uint32_t bytes) {
    const uintptr_t al = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | bytes;
    if ((al & 15u) == 0) {
        for (uint32_t o = threadIdx.x * 16u; o < bytes; o += kDecThreads * 16u)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst + o)), "l"(src + o) : "memory");
    } else if ((al & 3u) == 0) {
        for (uint32_t o = threadIdx.x * 4u; o < bytes; o += kDecThreads * 4u)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst + o)), "l"(src + o) : "memory");
    } else {
        for (uint32_t o = threadIdx.x; o < bytes; o += kDecThreads) dst[o] = src[o];
    }
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Q2_0 row of n values (in shared memory) against a q8_1 image (KAct layout, in shared memory): the reference's
// row dot, every lane returning the sum.
__device__ __forceinline__ float dec_row_dot(const uint8_t* row, const uint8_t* act, int n, int lane) {
    float v = 0.f;
    for (int kk = lane; kk < n / 32; kk += 32) {
        Dec d;
        decode_q2(row, kk, d);
        v = __fadd_rn(v, partial_layer<kQ2_0>(d, load_act(act + (size_t) kk * kKaBlock)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// The k largest logits of l[0..E) in route_warp's order (key descending, lower index first among equal keys), by
// one warp.  Lane j holds experts j + 32 i packed as (route_key << 32 | ~index), so one unsigned 64-bit comparison
// orders keys and breaks ties by index (0 marks past E), sorts its C values descending with a bitonic network, then
// k rounds each take the warp's largest head (xor-butterfly max) and advance the winning lane's list.
template <int C>
__device__ __forceinline__ void dec_topk_warp(const float* __restrict__ l, int E, int k, int32_t* s_ids, int lane) {
    uint64_t v[C];
#pragma unroll
    for (int i = 0; i < C; i++) {
        const int e = lane + 32 * i;
        v[i] = e < E ? ((uint64_t) route_key(l[e]) << 32) | (uint64_t) (~(uint32_t) e) : 0ull;
    }
#pragma unroll
    for (int sz = 2; sz <= C; sz <<= 1)
#pragma unroll
        for (int j = sz >> 1; j > 0; j >>= 1)
#pragma unroll
            for (int i = 0; i < C; i++) {
                const int q = i ^ j;
                if (q > i) {
                    const uint64_t x = v[i], y = v[q];
                    const bool sw = (i & sz) == 0 ? x < y : x > y;
                    v[i] = sw ? y : x;
                    v[q] = sw ? x : y;
                }
            }
    for (int r = 0; r < k; r++) {
        uint64_t m = v[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint64_t y = __shfl_xor_sync(0xffffffffu, m, o);
            m = y > m ? y : m;
        }
        if (v[0] == m) {  // the winner (values are unique through their index part)
#pragma unroll
            for (int i = 0; i + 1 < C; i++) v[i] = v[i + 1];
            v[C - 1] = 0ull;
        }
        if (lane == 0) s_ids[r] = (int32_t) ~(uint32_t) m;
    }
}

// Routing by the whole CTA in three short steps (then `dec_rank_candidates` and `dec_weights`):
//   1. thread t packs expert e = 16 (t & 31) + (t >> 5) (warp w holds the experts e = w mod 16, so experts of
//      similar index, which popularity skews alike, spread over the warps): v = route_key << 32 | ~e; each warp
//      finds its largest v and its largest logit (fmaxf, route_warp's max).
//   2. T = the k-th largest of the sixteen warp maxima is at most the k-th largest key overall, so every key of the
//      top k is >= T; a key is a candidate when fewer than k warp maxima exceed it.  Candidates take slots in
//      s_cand (up to kDecMaxCand); p[e] = exp(l[e] - max) in fp64.
//   3. (dec_rank_candidates) one warp ranks the candidates by counting the larger ones; with more than
//      kDecMaxCand candidates, or k above the number of non-empty warps, dec_topk_warp ranks all keys instead.
// The result is route_warp's: key descending, lower index first among equal keys.
constexpr int kDecMaxCand = 64;

__device__ __forceinline__ void dec_route_step1(const float* __restrict__ l, int E, uint64_t& v, uint64_t* s_gmax,
                                                float* s_fmax) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int e = 16 * lane + w;
    const float x = e < E ? l[e] : -INFINITY;
    v = e < E ? ((uint64_t) route_key(x) << 32) | (uint64_t) (~(uint32_t) e) : 0ull;
    uint64_t g = v;
    float m = x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t y = __shfl_xor_sync(0xffffffffu, g, o);
        g = y > g ? y : g;
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    }
    if (lane == 0) {
        s_gmax[w] = g;
        s_fmax[w] = m;
    }
}

__device__ __forceinline__ void dec_route_step2(const float* __restrict__ l, int E, int k, uint64_t v,
                                                const uint64_t* s_gmax, const float* s_fmax, uint64_t* s_cand,
                                                int* s_cnt, double* s_p) {
    int above = 0;
#pragma unroll
    for (int w = 0; w < kDecWarps; w++) above += s_gmax[w] > v ? 1 : 0;
    if (v != 0ull && above < k) {
        const int slot = atomicAdd(s_cnt, 1);
        if (slot < kDecMaxCand) s_cand[slot] = v;
    }
    float mx = s_fmax[0];
#pragma unroll
    for (int i = 1; i < kDecWarps; i++) mx = fmaxf(mx, s_fmax[i]);
    const int t = threadIdx.x;
    if (t < E) s_p[t] = exp((double) l[t] - (double) mx);
}

// step 3, by one warp: candidate c's rank is the number of larger candidates (values are unique through their
// index part)
__device__ __forceinline__ void dec_rank_candidates(const float* __restrict__ l, int E, int k, int n,
                                                    const uint64_t* s_cand, int32_t* s_ids, int lane) {
    if (n > kDecMaxCand || k > min(kDecWarps, E)) {
        dec_topk_warp<kDecMaxExperts / 32>(l, E, k, s_ids, lane);
        return;
    }
    const uint64_t c0 = lane < n ? s_cand[lane] : 0ull, c1 = 32 + lane < n ? s_cand[32 + lane] : 0ull;
    int r0 = 0, r1 = 0;
    for (int j = 0; j < n; j++) {
        const uint64_t c = s_cand[j];
        r0 += c > c0 ? 1 : 0;
        r1 += c > c1 ? 1 : 0;
    }
    if (lane < n && r0 < k) s_ids[r0] = (int32_t) ~(uint32_t) c0;
    if (32 + lane < n && r1 < k) s_ids[r1] = (int32_t) ~(uint32_t) c1;
}

// route_warp's sum of the softmax terms, by one warp: lane j adds p[j + 32 i] in i order, then the xor butterfly
__device__ __forceinline__ double dec_softmax_sum(const double* s_p, int E, int lane) {
    double part = 0.0;
    for (int e = lane; e < E; e += 32) part += s_p[e];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    return part;
}

// route_warp's weights for the ranked ids, by one warp: w_i = (float)((double)(float)(p_i / sum) / max(sum of the
// chosen in rank order, 2^-14)).
__device__ __forceinline__ void dec_weights(int k, const int32_t* s_ids, const double* s_p, double sum, float* s_w,
                                            int lane) {
    const double pn0 = lane < k ? s_p[s_ids[lane]] / sum : 0.0;
    const double pn1 = 32 + lane < k ? s_p[s_ids[32 + lane]] / sum : 0.0;
    double chosen = 0.0;
    for (int i = 0; i < k; i++) chosen += __shfl_sync(0xffffffffu, i < 32 ? pn0 : pn1, i & 31);
    chosen = fmax(chosen, 6.103515625e-05);
    if (lane < k) s_w[lane] = (float) ((double) (float) pn0 / chosen);
    if (32 + lane < k) s_w[32 + lane] = (float) ((double) (float) pn1 / chosen);
}

// the range [c n / G, (c + 1) n / G) of this CTA
__device__ __forceinline__ void dec_range(int n, int& lo, int& hi) {
    lo = (int) ((int64_t) blockIdx.x * n / gridDim.x);
    hi = (int) ((int64_t) (blockIdx.x + 1) * n / gridDim.x);
}

struct DecSmem {
    float* x;          // [H]
    uint8_t* xa;       // [H / 32][48] q8_1 image of x (copied from the global table in phase B)
    uint8_t* router;   // [rr][H] bf16: this CTA's router rows
    uint8_t* items;    // [nit][64][row bytes over H]: per item its 32 gate rows, then its 32 up rows
    uint8_t* down;     // [slots][dr][row bytes over F]; the stack's v = MoE(x) + x [H] in the norm
    float* v;
    uint8_t* ha;       // [slots * F / 32][48] q8_1 images of h
    double* p;         // [E] routing exps
    float* logits;     // [E + 1]
    float* hv;         // [nit][32] h of this CTA's items
    int rr, nit, dr;   // per-CTA maxima: router rows, items, down rows
};

struct DecCounts {
    int rr, nit, dr;
};
SMOE_HD DecCounts dec_counts(int H, int F, int E, int k, int G) {
    return DecCounts{(E + 1 + G - 1) / G, ((k + 1) * (F / 32) + G - 1) / G, (H + G - 1) / G};
}

static size_t dec_up(size_t n) { return (n + 127) & ~(size_t) 127; }

size_t decode_smem_bytes(int H, int F, int E, int k, int grid) {
    const size_t rbh = (size_t) (H / 64) * 18, rbf = (size_t) (F / 64) * 18;
    const DecCounts c = dec_counts(H, F, E, k, grid);
    return dec_up((size_t) H * 4) + dec_up((size_t) H / 32 * kKaBlock) + dec_up((size_t) c.rr * H * 2) +
           dec_up((size_t) c.nit * 64 * rbh) + dec_up(std::max((size_t) (k + 1) * c.dr * rbf, (size_t) H * 4)) +
           dec_up((size_t) (k + 1) * (F / 32) * kKaBlock) + dec_up((size_t) E * 8) + dec_up((size_t) (E + 1) * 4) +
           dec_up((size_t) c.nit * 32 * 4) + 128;
}

__device__ __forceinline__ DecSmem dec_smem(uint8_t* base, int H, int F, int E, int k) {
    const size_t rbh = (size_t) (H / 64) * 18, rbf = (size_t) (F / 64) * 18;
    const DecCounts c = dec_counts(H, F, E, k, gridDim.x);
    auto up = [](size_t n) { return (n + 127) & ~(size_t) 127; };
    DecSmem s;
    s.rr = c.rr;
    s.nit = c.nit;
    s.dr = c.dr;
    uint8_t* p = base;
    s.x = reinterpret_cast<float*>(p);
    p += up((size_t) H * 4);
    s.xa = p;
    p += up((size_t) H / 32 * kKaBlock);
    s.router = p;
    p += up((size_t) c.rr * H * 2);
    s.items = p;
    p += up((size_t) c.nit * 64 * rbh);
    s.down = p;
    s.v = reinterpret_cast<float*>(p);
    p += up(max((size_t) (k + 1) * c.dr * rbf, (size_t) H * 4));
    s.ha = p;
    p += up((size_t) (k + 1) * (F / 32) * kKaBlock);
    s.p = reinterpret_cast<double*>(p);
    p += up((size_t) E * 8);
    s.logits = reinterpret_cast<float*>(p);
    p += up((size_t) (E + 1) * 4);
    s.hv = reinterpret_cast<float*>(p);
    return s;
}

// The gate and up rows of item `it` (slot it / nb, 32-row block it % nb) of expert e (routed) or of the shared expert.
__device__ __forceinline__ void dec_stage_item(const DecodeArgs& a, const DecLayer& L, const DecSmem& s, int j, int it,
                                               int e) {
    const int nb = a.F / 32;
    const size_t rbh = (size_t) (a.H / 64) * 18;
    const int slot = it / nb, blk = it % nb;
    const int64_t stride = (int64_t) a.F * (int64_t) rbh;
    const uint8_t* g = slot < a.k ? L.gate + (int64_t) e * stride : L.sgate;
    const uint8_t* u = slot < a.k ? L.up + (int64_t) e * stride : L.sup;
    uint8_t* dst = s.items + (size_t) j * 64 * rbh;
    dec_stage(dst, g + (size_t) blk * 32 * rbh, (uint32_t) (32 * rbh));
    dec_stage(dst + 32 * rbh, u + (size_t) blk * 32 * rbh, (uint32_t) (32 * rbh));
}

// a layer's routing-independent rows: this CTA's router rows and its shared-expert items
__device__ __forceinline__ void dec_stage_static(const DecodeArgs& a, const DecLayer& L, const DecSmem& s) {
    const int H = a.H;
    int r0, r1;
    dec_range(a.E + (a.has_shared ? 1 : 0), r0, r1);
    for (int r = r0; r < r1; r++) {
        const uint16_t* src = r < a.E ? L.router + (size_t) r * H : L.ginp;
        dec_stage(s.router + (size_t) (r - r0) * H * 2, reinterpret_cast<const uint8_t*>(src), (uint32_t) H * 2);
    }
    int i0, i1;
    dec_range((a.k + (a.has_shared ? 1 : 0)) * (a.F / 32), i0, i1);
    for (int it = i0; it < i1; it++)
        if (it / (a.F / 32) == a.k) dec_stage_item(a, L, s, it - i0, it, 0);
}

__global__ void __launch_bounds__(kDecThreads, 1) decode_stack_kernel(const __grid_constant__ DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t dec_sm[];
    __shared__ int32_t s_ids[kMaxK];
    __shared__ float s_w[kMaxK];
    __shared__ float s_red[kDecWarps];
    __shared__ float s_parts[kDecMaxDownRows][kDecMaxSlots + 1];
    __shared__ double s_part[8];
    __shared__ double s_den, s_rden;
    __shared__ float s_sig;
    __shared__ double s_sum;
    __shared__ uint64_t s_gmax[kDecWarps];
    __shared__ uint64_t s_cand[kDecMaxCand];
    __shared__ int s_cnt;
    __shared__ __align__(8) uint64_t s_mb[2];  // bulk copies: [0] this CTA's routed items, [1] its down rows
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int H = a.H, F = a.F, E = a.E, K = a.k;
    const int nslot = K + (a.has_shared ? 1 : 0);
    const int nb = F / 32, nbx = H / 32;
    const size_t rbh = (size_t) (H / 64) * 18, rbf = (size_t) (F / 64) * 18;
    const int64_t d_stride = (int64_t) H * (int64_t) rbf;
    const DecSmem s = dec_smem(dec_sm, H, F, E, K);
    int r0, r1, i0, i1, j0, j1, x0, x1;
    dec_range(E + (a.has_shared ? 1 : 0), r0, r1);
    dec_range(nslot * nb, i0, i1);
    dec_range(H, j0, j1);
    dec_range(nbx, x0, x1);
    const int nj = j1 - j0;
    bool ok = true;
    unsigned nbar = 0;  // grid barriers passed in this launch

    uint32_t ph[2] = {0u, 0u};  // phases of s_mb[0] / s_mb[1] completed so far
    bool pend[2] = {false, false};  // a phase with copies in flight that nobody has waited for
    if (threadIdx.x == 0) {
        mbar_init(&s_mb[0], 1);
        mbar_init(&s_mb[1], 1);
        fence_mbar_init();
    }
    for (int i = threadIdx.x; i < H; i += kDecThreads) s.x[i] = a.x[i];
    dec_stage_static(a, a.layers[0], s);
    cp_commit();

    for (int l = 0; l < a.n_layers && ok; l++) {
        const DecLayer& L = a.layers[l];
        // ---------------- phase A: router rows, this CTA's blocks of x's q8_1 image ----------------
        cp_wait<0>();
        __syncthreads();
        if (warp < r1 - r0) {  // one router row per warp: fp64 sum of bf16(x) * w, rounded once
            const uint16_t* wr = reinterpret_cast<const uint16_t*>(s.router + (size_t) warp * H * 2);
            double acc = 0.0;
            for (int c = lane * 8; c < H; c += 256) {
                const uint4 wv = *reinterpret_cast<const uint4*>(wr + c);
                const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    acc = fma((double) bf16_round(s.x[c + 2 * q]), (double) __uint_as_float(wu[q] << 16), acc);
                    acc = fma((double) bf16_round(s.x[c + 2 * q + 1]), (double) __uint_as_float(wu[q] & 0xFFFF0000u), acc);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (lane == 0) a.logits[r0 + warp] = (float) acc;
        } else if (warp >= kDecWarps - (x1 - x0)) {
            const int b = x0 + (warp - (kDecWarps - (x1 - x0)));
            quant_ka_warp(s.x[b * 32 + lane], a.xa + (size_t) b * kKaBlock, lane, true);
        }
        if (a.xq && blockIdx.x == 0)
            for (int b = warp; b < nbx; b += kDecWarps) quant_q8_1_warp(s.x[b * 32 + lane], a.xq + (size_t) b * kQ8Block, lane);
        if (!(ok = dec_grid_sync(a.bar, ++nbar))) break;

        // ---------------- phase B: routing, this CTA's items of h ----------------
        // the logits and x's image in one copy each through L2 (other CTAs wrote them; this SM's L1 may hold the
        // previous layer's)
        dec_stage(reinterpret_cast<uint8_t*>(s.logits), reinterpret_cast<const uint8_t*>(a.logits), (uint32_t) (E + 1) * 4);
        dec_stage(s.xa, a.xa, (uint32_t) nbx * kKaBlock);
        cp_commit();
        cp_wait<0>();
        __syncthreads();
        // routing: candidates by the whole CTA, then warp 0 ranks them while warp 1 sums the softmax terms
        uint64_t rv;
        if (threadIdx.x == 0) s_cnt = (K <= min(kDecWarps, E)) ? 0 : kDecMaxCand + 1;
        dec_route_step1(s.logits, E, rv, s_gmax, s_red);
        __syncthreads();
        dec_route_step2(s.logits, E, K, rv, s_gmax, s_red, s_cand, &s_cnt, s.p);
        __syncthreads();
        if (warp == 0) {
            dec_rank_candidates(s.logits, E, K, s_cnt, s_cand, s_ids, lane);
        } else if (warp == 1) {
            const double sum = dec_softmax_sum(s.p, E, lane);
            if (lane == 0) s_sum = sum;
        } else if (threadIdx.x == 64 && a.has_shared) {
            const float e = (float) exp(-(double) s.logits[E]);
            s_sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
        }
        __syncthreads();
        // this CTA's routed items and its down rows of every slot: bulk copies issued by warp 0's lanes, completing on
        // s_mb[0] / s_mb[1], where the planes allow them (16-byte aligned); cp.async otherwise
        const bool items_bulk = (L.bulk & 1) != 0, down_bulk = (L.bulk & 2) != 0;
        const int n_routed = max(0, min(i1, K * nb) - i0);  // the items [i0, i0 + n_routed) are routed slots'
        if (warp == 0 && (items_bulk || down_bulk)) {
            fence_proxy_async();  // this CTA's earlier reads of the buffers before the copies overwrite them
            if (lane == 0) {
                if (items_bulk) mbar_expect_tx(&s_mb[0], (uint32_t) (n_routed * 64 * rbh));
                if (down_bulk) mbar_expect_tx(&s_mb[1], (uint32_t) (nslot * nj * rbf));
            }
            __syncwarp();
            const int n_ic = items_bulk ? 2 * n_routed : 0, n_dc = down_bulk && nj > 0 ? nslot : 0;
            const int64_t stride = (int64_t) F * (int64_t) rbh;
            for (int c = lane; c < n_ic + n_dc; c += 32) {
                if (c < n_ic) {  // item i0 + c / 2: its 32 gate (c even) or up (c odd) rows
                    const int it = i0 + c / 2, slot = it / nb, blk = it % nb;
                    const int64_t off = (int64_t) s_ids[slot] * stride + (int64_t) blk * 32 * (int64_t) rbh;
                    bulk_g2s(s.items + (size_t) (c / 2) * 64 * rbh + (size_t) (c & 1) * 32 * rbh,
                             ((c & 1) ? L.up : L.gate) + off, (uint32_t) (32 * rbh), &s_mb[0]);
                } else {
                    const int sl = c - n_ic;
                    const uint8_t* plane = sl < K ? L.down + (int64_t) s_ids[sl] * d_stride : L.sdown;
                    bulk_g2s(s.down + (size_t) sl * s.dr * rbf, plane + (size_t) j0 * rbf, (uint32_t) (nj * rbf),
                             &s_mb[1]);
                }
            }
        }
        if (!items_bulk)
            for (int it = i0; it < i0 + n_routed; it++) dec_stage_item(a, L, s, it - i0, it, s_ids[it / nb]);
        if (!down_bulk)
            for (int sl = 0; sl < nslot && nj > 0; sl++) {
                const uint8_t* plane = sl < K ? L.down + (int64_t) s_ids[sl] * d_stride : L.sdown;
                dec_stage(s.down + (size_t) sl * s.dr * rbf, plane + (size_t) j0 * rbf, (uint32_t) (nj * rbf));
            }
        cp_commit();
        // the routing weights while the rows arrive
        if (warp == 1) dec_weights(K, s_ids, s.p, s_sum, s_w, lane);
        __syncthreads();
        if (blockIdx.x == 0 && threadIdx.x < K) {
            if (a.ids) a.ids[threadIdx.x] = s_ids[threadIdx.x];
            if (a.w) a.w[threadIdx.x] = s_w[threadIdx.x];
        }
        if (a.sh_logit && blockIdx.x == 0 && threadIdx.x == 0 && a.has_shared) a.sh_logit[0] = s.logits[E];
        pend[0] = items_bulk;
        pend[1] = down_bulk;
        if (!items_bulk) cp_wait<0>();
        if (!(ok = __syncthreads_and(!items_bulk || mbar_wait_bounded(&s_mb[0], ph[0] & 1u, kWaitLimitNs)) != 0)) {
            if (threadIdx.x == 0) atomicOr(&g_smoe_status, kDevTimeout);
            break;
        }
        if (items_bulk) ph[0]++, pend[0] = false;
        for (int u = warp; u < (i1 - i0) * 32; u += kDecWarps) {  // one row pair per warp
            const int j = u / 32, pr = u % 32;
            const uint8_t* item = s.items + (size_t) j * 64 * rbh;
            const float g = dec_row_dot(item + (size_t) pr * rbh, s.xa, H, lane);
            const float uu = dec_row_dot(item + (size_t) (32 + pr) * rbh, s.xa, H, lane);
            if (lane == 0) s.hv[u] = silu_mul(g, uu);
        }
        __syncthreads();
        if (warp < i1 - i0) quant_ka_warp(s.hv[warp * 32 + lane], a.hq + (size_t) (i0 + warp) * kKaBlock, lane, true);
        if (!(ok = dec_grid_sync(a.bar, ++nbar))) break;

        // ---------------- phase C: down rows, combine (and the stack's add + RMSNorm) ----------------
        dec_stage(s.ha, a.hq, (uint32_t) (nslot * nb) * kKaBlock);  // every slot's h image, through L2
        cp_commit();
        if (l + 1 < a.n_layers) dec_stage_static(a, a.layers[l + 1], s);  // the next layer's static rows
        cp_commit();
        cp_wait<1>();  // h (and the down rows when they came by cp.async)
        if (!(ok = __syncthreads_and(!down_bulk || mbar_wait_bounded(&s_mb[1], ph[1] & 1u, kWaitLimitNs)) != 0)) {
            if (threadIdx.x == 0) atomicOr(&g_smoe_status, kDevTimeout);
            break;
        }
        if (down_bulk) ph[1]++, pend[1] = false;
        const int n_dots = nj * nslot;
        if (F <= 512) {  // one half-warp per dot: at most 16 partials, the xor-16 level would add zeros
            const int hl = lane & 15, half = lane >> 4;
            for (int u2 = warp; 2 * u2 < n_dots; u2 += kDecWarps) {
                const int u = 2 * u2 + half;
                const bool valid = u < n_dots;
                const int jl = valid ? u / nslot : 0, sl = valid ? u % nslot : 0;
                float v = 0.f;
                if (valid && hl < nb) {
                    Dec d;
                    decode_q2(s.down + ((size_t) sl * s.dr + jl) * rbf, hl, d);
                    v = partial_layer<kQ2_0>(d, load_act(s.ha + ((size_t) sl * nb + hl) * kKaBlock));
                }
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
                if (valid && hl == 0) s_parts[jl][sl] = v;
            }
        } else {  // one warp per dot
            for (int u = warp; u < n_dots; u += kDecWarps) {
                const int jl = u / nslot, sl = u % nslot;
                const float v = dec_row_dot(s.down + ((size_t) sl * s.dr + jl) * rbf, s.ha + (size_t) sl * nb * kKaBlock,
                                            F, lane);
                if (lane == 0) s_parts[jl][sl] = v;
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
                const float shv = __fmul_rn(s_parts[jl][K], s_sig);
                if (a.shared_out) a.shared_out[j] = shv;
                acc += (double) shv;
            }
            const float y = (float) acc;
            if (a.norm) a.vbuf[j] = __fadd_rn(y, s.x[j]);
            else a.out[j] = y;
        }
        if (!a.norm) continue;
        if (!(ok = dec_grid_sync(a.bar, ++nbar))) break;
        dec_stage(reinterpret_cast<uint8_t*>(s.v), reinterpret_cast<const uint8_t*>(a.vbuf), (uint32_t) H * 4);
        cp_commit();
        cp_wait<0>();
        __syncthreads();
        // x = rms_norm(v): the RMSNorm kernel's tree (256 threads: column c on thread c % 256, fma in column
        // order, xor butterfly per warp, the eight warp sums in order), in every CTA
        if (threadIdx.x < 256) {
            double ss = 0.0;
            for (int c = threadIdx.x; c < H; c += 256) {
                const float v = s.v[c];
                ss = fma((double) v, (double) v, ss);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) s_part[warp] = ss;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            double t = 0.0;
            for (int i = 0; i < 8; i++) t += s_part[i];
            s_den = sqrt(t / (double) H + (double) a.eps);
            s_rden = 1.0 / s_den;
        }
        __syncthreads();
        // v / den correctly rounded without a division per element (Markstein's theorem: with r = RN(1/den) and
        // q = RN(v r) within an ulp of v / den, the residual e = v - q den is exact under an fma and RN(q + e r) is
        // RN(v / den)); checked against the fp64 division on 1.7e10 pairs
        const double den = s_den, rden = s_rden;
        for (int c = threadIdx.x; c < H; c += kDecThreads) {
            const double v = (double) s.v[c];
            const double q = v * rden;
            const double vq = fma(fma(-q, den, v), rden, q);
            const float xn = (float) (vq * (L.norm_w ? (double) L.norm_w[c] : 1.0));
            s.x[c] = xn;
            if (l + 1 == a.n_layers && blockIdx.x == 0) a.out[c] = xn;
        }
        // the next layer's phase A reads s.x after its first __syncthreads; vbuf is next written in that layer's
        // phase C, two grid barriers after every CTA has read it here
    }
    cp_wait<0>();
    if (threadIdx.x == 0)  // a CTA that gave up drains its bulk copies in flight (bounded) before it exits
        for (int b = 0; b < 2; b++)
            if (pend[b]) mbar_wait_bounded(&s_mb[b], ph[b] & 1u, kWaitLimitNs);
}

// Every matrix Q2_0; n_embd a multiple of 512 (gate/up rows of whole 16-byte pieces), n_ff a multiple of 128 (down
// rows of whole 4-byte words) and at most 1024, at most 1024 experts; the per-CTA work must fit the warps and the
// shared-memory tables.
bool decode_qualifies(int H, int F, int E, int k, int gu_type, int d_type, int has_shared, int sg, int su, int sd) {
    const bool q2 = gu_type == kQ2_0 && d_type == kQ2_0 && (!has_shared || (sg == kQ2_0 && su == kQ2_0 && sd == kQ2_0));
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const DecCounts c = dec_counts(H, F, E, k, nsm);
    const int xq = (H / 32 + nsm - 1) / nsm;
    const bool fits = c.rr + xq <= kDecWarps && c.nit <= kDecWarps && c.dr <= kDecMaxDownRows && H <= 4096 &&
                      F <= 1024 && decode_smem_bytes(H, F, E, k, nsm) <= 220 * 1024;
    return q2 && fits && H % 512 == 0 && F % 128 == 0 && E <= kDecMaxExperts && k <= kMaxK && k <= E;
}

size_t decode_scratch_bytes(int H, int F, int E, int k) {
    auto up = [](size_t n) { return (n + 255) / 256 * 256; };
    return up((size_t) (E + 1) * 4) + up((size_t) H / 32 * kKaBlock) + up((size_t) (k + 1) * (F / 32) * kKaBlock) +
           up((size_t) H * 4) + 256;
}

cudaError_t launch_decode(const DecodeHost& h, cudaStream_t s) {
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    if (h.n_layers < 1 || h.n_layers > kDecodeMaxLayers || (!h.norm && h.n_layers != 1)) return cudaErrorInvalidValue;
    DecodeArgs a{};
    for (int l = 0; l < h.n_layers; l++) {
        const smoe_layer& L = h.layers[l];
        auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
        const size_t rbf = (size_t) (L.n_ff / 64) * 18;
        const int bulk = (a16(L.gate) && a16(L.up) ? 1 : 0) |
                         (rbf % 16 == 0 && a16(L.down) && (!L.has_shared || a16(L.sdown)) ? 2 : 0);
        a.layers[l] = DecLayer{L.router, L.has_shared ? L.gate_inp_shexp : nullptr, L.gate, L.up, L.down,
                               L.sgate, L.sup, L.sdown, h.norm_w ? h.norm_w[l] : nullptr, bulk};
    }
    const smoe_layer& L0 = h.layers[0];
    a.n_layers = h.n_layers;
    a.H = L0.n_embd;
    a.F = L0.n_ff;
    a.E = L0.n_expert;
    a.k = L0.k;
    a.has_shared = L0.has_shared ? 1 : 0;
    a.norm = h.norm;
    a.eps = h.eps;
    a.x = h.x;
    a.out = h.out;
    auto up = [](size_t n) { return (n + 255) / 256 * 256; };
    uint8_t* p = static_cast<uint8_t*>(h.scratch);
    a.logits = reinterpret_cast<float*>(p);
    p += up((size_t) (a.E + 1) * 4);
    a.xa = p;
    p += up((size_t) a.H / 32 * kKaBlock);
    a.hq = p;
    p += up((size_t) (a.k + 1) * (a.F / 32) * kKaBlock);
    a.vbuf = reinterpret_cast<float*>(p);
    p += up((size_t) a.H * 4);
    a.bar = reinterpret_cast<unsigned*>(p);
    a.ids = h.ids;
    a.w = h.w;
    a.sh_logit = h.sh_logit;
    a.xq = h.xq;
    a.parts = h.parts;
    a.shared_out = h.shared_out;
    const size_t smem = decode_smem_bytes(a.H, a.F, a.E, a.k, nsm);
    cudaError_t e = cudaMemsetAsync(a.bar, 0, sizeof(unsigned), s);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(decode_stack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) nsm);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_stack_kernel, a);
}

}  // namespace smoe
