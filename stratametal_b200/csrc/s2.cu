// s2.cu - the Strata pack's planar S2 experts on the device: the GGUF -> S2 re-layout, the Q8_0 activation rule,
// and the grouped expert evaluation the upstream decode path calls with device-side group / hit lists
// (include/strata/kernels/s2_expert_grouped.hpp:72-112, quantize_act.hpp:20-30).
//
// Blob layout (include/strata/kernels/cpu/expert.hpp:34-51, with H = n_embd and F = n_ff as parameters): the 2F
// gate/up code rows interleaved (row 2r gate r, 2r + 1 up r), H / 4 bytes each; the H down code rows, F / 4 bytes
// each; the fp16 scales of the gate/up rows (H / 64 per row) and of the down rows (F / 64 per row).  Two-bit codes,
// four per byte, first value in the low bits; a weight is (code - 1) * d of its 64-value block.
//
// Arithmetic: every row is the reference's row_dot (iq_parity.cpp:275-292) over 32-value partials
// (d_w * d_x) * sum (code - 1) q, partial k on lane k & 31, lanes meeting in the xor butterfly 16..1; d_x is the
// activation block's fp16 d, or the caller's fp32 scale when x_scales is given.  h = silu(g) * u is quantized in the
// same contract as x (quantize_q8_0, or its fp32-scale variant).  An S2 blob therefore computes exactly what the
// GGUF Q2_0 rows it was packed from compute on the same activation bytes.
//
// Grouping: group g's blob sits at grp_ptr[g]; its entries are [grp_start[g], grp_start[g + 1]), entry i reading
// activation row ent_tok[i] and writing out row ent_dst[i].  Counts come from device memory, so one captured graph
// serves any routing; the grids are persistent and skip what the counts exclude.
#include "common.cuh"
#include "kernels.cuh"
#include "q8.cuh"

namespace smoe {

constexpr int kS2Threads = 256;

struct S2Geom {
    int H, F;
    size_t gu_codes, d_codes, gu_scales, d_scales;
};
SMOE_HD S2Geom s2_geom(int H, int F) {
    S2Geom g;
    g.H = H;
    g.F = F;
    g.gu_codes = 0;
    g.d_codes = (size_t) 2 * F * (H / 4);
    g.gu_scales = g.d_codes + (size_t) H * (F / 4);
    g.d_scales = g.gu_scales + (size_t) 2 * F * (H / 64) * 2;
    return g;
}
size_t s2_blob_bytes(int H, int F) { return (size_t) 3 * H * F / 64 * 18; }

// ---- GGUF Q2_0 rows -> S2 blob: one thread per 64-value block --------------------------------------------------
__global__ void s2_pack_kernel(const uint8_t* __restrict__ gate, const uint8_t* __restrict__ up,
                               const uint8_t* __restrict__ down, int H, int F, uint8_t* __restrict__ blob) {
    const S2Geom g = s2_geom(H, F);
    const int bgu = H / 64, bd = F / 64;
    const int64_t n_gu = (int64_t) 2 * F * bgu, n_all = n_gu + (int64_t) H * bd;
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n_all; i += (int64_t) gridDim.x * blockDim.x) {
        const uint8_t* src;
        uint8_t *codes, *sc;
        if (i < n_gu) {
            const int64_t row = i / bgu, b = i % bgu;  // interleaved row: 2r gate, 2r + 1 up
            const uint8_t* plane = (row & 1) ? up : gate;
            src = plane + (size_t) (row >> 1) * bgu * 18 + b * 18;
            codes = blob + g.gu_codes + (size_t) row * (H / 4) + b * 16;
            sc = blob + g.gu_scales + ((size_t) row * bgu + b) * 2;
        } else {
            const int64_t j = (i - n_gu) / bd, b = (i - n_gu) % bd;
            src = down + (size_t) j * bd * 18 + b * 18;
            codes = blob + g.d_codes + (size_t) j * (F / 4) + b * 16;
            sc = blob + g.d_scales + ((size_t) j * bd + b) * 2;
        }
        sc[0] = src[0];
        sc[1] = src[1];
#pragma unroll
        for (int c = 0; c < 16; c++) codes[c] = src[2 + c];
    }
}

// ---- Q8_0 of 32 values by one warp (sgemv.mm:145-172; with `scales` the fp32-scale variant) --------------------
__device__ __forceinline__ void quant_q8_0_warp(float xi, uint8_t* __restrict__ yb, float* __restrict__ scale, int lane) {
    float amax = fabsf(xi);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d32 = __fdiv_rn(amax, 127.f);
    if (scale && lane == 0) *scale = d32;
    if (amax == 0.f) {
        if (lane < 17) reinterpret_cast<uint16_t*>(yb)[lane] = 0;  // 34 zero bytes
        return;
    }
    int q;
    if (scale) {
        q = (int) fminf(fmaxf(roundf(__fdiv_rn(xi, d32)), -127.f), 127.f);
    } else {
        const double r = rint(__ddiv_rn((double) xi, (double) d32));
        q = (int) fmin(fmax(r, -128.0), 127.0);
    }
    yb[2 + lane] = (uint8_t) (int8_t) q;
    if (lane == 0) {
        const uint16_t dh = f16_bits(d32);
        yb[0] = (uint8_t) dh;
        yb[1] = (uint8_t) (dh >> 8);
    }
}

__global__ void quant_q8_0_kernel(const float* __restrict__ x, int64_t n_blocks, uint8_t* __restrict__ y,
                                  float* __restrict__ scales) {
    const int lane = threadIdx.x & 31;
    for (int64_t b = (int64_t) blockIdx.x * 8 + (threadIdx.x >> 5); b < n_blocks; b += (int64_t) gridDim.x * 8)
        quant_q8_0_warp(x[b * 32 + lane], y + b * 34, scales ? scales + b : nullptr, lane);
}

// ---- one planar row against one Q8_0 activation row, the reference's row_dot order -------------------------------
// q bytes of block k start at 34 k + 2 (two-byte aligned): eight words from sixteen halfwords
__device__ __forceinline__ void s2_load_q(const uint8_t* blk, uint32_t (&q)[8]) {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(blk + 2);
#pragma unroll
    for (int i = 0; i < 8; i++) q[i] = (uint32_t) h[2 * i] | ((uint32_t) h[2 * i + 1] << 16);
}

__device__ __forceinline__ float s2_row_dot(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ sc, int n,
                                            const uint8_t* __restrict__ xq, const float* __restrict__ xs, int lane) {
    float acc = 0.f;
    for (int k = lane; k < n / 32; k += 32) {
        const uint2 cw = *reinterpret_cast<const uint2*>(codes + 8 * k);  // 32 codes, 8-byte aligned
        uint32_t q[8];
        s2_load_q(xq + (size_t) k * 34, q);
        int cq = 0, sq = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t b = ((i < 4 ? cw.x : cw.y) >> (8 * (i & 3))) & 0xFFu;
            uint32_t w = (b | (b << 12)) & 0x000F000Fu;
            w = (w | (w << 6)) & 0x03030303u;  // codes 4i .. 4i + 3, one per byte
            cq = __dp4a((int) w, (int) q[i], cq);
            sq = __dp4a(0x01010101, (int) q[i], sq);
        }
        const float dx = xs ? xs[k] : f16_to_f32(*reinterpret_cast<const uint16_t*>(xq + (size_t) k * 34));
        const float dw = f16_to_f32(*reinterpret_cast<const uint16_t*>(sc + 2 * (k >> 1)));
        acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(dw, dx), (float) (cq - sq)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    return acc;
}

struct S2Args {
    const unsigned long long* grp_ptr;
    const int32_t* grp_start;
    const int32_t* n_groups;
    const int32_t* ent_dst;
    const int32_t* ent_tok;
    int cap_groups, cap_entries;
    int H, F;
    const uint8_t* xq;   // [tokens][H / 32] Q8_0
    const float* xs;     // [tokens][H / 32] or null
    float* hf;           // [cap_entries][F]
    uint8_t* hq;         // [cap_entries][F / 32] Q8_0
    float* hs;           // [cap_entries][F / 32] (with xs)
    float* out;          // [rows][H]
};

// groups the counts admit (a count past its capacity is clamped and recorded as BAD_ID)
__device__ __forceinline__ int s2_groups(const S2Args& a) {
    int n = a.n_groups[0];
    if (n < 0 || n > a.cap_groups) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(&g_smoe_status, kDevBadId);
        n = n < 0 ? 0 : a.cap_groups;
    }
    return n;
}
__device__ __forceinline__ void s2_entries(const S2Args& a, int g, int& e0, int& e1) {
    e0 = a.grp_start[g];
    e1 = a.grp_start[g + 1];
    if (e0 < 0 || e1 > a.cap_entries || e1 < e0) {
        if (threadIdx.x == 0) atomicOr(&g_smoe_status, kDevBadId);
        e0 = e1 = 0;
    }
}

// gate and up row r of group g for each entry: hf[i][r] = silu(gate . x) * (up . x); one warp per row pair
__global__ void __launch_bounds__(kS2Threads) s2_gate_up_kernel(S2Args a) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const S2Geom g = s2_geom(a.H, a.F);
    const int n_groups = s2_groups(a);
    const int tiles = (a.F + 7) / 8;
    const int nb = a.H / 32;
    for (int item = blockIdx.x; item < n_groups * tiles; item += gridDim.x) {
        const int grp = item / tiles, r = (item % tiles) * 8 + warp;
        if (r >= a.F) continue;
        int e0, e1;
        s2_entries(a, grp, e0, e1);
        const uint8_t* blob = reinterpret_cast<const uint8_t*>(a.grp_ptr[grp]);
        const uint8_t* cg = blob + g.gu_codes + (size_t) (2 * r) * (a.H / 4);
        const uint8_t* sg = blob + g.gu_scales + (size_t) (2 * r) * (a.H / 64) * 2;
        for (int i = e0; i < e1; i++) {
            const int t = a.ent_tok[i];
            const uint8_t* xq = a.xq + (size_t) t * nb * 34;
            const float* xs = a.xs ? a.xs + (size_t) t * nb : nullptr;
            const float gv = s2_row_dot(cg, sg, a.H, xq, xs, lane);
            const float uv = s2_row_dot(cg + a.H / 4, sg + (a.H / 64) * 2, a.H, xq, xs, lane);
            if (lane == 0) a.hf[(size_t) i * a.F + r] = silu_mul(gv, uv);
        }
    }
}

// h of every entry in the activation contract of x
__global__ void __launch_bounds__(kS2Threads) s2_quant_h_kernel(S2Args a) {
    const int lane = threadIdx.x & 31;
    const int n_groups = s2_groups(a);
    int n_ent = n_groups > 0 ? a.grp_start[n_groups] : 0;
    n_ent = max(0, min(n_ent, a.cap_entries));
    const int64_t nbh = a.F / 32, total = (int64_t) n_ent * nbh;
    for (int64_t b = (int64_t) blockIdx.x * 8 + (threadIdx.x >> 5); b < total; b += (int64_t) gridDim.x * 8)
        quant_q8_0_warp(a.hf[b * 32 + lane], a.hq + b * 34, a.xs ? a.hs + b : nullptr, lane);
}

// down row j of group g for each entry: out[ent_dst[i]][j]; one warp per row
__global__ void __launch_bounds__(kS2Threads) s2_down_kernel(S2Args a) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const S2Geom g = s2_geom(a.H, a.F);
    const int n_groups = s2_groups(a);
    const int tiles = (a.H + 7) / 8;
    const int nbh = a.F / 32;
    for (int item = blockIdx.x; item < n_groups * tiles; item += gridDim.x) {
        const int grp = item / tiles, j = (item % tiles) * 8 + warp;
        if (j >= a.H) continue;
        int e0, e1;
        s2_entries(a, grp, e0, e1);
        const uint8_t* blob = reinterpret_cast<const uint8_t*>(a.grp_ptr[grp]);
        const uint8_t* cd = blob + g.d_codes + (size_t) j * (a.F / 4);
        const uint8_t* sd = blob + g.d_scales + (size_t) j * (a.F / 64) * 2;
        for (int i = e0; i < e1; i++) {
            const float v = s2_row_dot(cd, sd, a.F, a.hq + (size_t) i * nbh * 34, a.xs ? a.hs + (size_t) i * nbh : nullptr,
                                       lane);
            if (lane == 0) a.out[(size_t) a.ent_dst[i] * a.H + j] = v;
        }
    }
}

// ---- group / hit lists ----------------------------------------------------------------------------------------
// moe_group_resident: every id of ids[n] is resident at base + id * blob.  Groups are the distinct ids in ascending
// order; a group's entries are its routing indices in order (dst = index, tok = index / k_per_tok).  One CTA.
__global__ void __launch_bounds__(1024) s2_group_resident_kernel(const int32_t* __restrict__ ids, int n, int k_per_tok,
                                                                 const uint8_t* base, int64_t blob,
                                                                 unsigned long long* grp_ptr, int32_t* grp_start,
                                                                 int32_t* counts, int32_t* ent_dst, int32_t* ent_tok) {
    __shared__ int s_id[1024];
    __shared__ int s_sorted[1024];
    __shared__ int s_head[1024];
    __shared__ int warp_sums[32];
    const int i = threadIdx.x;
    const int id = i < n ? ids[i] : -1;
    s_id[i] = id;
    __syncthreads();
    // rank of (id, i) among the valid entries
    int rank = 0;
    if (id >= 0)
        for (int j = 0; j < n; j++) {
            const int o = s_id[j];
            rank += (o >= 0 && (o < id || (o == id && j < i))) ? 1 : 0;
        }
    if (id >= 0) s_sorted[rank] = i;
    int n_valid = 0;
    {
        int v = id >= 0 ? 1 : 0;
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if ((i & 31) == 0) warp_sums[i >> 5] = v;
    }
    __syncthreads();
    for (int w = 0; w < (int) (blockDim.x >> 5); w++) n_valid += warp_sums[w];
    // heads: the first entry of each group in sorted order
    const int src = i < n_valid ? s_sorted[i] : -1;
    const int sid = src >= 0 ? s_id[src] : -1;
    const int head = (i < n_valid && (i == 0 || s_id[s_sorted[i - 1]] != sid)) ? 1 : 0;
    s_head[i] = head;
    __syncthreads();
    int gidx = 0;  // groups before this sorted position (inclusive of its own head)
    for (int j = 0; j <= i && j < n_valid; j++) gidx += s_head[j];
    if (i < n_valid) {
        ent_dst[i] = src;
        ent_tok[i] = k_per_tok > 0 ? src / k_per_tok : 0;
        if (head) {
            grp_ptr[gidx - 1] = (unsigned long long) (base + (int64_t) sid * blob);
            grp_start[gidx - 1] = i;
        }
    }
    __syncthreads();
    if (i == 0) {
        int ng = 0;
        for (int j = 0; j < n_valid; j++) ng += s_head[j];
        grp_start[ng] = n_valid;
        counts[0] = ng;
        counts[1] = n_valid;
    }
}

// moe_hit_select: the routing entries whose expert is resident (res_row[e] = slot or -1), in routing order.
__global__ void __launch_bounds__(1024) s2_hit_select_kernel(const int32_t* __restrict__ ids,
                                                             const int32_t* __restrict__ res_row, int n, int n_expert,
                                                             int32_t* slot, int32_t* dst, int32_t* count) {
    __shared__ int warp_sums[32];
    const int i = threadIdx.x, lane = i & 31, warp = i >> 5;
    const int e = i < n ? ids[i] : -1;
    const int s = (e >= 0 && e < n_expert) ? res_row[e] : -1;
    const int hit = s >= 0 ? 1 : 0;
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    if (lane == 0) warp_sums[warp] = __popc(m);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < (int) (blockDim.x >> 5); w++) {
        if (w < warp) before += warp_sums[w];
        total += warp_sums[w];
    }
    if (hit) {
        const int pos = before + __popc(m & ((1u << lane) - 1u));
        slot[pos] = s;
        dst[pos] = i;
    }
    if (i == 0) count[0] = total;
}

// hits -> one group each: blob base + slot * blob_bytes, entry dst = dst_index[h], tok = dst / k_per_token (0: one
// activation for every hit)
__global__ void s2_hits_to_groups_kernel(const uint8_t* base, const int32_t* __restrict__ slot_index,
                                         const int32_t* __restrict__ dst_index, const int32_t* __restrict__ d_count,
                                         int cap, int64_t blob_bytes, int k_per_token, unsigned long long* grp_ptr,
                                         int32_t* grp_start, int32_t* n_groups, int32_t* ent_dst, int32_t* ent_tok) {
    int n = d_count[0];
    if (n < 0 || n > cap) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(&g_smoe_status, kDevBadId);
        n = n < 0 ? 0 : cap;
    }
    for (int h = blockIdx.x * blockDim.x + threadIdx.x; h <= n; h += gridDim.x * blockDim.x) {
        grp_start[h] = h;
        if (h == n) {
            n_groups[0] = n;
            continue;
        }
        grp_ptr[h] = (unsigned long long) (base + (int64_t) slot_index[h] * blob_bytes);
        const int d = dst_index[h];
        ent_dst[h] = d;
        ent_tok[h] = k_per_token > 0 ? d / k_per_token : 0;
    }
}

// moe_hit_add: parts[dst[h]] += hit_out[dst[h]] for the hits (rows a CPU tier left at zero)
__global__ void s2_hit_add_kernel(float* __restrict__ parts, const float* __restrict__ hit_out,
                                  const int32_t* __restrict__ dst, const int32_t* __restrict__ count, int cap, int64_t H) {
    int n = count[0];
    n = max(0, min(n, cap));
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t) n * H;
         i += (int64_t) gridDim.x * blockDim.x) {
        const int64_t row = dst[i / H];
        parts[row * H + i % H] = __fadd_rn(parts[row * H + i % H], hit_out[row * H + i % H]);
    }
}

// ---- launches ---------------------------------------------------------------------------------------------------
static int s2_grid() {
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    return nsm * 8;
}

// scratch: hf [cap][F] f32, hq [cap][F/32][34], hs [cap][F/32] f32, then the hit lists' groups
struct S2Scratch {
    float* hf;
    uint8_t* hq;
    float* hs;
    unsigned long long* grp_ptr;
    int32_t *grp_start, *n_groups, *ent_dst, *ent_tok;
};
static size_t a256(size_t n) { return (n + 255) & ~(size_t) 255; }
size_t s2_scratch_bytes(int64_t cap, int H, int F) {
    (void) H;
    return a256((size_t) cap * F * 4) + a256((size_t) cap * (F / 32) * 34) + a256((size_t) cap * (F / 32) * 4) +
           a256((size_t) cap * 8) + a256((size_t) (cap + 1) * 4) + a256(4) + 2 * a256((size_t) cap * 4);
}
static S2Scratch s2_scratch_at(void* p, int64_t cap, int F) {
    uint8_t* b = static_cast<uint8_t*>(p);
    S2Scratch s;
    s.hf = reinterpret_cast<float*>(b);
    b += a256((size_t) cap * F * 4);
    s.hq = b;
    b += a256((size_t) cap * (F / 32) * 34);
    s.hs = reinterpret_cast<float*>(b);
    b += a256((size_t) cap * (F / 32) * 4);
    s.grp_ptr = reinterpret_cast<unsigned long long*>(b);
    b += a256((size_t) cap * 8);
    s.grp_start = reinterpret_cast<int32_t*>(b);
    b += a256((size_t) (cap + 1) * 4);
    s.n_groups = reinterpret_cast<int32_t*>(b);
    b += a256(4);
    s.ent_dst = reinterpret_cast<int32_t*>(b);
    b += a256((size_t) cap * 4);
    s.ent_tok = reinterpret_cast<int32_t*>(b);
    return s;
}

cudaError_t launch_s2_pack(const uint8_t* gate, const uint8_t* up, const uint8_t* down, int H, int F, uint8_t* blob,
                           cudaStream_t s) {
    const int64_t n = (int64_t) 2 * F * (H / 64) + (int64_t) H * (F / 64);
    s2_pack_kernel<<<(unsigned) std::min<int64_t>((n + 255) / 256, 148 * 16), 256, 0, s>>>(gate, up, down, H, F, blob);
    return cudaGetLastError();
}

cudaError_t launch_quant_q8_0(const float* x, int64_t n, uint8_t* y, float* scales, cudaStream_t s) {
    const int64_t blocks = (n / 32 + 7) / 8;
    quant_q8_0_kernel<<<(unsigned) std::min<int64_t>(std::max<int64_t>(blocks, 1), 148 * 16), 256, 0, s>>>(x, n / 32, y,
                                                                                                         scales);
    return cudaGetLastError();
}

cudaError_t launch_s2_grouped(const unsigned long long* grp_ptr, const int32_t* grp_start, const int32_t* n_groups,
                              const int32_t* ent_dst, const int32_t* ent_tok, int cap_groups, int cap_entries, int H,
                              int F, const uint8_t* xq, const float* xs, void* scratch, float* out, cudaStream_t s) {
    const S2Scratch sc = s2_scratch_at(scratch, cap_entries, F);
    S2Args a{grp_ptr, grp_start, n_groups, ent_dst, ent_tok, cap_groups, cap_entries, H, F, xq, xs, sc.hf, sc.hq,
             sc.hs, out};
    const int grid = s2_grid();
    s2_gate_up_kernel<<<grid, kS2Threads, 0, s>>>(a);
    s2_quant_h_kernel<<<grid, kS2Threads, 0, s>>>(a);
    s2_down_kernel<<<grid, kS2Threads, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_s2_group_resident(const int32_t* ids, int n, int k_per_tok, const uint8_t* base, int64_t blob,
                                     unsigned long long* grp_ptr, int32_t* grp_start, int32_t* counts, int32_t* ent_dst,
                                     int32_t* ent_tok, cudaStream_t s) {
    s2_group_resident_kernel<<<1, 1024, 0, s>>>(ids, n, k_per_tok, base, blob, grp_ptr, grp_start, counts, ent_dst,
                                                ent_tok);
    return cudaGetLastError();
}

cudaError_t launch_s2_hit_select(const int32_t* ids, const int32_t* res_row, int n, int n_expert, int32_t* slot,
                                 int32_t* dst, int32_t* count, cudaStream_t s) {
    s2_hit_select_kernel<<<1, 1024, 0, s>>>(ids, res_row, n, n_expert, slot, dst, count);
    return cudaGetLastError();
}

cudaError_t launch_s2_hits(const uint8_t* base, const int32_t* slot_index, const int32_t* dst_index,
                           const int32_t* d_count, int cap, int64_t blob_bytes, int H, int F, const uint8_t* xq,
                           const float* xs, int k_per_token, void* scratch, float* out, cudaStream_t s) {
    const S2Scratch sc = s2_scratch_at(scratch, cap, F);
    s2_hits_to_groups_kernel<<<(cap + 256) / 256, 256, 0, s>>>(base, slot_index, dst_index, d_count, cap, blob_bytes,
                                                               k_per_token, sc.grp_ptr, sc.grp_start, sc.n_groups,
                                                               sc.ent_dst, sc.ent_tok);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return launch_s2_grouped(sc.grp_ptr, sc.grp_start, sc.n_groups, sc.ent_dst, sc.ent_tok, cap, cap, H, F, xq, xs,
                             scratch, out, s);
}

cudaError_t launch_s2_hit_add(float* parts, const float* hit_out, const int32_t* dst, const int32_t* count, int cap,
                              int64_t H, cudaStream_t s) {
    const int64_t n = (int64_t) cap * H;
    s2_hit_add_kernel<<<(unsigned) std::min<int64_t>((n + 255) / 256, 148 * 16), 256, 0, s>>>(parts, hit_out, dst,
                                                                                            count, cap, H);
    return cudaGetLastError();
}

}  // namespace smoe
