// expert.cu - dequant-fused grouped expert GEMVs on sm_100a (rows a5-a9 of the block).
//
// Work is grouped by expert: every (expert, row tile) item stages its weight rows into shared memory with
// one bulk copy (cp.async.bulk, the TMA engine without a tensor map: 16-byte aligned tiles of whole rows),
// keeps its rows' codes in registers, and walks the expert's tokens (slots).  Each weight byte is read from
// HBM once per launch however many tokens the expert has.
//
// Summation order.  Row r against a q8_1 column is the reference's iq_mmvq (iq.metal:459-514) and its host
// transcription row_dot (iq_parity.cpp:275-292): the 32-value partial k (a Q2_0 half block, an IQ2_S 32-group)
// is added to lane k & 31 in order, then the 32 lane sums meet in an xor butterfly 16, 8, 4, 2, 1.  The kernels
// here give every lane exactly those partials and reduce several rows at once with a transposed butterfly:
// at level L a lane keeps half of its rows, sends the other half to lane ^ L and adds what it receives, so
// every row's sum is formed from the same pairs as the reference's butterfly.  The result is bitwise the host
// reference.
//
// Q2_0 integer dot.  A qs word holds 16 codes (4 per byte, LSB first).  Instead of unpacking codes to bytes,
// the activation is re-laid out once per token so that byte b of word j holds value 4b + j of a 16-value run;
// then (qs & (3 << 2j)) against that word is a dp4a of code * 4^j, and
//   sum (code - 1) q = sum_j (dp4a_j >> 2j) - sum q       (exact integer arithmetic).
#include "common.cuh"
#include "kernels.cuh"
#include "q8.cuh"

#include <type_traits>

namespace smoe {

__device__ const uint64_t k_iq2s_grid_dev[1024] = {
#include "iq2s_grid.inc"
};

constexpr int kThreads = 256;  // 8 warps
constexpr int kSlotChunk = 8;  // tokens staged per pass

// ------------------------------------------------------------------------------------------------
// group helpers
// ------------------------------------------------------------------------------------------------
struct Item {
    int e;        // routed expert id (or 0 for single); -1 for the shared expert
    int beg, end; // slots
    bool shared;
};

__device__ __forceinline__ int group_count(const GroupView& g) {
    if (g.single_cols > 0) return 1;
    return (g.no_routed ? 0 : *g.n_active) + (g.shared_slots > 0 ? 1 : 0);
}

__device__ __forceinline__ Item group_item(const GroupView& g, int j) {
    Item it;
    if (g.single_cols > 0) {
        it.e = 0; it.beg = 0; it.end = g.single_cols; it.shared = false;
        return it;
    }
    const int na = g.no_routed ? 0 : *g.n_active;
    if (j < na) {
        it.e = g.active[j]; it.beg = g.offsets[it.e]; it.end = g.offsets[it.e + 1]; it.shared = false;
    } else {
        it.e = -1; it.beg = g.shared_base; it.end = g.shared_base + g.shared_slots; it.shared = true;
    }
    return it;
}

__device__ __forceinline__ int slot_token(const GroupView& g, const Item& it, int slot) {
    if (g.single_cols > 0) return slot;
    if (it.shared) return slot - g.shared_base;
    return g.slot_token[slot];
}

// ------------------------------------------------------------------------------------------------
// shared-memory loads and the partial dots
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lds_u32_unaligned(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t) 3);
    const uint32_t sh = (uint32_t) (a & 3) * 8u;
    return __funnelshift_r(base[0], base[1], sh);
}

__device__ __forceinline__ uint16_t lds_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// One staged q8_1 block: 8 words (re-laid out for Q2_0, natural order for IQ2_S), d as f32, sum of the q.
struct ActBlock {
    uint32_t w[8];
};

// Q2_0 weights of one partial (a 32-value half block): two qs words and d.
struct Q2W {
    uint32_t w0, w1;
    float d;
};

__device__ __forceinline__ Q2W q2_weights(const uint8_t* row, int k) {
    const uint8_t* blk = row + (k >> 1) * 18;
    Q2W q;
    q.d = f16_to_f32(lds_u16(blk));
    const uint8_t* qs = blk + 2 + 8 * (k & 1);
    q.w0 = lds_u32_unaligned(qs);
    q.w1 = lds_u32_unaligned(qs + 4);
    return q;
}

__device__ __forceinline__ float q2_partial(const Q2W& q, const uint32_t* a, float dx, int qsum) {
    const int s0 = dp4a_us(q.w1 & 0x03030303u, (int) a[4], dp4a_us(q.w0 & 0x03030303u, (int) a[0], 0));
    const int s1 = dp4a_us(q.w1 & 0x0C0C0C0Cu, (int) a[5], dp4a_us(q.w0 & 0x0C0C0C0Cu, (int) a[1], 0));
    const int s2 = dp4a_us(q.w1 & 0x30303030u, (int) a[6], dp4a_us(q.w0 & 0x30303030u, (int) a[2], 0));
    const int s3 = dp4a_us(q.w1 & 0xC0C0C0C0u, (int) a[7], dp4a_us(q.w0 & 0xC0C0C0C0u, (int) a[3], 0));
    const int sumi = s0 + (s1 >> 2) + (s2 >> 4) + (s3 >> 6) - qsum;
    return __fmul_rn(__fmul_rn(q.d, dx), (float) sumi);
}

// IQ2_S weights of one partial (32-group g of a 256-block): qs word, sign word, qh and scale bytes, d.
struct S2W {
    uint32_t qs, sg, hs;  // hs = qh | scale << 8
    float d;
};

__device__ __forceinline__ S2W s2_weights(const uint8_t* row, int k) {
    const uint8_t* blk = row + (k >> 3) * 82;
    const int g = k & 7;
    S2W w;
    w.d = f16_to_f32(lds_u16(blk));
    w.qs = lds_u32_unaligned(blk + 2 + 4 * g);
    w.sg = lds_u32_unaligned(blk + 34 + 4 * g);
    w.hs = (uint32_t) blk[66 + g] | ((uint32_t) blk[74 + g] << 8);
    return w;
}

// Bytes 0xFF where bit m of the 4-bit s is set (m = byte index).
__device__ __forceinline__ uint32_t sign_mask4(uint32_t s) { return ((s * 0x00204081u) & 0x01010101u) * 0xFFu; }

// IQ2_S partial (iq_parity.cpp:125-151): the codebook magnitudes are never 0, so negating a byte as
// (m ^ 0xFF) + 1 never carries into its neighbour.
__device__ __forceinline__ float s2_partial(const S2W& w, const uint32_t* a, float dx, const uint64_t* grid) {
    int sum0 = 0, sum1 = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t idx = ((w.qs >> (8 * j)) & 0xFFu) | (((w.hs >> (2 * j)) & 3u) << 8);
        const uint64_t e = grid[idx];
        const uint32_t sb = (w.sg >> (8 * j)) & 0xFFu;
        const uint32_t mlo = sign_mask4(sb & 0xFu), mhi = sign_mask4(sb >> 4);
        const uint32_t vlo = ((uint32_t) e ^ mlo) + (mlo & 0x01010101u);
        const uint32_t vhi = ((uint32_t) (e >> 32) ^ mhi) + (mhi & 0x01010101u);
        const int s = dp4a_ss((int) vhi, (int) a[2 * j + 1], dp4a_ss((int) vlo, (int) a[2 * j], 0));
        if (j < 2) sum0 += s;
        else sum1 += s;
    }
    const int sc = (int) (w.hs >> 8);
    const int ls0 = sc & 0x0F, ls1 = sc >> 4;
    const int sumi = (sum0 * ls0 + sum1 * ls1 + (sum0 + sum1) / 2) / 4;
    return __fmul_rn(__fmul_rn(w.d, dx), (float) sumi);
}

// Stage one q8_1 block (36 bytes at src, 4-byte aligned) into the kernel layout.
template <int TYPE>
__device__ __forceinline__ void stage_block(const uint8_t* __restrict__ src, uint32_t* __restrict__ dst_w,
                                            float* __restrict__ dst_d, int* __restrict__ dst_s) {
    const uint32_t* s32 = reinterpret_cast<const uint32_t*>(src);
    uint32_t x[8];
#pragma unroll
    for (int i = 0; i < 8; i++) x[i] = __ldg(s32 + 1 + i);
    int qs = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) qs = dp4a_ss((int) x[i], 0x01010101, qs);
    if (TYPE == kQ2_0) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t* X = x + 4 * h;
            const uint32_t t0 = __byte_perm(X[0], X[1], 0x5140), t1 = __byte_perm(X[2], X[3], 0x5140);
            const uint32_t t2 = __byte_perm(X[0], X[1], 0x7362), t3 = __byte_perm(X[2], X[3], 0x7362);
            dst_w[4 * h + 0] = __byte_perm(t0, t1, 0x5410);
            dst_w[4 * h + 1] = __byte_perm(t0, t1, 0x7632);
            dst_w[4 * h + 2] = __byte_perm(t2, t3, 0x5410);
            dst_w[4 * h + 3] = __byte_perm(t2, t3, 0x7632);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) dst_w[i] = x[i];
    }
    *dst_d = f16_to_f32((uint16_t) (s32[0] & 0xFFFFu));
    *dst_s = qs;
}

// Transposed butterfly: NV values per lane (power of two), levels LV0, LV0/2, ..., 1.  Afterwards v[0]
// holds, in every lane, the full sum of output index o(lane) whose bits are the lane bits of the halving
// levels, most significant first.
template <int NV, int LV0>
__device__ __forceinline__ void tbfly(float (&v)[NV], int lane) {
    int n = NV;
#pragma unroll
    for (int lvl = LV0; lvl >= 1; lvl >>= 1) {
        if (n > 1) {
            const bool upper = (lane & lvl) != 0;
            const int half = n >> 1;
#pragma unroll
            for (int i = 0; i < NV / 2; i++) {
                if (i < half) {
                    const float send = upper ? v[i] : v[i + half];
                    const float keep = upper ? v[i + half] : v[i];
                    v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, lvl));
                }
            }
            n = half;
        } else {
            v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], lvl));
        }
    }
}

// ------------------------------------------------------------------------------------------------
// gate/up + SwiGLU + q8_1 of h.  Item = (expert, 32-row tile of n_ff).  Warp w owns tile rows w, w+8,
// w+16, w+24 of both gate and up; lane L owns partials L, L+32, ... (PPL of them).
// ------------------------------------------------------------------------------------------------
template <int TYPE, int PPL>
__global__ void __launch_bounds__(kThreads) expert_gate_up_kernel(Matrix gate, Matrix up, Matrix sgate, Matrix sup,
                                                                  GroupView g, const uint8_t* __restrict__ xq,
                                                                  uint8_t* __restrict__ hq, int H, int F) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rb = (TYPE == kQ2_0) ? (H / 64) * 18 : (H / 256) * 82;
    const int nblk = H / 32;                 // q8_1 blocks of a token = partials of a row
    const int tile_bytes = 32 * rb;
    uint8_t* wbuf = smem;                                                      // [2][32][rb]
    uint32_t* aw = reinterpret_cast<uint32_t*>(smem + ((2 * tile_bytes + 16 + 127) & ~127));  // [chunk][nblk][8]
    float* ad = reinterpret_cast<float*>(aw + kSlotChunk * nblk * 8);          // [chunk][nblk]
    int* as = reinterpret_cast<int*>(ad + kSlotChunk * nblk);                  // [chunk][nblk]
    float* htile = reinterpret_cast<float*>(as + kSlotChunk * nblk);           // [chunk][32]
    uint64_t* grid_s = reinterpret_cast<uint64_t*>(htile + kSlotChunk * 32);   // [1024] (IQ2_S)
    uint64_t* bar = grid_s + (TYPE == kIQ2_S ? 1024 : 0);
    __shared__ int s_ok;

    if (TYPE == kIQ2_S)
        for (int i = tid; i < 1024; i += kThreads) grid_s[i] = k_iq2s_grid_dev[i];
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();

    const int n_tiles = F / 32;
    const int n_items = group_count(g) * n_tiles;
    const int hq_row = (F / 32) * kQ8Block;
    uint32_t phase = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int j = item / n_tiles, tt = item % n_tiles;
        const Item it = group_item(g, j);
        const uint8_t* gsrc = it.shared ? sgate.base : gate.base + (int64_t) it.e * gate.expert_stride;
        const uint8_t* usrc = it.shared ? sup.base : up.base + (int64_t) it.e * up.expert_stride;
        if (tid == 0) {
            fence_proxy_async();
            mbar_expect_tx(bar, 2u * (uint32_t) tile_bytes);
            bulk_g2s(wbuf, gsrc + (int64_t) tt * tile_bytes, (uint32_t) tile_bytes, bar);
            bulk_g2s(wbuf + tile_bytes, usrc + (int64_t) tt * tile_bytes, (uint32_t) tile_bytes, bar);
            bool ok = mbar_wait_bounded(bar, phase, kWaitLimitNs);
            if (!ok) {
                atomicOr(&g_smoe_status, kDevTimeout);
                mbar_wait_bounded(bar, phase, kWaitLimitNs);
            }
            s_ok = ok ? 1 : 0;
        }
        __syncthreads();
        if (!s_ok) return;
        (void) mbar_try_wait(bar, phase);  // acquire the copied bytes in every thread
        phase ^= 1u;

        // this warp's rows: tile rows warp + 8 i, i = 0..3, of gate (v[i]) and up (v[4 + i])
        using WT = typename std::conditional<TYPE == kQ2_0, Q2W, S2W>::type;
        WT wg[4][PPL], wu[4][PPL];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint8_t* rg = wbuf + (warp + 8 * i) * rb;
            const uint8_t* ru = wbuf + tile_bytes + (warp + 8 * i) * rb;
#pragma unroll
            for (int p = 0; p < PPL; p++) {
                const int k = lane + 32 * p;
                if (k < nblk) {
                    if constexpr (TYPE == kQ2_0) { wg[i][p] = q2_weights(rg, k); wu[i][p] = q2_weights(ru, k); }
                    else { wg[i][p] = s2_weights(rg, k); wu[i][p] = s2_weights(ru, k); }
                }
            }
        }

        for (int c0 = it.beg; c0 < it.end; c0 += kSlotChunk) {
            const int nc = min(kSlotChunk, it.end - c0);
            __syncthreads();  // previous chunk's staging and htile are consumed
            for (int q = tid; q < nc * nblk; q += kThreads) {
                const int s = q / nblk, b = q % nblk;
                const int tok = slot_token(g, it, c0 + s);
                stage_block<TYPE>(xq + ((int64_t) tok * nblk + b) * kQ8Block, aw + (s * nblk + b) * 8,
                                  ad + s * nblk + b, as + s * nblk + b);
            }
            __syncthreads();
            for (int s = 0; s < nc; s++) {
                float v[8];
#pragma unroll
                for (int i = 0; i < 8; i++) v[i] = 0.f;
#pragma unroll
                for (int p = 0; p < PPL; p++) {
                    const int k = lane + 32 * p;
                    if (k < nblk) {
                        const uint32_t* a = aw + (s * nblk + k) * 8;
                        uint32_t av[8];
#pragma unroll
                        for (int q = 0; q < 8; q++) av[q] = a[q];
                        const float dx = ad[s * nblk + k];
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            if constexpr (TYPE == kQ2_0) {
                                const int qsum = as[s * nblk + k];
                                v[i] = __fadd_rn(v[i], q2_partial(wg[i][p], av, dx, qsum));
                                v[4 + i] = __fadd_rn(v[4 + i], q2_partial(wu[i][p], av, dx, qsum));
                            } else {
                                v[i] = __fadd_rn(v[i], s2_partial(wg[i][p], av, dx, grid_s));
                                v[4 + i] = __fadd_rn(v[4 + i], s2_partial(wu[i][p], av, dx, grid_s));
                            }
                        }
                    }
                }
                tbfly<8, 16>(v, lane);
                // lane holds output 4*b4 + 2*b3 + b2: b4 = 0 gate, 1 up; row i = 2*b3 + b2
                const float other = __shfl_xor_sync(0xffffffffu, v[0], 16);
                if ((lane & 19) == 0) {
                    const int i = (lane >> 2) & 3;
                    htile[s * 32 + warp + 8 * i] = silu_mul(v[0], other);
                }
            }
            __syncthreads();
            for (int s = warp; s < nc; s += kThreads / 32)
                quant_q8_1_warp(htile[s * 32 + lane], hq + (int64_t) (c0 + s) * hq_row + tt * kQ8Block, lane);
        }
        __syncthreads();  // every thread is done with wbuf before the next copy is issued
    }
}

// ------------------------------------------------------------------------------------------------
// Matrix rows against staged q8_1 columns: y[slot][r] = W_e[r] . act[row(slot)].
// Lane groups of LPR lanes own one row each in RPG rows; lane l of a group owns partials l, l + LPR, ...
// (PPL of them).  LPR = 16 is exact against the reference when a row has at most 16 partials: its lanes
// 16..31 hold zeros and the butterfly's first level adds nothing.
// ------------------------------------------------------------------------------------------------
template <int TYPE, int LPR, int PPL>
__global__ void __launch_bounds__(kThreads) expert_rows_kernel(Matrix wm, Matrix swm, GroupView g,
                                                               const uint8_t* __restrict__ act, int act_by_token,
                                                               float* __restrict__ y, int64_t y_stride, int n_in,
                                                               int n_out) {
    constexpr int RPG = 4;
    constexpr int GROUPS = 32 / LPR;
    constexpr int ROWS = (kThreads / 32) * GROUPS * RPG;  // rows per tile
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane / LPR, gl = lane % LPR;
    const int rb = (TYPE == kQ2_0) ? (n_in / 64) * 18 : (n_in / 256) * 82;
    const int nblk = n_in / 32;
    uint8_t* wbuf = smem;  // [ROWS][rb] (+16 slack)
    uint32_t* aw = reinterpret_cast<uint32_t*>(smem + ((ROWS * rb + 16 + 127) & ~127));
    float* ad = reinterpret_cast<float*>(aw + kSlotChunk * nblk * 8);
    int* as = reinterpret_cast<int*>(ad + kSlotChunk * nblk);
    uint64_t* grid_s = reinterpret_cast<uint64_t*>(as + kSlotChunk * nblk + 2);
    uint64_t* bar = grid_s + (TYPE == kIQ2_S ? 1024 : 0);
    __shared__ int s_ok;

    if (TYPE == kIQ2_S)
        for (int i = tid; i < 1024; i += kThreads) grid_s[i] = k_iq2s_grid_dev[i];
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();

    const int n_tiles = (n_out + ROWS - 1) / ROWS;
    const int n_items = group_count(g) * n_tiles;
    uint32_t phase = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int j = item / n_tiles, tt = item % n_tiles;
        const Item it = group_item(g, j);
        const uint8_t* src = it.shared ? swm.base : wm.base + (int64_t) it.e * wm.expert_stride;
        const int r0 = tt * ROWS;
        const int nrows = min(ROWS, n_out - r0);
        // whole 16-byte units by one bulk copy; a ragged tail (rows whose bytes are not a multiple of 16)
        // by plain loads, so nothing past the matrix is read
        const uint32_t bytes = (uint32_t) (nrows * rb);
        const uint32_t bulk = bytes & ~15u;
        for (uint32_t b = bulk + tid; b < bytes; b += kThreads) wbuf[b] = src[(int64_t) r0 * rb + b];
        if (tid == 0) {
            fence_proxy_async();
            mbar_expect_tx(bar, bulk);
            if (bulk) bulk_g2s(wbuf, src + (int64_t) r0 * rb, bulk, bar);
            bool ok = mbar_wait_bounded(bar, phase, kWaitLimitNs);
            if (!ok) {
                atomicOr(&g_smoe_status, kDevTimeout);
                mbar_wait_bounded(bar, phase, kWaitLimitNs);
            }
            s_ok = ok ? 1 : 0;
        }
        __syncthreads();
        if (!s_ok) return;
        (void) mbar_try_wait(bar, phase);
        phase ^= 1u;

        using WT = typename std::conditional<TYPE == kQ2_0, Q2W, S2W>::type;
        WT wr[RPG][PPL];
        const int row_base = (warp * GROUPS + grp) * RPG;  // tile row of this group's v[0]
#pragma unroll
        for (int i = 0; i < RPG; i++) {
            const int r = min(row_base + i, nrows - 1);
            const uint8_t* rp = wbuf + r * rb;
#pragma unroll
            for (int p = 0; p < PPL; p++) {
                const int k = gl + LPR * p;
                if (k < nblk) {
                    if constexpr (TYPE == kQ2_0) wr[i][p] = q2_weights(rp, k);
                    else wr[i][p] = s2_weights(rp, k);
                }
            }
        }
        for (int c0 = it.beg; c0 < it.end; c0 += kSlotChunk) {
            const int nc = min(kSlotChunk, it.end - c0);
            __syncthreads();
            for (int q = tid; q < nc * nblk; q += kThreads) {
                const int s = q / nblk, b = q % nblk;
                const int arow = act_by_token ? slot_token(g, it, c0 + s) : c0 + s;
                stage_block<TYPE>(act + ((int64_t) arow * nblk + b) * kQ8Block, aw + (s * nblk + b) * 8,
                                  ad + s * nblk + b, as + s * nblk + b);
            }
            __syncthreads();
            for (int s = 0; s < nc; s++) {
                float v[RPG];
#pragma unroll
                for (int i = 0; i < RPG; i++) v[i] = 0.f;
#pragma unroll
                for (int p = 0; p < PPL; p++) {
                    const int k = gl + LPR * p;
                    if (k < nblk) {
                        const uint32_t* a = aw + (s * nblk + k) * 8;
                        uint32_t av[8];
#pragma unroll
                        for (int q = 0; q < 8; q++) av[q] = a[q];
                        const float dx = ad[s * nblk + k];
#pragma unroll
                        for (int i = 0; i < RPG; i++) {
                            if constexpr (TYPE == kQ2_0)
                                v[i] = __fadd_rn(v[i], q2_partial(wr[i][p], av, dx, as[s * nblk + k]));
                            else
                                v[i] = __fadd_rn(v[i], s2_partial(wr[i][p], av, dx, grid_s));
                        }
                    }
                }
                tbfly<RPG, LPR / 2>(v, lane);
                // lane holds row 2 * b(LPR/2) + b(LPR/4) of its group; lanes with the low bits clear store
                constexpr int low_mask = LPR / 4 - 1;
                if ((gl & low_mask) == 0) {
                    const int i = (gl / (LPR / 4)) & 3;
                    const int r = row_base + i;
                    if (r < nrows) y[(int64_t) (c0 + s) * y_stride + r0 + r] = v[0];
                }
            }
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------------------------------------
// launchers
// ------------------------------------------------------------------------------------------------
static int sm_count() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

template <typename K>
static cudaError_t launch_persistent(K kernel, size_t smem, int max_items, cudaStream_t s, dim3* out_grid) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (err != cudaSuccess) return err;
    int per_sm = 0;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (err != cudaSuccess) return err;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    int blocks = sm_count() * per_sm;
    if (max_items < blocks) blocks = max_items > 0 ? max_items : 1;
    *out_grid = dim3((unsigned) blocks);
    return cudaSuccess;
}

static int max_groups(const GroupView& g) {
    if (g.single_cols > 0) return 1;
    return (g.no_routed ? 0 : g.max_active) + (g.shared_slots > 0 ? 1 : 0);
}

cudaError_t launch_expert_gate_up(Matrix gate, Matrix up, Matrix sgate, Matrix sup, GroupView g, const uint8_t* xq,
                                  uint8_t* hq, int n_embd, int n_ff, cudaStream_t s) {
    const int type = gate.type;
    const int rb = type == kQ2_0 ? (n_embd / 64) * 18 : (n_embd / 256) * 82;
    const int nblk = n_embd / 32;
    size_t smem = ((size_t) (2 * 32 * rb + 16 + 127) & ~(size_t) 127) + (size_t) kSlotChunk * nblk * 40 +
                  kSlotChunk * 32 * 4 + (type == kIQ2_S ? 8192 : 0) + 16;
    const int ppl = (nblk + 31) / 32;
    const int max_items = max_groups(g) * (n_ff / 32);
    dim3 grid;
    cudaError_t err;
#define SMOE_GU(T_, P_)                                                                                        \
    do {                                                                                                       \
        err = launch_persistent(expert_gate_up_kernel<T_, P_>, smem, max_items, s, &grid);                    \
        if (err != cudaSuccess) return err;                                                                    \
        expert_gate_up_kernel<T_, P_><<<grid, kThreads, smem, s>>>(gate, up, sgate, sup, g, xq, hq, n_embd,    \
                                                                   n_ff);                                      \
    } while (0)
    if (type == kQ2_0) {
        if (ppl == 1) SMOE_GU(kQ2_0, 1);
        else if (ppl == 2) SMOE_GU(kQ2_0, 2);
        else if (ppl == 3) SMOE_GU(kQ2_0, 3);
        else SMOE_GU(kQ2_0, 4);
    } else {
        if (ppl == 1) SMOE_GU(kIQ2_S, 1);
        else if (ppl == 2) SMOE_GU(kIQ2_S, 2);
        else if (ppl == 3) SMOE_GU(kIQ2_S, 3);
        else SMOE_GU(kIQ2_S, 4);
    }
#undef SMOE_GU
    return cudaGetLastError();
}

cudaError_t launch_expert_down(Matrix down, Matrix sdown, GroupView g, const uint8_t* act, int act_by_token,
                               float* y, int64_t y_stride, int n_in, int n_out, cudaStream_t s) {
    const int type = down.type;
    const int rb = type == kQ2_0 ? (n_in / 64) * 18 : (n_in / 256) * 82;
    const int nblk = n_in / 32;
    const int lpr = nblk <= 16 ? 16 : 32;
    const int ppl = (nblk + lpr - 1) / lpr;
    const int rows = (kThreads / 32) * (32 / lpr) * 4;
    size_t smem = ((size_t) (rows * rb + 16 + 127) & ~(size_t) 127) + (size_t) kSlotChunk * nblk * 40 + 16 +
                  (type == kIQ2_S ? 8192 : 0) + 16;
    const int max_items = max_groups(g) * ((n_out + rows - 1) / rows);
    dim3 grid;
    cudaError_t err;
#define SMOE_ROWS(T_, L_, P_)                                                                                  \
    do {                                                                                                       \
        err = launch_persistent(expert_rows_kernel<T_, L_, P_>, smem, max_items, s, &grid);                   \
        if (err != cudaSuccess) return err;                                                                    \
        expert_rows_kernel<T_, L_, P_><<<grid, kThreads, smem, s>>>(down, sdown, g, act, act_by_token, y,      \
                                                                    y_stride, n_in, n_out);                    \
    } while (0)
    if (type == kQ2_0) {
        if (lpr == 16) SMOE_ROWS(kQ2_0, 16, 1);
        else if (ppl == 1) SMOE_ROWS(kQ2_0, 32, 1);
        else if (ppl == 2) SMOE_ROWS(kQ2_0, 32, 2);
        else if (ppl == 3) SMOE_ROWS(kQ2_0, 32, 3);
        else SMOE_ROWS(kQ2_0, 32, 4);
    } else {
        if (lpr == 16) SMOE_ROWS(kIQ2_S, 16, 1);
        else if (ppl == 1) SMOE_ROWS(kIQ2_S, 32, 1);
        else if (ppl == 2) SMOE_ROWS(kIQ2_S, 32, 2);
        else if (ppl == 3) SMOE_ROWS(kIQ2_S, 32, 3);
        else SMOE_ROWS(kIQ2_S, 32, 4);
    }
#undef SMOE_ROWS
    return cudaGetLastError();
}

}  // namespace smoe
