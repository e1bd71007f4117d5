// expert.cu - dequant-fused grouped expert GEMVs on sm_100a (rows a5-a9 of the block).
//
// Work is grouped by expert: every (expert, row tile) item is one bulk copy (cp.async.bulk, the TMA engine
// without a tensor map: a 16-byte aligned tile of whole rows) into a ring of kStages shared-memory stages, so
// a CTA keeps several tiles in flight while it computes.  Each warp decodes its rows' codes into registers
// once per item and walks the expert's tokens (slots).  Each weight byte is read from HBM once per launch
// however many tokens the expert has.
//
// Summation order.  Row r against a q8_1 column is the reference's iq_mmvq (iq.metal:459-514) and its host
// transcription row_dot (iq_parity.cpp:275-292): the 32-value partial k (a Q2_0 half block, an IQ2_S 32-group)
// is added to lane k & 31 in order, then the 32 lane sums meet in an xor butterfly 16, 8, 4, 2, 1.  The kernels
// here give every lane exactly those partials and reduce several rows at once with a transposed butterfly:
// at level L a lane keeps half of its rows, sends the other half to lane ^ L and adds what it receives, so
// every row's sum is formed from the same pairs as the reference's butterfly.  The result is bitwise the host
// reference.
//
// Q2_0 integer dot.  A qs word holds 16 codes (4 per byte, LSB first).  (qs >> 2j) & 0x03030303 holds, in
// byte b, the code of value 4b + j; the activation is re-laid out once per token to match (byte b of word j
// = value 4b + j of a 16-value run), so eight chained dp4a give sum code * q exactly and
//   sum (code - 1) q = sum code * q - sum q       (exact integer arithmetic; sum q is staged per block).
#include "common.cuh"
#include "ep.cuh"
#include "kernels.cuh"
#include "q8.cuh"

#include <type_traits>

namespace smoe {

__device__ const uint64_t k_iq2s_grid_dev[1024] = {
#include "iq2s_grid.inc"
};

constexpr int kSlotChunk = 8;  // tokens staged per pass
constexpr int kStages = 4;     // weight tiles in flight per CTA

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
// shared-memory loads, decoding and the partial dots
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lds_u32_unaligned(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t) 3);
    const uint32_t sh = (uint32_t) (a & 3) * 8u;
    return __funnelshift_r(base[0], base[1], sh);
}

__device__ __forceinline__ uint16_t lds_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// One 32-value partial of a weight row, decoded: eight code words that pair with the eight staged
// activation words of the matching q8_1 block, the block scale, and (IQ2_S) the two 4-bit sub-scales.
struct Dec {
    uint32_t c[8];
    float d;
    uint32_t ls;
};

// Q2_0 half block k & 1 of block k >> 1: c[j] = codes of values 4b + j (j < 4) of the first 16 values,
// c[4 + j] the same for the last 16.
__device__ __forceinline__ void decode_q2(const uint8_t* row, int k, Dec& w) {
    const uint8_t* blk = row + (k >> 1) * 18;
    w.d = f16_to_f32(lds_u16(blk));
    const uint8_t* qs = blk + 2 + 8 * (k & 1);
    const uint32_t w0 = lds_u32_unaligned(qs), w1 = lds_u32_unaligned(qs + 4);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        w.c[j] = (w0 >> (2 * j)) & 0x03030303u;
        w.c[4 + j] = (w1 >> (2 * j)) & 0x03030303u;
    }
    w.ls = 0;
}

// Bytes 0xFF where bit m of the 4-bit s is set (m = byte index).
__device__ __forceinline__ uint32_t sign_mask4(uint32_t s) { return ((s * 0x00204081u) & 0x01010101u) * 0xFFu; }

// IQ2_S 32-group k & 7 of block k >> 3 (format iq.metal:152-180): each 8-value chunk j is codebook entry
// qs[4g + j] | ((qh[g] >> 2j) & 3) << 8, value m negated when bit m of signs[4g + j] is set.  The codebook
// magnitudes are never 0, so negating a byte as (m ^ 0xFF) + 1 never carries into its neighbour.
__device__ __forceinline__ void decode_s2(const uint8_t* row, int k, const uint64_t* grid, Dec& w) {
    const uint8_t* blk = row + (k >> 3) * 82;
    const int g = k & 7;
    w.d = f16_to_f32(lds_u16(blk));
    const uint32_t qs = lds_u32_unaligned(blk + 2 + 4 * g);
    const uint32_t sg = lds_u32_unaligned(blk + 34 + 4 * g);
    const uint32_t qh = blk[66 + g];
    const uint32_t sc = blk[74 + g];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t idx = ((qs >> (8 * j)) & 0xFFu) | (((qh >> (2 * j)) & 3u) << 8);
        const uint64_t e = grid[idx];
        const uint32_t sb = (sg >> (8 * j)) & 0xFFu;
        const uint32_t mlo = sign_mask4(sb & 0xFu), mhi = sign_mask4(sb >> 4);
        w.c[2 * j] = ((uint32_t) e ^ mlo) + (mlo & 0x01010101u);
        w.c[2 * j + 1] = ((uint32_t) (e >> 32) ^ mhi) + (mhi & 0x01010101u);
    }
    w.ls = (sc & 0x0Fu) | ((sc >> 4) << 8);
}

template <int TYPE>
__device__ __forceinline__ void decode(const uint8_t* row, int k, const uint64_t* grid, Dec& w) {
    if constexpr (TYPE == kQ2_0) decode_q2(row, k, w);
    else decode_s2(row, k, grid, w);
}

// (float) v for |v| < 2^22 with two full-rate ops instead of a conversion: 1.5 * 2^23 + v is exact in f32.
__device__ __forceinline__ float int_to_float_exact(int v) {
    return __fsub_rn(__int_as_float(0x4B400000 + v), 12582912.0f);
}

// The partial (d_w * d_x) * sumi with the reference's two float multiplies (iq_parity.cpp:148-150, 247-251).
template <int TYPE>
__device__ __forceinline__ float partial(const Dec& w, const uint4& a0, const uint4& a1, float dx, int qsum) {
    int sumi;
    if constexpr (TYPE == kQ2_0) {
        int s = dp4a_us(w.c[0], (int) a0.x, 0);
        s = dp4a_us(w.c[1], (int) a0.y, s);
        s = dp4a_us(w.c[2], (int) a0.z, s);
        s = dp4a_us(w.c[3], (int) a0.w, s);
        s = dp4a_us(w.c[4], (int) a1.x, s);
        s = dp4a_us(w.c[5], (int) a1.y, s);
        s = dp4a_us(w.c[6], (int) a1.z, s);
        s = dp4a_us(w.c[7], (int) a1.w, s);
        sumi = s - qsum;
    } else {
        int s0 = dp4a_ss((int) w.c[0], (int) a0.x, 0);
        s0 = dp4a_ss((int) w.c[1], (int) a0.y, s0);
        s0 = dp4a_ss((int) w.c[2], (int) a0.z, s0);
        s0 = dp4a_ss((int) w.c[3], (int) a0.w, s0);
        int s1 = dp4a_ss((int) w.c[4], (int) a1.x, 0);
        s1 = dp4a_ss((int) w.c[5], (int) a1.y, s1);
        s1 = dp4a_ss((int) w.c[6], (int) a1.z, s1);
        s1 = dp4a_ss((int) w.c[7], (int) a1.w, s1);
        const int ls0 = (int) (w.ls & 0xFFu), ls1 = (int) (w.ls >> 8);
        sumi = (s0 * ls0 + s1 * ls1 + (s0 + s1) / 2) / 4;
    }
    return __fmul_rn(__fmul_rn(w.d, dx), int_to_float_exact(sumi));
}

// Stage one q8_1 block (36 bytes at src, 4-byte aligned): Q2_0 gets the code-matched layout (byte b of word
// j = value 4b + j of each 16-value run), IQ2_S the natural order; also d as f32 and the sum of the q.
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
    uint32_t o[8];
    if (TYPE == kQ2_0) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t* X = x + 4 * h;
            const uint32_t t0 = __byte_perm(X[0], X[1], 0x5140), t1 = __byte_perm(X[2], X[3], 0x5140);
            const uint32_t t2 = __byte_perm(X[0], X[1], 0x7362), t3 = __byte_perm(X[2], X[3], 0x7362);
            o[4 * h + 0] = __byte_perm(t0, t1, 0x5410);
            o[4 * h + 1] = __byte_perm(t0, t1, 0x7632);
            o[4 * h + 2] = __byte_perm(t2, t3, 0x5410);
            o[4 * h + 3] = __byte_perm(t2, t3, 0x7632);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = x[i];
    }
    reinterpret_cast<uint4*>(dst_w)[0] = make_uint4(o[0], o[1], o[2], o[3]);
    reinterpret_cast<uint4*>(dst_w)[1] = make_uint4(o[4], o[5], o[6], o[7]);
    *dst_d = f16_to_f32((uint16_t) (__ldg(s32) & 0xFFFFu));
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
// The tile ring.  Thread 0 issues item i + kStages - 1 at the top of iteration i into the stage that item
// i - 1 released (every thread passed the barrier at the end of iteration i - 1).  Waits are bounded: on a
// timeout the status word is set, thread 0 waits (bounded again) for every copy still in flight, and the CTA
// returns.
// ------------------------------------------------------------------------------------------------
struct Ring {
    uint8_t* base;
    uint32_t stage_bytes;
    uint64_t* bars;
};

__device__ __forceinline__ void ring_issue(const Ring& r, int i, const uint8_t* src0, uint32_t bytes0,
                                           const uint8_t* src1, uint32_t bytes1) {
    const int st = i % kStages;
    uint8_t* dst = r.base + (size_t) st * r.stage_bytes;
    const uint32_t b0 = bytes0 & ~15u, b1 = bytes1 & ~15u;
    // a ragged tail (rows whose bytes are not a multiple of 16) by plain loads, nothing past the matrix
    for (uint32_t b = b0; b < bytes0; b++) dst[b] = src0[b];
    fence_proxy_async();
    mbar_expect_tx(&r.bars[st], b0 + b1);
    if (b0) bulk_g2s(dst, src0, b0, &r.bars[st]);
    if (b1) bulk_g2s(dst + bytes0, src1, b1, &r.bars[st]);
}

// Thread 0 waits for item i; every thread then acquires it.  Returns false (for every thread) on timeout.
__device__ __forceinline__ bool ring_wait(const Ring& r, int i, int issued, int* s_ok) {
    const int st = i % kStages;
    const uint32_t parity = (uint32_t) ((i / kStages) & 1);
    if (threadIdx.x == 0) {
        bool ok = mbar_wait_bounded(&r.bars[st], parity, kWaitLimitNs);
        if (!ok) {
            atomicOr(&g_smoe_status, kDevTimeout);
            for (int j = i; j < issued; j++)
                mbar_wait_bounded(&r.bars[j % kStages], (uint32_t) ((j / kStages) & 1), kWaitLimitNs);
        }
        *s_ok = ok ? 1 : 0;
    }
    __syncthreads();
    if (!*s_ok) return false;
    (void) mbar_try_wait(&r.bars[st], parity);  // acquire the copied bytes in every thread
    return true;
}

constexpr int kGuThreads = 512;

// ------------------------------------------------------------------------------------------------
// Matrix rows against staged q8_1 columns: y[slot][r] = W_e[r] . act[row(slot)].  This is the stage entry
// point's kernel (smoe_iq_mmvq: one matrix, columns in the standard q8_1 layout staged through shared memory);
// the layer path uses layer_gate_up_kernel / layer_down_kernel below.
// Lane groups of LPR lanes own RPG rows each; lane l of a group owns partials l, l + LPR, ... (PPL of them).
// LPR = 16 is exact against the reference when a row has at most 16 partials: its lanes 16..31 hold zeros
// and the butterfly's first level adds nothing.
// ------------------------------------------------------------------------------------------------
constexpr int kRowThreads = 256;

template <int TYPE, int LPR, int PPL>
__global__ void __launch_bounds__(kRowThreads) expert_rows_kernel(Matrix wm, Matrix swm, GroupView g,
                                                                  const uint8_t* __restrict__ act, int act_by_token,
                                                                  float* __restrict__ y, int64_t y_stride, int n_in,
                                                                  int n_out) {
    constexpr int RPG = 4;
    constexpr int GROUPS = 32 / LPR;
    constexpr int ROWS = (kRowThreads / 32) * GROUPS * RPG;  // rows per tile
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane / LPR, gl = lane % LPR;
    const int rb = (TYPE == kQ2_0) ? (n_in / 64) * 18 : (n_in / 256) * 82;
    const int nblk = n_in / 32;
    const uint32_t stage_bytes = ((uint32_t) (ROWS * rb) + 16u + 127u) & ~127u;
    Ring ring{smem, stage_bytes, nullptr};
    uint32_t* aw = reinterpret_cast<uint32_t*>(smem + (size_t) kStages * stage_bytes);
    float* ad = reinterpret_cast<float*>(aw + kSlotChunk * nblk * 8);
    int* as = reinterpret_cast<int*>(ad + kSlotChunk * nblk);
    uint64_t* grid_s = reinterpret_cast<uint64_t*>(as + kSlotChunk * nblk + 2);
    ring.bars = grid_s + (TYPE == kIQ2_S ? 1024 : 0);
    __shared__ int s_ok;

    if (TYPE == kIQ2_S)
        for (int i = tid; i < 1024; i += kRowThreads) grid_s[i] = k_iq2s_grid_dev[i];
    if (tid == 0) {
        for (int i = 0; i < kStages; i++) mbar_init(&ring.bars[i], 1);
        fence_mbar_init();
    }
    __syncthreads();

    const int n_tiles = (n_out + ROWS - 1) / ROWS;
    const int n_items = group_count(g) * n_tiles;
    const int my_n = blockIdx.x < n_items ? (n_items - 1 - (int) blockIdx.x) / (int) gridDim.x + 1 : 0;
    auto item_src = [&](int i, uint32_t* bytes) -> const uint8_t* {
        const int item = blockIdx.x + i * gridDim.x;
        const int tt = item % n_tiles;
        const Item it = group_item(g, item / n_tiles);
        const int r0 = tt * ROWS;
        *bytes = (uint32_t) (min(ROWS, n_out - r0) * rb);
        return (it.shared ? swm.base : wm.base + (int64_t) it.e * wm.expert_stride) + (int64_t) r0 * rb;
    };
    int issued = 0;
    if (tid == 0) {
        for (; issued < kStages - 1 && issued < my_n; issued++) {
            uint32_t bytes;
            const uint8_t* src = item_src(issued, &bytes);
            ring_issue(ring, issued, src, bytes, nullptr, 0);
        }
    }
    for (int i = 0; i < my_n; i++) {
        if (tid == 0 && issued < my_n) {
            uint32_t bytes;
            const uint8_t* src = item_src(issued, &bytes);
            ring_issue(ring, issued, src, bytes, nullptr, 0);
            issued++;
        }
        if (!ring_wait(ring, i, issued, &s_ok)) return;
        const int item = blockIdx.x + i * gridDim.x;
        const int tt = item % n_tiles;
        const Item it = group_item(g, item / n_tiles);
        const int r0 = tt * ROWS;
        const int nrows = min(ROWS, n_out - r0);
        const uint8_t* wt = ring.base + (size_t) (i % kStages) * stage_bytes;

        Dec wr[RPG][PPL];
        const int row_base = (warp * GROUPS + grp) * RPG;  // tile row of this group's v[0]
#pragma unroll
        for (int q = 0; q < RPG; q++) {
            const uint8_t* rp = wt + min(row_base + q, nrows - 1) * rb;
#pragma unroll
            for (int p = 0; p < PPL; p++) {
                const int k = gl + LPR * p;
                if (k < nblk) decode<TYPE>(rp, k, grid_s, wr[q][p]);
            }
        }
        for (int c0 = it.beg; c0 < it.end; c0 += kSlotChunk) {
            const int nc = min(kSlotChunk, it.end - c0);
            __syncthreads();
            for (int q = tid; q < nc * nblk; q += kRowThreads) {
                const int s = q / nblk, b = q % nblk;
                const int arow = act_by_token ? slot_token(g, it, c0 + s) : c0 + s;
                stage_block<TYPE>(act + ((int64_t) arow * nblk + b) * kQ8Block, aw + (s * nblk + b) * 8,
                                  ad + s * nblk + b, as + s * nblk + b);
            }
            __syncthreads();
            for (int s = 0; s < nc; s++) {
                float v[RPG];
#pragma unroll
                for (int q = 0; q < RPG; q++) v[q] = 0.f;
#pragma unroll
                for (int p = 0; p < PPL; p++) {
                    const int k = gl + LPR * p;
                    if (k < nblk) {
                        const uint4* a = reinterpret_cast<const uint4*>(aw + (s * nblk + k) * 8);
                        const uint4 a0 = a[0], a1 = a[1];
                        const float dx = ad[s * nblk + k];
                        const int qsum = as[s * nblk + k];
#pragma unroll
                        for (int q = 0; q < RPG; q++) v[q] = __fadd_rn(v[q], partial<TYPE>(wr[q][p], a0, a1, dx, qsum));
                    }
                }
                tbfly<RPG, LPR / 2>(v, lane);
                // lane holds row 2 * b(LPR/2) + b(LPR/4) of its group; lanes with the low bits clear store
                constexpr int low_mask = LPR / 4 - 1;
                if ((gl & low_mask) == 0) {
                    const int r = row_base + ((gl / (LPR / 4)) & 3);
                    if (r < nrows) y[(int64_t) (c0 + s) * y_stride + r0 + r] = v[0];
                }
            }
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------------------------------------
// The layer path.  Items are (work-list entry, row tile): a work-list entry is at most kChunk slots of one
// expert, entries are ordered heaviest expert first (the shared expert's chunks lead), and CTAs claim items
// from a counter, so large groups start first and small ones fill in.  Activations come straight from HBM/L2
// in the KAct layout through the read-only path: no staging and no barrier per token.
// ------------------------------------------------------------------------------------------------
struct Entry {
    int e, beg, n;
    bool shared;
};

__device__ __forceinline__ int shared_entries(const Work& w) {
    return w.shared_slots > 0 ? (w.shared_slots + w.sched.chunk - 1) / w.sched.chunk : 0;
}

__device__ __forceinline__ int work_entries(const Work& w) {
    return shared_entries(w) + (w.no_routed ? 0 : *w.sched.count);
}

__device__ __forceinline__ Entry work_entry(const Work& w, int j) {
    Entry en;
    const int sh = shared_entries(w);
    if (j < sh) {
        en.e = -1;
        en.beg = w.shared_base + j * w.sched.chunk;
        en.n = min(w.sched.chunk, w.shared_slots - j * w.sched.chunk);
        en.shared = true;
    } else {
        const int jj = j - sh;
        en.e = w.sched.e[jj];
        en.beg = w.sched.beg[jj];
        en.n = w.sched.n[jj];
        en.shared = false;
    }
    return en;
}

__device__ __forceinline__ int entry_token(const Work& w, const Entry& en, int slot) {
    return en.shared ? slot - w.shared_base : w.slot_token[slot];
}

// Copy the work list and the slot -> token map into shared memory (tab: 3 * cap + n_slot ints) and point the
// Work at the copies, so the producer's per-item table reads are shared-memory reads.
__device__ __forceinline__ void tables_to_smem(Work& w, int32_t* tab, int cap, int n_slot, int nthreads) {
    const int n_ent = *w.sched.count;
    for (int i = threadIdx.x; i < n_ent; i += nthreads) {
        tab[i] = w.sched.e[i];
        tab[cap + i] = w.sched.beg[i];
        tab[2 * cap + i] = w.sched.n[i];
    }
    for (int i = threadIdx.x; i < n_slot; i += nthreads) tab[3 * cap + i] = w.slot_token[i];
    __syncthreads();
    if (threadIdx.x == 0) tab[3 * cap + n_slot] = n_ent;
    __syncthreads();
    w.sched.e = tab;
    w.sched.beg = tab + cap;
    w.sched.n = tab + 2 * cap;
    w.sched.count = tab + 3 * cap + n_slot;
    w.slot_token = tab + 3 * cap;
}

// Thread 0 waits for item i's stage (bounded); on a timeout it also waits, bounded, for every copy it still
// has in flight.  Every thread then acquires the stage, or every thread returns false.
template <int NST>
__device__ __forceinline__ bool stage_wait(uint64_t* bars, int i, const int* s_item, int n_items, int* s_ok) {
    const int st = i % NST;
    const uint32_t parity = (uint32_t) ((i / NST) & 1);
    if (threadIdx.x == 0) {
        const bool ok = mbar_wait_bounded(&bars[st], parity, kWaitLimitNs);
        if (!ok) {
            atomicOr(&g_smoe_status, kDevTimeout);
            for (int j = i + 1; j < i + NST; j++)
                if (s_item[j % NST] < n_items)
                    mbar_wait_bounded(&bars[j % NST], (uint32_t) ((j / NST) & 1), kWaitLimitNs);
        }
        *s_ok = ok ? 1 : 0;
    }
    __syncthreads();
    if (!*s_ok) return false;
    (void) mbar_try_wait(&bars[st], parity);
    return true;
}

// One staged activation block (kKaBlock bytes, 16-byte aligned) and a partial against it.
template <int TYPE>
__device__ __forceinline__ float partial_ka(const Dec& w, const uint8_t* blk) {
    const uint4 a0 = reinterpret_cast<const uint4*>(blk)[0];
    const uint4 a1 = reinterpret_cast<const uint4*>(blk)[1];
    const float2 ds = reinterpret_cast<const float2*>(blk)[4];
    return partial<TYPE>(w, a0, a1, ds.x, 0x4B400000 - __float_as_int(ds.y));
}

// Layer-path dot: the dp4a chain starts from the bits of 1.5 * 2^23 minus the block's sum of q, so after the
// eight unsigned-code dp4a it holds the float 1.5 * 2^23 + sum (code - 1) q exactly (|sum| < 2^22), and one
// subtraction gives (float) sumi.  The seed is per (token, block) and shared by every row.
template <int TYPE>
__device__ __forceinline__ void decode_layer(const uint8_t* row, int k, const uint64_t* grid, Dec& w) {
    decode<TYPE>(row, k, grid, w);
}

struct ActRegs {
    uint4 a0, a1;
    float dx;
    int seed;  // Q2_0: 0x4B400000 - sum q
};

__device__ __forceinline__ ActRegs load_act(const uint8_t* blk) {
    ActRegs r;
    r.a0 = reinterpret_cast<const uint4*>(blk)[0];
    r.a1 = reinterpret_cast<const uint4*>(blk)[1];
    const float2 ds = reinterpret_cast<const float2*>(blk)[4];
    r.dx = ds.x;
    r.seed = __float_as_int(ds.y);
    return r;
}

template <int TYPE>
__device__ __forceinline__ float partial_layer(const Dec& w, const ActRegs& a) {
    float f;
    if constexpr (TYPE == kQ2_0) {
        int s = dp4a_us(w.c[0], (int) a.a0.x, a.seed);
        s = dp4a_us(w.c[1], (int) a.a0.y, s);
        s = dp4a_us(w.c[2], (int) a.a0.z, s);
        s = dp4a_us(w.c[3], (int) a.a0.w, s);
        s = dp4a_us(w.c[4], (int) a.a1.x, s);
        s = dp4a_us(w.c[5], (int) a.a1.y, s);
        s = dp4a_us(w.c[6], (int) a.a1.z, s);
        s = dp4a_us(w.c[7], (int) a.a1.w, s);
        f = __fsub_rn(__int_as_float(s), 12582912.0f);
    } else {
        int s0 = dp4a_ss((int) w.c[0], (int) a.a0.x, 0);
        s0 = dp4a_ss((int) w.c[1], (int) a.a0.y, s0);
        s0 = dp4a_ss((int) w.c[2], (int) a.a0.z, s0);
        s0 = dp4a_ss((int) w.c[3], (int) a.a0.w, s0);
        int s1 = dp4a_ss((int) w.c[4], (int) a.a1.x, 0);
        s1 = dp4a_ss((int) w.c[5], (int) a.a1.y, s1);
        s1 = dp4a_ss((int) w.c[6], (int) a.a1.z, s1);
        s1 = dp4a_ss((int) w.c[7], (int) a.a1.w, s1);
        const int ls0 = (int) (w.ls & 0xFFu), ls1 = (int) (w.ls >> 8);
        f = int_to_float_exact((s0 * ls0 + s1 * ls1 + (s0 + s1) / 2) / 4);
    }
    return __fmul_rn(__fmul_rn(w.d, a.dx), f);
}

constexpr int kGuStages = 4;
constexpr int kGuConsumers = kGuThreads / 32;   // 16 consumer warps
constexpr int kGuBlock = kGuThreads + 32;       // + 1 producer warp

// gate and up.  Item = (work entry, 32-row tile of gate or of up).  Warp-specialised: one producer warp claims
// items and bulk-copies, per ring stage, the tile and the entry's token activations; 16 consumer warps compute,
// warp w owning tile rows w and w + 16, lane L partials L, L + 32, ... (PPL of them).  Stages are handed back
// through `empty` barriers, so the producer runs ahead and its claim / table reads stay off the consumers'
// path.  Results go to gu[slot][gate n_ff | up n_ff] as f32; consumer warps never wait for each other.
template <int TYPE, int PPL>
__global__ void __launch_bounds__(kGuBlock, 1) layer_gate_up_kernel(Matrix gate, Matrix up, Matrix sgate,
                                                                    Matrix sup, Work w, KAct xa,
                                                                    float* __restrict__ gu, int H, int F,
                                                                    int tab_in_smem) {
    constexpr int NST = kGuStages;
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rb = (TYPE == kQ2_0) ? (H / 64) * 18 : (H / 256) * 82;
    const int nblk = H / 32;
    const uint32_t tile_bytes = 32u * (uint32_t) rb;
    const uint32_t act_row = (uint32_t) nblk * kKaBlock;
    const uint32_t stage_bytes = (tile_bytes + kChunk * act_row + 16u + 127u) & ~127u;
    uint64_t* grid_s = reinterpret_cast<uint64_t*>(smem + (size_t) NST * stage_bytes);  // [1024] (IQ2_S)
    uint64_t* full = grid_s + (TYPE == kIQ2_S ? 1024 : 0);
    uint64_t* empty = full + NST;
    int32_t* tab = reinterpret_cast<int32_t*>(empty + NST);  // work list + slot -> token map
    __shared__ int s_item[NST];

    if (TYPE == kIQ2_S)
        for (int i = tid; i < 1024; i += kGuBlock) grid_s[i] = k_iq2s_grid_dev[i];
    if (tab_in_smem) tables_to_smem(w, tab, w.max_entries, w.shared_base, kGuBlock);
    if (tid == 0) {
        for (int i = 0; i < NST; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kGuConsumers);
        }
        fence_mbar_init();
    }
    __syncthreads();
    const int rt = F / 32;            // row tiles per matrix
    const int n_tiles = 2 * rt;       // gate tiles then up tiles
    const int n_items = work_entries(w) * n_tiles;

    if (warp == kGuConsumers) {  // producer
        if (lane != 0) return;
        for (int j = 0;; j++) {
            const int st = j % NST;
            if (j >= NST && !mbar_wait_bounded(&empty[st], (uint32_t) ((j / NST - 1) & 1), kWaitLimitNs)) {
                atomicOr(&g_smoe_status, kDevTimeout);
                for (int q = j - NST + 1; q < j; q++)  // copies still in flight
                    mbar_wait_bounded(&full[q % NST], (uint32_t) ((q / NST) & 1), kWaitLimitNs);
                return;
            }
            const int id = (int) blockIdx.x + j * (int) gridDim.x;  // heaviest items first, round robin
            s_item[st] = id;
            if (id >= n_items) {
                mbar_arrive(&full[st]);  // hands the consumers the end marker
                return;
            }
            const Entry en = work_entry(w, id / n_tiles);
            const int tt = id % n_tiles;
            const Matrix m = tt < rt ? (en.shared ? sgate : gate) : (en.shared ? sup : up);
            const uint8_t* src = (en.shared ? m.base : m.base + (int64_t) en.e * m.expert_stride) +
                                 (int64_t) (tt % rt) * tile_bytes;
            uint8_t* dst = smem + (size_t) st * stage_bytes;
            fence_proxy_async();
            mbar_expect_tx(&full[st], tile_bytes + (uint32_t) en.n * act_row);
            bulk_g2s(dst, src, tile_bytes, &full[st]);
            for (int s = 0; s < en.n; s++) {
                const int tok = entry_token(w, en, en.beg + s);
                bulk_g2s(dst + tile_bytes + s * act_row, xa.base + (size_t) tok * act_row, act_row, &full[st]);
            }
        }
    }

    for (int i = 0;; i++) {
        const int st = i % NST;
        const uint32_t parity = (uint32_t) ((i / NST) & 1);
        bool ok = true;
        if (lane == 0) ok = mbar_wait_bounded(&full[st], parity, kWaitLimitNs);
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
            if (lane == 0) atomicOr(&g_smoe_status, kDevTimeout);
            return;
        }
        (void) mbar_try_wait(&full[st], parity);  // acquire in every lane
        const int id = s_item[st];
        if (id >= n_items) break;
        const Entry en = work_entry(w, id / n_tiles);
        const int tt = id % n_tiles;
        const uint8_t* wt = smem + (size_t) st * stage_bytes;
        const uint8_t* acts = wt + tile_bytes;

        Dec wd[2][PPL];  // tile rows warp, warp + 16
#pragma unroll
        for (int q = 0; q < 2; q++) {
            const uint8_t* rp = wt + (warp + 16 * q) * rb;
#pragma unroll
            for (int p = 0; p < PPL; p++) {
                const int k = lane + 32 * p;
                if (k < nblk) decode_layer<TYPE>(rp, k, grid_s, wd[q][p]);
            }
        }
        float* out = gu + (tt < rt ? 0 : F) + (tt % rt) * 32 + warp;
        for (int s = 0; s < en.n; s++) {
            float v[2] = {0.f, 0.f};
#pragma unroll
            for (int p = 0; p < PPL; p++) {
                const int k = lane + 32 * p;
                if (k < nblk) {
                    const ActRegs a = load_act(acts + s * act_row + k * kKaBlock);
#pragma unroll
                    for (int q = 0; q < 2; q++) v[q] = __fadd_rn(v[q], partial_layer<TYPE>(wd[q][p], a));
                }
            }
            tbfly<2, 16>(v, lane);  // lane holds tile row warp + 16 * b4
            if ((lane & 15) == 0) out[(int64_t) (en.beg + s) * 2 * F + 16 * (lane >> 4)] = v[0];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the stage
    }
}

// SwiGLU then q8_1 of h, in the down kernel's layout: one warp per (slot, 32-value block).
template <int DQ2>
__global__ void swiglu_ka_kernel(const float* __restrict__ gu, KAct ha, int64_t rows, int F) {
    const int lane = threadIdx.x & 31;
    const int nb = F / 32;
    const int64_t warps = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t q = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); q < rows * nb; q += warps) {
        const int64_t r = q / nb;
        const int b = (int) (q % nb);
        const float* g = gu + r * 2 * F + b * 32;
        quant_ka_warp(silu_mul(g[lane], g[F + lane]), ha.base + q * kKaBlock, lane, DQ2 != 0);
    }
}

constexpr int kDownStages = 4;
constexpr int kDownConsumers = kRowThreads / 32;  // 8 consumer warps
constexpr int kDownBlock = kRowThreads + 32;      // + 1 producer warp

// down.  Item = (work entry, ROWS-row tile of n_embd).  A stage holds the tile and the entry's h rows (its slots
// are contiguous: one bulk copy).  Same producer / consumer split as the gate/up kernel; consumer warps never
// synchronise with each other.
template <int TYPE, int LPR, int PPL>
__global__ void __launch_bounds__(kDownBlock) layer_down_kernel(Matrix wm, Matrix swm, Work w, KAct ha,
                                                                float* __restrict__ y, int n_in, int n_out,
                                                                int tab_in_smem) {
    constexpr int NST = kDownStages;
    constexpr int RPG = 4;
    constexpr int GROUPS = 32 / LPR;
    constexpr int ROWS = kDownConsumers * GROUPS * RPG;
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane / LPR, gl = lane % LPR;
    const int rb = (TYPE == kQ2_0) ? (n_in / 64) * 18 : (n_in / 256) * 82;
    const int nblk = n_in / 32;
    const uint32_t tile_bytes = (uint32_t) (ROWS * rb);
    const uint32_t act_row = (uint32_t) nblk * kKaBlock;
    const uint32_t stage_bytes = (tile_bytes + kChunk * act_row + 16u + 127u) & ~127u;
    uint64_t* grid_s = reinterpret_cast<uint64_t*>(smem + (size_t) NST * stage_bytes);
    uint64_t* full = grid_s + (TYPE == kIQ2_S ? 1024 : 0);
    uint64_t* empty = full + NST;
    int32_t* tab = reinterpret_cast<int32_t*>(empty + NST);
    __shared__ int s_item[NST];

    if (TYPE == kIQ2_S)
        for (int i = tid; i < 1024; i += kDownBlock) grid_s[i] = k_iq2s_grid_dev[i];
    if (tab_in_smem) tables_to_smem(w, tab, w.max_entries, 0, kDownBlock);
    if (tid == 0) {
        for (int i = 0; i < NST; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kDownConsumers);
        }
        fence_mbar_init();
    }
    __syncthreads();
    const int n_tiles = n_out / ROWS;  // the layer check guarantees whole tiles
    const int n_items = work_entries(w) * n_tiles;

    if (warp == kDownConsumers) {  // producer
        if (lane != 0) return;
        for (int j = 0;; j++) {
            const int st = j % NST;
            if (j >= NST && !mbar_wait_bounded(&empty[st], (uint32_t) ((j / NST - 1) & 1), kWaitLimitNs)) {
                atomicOr(&g_smoe_status, kDevTimeout);
                for (int q = j - NST + 1; q < j; q++)
                    mbar_wait_bounded(&full[q % NST], (uint32_t) ((q / NST) & 1), kWaitLimitNs);
                return;
            }
            const int id = (int) blockIdx.x + j * (int) gridDim.x;
            s_item[st] = id;
            if (id >= n_items) {
                mbar_arrive(&full[st]);
                return;
            }
            const Entry en = work_entry(w, id / n_tiles);
            const int r0 = (id % n_tiles) * ROWS;
            const uint8_t* src =
                (en.shared ? swm.base : wm.base + (int64_t) en.e * wm.expert_stride) + (int64_t) r0 * rb;
            uint8_t* dst = smem + (size_t) st * stage_bytes;
            fence_proxy_async();
            mbar_expect_tx(&full[st], tile_bytes + (uint32_t) en.n * act_row);
            bulk_g2s(dst, src, tile_bytes, &full[st]);
            bulk_g2s(dst + tile_bytes, ha.base + (size_t) en.beg * act_row, (uint32_t) en.n * act_row, &full[st]);
        }
    }

    for (int i = 0;; i++) {
        const int st = i % NST;
        const uint32_t parity = (uint32_t) ((i / NST) & 1);
        bool ok = true;
        if (lane == 0) ok = mbar_wait_bounded(&full[st], parity, kWaitLimitNs);
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
            if (lane == 0) atomicOr(&g_smoe_status, kDevTimeout);
            break;
        }
        (void) mbar_try_wait(&full[st], parity);
        const int id = s_item[st];
        if (id >= n_items) break;
        const Entry en = work_entry(w, id / n_tiles);
        const int r0 = (id % n_tiles) * ROWS;
        const uint8_t* wt = smem + (size_t) st * stage_bytes;
        const uint8_t* acts = wt + tile_bytes;

        Dec wr[RPG][PPL];
        const int row_base = (warp * GROUPS + grp) * RPG;
#pragma unroll
        for (int q = 0; q < RPG; q++) {
            const uint8_t* rp = wt + (row_base + q) * rb;
#pragma unroll
            for (int p = 0; p < PPL; p++) {
                const int k = gl + LPR * p;
                if (k < nblk) decode_layer<TYPE>(rp, k, grid_s, wr[q][p]);
            }
        }
        for (int s = 0; s < en.n; s++) {
            float v[RPG];
#pragma unroll
            for (int q = 0; q < RPG; q++) v[q] = 0.f;
#pragma unroll
            for (int p = 0; p < PPL; p++) {
                const int k = gl + LPR * p;
                if (k < nblk) {
                    const ActRegs a = load_act(acts + s * act_row + k * kKaBlock);
#pragma unroll
                    for (int q = 0; q < RPG; q++) v[q] = __fadd_rn(v[q], partial_layer<TYPE>(wr[q][p], a));
                }
            }
            tbfly<RPG, LPR / 2>(v, lane);
            constexpr int low_mask = LPR / 4 - 1;
            if ((gl & low_mask) == 0)
                down_row(w, y, en.beg + s, n_out)[r0 + row_base + ((gl / (LPR / 4)) & 3)] = v[0];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    ep_signal_done(w.ep_done, gridDim.x * kDownConsumers);
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
static cudaError_t launch_persistent(K kernel, int threads, size_t smem, int max_items, dim3* out_grid) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (err != cudaSuccess) return err;
    int per_sm = 0;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
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

cudaError_t launch_expert_down(Matrix down, Matrix sdown, GroupView g, const uint8_t* act, int act_by_token,
                               float* y, int64_t y_stride, int n_in, int n_out, cudaStream_t s) {
    const int type = down.type;
    const int rb = type == kQ2_0 ? (n_in / 64) * 18 : (n_in / 256) * 82;
    const int nblk = n_in / 32;
    const int lpr = nblk <= 16 ? 16 : 32;
    const int ppl = (nblk + lpr - 1) / lpr;
    const int rows = (kRowThreads / 32) * (32 / lpr) * 4;
    const size_t stage = ((size_t) rows * rb + 16 + 127) & ~(size_t) 127;
    const size_t smem = kStages * stage + (size_t) kSlotChunk * nblk * 40 + 16 + (type == kIQ2_S ? 8192 : 0) +
                        kStages * 8;
    const int max_items = max_groups(g) * ((n_out + rows - 1) / rows);
    dim3 grid;
    cudaError_t err;
#define SMOE_ROWS(T_, L_, P_)                                                                                  \
    do {                                                                                                       \
        err = launch_persistent(expert_rows_kernel<T_, L_, P_>, kRowThreads, smem, max_items, &grid);         \
        if (err != cudaSuccess) return err;                                                                    \
        expert_rows_kernel<T_, L_, P_><<<grid, kRowThreads, smem, s>>>(down, sdown, g, act, act_by_token, y,   \
                                                                       y_stride, n_in, n_out);                 \
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

namespace smoe {

constexpr size_t kTableSmemMax = 24 * 1024;  // work tables larger than this are read from global memory

static int max_work_entries(const Work& w) {
    return (w.no_routed ? 0 : w.max_entries) + (w.shared_slots > 0 ? (w.shared_slots + kChunk - 1) / kChunk : 0);
}

cudaError_t launch_layer_gate_up(Matrix gate, Matrix up, Matrix sgate, Matrix sup, Work w, KAct xa, float* gu,
                                 int n_embd, int n_ff, cudaStream_t s) {
    const int type = gate.type;
    const int rb = type == kQ2_0 ? (n_embd / 64) * 18 : (n_embd / 256) * 82;
    const int nblk = n_embd / 32;
    const size_t stage = ((size_t) 32 * rb + (size_t) kChunk * nblk * kKaBlock + 16 + 127) & ~(size_t) 127;
    const size_t tab = ((size_t) 3 * w.max_entries + w.shared_base + 1) * 4;
    const int tab_in_smem = tab <= kTableSmemMax ? 1 : 0;
    const size_t smem = kGuStages * stage + (type == kIQ2_S ? 8192 : 0) + 2 * kGuStages * 8 + (tab_in_smem ? tab : 0);
    const int ppl = (nblk + 31) / 32;
    const int max_items = max_work_entries(w) * 2 * (n_ff / 32);
    dim3 grid;
    cudaError_t err;
#define SMOE_LGU(T_, P_)                                                                                        \
    do {                                                                                                        \
        err = launch_persistent(layer_gate_up_kernel<T_, P_>, kGuBlock, smem, max_items, &grid);               \
        if (err != cudaSuccess) return err;                                                                     \
        layer_gate_up_kernel<T_, P_><<<grid, kGuBlock, smem, s>>>(gate, up, sgate, sup, w, xa, gu, n_embd,      \
                                                                  n_ff, tab_in_smem);                           \
    } while (0)
    if (type == kQ2_0) {
        if (ppl == 1) SMOE_LGU(kQ2_0, 1);
        else if (ppl == 2) SMOE_LGU(kQ2_0, 2);
        else if (ppl == 3) SMOE_LGU(kQ2_0, 3);
        else SMOE_LGU(kQ2_0, 4);
    } else {
        if (ppl == 1) SMOE_LGU(kIQ2_S, 1);
        else if (ppl == 2) SMOE_LGU(kIQ2_S, 2);
        else if (ppl == 3) SMOE_LGU(kIQ2_S, 3);
        else SMOE_LGU(kIQ2_S, 4);
    }
#undef SMOE_LGU
    return cudaGetLastError();
}

cudaError_t launch_swiglu_ka(const float* gu, KAct ha, int64_t rows, int n_ff, int down_q2, cudaStream_t s) {
    const int64_t warps = rows * (n_ff / 32);
    int64_t blocks = (warps + 7) / 8;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    if (down_q2) swiglu_ka_kernel<1><<<(unsigned) blocks, 256, 0, s>>>(gu, ha, rows, n_ff);
    else swiglu_ka_kernel<0><<<(unsigned) blocks, 256, 0, s>>>(gu, ha, rows, n_ff);
    return cudaGetLastError();
}

cudaError_t launch_layer_down(Matrix down, Matrix sdown, Work w, KAct ha, float* y, int n_ff, int n_embd,
                              cudaStream_t s) {
    const int type = down.type;
    const int n_in = n_ff, n_out = n_embd;
    const int rb = type == kQ2_0 ? (n_in / 64) * 18 : (n_in / 256) * 82;
    const int nblk = n_in / 32;
    const int lpr = nblk <= 16 ? 16 : 32;
    const int ppl = (nblk + lpr - 1) / lpr;
    const int rows = (kRowThreads / 32) * (32 / lpr) * 4;
    const size_t stage = ((size_t) rows * rb + (size_t) kChunk * nblk * kKaBlock + 16 + 127) & ~(size_t) 127;
    const size_t tab = ((size_t) 3 * w.max_entries + 1) * 4;
    const int tab_in_smem = tab <= kTableSmemMax ? 1 : 0;
    const size_t smem = kDownStages * stage + (type == kIQ2_S ? 8192 : 0) + 2 * kDownStages * 8 + (tab_in_smem ? tab : 0);
    const int max_items = max_work_entries(w) * (n_out / rows);
    dim3 grid;
    cudaError_t err;
#define SMOE_LD(T_, L_, P_)                                                                                     \
    do {                                                                                                        \
        err = launch_persistent(layer_down_kernel<T_, L_, P_>, kDownBlock, smem, max_items, &grid);            \
        if (err != cudaSuccess) return err;                                                                     \
        layer_down_kernel<T_, L_, P_><<<grid, kDownBlock, smem, s>>>(down, sdown, w, ha, y, n_in, n_out,        \
                                                                     tab_in_smem);                              \
    } while (0)
    if (type == kQ2_0) {
        if (lpr == 16) SMOE_LD(kQ2_0, 16, 1);
        else if (ppl == 1) SMOE_LD(kQ2_0, 32, 1);
        else if (ppl == 2) SMOE_LD(kQ2_0, 32, 2);
        else if (ppl == 3) SMOE_LD(kQ2_0, 32, 3);
        else SMOE_LD(kQ2_0, 32, 4);
    } else {
        if (lpr == 16) SMOE_LD(kIQ2_S, 16, 1);
        else if (ppl == 1) SMOE_LD(kIQ2_S, 32, 1);
        else if (ppl == 2) SMOE_LD(kIQ2_S, 32, 2);
        else if (ppl == 3) SMOE_LD(kIQ2_S, 32, 3);
        else SMOE_LD(kIQ2_S, 32, 4);
    }
#undef SMOE_LD
    return cudaGetLastError();
}

}  // namespace smoe
