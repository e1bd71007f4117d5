// tc.cu - grouped expert GEMMs on the 5th-generation tensor cores (tcgen05.mma kind::f16, f32 accumulators in
// tensor memory) for work entries with many tokens: the prefill path.
//
// Shapes (swap-AB): M = 128 weight rows per tile (tensor-memory lanes), N = 2 x the entry's tokens (hi and lo
// halves of <= 64 tokens each, padded to a multiple of 16), K streamed in 64-wide stages (one Q2_0 block per row).
//
//   gate/up item (MODE 0): 128 rows of gate and of up (two accumulators, so the thread that owns row r holds
//                g_r and u_r), epilogue SwiGLU and the q8_1 rule over each warp's 32 rows (one block of h),
//                written as the down GEMM's activation.
//   down item (MODE 1):    128 output rows, K = n_ff, epilogue stores f32 per (slot, row).
//
// Operands.  Weights: Q2_0 blocks are TMA-loaded raw (2D boxes of 144 B x 128 rows = 8 blocks per row) and
// decoded by eight warps to fp16 (code - 1) * d, exact in fp16, into a K-major unswizzled shared-memory tile.
// The decode ORs a code pair straight into the mantissas of an fp16 pair of power-of-two magnitude 2^E (the code
// lands at the mantissa bit of weight 1), so one HADD2 of -(2^E + 1) gives code - 1 exactly and one HMUL2 by d
// gives the weight.  That fixes the K order inside each 64-value block (tc_kpos): the activation images are
// written in the same order, and a dot product does not depend on it.
// Activations: the q8_1 image x~ = q * d (q the int8 code, d the fp16 scale) is exact in f32 but not in fp16, so
// it is carried as two fp16 halves, hi = fp16(x~) and lo = fp16(x~ - hi), which together are exact.  The B
// tile stacks them, hi in rows [0, npad) and lo in rows [npad, 2 npad), so one MMA per K step yields both
// partial products in adjacent accumulator columns and the epilogue adds them: the result is the integer
// contract's dot product up to the order of the f32 additions.  Activation rows are gathered per token by TMA
// (tile::gather4) into a 128-byte-swizzled tile.
//
// Warps: 0 producer (TMA; also allocates tensor memory), 1 MMA issuer (lane 0), 4-11 decoders, 12-15 epilogue
// (warp 12 + q reads tensor-memory lanes 32q..32q+31).  Rings: raw weight quarters (2), A/B stages (3),
// accumulators (2).  Every wait is bounded; on a timeout the kernel records kDevTimeout, drains the copies and
// MMAs it issued (bounded), frees tensor memory and returns.
#include "common.cuh"
#include "kernels.cuh"
#include "q8.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

namespace smoe {

constexpr int kTcThreads = 512;
constexpr int kTcDecWarps = 8;
constexpr int kTcM = 128;
constexpr int kTcK = 64;                          // K per A/B stage: one Q2_0 block per row
constexpr int kTcQ = 512;                         // K per raw quarter: 8 blocks = 144 bytes per row
constexpr int kTcAB = 3;                          // A/B stages
constexpr int kTcRaw = 2;                         // raw weight stages
constexpr uint32_t kRawMat = kTcM * 144;          // 18,432 B: one matrix quarter
constexpr uint32_t kAMat = kTcM * kTcK * 2;       // 16,384 B: one fp16 A tile
constexpr uint32_t kBTile = 2 * kTcChunk * kTcK * 2;  // 16,384 B: up to 64 hi + 64 lo activation rows

struct TcArgs {
    Work w;
    int K;          // n_embd (gate/up) or n_ff (down)
    int m_tiles;    // row tiles per expert matrix
    int act_rows;   // rows of one activation half: T (gate/up, per token) or R (down, per slot)
    int n_out;      // gate/up: n_ff (h row length); down: n_embd (parts row length)
    int hh_rows;    // gate/up: R, the slot rows of one half of the h image
    __half* hh;     // gate/up output: hi [R][n_ff] then lo [R][n_ff]
    float* parts;   // down output [slot][n_embd]
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, int x, int y0, int y1, int y2, int y3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3, %4, %5, %6}], [%7];" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(smem_addr(bar))
        : "memory");
}

// K-major 128-byte-swizzled descriptor (a TMA-written activation tile, 128 B per row): 1024 B between 8-row groups.
__device__ __forceinline__ uint64_t umma_desc_sw128(const void* smem_ptr) {
    const uint32_t a = smem_addr(smem_ptr);
    return (uint64_t) ((a >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t) (1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

// K order inside a 64-value block.  A code word (16 codes, code v at bits 2v) decodes as 8 fp16 pairs: pair s
// holds values s (low) and 8 + s (high), from bits 2s and 16 + 2s (s < 5) or of the word shifted right by 10
// (s >= 5).  Word j fills 16-byte chunks 2j (pairs 0-3) and 2j + 1 (pairs 4-7), so value v of the block sits at
// position tc_kpos(v).
__host__ __device__ constexpr int tc_kpos(int v) {
    return 16 * (v >> 4) + 8 * ((v & 7) >> 2) + 2 * (v & 3) + ((v >> 3) & 1);
}

// Pair s of code word w (see tc_kpos) as fp16 (code - 1) * d; d2 = d in both halves.
template <int S>
__device__ __forceinline__ uint32_t dec_pair(uint32_t w, uint32_t w10, __half2 d2) {
    constexpr int s = S < 5 ? S : S - 5;                        // code bit position 2s after the shift
    constexpr uint32_t mask = 0x00030003u << (2 * s);
    constexpr uint32_t magic[5] = {0x64006400u, 0x5C005C00u, 0x54005400u, 0x4C004C00u, 0x44004400u};  // 2^(10-2s)
    constexpr float bias[5] = {-1025.f, -257.f, -65.f, -17.f, -5.f};                                    // -(2^E + 1)
    const uint32_t x = ((S < 5 ? w : w10) & mask) | magic[s];  // fp16 pair (2^E + c_lo, 2^E + c_hi)
    const __half2 c = __hadd2(*reinterpret_cast<const __half2*>(&x), __float2half2_rn(bias[s]));
    const __half2 v = __hmul2(c, d2);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// A whole warp waits (bounded) for a phase; the verdict is the same for every lane.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
    const bool ok = mbar_wait_sleep(bar, parity, kWaitLimitNs);
    return __all_sync(0xffffffffu, ok);
}

// Wait (bounded) for the latest phase of each slot of a ring of `n` barriers fed `count` times: the drain
// before a role returns while copies or MMAs it issued may still be in flight.
__device__ __forceinline__ void drain_ring(uint64_t* bars, int n, int count) {
    for (int i = max(0, count - n); i < count; i++)
        mbar_wait_sleep(&bars[i % n], (uint32_t) ((i / n) & 1), kWaitLimitNs);
}

template <int MODE>
__global__ void __launch_bounds__(kTcThreads, 1) tc_expert_kernel(const __grid_constant__ CUtensorMap mw0,
                                                                  const __grid_constant__ CUtensorMap mw1,
                                                                  const __grid_constant__ CUtensorMap sw0,
                                                                  const __grid_constant__ CUtensorMap sw1,
                                                                  const __grid_constant__ CUtensorMap mact,
                                                                  TcArgs args) {
    constexpr int NMAT = MODE == 0 ? 2 : 1;
    constexpr uint32_t kMatCols = 2 * kTcChunk;     // one matrix: hi columns [0, npad), lo [npad, 2 npad)
    constexpr uint32_t kAccCols = NMAT * kMatCols;  // one accumulator buffer
    constexpr uint32_t kTmemCols = 2 * kAccCols;    // two buffers: 512 (gate/up) or 256 (down)
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint8_t* sB = smem;                                   // [kTcAB][hi npad rows | lo npad rows] x 128 B, swizzled
    uint8_t* sA = sB + kTcAB * kBTile;                    // [kTcAB][NMAT] 128 x 64 fp16, core-matrix layout
    uint8_t* sRaw = sA + kTcAB * NMAT * kAMat;            // [kTcRaw][NMAT] 128 rows x 144 B
    uint64_t* bars = reinterpret_cast<uint64_t*>(sRaw + kTcRaw * NMAT * kRawMat);
    uint64_t* raw_full = bars;                 // producer arrive + tx
    uint64_t* raw_empty = raw_full + kTcRaw;   // the decoder warps
    uint64_t* b_full = raw_empty + kTcRaw;     // producer arrive + tx
    uint64_t* a_full = b_full + kTcAB;         // the decoder warps
    uint64_t* ab_empty = a_full + kTcAB;       // MMA commit
    uint64_t* acc_full = ab_empty + kTcAB;     // MMA commit
    uint64_t* acc_empty = acc_full + 2;        // 4 epilogue warps
    uint64_t* mma_done = acc_empty + 2;        // MMA commit (the final drain)
    __shared__ uint32_t s_tmem;

    const Work w = args.w;
    const int K = args.K;
    const int KS = K / kTcK;                 // A/B stages per item
    const int QS = (K + kTcQ - 1) / kTcQ;    // raw quarters per item
    constexpr int kQS = kTcQ / kTcK;         // A/B stages per quarter
    const int n_items = work_entries(w) * args.m_tiles;

    if (tid == 0) {
        for (int i = 0; i < kTcRaw; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kTcDecWarps);
        }
        for (int i = 0; i < kTcAB; i++) {
            mbar_init(&b_full[i], 1);
            mbar_init(&a_full[i], kTcDecWarps);
            mbar_init(&ab_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 4);
        }
        mbar_init(mma_done, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&s_tmem, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == 0) {
        // ---------------- producer warp: raw weight quarters (lane 0) and activation rows ----------------
        int rc = 0, sc = 0;
        bool ok = true;
        for (int j = 0; ok; j++) {
            const int id = (int) blockIdx.x + j * (int) gridDim.x;
            if (id >= n_items) break;
            const Entry en = work_entry(w, id / args.m_tiles);
            const int mt = id % args.m_tiles;
            const int npad = (en.n + 15) & ~15;
            // lane l < 16 gathers hi rows 4l..4l+3, lane l >= 16 the same tokens' lo rows
            const int g = lane & 15;
            int tk[4] = {0, 0, 0, 0};
            if (MODE == 0) {
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int rr = min(4 * g + u, en.n - 1);  // padding rows repeat the last token
                    tk[u] = entry_token(w, en, en.beg + rr) + (lane >= 16 ? args.act_rows : 0);
                }
            }
            const bool gather_lane = 4 * g < npad;
            const int row = (en.shared ? 0 : en.e * args.m_tiles * kTcM) + mt * kTcM;
            for (int q = 0; q < QS && ok; q++) {
                const int rs = rc % kTcRaw;
                if (rc >= kTcRaw && !warp_wait(&raw_empty[rs], (uint32_t) ((rc / kTcRaw - 1) & 1))) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    uint8_t* dst = sRaw + (size_t) rs * NMAT * kRawMat;
                    mbar_expect_tx(&raw_full[rs], NMAT * kRawMat);
                    tma_load_2d(dst, en.shared ? &sw0 : &mw0, q * 144, row, &raw_full[rs]);
                    if (NMAT == 2) tma_load_2d(dst + kRawMat, en.shared ? &sw1 : &mw1, q * 144, row, &raw_full[rs]);
                }
                rc++;
                const int k_end = min(KS, (q + 1) * kQS);
                for (int ks = q * kQS; ks < k_end; ks++) {
                    const int st = sc % kTcAB;
                    if (sc >= kTcAB && !warp_wait(&ab_empty[st], (uint32_t) ((sc / kTcAB - 1) & 1))) {
                        ok = false;
                        break;
                    }
                    uint8_t* bdst = sB + (size_t) st * kBTile;
                    if (lane == 0) mbar_expect_tx(&b_full[st], (uint32_t) (2 * npad * kTcK * 2));
                    __syncwarp();
                    if (MODE == 0) {
                        // lane g < 16: hi rows 4g..4g+3; lane 16 + g: the same tokens' lo rows at npad + 4g
                        if (gather_lane)
                            tma_gather4(bdst + ((lane >= 16 ? npad : 0) + 4 * g) * 128, &mact, ks * kTcK, tk[0], tk[1],
                                        tk[2], tk[3], &b_full[st]);
                    } else {
                        // 16-row boxes of consecutive slots: lane i < npad/16 hi rows, lane 8 + i lo rows
                        const int i = lane & 7;
                        if (lane < 16 && 16 * i < npad)
                            tma_load_2d(bdst + ((lane >= 8 ? npad : 0) + 16 * i) * 128, &mact, ks * kTcK,
                                        (lane >= 8 ? args.act_rows : 0) + en.beg + 16 * i, &b_full[st]);
                    }
                    sc++;
                }
            }
        }
        if (!ok && lane == 0) atomicOr(&g_smoe_status, kDevTimeout);
        // every copy this warp issued has landed before the shared memory is released
        if (lane == 0) {
            drain_ring(raw_full, kTcRaw, rc);
            drain_ring(b_full, kTcAB, sc);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (lane 0) ----------------
        if (lane == 0) {
            int sc = 0;
            bool ok = true, issued = false;
            for (int j = 0; ok; j++) {
                const int id = (int) blockIdx.x + j * (int) gridDim.x;
                if (id >= n_items) break;
                const Entry en = work_entry(w, id / args.m_tiles);
                const int npad = (en.n + 15) & ~15;
                const int a = j & 1;
                if (j >= 2 && !mbar_wait_sleep(&acc_empty[a], (uint32_t) ((j / 2 - 1) & 1), kWaitLimitNs)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t idesc = umma_idesc_f16(kTcM, 2 * npad);
                const uint32_t d0 = tmem + (uint32_t) a * kAccCols;
                for (int ks = 0; ks < KS; ks++) {
                    const int st = sc % kTcAB;
                    const uint32_t par = (uint32_t) ((sc / kTcAB) & 1);
                    if (!mbar_wait_sleep(&b_full[st], par, kWaitLimitNs) ||
                        !mbar_wait_sleep(&a_full[st], par, kWaitLimitNs)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint8_t* bt = sB + (size_t) st * kBTile;
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        const uint8_t* at = sA + ((size_t) st * NMAT + m) * kAMat;
                        const uint32_t d = d0 + (uint32_t) m * kMatCols;
#pragma unroll
                        for (int s = 0; s < kTcK / 16; s++)
                            umma_f16(d, umma_desc(at + s * 256, 128, 1024), umma_desc_sw128(bt + s * 32), idesc,
                                     (ks > 0 || s > 0) ? 1u : 0u);
                    }
                    umma_commit(&ab_empty[st]);  // the stage is free once these MMAs have read it
                    issued = true;
                    sc++;
                }
                if (!ok) break;
                umma_commit(&acc_full[a]);
            }
            if (!ok) atomicOr(&g_smoe_status, kDevTimeout);
            if (issued) {  // every MMA has retired before tensor memory is freed
                umma_commit(mma_done);
                mbar_wait_sleep(mma_done, 0, kWaitLimitNs);
            }
        }
        __syncwarp();
    } else if (warp >= 4 && warp < 4 + kTcDecWarps) {
        // ---------------- decoders: raw Q2_0 -> fp16 A tiles ----------------
        // Pass i covers rows 8 (2 dw + i) + (lane&7), code word j = lane>>3 (chunks 2j, 2j + 1): a quarter-warp
        // stores 128-byte runs of a core matrix, and the code reads of a warp fall in distinct banks.
        const int dw = warp - 4;
        const int j4 = lane >> 3;
        int rc = 0, sc = 0;
        bool ok = true;
        for (int j = 0; ok; j++) {
            const int id = (int) blockIdx.x + j * (int) gridDim.x;
            if (id >= n_items) break;
            for (int q = 0; q < QS && ok; q++) {
                const int rs = rc % kTcRaw;
                if (!warp_wait(&raw_full[rs], (uint32_t) ((rc / kTcRaw) & 1))) {
                    ok = false;
                    break;
                }
                const uint8_t* raw = sRaw + (size_t) rs * NMAT * kRawMat;
                const int k_end = min(KS, (q + 1) * kQS);
                for (int ks = q * kQS; ks < k_end; ks++) {
                    const int st = sc % kTcAB;
                    if (sc >= kTcAB && !warp_wait(&ab_empty[st], (uint32_t) ((sc / kTcAB - 1) & 1))) {
                        ok = false;
                        break;
                    }
                    const int boff = (ks - q * kQS) * 18;
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        uint8_t* at = sA + ((size_t) st * NMAT + m) * kAMat;
                        const uint8_t* rm = raw + m * kRawMat;
#pragma unroll
                        for (int i = 0; i < 16 / kTcDecWarps; i++) {
                            const int r = (2 * dw + i) * 8 + (lane & 7);
                            const uint8_t* blk = rm + r * 144 + boff;
                            const uint16_t* cw = reinterpret_cast<const uint16_t*>(blk + 2 + 4 * j4);
                            const uint32_t w = (uint32_t) cw[0] | ((uint32_t) cw[1] << 16);
                            const uint32_t w10 = w >> 10;
                            const __half2 d2 = __half2half2(__ushort_as_half(*reinterpret_cast<const uint16_t*>(blk)));
                            uint8_t* dst = at + (2 * j4) * 128 + (r >> 3) * 1024 + (r & 7) * 16;
                            *reinterpret_cast<uint4*>(dst) =
                                make_uint4(dec_pair<0>(w, w10, d2), dec_pair<1>(w, w10, d2), dec_pair<2>(w, w10, d2),
                                           dec_pair<3>(w, w10, d2));
                            *reinterpret_cast<uint4*>(dst + 128) =
                                make_uint4(dec_pair<4>(w, w10, d2), dec_pair<5>(w, w10, d2), dec_pair<6>(w, w10, d2),
                                           dec_pair<7>(w, w10, d2));
                        }
                    }
                    fence_proxy_async();  // generic-proxy stores -> the tensor core's reads
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[st]);
                    sc++;
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_empty[rs]);
                rc++;
            }
        }
        if (!ok && lane == 0) atomicOr(&g_smoe_status, kDevTimeout);
    } else if (warp >= 4 + kTcDecWarps) {
        // ---------------- epilogue: tensor memory -> h (gate/up) or the slot rows (down) ----------------
        const int wq = warp & 3;  // tensor-memory lanes 32 wq .. 32 wq + 31
        bool ok = true;
        for (int j = 0; ok; j++) {
            const int id = (int) blockIdx.x + j * (int) gridDim.x;
            if (id >= n_items) break;
            const Entry en = work_entry(w, id / args.m_tiles);
            const int mt = id % args.m_tiles;
            const int npad = (en.n + 15) & ~15;
            const int a = j & 1;
            if (!warp_wait(&acc_full[a], (uint32_t) ((j / 2) & 1))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem + ((uint32_t) (32 * wq) << 16) + (uint32_t) a * kAccCols;
            const int row = mt * kTcM + 32 * wq + lane;  // this thread's output row
            for (int c0 = 0; c0 < en.n; c0 += 8) {
                uint32_t g8[8], gl8[8], u8[8], ul8[8];
                tmem_ld8(tbase + (uint32_t) c0, g8);
                tmem_ld8(tbase + (uint32_t) (npad + c0), gl8);
                if (MODE == 0) {
                    tmem_ld8(tbase + kMatCols + (uint32_t) c0, u8);
                    tmem_ld8(tbase + kMatCols + (uint32_t) (npad + c0), ul8);
                }
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int t = c0 + i;
                    if (t >= en.n) break;  // uniform across the warp
                    const int slot = en.beg + t;
                    if (MODE == 0) {
                        // SwiGLU, then the q8_1 rule over the warp's 32 rows (one block of h), stored as hi/lo
                        const float h = silu_mul(__fadd_rn(__uint_as_float(g8[i]), __uint_as_float(gl8[i])),
                                                 __fadd_rn(__uint_as_float(u8[i]), __uint_as_float(ul8[i])));
                        float amax = fabsf(h);
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                        float d = __fdiv_rn(amax, 127.f);
                        if (fabsf(d) > 65504.f) d = copysignf(65504.f, d);
                        float qv = 0.f;
                        if (amax != 0.f) qv = fminf(fmaxf(roundf(__fdiv_rn(h, d)), -127.f), 127.f);
                        const float v = __fmul_rn(qv, f16_to_f32(f16_bits(d)));
                        const __half hi = __float2half_rn(v);
                        const __half lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
                        const int col = (row & ~63) + tc_kpos(row & 63);
                        args.hh[(size_t) slot * args.n_out + col] = hi;
                        args.hh[((size_t) args.hh_rows + slot) * args.n_out + col] = lo;
                    } else {
                        args.parts[(size_t) slot * args.n_out + row] =
                            __fadd_rn(__uint_as_float(g8[i]), __uint_as_float(gl8[i]));
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[a]);
        }
        if (!ok && lane == 0) atomicOr(&g_smoe_status, kDevTimeout);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// q8_1 image of x as hi/lo fp16 halves, in the K order of tc_kpos: value i of token t goes to column
// c = (i & ~63) + tc_kpos(i & 63), xh[t][c] = hi, xh[T + t][c] = lo, hi + lo = q * fp16(d) exactly.
// One warp per 32-value block, the q8_1 rule of quant_q8_1_warp.
__global__ void quant_xh_kernel(const float* __restrict__ x, int T, int H, __half* __restrict__ xh) {
    const int lane = threadIdx.x & 31;
    const int64_t nblk = (int64_t) T * (H / 32);
    for (int64_t b = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nblk;
         b += (int64_t) gridDim.x * (blockDim.x >> 5)) {
        const int64_t i = b * 32 + lane;
        const float xi = x[i];
        float amax = fabsf(xi);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        float d = __fdiv_rn(amax, 127.f);
        if (fabsf(d) > 65504.f) d = copysignf(65504.f, d);
        float qv = 0.f;
        if (amax != 0.f) qv = fminf(fmaxf(roundf(__fdiv_rn(xi, d)), -127.f), 127.f);
        const float v = __fmul_rn(qv, f16_to_f32(f16_bits(d)));
        const __half hi = __float2half_rn(v);
        const int64_t c = (i & ~(int64_t) 63) + tc_kpos((int) (i & 63));
        xh[c] = hi;
        xh[(int64_t) T * H + c] = __float2half_rn(__fsub_rn(v, __half2float(hi)));
    }
}

// ------------------------------------------------------------------------------------------------
// host side: tensor maps (encoded through the runtime's driver entry point) and the launches
// ------------------------------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    auto fn = encode_fn();
    if (!fn || !base) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Q2_0 rows as bytes: `rows` rows of row_bytes, box = one raw quarter (144 B) of 128 rows.
bool weight_map(CUtensorMap* m, const uint8_t* base, int64_t rows, int row_bytes) {
    return make_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, (uint64_t) row_bytes, (uint64_t) rows,
                    (uint64_t) row_bytes, 144, kTcM, CU_TENSOR_MAP_SWIZZLE_NONE);
}

size_t tc_smem_bytes(int nmat) {
    return (size_t) kTcAB * kBTile + (size_t) kTcAB * nmat * kAMat + (size_t) kTcRaw * nmat * kRawMat + 32 * 8 +
           1024;
}

template <int MODE>
cudaError_t launch_tc(const CUtensorMap* maps, const TcArgs& a, cudaStream_t s) {
    const size_t smem = tc_smem_bytes(MODE == 0 ? 2 : 1);
    cudaError_t err =
        cudaFuncSetAttribute(tc_expert_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (err != cudaSuccess) return err;
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    tc_expert_kernel<MODE><<<nsm, kTcThreads, smem, s>>>(maps[0], maps[1], maps[2], maps[3], maps[4], a);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_quant_xh(const float* x, int T, int H, __half* xh, cudaStream_t s) {
    const int64_t nblk = (int64_t) T * (H / 32);
    const int grid = (int) std::min<int64_t>((nblk + 7) / 8, 148 * 16);
    quant_xh_kernel<<<grid, 256, 0, s>>>(x, T, H, xh);
    return cudaGetLastError();
}

cudaError_t launch_tc_gate_up(Matrix gate, Matrix up, Matrix sgate, Matrix sup, Work w, int n_expert,
                              const __half* xh, int T, __half* hh, int R, int n_embd, int n_ff, cudaStream_t s) {
    const int rb = (n_embd / 64) * 18;
    const int64_t routed_rows = (int64_t) n_ff * n_expert;
    CUtensorMap maps[5];
    const bool ok = weight_map(&maps[0], gate.base, routed_rows, rb) && weight_map(&maps[1], up.base, routed_rows, rb) &&
                    weight_map(&maps[2], sgate.base ? sgate.base : gate.base, n_ff, rb) &&
                    weight_map(&maps[3], sup.base ? sup.base : up.base, n_ff, rb) &&
                    make_map(&maps[4], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh, (uint64_t) n_embd, (uint64_t) 2 * T,
                             (uint64_t) n_embd * 2, kTcK, 1, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!ok) return cudaErrorInvalidValue;
    TcArgs a{};
    a.w = w;
    a.K = n_embd;
    a.m_tiles = n_ff / kTcM;
    a.act_rows = T;
    a.n_out = n_ff;
    a.hh_rows = R;
    a.hh = hh;
    return launch_tc<0>(maps, a, s);
}

cudaError_t launch_tc_down(Matrix down, Matrix sdown, Work w, int n_expert, const __half* hh, int R, float* parts,
                           int n_ff, int n_embd, cudaStream_t s) {
    const int rb = (n_ff / 64) * 18;
    const int64_t routed_rows = (int64_t) n_embd * n_expert;
    CUtensorMap maps[5];
    const uint8_t* sd = sdown.base ? sdown.base : down.base;
    const bool ok = weight_map(&maps[0], down.base, routed_rows, rb) && weight_map(&maps[1], down.base, routed_rows, rb) &&
                    weight_map(&maps[2], sd, n_embd, rb) && weight_map(&maps[3], sd, n_embd, rb) &&
                    make_map(&maps[4], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, hh, (uint64_t) n_ff, (uint64_t) 2 * R,
                             (uint64_t) n_ff * 2, kTcK, 16, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!ok) return cudaErrorInvalidValue;
    TcArgs a{};
    a.w = w;
    a.K = n_ff;
    a.m_tiles = n_embd / kTcM;
    a.act_rows = R;
    a.n_out = n_embd;
    a.parts = parts;
    return launch_tc<1>(maps, a, s);
}

}  // namespace smoe
