// tc.cu - grouped expert GEMMs on the 5th-generation tensor cores (tcgen05.mma kind::f16, f32 accumulators in
// tensor memory) for work entries with many tokens: the prefill path.
//
// Shapes (swap-AB): M = 128 weight rows per tile (tensor-memory lanes), N = the entry's tokens (<= 64, padded to a
// multiple of 16), K streamed in 64-wide stages (one Q2_0 block per row).
//
//   gate/up item (MODE 0): 128 rows of gate and of up (two accumulators, so the thread that owns row r holds
//                g_r and u_r), epilogue SwiGLU and the q8_1 rule over each warp's 32 rows (one block of h),
//                written as the down GEMM's activation.
//   down item (MODE 1):    128 output rows, K = n_ff, epilogue stores f32 per (slot, row).
//
// Operands.  Weights: Q2_0 blocks are TMA-loaded raw (2D boxes of 144 B x 128 rows = 8 blocks per row) and
// decoded by eight warps to fp16 (code - 1) * d, exact in fp16, straight into tensor memory (tcgen05.st; the
// thread that owns tensor-memory lane r decodes weight row r), where the MMA reads A: the decoded tile never
// touches shared memory, which is left to the activation tiles.  The decode ORs a code pair straight into the
// mantissas of an fp16 pair of power-of-two magnitude 2^E (the code lands at the mantissa bit of weight 1), so
// one HADD2 of -(2^E + 1) gives code - 1 exactly and one HMUL2 by d gives the weight.  That fixes the K order
// inside each 64-value block (tc_kpos): the activation images are written in the same order, and a dot product
// does not depend on it.
// Activations: the q8_1 image x~ = q * d (q the int8 code, d the fp16 scale) is exact in f32 but not in fp16, so
// it is carried as two fp16 halves, hi = fp16(x~) and lo = fp16(x~ - hi), which together are exact.  The B
// tile stacks them, hi in rows [0, npad) and lo in rows [npad, 2 npad), so one MMA of N = 2 npad per K step
// yields both partial products in adjacent accumulator columns and the epilogue adds them: the result is the
// integer contract's dot product up to the order of the f32 additions.  Gate/up gathers its rows per token with
// 16-byte cp.async copies into a 128-byte-swizzled tile; down reads consecutive slots with TMA boxes.
//
// Warps: 0 raw weight producer (TMA; also allocates tensor memory), 1 MMA issuer (lane 0), 2-3 activation
// producers, 4-11 decoders, 12-19 epilogue (warp 12 + 4h + q reads tensor-memory lanes 32q..32q+31, token groups
// h, h + 2, ...).  Rings: raw weight quarters (2 or 4), decoded A stages (3, tensor memory), activation stages
// (4 or 6), accumulators (1 for gate/up, whose epilogue frees it after copying g and u to shared memory; 2 for
// down), each with its own full/empty barriers, so weight prefetch runs ahead of the activations.
// Every wait is bounded; on a timeout the kernel records kDevTimeout, drains the copies and MMAs it issued
// (bounded), frees tensor memory and returns.
#include "common.cuh"
#include "ep.cuh"
#include "kernels.cuh"
#include "q8.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

namespace smoe {

constexpr int kTcDecWarps = 8;                    // warps 4..11
constexpr int kTcEpiWarp0 = 4 + kTcDecWarps;      // warps 12..19
constexpr int kTcEpiWarps = 8;
constexpr int kTcThreads = 32 * (kTcEpiWarp0 + kTcEpiWarps);
constexpr int kTcM = 128;
constexpr int kTcK = 64;                          // K per A/B stage: one Q2_0 block per row
constexpr int kTcQ = 512;                         // K per raw quarter: 8 blocks = 144 bytes per row
constexpr uint32_t kRawMat = kTcM * 144;          // 18,432 B: one matrix quarter
constexpr uint32_t kBTile = 2 * kTcChunk * kTcK * 2;  // 16,384 B: up to 64 hi + 64 lo activation rows
constexpr int kBRowsPerThread = 2 * kTcChunk / 8;     // tile rows per activation-producer thread

struct TcArgs {
    Work w;
    const __half* act;  // activation image: hi rows [0, act_rows), lo rows [act_rows, 2 act_rows), K columns
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

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// One arrival on `bar` once every cp.async this thread issued before has completed (counted in the barrier's
// expected arrivals).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

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

// Ring depths, shared memory and tensor memory per mode (gate/up holds two matrices per stage).
// Gate/up keeps one accumulator buffer (gate and up, hi and lo columns: 256) beside three A stages; its epilogue
// frees the buffer as soon as g and u sit in a shared-memory staging area.  Down keeps two buffers.
template <int MODE> struct TcCfg {
    static constexpr int NMAT = MODE == 0 ? 2 : 1;
    static constexpr int kRaw = MODE == 0 ? 2 : 4;                // raw weight quarters (shared memory)
    static constexpr int kA = 3;                                  // decoded A stages (tensor memory)
    static constexpr int kB = MODE == 0 ? 4 : 6;                  // activation stages (shared memory)
    static constexpr int kAccBufs = MODE == 0 ? 1 : 2;
    static constexpr uint32_t kMatCols = 2 * kTcChunk;            // one matrix: hi [0, npad), lo [npad, 2 npad)
    static constexpr uint32_t kAccCols = NMAT * kMatCols;         // one accumulator buffer
    static constexpr uint32_t kAOff = kAccBufs * kAccCols;        // A stages follow the accumulator buffers
    static constexpr uint32_t kACols = NMAT * kTcK / 2;           // one A stage: 64 fp16 per row per matrix
    static constexpr uint32_t kTmemCols = 512;
    static_assert(kAOff + kA * kACols <= kTmemCols, "tensor memory budget");
    static constexpr size_t kStage = MODE == 0 ? (size_t) kTcEpiWarps * 2 * 32 * (kTcChunk / 2) * 4 : 0;  // g, u
    static constexpr size_t smem =
        (size_t) kB * kBTile + (size_t) kRaw * NMAT * kRawMat + kStage + 64 * 8 + 1024;
};

template <int MODE>
__global__ void __launch_bounds__(kTcThreads, 1) tc_expert_kernel(const __grid_constant__ CUtensorMap mw0,
                                                                  const __grid_constant__ CUtensorMap mw1,
                                                                  const __grid_constant__ CUtensorMap sw0,
                                                                  const __grid_constant__ CUtensorMap sw1,
                                                                  const __grid_constant__ CUtensorMap mact,
                                                                  TcArgs args) {
    using Cfg = TcCfg<MODE>;
    constexpr int NMAT = Cfg::NMAT, kRaw = Cfg::kRaw, kA = Cfg::kA, kB = Cfg::kB, kAccBufs = Cfg::kAccBufs;
    constexpr uint32_t kMatCols = Cfg::kMatCols, kAccCols = Cfg::kAccCols, kAOff = Cfg::kAOff, kACols = Cfg::kACols;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint8_t* sB = smem;                          // [kB][hi npad rows | lo npad rows] x 128 B, 128-byte swizzle
    uint8_t* sRaw = sB + kB * kBTile;            // [kRaw][NMAT] 128 rows x 144 B
    float* sStage = reinterpret_cast<float*>(sRaw + kRaw * NMAT * kRawMat);  // gate/up: per epilogue warp g, u
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sStage) + Cfg::kStage);
    uint64_t* raw_full = bars;                   // raw producer arrive + tx
    uint64_t* raw_empty = raw_full + kRaw;       // the decoder warps
    uint64_t* a_full = raw_empty + kRaw;         // the decoder warps
    uint64_t* a_empty = a_full + kA;             // MMA commit
    uint64_t* b_full = a_empty + kA;             // gate/up: 64 cp.async arrivals; down: producer arrive + tx
    uint64_t* b_empty = b_full + kB;             // MMA commit
    uint64_t* acc_full = b_empty + kB;           // MMA commit
    uint64_t* acc_empty = acc_full + 2;          // the epilogue warps
    uint64_t* mma_done = acc_empty + 2;          // MMA commit (the final drain)
    __shared__ uint32_t s_tmem;

    const Work w = args.w;
    const int K = args.K;
    const int KS = K / kTcK;                 // A/B stages per item
    const int QS = (K + kTcQ - 1) / kTcQ;    // raw quarters per item
    constexpr int kQS = kTcQ / kTcK;         // A/B stages per quarter
    const int n_items = work_entries(w) * args.m_tiles;

    if (tid == 0) {
        for (int i = 0; i < kRaw; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kTcDecWarps);
        }
        for (int i = 0; i < kA; i++) {
            mbar_init(&a_full[i], kTcDecWarps);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < kB; i++) {
            mbar_init(&b_full[i], MODE == 0 ? 64 : 1);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kTcEpiWarps);
        }
        mbar_init(mma_done, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&s_tmem, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == 0) {
        // ---------------- raw weight producer: one quarter of every matrix per raw stage ----------------
        int rc = 0;
        bool ok = true;
        for (int j = 0; ok; j++) {
            const int id = (int) blockIdx.x + j * (int) gridDim.x;
            if (id >= n_items) break;
            const Entry en = work_entry(w, id / args.m_tiles);
            const int row = (en.shared ? 0 : en.e * args.m_tiles * kTcM) + (id % args.m_tiles) * kTcM;
            for (int q = 0; q < QS; q++) {
                const int rs = rc % kRaw;
                if (rc >= kRaw && !warp_wait(&raw_empty[rs], (uint32_t) ((rc / kRaw - 1) & 1))) {
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
            }
        }
        if (!ok && lane == 0) atomicOr(&g_smoe_status, kDevTimeout);
        if (lane == 0) drain_ring(raw_full, kRaw, rc);  // every copy has landed before shared memory is released
        __syncwarp();
    } else if (warp == 2 || (MODE == 0 && warp == 3)) {
        // ---------------- activation producers: the entry's hi and lo rows for each K stage ----------------
        // Tile row rho < npad is the hi row of entry row rho, row npad + rho its lo row (128-byte swizzle).
        // gate/up (rows are tokens): 16-byte cp.async copies, thread pt copying chunk pt & 7 of rows
        // (pt >> 3) + 8i, each thread's arrival firing when its copies have landed.  down (rows are consecutive
        // slots): TMA boxes of 16 rows.
        const int pt = tid - 64;
        const int ch = pt & 7;
        int bc = 0;
        bool ok = true;
        for (int j = 0; ok; j++) {
            const int id = (int) blockIdx.x + j * (int) gridDim.x;
            if (id >= n_items) break;
            const Entry en = work_entry(w, id / args.m_tiles);
            const int npad = (en.n + 15) & ~15;
            const int nrow = 2 * npad;  // tile rows, a multiple of 32
            const __half* src[kBRowsPerThread];
            if (MODE == 0) {
#pragma unroll
                for (int i = 0; i < kBRowsPerThread; i++) {
                    const int rho = (pt >> 3) + 8 * i;
                    const int er = min(rho < npad ? rho : rho - npad, en.n - 1);  // padding repeats the last row
                    src[i] = args.act + (size_t) (entry_token(w, en, en.beg + er) + (rho < npad ? 0 : args.act_rows)) *
                                            K + ch * 8;
                }
            }
            for (int ks = 0; ks < KS; ks++) {
                const int st = bc % kB;
                if (bc >= kB && !warp_wait(&b_empty[st], (uint32_t) ((bc / kB - 1) & 1))) {
                    ok = false;
                    break;
                }
                uint8_t* bt = sB + (size_t) st * kBTile;
                if (MODE == 0) {
                    const uint32_t bdst = smem_addr(bt);
#pragma unroll
                    for (int i = 0; i < kBRowsPerThread; i++) {
                        const int rho = (pt >> 3) + 8 * i;
                        if (rho < nrow) cp_async16(bdst + rho * 128 + ((ch ^ (rho & 7)) << 4), src[i] + ks * kTcK);
                    }
                    cp_async_arrive_noinc(&b_full[st]);
                } else {
                    if (lane == 0) mbar_expect_tx(&b_full[st], (uint32_t) (nrow * kTcK * 2));
                    __syncwarp();
                    const int i = lane & 7;  // lane i < 8: hi rows 16i.., lane 8 + i: lo rows npad + 16i..
                    if (lane < 16 && 16 * i < npad)
                        tma_load_2d(bt + ((lane >= 8 ? npad : 0) + 16 * i) * 128, &mact, ks * kTcK,
                                    (lane >= 8 ? args.act_rows : 0) + en.beg + 16 * i, &b_full[st]);
                }
                bc++;
            }
        }
        if (!ok && lane == 0) atomicOr(&g_smoe_status, kDevTimeout);
        if (MODE == 0) {
            cp_async_wait_all();  // every copy has landed before shared memory is released
        } else {
            if (lane == 0) drain_ring(b_full, kB, bc);
            __syncwarp();
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (lane 0): A from tensor memory, B from shared memory ----------------
        if (lane == 0) {
            int sc = 0;
            bool ok = true, issued = false;
            for (int j = 0; ok; j++) {
                const int id = (int) blockIdx.x + j * (int) gridDim.x;
                if (id >= n_items) break;
                const Entry en = work_entry(w, id / args.m_tiles);
                const int npad = (en.n + 15) & ~15;
                const int a = j % kAccBufs;
                if (j >= kAccBufs &&
                    !mbar_wait_sleep(&acc_empty[a], (uint32_t) ((j / kAccBufs - 1) & 1), kWaitLimitNs)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t idesc = umma_idesc_f16(kTcM, 2 * npad);  // hi and lo rows in one MMA
                const uint32_t d0 = tmem + (uint32_t) a * kAccCols;
                for (int ks = 0; ks < KS; ks++, sc++) {
                    const int sa = sc % kA, sb = sc % kB;
                    if (!mbar_wait_sleep(&b_full[sb], (uint32_t) ((sc / kB) & 1), kWaitLimitNs) ||
                        !mbar_wait_sleep(&a_full[sa], (uint32_t) ((sc / kA) & 1), kWaitLimitNs)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    fence_proxy_async();  // cp.async (generic proxy) writes -> the tensor core's reads
                    // descriptors advance by constants: 16 K values = 8 A columns = 32 B of a B row (2 in the
                    // descriptor's 16-byte address units)
                    const uint64_t bd = umma_desc_sw128(sB + (size_t) sb * kBTile);
                    const uint32_t at0 = tmem + kAOff + (uint32_t) sa * kACols;
                    const uint32_t first = ks > 0 ? 1u : 0u;
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        const uint32_t d = d0 + (uint32_t) m * kMatCols;
                        const uint32_t at = at0 + (uint32_t) m * (kTcK / 2);
#pragma unroll
                        for (int s = 0; s < kTcK / 16; s++) umma_f16_ts(d, at + 8 * s, bd + 2 * s, idesc, s > 0 ? 1u : first);
                    }
                    umma_commit(&a_empty[sa]);  // each stage is free once these MMAs have read it
                    umma_commit(&b_empty[sb]);
                    issued = true;
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
        // ---------------- decoders: raw Q2_0 -> fp16 A in tensor memory ----------------
        // Warp 4 + 4 role + q decodes rows 32q + lane (its tensor-memory lanes): gate/up, matrix `role` (all 64
        // values of the block); down, the block's code words 2 role and 2 role + 1.  Code word j, pair s lands in
        // A column 8j + s (low half value 16j + s, high half 16j + 8 + s: the K order of tc_kpos).
        const int q = warp & 3, role = (warp - 4) >> 2;
        const int m = MODE == 0 ? role : 0;
        constexpr int NW = MODE == 0 ? 4 : 2;  // code words per thread per stage
        const int j0 = MODE == 0 ? 0 : 2 * role;
        const int r = 32 * q + lane;
        int rc = 0, sc = 0;
        bool ok = true;
        for (int j = 0; ok; j++) {
            const int id = (int) blockIdx.x + j * (int) gridDim.x;
            if (id >= n_items) break;
            for (int qq = 0; qq < QS && ok; qq++) {
                const int rs = rc % kRaw;
                if (!warp_wait(&raw_full[rs], (uint32_t) ((rc / kRaw) & 1))) {
                    ok = false;
                    break;
                }
                const uint8_t* rowp = sRaw + ((size_t) rs * NMAT + m) * kRawMat + r * 144;
                const int k_end = min(KS, (qq + 1) * kQS);
                for (int ks = qq * kQS; ks < k_end; ks++, sc++) {
                    const int sa = sc % kA;
                    // the block's 18 bytes from aligned 4-byte words: rows are 144 B apart, so a block starts on a
                    // 4-byte boundary for even b (d and the first code pair share a word) and 2 bytes past one
                    // for odd b (d ends a word, the codes are aligned)
                    const int b = ks - qq * kQS;
                    const uint32_t* wp = reinterpret_cast<const uint32_t*>(rowp + ((b * 18) & ~3));
                    uint32_t wv[NW];
                    uint16_t dbits;
                    if ((b & 1) == 0) {
                        uint32_t raw5[NW + 1];
#pragma unroll
                        for (int i = 0; i <= NW; i++) raw5[i] = wp[j0 + i];
                        dbits = (uint16_t) raw5[0];  // only meaningful when j0 == 0 (see below)
#pragma unroll
                        for (int i = 0; i < NW; i++) wv[i] = __funnelshift_r(raw5[i], raw5[i + 1], 16);
                        if (j0 != 0) dbits = (uint16_t) wp[0];
                    } else {
#pragma unroll
                        for (int i = 0; i < NW; i++) wv[i] = wp[1 + j0 + i];
                        dbits = (uint16_t) (wp[0] >> 16);
                    }
                    const __half2 d2 = __half2half2(__ushort_as_half(dbits));
                    uint32_t col[8 * NW];
#pragma unroll
                    for (int i = 0; i < NW; i++) {
                        const uint32_t wq = wv[i], w10 = wq >> 10;
                        col[8 * i + 0] = dec_pair<0>(wq, w10, d2);
                        col[8 * i + 1] = dec_pair<1>(wq, w10, d2);
                        col[8 * i + 2] = dec_pair<2>(wq, w10, d2);
                        col[8 * i + 3] = dec_pair<3>(wq, w10, d2);
                        col[8 * i + 4] = dec_pair<4>(wq, w10, d2);
                        col[8 * i + 5] = dec_pair<5>(wq, w10, d2);
                        col[8 * i + 6] = dec_pair<6>(wq, w10, d2);
                        col[8 * i + 7] = dec_pair<7>(wq, w10, d2);
                    }
                    if (sc >= kA && !warp_wait(&a_empty[sa], (uint32_t) ((sc / kA - 1) & 1))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ta = tmem + ((uint32_t) (32 * q) << 16) + kAOff + (uint32_t) sa * kACols +
                                        (uint32_t) m * (kTcK / 2) + (uint32_t) (8 * j0);
                    tmem_st16(ta, col);
                    if (NW == 4) tmem_st16(ta + 16, col + 16);
                    if constexpr (NW == 4) tmem_wait_st32(col);
                    else tmem_wait_st16(col);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[sa]);
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_empty[rs]);
                rc++;
            }
        }
        if (!ok && lane == 0) atomicOr(&g_smoe_status, kDevTimeout);
    } else if (warp >= kTcEpiWarp0) {
        // ---------------- epilogue: tensor memory -> h (gate/up) or the slot rows (down) ----------------
        // Warp kTcEpiWarp0 + 4 hf + q reads tensor-memory lanes 32q..32q+31 (its rows) and the 8-token column
        // groups hf, hf + 2, hf + 4, ...
        const int wq = warp & 3;
        const int hf = (warp - kTcEpiWarp0) >> 2;
        // gate/up staging of this warp: g and u of its 32 rows for its tokens, [token][row]
        float* sg = sStage + (size_t) (warp - kTcEpiWarp0) * 2 * 32 * (kTcChunk / 2);
        float* su = sg + 32 * (kTcChunk / 2);
        bool ok = true;
        for (int j = 0; ok; j++) {
            const int id = (int) blockIdx.x + j * (int) gridDim.x;
            if (id >= n_items) break;
            const Entry en = work_entry(w, id / args.m_tiles);
            const int mt = id % args.m_tiles;
            const int npad = (en.n + 15) & ~15;
            const int a = j % kAccBufs;
            if (!warp_wait(&acc_full[a], (uint32_t) ((j / kAccBufs) & 1))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem + ((uint32_t) (32 * wq) << 16) + (uint32_t) a * kAccCols;
            const int row = mt * kTcM + 32 * wq + lane;  // this thread's output row
            // pass 1: accumulators (hi + lo columns) out of tensor memory
            for (int c0 = 8 * hf, tt = 0; c0 < en.n; c0 += 16, tt += 8) {
                uint32_t g8[8], gl8[8], u8[8], ul8[8];
                tmem_ld8(tbase + (uint32_t) c0, g8);
                tmem_ld8(tbase + (uint32_t) (npad + c0), gl8);
                if (MODE == 0) {
                    tmem_ld8(tbase + kMatCols + (uint32_t) c0, u8);
                    tmem_ld8(tbase + kMatCols + (uint32_t) (npad + c0), ul8);
                }
                tmem_wait_ld8x4(g8, gl8, u8, ul8);
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float g = __fadd_rn(__uint_as_float(g8[i]), __uint_as_float(gl8[i]));
                    if (MODE == 0) {
                        sg[(tt + i) * 32 + lane] = g;
                        su[(tt + i) * 32 + lane] = __fadd_rn(__uint_as_float(u8[i]), __uint_as_float(ul8[i]));
                    } else if (c0 + i < en.n) {
                        down_row(w, args.parts, en.beg + c0 + i, args.n_out)[row] = g;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[a]);  // the MMA may overwrite the buffer from here on
            if (MODE == 0) {
                // pass 2: SwiGLU, then the q8_1 rule over the warp's 32 rows (one block of h), stored as hi/lo
                const int col = (row & ~63) + tc_kpos(row & 63);
                for (int c0 = 8 * hf, tt = 0; c0 < en.n; c0 += 16, tt += 8) {
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int t = c0 + i;
                        if (t >= en.n) break;  // uniform across the warp
                        const int slot = en.beg + t;
                        // SwiGLU with the library expf (within 2 ulp; the dot products here already differ from
                        // the reference in f32 summation order), block max by one warp reduction (the order of
                        // non-negative floats is the order of their bit patterns)
                        const float gg = sg[(tt + i) * 32 + lane];
                        const float h = __fmul_rn(__fdiv_rn(gg, __fadd_rn(1.f, expf(-gg))), su[(tt + i) * 32 + lane]);
                        const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(h))));
                        float d = __fdiv_rn(amax, 127.f);
                        if (fabsf(d) > 65504.f) d = copysignf(65504.f, d);
                        float qv = 0.f;
                        if (amax != 0.f) qv = fminf(fmaxf(roundf(__fdiv_rn(h, d)), -127.f), 127.f);
                        const float v = __fmul_rn(qv, __half2float(__float2half_rn(d)));
                        const __half hi = __float2half_rn(v);
                        const __half lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
                        args.hh[(size_t) slot * args.n_out + col] = hi;
                        args.hh[((size_t) args.hh_rows + slot) * args.n_out + col] = lo;
                    }
                }
                __syncwarp();  // the staging area is rewritten by this warp's next item
            }
        }
        if (!ok && lane == 0) atomicOr(&g_smoe_status, kDevTimeout);
        if (MODE == 1) ep_signal_done(w.ep_done, gridDim.x * kTcEpiWarps);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
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

template <int MODE>
cudaError_t launch_tc(const CUtensorMap* maps, const TcArgs& a, cudaStream_t s) {
    const size_t smem = TcCfg<MODE>::smem;
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
                    weight_map(&maps[3], sup.base ? sup.base : up.base, n_ff, rb);
    if (!ok) return cudaErrorInvalidValue;
    maps[4] = maps[0];  // gate/up gathers its activation rows with cp.async: no activation tensor map
    TcArgs a{};
    a.w = w;
    a.act = xh;
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
    a.act = hh;
    a.K = n_ff;
    a.m_tiles = n_embd / kTcM;
    a.act_rows = R;
    a.n_out = n_embd;
    a.parts = parts;
    return launch_tc<1>(maps, a, s);
}

}  // namespace smoe
