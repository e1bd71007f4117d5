// tq.cu - grouped expert GEMVs of the q8_1 integer contract on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, s32 accumulators in tensor memory): the decode-shaped path (a few tokens per expert),
// with results bit for bit those of the reference's row dot (iq.metal:459-514, host row_dot iq_parity.cpp:275-292).
//
// The contract.  A weight row against a q8_1 activation is a sum of 32-value partials
//   p_k = (d_w(k) * d_x(k)) * (float)(sum_i code_i * q_i - sum_i q_i)            (two f32 multiplies)
// added in the reference's order: partial k goes to lane k & 31 (in-lane sums start from 0 and follow k), then
// the 32 lane sums meet in an xor butterfly 16, 8, 4, 2, 1.  Here one MMA of K = 32 gives sum code * q of one
// partial for 128 rows x 8 tokens exactly (int32), each K step into its own tensor-memory columns (no
// accumulation across K), and the epilogue evaluates the partials and the reference's tree of f32 additions:
// lane sums s_l, level-1 nodes a_j = s_j + s_(j+16) (j < 16), then b_j = a_j + a_(j+8), c_j = b_j + b_(j+4),
// d_j = c_j + c_(j+2), result d_0 + d_1 (float addition commutes, so only the grouping matters).
//
// Shapes (swap-AB): M = 128 weight rows (tensor-memory lanes), N = 8 tokens (slots) of one work entry, K = 32
// per MMA.  P = K / 32 partials per row (16, 32 or 64).  A stage is 8 whole Q2_0 blocks of a row (16 K steps),
// two groups of four chosen so that the epilogue finishes level-2 tree nodes from each stage (tq_block below):
// P / 16 stages per item, one for down at n_ff = 512.  The epilogue keeps per token two level-2/3 nodes of its
// K parity across the stages and hands them over once per item (d_h below).
//
// Items.  Each CTA takes its groups in serpentine order over the heaviest-first work list; the down kernel is a
// programmatic dependent launch of gate/up (only its activation producers wait for the gate/up grid).
//
// Operands.  Weights: Q2_0 rows TMA-loaded raw (2D boxes of 144 B x 128 rows), decoded by eight warps into int8
// codes 0..3 straight into tensor memory (tcgen05.st; A of the MMA is read from tensor memory).  The word
// (qs >> 2j) & 0x03030303 holds in byte b the code of value 4b + j of a 16-value run; the activation rows are the
// expert kernels' layout (KAct), whose q words use the same order, so the MMA's K order matches without a
// shuffle.  Activations: per entry, the tokens' q words of every K step gathered by cp.async into the canonical
// K-major layout (8 tokens x 16 B core matrices), and each (token, K step)'s scale and sum of q beside them.
//
//   gate/up (MODE 0): gate and up rows of one 128-row tile per item, the epilogue applies SwiGLU and the q8_1
//                     rule to each warp's 32 rows (one 32-value block of h) and writes h in the KAct layout;
//   down (MODE 1):    128 output rows per item, the epilogue stores f32 per (slot, row).
//
// Warps: 0 raw weight producer (TMA; tensor memory allocation), 1 MMA issuer, 2-3 activation producers, 4-11
// decoders, 12-19 epilogue.  Every wait is bounded; on a timeout the kernel records kDevTimeout, drains what it
// issued (bounded), frees tensor memory and returns.
#include "common.cuh"
#include "ep.cuh"
#include "kernels.cuh"
#include "q8.cuh"

namespace smoe {

constexpr int kTqThreads = 640;
constexpr int kTqEpiWarp0 = 12;
constexpr int kTqM = 128;
constexpr int kTqN = 8;                 // tokens per MMA (work entries of kChunk = 8 slots)
constexpr uint32_t kTqQuarter = kTqM * 144;  // one 2D box: 8 blocks of 128 rows

// idesc of kind::i8: s32 accumulator (c_format 2), A and B signed 8-bit, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (N >> 3) << 17) | ((uint32_t) (M >> 4) << 24);
}

__device__ __forceinline__ void umma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc) {
    asm volatile("{ .reg .pred p; setp.ne.b32 p, 0, 0; tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p; }" ::"r"(
                     d_tmem),
                 "r"(a_tmem), "l"(b_desc), "r"(idesc)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tq_tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tq_cp16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void tq_cp8(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void tq_cp_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool tq_wait(uint64_t* bar, uint32_t parity) {
    const bool ok = mbar_wait_sleep(bar, parity, kWaitLimitNs);
    return __all_sync(0xffffffffu, ok);
}

// Packed f32x2 multiply and add with round-to-nearest: each lane rounds as the scalar operation does.  ptxas may
// still fuse a packed multiply into a packed add that consumes it, so they are used only where no addition
// takes a product.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
    float2 o;
    asm("{ .reg .b64 x, y, z; mov.b64 x, {%2, %3}; mov.b64 y, {%4, %5}; mul.rn.f32x2 z, x, y; mov.b64 {%0, %1}, z; }"
        : "=f"(o.x), "=f"(o.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return o;
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
    float2 o;
    asm("{ .reg .b64 x, y, z; mov.b64 x, {%2, %3}; mov.b64 y, {%4, %5}; add.rn.f32x2 z, x, y; mov.b64 {%0, %1}, z; }"
        : "=f"(o.x), "=f"(o.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return o;
}

// A stage is eight Q2_0 blocks of a row (16 K steps), in two groups of four slots whose partials, for the K steps
// of parity h (partials 2 b + h), finish tree nodes together:
//   P = 64 (stages m = 0..3): group 0 = blocks m, m+8, m+16, m+24 -> a_(2m+h), group 1 = m+4, m+12, m+20, m+28
//           -> a_(2m+8+h): b_(2m+h) = a_(2m+h) + a_(2m+8+h);
//   P = 32 (stages m = 0, 1): group g = blocks n, n+8, n+4, n+12 with n = m + 2g -> b_(2n+h) (one partial per
//           lane: a_j = (0 + p_j) + (0 + p_(j+16))), group 1 completing c_(2m+h) = b_(2m+h) + b_(2m+4+h);
//   P = 16 (one stage): group g = blocks 2g, 2g+1, 2g+4, 2g+5 -> b_(4g+h), b_(4g+2+h) (one partial on lanes
//           0..15: a_j = (0 + p_j) + 0), group 1 completing c_h and c_(2+h).
template <int P>
__host__ __device__ constexpr int tq_block(int m, int s) {
    return P == 64 ? m + (s >= 4 ? 4 + 8 * (s - 4) : 8 * s)
         : P == 32 ? (m + 2 * (s >> 2)) + ((s & 3) == 1 ? 8 : (s & 3) == 2 ? 4 : (s & 3) == 3 ? 12 : 0)
                   : 2 * (s >> 2) + (s & 3) + ((s & 3) >= 2 ? 2 : 0);
}

// A stage's blocks are its first block plus offsets that do not depend on the stage (the MMA issuer adds them
// to one descriptor).
template <int P>
constexpr bool tq_block_shifts() {
    for (int m = 0; m < 4; m++)
        for (int s = 0; s < 8; s++)
            if (tq_block<P>(m, s) - tq_block<P>(m, 0) != tq_block<P>(0, s) - tq_block<P>(0, 0)) return false;
    return true;
}
static_assert(tq_block_shifts<64>() && tq_block_shifts<32>() && tq_block_shifts<16>(), "stage block offsets");

// The order in which an item's stages run: P = 64: m = 0 2 1 3 (b_h, b_(4+h) -> c_h; b_(2+h), b_(6+h) ->
// c_(2+h)); otherwise in order.  The epilogue keeps 2 values per token (plus a_(2m+h) within a P = 64 stage).
template <int P>
__host__ __device__ constexpr int tq_order(int i) {
    return P == 64 ? (i >> 1) + 2 * (i & 1) : i;
}

// One item = one 128-row tile of one matrix for one work entry.  Gate/up runs an entry's gate tile and its up
// tile as two consecutive items on the same CTA (a group): the epilogue keeps g in registers and applies SwiGLU
// when u is done, and the activation buffer is loaded once per group.
template <int MODE, int P>
struct TqCfg {
    static constexpr int G = MODE == 0 ? 2 : 1;       // items per group (matrices of one tile)
    static constexpr int QS = P / 16;                 // raw quarters (8 blocks = 16 partials) per row
    static constexpr int NB = 8;                      // blocks (slots) per stage
    static constexpr int S = P / (2 * NB);            // stages per item
    static constexpr uint32_t kRawItem = QS * kTqQuarter;
    static constexpr int kRaw = kRawItem > 40 * 1024 ? 2 : 4;  // items of raw weights in flight
    static constexpr int kA = 2, kD = 2, kDW = 4;
    static constexpr int kBB = MODE == 0 || kRawItem > 40 * 1024 ? 2 : 4;  // activation buffers (groups)
    static constexpr uint32_t kStCols = NB * 16;      // one A or D stage: 2 NB K steps x 8 columns
    static constexpr uint32_t kTmemCols = 512;
    static_assert((kA + kD) * kStCols <= kTmemCols, "tensor memory budget");
    static constexpr uint32_t kBBytes = P * 256;      // q words: [K step][2 core matrices][8 tokens][16 B]
    static constexpr uint32_t kSBytes = P * kTqN * 8; // [K step][token] {d_x f32, sum q}
    static constexpr uint32_t kBBuf = kBBytes + kSBytes;
    static constexpr uint32_t kDWStage = NB * kTqM * 2;  // fp16 block scales [slot][row]
    static constexpr uint32_t kXch = 3 * 4 * kTqN * 32 * 4;  // d hand-over (2 buffers) and g, per lane quarter
    static constexpr int kBars = 80;                         // mbarriers
    static constexpr size_t smem = (size_t) kRaw * kRawItem + kBB * kBBuf + kDW * kDWStage + kXch + kBars * 8 + 1024;
    static_assert(smem <= 232448, "shared memory per block");
};

struct TqArgs {
    Work w;
    const uint8_t* act;  // activation rows in the KAct layout (tokens for gate/up, slots for down)
    int m_tiles;         // 128-row tiles per expert matrix
    int rows_per_expert; // n_ff (gate/up) or n_embd (down)
    int n_out;           // gate/up: n_ff (h row length); down: n_embd
    uint8_t* ha;         // gate/up: h in the KAct layout [slot][n_ff / 32][48]
    int ha_q2;           // the down matrix is Q2_0 (permuted q words)
    float* y;            // down: [slot][n_embd]
};

template <int MODE, int P>
__global__ void __launch_bounds__(kTqThreads, 1) tq_expert_kernel(const __grid_constant__ CUtensorMap mw0,
                                                                  const __grid_constant__ CUtensorMap mw1,
                                                                  const __grid_constant__ CUtensorMap sw0,
                                                                  const __grid_constant__ CUtensorMap sw1,
                                                                  TqArgs args) {
    using Cfg = TqCfg<MODE, P>;
    constexpr int G = Cfg::G, QS = Cfg::QS, S = Cfg::S, kRaw = Cfg::kRaw, kA = Cfg::kA, kD = Cfg::kD,
                  kDW = Cfg::kDW, kBB = Cfg::kBB, NB = Cfg::NB;
    constexpr uint32_t kStCols = Cfg::kStCols;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint8_t* sRaw = smem;                                          // [kRaw][QS][128 rows][144 B]
    uint8_t* sB = sRaw + (size_t) kRaw * Cfg::kRawItem;            // [kBB][kBBuf]
    uint16_t* sDW = reinterpret_cast<uint16_t*>(sB + kBB * Cfg::kBBuf);  // [kDW][4][128]
    float* sX = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(sDW) + kDW * Cfg::kDWStage);  // [2][4][8][32]
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sX) + Cfg::kXch);
    uint64_t* raw_full = bars;            // TMA tx
    uint64_t* raw_empty = raw_full + 4;   // decoders (8 warps)
    uint64_t* b_full = raw_empty + 4;     // 64 producer threads (cp.async)
    uint64_t* b_empty = b_full + 4;       // MMA commit + 8 epilogue warps
    uint64_t* a_full = b_empty + 4;       // the 4 decoder warps of the stage
    uint64_t* a_empty = a_full + kA;      // MMA commit
    uint64_t* d_full = a_empty + kA;      // MMA commit
    uint64_t* d_empty = d_full + kD;      // epilogue warps
    uint64_t* dw_full = d_empty + kD;     // the 4 decoder warps of the stage
    uint64_t* dw_empty = dw_full + kDW;   // epilogue warps
    uint64_t* x_full = dw_empty + kDW;    // [h][2][4] the h warp wrote its half of the hand-over buffer
    uint64_t* x_empty = x_full + 16;      // [h][2][4] the other warp read it
    uint64_t* mma_done = x_empty + 16;
    static_assert(4 * 4 + 2 * (kA + kD + kDW) + 2 * 16 + 1 <= Cfg::kBars, "mbarrier region");
    __shared__ uint32_t s_tmem;

    const Work w = args.w;
    const int n_groups = work_entries(w) * args.m_tiles;
    // gate/up: the down launch that follows may start now (programmatic dependent launch); its CTAs take SMs as
    // this grid's CTAs exit and set up while the last ones finish
    if (MODE == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // item j of this CTA: matrix j % G of group (j / G) gridDim.x + c, c = blockIdx.x in even rounds and
    // gridDim.x - 1 - blockIdx.x in odd ones.  The work list runs from the heaviest entries (eight tokens) to the
    // lightest, so the serpentine order gives each CTA a similar mix; a CTA's groups still increase with j.
    auto group_of = [&](int j) {
        const int round = j / G;
        return round * (int) gridDim.x + ((round & 1) ? (int) gridDim.x - 1 - (int) blockIdx.x : (int) blockIdx.x);
    };

    if (tid == 0) {
        for (int i = 0; i < 4; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], 8);
            mbar_init(&b_full[i], 64);
            mbar_init(&b_empty[i], 1 + 8);
        }
        for (int i = 0; i < kA; i++) {
            mbar_init(&a_full[i], 4);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < kD; i++) {
            mbar_init(&d_full[i], 1);
            mbar_init(&d_empty[i], 8);
        }
        for (int i = 0; i < kDW; i++) {
            mbar_init(&dw_full[i], 4);
            mbar_init(&dw_empty[i], 8);
        }
        for (int i = 0; i < 16; i++) {
            mbar_init(&x_full[i], 1);
            mbar_init(&x_empty[i], 1);
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
    const uint32_t tA = tmem, tD = tmem + kA * kStCols;

    if (warp == 0) {
        // ---------------- raw weights: the item's row tile, one box per quarter ----------------
        bool ok = true;
        int j = 0;
        for (;; j++) {
            const int gid = group_of(j);
            if (gid >= n_groups) break;
            const Entry en = work_entry(w, gid / args.m_tiles);
            const int mat = j % G;
            const int row = (en.shared ? 0 : en.e * args.rows_per_expert) + (gid % args.m_tiles) * kTqM;
            const int rs = j % kRaw;
            if (j >= kRaw && !tq_wait(&raw_empty[rs], (uint32_t) ((j / kRaw - 1) & 1))) {
                ok = false;
                break;
            }
            if (lane == 0) {
                uint8_t* dst = sRaw + (size_t) rs * Cfg::kRawItem;
                const CUtensorMap* map = en.shared ? (mat ? &sw1 : &sw0) : (mat ? &mw1 : &mw0);
                mbar_expect_tx(&raw_full[rs], Cfg::kRawItem);
                for (int q = 0; q < QS; q++) tq_tma_2d(dst + (size_t) q * kTqQuarter, map, q * 144, row, &raw_full[rs]);
            }
            __syncwarp();
        }
        if (!ok && lane == 0) atomicOr(&g_smoe_status, kDevTimeout);
        if (lane == 0)
            for (int i = max(0, j - kRaw); i < j; i++)
                mbar_wait_sleep(&raw_full[i % kRaw], (uint32_t) ((i / kRaw) & 1), kWaitLimitNs);
        __syncwarp();
    } else if (warp == 2 || warp == 3) {
        // ---------------- activations: the entry's slots, every K step, once per group ----------------
        // down: h is the previous grid's output.  Only these warps read it, so only they wait for that grid (a
        // no-op without a programmatic launch); the weight loads, decoding and set-up of the others overlap it.
        if (MODE == 1) asm volatile("griddepcontrol.wait;" ::: "memory");
        const int pt = tid - 64;  // 0..63
        bool ok = true;
        for (int g = 0; ok; g++) {
            const int gid = group_of(g * G);
            if (gid >= n_groups) break;
            const Entry en = work_entry(w, gid / args.m_tiles);
            const int bb = g % kBB;
            if (g >= kBB && !tq_wait(&b_empty[bb], (uint32_t) ((g / kBB - 1) & 1))) {
                ok = false;
                break;
            }
            uint8_t* buf = sB + (size_t) bb * Cfg::kBBuf;
            const uint32_t bq = smem_addr(buf), bs = smem_addr(buf + Cfg::kBBytes);
            // thread pt copies token t = pt / 8, K steps pt % 8, pt % 8 + 8, ...: its q bytes (two 16-byte halves)
            // and {d, sum q}.  gate/up reads the slot's token row of x, down the slot's own row of h.
            const int t = pt >> 3;
            if (t < en.n) {
                const int tok = MODE == 0 ? entry_token(w, en, en.beg + t) : en.beg + t;
                const uint8_t* row = args.act + (size_t) tok * ((size_t) P * kKaBlock);
#pragma unroll
                for (int k = pt & 7; k < P; k += 8) {
                    const uint8_t* src = row + (size_t) k * kKaBlock;
                    tq_cp16(bq + k * 256 + t * 16, src);
                    tq_cp16(bq + k * 256 + 128 + t * 16, src + 16);
                    tq_cp8(bs + (k * kTqN + t) * 8, src + 32);
                }
            }
            tq_cp_arrive(&b_full[bb]);
        }
        if (!ok && lane == 0) atomicOr(&g_smoe_status, kDevTimeout);
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_i8(kTqM, kTqN);
            int sa_c = 0, sd_c = 0;
            bool ok = true, issued = false;
            for (int j = 0; ok; j++) {
                const int gid = group_of(j);
                if (gid >= n_groups) break;
                const int g = j / G, bb = g % kBB;
                if (j % G == 0) {
                    if (!mbar_wait_sleep(&b_full[bb], (uint32_t) ((g / kBB) & 1), kWaitLimitNs)) {
                        ok = false;
                        break;
                    }
                    // the producers' cp.async writes of this group's activations -> the MMA's (async proxy) reads;
                    // the A operands come through tensor memory, so once per group is enough
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                }
                // K step k of the group's activations: the descriptor of K step 0 plus k * 256 B (start address
                // field, in 16-byte units, of an address below 256 KB: no carry out of the field)
                const uint64_t bd0 = umma_desc(sB + (size_t) bb * Cfg::kBBuf, 128, 256);
                for (int i = 0; i < S; i++, sa_c++, sd_c++) {
                    const int m = tq_order<P>(i);
                    const int sa = sa_c % kA, sd = sd_c % kD;
                    if (!mbar_wait_sleep(&a_full[sa], (uint32_t) ((sa_c / kA) & 1), kWaitLimitNs) ||
                        (sd_c >= kD && !mbar_wait_sleep(&d_empty[sd], (uint32_t) ((sd_c / kD - 1) & 1), kWaitLimitNs))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bdm = bd0 + (uint64_t) (2 * 16 * tq_block<P>(m, 0));
                    const uint32_t dst = tD + sd * kStCols, ast = tA + sa * kStCols;
#pragma unroll
                    for (int s = 0; s < NB; s++)
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int k_off = 2 * (tq_block<P>(0, s) - tq_block<P>(0, 0)) + h;
                            umma_i8_ts(dst + (uint32_t) (h * NB + s) * 8, ast + (uint32_t) (s * 2 + h) * 8,
                                       bdm + (uint64_t) (16 * k_off), idesc);
                        }
                    umma_commit(&a_empty[sa]);
                    umma_commit(&d_full[sd]);
                    issued = true;
                }
                if (!ok) break;
                if (j % G == G - 1) umma_commit(&b_empty[bb]);
            }
            if (!ok) atomicOr(&g_smoe_status, kDevTimeout);
            if (issued) {
                umma_commit(mma_done);
                mbar_wait_sleep(mma_done, 0, kWaitLimitNs);
            }
        }
        __syncwarp();
    } else if (warp >= 4 && warp < kTqEpiWarp0) {
        // ---------------- decoders: raw Q2_0 -> int8 codes in tensor memory, block scales to shared memory ------
        // warp 4 + 4 role + q decodes rows 32q + lane of every other stage (global stage count % 2 == role).
        const int q = warp & 3, role = (warp - 4) >> 2;
        const int r = 32 * q + lane;
        int sa_c = 0, dw_c = 0;
        bool ok = true;
        for (int j = 0; ok; j++) {
            if (group_of(j) >= n_groups) break;
            const int rs = j % kRaw;
            if (!tq_wait(&raw_full[rs], (uint32_t) ((j / kRaw) & 1))) {
                ok = false;
                break;
            }
            const uint8_t* rowq = sRaw + (size_t) rs * Cfg::kRawItem + (size_t) r * 144;
#pragma unroll
            for (int i = 0; i < S; i++, sa_c++, dw_c++) {
                if (!ok) break;
                if ((sa_c & 1) != role) continue;  // the two decoder roles take alternate stages
                const int m = tq_order<P>(i);
                const int sa = sa_c % kA, sw = dw_c % kDW;
                if (sa_c >= kA && !tq_wait(&a_empty[sa], (uint32_t) ((sa_c / kA - 1) & 1))) {
                    ok = false;
                    break;
                }
                if (dw_c >= kDW && !tq_wait(&dw_empty[sw], (uint32_t) ((dw_c / kDW - 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint16_t* dw = sDW + (size_t) sw * (Cfg::kDWStage / 2);
#pragma unroll
                for (int g4 = 0; g4 < NB / 4; g4++) {  // four slots at a time
                    uint32_t col[64];  // slot 4 g4 + sl, half h, word c at 16 sl + 8 h + c
#pragma unroll
                    for (int sl = 0; sl < 4; sl++) {
                        const int b = tq_block<P>(m, 4 * g4 + sl);
                        const int o = ((b & 7) * 18) & 15;  // the block's offset inside its 16-byte chunk (even)
                        const uint4* cp =
                            reinterpret_cast<const uint4*>(rowq + (size_t) (b >> 3) * kTqQuarter + (b & 7) * 18 - o);
                        const uint4 c0 = cp[0], c1 = cp[1];
                        const uint32_t wv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                        const int wi = (o + 2) >> 2;                      // the 16 code bytes start at byte o + 2
                        const uint32_t sh = (uint32_t) ((o + 2) & 3) * 8u;  // 0 or 16
                        uint32_t qw[4];
#pragma unroll
                        for (int x = 0; x < 4; x++)
                            qw[x] = sh ? __funnelshift_r(wv[wi + x], wv[wi + x + 1 < 8 ? wi + x + 1 : 7], sh) : wv[wi + x];
                        dw[(4 * g4 + sl) * kTqM + r] = (uint16_t) (wv[o >> 2] >> ((o & 3) * 8));
#pragma unroll
                        for (int h = 0; h < 2; h++)
#pragma unroll
                            for (int hw = 0; hw < 2; hw++)
#pragma unroll
                                for (int jj = 0; jj < 4; jj++)
                                    col[16 * sl + 8 * h + 4 * hw + jj] = (qw[2 * h + hw] >> (2 * jj)) & 0x03030303u;
                    }
                    const uint32_t ta = tA + ((uint32_t) (32 * q) << 16) + sa * kStCols + (uint32_t) g4 * 64;
                    tmem_st16(ta, col);
                    tmem_st16(ta + 16, col + 16);
                    tmem_st16(ta + 32, col + 32);
                    tmem_st16(ta + 48, col + 48);
                    tmem_wait_st32(col);
                    tmem_wait_st32(col + 32);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&a_full[sa]);
                    mbar_arrive(&dw_full[sw]);
                }
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[rs]);
        }
        if (!ok && lane == 0) atomicOr(&g_smoe_status, kDevTimeout);
    } else if (warp >= kTqEpiWarp0) {
        // ---------------- epilogue ----------------
        // Warp 12 + 4 h + q owns rows 32q + lane and the partials of half h (K steps 2 b + h) of every token.  The
        // reference's tree keeps the two parities apart until its last addition (a_j, b_j, c_j and d_j only meet
        // nodes of the same parity), so each warp finishes d_h and the h = 1 warp hands d_1 over once per item.
        const int q = warp & 3, hh = (warp - kTqEpiWarp0) >> 2;
        const int r = 32 * q + lane;
        int sd_c = 0, dw_c = 0;
        bool ok = true;
        float* gs = sX + (size_t) 2 * 4 * kTqN * 32 + (size_t) q * kTqN * 32;  // gate/up: g until the up item
        for (int j = 0; ok; j++) {
            const int gid = group_of(j);
            if (gid >= n_groups) break;
            const Entry en = work_entry(w, gid / args.m_tiles);
            const int mt = gid % args.m_tiles;
            const int mat = j % G, bb = (j / G) % kBB;
            const uint8_t* buf = sB + (size_t) bb * Cfg::kBBuf;
            const float2* sc = reinterpret_cast<const float2*>(buf + Cfg::kBBytes);  // [K step][token] {d, sum q}
            // Per token: B[] holds b_h, b_(2+h), then c_h, c_(2+h).  Each stage finishes level-2 nodes; the stages
            // run in an order that finishes level-3 pairs early (tq_order).
            float B[kTqN][2];
            // one copy of the stage code serves every stage (a smaller instruction footprint): the node a stage
            // writes is chosen by selects on m & 1, so the register arrays keep constant indices
#pragma unroll 1
            for (int i = 0; i < S; i++) {
                const int m = tq_order<P>(i);
                const int c = sd_c + i, cw = dw_c + i;
                const int sd = c % kD, sw = cw % kDW;
                if (!tq_wait(&d_full[sd], (uint32_t) ((c / kD) & 1)) || !tq_wait(&dw_full[sw], (uint32_t) ((cw / kDW) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint16_t* dw = sDW + (size_t) sw * (Cfg::kDWStage / 2);
                float a0[kTqN];  // P = 64: a_(2m+h) of the first four slots, until a_(2m+8+h) arrives
#pragma unroll
                for (int g4 = 0; g4 < NB / 4; g4++) {
                    uint32_t v[32];  // slot 4 g4 + sl, token t at column 8 sl + t (the K steps 2 b + h)
                    tmem_ld32(tD + ((uint32_t) (32 * q) << 16) + sd * kStCols + (uint32_t) (hh * NB + 4 * g4) * 8, v);
                    float dws[4];
#pragma unroll
                    for (int sl = 0; sl < 4; sl++) dws[sl] = f16_to_f32(dw[(4 * g4 + sl) * kTqM + r]);
                    tmem_wait_ld32(v);
                    if (g4 == NB / 4 - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            mbar_arrive(&d_empty[sd]);
                            mbar_arrive(&dw_empty[sw]);
                        }
                    }
#pragma unroll
                    for (int t = 0; t < kTqN; t++) {
                        if (t >= en.n) break;  // uniform across the warp
                        // p_s = (d_w * d_x) * (float) (sum code q - sum q), slots in pairs
                        float2 sq[4];
#pragma unroll
                        for (int sl = 0; sl < 4; sl++)
                            sq[sl] = sc[(2 * tq_block<P>(m, 4 * g4 + sl) + hh) * kTqN + t];  // {d_x, seed}
                        const float2 kBias = make_float2(-12582912.0f, -12582912.0f);
                        // Packed f32x2 only where no addition consumes the result (ptxas may fuse a packed multiply
                        // into a following packed add, which would round once instead of twice): the integer-to-
                        // float step and d_w * d_x.  The product with f and every addition stay scalar _rn
                        // operations, which are never contracted.
                        float2 pp[2];
#pragma unroll
                        for (int u = 0; u < 2; u++) {
                            const float2 f = add2_rn(
                                make_float2(__int_as_float(__float_as_int(sq[2 * u].y) + (int) v[8 * (2 * u) + t]),
                                            __int_as_float(__float_as_int(sq[2 * u + 1].y) + (int) v[8 * (2 * u + 1) + t])),
                                kBias);
                            const float2 dd = mul2_rn(make_float2(dws[2 * u], dws[2 * u + 1]),
                                                      make_float2(sq[2 * u].x, sq[2 * u + 1].x));
                            pp[u] = make_float2(__fmul_rn(dd.x, f.x), __fmul_rn(dd.y, f.y));
                        }
                        if (P == 64) {
                            // four slots: a = ((0 + p_l) + p_(l+32)) + ((0 + p_(l+16)) + p_(l+48)), l = 2m+h (+8)
                            const float a = __fadd_rn(__fadd_rn(__fadd_rn(0.f, pp[0].x), pp[1].x),
                                                      __fadd_rn(__fadd_rn(0.f, pp[0].y), pp[1].y));
                            if (g4 == 0) {
                                a0[t] = a;
                            } else {
                                const float bj = __fadd_rn(a0[t], a);  // b_(2m+h)
                                // order m = 0 2 1 3: b_h, b_(4+h) -> c_h; b_(2+h), b_(6+h) -> c_(2+h)
                                const float nv = m < 2 ? bj : __fadd_rn((m & 1) ? B[t][1] : B[t][0], bj);
                                if (m & 1) B[t][1] = nv;
                                else B[t][0] = nv;
                            }
                        } else if (P == 32) {
                            // blocks n, n+8, n+4, n+12 (n = m + 2 g4): b_(2n+h) = a_(2n+h) + a_(2n+8+h),
                            // a_j = (0 + p_j) + (0 + p_(j+16))
                            const float bj = __fadd_rn(__fadd_rn(__fadd_rn(0.f, pp[0].x), __fadd_rn(0.f, pp[0].y)),
                                                       __fadd_rn(__fadd_rn(0.f, pp[1].x), __fadd_rn(0.f, pp[1].y)));
                            // group 0: b_(2m+h); group 1: b_(2m+4+h) completes c_(2m+h)  (m = 0, 1)
                            const float nv = g4 == 0 ? bj : __fadd_rn(m ? B[t][1] : B[t][0], bj);
                            if (m) B[t][1] = nv;
                            else B[t][0] = nv;
                        } else {
                            // blocks 2 g4 + {0, 1, 4, 5}: lanes 4 g4 + 2s + h and 4 g4 + 2s + 8 + h (s < 2) hold
                            // one partial each, lanes 16..31 nothing: a = (0 + p) + 0, b = a + a'
                            const float2 b01 = make_float2(  // b_(4m+h) from slots 0, 2; b_(4m+2+h) from 1, 3
                                __fadd_rn(__fadd_rn(__fadd_rn(0.f, pp[0].x), 0.f), __fadd_rn(__fadd_rn(0.f, pp[1].x), 0.f)),
                                __fadd_rn(__fadd_rn(__fadd_rn(0.f, pp[0].y), 0.f), __fadd_rn(__fadd_rn(0.f, pp[1].y), 0.f)));
                            if (g4 == 0) {
                                B[t][0] = b01.x;
                                B[t][1] = b01.y;
                            } else {  // c_h = b_h + b_(4+h), c_(2+h) = b_(2+h) + b_(6+h)
                                B[t][0] = __fadd_rn(B[t][0], b01.x);
                                B[t][1] = __fadd_rn(B[t][1], b01.y);
                            }
                        }
                    }
                }
            }
            sd_c += S;
            dw_c += S;
            if (!ok) break;
            if (mat == G - 1) {  // the activation buffer (scales) is no longer needed
                __syncwarp();
                if (lane == 0) mbar_arrive(&b_empty[bb]);
            }
            // d_h = c_h + c_(2+h); the result is d_0 + d_1.  Gate and down items: the h = 1 warp hands d_1 to the
            // h = 0 warp, which finishes every token.  Up items (the SwiGLU and q8_1 step): token t is finished by
            // the warp of half t & 1, each warp handing the other its d_h of the other's tokens (d_1 + d_0 = d_0 +
            // d_1 exactly: a two-operand IEEE addition is commutative).  The g of a token reaches its up finisher
            // through gs, written by the h = 0 warp before it signals the up item's hand-over.
            const bool split = MODE == 0 && mat == 1;
            const int xb = j & 1;  // gate/up: xb = mat, so the gate and up items keep to their own barriers
            float* xs = sX + ((size_t) xb * 4 + q) * kTqN * 32;  // [token][lane]: d of the token's other half
            const uint32_t xpar = (uint32_t) ((j / 2) & 1);
            float dsum[kTqN];
#pragma unroll
            for (int t = 0; t < kTqN; t++) {
                if (t >= en.n) break;  // uniform across the warp
                dsum[t] = __fadd_rn(B[t][0], B[t][1]);
            }
            // x_full[h]: warp h wrote its part of xs; x_empty[h]: the other warp read it (the part is free again)
            if (split || hh == 1) {
                if (j >= 2 && !tq_wait(&x_empty[(hh * 2 + xb) * 4 + q], xpar ^ 1u)) {
                    ok = false;
                    break;
                }
#pragma unroll
                for (int t = 0; t < kTqN; t++) {
                    if (t >= en.n) break;
                    if (!split || (t & 1) != hh) xs[t * 32 + lane] = dsum[t];
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&x_full[(hh * 2 + xb) * 4 + q]);
                if (!split) continue;
            }
            if (!tq_wait(&x_full[((1 - hh) * 2 + xb) * 4 + q], xpar)) {
                ok = false;
                break;
            }
            if (!split) {
#pragma unroll
                for (int t = 0; t < kTqN; t++) {
                    if (t >= en.n) break;
                    const float res = __fadd_rn(dsum[t], xs[t * 32 + lane]);
                    if (MODE == 1) down_row(w, args.y, en.beg + t, args.n_out)[mt * kTqM + r] = res;
                    else gs[t * 32 + lane] = res;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&x_empty[(2 + xb) * 4 + q]);
                continue;
            }
            float own[kTqN / 2] = {0.f, 0.f, 0.f, 0.f};  // the results of tokens hh + 2u
#pragma unroll
            for (int u = 0; u < kTqN / 2; u++) {
                if (2 * u + hh >= en.n) break;
                own[u] = __fadd_rn(hh ? dsum[2 * u + 1] : dsum[2 * u], xs[(2 * u + hh) * 32 + lane]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&x_empty[((1 - hh) * 2 + xb) * 4 + q]);
            const int n_own = (en.n - hh + 1) >> 1;
            if (n_own > 0) {
                // SwiGLU of the warp's (at most four) tokens without branches between them, so their fp64 exps
                // overlap (a token past the entry's count computes on stale values and is not stored), then the
                // q8_1 rule over the warp's 32 rows (one 32-value block of h) per token
                float hv[kTqN / 2];
#pragma unroll
                for (int u = 0; u < kTqN / 2; u++) hv[u] = silu_mul(gs[(2 * u + hh) * 32 + lane], own[u]);
#pragma unroll
                for (int u = 0; u < kTqN / 2; u++) gs[(2 * u + hh) * 32 + lane] = hv[u];
                const int nb = args.n_out / 32;
                const int blk = (mt * kTqM + 32 * q) / 32;
#pragma unroll 1
                for (int u = 0; u < n_own; u++)
                    quant_ka_warp(gs[(2 * u + hh) * 32 + lane],
                                  args.ha + ((size_t) (en.beg + 2 * u + hh) * nb + blk) * kKaBlock, lane,
                                  args.ha_q2 != 0);
            }
        }
        if (!ok && lane == 0) atomicOr(&g_smoe_status, kDevTimeout);
        if (MODE == 1) ep_signal_done(w.ep_done, gridDim.x * 8);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

namespace {

template <int MODE, int P>
cudaError_t launch_tq(const CUtensorMap* maps, const TqArgs& a, cudaStream_t s) {
    const size_t smem = TqCfg<MODE, P>::smem;
    cudaError_t err =
        cudaFuncSetAttribute(tq_expert_kernel<MODE, P>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (err != cudaSuccess) return err;
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    if (MODE == 0) {
        tq_expert_kernel<MODE, P><<<nsm, kTqThreads, smem, s>>>(maps[0], maps[1], maps[2], maps[3], a);
        return cudaGetLastError();
    }
    // down: launched as a programmatic dependent of the gate/up grid before it (see griddepcontrol above)
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned) nsm);
    cfg.blockDim = dim3(kTqThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tq_expert_kernel<MODE, P>, maps[0], maps[1], maps[2], maps[3], a);
}

template <int MODE>
cudaError_t launch_tq_p(int P, const CUtensorMap* maps, const TqArgs& a, cudaStream_t s) {
    if (P == 16) return launch_tq<MODE, 16>(maps, a, s);
    if (P == 32) return launch_tq<MODE, 32>(maps, a, s);
    if (P == 64) return launch_tq<MODE, 64>(maps, a, s);
    return cudaErrorInvalidValue;
}

}  // namespace

bool tq_qualifies(int H, int F) {
    const auto okp = [](int n) { return n == 512 || n == 1024 || n == 2048; };
    return okp(H) && okp(F);
}

cudaError_t launch_tq_gate_up(Matrix gate, Matrix up, Matrix sgate, Matrix sup, Work w, int n_expert, KAct xa,
                              KAct ha, int down_q2, int n_embd, int n_ff, cudaStream_t s) {
    const int rb = (n_embd / 64) * 18;
    const int64_t routed_rows = (int64_t) n_ff * n_expert;
    CUtensorMap maps[4];
    const bool ok = weight_map(&maps[0], gate.base, routed_rows, rb) && weight_map(&maps[1], up.base, routed_rows, rb) &&
                    weight_map(&maps[2], sgate.base ? sgate.base : gate.base, n_ff, rb) &&
                    weight_map(&maps[3], sup.base ? sup.base : up.base, n_ff, rb);
    if (!ok) return cudaErrorInvalidValue;
    TqArgs a{};
    a.w = w;
    a.act = xa.base;
    a.m_tiles = n_ff / kTqM;
    a.rows_per_expert = n_ff;
    a.n_out = n_ff;
    a.ha = ha.base;
    a.ha_q2 = down_q2;
    return launch_tq_p<0>(n_embd / 32, maps, a, s);
}

cudaError_t launch_tq_down(Matrix down, Matrix sdown, Work w, int n_expert, KAct ha, float* y, int n_ff, int n_embd,
                           cudaStream_t s) {
    const int rb = (n_ff / 64) * 18;
    const int64_t routed_rows = (int64_t) n_embd * n_expert;
    CUtensorMap maps[4];
    const uint8_t* sd = sdown.base ? sdown.base : down.base;
    const bool ok = weight_map(&maps[0], down.base, routed_rows, rb) && weight_map(&maps[2], sd, n_embd, rb);
    if (!ok) return cudaErrorInvalidValue;
    maps[1] = maps[0];
    maps[3] = maps[2];
    TqArgs a{};
    a.w = w;
    a.act = ha.base;
    a.m_tiles = n_embd / kTqM;
    a.rows_per_expert = n_embd;
    a.n_out = n_embd;
    a.y = y;
    return launch_tq_p<1>(n_ff / 32, maps, a, s);
}

}  // namespace smoe
