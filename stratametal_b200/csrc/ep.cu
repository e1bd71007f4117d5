// ep.cu - expert parallelism over peer memory: the MoE block's two exchanges (dispatch of token rows to the
// ranks that own their experts, return of the down outputs to the token's rank) as stores into the other
// ranks' exchange areas, mapped into this process (CUDA IPC over NVLink / NVSwitch).  No collective library on
// the data path and no TMA multicast: every remote access is a plain store or a system-scope atomic.
//
// Protocol per step (each rank runs the same steps in the same order):
//   1. dispatch (this rank's tokens): every token's k ids to every rank, its q8_1 row to every rank that owns
//      one of its experts and to this rank (the shared expert), its count to every rank; then +1 on each rank's
//      disp_flag[this rank] (last warp, after a system-wide fence by every warp).
//   2. receive (as an expert owner): wait until every disp_flag reached this step, then turn the received rows
//      into local ids (-1: not here) and the expert kernels' activation image.  The down kernels write each
//      routed slot's row into the token rank's parts area, in router order, then +1 on its done_flag[this rank].
//   3. wait for every done_flag, then combine locally (router order, the shared expert computed here).
// Reuse is safe without more flags: a rank dispatches step n + 1 only after its step-n combine saw every
// owner's done signal, which each owner sends after it finished reading the step-n rows it received.
//
// Received rows are numbered from this rank's point of view: row r = b * max_tokens + t is token t of rank
// (rank + b) % world, so this rank's own tokens are rows [0, T) and the shared expert's slots map onto them.
#include "ep.cuh"

#include <algorithm>
#include <cstddef>

namespace smoe {

constexpr int kEpMaxWorld = 8;

// Header of every rank's exchange area (the rest: counts, ids, q8_1 rows, parts).  The first two arrays are
// written by other ranks; the rest only by this rank.
struct EpHeader {
    unsigned disp_flag[64];  // [source rank]
    unsigned done_flag[64];  // [owner rank]
    unsigned epoch;          // steps this rank began (its dispatch adds 1)
    unsigned disp_counter;   // finished warps of the running dispatch
    unsigned done_counter;   // finished warps of the running down launch
    int rank, world, max_tokens, H, k, qrow;
    long long off_count, off_ids, off_q8, off_parts;
    float* parts_of[kEpMaxWorld];    // [b]: parts area of rank (rank + b) % world, as this process maps it
    unsigned* done_of[kEpMaxWorld];  // [p]: &done_flag[rank] in rank p's area
    unsigned* disp_of[kEpMaxWorld];  // [p]: &disp_flag[rank] in rank p's area
    uint8_t* area_of[kEpMaxWorld];   // [p]: rank p's area
};
constexpr size_t kEpHeaderBytes = 4096;
static_assert(sizeof(EpHeader) <= kEpHeaderBytes, "exchange header");

namespace {
size_t ep_up256(size_t n) { return (n + 255) & ~(size_t) 255; }
struct EpOffsets {
    size_t count, ids, q8, parts, total;
};
EpOffsets ep_offsets(int H, int k, int Tm, int world) {
    EpOffsets o;
    const size_t qrow = (size_t) H / 32 * kQ8Block;
    size_t at = kEpHeaderBytes;
    o.count = at; at += ep_up256((size_t) kEpMaxWorld * 4);
    o.ids = at; at += ep_up256((size_t) world * Tm * k * 4);
    o.q8 = at; at += ep_up256((size_t) world * Tm * qrow);
    o.parts = at; at += ep_up256((size_t) Tm * k * H * 4);
    o.total = at;
    return o;
}
}  // namespace

size_t ep_arena_bytes(int H, int k, int max_tokens, int world) { return ep_offsets(H, k, max_tokens, world).total; }

float* const* ep_parts_table(void* arena) { return static_cast<EpHeader*>(arena)->parts_of; }
unsigned* const* ep_done_table(void* arena) { return static_cast<EpHeader*>(arena)->done_of; }
unsigned* ep_done_counter(void* arena) { return &static_cast<EpHeader*>(arena)->done_counter; }

// Host side, once per area before the first step (the area was zeroed when it was allocated): this rank's
// view of every rank's area.
cudaError_t ep_init(void* arena, void* const* peers, int rank, int world, int H, int k, int max_tokens) {
    const EpOffsets o = ep_offsets(H, k, max_tokens, world);
    EpHeader h;
    cudaError_t e = cudaMemcpy(&h, arena, sizeof h, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return e;
    h.rank = rank;
    h.world = world;
    h.max_tokens = max_tokens;
    h.H = H;
    h.k = k;
    h.qrow = H / 32 * kQ8Block;
    h.off_count = (long long) o.count;
    h.off_ids = (long long) o.ids;
    h.off_q8 = (long long) o.q8;
    h.off_parts = (long long) o.parts;
    for (int i = 0; i < kEpMaxWorld; i++) {
        h.parts_of[i] = nullptr;
        h.done_of[i] = h.disp_of[i] = nullptr;
        h.area_of[i] = nullptr;
    }
    for (int p = 0; p < world; p++) {
        uint8_t* a = static_cast<uint8_t*>(peers[p]);
        h.area_of[p] = a;
        h.done_of[p] = reinterpret_cast<EpHeader*>(a)->done_flag + rank;
        h.disp_of[p] = reinterpret_cast<EpHeader*>(a)->disp_flag + rank;
    }
    for (int b = 0; b < world; b++)
        h.parts_of[b] = reinterpret_cast<float*>(static_cast<uint8_t*>(peers[(rank + b) % world]) + o.parts);
    // only the fields this rank owns: the flags belong to the other ranks' writers
    const size_t from = offsetof(EpHeader, rank);
    return cudaMemcpy(static_cast<uint8_t*>(arena) + from, reinterpret_cast<uint8_t*>(&h) + from, sizeof h - from,
                      cudaMemcpyHostToDevice);
}

float* ep_parts(void* arena, int H, int k, int max_tokens, int world) {
    return reinterpret_cast<float*>(static_cast<uint8_t*>(arena) + ep_offsets(H, k, max_tokens, world).parts);
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned ld_volatile_u32(const unsigned* p) {
    return *reinterpret_cast<const volatile unsigned*>(p);
}

// Every flags[p] (p < n) must reach `target` (modulo 2^32).  Bounded: after kWaitLimitNs, or at once when an
// earlier wait of this library already gave up, the status word says so and the caller goes on without the data.
__device__ bool ep_wait_flags(const unsigned* flags, int n, unsigned target) {
    const uint64_t t0 = global_timer_ns();
    for (int p = 0; p < n; p++) {
        while ((int) (ld_acquire_sys(flags + p) - target) < 0) {
            if (ld_volatile_u32(&g_smoe_status) & kDevTimeout) return false;
            if (global_timer_ns() - t0 > kWaitLimitNs) {
                atomicOr(&g_smoe_status, kDevTimeout);
                return false;
            }
            __nanosleep(128);
        }
    }
    return true;
}

__global__ void __launch_bounds__(256) ep_dispatch_kernel(uint8_t* __restrict__ area, const int32_t* __restrict__ ids,
                                                          const uint8_t* __restrict__ xq, int T, int n_local) {
    EpHeader* h = reinterpret_cast<EpHeader*>(area);
    const int G = h->world, rank = h->rank, k = h->k, Tm = h->max_tokens, qrow = h->qrow;
    const int lane = threadIdx.x & 31;
    const int nwarps = (int) (gridDim.x * blockDim.x) >> 5;
    const int gw = (int) ((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    if (blockIdx.x == 0 && (int) threadIdx.x < G) {
        const int p = threadIdx.x;
        reinterpret_cast<int*>(h->area_of[p] + h->off_count)[(rank - p + G) % G] = T;
    }
    for (int t = gw; t < T; t += nwarps) {
        const int id0 = lane < k ? ids[(size_t) t * k + lane] : -1;
        const int id1 = lane + 32 < k ? ids[(size_t) t * k + lane + 32] : -1;
        unsigned m = 0;
        if (id0 >= 0 && id0 / n_local < G) m |= 1u << (id0 / n_local);
        if (id1 >= 0 && id1 / n_local < G) m |= 1u << (id1 / n_local);
        const unsigned mask = __reduce_or_sync(0xffffffffu, m) | (1u << rank);
        const int4* src = reinterpret_cast<const int4*>(xq + (size_t) t * qrow);
        for (int p = 0; p < G; p++) {
            const int b = (rank - p + G) % G;
            uint8_t* pa = h->area_of[p];
            int32_t* rid = reinterpret_cast<int32_t*>(pa + h->off_ids) + ((size_t) b * Tm + t) * k;
            if (lane < k) rid[lane] = id0;
            if (lane + 32 < k) rid[lane + 32] = id1;
            if ((mask >> p) & 1u) {
                int4* dst = reinterpret_cast<int4*>(pa + h->off_q8 + ((size_t) b * Tm + t) * qrow);
                for (int i = lane; i < qrow / 16; i += 32) dst[i] = src[i];
            }
        }
    }
    if (ep_last_warp(&h->disp_counter, (unsigned) nwarps)) {
        h->epoch += 1;
        for (int p = 0; p < G; p++) atomicAdd_system(h->disp_of[p], 1u);
    }
}

// One 32-value q8_1 block (36 bytes) into the SIMT kernels' layout: the words of quant_ka_warp, the scale read
// back from its fp16 bits, 0x4B400000 - the sum of the q.
__device__ __forceinline__ void ka_from_q8_warp(const uint8_t* __restrict__ qb, uint8_t* __restrict__ blk48, int lane,
                                                bool q2_layout) {
    const int q = (int) (int8_t) qb[4 + lane];
    int qs = q;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
    const int L = lane & 7;
    const int src0 = q2_layout ? 16 * (L >> 2) + (L & 3) : 4 * L;
    const int stride = q2_layout ? 4 : 1;
    uint32_t word = 0;
#pragma unroll
    for (int b = 0; b < 4; b++) {
        const int qb2 = __shfl_sync(0xffffffffu, q, src0 + b * stride);
        word |= ((uint32_t) qb2 & 0xFFu) << (8 * b);
    }
    if (lane < 8) reinterpret_cast<uint32_t*>(blk48)[lane] = word;
    if (lane == 8) reinterpret_cast<float*>(blk48)[8] = f16_to_f32((uint16_t) (qb[0] | (qb[1] << 8)));
    if (lane == 9) reinterpret_cast<int*>(blk48)[9] = 0x4B400000 - qs;
}

__global__ void __launch_bounds__(256) ep_receive_kernel(uint8_t* __restrict__ area, int expert_first, int n_local,
                                                         int32_t* __restrict__ oids, KAct xa, int xa_q2,
                                                         __half* __restrict__ xh) {
    EpHeader* h = reinterpret_cast<EpHeader*>(area);
    const int G = h->world, k = h->k, Tm = h->max_tokens, H = h->H, qrow = h->qrow;
    __shared__ int s_ok;
    if (threadIdx.x == 0) s_ok = ep_wait_flags(h->disp_flag, G, ld_volatile_u32(&h->epoch)) ? 1 : 0;
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int rows = G * Tm;
    const int nwarps = (int) (gridDim.x * blockDim.x) >> 5;
    const int* counts = reinterpret_cast<const int*>(area + h->off_count);
    const int32_t* rids = reinterpret_cast<const int32_t*>(area + h->off_ids);
    const int nblk = H / 32;
    for (int r = (int) ((blockIdx.x * blockDim.x + threadIdx.x) >> 5); r < rows; r += nwarps) {
        const int b = r / Tm, t = r % Tm;
        const int cnt = s_ok ? min(max(counts[b], 0), Tm) : 0;
        const bool valid = t < cnt;
        int o0 = -1, o1 = -1;
        if (valid) {
            if (lane < k) o0 = rids[(size_t) r * k + lane] - expert_first;
            if (lane + 32 < k) o1 = rids[(size_t) r * k + lane + 32] - expert_first;
            if (o0 >= n_local) o0 = -1;
            if (o1 >= n_local) o1 = -1;
            o0 = max(o0, -1);
            o1 = max(o1, -1);
        }
        if (lane < k) oids[(size_t) r * k + lane] = o0;
        if (lane + 32 < k) oids[(size_t) r * k + lane + 32] = o1;
        const bool present = __any_sync(0xffffffffu, o0 >= 0 || o1 >= 0) || (valid && b == 0);
        if (!present) continue;
        const uint8_t* q8 = area + h->off_q8 + (size_t) r * qrow;
        if (xa.base) {
            for (int blk = 0; blk < nblk; blk++)
                ka_from_q8_warp(q8 + blk * kQ8Block, xa.base + ((size_t) r * nblk + blk) * kKaBlock, lane, xa_q2 != 0);
        } else {
            // hi/lo fp16 image in the K order of tc_kpos: hi rows [0, rows), lo rows [rows, 2 rows)
            for (int blk = 0; blk < nblk; blk++) {
                const uint8_t* qb = q8 + blk * kQ8Block;
                const float d = f16_to_f32((uint16_t) (qb[0] | (qb[1] << 8)));
                const float v = __fmul_rn((float) (int8_t) qb[4 + lane], d);
                const __half hi = __float2half_rn(v);
                const int i = blk * 32 + lane;
                const size_t c = (size_t) (i & ~63) + tc_kpos(i & 63);
                xh[(size_t) r * H + c] = hi;
                xh[((size_t) rows + r) * H + c] = __float2half_rn(__fsub_rn(v, __half2float(hi)));
            }
        }
    }
}

__global__ void ep_wait_done_kernel(uint8_t* __restrict__ area) {
    EpHeader* h = reinterpret_cast<EpHeader*>(area);
    if (threadIdx.x == 0) (void) ep_wait_flags(h->done_flag, h->world, ld_volatile_u32(&h->epoch));
}

cudaError_t launch_ep_dispatch(void* arena, const int32_t* ids, const uint8_t* xq, int T, int k, int H, int n_local,
                               cudaStream_t s) {
    (void) k;
    (void) H;
    const int grid = std::max(1, std::min((T + 7) / 8, 148 * 4));
    ep_dispatch_kernel<<<grid, 256, 0, s>>>(static_cast<uint8_t*>(arena), ids, xq, T, n_local);
    return cudaGetLastError();
}

cudaError_t launch_ep_receive(void* arena, int k, int H, int expert_first, int n_local, int32_t* oids,
                              const KAct* xa, int xa_q2, __half* xh, cudaStream_t s, int rows) {
    (void) k;
    (void) H;
    const int grid = std::max(1, std::min((rows + 7) / 8, 148 * 8));
    ep_receive_kernel<<<grid, 256, 0, s>>>(static_cast<uint8_t*>(arena), expert_first, n_local, oids,
                                           xa ? *xa : KAct{nullptr}, xa_q2, xh);
    return cudaGetLastError();
}

cudaError_t launch_ep_wait_done(void* arena, cudaStream_t s) {
    ep_wait_done_kernel<<<1, 32, 0, s>>>(static_cast<uint8_t*>(arena));
    return cudaGetLastError();
}

}  // namespace smoe
