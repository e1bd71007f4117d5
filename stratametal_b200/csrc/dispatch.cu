// dispatch.cu - token -> expert grouping (row a11): per-expert counts, exclusive prefix sums, the list of
// experts with rows, and a stable permutation of the (token, k) pairs into contiguous per-expert groups.
//
// Contract: fused::group (include/strata/prefill/moe_fused.hpp:46-50) - slot[i] is the grouped row of pair
// i = t * k + j and src[row] its token.  The reference leaves the order inside an expert free; here it is
// token order, so every replay groups identically (and combine reads rows in router order).
//
// One CTA of 1024 threads walks the tokens in chunks of 64: each chunk builds, per expert, a 64-bit mask of
// the chunk's tokens that route to it; popcounts of those masks give the counts, and the popcount of the
// mask below a token gives that token's rank inside its expert.
#include "common.cuh"
#include "kernels.cuh"

namespace smoe {

size_t group_tables_bytes(int n_expert) {
    const size_t n = (size_t) n_expert * 3 + 1 + 1 + 4;
    return (n * 4 + 255) & ~(size_t) 255;
}

GroupTables group_tables_at(void* base, int n_expert) {
    int32_t* p = static_cast<int32_t*>(base);
    GroupTables g;
    g.counts = p;
    g.offsets = p + n_expert;
    g.active = p + 2 * n_expert + 1;
    g.n_active = p + 3 * n_expert + 1;
    g.work = p + 3 * n_expert + 2;
    return g;
}

size_t sched_bytes(int E, int T, int k, int chunk) {
    return ((size_t) 3 * sched_capacity(E, T, k, chunk) * 4 + 4 + 255) & ~(size_t) 255;
}

Sched sched_at(void* base, int E, int T, int k, int chunk) {
    const int cap = sched_capacity(E, T, k, chunk);
    int32_t* p = static_cast<int32_t*>(base);
    return Sched{p, p + cap, p + 2 * cap, p + 3 * cap, chunk};
}

// True when pair i names an expert that an earlier pair of the same token already named.  The router never does
// (its k ids are distinct); a caller-supplied routing that does is malformed: the repeated pair gets no row
// (slot -1), the device status records BAD_ID, and the counts include each (token, expert) once.
__device__ __forceinline__ bool repeats_earlier(const int32_t* __restrict__ ids, size_t i, int k, int e) {
    for (size_t j = i - i % (size_t) k; j < i; j++)
        if (ids[j] == e) return true;
    return false;
}

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

__device__ __forceinline__ int block_excl_scan(int v, int* warp_sums, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < (int) (blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        warp_sums[lane] = w;  // inclusive
    }
    __syncthreads();
    const int before = warp > 0 ? warp_sums[warp - 1] : 0;
    if (total) *total = warp_sums[(blockDim.x >> 5) - 1];
    __syncthreads();
    return before + x - v;
}

// The work list from the grouping tables (one CTA of 1024 threads, thread e = expert e): experts bucketed by
// min(count, 63), heaviest bucket first, ascending id inside a bucket (per-warp bucket counts, scanned
// bucket-major then warp-minor, plus the rank among same-bucket lanes), then each expert cut into chunks of at
// most sched.chunk slots.
// counts / offsets: the tables as this CTA holds them (shared memory when it just computed them); whist
// (32 x 64 ints) and sorted (kMaxExperts ints): shared scratch.
__device__ void build_sched(const int* counts, const int* offsets, int n_active, Sched sched, int E, int* warp_sums,
                           int (*whist)[64], int* sorted) {
    __shared__ int bucket_off[64];
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    for (int i = tid; i < 32 * 64; i += blockDim.x) whist[i / 64][i % 64] = 0;
    __syncthreads();
    const int e = tid;
    const int cnt = e < E ? counts[e] : 0;
    const int b = cnt > 0 ? 63 - min(cnt, 63) : -1;
    if (b >= 0) atomicAdd(&whist[warp][b], 1);
    __syncthreads();
    if (tid < 64) {
        int acc = 0;
        for (int w = 0; w < 32; w++) {
            const int t = whist[w][tid];
            whist[w][tid] = acc;
            acc += t;
        }
        bucket_off[tid] = acc;
    }
    __syncthreads();
    if (tid < 32) {  // exclusive scan of the 64 bucket totals by one warp (two per lane)
        const int a = bucket_off[2 * tid], b = bucket_off[2 * tid + 1];
        int x = a + b;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (tid >= o) x += y;
        }
        const int before = x - a - b;
        bucket_off[2 * tid] = before;
        bucket_off[2 * tid + 1] = before + a;
    }
    __syncthreads();
    const uint32_t same = __match_any_sync(0xffffffffu, b);
    if (b >= 0) sorted[bucket_off[b] + whist[warp][b] + __popc(same & lanemask_lt())] = e;
    __syncthreads();
    const int ej = tid < n_active ? sorted[tid] : -1;
    const int cj = ej >= 0 ? counts[ej] : 0;
    const int chunk = sched.chunk;
    const int nch = (cj + chunk - 1) / chunk;
    int total = 0;
    const int off = block_excl_scan(nch, warp_sums, &total);
    if (ej >= 0) {
        const int base = offsets[ej];
        for (int c = 0; c < nch; c++) {
            sched.e[off + c] = ej;
            sched.beg[off + c] = base + c * chunk;
            sched.n[off + c] = min(chunk, cj - c * chunk);
        }
    }
    if (tid == 0) sched.count[0] = total;
}

// One CTA, up to kGroupWideMinTokens tokens (4 chunks of 64): every chunk's per-expert token masks are built once
// and kept in shared memory; the counts, the exclusive offsets, the slots and the work list all come from them.
constexpr int kGroupMaxChunks = kGroupWideMinTokens / 64;
__global__ void __launch_bounds__(1024) group_kernel(const int32_t* __restrict__ ids, int T, int k, int E,
                                                     GroupTables g, int32_t* __restrict__ slot,
                                                     int32_t* __restrict__ src, Sched sched, int with_sched,
                                                     int skip_negative, int32_t* __restrict__ pair) {
    __shared__ unsigned long long mask[kGroupMaxChunks][kMaxExperts];
    __shared__ int cnt_s[kMaxExperts];
    __shared__ int off_s[kMaxExperts];
    __shared__ int warp_sums[32];
    __shared__ int n_active_s;
    const int tid = threadIdx.x;
    const int nchunks = (T + 63) / 64;

    for (int i = tid; i < nchunks * E; i += blockDim.x) mask[i / E][i % E] = 0ull;
    __syncthreads();
    for (int p = tid; p < T * k; p += blockDim.x) {
        const int t = p / k;
        const int e = ids[p];
        if (e >= 0 && e < E) atomicOr(&mask[t >> 6][e], 1ull << (t & 63));
    }
    __syncthreads();
    // counts -> exclusive offsets and the active list (experts with rows, ascending id)
    int carry = 0, carry_act = 0;
    for (int e0 = 0; e0 < E; e0 += blockDim.x) {
        const int e = e0 + tid;
        int cnt = 0;
        if (e < E)
            for (int c = 0; c < nchunks; c++) cnt += __popcll(mask[c][e]);
        int tot, tot_act;
        const int off = block_excl_scan(cnt, warp_sums, &tot);
        const int act = block_excl_scan(cnt > 0 ? 1 : 0, warp_sums, &tot_act);
        if (e < E) {
            cnt_s[e] = cnt;
            off_s[e] = carry + off;
            g.counts[e] = cnt;
            g.offsets[e] = carry + off;
            if (cnt > 0) g.active[carry_act + act] = e;
        }
        carry += tot;
        carry_act += tot_act;
    }
    if (tid == 0) {
        g.offsets[E] = carry;
        g.n_active[0] = carry_act;
        n_active_s = carry_act;
        g.work[0] = g.work[1] = g.work[2] = g.work[3] = 0;
    }
    __syncthreads();
    // slots: expert base + the pairs of that expert in earlier chunks + the rank among this chunk's tokens
    for (int i = tid; i < T * k; i += blockDim.x) {
        const int t = i / k, c = t >> 6, tl = t & 63;
        const int e = ids[i];
        if (e < 0 || e >= E || repeats_earlier(ids, (size_t) i, k, e)) {
            slot[i] = -1;
            if (!(skip_negative && e < 0)) atomicOr(&g_smoe_status, kDevBadId);
            continue;
        }
        int pos = off_s[e] + __popcll(mask[c][e] & ((1ull << tl) - 1ull));
        for (int cc = 0; cc < c; cc++) pos += __popcll(mask[cc][e]);
        slot[i] = pos;
        if (src) src[pos] = t;
        if (pair) pair[pos] = i;
    }
    __syncthreads();
    // the work list reuses the mask memory as its scratch
    if (with_sched)
        build_sched(cnt_s, off_s, n_active_s, sched, E, warp_sums, reinterpret_cast<int (*)[64]>(&mask[0][0]),
                    reinterpret_cast<int*>(&mask[0][0]) + 32 * 64);
}

// Any number of tokens in one CTA (the stage entry points without chunk scratch): two passes over 64-token chunks.
__global__ void __launch_bounds__(1024) group_kernel_any(const int32_t* __restrict__ ids, int T, int k, int E,
                                                     GroupTables g, int32_t* __restrict__ slot,
                                                     int32_t* __restrict__ src, Sched sched, int with_sched,
                                                     int skip_negative, int32_t* __restrict__ pair) {
    __shared__ unsigned long long mask[kMaxExperts];
    __shared__ int run[kMaxExperts];
    __shared__ int warp_sums[32];
    const int tid = threadIdx.x;
    const int nchunks = (T + 63) / 64;

    for (int e = tid; e < E; e += blockDim.x) run[e] = 0;
    for (int pass = 0; pass < 2; pass++) {
        for (int c = 0; c < nchunks; c++) {
            const int t0 = c * 64;
            const int nt = min(64, T - t0);
            for (int e = tid; e < E; e += blockDim.x) mask[e] = 0ull;
            __syncthreads();
            for (int p = tid; p < nt * k; p += blockDim.x) {
                const int tl = p / k;
                const int e = ids[(size_t) (t0 + tl) * k + (p % k)];
                if (e >= 0 && e < E) atomicOr(&mask[e], 1ull << tl);
            }
            __syncthreads();
            if (pass == 1) {
                for (int p = tid; p < nt * k; p += blockDim.x) {
                    const int tl = p / k;
                    const size_t i = (size_t) (t0 + tl) * k + (p % k);
                    const int e = ids[i];
                    if (e < 0 || e >= E || repeats_earlier(ids, i, k, e)) {
                        slot[i] = -1;
                        if (!(skip_negative && e < 0)) atomicOr(&g_smoe_status, kDevBadId);
                        continue;
                    }
                    const int pos = run[e] + __popcll(mask[e] & ((1ull << tl) - 1ull));
                    slot[i] = pos;
                    if (src) src[pos] = t0 + tl;
                    if (pair) pair[pos] = (int) i;
                }
                __syncthreads();
            }
            for (int e = tid; e < E; e += blockDim.x) run[e] += __popcll(mask[e]);
            __syncthreads();
        }
        if (pass == 0) {
            // counts -> exclusive offsets and the active list (experts with rows, ascending id)
            int carry = 0, carry_act = 0;
            for (int e0 = 0; e0 < E; e0 += blockDim.x) {
                const int e = e0 + tid;
                const int cnt = e < E ? run[e] : 0;
                int tot, tot_act;
                const int off = block_excl_scan(cnt, warp_sums, &tot);
                const int act = block_excl_scan(cnt > 0 ? 1 : 0, warp_sums, &tot_act);
                if (e < E) {
                    g.counts[e] = cnt;
                    g.offsets[e] = carry + off;
                    run[e] = carry + off;
                    if (cnt > 0) g.active[carry_act + act] = e;
                }
                carry += tot;
                carry_act += tot_act;
            }
            if (tid == 0) {
                g.offsets[E] = carry;
                g.n_active[0] = carry_act;
                g.work[0] = g.work[1] = g.work[2] = g.work[3] = 0;
            }
            __syncthreads();
        }
    }
    if (with_sched) {
        __shared__ int whist[32][64];
        __shared__ int sorted[kMaxExperts];
        build_sched(g.counts, g.offsets, g.n_active[0], sched, E, warp_sums, whist, sorted);
    }
}

// ------------------------------------------------------------------------------------------------
// The same grouping for many tokens, over CTAs of 64-token chunks: (1) per-chunk expert counts, (2) one CTA
// turns them into per-(chunk, expert) base slots, the tables and the work list, (3) each chunk places its pairs
// at base + rank among the chunk's pairs of that expert (token order).  The slots equal group_kernel's.
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) group_count_kernel(const int32_t* __restrict__ ids, int T, int k, int E,
                                                          int32_t* __restrict__ cc) {
    __shared__ int cnt[kMaxExperts];
    const int c = blockIdx.x, t0 = c * 64, nt = min(64, T - t0);
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < nt * k; p += blockDim.x) {
        const int e = ids[(size_t) t0 * k + p];
        if (e >= 0 && e < E && !repeats_earlier(ids, (size_t) t0 * k + p, k, e)) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) cc[(size_t) c * E + e] = cnt[e];
}

__global__ void __launch_bounds__(1024) group_scan_kernel(int E, int nchunks, int32_t* __restrict__ cc,
                                                          GroupTables g, Sched sched, int with_sched) {
    __shared__ int warp_sums[32];
    const int e = threadIdx.x;
    int run = 0;
    if (e < E)
        for (int c = 0; c < nchunks; c++) {
            const int v = cc[(size_t) c * E + e];
            cc[(size_t) c * E + e] = run;
            run += v;
        }
    const int cnt = e < E ? run : 0;
    int tot, tot_act;
    const int off = block_excl_scan(cnt, warp_sums, &tot);
    const int act = block_excl_scan(cnt > 0 ? 1 : 0, warp_sums, &tot_act);
    if (e < E) {
        g.counts[e] = cnt;
        g.offsets[e] = off;
        if (cnt > 0) g.active[act] = e;
        for (int c = 0; c < nchunks; c++) cc[(size_t) c * E + e] += off;
    }
    if (e == 0) {
        g.offsets[E] = tot;
        g.n_active[0] = tot_act;
        g.work[0] = g.work[1] = g.work[2] = g.work[3] = 0;
    }
    __syncthreads();
    if (with_sched) {
        __shared__ int whist[32][64];
        __shared__ int sorted[kMaxExperts];
        __shared__ int n_act;
        if (e == 0) n_act = tot_act;
        __syncthreads();
        build_sched(g.counts, g.offsets, n_act, sched, E, warp_sums, whist, sorted);
    }
}

__global__ void __launch_bounds__(256) group_assign_kernel(const int32_t* __restrict__ ids, int T, int k, int E,
                                                           const int32_t* __restrict__ cc, int32_t* __restrict__ slot,
                                                           int32_t* __restrict__ src, int skip_negative,
                                                           int32_t* __restrict__ pair) {
    __shared__ unsigned long long mask[kMaxExperts];
    const int c = blockIdx.x, t0 = c * 64, nt = min(64, T - t0);
    for (int e = threadIdx.x; e < E; e += blockDim.x) mask[e] = 0ull;
    __syncthreads();
    for (int p = threadIdx.x; p < nt * k; p += blockDim.x) {
        const int e = ids[(size_t) t0 * k + p];
        if (e >= 0 && e < E) atomicOr(&mask[e], 1ull << (p / k));
    }
    __syncthreads();
    for (int p = threadIdx.x; p < nt * k; p += blockDim.x) {
        const int tl = p / k;
        const size_t i = (size_t) t0 * k + p;
        const int e = ids[i];
        if (e < 0 || e >= E || repeats_earlier(ids, i, k, e)) {
            slot[i] = -1;
            if (!(skip_negative && e < 0)) atomicOr(&g_smoe_status, kDevBadId);
            continue;
        }
        const int pos = cc[(size_t) c * E + e] + __popcll(mask[e] & ((1ull << tl) - 1ull));
        slot[i] = pos;
        if (src) src[pos] = t0 + tl;
        if (pair) pair[pos] = (int) i;
    }
}

size_t group_chunk_bytes(int T, int E) { return (((size_t) (T + 63) / 64) * E * 4 + 255) & ~(size_t) 255; }

cudaError_t launch_group(const int32_t* ids, int T, int k, int E, GroupTables g, int32_t* slot, int32_t* src,
                         cudaStream_t s, const Sched* sched, int32_t* chunk_counts, int skip_negative, int32_t* pair) {
    if (chunk_counts && T > kGroupWideMinTokens) {
        const int nchunks = (T + 63) / 64;
        group_count_kernel<<<nchunks, 256, 0, s>>>(ids, T, k, E, chunk_counts);
        group_scan_kernel<<<1, 1024, 0, s>>>(E, nchunks, chunk_counts, g, sched ? *sched : Sched{}, sched ? 1 : 0);
        group_assign_kernel<<<nchunks, 256, 0, s>>>(ids, T, k, E, chunk_counts, slot, src, skip_negative, pair);
        return cudaGetLastError();
    }
    if (T <= kGroupWideMinTokens)
        group_kernel<<<1, 1024, 0, s>>>(ids, T, k, E, g, slot, src, sched ? *sched : Sched{}, sched ? 1 : 0,
                                        skip_negative, pair);
    else
        group_kernel_any<<<1, 1024, 0, s>>>(ids, T, k, E, g, slot, src, sched ? *sched : Sched{}, sched ? 1 : 0,
                                            skip_negative, pair);
    return cudaGetLastError();
}

}  // namespace smoe
