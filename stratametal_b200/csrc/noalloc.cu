// noalloc.cu - smoe_moe_group_noalloc: the token -> expert grouping with its scratch in a static device array.
//
// Why it exists.  smoe_moe_group takes its grouping tables (counts, offsets, the active-expert list, work
// counters) from a scratch buffer the caller allocates.  Some callers cannot allocate device memory at the
// point where they group tokens: code recorded into a CUDA graph (cudaMalloc is not an operation a stream
// capture can record), engines whose memory planner hands out every device byte at start-up and forbids
// allocation on the token path, and plug-ins running inside a host process that owns the device allocator.
// This entry point needs no scratch from them: the tables live in g_noalloc_tables below, a fixed 12,544-byte
// array that every GPU which loads this library holds until the process exits.
//
// Limits and sharing.  At most kNoAllocMaxExperts (1024) experts; larger requests are refused.  Every call on a
// device uses the same array and leaves the last call's tables in it.  The kernel writes every table entry it
// later reads and zeroes its own work counters, so nothing has to be cleared between calls.  Two calls whose
// kernels overlap on the GPU (different streams with no ordering between them) race on the array: order them.
//
// Set-up.  Host code cannot use the array's name as a device address, so the first call on each device looks
// the address up with cudaGetSymbolAddress while that device is current, and keeps it.  Make that first call
// before any stream capture begins.  The call allocates nothing: no cudaMalloc, no cudaFree, no allocating
// library routine.
#include "../../include/smoe.h"
#include "common.cuh"
#include "kernels.cuh"

#include <mutex>

namespace smoe {

constexpr int kNoAllocMaxExperts = 1024;
constexpr int kNoAllocTableInts = 3136;  // group_tables_bytes(1024) / 4
static_assert(kNoAllocTableInts * 4 >= (3 * kNoAllocMaxExperts + 6) * 4, "table too small");

static __device__ __align__(256) int32_t g_noalloc_tables[kNoAllocTableInts];

namespace {
constexpr int kMaxDevices = 64;
int32_t* g_noalloc_dev_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;
}  // namespace

}  // namespace smoe

extern "C" smoe_status smoe_moe_group_noalloc(const int32_t* ids, int n_tok, int k, int n_expert, int32_t* slot,
                                              int32_t* src, void* stream) {
    using namespace smoe;
    if (n_tok < 0 || k < 0 || n_expert < 0) return fail(SMOE_INVALID_ARG, "moe_group_noalloc: negative size");
    if (n_tok == 0 || k == 0 || n_expert == 0) return ok();
    if (k > kMaxK) return fail(SMOE_INVALID_ARG, "moe_group_noalloc: k exceeds 64");
    if (n_expert > kNoAllocMaxExperts)
        return fail(SMOE_INVALID_ARG, "moe_group_noalloc: n_expert exceeds the static table's 1024 experts");
    if (!stream) return fail(SMOE_INVALID_ARG, "moe_group_noalloc: a non-null stream is required");
    if (!ids || !slot) return fail(SMOE_INVALID_ARG, "moe_group_noalloc: null buffer");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "moe_group_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(SMOE_UNSUPPORTED, "moe_group_noalloc: device ordinal above 63");
    int32_t* tables = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_dev_ptr[dev]) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_noalloc_tables);
            if (e != cudaSuccess) return cuda_fail(e, "moe_group_noalloc: cudaGetSymbolAddress");
            g_noalloc_dev_ptr[dev] = static_cast<int32_t*>(p);
        }
        tables = g_noalloc_dev_ptr[dev];
    }
    e = launch_group(ids, n_tok, k, n_expert, group_tables_at(tables, n_expert), slot, src, (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "moe_group_noalloc");
}
