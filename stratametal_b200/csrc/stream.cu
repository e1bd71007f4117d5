// stream.cu - the C ABI of the expert-streaming tier (include/smoe_stream.hpp): the pack's expert file and the
// VRAM slot cache as opaque handles.  No C++ exception crosses the ABI: each is turned into its status and message.
#include "../../include/smoe.h"
#include "../../include/smoe_stream.hpp"

#include <new>

namespace {
template <typename F>
smoe_status guarded(const char* who, F&& f) {
    try {
        f();
        return smoe::ok();
    } catch (const smoe::Error& e) {
        return smoe::fail(e.status, e.what());
    } catch (const std::bad_alloc&) {
        return smoe::fail(SMOE_CUDA_ERROR, std::string(who) + ": out of host memory");
    } catch (const std::exception& e) {
        return smoe::fail(SMOE_INVALID_ARG, std::string(who) + ": " + e.what());
    }
}
}  // namespace

extern "C" {

smoe_status smoe_native_experts_open(const char* pack_dir, void** handle) {
    if (!pack_dir || !handle) return smoe::fail(SMOE_INVALID_ARG, "native_experts_open: null argument");
    return guarded("native_experts_open", [&] {
        auto* n = new smoe::NativeExperts();
        try {
            n->open(pack_dir);
        } catch (...) {
            delete n;
            throw;
        }
        *handle = n;
    });
}

void smoe_native_experts_close(void* handle) { delete static_cast<smoe::NativeExperts*>(handle); }

smoe_status smoe_native_experts_pick(const void* handle, int64_t layer, int64_t expert, int* gu_type, int* d_type,
                                     uint64_t* file_off, uint64_t* blob_bytes, const uint8_t** host_blob) {
    if (!handle) return smoe::fail(SMOE_INVALID_ARG, "native_experts_pick: null handle");
    return guarded("native_experts_pick", [&] {
        const auto* n = static_cast<const smoe::NativeExperts*>(handle);
        const smoe::NativeExperts::Pick p = n->pick(layer, expert);
        if (gu_type) *gu_type = p.gu_type;
        if (d_type) *d_type = p.d_type;
        if (file_off) *file_off = p.file_off;
        if (blob_bytes) *blob_bytes = p.blob_bytes;
        if (host_blob) *host_blob = n->blob(p);
    });
}

smoe_status smoe_expert_cache_open(int64_t n_slots, int64_t n_layers, int64_t n_expert, int64_t blob_bytes,
                                   int per_layer, void** handle) {
    if (!handle) return smoe::fail(SMOE_INVALID_ARG, "expert_cache_open: null handle");
    return guarded("expert_cache_open", [&] {
        auto* c = new smoe::ExpertCache();
        try {
            c->residency().set_per_layer_admission(per_layer != 0);
            c->open(n_slots, n_layers, n_expert, blob_bytes);
            c->residency().set_per_layer_admission(per_layer != 0);
        } catch (...) {
            delete c;
            throw;
        }
        *handle = c;
    });
}

void smoe_expert_cache_close(void* handle) { delete static_cast<smoe::ExpertCache*>(handle); }

smoe_status smoe_expert_cache_ensure(void* handle, int64_t layer, int64_t expert, const uint8_t* host_blob,
                                     int64_t bytes, void* stream, int32_t* slot) {
    if (!handle || !host_blob || !slot) return smoe::fail(SMOE_INVALID_ARG, "expert_cache_ensure: null argument");
    return guarded("expert_cache_ensure", [&] {
        *slot = static_cast<smoe::ExpertCache*>(handle)->ensure(layer, expert, host_blob, bytes, (cudaStream_t) stream);
    });
}

int32_t smoe_expert_cache_slot_of(const void* handle, int64_t layer, int64_t expert) {
    return handle ? static_cast<const smoe::ExpertCache*>(handle)->residency_const().slot_of(layer, expert) : -1;
}

uint8_t* smoe_expert_cache_arena(const void* handle) {
    return handle ? static_cast<const smoe::ExpertCache*>(handle)->arena() : nullptr;
}

const int32_t* smoe_expert_cache_row(const void* handle, int64_t layer) {
    if (!handle) return nullptr;
    const auto* c = static_cast<const smoe::ExpertCache*>(handle);
    if (layer < 0 || layer >= c->residency_const().n_layers()) return nullptr;
    return c->device_row(layer);
}

}  // extern "C"
