// gguf.cu - the C ABI of the model boundary (include/smoe_gguf.hpp): a GGUF file and one MoE layer uploaded from it
// by tensor name, as opaque handles.  No C++ exception crosses the ABI.
#include "../../include/smoe.h"
#include "../../include/smoe_gguf.hpp"

extern "C" {

smoe_status smoe_gguf_open(const char* path, void** handle) {
    if (!path || !handle) return smoe::fail(SMOE_INVALID_ARG, "gguf_open: null argument");
    return guarded("gguf_open", [&] {
        auto* g = new smoe::Gguf();
        try {
            g->open(path);
        } catch (...) {
            delete g;
            throw;
        }
        *handle = g;
    });
}

void smoe_gguf_close(void* handle) { delete static_cast<smoe::Gguf*>(handle); }

smoe_status smoe_gguf_tensor(const void* handle, const char* name, int* type, int64_t* ne4, uint64_t* bytes,
                             const uint8_t** data) {
    if (!handle || !name) return smoe::fail(SMOE_INVALID_ARG, "gguf_tensor: null argument");
    return guarded("gguf_tensor", [&] {
        const smoe::Gguf::Tensor& t = static_cast<const smoe::Gguf*>(handle)->at(name);
        if (type) *type = (int) t.type;
        if (ne4)
            for (int d = 0; d < 4; d++) ne4[d] = t.ne[d];
        if (bytes) *bytes = t.bytes;
        if (data) *data = t.data;
    });
}

smoe_status smoe_gguf_load_layer(const void* handle, int layer, int with_shared, int k, smoe_layer* out,
                                 void** owner) {
    if (!handle || !out || !owner) return smoe::fail(SMOE_INVALID_ARG, "gguf_load_layer: null argument");
    return guarded("gguf_load_layer", [&] {
        std::unique_ptr<smoe::GgufLayer> g =
            smoe::GgufLayer::load(*static_cast<const smoe::Gguf*>(handle), layer, with_shared != 0, k);
        *out = g->desc();
        *owner = g.release();
    });
}

void smoe_gguf_free_layer(void* owner) { delete static_cast<smoe::GgufLayer*>(owner); }

}  // extern "C"
