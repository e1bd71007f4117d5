// Builds the reference's own router reference (TEST INFRASTRUCTURE ONLY).
//
// metal/src/router_parity.cpp is compiled here unmodified; main() is renamed so the host reference
// `reference()` (:48-72: softmax in double, stable descending sort, renorm clamped at 2^-14) is callable.
#define main strata_router_parity_main
#include "metal/src/router_parity.cpp"
#undef main

extern "C" void ref_route(const float* logits, int n_expert, int k, int* ids, float* w) {
    std::vector<float> raw((size_t) k);
    reference(logits, n_expert, k, ids, w, raw.data());
}
