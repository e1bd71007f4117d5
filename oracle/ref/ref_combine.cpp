// Builds the reference's own combine reference (TEST INFRASTRUCTURE ONLY).
//
// metal/src/moe_combine_parity.cpp is compiled here unmodified; main() is renamed so `reference()`
// (:55-71: double sum of w * part in router order, shared added plain) is callable, with its trap flags.
#define main strata_moe_combine_parity_main
#include "metal/src/moe_combine_parity.cpp"
#undef main

extern "C" void ref_combine(const float* parts, const float* w, const float* shared, float* y, int n_embd, int k,
                            int weight_routed, int weight_shared) {
    std::vector<float> p(parts, parts + (size_t) k * n_embd), ww(w, w + k), s;
    if (shared) s.assign(shared, shared + n_embd);
    std::vector<float> out = reference(p, ww, shared ? &s : nullptr, n_embd, k, weight_routed != 0, weight_shared != 0);
    std::memcpy(y, out.data(), out.size() * sizeof(float));
}
