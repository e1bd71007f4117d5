// Link stand-ins for the Metal side of the reference's parity sources (TEST INFRASTRUCTURE ONLY).
//
// The parity .cpp files compiled beside this name Metal launchers and the shared-buffer class in code
// paths this build never runs (their renamed main()).  Every launcher here throws.  The block geometry
// helpers are real, because the host reference ref_expert() sizes its rows with them; their values are
// the GGUF block sizes of metal/src/iq.mm:99-131 for the six formats this build takes (Q2_0 64 values /
// 18 bytes, IQ2_S 256 / 82, IQ4_NL 32 / 18, IQ4_XS 256 / 136, IQ3_XXS 256 / 98, IQ3_S 256 / 110) and the q8_1
// block (32 values / 36 bytes).
#include "strata/metal/bytes.hpp"
#include "strata/metal/device.hpp"
#include "strata/metal/iq.hpp"
#include "strata/metal/moe_combine.hpp"
#include "strata/metal/router.hpp"

#include <cstdlib>

namespace strata::metal {

struct Bytes::Impl {
    void* p;
    uint64_t n;
};
Bytes::Bytes(uint64_t bytes) : impl_(new Impl{std::calloc(bytes ? bytes : 1, 1), bytes}) {}
Bytes::Bytes(Bytes&& o) noexcept : impl_(o.impl_) { o.impl_ = nullptr; }
Bytes& Bytes::operator=(Bytes&& o) noexcept {
    std::swap(impl_, o.impl_);
    return *this;
}
Bytes::~Bytes() {
    if (impl_) std::free(impl_->p);
    delete impl_;
}
void* Bytes::data() const { return impl_->p; }
uint64_t Bytes::size() const { return impl_->n; }
void* Bytes::handle() const { return nullptr; }

[[noreturn]] static void no_device() { throw MetalError("no Metal device in this build"); }

bool iq_type_supported(int t) noexcept {
    return t == kQ2_0 || t == kIq2S || t == kIq4Nl || t == kIq4Xs || t == kIq3Xxs || t == kIq3S;
}
int iq_block_values(int t) {
    return t == kQ2_0 ? 64 : t == kIq4Nl ? 32 : (t == kIq2S || t == kIq4Xs || t == kIq3Xxs || t == kIq3S) ? 256 : 0;
}
size_t iq_block_bytes(int t) {
    return t == kQ2_0 ? 18 : t == kIq2S ? 82 : t == kIq4Nl ? 18 : t == kIq4Xs ? 136 : t == kIq3Xxs ? 98 : t == kIq3S ? 110 : 0;
}
size_t iq_row_bytes(int t, int64_t n) {
    const int v = iq_block_values(t);
    if (v == 0 || n <= 0 || n % v) throw MetalError("iq_row_bytes: bad type or length");
    return (size_t) (n / v) * iq_block_bytes(t);
}
size_t iq_q8_1_bytes(int64_t n) {
    if (n <= 0 || n % 32) throw MetalError("iq_q8_1_bytes: bad length");
    return (size_t) (n / 32) * 36;
}
size_t iq_expert_bytes(const IqExpert&) { no_device(); }
void iq_quantize_q8_1(const Bytes&, int64_t, Bytes&) { no_device(); }
void iq_mmvq(int, const Bytes&, int64_t, const Bytes&, int64_t, int64_t, int64_t, Bytes&) { no_device(); }
void iq_swiglu_q8(const Bytes&, const Bytes&, int64_t, Bytes&) { no_device(); }
void iq_expert(const Bytes&, const Bytes&, const IqExpert&, int64_t, Bytes&) { no_device(); }
void router_top10(const Bytes&, int, int, int, Bytes&, Bytes&) { no_device(); }
void moe_combine(const Bytes&, const Bytes&, const Bytes*, Bytes&, int, int) { no_device(); }

}  // namespace strata::metal
