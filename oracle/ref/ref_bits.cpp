// The reference's own bf16 / fp16 converters, compiled from its headers (TEST INFRASTRUCTURE ONLY):
// include/strata/kernels/bf16_bits.hpp and f16_bits.hpp are header-only and used here unmodified.
#include "strata/kernels/bf16_bits.hpp"
#include "strata/kernels/f16_bits.hpp"

extern "C" {
uint16_t ref_bf16_from_f32(float f) { return strata::kernels::bf16_from_f32(f); }
uint16_t ref_f16_from_f32(float f) { return strata::kernels::f16_from_f32(f); }
float ref_f32_from_f16(uint16_t h) { return strata::kernels::f32_from_f16(h); }
}
