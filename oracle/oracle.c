/* oracle.c - CPU restatement of StrataMetal's host MoE-block reference.  TEST INFRASTRUCTURE ONLY:
 * the checker for the B200 kernels, never linked into or called by the product library.
 *
 * Every function below restates one host function of the reference's parity tests, named in its
 * comment with file:line inside the StrataMetal tree.  Arithmetic, rounding and summation order follow
 * those functions exactly; compile with -ffp-contract=off so no multiply-add is fused. */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

static const uint64_t k_iq2s_grid[1024] = {
#include "../stratametal_b200/csrc/iq2s_grid.inc"
};
static const uint32_t k_iq3xxs_grid[256] = {
#include "../stratametal_b200/csrc/iq3xxs_grid.inc"
};
static const uint32_t k_iq3s_grid[512] = {
#include "../stratametal_b200/csrc/iq3s_grid.inc"
};

/* ------------------------------------------------------------------------------------------------ */
/* bit conversions                                                                                  */
/* ------------------------------------------------------------------------------------------------ */

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* RNE f32 -> bf16 with NaN quieted (bf16_bits.hpp:37-47): the carry bit is bit 16, the lowest kept bit. */
uint16_t orc_bf16_from_f32(float f) {
    uint32_t i = f2u(f);
    if ((i & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t) ((i >> 16) | 64u);
    i = (i + ((i >> 16) & 1u) + 0x7FFFu) & 0xFFFF0000u;
    return (uint16_t) (i >> 16);
}

float orc_f32_from_bf16(uint16_t h) { return u2f((uint32_t) h << 16); }

/* RNE f32 -> fp16 with subnormals, finite overflow to inf, NaN kept (f16_bits.hpp:37-73). */
uint16_t orc_f16_from_f32(float f) {
    const uint32_t x = f2u(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t rawexp = (x >> 23) & 0xFFu;
    const int exp = (int) rawexp - 127 + 15;
    uint32_t man = x & 0x7FFFFFu;
    if (rawexp == 0xFFu) return (uint16_t) (sign | 0x7C00u | (man ? 0x200u : 0u));
    if (exp >= 31) return (uint16_t) (sign | 0x7C00u);
    if (exp <= 0) {
        if (exp < -10) return (uint16_t) sign;
        man |= 0x800000u;
        const uint32_t sh = (uint32_t) (14 - exp);
        uint32_t h = (man >> sh) & 0x3FFu;
        const uint32_t rem = man & ((1u << sh) - 1u);
        const uint32_t half = 1u << (sh - 1);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return (uint16_t) (sign | h);
    }
    uint32_t h = sign | ((uint32_t) exp << 10) | (man >> 13);
    const uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t) h;
}

/* Exact fp16 -> f32 including subnormals (f16_bits.hpp:77-104). */
float orc_f32_from_f16(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t out;
    if (ex == 0) {
        if (man == 0) {
            out = sign;
        } else {
            uint32_t m = man;
            int s = 0;
            while ((m & 0x400u) == 0) { m <<= 1; ++s; }
            out = sign | ((uint32_t) (113 - s) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (ex == 31) {
        out = sign | 0x7F800000u | (man << 13);
    } else {
        out = sign | ((ex - 15 + 127) << 23) | (man << 13);
    }
    return u2f(out);
}

/* Block geometry (metal/src/iq.mm:99-131; gguf_reader.hpp:197-199). */
size_t orc_row_bytes(int type, int64_t n) {
    if (n <= 0) return 0;
    if (type == ORC_Q2_0) return (n % 64) ? 0 : (size_t) (n / 64) * 18u;
    if (type == ORC_IQ2_S) return (n % 256) ? 0 : (size_t) (n / 256) * 82u;
    if (type == ORC_IQ4_NL) return (n % 32) ? 0 : (size_t) (n / 32) * 18u;
    if (type == ORC_IQ4_XS) return (n % 256) ? 0 : (size_t) (n / 256) * 136u;
    if (type == ORC_IQ3_XXS) return (n % 256) ? 0 : (size_t) (n / 256) * 98u;
    if (type == ORC_IQ3_S) return (n % 256) ? 0 : (size_t) (n / 256) * 110u;
    return 0;
}

size_t orc_q8_1_bytes(int64_t n) { return (n <= 0 || n % 32) ? 0 : (size_t) (n / 32) * 36u; }

static uint16_t rd16(const uint8_t* p) { return (uint16_t) (p[0] | (p[1] << 8)); }
static void wr16(uint8_t* p, uint16_t h) { p[0] = (uint8_t) h; p[1] = (uint8_t) (h >> 8); }

/* ------------------------------------------------------------------------------------------------ */
/* q8_1 (iq_parity.cpp:350-382)                                                                     */
/* ------------------------------------------------------------------------------------------------ */

/* amax and the float sum come from a 32-lane xor butterfly (offsets 16..1); d = amax / 127 clamped to
 * +-65504; q = round-half-away(x / d) clamped to +-127 (0 when amax == 0); stored as fp16 d, fp16 sum,
 * 32 int8. */
void orc_quant_q8_1_block(const float* x, uint8_t* y) {
    float a[32], s[32], na[32], ns[32];
    for (int i = 0; i < 32; i++) { a[i] = fabsf(x[i]); s[i] = x[i]; }
    for (int o = 16; o > 0; o >>= 1) {
        for (int i = 0; i < 32; i++) {
            na[i] = a[i] > a[i ^ o] ? a[i] : a[i ^ o];
            ns[i] = s[i] + s[i ^ o];
        }
        memcpy(a, na, sizeof a);
        memcpy(s, ns, sizeof s);
    }
    const float amax = a[0];
    const float sum = s[0];
    float d = amax / 127.f;
    if (fabsf(d) > 65504.f) d = copysignf(65504.f, d);
    for (int i = 0; i < 32; i++) {
        int q = 0;
        if (amax != 0.f) {
            float r = roundf(x[i] / d);
            if (r > 127.f) r = 127.f;
            if (r < -127.f) r = -127.f;
            q = (int) r;
        }
        y[4 + i] = (uint8_t) (int8_t) q;
    }
    const float sc = fabsf(sum) > 65504.f ? copysignf(65504.f, sum) : sum;
    wr16(y, orc_f16_from_f32(d));
    wr16(y + 2, orc_f16_from_f32(sc));
}

void orc_quant_q8_1(const float* x, int64_t n, uint8_t* y) {
    for (int64_t b = 0; b < n / 32; b++) orc_quant_q8_1_block(x + b * 32, y + b * 36);
}

/* ------------------------------------------------------------------------------------------------ */
/* integer partial dots                                                                             */
/* ------------------------------------------------------------------------------------------------ */

static int8_t q8_at(const uint8_t* xblk, int i) { return (int8_t) xblk[4 + i]; }

/* Q2_0 half-block `half` (32 values) of block `blk` against q8_1 block `xblk`:
 * sumi = sum (code - 1) * q, partial = (f32(d_w) * f32(d_x)) * (float) sumi
 * (iq_parity.cpp:225-252 with minus_one; codes 4 per byte, LSB first, dequant.hpp:69-78). */
static float q2_0_partial(const uint8_t* blk, const uint8_t* xblk, int half, int minus_one) {
    const uint8_t* qs = blk + 2 + 8 * half;
    int32_t sumi = 0;
    for (int i = 0; i < 32; i++) {
        const int code = (qs[i / 4] >> (2 * (i % 4))) & 3;
        sumi += (code - (minus_one ? 1 : 0)) * (int32_t) q8_at(xblk, i);
    }
    const float d = orc_f32_from_f16(rd16(blk)) * orc_f32_from_f16(rd16(xblk));
    return d * (float) sumi;
}

/* IQ2_S 32-value group `g` of a 256-value block (iq_parity.cpp:125-151, format iq.metal:152-180):
 * for each 8-value chunk j: 10-bit index = qs[4g+j] | ((qh[g] >> 2j) & 3) << 8 into the codebook, value m
 * negated when bit m of sign byte signs[4g+j] is set; sum0 over chunks 0-1, sum1 over chunks 2-3;
 * sumi = (sum0*ls0 + sum1*ls1 + (sum0+sum1)/2) / 4 with C truncating division. */
static float iq2_s_partial(const uint8_t* blk, const uint8_t* xblk, int g) {
    const uint8_t* qs = blk + 2;
    const uint8_t* sg = blk + 34;
    const int qh = blk[66 + g];
    const int sc = blk[74 + g];
    const int ls0 = sc & 0x0F, ls1 = sc >> 4;
    int32_t sum0 = 0, sum1 = 0;
    for (int j = 0; j < 4; j++) {
        const uint32_t idx = (uint32_t) qs[4 * g + j] | ((uint32_t) ((qh >> (2 * j)) & 3) << 8);
        const uint64_t e = k_iq2s_grid[idx];
        const uint32_t sb = sg[4 * g + j];
        int32_t part = 0;
        for (int m = 0; m < 8; m++) {
            int v = (int) ((e >> (8 * m)) & 0xFFu);
            if ((sb >> m) & 1u) v = -v;
            part += v * (int32_t) q8_at(xblk, 8 * j + m);
        }
        if (j < 2) sum0 += part;
        else sum1 += part;
    }
    const int32_t sumi = (sum0 * ls0 + sum1 * ls1 + (sum0 + sum1) / 2) / 4;
    const float d = orc_f32_from_f16(rd16(blk)) * orc_f32_from_f16(rd16(xblk));
    return d * (float) sumi;
}

/* The IQ4 code values (iq_parity.cpp:106): the format's fixed non-linear table, index = one 4-bit code. */
static const int8_t k_iq4_values[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

/* IQ4_NL (fp16 d, qs[16]: byte i holds value i in its low nibble and value i + 16 in its high nibble) has two
 * 16-value partials per 32-value block (iq_parity.cpp:196-206): partial p reads qs bytes 8p .. 8p + 7, i.e. values
 * 8p .. 8p + 7 and 16 + 8p .. 16 + 8p + 7 of the block's q8_1 block; partial = (f32(d_w) * f32(d_x)) * sumi. */
static float iq4_nl_partial(const uint8_t* blk, const uint8_t* xblk, int p) {
    const uint8_t* qs = blk + 2;
    int32_t sumi = 0;
    for (int i = 8 * p; i < 8 * p + 8; i++) {
        sumi += k_iq4_values[qs[i] & 15] * (int32_t) q8_at(xblk, i);
        sumi += k_iq4_values[qs[i] >> 4] * (int32_t) q8_at(xblk, i + 16);
    }
    const float d = orc_f32_from_f16(rd16(blk)) * orc_f32_from_f16(rd16(xblk));
    return d * (float) sumi;
}

/* IQ4_XS (fp16 d @0, 2-bit high scales u16 @2, 4-bit low scales [4] @4, qs[128] @8; 256 values) 32-value group
 * ib (iq_parity.cpp:208-222): qs bytes 16 ib .. 16 ib + 15 as in IQ4_NL (low nibble value i, high nibble value
 * i + 16), the 6-bit scale ls = low nibble ib of scales_l | bits 2 ib, 2 ib + 1 of scales_h << 4, and
 * sumi * (ls - 32). */
static float iq4_xs_partial(const uint8_t* blk, const uint8_t* xblk, int ib) {
    const uint8_t* qs = blk + 8 + 16 * ib;
    int32_t sumi = 0;
    for (int i = 0; i < 16; i++) {
        sumi += k_iq4_values[qs[i] & 15] * (int32_t) q8_at(xblk, i);
        sumi += k_iq4_values[qs[i] >> 4] * (int32_t) q8_at(xblk, i + 16);
    }
    const int sh = rd16(blk + 2);
    const int ls = ((blk[4 + ib / 2] >> (4 * (ib % 2))) & 15) | (((sh >> (2 * ib)) & 3) << 4);
    sumi *= ls - 32;
    const float d = orc_f32_from_f16(rd16(blk)) * orc_f32_from_f16(rd16(xblk));
    return d * (float) sumi;
}

/* Sum over one 4-value codebook entry: magnitudes (bytes of `e`) times q, value j negated when bit j of `neg`
 * is set. */
static int32_t grid4(uint32_t e, unsigned neg, const uint8_t* xblk, int v0) {
    int32_t s = 0;
    for (int j = 0; j < 4; j++) {
        int v = (int) ((e >> (8 * j)) & 0xFFu);
        if ((neg >> j) & 1u) v = -v;
        s += v * (int32_t) q8_at(xblk, v0 + j);
    }
    return s;
}

/* IQ3_XXS (fp16 d, qs[64] grid indices, 8 words of signs and scale @66; 256 values) 32-value group g
 * (iq_parity.cpp:153-173): word w = bytes 66 + 4g; chunk c (8 values) uses grid entries qs[8g + 2c] (values
 * 8c..8c+3) and qs[8g + 2c + 1] (8c+4..8c+7) with the 7 sign bits (w >> 7c) & 127 completed by their parity as
 * bit 7; sumi = (ls * sumi + sumi / 2) / 2 (C truncating division), ls = w >> 28. */
static float iq3_xxs_partial(const uint8_t* blk, const uint8_t* xblk, int g) {
    const uint8_t* qs = blk + 2;
    const uint32_t w = (uint32_t) qs[64 + 4 * g] | ((uint32_t) qs[65 + 4 * g] << 8) | ((uint32_t) qs[66 + 4 * g] << 16) |
                       ((uint32_t) qs[67 + 4 * g] << 24);
    int32_t sumi = 0;
    for (int c = 0; c < 4; c++) {
        unsigned s7 = (w >> (7 * c)) & 127u, par = 0;
        for (int b = 0; b < 7; b++) par ^= (s7 >> b) & 1u;
        const unsigned sg = s7 | (par << 7);
        sumi += grid4(k_iq3xxs_grid[qs[8 * g + 2 * c]], sg & 15u, xblk, 8 * c);
        sumi += grid4(k_iq3xxs_grid[qs[8 * g + 2 * c + 1]], sg >> 4, xblk, 8 * c + 4);
    }
    const int32_t ls = (int32_t) (w >> 28);
    sumi = (ls * sumi + sumi / 2) / 2;
    const float d = orc_f32_from_f16(rd16(blk)) * orc_f32_from_f16(rd16(xblk));
    return d * (float) sumi;
}

/* IQ3_S (fp16 d, qs[64], qh[8] @66, signs[32] @74, scales[4] @106; 256 values) 32-value group g
 * (iq_parity.cpp:175-194): chunk c takes 9-bit indices qs[8g + 2c] | bit 2c of qh[g] << 8 and qs[8g + 2c + 1] |
 * bit 2c + 1 << 8, sign byte signs[4g + c] (bits 0-3 the first entry's values, 4-7 the second's); sumi * (1 + 2
 * nib), nib = nibble g & 1 of scales[g / 2]. */
static float iq3_s_partial(const uint8_t* blk, const uint8_t* xblk, int g) {
    const uint8_t* qs = blk + 2;
    const unsigned qh = blk[66 + g];
    int32_t sumi = 0;
    for (int c = 0; c < 4; c++) {
        const unsigned i0 = qs[8 * g + 2 * c] | (((qh >> (2 * c)) & 1u) << 8);
        const unsigned i1 = qs[8 * g + 2 * c + 1] | (((qh >> (2 * c + 1)) & 1u) << 8);
        const unsigned sb = blk[74 + 4 * g + c];
        sumi += grid4(k_iq3s_grid[i0], sb & 15u, xblk, 8 * c);
        sumi += grid4(k_iq3s_grid[i1], sb >> 4, xblk, 8 * c + 4);
    }
    const int nib = (blk[106 + g / 2] >> (4 * (g & 1))) & 15;
    sumi *= 1 + 2 * nib;
    const float d = orc_f32_from_f16(rd16(blk)) * orc_f32_from_f16(rd16(xblk));
    return d * (float) sumi;
}

/* row_dot (iq_parity.cpp:275-292): the row's partials in order (32 values each, IQ4_NL 16), partial k added to
 * lane k & 31, then the 32 lane sums meet in an xor butterfly (16, 8, 4, 2, 1). */
static float row_dot_impl(int type, const uint8_t* row, const uint8_t* col, int n_in, int variant) {
    float lane[32], nxt[32];
    memset(lane, 0, sizeof lane);
    const int npart = type == ORC_IQ4_NL ? n_in / 16 : n_in / 32;
    for (int k = 0; k < npart; k++) {
        float p;
        if (type == ORC_IQ2_S) p = iq2_s_partial(row + (size_t) (k / 8) * 82, col + (size_t) k * 36, k % 8);
        else if (type == ORC_IQ4_NL) p = iq4_nl_partial(row + (size_t) (k / 2) * 18, col + (size_t) (k / 2) * 36, k % 2);
        else if (type == ORC_IQ4_XS) p = iq4_xs_partial(row + (size_t) (k / 8) * 136, col + (size_t) k * 36, k % 8);
        else if (type == ORC_IQ3_XXS) p = iq3_xxs_partial(row + (size_t) (k / 8) * 98, col + (size_t) k * 36, k % 8);
        else if (type == ORC_IQ3_S) p = iq3_s_partial(row + (size_t) (k / 8) * 110, col + (size_t) k * 36, k % 8);
        else p = q2_0_partial(row + (size_t) (k / 2) * 18, col + (size_t) k * 36, k % 2, variant != 1);
        lane[k & 31] += p;
    }
    for (int o = 16; o > 0; o >>= 1) {
        for (int i = 0; i < 32; i++) nxt[i] = lane[i] + lane[i ^ o];
        memcpy(lane, nxt, sizeof lane);
    }
    return lane[0];
}

float orc_row_dot(int type, const uint8_t* row, const uint8_t* col, int n_in) {
    return row_dot_impl(type, row, col, n_in, 0);
}

float orc_row_dot_variant(int type, const uint8_t* row, const uint8_t* col, int n_in, int variant) {
    return row_dot_impl(type, row, col, n_in, variant);
}

void orc_mmvq(int type, const uint8_t* w, const uint8_t* x, int n_in, int n_out, int n_col, float* y) {
    const size_t rb = orc_row_bytes(type, n_in);
    const size_t xb = orc_q8_1_bytes(n_in);
    for (int c = 0; c < n_col; c++)
        for (int r = 0; r < n_out; r++)
            y[(size_t) c * n_out + r] = orc_row_dot(type, w + (size_t) r * rb, x + (size_t) c * xb, n_in);
}

/* silu(g) * u in float with the libm exp, then the q8_1 block rule (iq_parity.cpp:384, iq.metal:630-663). */
static float silu_mul(float g, float u) { return (g / (1.f + expf(-g))) * u; }

void orc_swiglu_q8(const float* gate, const float* up, int64_t n, uint8_t* y) {
    float h[32];
    for (int64_t b = 0; b < n / 32; b++) {
        for (int i = 0; i < 32; i++) h[i] = silu_mul(gate[b * 32 + i], up[b * 32 + i]);
        orc_quant_q8_1_block(h, y + b * 36);
    }
}

/* bf16_dot (pack_parity.cpp:3795-3799): products of the rounded activation and the bf16 row summed in
 * double in index order, then rounded to float. */
float orc_bf16_dot(const float* x, const uint16_t* row, int n) {
    double acc = 0;
    for (int i = 0; i < n; i++) acc += (double) x[i] * (double) orc_f32_from_bf16(row[i]);
    return (float) acc;
}

/* route_ref (pack_parity.cpp:5144-5165): softmax in double over all experts, a stable descending sort
 * (equal probabilities keep the lower index), w_i = (float) p, then (float)((double) w_i / max(sum, 2^-14))
 * where sum is the double sum of the chosen p in rank order. */
void orc_route(const float* logits, int n_expert, int k, int32_t* ids, float* w) {
    double mx = (double) logits[0];
    for (int e = 1; e < n_expert; e++) if ((double) logits[e] > mx) mx = (double) logits[e];
    double* p = (double*) malloc(sizeof(double) * (size_t) n_expert);
    unsigned char* taken = (unsigned char*) calloc((size_t) n_expert, 1);
    double sum = 0;
    for (int e = 0; e < n_expert; e++) { p[e] = exp((double) logits[e] - mx); sum += p[e]; }
    for (int e = 0; e < n_expert; e++) p[e] /= sum;
    /* selection of the k largest in stable order == the first k of a stable descending sort */
    double chosen = 0;
    for (int i = 0; i < k; i++) {
        int best = -1;
        for (int e = 0; e < n_expert; e++) {
            if (taken[e]) continue;
            if (best < 0 || p[e] > p[best]) best = e;
        }
        taken[best] = 1;
        ids[i] = best;
        w[i] = (float) p[best];
        chosen += p[best];
    }
    if (chosen < 6.103515625e-05) chosen = 6.103515625e-05;
    for (int i = 0; i < k; i++) w[i] = (float) ((double) w[i] / chosen);
    free(p);
    free(taken);
}

/* combine (pack_parity.cpp:8607-8616): double sum of w_e * part_e in router order, the shared output added
 * plain (not router weighted) in double, rounded once to float.  shared may be NULL. */
void orc_combine(const float* parts, const float* w, const float* shared, float* y, int n_embd, int k) {
    for (int d = 0; d < n_embd; d++) {
        double acc = 0;
        for (int e = 0; e < k; e++) acc += (double) w[e] * (double) parts[(size_t) e * n_embd + d];
        if (shared) acc += (double) shared[d];
        y[d] = (float) acc;
    }
}

/* Exact dequantization (dequant.hpp:69-78 for Q2_0; IQ2_S as its dot implies: d * (0.5 + ls) * 0.25 times
 * the signed codebook value, ls the 4-bit scale of the 16-value half). */
void orc_dequant_row(int type, const uint8_t* row, int n, float* out) {
    if (type == ORC_Q2_0) {
        for (int b = 0; b < n / 64; b++) {
            const uint8_t* blk = row + (size_t) b * 18;
            const float d = orc_f32_from_f16(rd16(blk));
            for (int j = 0; j < 64; j++) {
                const int code = (blk[2 + j / 4] >> (2 * (j % 4))) & 3;
                out[b * 64 + j] = (float) (code - 1) * d;
            }
        }
        return;
    }
    for (int b = 0; b < n / 256; b++) {
        const uint8_t* blk = row + (size_t) b * 82;
        const double d = (double) orc_f32_from_f16(rd16(blk));
        for (int g = 0; g < 8; g++) {
            const int qh = blk[66 + g];
            const int sc = blk[74 + g];
            for (int j = 0; j < 4; j++) {
                const int ls = j < 2 ? (sc & 15) : (sc >> 4);
                const uint32_t idx = (uint32_t) blk[2 + 4 * g + j] | ((uint32_t) ((qh >> (2 * j)) & 3) << 8);
                const uint64_t e = k_iq2s_grid[idx];
                const uint32_t sb = blk[34 + 4 * g + j];
                for (int m = 0; m < 8; m++) {
                    double v = (double) ((e >> (8 * m)) & 0xFFu);
                    if ((sb >> m) & 1u) v = -v;
                    out[b * 256 + g * 32 + j * 8 + m] = (float) (d * (0.5 + ls) * 0.25 * v);
                }
            }
        }
    }
}

/* ------------------------------------------------------------------------------------------------ */
/* the block                                                                                        */
/* ------------------------------------------------------------------------------------------------ */

typedef struct {
    const orc_layer* L;
    int T, mode;
    const float* x;
    /* per token */
    float* xr;          /* [T][n_embd] bf16-rounded x */
    uint8_t* xq;        /* [T][n_embd/32*36] */
    float* logits;      /* [T][E] */
    int32_t* ids;       /* [T][k] */
    float* w;           /* [T][k] */
    float* scale;       /* [T] shared gate logit */
    /* per (token, slot) with slot k = the shared expert */
    float* g;           /* [T][k+1][n_ff] */
    float* u;
    uint8_t* hq;        /* [T][k+1][n_ff/32*36] */
    float* h32;         /* [T][k+1][n_ff] fp32-mode SwiGLU output */
    float* parts;       /* [T][k+1][n_embd] */
    int chunks_gu, chunks_d;
    int rows_gu, rows_d;
    atomic_int next;
    int n_items;
    int phase;
    int bad;
} layer_job;

static const uint8_t* slot_plane(const layer_job* J, int t, int slot, int which, int* type) {
    const orc_layer* L = J->L;
    const size_t gu_n = orc_row_bytes(L->gu_type, L->n_embd) * (size_t) L->n_ff;
    const size_t d_n = orc_row_bytes(L->d_type, L->n_ff) * (size_t) L->n_embd;
    if (slot == L->k) {
        *type = which == 0 ? L->sg_type : which == 1 ? L->su_type : L->sd_type;
        return which == 0 ? L->sgate : which == 1 ? L->sup : L->sdown;
    }
    const int id = J->ids[(size_t) t * L->k + slot];
    *type = which == 2 ? L->d_type : L->gu_type;
    if (which == 0) return L->gate + (size_t) id * gu_n;
    if (which == 1) return L->up + (size_t) id * gu_n;
    return L->down + (size_t) id * d_n;
}

static double dot_f32(int type, const uint8_t* row, const float* x, int n, float* scratch) {
    orc_dequant_row(type, row, n, scratch);
    double acc = 0;
    for (int i = 0; i < n; i++) acc += (double) scratch[i] * (double) x[i];
    return acc;
}

/* The router stage alone for T tokens (layer_exec.cpp:470-472): x rounded to bf16, logits by bf16_dot
 * (pack_parity.cpp:3793-3799), then route_ref (pack_parity.cpp:5144-5165); the same steps as phase 0 below. */
void orc_router(const float* x, int T, const uint16_t* router, int n_expert, int n_embd, int k, float* logits,
                int32_t* ids, float* w) {
    float* xr = (float*) malloc(sizeof(float) * (size_t) n_embd);
    for (int t = 0; t < T; t++) {
        const float* xt = x + (size_t) t * n_embd;
        float* lt = logits + (size_t) t * n_expert;
        for (int i = 0; i < n_embd; i++) xr[i] = orc_f32_from_bf16(orc_bf16_from_f32(xt[i]));
        for (int e = 0; e < n_expert; e++) lt[e] = orc_bf16_dot(xr, router + (size_t) e * n_embd, n_embd);
        orc_route(lt, n_expert, k, ids + (size_t) t * k, w + (size_t) t * k);
    }
    free(xr);
}

/* phase 0: per token routing + q8_1; phase 1: gate/up rows; phase 2: SwiGLU (+ q8_1 of h);
 * phase 3: down rows. */
static void run_item(layer_job* J, int item, float* scratch) {
    const orc_layer* L = J->L;
    const int S = L->k + 1;
    const int E = L->n_expert, H = L->n_embd, F = L->n_ff;
    if (J->phase == 0) {
        const int t = item;
        const float* xt = J->x + (size_t) t * H;
        float* xr = J->xr + (size_t) t * H;
        for (int i = 0; i < H; i++) xr[i] = orc_f32_from_bf16(orc_bf16_from_f32(xt[i]));
        for (int e = 0; e < E; e++) J->logits[(size_t) t * E + e] = orc_bf16_dot(xr, L->router + (size_t) e * H, H);
        orc_route(J->logits + (size_t) t * E, E, L->k, J->ids + (size_t) t * L->k, J->w + (size_t) t * L->k);
        for (int i = 0; i < L->k; i++) {
            const int id = J->ids[(size_t) t * L->k + i];
            if (id < 0 || id >= E) J->bad = 1;
        }
        orc_quant_q8_1(xt, H, J->xq + (size_t) t * orc_q8_1_bytes(H));
        if (L->has_shared) J->scale[t] = orc_bf16_dot(xr, L->ginp, H);
        return;
    }
    if (J->phase == 2) {
        const int t = item / S, slot = item % S;
        const size_t o = ((size_t) t * S + slot) * F;
        if (slot == L->k && !L->has_shared) return;
        if (J->mode == 0) {
            orc_swiglu_q8(J->g + o, J->u + o, F, J->hq + ((size_t) t * S + slot) * orc_q8_1_bytes(F));
        } else {
            for (int r = 0; r < F; r++) {
                const double g = (double) J->g[o + r];
                J->h32[o + r] = (float) (g / (1.0 + exp(-g)) * (double) J->u[o + r]);
            }
        }
        return;
    }
    const int chunks = J->phase == 1 ? J->chunks_gu : J->chunks_d;
    const int rows_per = J->phase == 1 ? J->rows_gu : J->rows_d;
    const int ts = item / chunks, c = item % chunks;
    const int t = ts / S, slot = ts % S;
    if (slot == L->k && !L->has_shared) return;
    if (J->bad) return;
    if (J->phase == 1) {
        int tg, tu;
        const uint8_t* gp = slot_plane(J, t, slot, 0, &tg);
        const uint8_t* up = slot_plane(J, t, slot, 1, &tu);
        const size_t rbg = orc_row_bytes(tg, H), rbu = orc_row_bytes(tu, H);
        const size_t o = ((size_t) t * S + slot) * F;
        for (int r = c * rows_per; r < F && r < (c + 1) * rows_per; r++) {
            if (J->mode == 0) {
                const uint8_t* xq = J->xq + (size_t) t * orc_q8_1_bytes(H);
                J->g[o + r] = orc_row_dot(tg, gp + r * rbg, xq, H);
                J->u[o + r] = orc_row_dot(tu, up + r * rbu, xq, H);
            } else {
                const float* xt = J->x + (size_t) t * H;
                J->g[o + r] = (float) dot_f32(tg, gp + r * rbg, xt, H, scratch);
                J->u[o + r] = (float) dot_f32(tu, up + r * rbu, xt, H, scratch);
            }
        }
        return;
    }
    int td;
    const uint8_t* dp = slot_plane(J, t, slot, 2, &td);
    const size_t rbd = orc_row_bytes(td, F);
    const size_t o = ((size_t) t * S + slot) * H;
    for (int r = c * rows_per; r < H && r < (c + 1) * rows_per; r++) {
        if (J->mode == 0) {
            const uint8_t* hq = J->hq + ((size_t) t * S + slot) * orc_q8_1_bytes(F);
            J->parts[o + r] = orc_row_dot(td, dp + r * rbd, hq, F);
        } else {
            J->parts[o + r] = (float) dot_f32(td, dp + r * rbd, J->h32 + ((size_t) t * S + slot) * F, F, scratch);
        }
    }
}

typedef struct { layer_job* J; } worker_arg;

static void* worker(void* p) {
    layer_job* J = ((worker_arg*) p)->J;
    const int n = J->L->n_embd > J->L->n_ff ? J->L->n_embd : J->L->n_ff;
    float* scratch = (float*) malloc(sizeof(float) * (size_t) n);
    for (;;) {
        const int i = atomic_fetch_add(&J->next, 1);
        if (i >= J->n_items) break;
        run_item(J, i, scratch);
    }
    free(scratch);
    return NULL;
}

static void run_phase(layer_job* J, int phase, int n_items, int n_threads) {
    J->phase = phase;
    J->n_items = n_items;
    atomic_store(&J->next, 0);
    if (n_threads <= 1 || n_items <= 1) {
        worker_arg a = {J};
        worker(&a);
        return;
    }
    int nt = n_threads < n_items ? n_threads : n_items;
    pthread_t* th = (pthread_t*) malloc(sizeof(pthread_t) * (size_t) nt);
    worker_arg a = {J};
    for (int i = 1; i < nt; i++) pthread_create(&th[i], NULL, worker, &a);
    worker(&a);
    for (int i = 1; i < nt; i++) pthread_join(th[i], NULL);
    free(th);
}

int orc_moe_layer(const orc_layer* L, const float* x, int T, float* out, const orc_trace* tr, int mode,
                  int n_threads) {
    if (!L || L->n_embd <= 0 || L->n_ff <= 0 || L->n_expert <= 0 || L->k <= 0 || L->k > L->n_expert || T < 0)
        return -1;
    if (T == 0) return 0;
    if (!orc_row_bytes(L->gu_type, L->n_embd) || !orc_row_bytes(L->d_type, L->n_ff)) return -1;
    if (L->has_shared && (!orc_row_bytes(L->sg_type, L->n_embd) || !orc_row_bytes(L->su_type, L->n_embd) ||
                          !orc_row_bytes(L->sd_type, L->n_ff)))
        return -1;
    const int H = L->n_embd, F = L->n_ff, E = L->n_expert, K = L->k, S = K + 1;
    layer_job J;
    memset(&J, 0, sizeof J);
    J.L = L;
    J.T = T;
    J.mode = mode;
    J.x = x;
    J.xr = (float*) malloc(sizeof(float) * (size_t) T * H);
    J.xq = (uint8_t*) malloc(orc_q8_1_bytes(H) * (size_t) T);
    J.logits = (float*) malloc(sizeof(float) * (size_t) T * E);
    J.ids = (int32_t*) malloc(sizeof(int32_t) * (size_t) T * K);
    J.w = (float*) malloc(sizeof(float) * (size_t) T * K);
    J.scale = (float*) calloc((size_t) T, sizeof(float));
    J.g = (float*) malloc(sizeof(float) * (size_t) T * S * F);
    J.u = (float*) malloc(sizeof(float) * (size_t) T * S * F);
    J.hq = (uint8_t*) malloc(orc_q8_1_bytes(F) * (size_t) T * S);
    J.h32 = (float*) malloc(sizeof(float) * (size_t) T * S * F);
    J.parts = (float*) malloc(sizeof(float) * (size_t) T * S * H);
    J.rows_gu = 64;
    J.rows_d = 128;
    J.chunks_gu = (F + J.rows_gu - 1) / J.rows_gu;
    J.chunks_d = (H + J.rows_d - 1) / J.rows_d;
    run_phase(&J, 0, T, n_threads);
    int rc = 0;
    if (J.bad) {
        rc = -1;
        goto done;
    }
    run_phase(&J, 1, T * S * J.chunks_gu, n_threads);
    run_phase(&J, 2, T * S, n_threads);
    run_phase(&J, 3, T * S * J.chunks_d, n_threads);
    {
        float* shared = (float*) malloc(sizeof(float) * (size_t) H);
        for (int t = 0; t < T; t++) {
            const float* sh = NULL;
            if (L->has_shared) {
                /* sigmoid in float with the libm exp (pack_parity.cpp:3646), applied to the down output */
                const float sig = 1.0f / (1.0f + expf(-J.scale[t]));
                const float* sd = J.parts + ((size_t) t * S + K) * H;
                for (int d = 0; d < H; d++) shared[d] = sd[d] * sig;
                sh = shared;
                if (tr && tr->shared) memcpy(tr->shared + (size_t) t * H, shared, sizeof(float) * (size_t) H);
            }
            orc_combine(J.parts + (size_t) t * S * H, J.w + (size_t) t * K, sh, out + (size_t) t * H, H, K);
            if (tr && tr->parts)
                memcpy(tr->parts + (size_t) t * K * H, J.parts + (size_t) t * S * H, sizeof(float) * (size_t) K * H);
        }
        free(shared);
    }
    if (tr) {
        if (tr->logits) memcpy(tr->logits, J.logits, sizeof(float) * (size_t) T * E);
        if (tr->ids) memcpy(tr->ids, J.ids, sizeof(int32_t) * (size_t) T * K);
        if (tr->weights) memcpy(tr->weights, J.w, sizeof(float) * (size_t) T * K);
        if (tr->xq) memcpy(tr->xq, J.xq, orc_q8_1_bytes(H) * (size_t) T);
    }
done:
    free(J.xr); free(J.xq); free(J.logits); free(J.ids); free(J.w); free(J.scale);
    free(J.g); free(J.u); free(J.hq); free(J.h32); free(J.parts);
    return rc;
}

/* elementwise_parity.cpp:84-100 (rms_ref with use_sum = false, use_w = w != NULL); add_inplace before it. */
void orc_add_rms_norm(const float* x, const float* residual, const float* w, int64_t rows, int64_t cols, float eps,
                      float* out) {
    for (int64_t r = 0; r < rows; r++) {
        const float* xr = x + r * cols;
        float* o = out + r * cols;
        for (int64_t c = 0; c < cols; c++) o[c] = residual ? xr[c] + residual[r * cols + c] : xr[c];
        double ss = 0.0;
        for (int64_t c = 0; c < cols; c++) {
            const double v = o[c];
            ss += v * v;
        }
        const double den = sqrt(ss / (double) cols + (double) eps);
        for (int64_t c = 0; c < cols; c++) {
            const double v = o[c];
            o[c] = (float) ((v / den) * (w ? (double) w[c] : 1.0));
        }
    }
}

/* ---- the Strata pack's planar S2 experts (include/strata/kernels/cpu/expert.hpp:34-51) -------------------------
 * One expert of geometry (H, F) in one blob: the 2F gate/up code rows interleaved (row 2r gate r, 2r + 1 up r),
 * H / 4 bytes each; then the H down code rows, F / 4 bytes each; then the fp16 scales of the gate/up rows (H / 64
 * per row, same row order) and of the down rows (F / 64 per row).  Codes are 2 bits, four per byte, first value in
 * the low bits (the GGUF Q2_0 qs order, dequant.hpp:69-78); a weight is (code - 1) * d of its 64-value block.  The
 * pack is therefore a lossless re-layout of the GGUF Q2_0 planes, and orc_s2_pack performs it. */
size_t orc_s2_blob_bytes(int H, int F) { return (size_t) 3 * H * F / 64 * 18; }

static void s2_offsets(int H, int F, size_t* gu_codes, size_t* d_codes, size_t* gu_scales, size_t* d_scales) {
    *gu_codes = 0;
    *d_codes = (size_t) 2 * F * (H / 4);
    *gu_scales = *d_codes + (size_t) H * (F / 4);
    *d_scales = *gu_scales + (size_t) 2 * F * (H / 64) * 2;
}

/* One GGUF Q2_0 row of n values -> its codes (n / 4 bytes) and scales (n / 64 fp16) in the planar form. */
static void s2_put_row(const uint8_t* row, int n, uint8_t* codes, uint8_t* scales) {
    for (int b = 0; b < n / 64; b++) {
        memcpy(scales + 2 * b, row + (size_t) b * 18, 2);
        memcpy(codes + 16 * b, row + (size_t) b * 18 + 2, 16);
    }
}

void orc_s2_pack(const uint8_t* gate, const uint8_t* up, const uint8_t* down, int H, int F, uint8_t* blob) {
    size_t oc, od, os, ods;
    s2_offsets(H, F, &oc, &od, &os, &ods);
    const size_t rgu = orc_row_bytes(ORC_Q2_0, H), rd = orc_row_bytes(ORC_Q2_0, F);
    for (int r = 0; r < F; r++) {
        s2_put_row(gate + (size_t) r * rgu, H, blob + oc + (size_t) (2 * r) * (H / 4),
                   blob + os + (size_t) (2 * r) * (H / 64) * 2);
        s2_put_row(up + (size_t) r * rgu, H, blob + oc + (size_t) (2 * r + 1) * (H / 4),
                   blob + os + (size_t) (2 * r + 1) * (H / 64) * 2);
    }
    for (int j = 0; j < H; j++)
        s2_put_row(down + (size_t) j * rd, F, blob + od + (size_t) j * (F / 4), blob + ods + (size_t) j * (F / 64) * 2);
}

/* quantize_q8_0 (metal/src/sgemv.mm:145-172, the GPU contract of include/strata/kernels/quantize_act.hpp:20-22):
 * per 32 values amax, d32 = amax / 127 in float, stored as fp16; q = rint((double) x / (double) d32) clamped to
 * [-128, 127]; an all-zero block is 34 zero bytes.  With `scales` (quantize_q8_0_scaled, quantize_act.hpp:24-30:
 * the same blocks plus the CPU's fp32 scale and its rounding rule): scales[b] = d32 and q is rounded half away
 * from zero (the CPU activation contract, expert.hpp:53-58), clamped to [-127, 127]. */
void orc_quant_q8_0(const float* x, int64_t n, uint8_t* blocks, float* scales) {
    for (int64_t b = 0; b < n / 32; b++) {
        const float* xb = x + b * 32;
        uint8_t* o = blocks + b * 34;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(xb[i]));
        if (scales) scales[b] = amax / 127.0f;
        if (amax == 0.0f) {
            memset(o, 0, 34);
            continue;
        }
        const float d32 = amax / 127.0f;
        const uint16_t d16 = orc_f16_from_f32(d32);
        o[0] = (uint8_t) d16;
        o[1] = (uint8_t) (d16 >> 8);
        for (int i = 0; i < 32; i++) {
            double q;
            if (scales) {
                q = roundf(xb[i] / d32);
                if (q > 127.0) q = 127.0;
                if (q < -127.0) q = -127.0;
            } else {
                q = rint((double) xb[i] / (double) d32);
                if (q > 127.0) q = 127.0;
                if (q < -128.0) q = -128.0;
            }
            o[2 + i] = (uint8_t) (int8_t) q;
        }
    }
}

/* One planar Q2_0 row (codes, fp16 scales) of n values against Q8_0 blocks: the reference's row_dot order
 * (iq_parity.cpp:275-292) over 32-value partials (d_w * d_x) * sum (code - 1) q, d_x the block's fp16 d or, with
 * x_scales, the fp32 scale. */
static float s2_row_dot(const uint8_t* codes, const uint8_t* sc, int n, const uint8_t* xq, const float* xs) {
    float lane[32], nxt[32];
    memset(lane, 0, sizeof lane);
    for (int k = 0; k < n / 32; k++) {
        int32_t sumi = 0;
        const uint8_t* xb = xq + (size_t) k * 34;
        for (int i = 0; i < 32; i++) {
            const int code = (codes[8 * k + i / 4] >> (2 * (i % 4))) & 3;
            sumi += (code - 1) * (int32_t) (int8_t) xb[2 + i];
        }
        const float dx = xs ? xs[k] : orc_f32_from_f16(rd16(xb));
        const float d = orc_f32_from_f16(rd16(sc + 2 * (k / 2))) * dx;
        lane[k & 31] += d * (float) sumi;
    }
    for (int o = 16; o > 0; o >>= 1) {
        for (int l = 0; l < 32; l++) nxt[l] = lane[l] + lane[l ^ o];
        memcpy(lane, nxt, sizeof lane);
    }
    return lane[0];
}

/* One S2 expert for one token (the chain of include/strata/kernels/s2_expert_grouped.hpp:11-16): gate and up rows
 * against x (Q8_0 blocks, optional fp32 scales), h = silu(g) * u, h quantized in the same contract as x (fp16 d
 * without scales, fp32 scales with them), down rows -> out[H]. */
void orc_s2_expert(const uint8_t* blob, int H, int F, const uint8_t* xq, const float* xs, float* out) {
    size_t oc, od, os, ods;
    s2_offsets(H, F, &oc, &od, &os, &ods);
    float* h = (float*) malloc(sizeof(float) * (size_t) F);
    uint8_t* hq = (uint8_t*) malloc((size_t) F / 32 * 34);
    float* hs = xs ? (float*) malloc(sizeof(float) * (size_t) F / 32) : NULL;
    for (int r = 0; r < F; r++) {
        const float g = s2_row_dot(blob + oc + (size_t) (2 * r) * (H / 4), blob + os + (size_t) (2 * r) * (H / 64) * 2,
                                   H, xq, xs);
        const float u = s2_row_dot(blob + oc + (size_t) (2 * r + 1) * (H / 4),
                                   blob + os + (size_t) (2 * r + 1) * (H / 64) * 2, H, xq, xs);
        h[r] = silu_mul(g, u);
    }
    orc_quant_q8_0(h, F, hq, hs);
    for (int j = 0; j < H; j++)
        out[j] = s2_row_dot(blob + od + (size_t) j * (F / 4), blob + ods + (size_t) j * (F / 64) * 2, F, hq, hs);
    free(h);
    free(hq);
    free(hs);
}
