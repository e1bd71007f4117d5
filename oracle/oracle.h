/* oracle.h - CPU restatement of StrataMetal's host MoE-block reference (TEST INFRASTRUCTURE ONLY).
 *
 * This library is the checker for the B200 kernels, never part of the product path.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may load it.
 *
 * It restates, in plain C, the host functions the reference's own parity tests judge the MoE block
 * against (file:line inside the StrataMetal tree):
 *   - bf16 / fp16 bit conversions            include/strata/kernels/bf16_bits.hpp:37-47, f16_bits.hpp:37-104
 *   - q8_1 activation block                  metal/src/iq_parity.cpp:350-382 (quant_host_block)
 *   - Q2_0 partial dot (code - 1)            metal/src/iq_parity.cpp:225-252 (dot_q2_0), pack_parity.cpp:2736-2757
 *   - IQ2_S partial dot                      metal/src/iq_parity.cpp:125-151 (dot_iq2_s)
 *   - IQ4_NL / IQ4_XS partial dots           metal/src/iq_parity.cpp:106-115, 196-222 (dot_iq4_nl, dot_iq4_xs);
 *   - IQ3_XXS / IQ3_S partial dots           metal/src/iq_parity.cpp:79-101, 153-194 (dot_iq3_xxs, dot_iq3_s);
 *                                            geometry :256-263 (geom_of).  The layer path takes none of these
 *                                            four; the stage entry point smoe_iq_mmvq takes IQ4_NL and IQ4_XS
 *   - 32-lane row accumulation + butterfly   metal/src/iq_parity.cpp:275-292 (row_dot), pack_parity.cpp:2759-2772
 *   - SwiGLU then q8_1 of h                  metal/src/iq_parity.cpp:384-411 (silu, ref_expert)
 *   - bf16 router dot, double accumulation   metal/src/pack_parity.cpp:3793-3799 (round_bf16, bf16_dot)
 *   - softmax / stable top-k / renorm        metal/src/pack_parity.cpp:5144-5165 (route_ref) == router_parity.cpp:48-72
 *   - shared expert + sigmoid gate           metal/src/pack_parity.cpp:8597-8606, 3646 (gdn_sigmoid)
 *   - combine, double sum in router order    metal/src/pack_parity.cpp:8607-8616 == moe_combine_parity.cpp:55-71
 *
 * Two modes: CONTRACT mode is the chain above (q8_1 activations, integer dots), the reference's own host
 * implementation of the block.  FP32 mode dequantizes the weights exactly and accumulates unquantized
 * activations in double (the "fp32 host accumulation" the spec names); it shares the router with the
 * contract mode.  Everything here must be compiled with -ffp-contract=off: the reference adds float
 * partials one by one, and a fused multiply-add would change the sums it defines. */
#ifndef STRATA_ORACLE_H
#define STRATA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_Q2_0 = 42, ORC_IQ2_S = 22, ORC_IQ4_NL = 20, ORC_IQ4_XS = 23, ORC_IQ3_XXS = 18, ORC_IQ3_S = 21 };

/* ---- formats and bit conversions ---- */
uint16_t orc_bf16_from_f32(float f);
float orc_f32_from_bf16(uint16_t h);
uint16_t orc_f16_from_f32(float f);
float orc_f32_from_f16(uint16_t h);
/* Bytes of one row of n values of `type` (Q2_0: 18 B / 64, IQ2_S: 82 B / 256); 0 when not a multiple. */
size_t orc_row_bytes(int type, int64_t n);
size_t orc_q8_1_bytes(int64_t n);

/* ---- stage references ---- */
void orc_quant_q8_1_block(const float* x32, uint8_t* y36);
void orc_quant_q8_1(const float* x, int64_t n, uint8_t* y);
/* One weight row against one q8_1 column, in the reference's 32-lane order. */
float orc_row_dot(int type, const uint8_t* row, const uint8_t* col_q8, int n_in);
/* y[c * n_out + r] = W[r] . x[c] (iq_mmvq semantics). */
void orc_mmvq(int type, const uint8_t* w, const uint8_t* x_q8, int n_in, int n_out, int n_col, float* y);
void orc_swiglu_q8(const float* gate, const float* up, int64_t n, uint8_t* y);
float orc_bf16_dot(const float* x_rounded, const uint16_t* row, int n);
void orc_route(const float* logits, int n_expert, int k, int32_t* ids, float* w);
/* bf16 rounding of x, the router logits and the routing of T tokens (the block's first stage). */
void orc_router(const float* x, int T, const uint16_t* router, int n_expert, int n_embd, int k, float* logits,
                int32_t* ids, float* w);
void orc_combine(const float* parts, const float* w, const float* shared, float* y, int n_embd, int k);

/* Dequantize one row to floats (exact: (code - 1) * d for Q2_0; d * (0.5 + ls) / 4 * signed grid for IQ2_S). */
void orc_dequant_row(int type, const uint8_t* row, int n, float* out);

/* ---- the whole block ---- */
typedef struct {
    int n_embd, n_ff, n_expert, k;
    int gu_type, d_type;                 /* routed experts: gate/up type, down type */
    const uint16_t* router;              /* [n_expert][n_embd] bf16 (ffn_gate_inp.weight) */
    const uint8_t* gate;                 /* ffn_gate_exps: n_expert x n_ff rows of gu_type over n_embd */
    const uint8_t* up;                   /* ffn_up_exps:   same */
    const uint8_t* down;                 /* ffn_down_exps: n_expert x n_embd rows of d_type over n_ff */
    int has_shared;
    int sg_type, su_type, sd_type;
    const uint8_t* sgate;                /* ffn_gate_shexp: n_ff rows over n_embd */
    const uint8_t* sup;                  /* ffn_up_shexp */
    const uint8_t* sdown;                /* ffn_down_shexp: n_embd rows over n_ff */
    const uint16_t* ginp;                /* ffn_gate_inp_shexp: [n_embd] bf16 */
} orc_layer;

/* Optional per-stage outputs (any pointer may be NULL). Shapes for T tokens. */
typedef struct {
    float* logits;                       /* [T][n_expert] */
    int32_t* ids;                        /* [T][k] */
    float* weights;                      /* [T][k] */
    float* parts;                        /* [T][k][n_embd] routed expert outputs, router order */
    float* shared;                       /* [T][n_embd] shared expert output after the sigmoid gate */
    uint8_t* xq;                         /* [T][n_embd/32 * 36] q8_1 image of x */
} orc_trace;

/* mode 0 = contract (q8_1 chain), 1 = fp32 (exact dequant, double accumulation).  n_threads <= 1 runs
 * serially; more threads split the work over (token, expert, row range) like the reference's expert pool.
 * Returns 0, or -1 on a bad geometry / routed id outside the pool. */
int orc_moe_layer(const orc_layer* L, const float* x, int T, float* out, const orc_trace* tr, int mode,
                  int n_threads);

/* rms_norm_weighted host rule (metal/src/elementwise_parity.cpp:84-100, mean form): per row, ss = sequential
 * fp64 sum of v^2, den = sqrt(ss / cols + eps), out = (float)((v / den) * w) (w NULL: unit weight).  With
 * residual non-NULL the row is first (float)(x + residual), the reference's add_inplace (elementwise.hpp:52). */
void orc_add_rms_norm(const float* x, const float* residual, const float* w, int64_t rows, int64_t cols, float eps,
                      float* out);

/* Trap variants for the tests (variant 1: Q2_0 codes without the -1, iq_parity.cpp:225-248 minus_one=false). */
/* The Strata pack's planar S2 experts (expert.hpp:34-51): blob size, GGUF Q2_0 -> S2 re-layout of one expert,
 * the Q8_0 activation rule (sgemv.mm:145-172; with `scales`, the fp32-scale variant of quantize_act.hpp:24-30) and
 * one expert for one token over Q8_0 activations. */
size_t orc_s2_blob_bytes(int H, int F);
void orc_s2_pack(const uint8_t* gate, const uint8_t* up, const uint8_t* down, int H, int F, uint8_t* blob);
void orc_quant_q8_0(const float* x, int64_t n, uint8_t* blocks, float* scales);
void orc_s2_expert(const uint8_t* blob, int H, int F, const uint8_t* xq, const float* xs, float* out);

float orc_row_dot_variant(int type, const uint8_t* row, const uint8_t* col_q8, int n_in, int variant);

#ifdef __cplusplus
}
#endif
#endif
