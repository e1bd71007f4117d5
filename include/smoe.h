/* smoe.h - C ABI of the B200-native StrataMetal MoE block (sm_100a).
 *
 * Every entry point takes device pointers, plain sizes and an explicit, non-null CUDA stream
 * (cudaStream_t passed as void*), enqueues work on that stream, never synchronises and never
 * allocates.  Scratch comes from a caller-owned arena sized by the matching *_scratch_bytes().
 *
 * Each declaration names the reference interface it replaces (file:line inside the StrataMetal tree).
 * Argument meaning and error behaviour follow those interfaces:
 *   - negative counts, k > 64, n_expert > 1024, k > n_expert, an unsupported type or a bad multiple
 *     return SMOE_INVALID_ARG / SMOE_UNSUPPORTED (the reference throws MetalError: router.mm:33-37,
 *     iq.mm:148-158, moe_combine.mm:31-38);
 *   - a zero count returns SMOE_OK before any launch and leaves every output untouched
 *     (router_parity.cpp:220-225, moe_combine_parity.cpp:168-176, iq_parity.cpp:560-569);
 *   - outputs are never written past their extent.
 * A kernel that gives up on a bounded wait, or meets a routed id outside the pool, records a code in the
 * per-device status word read by smoe_device_status(). */
#ifndef SMOE_H
#define SMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    SMOE_OK = 0,
    SMOE_INVALID_ARG = 1,
    SMOE_UNSUPPORTED = 2,
    SMOE_CUDA_ERROR = 3,
    SMOE_DEVICE_TIMEOUT = 4
} smoe_status;

/* ggml block formats (type ids) the layer and the stage entry points take. */
enum { SMOE_Q2_0 = 42, SMOE_IQ2_S = 22, SMOE_IQ4_NL = 20, SMOE_IQ4_XS = 23, SMOE_IQ3_XXS = 18, SMOE_IQ3_S = 21 };

/* Message of the last non-OK status returned on this thread ("" after an OK call). */
const char* smoe_last_error(void);

/* Reads (and with clear != 0 resets) the device status word of the current device after a sync:
 * 0 ok, 1 a bounded wait ran out, 2 a routed id outside the pool was met.
 * Replaces the reference's std::exit on CUDA errors (src/kernels/cuda/bf16_gemv.cu:68-80). */
unsigned smoe_device_status(int clear);

/* ---- geometry ------------------------------------------------------------------------------------ */

/* iq_row_bytes (metal/include/strata/metal/iq.hpp:41, iq.mm:124-129): bytes of one row of n values; 0 for an
 * unsupported type or a bad multiple.  Q2_0: 18 B / 64 values; IQ2_S: 82 B / 256; IQ4_NL: 18 B / 32; IQ4_XS:
 * 136 B / 256; IQ3_XXS: 98 B / 256; IQ3_S: 110 B / 256 (iq.mm:99-122). */
size_t smoe_row_bytes(int ggml_type, int64_t n);
/* iq_q8_1_bytes (iq.hpp:43, iq.mm:131-134): 36 B per 32 values; 0 unless n is a positive multiple of 32. */
size_t smoe_q8_1_bytes(int64_t n);

/* ---- stage entry points (one reference kernel each) ---------------------------------------------- */

/* f32_to_bf16_bulk (metal/include/strata/metal/elementwise.hpp:27; layer_exec.cpp:470):
 * round-to-nearest-even bf16 bits of n floats (bf16_bits.hpp:37-47). */
smoe_status smoe_f32_to_bf16_bulk(const float* x, uint16_t* y, int64_t n, void* stream);

/* bf16_gemv (metal/include/strata/metal/bf16_gemv.hpp:83-89, bf16_gemv.mm:195-203), n_col columns:
 * y[c][o] = sum_i f32(x[c][i]) * f32(w[o][i]).  The sum is accumulated in fp64 and rounded once, which is
 * the host oracle's bf16_dot (pack_parity.cpp:3795-3799); w is [n_out][n_in] row-major; n_in % 8 == 0. */
smoe_status smoe_bf16_gemv(const uint16_t* x, const uint16_t* w, float* y, int64_t n_in, int64_t n_out,
                           int64_t n_col, void* stream);

/* router_top10 (metal/include/strata/metal/router.hpp:14-16, router.mm:32-49; CUDA contract
 * include/strata/kernels/router_top10.hpp:20-21, native_router.hpp:17-18): per token softmax over all
 * n_expert logits (fp64), top-k by probability with the lower index on a tie, weights divided by
 * max(sum of the k, 2^-14).  logits [n_tokens][n_expert] f32; ids, weights [n_tokens][k]. */
smoe_status smoe_router_top10(const float* logits, int n_tokens, int n_expert, int k, int32_t* ids, float* weights,
                              void* stream);

/* The router as one call (a1 + a2 + a3 of the block, layer_exec.cpp:470-472): bf16 rounding of x, the
 * fp64-accumulated bf16 GEMV against w_router [n_expert][n_embd] into logits [n_tokens][n_expert], and
 * router_top10 on them.  n_embd % 8 == 0. */
smoe_status smoe_router(const float* x, const uint16_t* w_router, int n_tokens, int n_embd, int n_expert, int k,
                        float* logits, int32_t* ids, float* weights, void* stream);

/* iq_quantize_q8_1 (iq.hpp:46, iq.mm:138-146; kernel iq.metal:597-627): n floats (a multiple of 32) into
 * n/32 q8_1 blocks. */
smoe_status smoe_iq_quantize_q8_1(const float* x, int64_t n, uint8_t* y, void* stream);

/* iq_mmvq (iq.hpp:50-51, iq.mm:148-169; CUDA contract include/strata/kernels/iq_kernels.hpp:30):
 * y[c * n_out + r] = W[r] . x[c] for n_col q8_1 columns, W n_out rows of ggml_type over n_in values.
 * The sum of a row follows the reference's 32-lane order (iq.metal:459-514) and is bitwise its host
 * reference (iq_parity.cpp:275-292).  Types: Q2_0 (42), IQ2_S (22), IQ4_NL (20), IQ4_XS (23), IQ3_XXS (18) and
 * IQ3_S (21) (iq.metal:516-549, host dots iq_parity.cpp:125-222).  Every type: n_in at most 4096, n_out and
 * n_col at most 2^31 - 1, w 16-byte and x_q8 4-byte aligned. */
smoe_status smoe_iq_mmvq(int ggml_type, const uint8_t* w, const uint8_t* x_q8, int64_t n_in, int64_t n_out,
                         int64_t n_col, float* y, void* stream);

/* iq_swiglu_q8 (iq.hpp:54, iq.mm:201-210; kernel iq.metal:630-663): silu(gate) * up, stored as q8_1. */
smoe_status smoe_iq_swiglu_q8(const float* gate, const float* up, int64_t n, uint8_t* y, void* stream);

/* moe_combine (metal/include/strata/metal/moe_combine.hpp:14-15, moe_combine.mm:31-48; CUDA contract
 * native_moe.hpp:15-20, shared_expert.hpp:97-101) for n_tok tokens:
 * y[t][j] = sum_e w[t][e] * parts[t][e][j] + shared[t][j], summed in fp64 in router order and rounded once
 * (pack_parity.cpp:8607-8616).  shared may be NULL; it is added plain, not router weighted. */
smoe_status smoe_moe_combine(const float* parts, const float* weights, const float* shared, float* y,
                             int64_t n_embd, int k, int n_tok, void* stream);

/* fused::group (include/strata/prefill/moe_fused.hpp:46-50): routing ids [n_tok][k] -> expert groups.
 * Writes, inside `scratch` (smoe_moe_group_scratch_bytes), counts[n_expert], offsets[n_expert + 1] and the
 * active-expert list; slot[i] = the grouped row of pair i (i = t * k + j); src[row] = its token.  Rows of
 * one expert are in token order (the reference leaves that order free; this build fixes it).  A token's k ids
 * must name k different experts, as the router's do: a pair that repeats an expert named earlier in its token
 * gets slot -1 and no row, and the device status records 2 (an id outside the pool gets the same). */
size_t smoe_moe_group_scratch_bytes(int n_tok, int k, int n_expert);
smoe_status smoe_moe_group(const int32_t* ids, int n_tok, int k, int n_expert, void* scratch, int32_t* slot,
                           int32_t* src, void* stream);

/* No counterpart in the reference.  The same grouping as smoe_moe_group for callers that cannot allocate
 * device memory where they group tokens (code being captured into a CUDA graph, engines whose planner forbids
 * allocation on the token path, plug-ins inside a process that owns the allocator): the grouping tables live
 * in a static 12,544-byte device array instead of caller scratch, so at most 1024 experts (more is refused
 * with SMOE_INVALID_ARG).  Allocates nothing.  The first call on each device looks up the array's device
 * address (cudaGetSymbolAddress) and must come before any stream capture.  The address is kept for the life of
 * the process: after cudaDeviceReset (or anything else that destroys the device's primary context) it is
 * stale, so do not call this entry point on that device again in the same process.  All calls on a device
 * share the array; calls that overlap on the GPU race, so order them on one stream. */
smoe_status smoe_moe_group_noalloc(const int32_t* ids, int n_tok, int k, int n_expert, int32_t* slot, int32_t* src,
                                   void* stream);

/* ---- the block ----------------------------------------------------------------------------------- */

/* One MoE layer's weights on the device, named as the GGUF names them (layer_exec.cpp:369-452,
 * expert_spans :109-123).  Routed planes hold n_expert experts back to back; expert e's gate rows start
 * at gate + e * n_ff * smoe_row_bytes(gu_type, n_embd). */
typedef struct smoe_layer {
    int n_embd, n_ff, n_expert, k;
    int gu_type, d_type;              /* routed gate/up and down types: any SMOE_* format above */
    const uint16_t* router;           /* ffn_gate_inp.weight       [n_expert][n_embd] bf16 */
    const uint8_t* gate;              /* ffn_gate_exps.weight      [n_expert][n_ff rows] */
    const uint8_t* up;                /* ffn_up_exps.weight        [n_expert][n_ff rows] */
    const uint8_t* down;              /* ffn_down_exps.weight      [n_expert][n_embd rows] */
    int has_shared;
    int sg_type, su_type, sd_type;
    const uint8_t* sgate;             /* ffn_gate_shexp.weight     [n_ff rows over n_embd] */
    const uint8_t* sup;               /* ffn_up_shexp.weight       [n_ff rows over n_embd] */
    const uint8_t* sdown;             /* ffn_down_shexp.weight     [n_embd rows over n_ff] */
    const uint16_t* gate_inp_shexp;   /* ffn_gate_inp_shexp.weight [n_embd] bf16 */
} smoe_layer;

/* Optional stage outputs, the device-side FfnTrace (metal/include/strata/metal/layer_exec.hpp:100-109).
 * Any pointer may be NULL.  Shapes for n_tokens tokens. */
typedef struct smoe_trace {
    float* logits;     /* [T][n_expert] router logits (FfnTrace::route) */
    int32_t* ids;      /* [T][k] */
    float* weights;    /* [T][k] (FfnTrace::route_w) */
    uint8_t* xq;       /* [T][n_embd / 32 * 36] q8_1 image of x (FfnTrace::exq) */
    float* parts;      /* [T][k][n_embd] routed expert outputs in router order (FfnTrace::edown) */
    float* shared;     /* [T][n_embd] gated shared-expert output (FfnTrace::shared) */
} smoe_trace;

/* Stage timing, the device-side counterpart of the reference's per-(layer, stage) event pairs
 * (include/strata/core/layer.hpp:317-337).  While set (n >= SMOE_STAGES, events are cudaEvent_t),
 * smoe_moe_forward records events[i] on its stream when stage i has been enqueued:
 * 0 router GEMV, 1 top-k + q8_1 of x, 2 dispatch, 3 gate/up + SwiGLU, 4 down, 5 combine.
 * The setting is per host thread; NULL or n = 0 turns it off. */
enum { SMOE_STAGES = 6 };
void smoe_set_stage_events(void** events, int n);

/* The glue of the layer stack.  rms_norm_weighted (include/strata/kernels/elementwise.hpp:82, host rule
 * metal/src/elementwise_parity.cpp:84-100): in place, per row of cols values, x = (x / sqrt(mean(x^2) + eps)) * w
 * with the mean and the division in fp64 and w[cols] (NULL: unit weight, an extension).  smoe_add_rms_norm fuses
 * the reference's add_inplace (elementwise.hpp:52) before it: x = rms_norm(x + residual) * w, the step between
 * two MoE blocks of the stack (residual NULL: plain rms_norm_weighted).  Zero sizes return SMOE_OK untouched. */
smoe_status smoe_rms_norm_weighted(float* x, const float* w, int64_t rows, int64_t cols, float eps, void* stream);
smoe_status smoe_add_rms_norm(float* x, const float* residual, const float* w, int64_t rows, int64_t cols, float eps,
                              void* stream);

/* Expert-kernel path of smoe_moe_forward (no reference counterpart: the reference has one GPU path).
 * 0 (default) automatic: one token takes the fused single-token kernel (path 3) when the layer qualifies,
 * batches of 512 tokens or more the fp16 tensor-core kernels (path 2) when the layer qualifies, smaller batches
 * the int8 tensor-core kernels (path 4) when the layer qualifies, the SIMT kernels otherwise;
 * 1 the SIMT kernels always; 2 the fp16 tensor-core kernels whenever the layer qualifies (every routed and
 * shared matrix Q2_0, n_embd and n_ff multiples of 512); 3 the fused single-token kernel whenever the batch is
 * one token and the layer qualifies (every matrix Q2_0, n_embd a multiple of 512 and at most 4096, n_ff a
 * multiple of 128 and at most 1024, n_expert at most 512), automatic otherwise; 4 the int8 tensor-core kernels whenever the layer qualifies (every matrix Q2_0,
 * n_embd and n_ff each 512, 1024 or 2048).  The SIMT, fused and int8 tensor-core kernels evaluate the
 * reference's q8_1 integer contract in the reference's summation order (bit for bit); the fp16 tensor-core
 * kernels evaluate the same products from an exact fp16 hi/lo split of the q8_1 activation with f32
 * accumulation, so their results agree up to the order of the f32 additions.  Process-wide.  Layers with any
 * matrix in a format other than Q2_0 / IQ2_S always take the any-format kernels (path 5: the reference's row dot
 * per format, grouped by expert, bit for bit), whatever the setting. */
smoe_status smoe_set_expert_path(int path);
/* The path smoe_moe_forward takes for this layer and batch: 1 SIMT, 2 fp16 tensor cores, 3 fused single-token
 * kernel, 4 int8 tensor cores, 5 any-format kernels, -1 invalid layer. */
int smoe_expert_path_for(const smoe_layer* L, int n_tokens);

/* Validates the layer's geometry and types: SMOE_OK when smoe_moe_forward can run it. */
smoe_status smoe_layer_check(const smoe_layer* L);

/* Scratch the block needs for up to max_tokens tokens. */
size_t smoe_moe_scratch_bytes(const smoe_layer* L, int max_tokens);

/* FfnExec::run's MoE block (layer_exec.cpp:462-563 between gr_read and gr_write; upstream moe_route +
 * moe_shared + moe_combine_parts, include/strata/core/layer.hpp:170-190): x [n_tokens][n_embd] f32 ->
 * out [n_tokens][n_embd] f32 = router -> dispatch -> routed experts (gate/up, SwiGLU, q8_1, down) ->
 * sigmoid-gated shared expert -> combine.  The shared expert is added only when the layer has one. */
smoe_status smoe_moe_forward(const smoe_layer* L, const float* x, int n_tokens, float* out, void* scratch,
                             size_t scratch_bytes, const smoe_trace* trace, void* stream);

/* ---- the Strata pack's planar S2 experts and the grouped decode API over them ---------------------------------
 * Blob layout (include/strata/kernels/cpu/expert.hpp:34-51, with n_embd = H and n_ff = F parameters instead of the
 * artifact's fixed 2560 / 640): the 2F gate/up code rows interleaved (row 2r = gate r, 2r + 1 = up r), H / 4 bytes
 * each; the H down code rows, F / 4 bytes each; the fp16 scales of the gate/up rows (H / 64 per row) and of the
 * down rows (F / 64 per row).  Two-bit codes, four per byte, first value in the low bits; a weight is
 * (code - 1) * d of its 64-value block (s2_expert_grouped.hpp:68-71).  Every row is the reference's row_dot order
 * over 32-value partials (iq_parity.cpp:275-292), so a blob computes exactly what the GGUF Q2_0 rows it was packed
 * from compute on the same activation bytes.  Activations are ggml Q8_0 blocks (34 B: fp16 d, 32 int8); with
 * x_scales (n_embd / 32 fp32 per token) those scales replace d for the gate/up dots and the intermediate is
 * quantized with fp32 scales too (s2_expert_grouped.hpp:59-66).  Blobs and slots are 16-byte aligned. */

/* BLOB (expert.hpp:45) for this geometry; 0 unless n_embd and n_ff are positive multiples of 64. */
size_t smoe_s2_blob_bytes(int n_embd, int n_ff);
/* One expert's GGUF Q2_0 rows (gate and up: n_ff rows over n_embd; down: n_embd rows over n_ff) -> its S2 blob
 * (the pack's re-layout of the same codes and scales). */
smoe_status smoe_s2_pack_expert(const uint8_t* gate, const uint8_t* up, const uint8_t* down, int n_embd, int n_ff,
                                uint8_t* blob, void* stream);
/* quantize_q8_0 (include/strata/kernels/quantize_act.hpp:20-22; host rule metal/src/sgemv.mm:145-172): d32 =
 * amax / 127 stored as fp16, q = rint(x / d32) in double, clamped to [-128, 127]; zero blocks are 34 zero bytes.
 * With scales non-NULL, quantize_q8_0_scaled (quantize_act.hpp:24-30): the same blocks' d, scales[b] = d32 and q
 * rounded half away from zero in float (the CPU contract), clamped to [-127, 127].  n % 32 == 0. */
smoe_status smoe_quantize_q8_0(const float* x, uint8_t* blocks, float* scales, int64_t n, void* stream);
/* moe_hit_grouped_scratch_bytes (s2_expert_grouped.hpp:30-35): caller-owned scratch of the grouped / hit calls for
 * up to cap_entries entries (or hits). */
size_t smoe_moe_grouped_scratch_bytes(int64_t cap_entries, int64_t n_embd, int64_t n_ff);
/* moe_grouped_s2 (s2_expert_grouped.hpp:96-102): group g's blob at device address grp_ptr[g], its entries
 * [grp_start[g], grp_start[g + 1]); entry i reads activation row ent_tok[i] of x_q8_0 (and x_scales) and writes the
 * n_embd floats of out row ent_dst[i].  n_groups[0] (device) is the group count, at most cap_groups; every row of a
 * blob is read once for all of its entries.  Counts past their capacities are clamped and record status 2. */
smoe_status smoe_moe_grouped_s2(const unsigned long long* grp_ptr, const int32_t* grp_start, const int32_t* n_groups,
                                const int32_t* ent_dst, const int32_t* ent_tok, int64_t cap_groups, int64_t cap_entries,
                                int n_embd, int n_ff, const uint8_t* x_q8_0, const float* x_scales, void* scratch,
                                float* out, void* stream);
/* moe_group_resident (s2_expert_grouped.hpp:103-107): the groups of moe_grouped_s2 when every expert is resident at
 * base + id * blob_bytes: groups are the distinct ids of ids[n] in ascending order, a group's entries its routing
 * indices in order (dst = index, tok = index / k_per_tok); counts[0] = groups, counts[1] = entries.  n <= 1024;
 * negative ids are skipped.  grp_start holds n + 1 ints. */
smoe_status smoe_moe_group_resident(const int32_t* ids, int n, int k_per_tok, const uint8_t* base, int64_t blob_bytes,
                                    unsigned long long* grp_ptr, int32_t* grp_start, int32_t* counts, int32_t* ent_dst,
                                    int32_t* ent_tok, void* stream);
/* moe_hit_select / moe_hit_select_multi (s2_expert_grouped.hpp:80-86, 108-109): the routing entries of ids[n]
 * whose expert is resident (res_row[e] = slot, or -1), in routing order: slot[c], dst[c] = the entry's index, and
 * count[0] = the hits.  n <= 1024. */
smoe_status smoe_moe_hit_select(const int32_t* ids, const int32_t* res_row, int n, int n_expert, int32_t* slot,
                                int32_t* dst, int32_t* count, void* stream);
/* moe_hit_grouped_s2_dev / _multi (s2_expert_grouped.hpp:86-89, 110-112): hit h < d_count[0] (at most cap) is the
 * blob at blob_base + slot_index[h] * blob_bytes and writes out row dst_index[h]; it reads activation row
 * dst_index[h] / k_per_token, or row 0 for every hit when k_per_token is 0 (one token). */
smoe_status smoe_moe_hit_grouped_s2(const uint8_t* blob_base, const int32_t* slot_index, const int32_t* dst_index,
                                    const int32_t* d_count, int64_t cap, int64_t blob_bytes, int n_embd, int n_ff,
                                    const uint8_t* x_q8_0, const float* x_scales, int k_per_token, void* scratch,
                                    float* out, void* stream);
/* moe_hit_add (s2_expert_grouped.hpp:90-91): parts[dst[h]] += hit_out[dst[h]] (n_embd floats) for h < count[0]. */
smoe_status smoe_moe_hit_add(float* parts, const float* hit_out, const int32_t* dst, const int32_t* count, int64_t cap,
                             int64_t n_embd, void* stream);

/* ---- streaming routed experts from the pack on disk into HBM (include/smoe_stream.hpp holds the C++ classes) ----
 * The pack's expert file (metal/src/pack.cpp:367-416): pack_dir/native_experts.txt, header "# strata native
 * experts vN ... (n_expert E)" (N <= 4) and one line per layer "layer gu_type d_type offset blob_bytes", over
 * pack_dir/experts.bin (layers back to back, a layer's experts back to back); experts.bin is mapped read-only.
 * Set-up, not the token path. */
smoe_status smoe_native_experts_open(const char* pack_dir, void** handle);
void smoe_native_experts_close(void* handle);
/* pick_native_expert (pack.cpp:368-416): the formats, file offset and size of (layer, expert)'s blob, and a host
 * pointer to its bytes inside the mapping (any output may be NULL). */
smoe_status smoe_native_experts_pick(const void* handle, int64_t layer, int64_t expert, int* gu_type, int* d_type,
                                     uint64_t* file_off, uint64_t* blob_bytes, const uint8_t** host_blob);
/* The VRAM expert tier (include/strata/core/expert_cache.hpp:72-150): n_slots x blob_bytes of device memory,
 * checked against the free memory and allocated here, once (set-up); a (layer, expert) -> slot table on the host
 * and on the device; a slot is claimed once and never evicted; with per_layer != 0 layer l only takes slots
 * [l q, (l + 1) q), q = n_slots / n_layers (the last layer the remainder).  blob_bytes % 16 == 0. */
smoe_status smoe_expert_cache_open(int64_t n_slots, int64_t n_layers, int64_t n_expert, int64_t blob_bytes,
                                   int per_layer, void** handle);
void smoe_expert_cache_close(void* handle);
/* admit + fill_slot (expert_cache.hpp:133-137, 168-171): *slot = the expert's slot; a new one is filled from host
 * memory (copied through pinned staging, so the source may be reused at once) and published in the device table,
 * both on `stream`.  *slot = -1 when the cache is full (nothing queued). */
smoe_status smoe_expert_cache_ensure(void* handle, int64_t layer, int64_t expert, const uint8_t* host_blob,
                                     int64_t bytes, void* stream, int32_t* slot);
/* slot_of (expert_cache.hpp:130-131): the slot, or -1 (also for a layer or expert out of range). */
int32_t smoe_expert_cache_slot_of(const void* handle, int64_t layer, int64_t expert);
/* The slot arena's device base (slot s at base + s * blob_bytes) and one layer's device residency row
 * (int32 [n_expert]: slot or -1), the res_row smoe_moe_hit_select reads; NULL for a bad handle or layer. */
uint8_t* smoe_expert_cache_arena(const void* handle);
const int32_t* smoe_expert_cache_row(const void* handle, int64_t layer);

/* ---- the model boundary: a MoE layer read from a GGUF file by tensor name (include/smoe_gguf.hpp) ------------
 * FfnExec::load (metal/src/layer_exec.cpp:369-452, expert_spans :109-123) over the reference's tensor names
 * blk.<L>.ffn_gate_inp / ffn_{gate,up,down}_exps / ffn_{gate,up,down}_shexp / ffn_gate_inp_shexp .weight
 * (metal/include/strata/metal/layer_tensors.hpp:48).  GGUF v2 / v3, mapped read-only; set-up, not the token path. */
smoe_status smoe_gguf_open(const char* path, void** handle);
void smoe_gguf_close(void* handle);
/* A tensor by its full name: ggml type, shape ne[0..3] (ne[0] fastest), bytes and a host pointer into the mapping
 * (any output may be NULL). */
smoe_status smoe_gguf_tensor(const void* handle, const char* name, int* type, int64_t* ne4, uint64_t* bytes,
                             const uint8_t** data);
/* Uploads layer `layer`'s MoE planes (allocates device memory: set-up) and fills *out with them: geometry from the
 * shapes (gate ne = {n_embd, n_ff, n_expert}), k from <general.architecture>.expert_used_count unless k > 0, the
 * router as bf16 (an F32 router is rounded to nearest even).  Each expert plane must hold exactly n_expert experts
 * of whole rows.  *owner keeps the device memory until smoe_gguf_free_layer(*owner). */
smoe_status smoe_gguf_load_layer(const void* handle, int layer, int with_shared, int k, smoe_layer* out, void** owner);
void smoe_gguf_free_layer(void* owner);

/* ---- the batch-1 layer stack in one launch -------------------------------------------------------------------
 * Session::forward's layer walk (metal/src/forward.cpp:554-565) with the MoE half only, for one token:
 * x = rms_norm_weighted(MoE_l(x) + x, norm_w[l]) for l = 0 .. n_layers - 1 (eps; norm_w NULL or any entry NULL: unit
 * weight), out = the last x.  Equals n_layers calls of smoe_moe_forward each followed by smoe_add_rms_norm, bit for
 * bit, in one persistent cooperative launch per 48 layers.  Every layer: one geometry, every matrix Q2_0, n_embd a
 * multiple of 512 up to 4096, n_ff a multiple of 128 up to 1024, n_expert at most 512 (the rule of path 3;
 * SMOE_UNSUPPORTED otherwise).  x and out may be the same buffer. */
size_t smoe_stack_decode_scratch_bytes(const smoe_layer* L);
smoe_status smoe_stack_decode(const smoe_layer* layers, int n_layers, const float* const* norm_w, float eps,
                              const float* x, float* out, void* scratch, size_t scratch_bytes, void* stream);

/* ---- Expert parallelism over the GPUs of one node (no reference counterpart: the reference reaches a second
 * GPU only through its peer / remote expert tiers, include/strata/core/peer_experts.hpp:35-104, which this
 * replaces for the MoE block).  Rank r of `world` holds the router and the shared expert whole and the routed
 * experts [r * E / world, (r + 1) * E / world); each rank routes its own tokens, sends each token's q8_1 row
 * once to every rank that owns one of its experts, the owners run their experts and store every routed slot's
 * down row straight into the token rank's exchange area, and the token's rank combines in router order.  The
 * exchange areas are mapped into every process (CUDA IPC); the data path uses no collective library.
 * Results equal smoe_moe_forward's on the same tokens bit for bit (the same kernels, the same orders). */
enum { SMOE_EP_MAX_WORLD = 8, SMOE_EP_HANDLE_BYTES = 64 };

typedef struct smoe_ep {
    int rank;        /* this process's rank, 0 <= rank < world */
    int world;       /* ranks (GPUs), 1..SMOE_EP_MAX_WORLD; n_expert % world == 0 */
    int max_tokens;  /* tokens per rank and step, at most; the same on every rank */
    void* areas[SMOE_EP_MAX_WORLD]; /* every rank's exchange area as this process addresses it (own at [rank]) */
} smoe_ep;

/* Bytes of one rank's exchange area (the same on every rank). */
size_t smoe_ep_area_bytes(const smoe_layer* L, int max_tokens, int world);
/* Set-up, not the token path: allocates a zeroed exchange area on the current device and, when ipc_handle is
 * not NULL, writes its SMOE_EP_HANDLE_BYTES-byte IPC handle there for the other processes. */
smoe_status smoe_ep_area_alloc(size_t bytes, void** area, void* ipc_handle);
/* Maps another process's area from its handle (peer access over NVLink), and unmaps it. */
smoe_status smoe_ep_area_open(const void* ipc_handle, void** area);
smoe_status smoe_ep_area_close(void* area);
smoe_status smoe_ep_area_free(void* area);
/* Once per rank after every area exists (and before any rank's first step): records this rank's view of the
 * areas in its own.  L->n_expert is the whole pool; L->gate / up / down hold this rank's experts. */
smoe_status smoe_ep_init(const smoe_ep* ep, const smoe_layer* L);
/* Local scratch of smoe_ep_forward. */
size_t smoe_ep_scratch_bytes(const smoe_layer* L, const smoe_ep* ep);
/* The MoE block of this rank's n_tokens tokens (0 <= n_tokens <= max_tokens; 0 still takes part in the
 * exchange): every rank calls it once per step, in the same order.  phases: 1 route + dispatch, 2 receive +
 * experts, 4 wait + combine, ORed; 7 is a whole step.  A caller that drives several ranks from one process on
 * one device runs phase 1 of every rank, then 2 of every rank, then 4, so that no kernel ever waits for one
 * launched after it.  Waits are bounded: a rank that does not take part makes the others record
 * SMOE_DEVICE_TIMEOUT in the status word within seconds.  Layers whose shared expert types differ from the
 * routed ones, formats other than Q2_0 / IQ2_S, and n_embd not a multiple of 128, are SMOE_UNSUPPORTED. */
smoe_status smoe_ep_forward(const smoe_layer* L, const smoe_ep* ep, const float* x, int n_tokens, float* out,
                            void* scratch, size_t scratch_bytes, const smoe_trace* trace, int phases, void* stream);

#ifdef __cplusplus
}
#endif
#endif
