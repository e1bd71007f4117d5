// kernels.cuh - launchers shared between the kernel files and the C ABI (api.cu).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/smoe.h"

namespace smoe {

constexpr int kRouterTokTile = 16;  // tokens per CTA in the router GEMV (x staged as bf16: 16 x n_embd x 2 bytes)
constexpr int kRouterGemmMinTokens = 64;  // above this the router logits use the tiled fp64 GEMM
constexpr int kMaxExperts = 1024;
constexpr int kMaxK = 64;

// Activations in the expert kernels' layout ("ka"): per 32-value block 48 bytes = 8 words (Q2_0 weights:
// byte b of word j of each half = value 4b + j of that 16-value half; IQ2_S weights: natural order), the q8_1
// scale as f32 (the fp16 d read back), 0x4B400000 - the sum of the 32 q, and 8 bytes of padding so every block is 16-byte
// aligned and a row of blocks is one bulk copy.
constexpr int kKaBlock = 48;
struct KAct {
    uint8_t* base;  // [rows][nblk][48]
};
inline size_t ka_bytes(int64_t rows, int nblk) { return (size_t) rows * nblk * kKaBlock; }
inline KAct ka_at(void* base, int64_t rows, int nblk) {
    (void) rows;
    (void) nblk;
    return KAct{static_cast<uint8_t*>(base)};
}

// ---- router.cu ----
// split_scratch (router_split_bytes of it, 256-byte aligned): few-token f32 calls take the fp64 tensor-path GEMM
// split over K instead of the GEMV, to fill the SMs.
// With defer non-null, a split-K router GEMM leaves the sum of its partials to the top-k launch (*defer = the
// number of splits, 0 when the GEMM wrote the logits itself).
cudaError_t launch_bf16_gemv(const void* x, bool f32_in, const uint16_t* w, const uint16_t* extra, float* y,
                             float* y_extra, int T, int H, int n_out, cudaStream_t s, void* split_scratch = nullptr,
                             int* defer = nullptr);
size_t router_split_bytes(int T, int n_rows, int H);
// The split-K partials of a deferred router GEMM: the top-k kernel adds them (in split order, as the reduce kernel
// does) into lout [T][E] and y_extra [T] (the shared gate's logit, when the GEMM had that row) before it routes.
struct RouterSplit {
    const double* part;
    int S;
    float* lout;
    float* y_extra;
};
// xa (optional): the activation in the expert kernels' layout, permuted for Q2_0 gate/up when xa_q2 != 0.
cudaError_t launch_router_topk(const float* logits, int T, int E, int k, int32_t* ids, float* w, const float* x,
                               uint8_t* xq, int H, cudaStream_t s, const KAct* xa = nullptr, int xa_q2 = 1,
                               const RouterSplit* split = nullptr);
cudaError_t launch_quant_q8_1(const float* x, int64_t n, uint8_t* y, cudaStream_t s);
cudaError_t launch_swiglu_q8(const float* g, const float* u, int64_t n, uint8_t* y, cudaStream_t s);
cudaError_t launch_f32_to_bf16(const float* x, uint16_t* y, int64_t n, cudaStream_t s);
cudaError_t launch_quant_ka(const float* x, int64_t rows, int H, const KAct& xa, int q2, cudaStream_t s);

// ---- dispatch.cu ----
// Grouping tables inside the caller's scratch: counts[E], offsets[E + 1], active[E], n_active[1],
// work[4] (counters for the expert kernels), all int32.
struct GroupTables {
    int32_t* counts;
    int32_t* offsets;
    int32_t* active;
    int32_t* n_active;
    int32_t* work;
};
size_t group_tables_bytes(int n_expert);
GroupTables group_tables_at(void* base, int n_expert);

// Work list of the layer path: the active experts ordered heaviest first (token count descending, expert id
// ascending), each split into chunks of at most kChunk slots.  Entry c covers slots [beg[c], beg[c] + n[c])
// of expert e[c].
constexpr int kChunk = 8;     // the SIMT expert kernels
constexpr int kTcChunk = 64;  // the tensor-core expert kernels
struct Sched {
    int32_t* e;
    int32_t* beg;
    int32_t* n;
    int32_t* count;  // [1] entries
    int chunk = kChunk;
};
inline int sched_capacity(int E, int T, int k, int chunk = kChunk) { return E + (T * k + chunk - 1) / chunk + 1; }
size_t sched_bytes(int E, int T, int k, int chunk = kChunk);
Sched sched_at(void* base, int E, int T, int k, int chunk = kChunk);

// `sched` may be null (the stage entry points): then only the grouping tables are written.
// With chunk_counts (group_chunk_bytes(T, E) of scratch) and more than kGroupWideMinTokens tokens the grouping
// runs over many CTAs (three launches) instead of one; the result is the same.
constexpr int kGroupWideMinTokens = 256;
size_t group_chunk_bytes(int T, int E);
// skip_negative: ids < 0 mark pairs that are not grouped (slot -1, no error); pair (optional): pair[row] = the
// pair index t * k + j of each grouped row.
cudaError_t launch_group(const int32_t* ids, int T, int k, int E, GroupTables g, int32_t* slot, int32_t* src,
                         cudaStream_t s, const Sched* sched = nullptr, int32_t* chunk_counts = nullptr,
                         int skip_negative = 0, int32_t* pair = nullptr);


// ---- expert.cu ----
// Which rows of which expert a grouped launch covers.  Routed experts are the n_active entries of `active`
// with slots [offsets[e], offsets[e + 1]); slot_token maps a routed slot to its token.  When shared_slots > 0
// one more "expert" follows: the shared expert, slots [shared_base, shared_base + shared_slots), token =
// slot - shared_base.  With single_cols > 0 there is exactly one expert (index 0) with slots [0, single_cols)
// and token = slot (the plain matrix-vector product over columns).
struct GroupView {
    const int32_t* offsets;
    const int32_t* active;
    const int32_t* n_active;
    const int32_t* slot_token;
    int max_active;
    int no_routed;  // 1: only the shared expert (a launch for a shared type that differs from the routed one)
    int shared_base;
    int shared_slots;
    int single_cols;
};

struct Matrix {
    const uint8_t* base;   // expert 0's first row
    int64_t expert_stride; // bytes between experts
    int type;              // ggml type
};

// y[slot][r] = down_e[r] . act[slot] for every slot, y row stride y_stride floats; act rows n_in / 32 blocks.
// ---- iqx.cu ---- (every block format against q8_1 columns, the reference's row_dot order)
bool gx_type_ok(int type);
size_t gx_row_bytes(int type, int64_t n);
cudaError_t launch_gx_mmvq(int type, const uint8_t* w, const uint8_t* x, int n_in, int n_out, int n_col,
                           float* y, cudaStream_t s);
cudaError_t launch_expert_down(Matrix down, Matrix sdown, GroupView g, const uint8_t* act, int act_by_token,
                               float* y, int64_t y_stride, int n_in, int n_out, cudaStream_t s);

// Expert parallelism: the warps that wrote routed rows to other ranks report here.  Each such warp fences its
// stores system-wide and counts itself in `counter` (this rank's memory); the last of `total` warps resets the
// counter and adds 1 to every rank's done flag for this rank (flags[p] points into rank p's exchange area).
struct EpDone {
    unsigned* counter = nullptr;
    unsigned* const* flags = nullptr;
    int world = 0;
};

// The layer path (v3): work items are (work-list entry, row tile), claimed dynamically from `counter`
// (zeroed by the dispatch) heaviest first; the shared expert's chunks come first when shared_slots > 0.
struct Work {
    Sched sched;
    const int32_t* slot_token;
    int max_entries;   // capacity of the routed work list (bounds the grid)
    int shared_base;   // first shared slot (T * k)
    int shared_slots;  // T, or 0 when the shared expert is not in this launch
    int no_routed;     // 1: the shared expert only
    int32_t* counter;
    // Expert parallelism (null otherwise): the down output of routed slot s goes to the rank that owns its
    // token, ep_out[p / (ep_rows * ep_k)] + (p % (ep_rows * ep_k)) * n_out with p = slot_pair[s] (received row
    // * k + j; received rows come in blocks of ep_rows per source rank); shared slot s goes to
    // ep_shared + (s - shared_base) * n_out.
    const int32_t* slot_pair = nullptr;
    float* const* ep_out = nullptr;
    float* ep_shared = nullptr;
    int ep_rows = 0;
    int ep_k = 0;
    EpDone ep_done;
};
// gate and up rows into gu[slot][gate n_ff | up n_ff] (f32), then SwiGLU + q8_1 of h into ha.
cudaError_t launch_layer_gate_up(Matrix gate, Matrix up, Matrix sgate, Matrix sup, Work w, KAct xa, float* gu,
                                 int n_embd, int n_ff, cudaStream_t s);
cudaError_t launch_swiglu_ka(const float* gu, KAct ha, int64_t rows, int n_ff, int down_q2, cudaStream_t s);
cudaError_t launch_layer_down(Matrix down, Matrix sdown, Work w, KAct ha, float* y, int n_ff, int n_embd,
                              cudaStream_t s);

// The any-format layer path (iqx.cu): gate/up rows into gu[slot][gate n_ff | up n_ff], SwiGLU + q8_1 of h into
// hq[slot][n_ff / 32] (q8_1 blocks), down rows into y[slot][n_embd]; xq holds the q8_1 blocks of every token.
// shared_only 1 runs the shared expert's slots with the given (shared) matrices, 0 the routed work list.
cudaError_t launch_gx_gate_up(Matrix gate, Matrix up, Work w, int shared_only, const uint8_t* xq, float* gu,
                              int n_embd, int n_ff, cudaStream_t s);
cudaError_t launch_gx_swiglu(const float* gu, uint8_t* h, int64_t rows, int n_ff, cudaStream_t s);
cudaError_t launch_gx_down(Matrix down, Work w, int shared_only, const uint8_t* hq, float* y, int n_ff, int n_embd,
                           cudaStream_t s);

// ---- tc.cu ---- (Q2_0 weights; n_embd and n_ff multiples of 512; work list built with chunk kTcChunk)
// xh: hi/lo fp16 image of the q8_1 activation, rows [0, T) hi and [T, 2T) lo.
cudaError_t launch_quant_xh(const float* x, int T, int H, __half* xh, cudaStream_t s);
// gate/up + SwiGLU + q8_1 of h into hh (hi rows [0, R), lo rows [R, 2R), R = slot rows).
cudaError_t launch_tc_gate_up(Matrix gate, Matrix up, Matrix sgate, Matrix sup, Work w, int n_expert,
                              const __half* xh, int T, __half* hh, int R, int n_embd, int n_ff, cudaStream_t s);
// down rows of every slot into parts[slot][n_embd].
cudaError_t launch_tc_down(Matrix down, Matrix sdown, Work w, int n_expert, const __half* hh, int R, float* parts,
                           int n_ff, int n_embd, cudaStream_t s);

// ---- tq.cu ---- (Q2_0 weights, n_embd and n_ff in {512, 1024, 2048}; work list built with chunk kChunk = 8)
// The q8_1 integer contract on the int8 tensor cores, bitwise the SIMT kernels' results.
bool tq_qualifies(int H, int F);
// gate/up + SwiGLU + q8_1 of h into ha (the down matrix's KAct layout).
cudaError_t launch_tq_gate_up(Matrix gate, Matrix up, Matrix sgate, Matrix sup, Work w, int n_expert, KAct xa,
                              KAct ha, int down_q2, int n_embd, int n_ff, cudaStream_t s);
// down rows of every slot into y[slot][n_embd] (or the expert-parallel destinations of the Work).
cudaError_t launch_tq_down(Matrix down, Matrix sdown, Work w, int n_expert, KAct ha, float* y, int n_ff, int n_embd,
                           cudaStream_t s);

// ---- s2.cu ---- (the pack's planar S2 experts and the grouped / hit decode API over them)
size_t s2_blob_bytes(int H, int F);
size_t s2_scratch_bytes(int64_t cap, int H, int F);
cudaError_t launch_s2_pack(const uint8_t* gate, const uint8_t* up, const uint8_t* down, int H, int F, uint8_t* blob,
                           cudaStream_t s);
cudaError_t launch_quant_q8_0(const float* x, int64_t n, uint8_t* y, float* scales, cudaStream_t s);
cudaError_t launch_s2_grouped(const unsigned long long* grp_ptr, const int32_t* grp_start, const int32_t* n_groups,
                              const int32_t* ent_dst, const int32_t* ent_tok, int cap_groups, int cap_entries, int H,
                              int F, const uint8_t* xq, const float* xs, void* scratch, float* out, cudaStream_t s);
cudaError_t launch_s2_group_resident(const int32_t* ids, int n, int k_per_tok, const uint8_t* base, int64_t blob,
                                     unsigned long long* grp_ptr, int32_t* grp_start, int32_t* counts, int32_t* ent_dst,
                                     int32_t* ent_tok, cudaStream_t s);
cudaError_t launch_s2_hit_select(const int32_t* ids, const int32_t* res_row, int n, int n_expert, int32_t* slot,
                                 int32_t* dst, int32_t* count, cudaStream_t s);
cudaError_t launch_s2_hits(const uint8_t* base, const int32_t* slot_index, const int32_t* dst_index,
                           const int32_t* d_count, int cap, int64_t blob_bytes, int H, int F, const uint8_t* xq,
                           const float* xs, int k_per_token, void* scratch, float* out, cudaStream_t s);
cudaError_t launch_s2_hit_add(float* parts, const float* hit_out, const int32_t* dst, const int32_t* count, int cap,
                              int64_t H, cudaStream_t s);

// ---- elementwise.cu ----
// x[r] = rms_norm(x[r] + residual[r]) * w (residual and w may be null): the host rule of rms_ref.
cudaError_t launch_add_rms_norm(float* x, const float* residual, const float* w, int64_t rows, int64_t cols,
                                float eps, cudaStream_t s);

// ---- decode.cu ---- (one token through one layer, or through a stack of layers, in one cooperative launch)
constexpr int kDecodeMaxLayers = 48;  // layers per launch (the table travels in the launch parameters)
struct DecodeHost {
    const smoe_layer* layers;     // n_layers layers of one geometry
    int n_layers;
    const float* const* norm_w;   // per-layer RMSNorm weights (null: unit)
    int norm;                     // 1: x = rms_norm(MoE(x) + x) after every layer; 0: one layer, out = MoE(x)
    float eps;
    const float* x;
    float* out;
    void* scratch;                // decode_scratch_bytes
    int32_t* ids;                 // single-layer trace (all may be null)
    float* w;
    float* sh_logit;
    uint8_t* xq;
    float* parts;
    float* shared_out;
};
bool decode_qualifies(int H, int F, int E, int k, int gu_type, int d_type, int has_shared, int sg, int su, int sd);
size_t decode_scratch_bytes(int H, int F, int E, int k);
// the router logits [E + 1] at the start of the scratch (the last one the shared gate)
cudaError_t launch_decode(const DecodeHost& h, cudaStream_t s);

// ---- ep.cu ---- (expert parallelism over peer memory)
size_t ep_arena_bytes(int H, int k, int max_tokens, int world);
// Route + q8_1 done; send every token's ids to every rank and its q8_1 row to each rank that owns one of its
// experts (and to this rank), then signal.
cudaError_t launch_ep_dispatch(void* arena, const int32_t* ids, const uint8_t* xq, int T, int k, int H,
                               int n_local, cudaStream_t s);
// Wait for every rank's dispatch, then the received rows' local ids (-1: not here) and their activation image:
// xa (the SIMT kernels' layout, q2 permuted when xa_q2) or xh (hi/lo, the tensor-core kernels).
cudaError_t launch_ep_receive(void* arena, int k, int H, int expert_first, int n_local, int32_t* oids,
                              const KAct* xa, int xa_q2, __half* xh, cudaStream_t s, int rows);
// Wait for every rank's down outputs of this rank's tokens.
cudaError_t launch_ep_wait_done(void* arena, cudaStream_t s);
float* const* ep_parts_table(void* arena);
unsigned* const* ep_done_table(void* arena);
unsigned* ep_done_counter(void* arena);
float* ep_parts(void* arena, int H, int k, int max_tokens, int world);
cudaError_t ep_init(void* arena, void* const* peers, int rank, int world, int H, int k, int max_tokens);

// ---- combine.cu ----
// out[t][j] = sum_i w[t][i] * parts[slot(t, i)][j] (+ shared[t][j] * sigmoid(gate_logit[t]) when shared)
// slot == nullptr means parts is [T][k][H] in router order; shared_scale == nullptr adds shared plain.
cudaError_t launch_combine(const float* parts, const int32_t* slot, const float* w, const float* shared,
                           const float* shared_logit, float* out, float* shared_out, int64_t H, int k, int T,
                           int64_t shared_stride, cudaStream_t s);
cudaError_t launch_gather_parts(const float* parts, const int32_t* slot, float* dst, int64_t H, int k, int T,
                                cudaStream_t s);

}  // namespace smoe
