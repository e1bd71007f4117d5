// api.cu - the C ABI (include/smoe.h): argument checks that mirror the reference's host API, scratch
// layout, and the MoE block's launch sequence.
#include "../../include/smoe.h"
#include "common.cuh"
#include "kernels.cuh"

#include <algorithm>
#include <atomic>
#include <cstring>
#include <string>

namespace smoe {
namespace {

thread_local std::string g_err;
thread_local cudaEvent_t* g_stage_events = nullptr;

cudaError_t mark(int stage, cudaStream_t s) {
    return g_stage_events ? cudaEventRecord(g_stage_events[stage], s) : cudaSuccess;
}

smoe_status fail(smoe_status s, const std::string& msg) {
    g_err = msg;
    return s;
}
smoe_status ok() {
    g_err.clear();
    return SMOE_OK;
}
smoe_status cuda_fail(cudaError_t e, const char* where) {
    return fail(SMOE_CUDA_ERROR, std::string(where) + ": " + cudaGetErrorString(e));
}

// Every block format of the reference's MMVQ family: Q2_0, IQ2_S, IQ4_NL, IQ4_XS, IQ3_XXS, IQ3_S (iqx.cu).
size_t row_bytes(int t, int64_t n) { return gx_row_bytes(t, n); }

// Layers with a routed or shared matrix outside Q2_0 / IQ2_S take the any-format path (iqx.cu).
bool any_format(const smoe_layer* L) {
    auto fast = [](int t) { return t == kQ2_0 || t == kIQ2_S; };
    return !fast(L->gu_type) || !fast(L->d_type) ||
           (L->has_shared && (!fast(L->sg_type) || !fast(L->su_type) || !fast(L->sd_type)));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

size_t up256(size_t n) { return (n + 255) & ~(size_t) 255; }

// Scratch regions of the block for T tokens.
struct Layout {
    size_t xq, xa, xa2, logits, sh_logit, ids, w, slot, slot_token, tables, sched, gu, ha, parts;
    size_t sched_tc, xh, hh;  // the tensor-core path (0 bytes when the layer does not qualify)
    size_t chunk;             // per-(64-token chunk, expert) counts of the many-CTA grouping
    size_t dec;               // the single-token fused kernel: logits, h, v and its grid barrier words
    size_t rsplit;            // fp64 partial sums of the few-token router GEMM
    size_t hq;                // q8_1 blocks of h per slot (the any-format path)
    size_t total;
};

// Expert path: 0 automatic (the fused single-token kernel at one token, tensor cores from kTcAutoTokens tokens
// on, the SIMT kernels between), 1 the SIMT kernels, 2 tensor cores whenever the layer qualifies, 3 the fused
// single-token kernel whenever the batch is one token and the layer qualifies.
std::atomic<int> g_expert_path{0};
constexpr int kTcAutoTokens = 512;

// The tensor-core kernels take Q2_0 everywhere and rows whose byte length is a multiple of 16 (TMA strides):
// n_embd and n_ff multiples of 512.
bool tc_qualifies(const smoe_layer* L) {
    const bool q2 = L->gu_type == kQ2_0 && L->d_type == kQ2_0 &&
                    (!L->has_shared || (L->sg_type == kQ2_0 && L->su_type == kQ2_0 && L->sd_type == kQ2_0));
    return q2 && L->n_embd % 512 == 0 && L->n_ff % 512 == 0;
}

bool use_decode(const smoe_layer* L, int T) {
    const int p = g_expert_path.load(std::memory_order_relaxed);
    return T == 1 && (p == 0 || p == 3) &&
           decode_qualifies(L->n_embd, L->n_ff, L->n_expert, L->k, L->gu_type, L->d_type, L->has_shared, L->sg_type,
                            L->su_type, L->sd_type);
}

bool use_tc(const smoe_layer* L, int T) {
    const int p = g_expert_path.load(std::memory_order_relaxed);
    if (p == 1 || p == 3 || p == 4 || !tc_qualifies(L)) return false;
    return p == 2 || T >= kTcAutoTokens;
}

// The int8 tensor-core kernels of the integer contract take Q2_0 everywhere and n_embd, n_ff in {512, 1024, 2048}.
bool tq_layer(const smoe_layer* L) {
    const bool q2 = L->gu_type == kQ2_0 && L->d_type == kQ2_0 &&
                    (!L->has_shared || (L->sg_type == kQ2_0 && L->su_type == kQ2_0 && L->sd_type == kQ2_0));
    return q2 && tq_qualifies(L->n_embd, L->n_ff);
}

// Below the tensor-core (fp16) range: the int8 tensor-core kernels unless the SIMT kernels are asked for.
bool use_tq(const smoe_layer* L, int T) {
    const int p = g_expert_path.load(std::memory_order_relaxed);
    if (p == 1 || p == 2 || !tq_layer(L)) return false;
    return p == 4 || (p == 0 && T < kTcAutoTokens) || p == 3;
}

Layout layout_of(const smoe_layer* L, int T) {
    Layout o;
    const size_t H = (size_t) L->n_embd, F = (size_t) L->n_ff, E = (size_t) L->n_expert, K = (size_t) L->k;
    const size_t rows = (size_t) T * K + (L->has_shared ? (size_t) T : 0);
    size_t at = 0;
    o.xq = at; at += up256((size_t) T * (H / 32) * kQ8Block);
    o.xa = at; at += up256(ka_bytes(T, (int) (H / 32)));
    o.xa2 = at; at += up256(ka_bytes(T, (int) (H / 32)));
    o.logits = at; at += up256((size_t) T * E * 4);
    o.sh_logit = at; at += up256((size_t) T * 4);
    o.ids = at; at += up256((size_t) T * K * 4);
    o.w = at; at += up256((size_t) T * K * 4);
    o.slot = at; at += up256((size_t) T * K * 4);
    o.slot_token = at; at += up256((size_t) T * K * 4);
    o.tables = at; at += group_tables_bytes((int) E);
    o.sched = at; at += sched_bytes((int) E, T, (int) K);
    o.gu = at; at += up256(rows * 2 * F * 4);
    o.ha = at; at += up256(ka_bytes((int64_t) rows, (int) (F / 32)));
    o.parts = at; at += up256(rows * H * 4);
    o.chunk = at; at += group_chunk_bytes(T, (int) E);
    o.dec = at; at += up256(decode_scratch_bytes((int) H, (int) F, (int) E, (int) K));
    o.rsplit = at; at += router_split_bytes(std::min(T, kRouterGemmMinTokens), (int) E + 1, (int) H);
    o.sched_tc = o.xh = o.hh = at;
    if (tc_qualifies(L)) {
        o.sched_tc = at; at += sched_bytes((int) E, T, (int) K, kTcChunk);
        o.xh = at; at += up256((size_t) 2 * T * H * 2);
        o.hh = at; at += up256(rows * 2 * F * 2);
    }
    o.hq = at;
    if (any_format(L)) at += up256(rows * (F / 32) * kQ8Block);
    o.total = at;
    return o;
}

smoe_status check_layer(const smoe_layer* L) {
    if (!L) return fail(SMOE_INVALID_ARG, "layer is null");
    if (L->n_embd <= 0 || L->n_ff <= 0 || L->n_expert <= 0 || L->k <= 0)
        return fail(SMOE_INVALID_ARG, "layer: sizes must be positive");
    if (L->k > kMaxK) return fail(SMOE_INVALID_ARG, "layer: k exceeds 64");
    if (L->n_expert > kMaxExperts) return fail(SMOE_INVALID_ARG, "layer: n_expert exceeds 1024");
    if (L->k > L->n_expert) return fail(SMOE_INVALID_ARG, "layer: k exceeds n_expert");
    if (!row_bytes(L->gu_type, L->n_embd) || !row_bytes(L->d_type, L->n_ff))
        return fail(SMOE_UNSUPPORTED, "layer: routed types must be Q2_0, IQ2_S, IQ4_NL, IQ4_XS, IQ3_XXS or IQ3_S "
                                      "with whole blocks per row");
    if (L->n_ff % 32 || L->n_embd % 64) return fail(SMOE_INVALID_ARG, "layer: n_ff % 32 and n_embd % 64 must be 0");
    if (L->n_embd > 4096 || L->n_ff > 4096) return fail(SMOE_UNSUPPORTED, "layer: n_embd and n_ff are at most 4096");
    if (!L->router || !L->gate || !L->up || !L->down) return fail(SMOE_INVALID_ARG, "layer: a routed plane is null");
    if (!aligned(L->router, 16) || !aligned(L->gate, 16) || !aligned(L->up, 16) || !aligned(L->down, 16))
        return fail(SMOE_INVALID_ARG, "layer: planes must be 16-byte aligned");
    if (L->has_shared) {
        if (!row_bytes(L->sg_type, L->n_embd) || !row_bytes(L->su_type, L->n_embd) || !row_bytes(L->sd_type, L->n_ff))
            return fail(SMOE_UNSUPPORTED, "layer: shared types must be Q2_0, IQ2_S, IQ4_NL, IQ4_XS, IQ3_XXS or IQ3_S "
                                          "with whole blocks per row");
        if (L->sg_type != L->su_type) return fail(SMOE_UNSUPPORTED, "layer: shared gate and up types differ");
        if (!L->sgate || !L->sup || !L->sdown || !L->gate_inp_shexp)
            return fail(SMOE_INVALID_ARG, "layer: a shared plane is null");
        if (!aligned(L->sgate, 16) || !aligned(L->sup, 16) || !aligned(L->sdown, 16) ||
            !aligned(L->gate_inp_shexp, 16))
            return fail(SMOE_INVALID_ARG, "layer: shared planes must be 16-byte aligned");
    }
    return SMOE_OK;
}

// Local scratch of the expert-parallel block: this rank's tokens (T = max_tokens) on the router side, the
// received rows (R = world * max_tokens) and this rank's n_local experts on the expert side.
struct EpLayout {
    size_t xq, logits, sh_logit, ids, w, shared, rsplit;                               // token side
    size_t oids, slot, slot_token, slot_pair, tables, sched, chunk, xa, gu, ha;        // expert side, SIMT
    size_t sched_tc, xh, hh;                                                           // tensor cores
    size_t total;
};

EpLayout ep_layout_of(const smoe_layer* L, const smoe_ep* ep) {
    EpLayout o;
    const size_t H = (size_t) L->n_embd, F = (size_t) L->n_ff, K = (size_t) L->k;
    const int T = ep->max_tokens, R = ep->world * ep->max_tokens, El = L->n_expert / ep->world;
    const size_t rows = (size_t) R * K + (L->has_shared ? (size_t) T : 0);
    size_t at = 0;
    o.xq = at; at += up256((size_t) T * (H / 32) * kQ8Block);
    o.logits = at; at += up256((size_t) T * L->n_expert * 4);
    o.sh_logit = at; at += up256((size_t) T * 4);
    o.ids = at; at += up256((size_t) T * K * 4);
    o.w = at; at += up256((size_t) T * K * 4);
    o.shared = at; at += up256((size_t) T * H * 4);
    o.rsplit = at; at += router_split_bytes(std::min(T, kRouterGemmMinTokens), L->n_expert + 1, (int) H);
    o.oids = at; at += up256((size_t) R * K * 4);
    o.slot = at; at += up256((size_t) R * K * 4);
    o.slot_token = at; at += up256((size_t) R * K * 4);
    o.slot_pair = at; at += up256((size_t) R * K * 4);
    o.tables = at; at += group_tables_bytes(El);
    o.sched = at; at += sched_bytes(El, R, (int) K);
    o.chunk = at; at += group_chunk_bytes(R, El);
    o.xa = at; at += up256(ka_bytes(R, (int) (H / 32)));
    o.gu = at; at += up256(rows * 2 * F * 4);
    o.ha = at; at += up256(ka_bytes((int64_t) rows, (int) (F / 32)));
    o.sched_tc = o.xh = o.hh = at;
    if (tc_qualifies(L)) {
        o.sched_tc = at; at += sched_bytes(El, R, (int) K, kTcChunk);
        o.xh = at; at += up256((size_t) 2 * R * H * 2);
        o.hh = at; at += up256(rows * 2 * F * 2);
    }
    o.total = at;
    return o;
}

smoe_status check_ep(const smoe_layer* L, const smoe_ep* ep) {
    smoe_status st = check_layer(L);
    if (st != SMOE_OK) return st;
    if (!ep) return fail(SMOE_INVALID_ARG, "ep: descriptor is null");
    if (ep->world < 1 || ep->world > SMOE_EP_MAX_WORLD || ep->rank < 0 || ep->rank >= ep->world)
        return fail(SMOE_INVALID_ARG, "ep: need 1 <= world <= 8 and 0 <= rank < world");
    if (ep->max_tokens < 1) return fail(SMOE_INVALID_ARG, "ep: max_tokens must be positive");
    if (L->n_expert % ep->world) return fail(SMOE_INVALID_ARG, "ep: n_expert must be a multiple of world");
    if (L->n_expert / ep->world < 1) return fail(SMOE_INVALID_ARG, "ep: no experts per rank");
    if (L->n_embd % 128) return fail(SMOE_UNSUPPORTED, "ep: n_embd must be a multiple of 128");
    if (L->has_shared && (L->sg_type != L->gu_type || L->su_type != L->gu_type || L->sd_type != L->d_type))
        return fail(SMOE_UNSUPPORTED, "ep: the shared expert's types must equal the routed ones");
    if (any_format(L)) return fail(SMOE_UNSUPPORTED, "ep: expert parallelism takes Q2_0 and IQ2_S layers");
    for (int p = 0; p < ep->world; p++)
        if (!ep->areas[p] || !aligned(ep->areas[p], 256)) return fail(SMOE_INVALID_ARG, "ep: an area is null or unaligned");
    return SMOE_OK;
}

}  // namespace
}  // namespace smoe

using namespace smoe;

extern "C" {

const char* smoe_last_error(void) { return g_err.c_str(); }

smoe_status smoe_set_expert_path(int path) {
    if (path < 0 || path > 4) return fail(SMOE_INVALID_ARG, "set_expert_path: path must be 0, 1, 2, 3 or 4");
    g_expert_path.store(path);
    return ok();
}

int smoe_expert_path_for(const smoe_layer* L, int n_tokens) {
    if (check_layer(L) != SMOE_OK || n_tokens <= 0) return -1;
    if (any_format(L)) return 5;
    return use_decode(L, n_tokens) ? 3 : use_tc(L, n_tokens) ? 2 : use_tq(L, n_tokens) ? 4 : 1;
}

void smoe_set_stage_events(void** events, int n) {
    g_stage_events = (events && n >= SMOE_STAGES) ? reinterpret_cast<cudaEvent_t*>(events) : nullptr;
}

unsigned smoe_device_status(int clear) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_smoe_status, sizeof v) != cudaSuccess) return 0xFFFFFFFFu;
    if (clear) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_smoe_status, &z, sizeof z);
    }
    return v;
}

size_t smoe_row_bytes(int ggml_type, int64_t n) { return row_bytes(ggml_type, n); }

size_t smoe_q8_1_bytes(int64_t n) { return (n <= 0 || n % 32) ? 0 : (size_t) (n / 32) * kQ8Block; }

smoe_status smoe_f32_to_bf16_bulk(const float* x, uint16_t* y, int64_t n, void* stream) {
    if (n < 0) return fail(SMOE_INVALID_ARG, "f32_to_bf16_bulk: negative size");
    if (n == 0) return ok();
    if (!stream) return fail(SMOE_INVALID_ARG, "f32_to_bf16_bulk: a non-null stream is required");
    if (!x || !y) return fail(SMOE_INVALID_ARG, "f32_to_bf16_bulk: null buffer");
    const cudaError_t e = launch_f32_to_bf16(x, y, n, (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "f32_to_bf16_bulk");
}

smoe_status smoe_bf16_gemv(const uint16_t* x, const uint16_t* w, float* y, int64_t n_in, int64_t n_out,
                           int64_t n_col, void* stream) {
    // bf16_gemv.mm:195-200: non-positive sizes return without a launch; sizes past int32 throw
    if (n_in <= 0 || n_out <= 0 || n_col <= 0) return ok();
    if (n_in > 0x7fffffff || n_out > 0x7fffffff || n_col > 0x7fffffff)
        return fail(SMOE_INVALID_ARG, "bf16_gemv: dimension does not fit in int32");
    if (n_in % 8) return fail(SMOE_INVALID_ARG, "bf16_gemv: n_in must be a multiple of 8");
    if (n_in > 16384) return fail(SMOE_UNSUPPORTED, "bf16_gemv: n_in is at most 16384");
    if (!stream) return fail(SMOE_INVALID_ARG, "bf16_gemv: a non-null stream is required");
    if (!x || !w || !y || !aligned(x, 16) || !aligned(w, 16))
        return fail(SMOE_INVALID_ARG, "bf16_gemv: x and w must be non-null and 16-byte aligned");
    const cudaError_t e = launch_bf16_gemv(x, false, w, nullptr, y, nullptr, (int) n_col, (int) n_in, (int) n_out,
                                           (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "bf16_gemv");
}

static smoe_status check_router_args(int n_tokens, int n_expert, int k, bool* noop) {
    // router.mm:32-37
    *noop = false;
    if (n_tokens < 0 || n_expert < 0 || k < 0) return fail(SMOE_INVALID_ARG, "router_top10: negative size");
    if (n_tokens == 0 || n_expert == 0 || k == 0) {
        *noop = true;
        return ok();
    }
    if (k > kMaxK) return fail(SMOE_INVALID_ARG, "router_top10: k exceeds 64");
    if (n_expert > kMaxExperts) return fail(SMOE_INVALID_ARG, "router_top10: n_expert exceeds 1024");
    if (k > n_expert) return fail(SMOE_INVALID_ARG, "router_top10: k exceeds n_expert");
    return ok();
}

smoe_status smoe_router_top10(const float* logits, int n_tokens, int n_expert, int k, int32_t* ids, float* weights,
                              void* stream) {
    bool noop;
    const smoe_status st = check_router_args(n_tokens, n_expert, k, &noop);
    if (st != SMOE_OK || noop) return st;
    if (!stream) return fail(SMOE_INVALID_ARG, "router_top10: a non-null stream is required");
    if (!logits || !ids || !weights) return fail(SMOE_INVALID_ARG, "router_top10: null buffer");
    const cudaError_t e = launch_router_topk(logits, n_tokens, n_expert, k, ids, weights, nullptr, nullptr, 0,
                                             (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "router_top10");
}

smoe_status smoe_router(const float* x, const uint16_t* w_router, int n_tokens, int n_embd, int n_expert, int k,
                        float* logits, int32_t* ids, float* weights, void* stream) {
    bool noop;
    smoe_status st = check_router_args(n_tokens, n_expert, k, &noop);
    if (st != SMOE_OK || noop) return st;
    if (n_embd <= 0 || n_embd % 8 || n_embd > 16384)
        return fail(SMOE_INVALID_ARG, "router: n_embd must be a positive multiple of 8, at most 16384");
    if (!stream) return fail(SMOE_INVALID_ARG, "router: a non-null stream is required");
    if (!x || !w_router || !logits || !ids || !weights || !aligned(w_router, 16) || !aligned(x, 16))
        return fail(SMOE_INVALID_ARG, "router: null buffer, or x / w_router not 16-byte aligned");
    cudaError_t e = launch_bf16_gemv(x, true, w_router, nullptr, logits, nullptr, n_tokens, n_embd, n_expert,
                                     (cudaStream_t) stream);
    if (e != cudaSuccess) return cuda_fail(e, "router");
    e = launch_router_topk(logits, n_tokens, n_expert, k, ids, weights, nullptr, nullptr, 0, (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "router");
}

smoe_status smoe_iq_quantize_q8_1(const float* x, int64_t n, uint8_t* y, void* stream) {
    // iq.mm:138-141: n <= 0 returns; a partial block throws
    if (n <= 0) return ok();
    if (n % 32) return fail(SMOE_INVALID_ARG, "iq_quantize_q8_1: length must be a multiple of 32");
    if (!stream) return fail(SMOE_INVALID_ARG, "iq_quantize_q8_1: a non-null stream is required");
    if (!x || !y) return fail(SMOE_INVALID_ARG, "iq_quantize_q8_1: null buffer");
    const cudaError_t e = launch_quant_q8_1(x, n, y, (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "iq_quantize_q8_1");
}

smoe_status smoe_iq_mmvq(int ggml_type, const uint8_t* w, const uint8_t* x_q8, int64_t n_in, int64_t n_out,
                         int64_t n_col, float* y, void* stream) {
    // iq.mm:150-158
    if (n_in == 0 || n_out == 0 || n_col == 0) return ok();
    if (n_in < 0 || n_out < 0 || n_col < 0) return fail(SMOE_INVALID_ARG, "iq_mmvq: negative size");
    if (!gx_type_ok(ggml_type))
        return fail(SMOE_UNSUPPORTED, "iq_mmvq: type is not Q2_0, IQ2_S, IQ4_NL, IQ4_XS, IQ3_XXS or IQ3_S");
    if (!row_bytes(ggml_type, n_in)) return fail(SMOE_INVALID_ARG, "iq_mmvq: n_in is not a whole number of blocks");
    if (n_in > 4096) return fail(SMOE_UNSUPPORTED, "iq_mmvq: n_in is at most 4096");
    if (n_out > 0x7fffffff || n_col > 0x7fffffff) return fail(SMOE_INVALID_ARG, "iq_mmvq: size does not fit in int");
    if (!stream) return fail(SMOE_INVALID_ARG, "iq_mmvq: a non-null stream is required");
    if (!w || !x_q8 || !y || !aligned(w, 16) || !aligned(x_q8, 4))
        return fail(SMOE_INVALID_ARG, "iq_mmvq: w must be 16-byte and x 4-byte aligned");
    if (ggml_type != kQ2_0 && ggml_type != kIQ2_S) {  // iqx.cu
        const cudaError_t e = launch_gx_mmvq(ggml_type, w, x_q8, (int) n_in, (int) n_out, (int) n_col, y,
                                             (cudaStream_t) stream);
        return e == cudaSuccess ? ok() : cuda_fail(e, "iq_mmvq");
    }
    GroupView g{};
    g.single_cols = (int) n_col;
    const Matrix m{w, 0, ggml_type};
    const cudaError_t e = launch_expert_down(m, m, g, x_q8, 0, y, n_out, (int) n_in, (int) n_out,
                                             (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "iq_mmvq");
}

smoe_status smoe_iq_swiglu_q8(const float* gate, const float* up, int64_t n, uint8_t* y, void* stream) {
    // iq.mm:201-203
    if (n == 0) return ok();
    if (n < 0 || n % 32) return fail(SMOE_INVALID_ARG, "iq_swiglu_q8: length must be a positive multiple of 32");
    if (!stream) return fail(SMOE_INVALID_ARG, "iq_swiglu_q8: a non-null stream is required");
    if (!gate || !up || !y) return fail(SMOE_INVALID_ARG, "iq_swiglu_q8: null buffer");
    const cudaError_t e = launch_swiglu_q8(gate, up, n, y, (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "iq_swiglu_q8");
}

smoe_status smoe_moe_combine(const float* parts, const float* weights, const float* shared, float* y,
                             int64_t n_embd, int k, int n_tok, void* stream) {
    // moe_combine.mm:31-34
    if (n_embd < 0 || k < 0 || n_tok < 0) return fail(SMOE_INVALID_ARG, "moe_combine: negative size");
    if (n_embd == 0 || k == 0 || n_tok == 0) return ok();
    if (k > kMaxK) return fail(SMOE_INVALID_ARG, "moe_combine: k exceeds 64");
    if (!stream) return fail(SMOE_INVALID_ARG, "moe_combine: a non-null stream is required");
    if (!parts || !weights || !y) return fail(SMOE_INVALID_ARG, "moe_combine: null buffer");
    const cudaError_t e = launch_combine(parts, nullptr, weights, shared, nullptr, y, nullptr, n_embd, k, n_tok,
                                         n_embd, (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "moe_combine");
}

size_t smoe_moe_group_scratch_bytes(int n_tok, int k, int n_expert) {
    (void) n_tok;
    (void) k;
    return (n_expert > 0 && n_expert <= kMaxExperts) ? group_tables_bytes(n_expert) : 0;
}

smoe_status smoe_moe_group(const int32_t* ids, int n_tok, int k, int n_expert, void* scratch, int32_t* slot,
                           int32_t* src, void* stream) {
    if (n_tok < 0 || k < 0 || n_expert < 0) return fail(SMOE_INVALID_ARG, "moe_group: negative size");
    if (n_tok == 0 || k == 0 || n_expert == 0) return ok();
    if (k > kMaxK || n_expert > kMaxExperts) return fail(SMOE_INVALID_ARG, "moe_group: k > 64 or n_expert > 1024");
    if (!stream) return fail(SMOE_INVALID_ARG, "moe_group: a non-null stream is required");
    if (!ids || !scratch || !slot || !aligned(scratch, 4)) return fail(SMOE_INVALID_ARG, "moe_group: null buffer");
    const cudaError_t e = launch_group(ids, n_tok, k, n_expert, group_tables_at(scratch, n_expert), slot, src,
                                       (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "moe_group");
}

smoe_status smoe_rms_norm_weighted(float* x, const float* w, int64_t rows, int64_t cols, float eps, void* stream) {
    return smoe_add_rms_norm(x, nullptr, w, rows, cols, eps, stream);
}

smoe_status smoe_add_rms_norm(float* x, const float* residual, const float* w, int64_t rows, int64_t cols, float eps,
                              void* stream) {
    if (rows < 0 || cols < 0) return fail(SMOE_INVALID_ARG, "rms_norm: negative size");
    if (rows == 0 || cols == 0) return ok();
    if (!(eps >= 0.f)) return fail(SMOE_INVALID_ARG, "rms_norm: eps must be >= 0");
    if (!stream) return fail(SMOE_INVALID_ARG, "rms_norm: a non-null stream is required");
    if (!x) return fail(SMOE_INVALID_ARG, "rms_norm: null buffer");
    const cudaError_t e = launch_add_rms_norm(x, residual, w, rows, cols, eps, (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "rms_norm");
}

smoe_status smoe_layer_check(const smoe_layer* L) {
    const smoe_status st = check_layer(L);
    return st == SMOE_OK ? ok() : st;
}

size_t smoe_moe_scratch_bytes(const smoe_layer* L, int max_tokens) {
    if (check_layer(L) != SMOE_OK || max_tokens < 0) return 0;
    return layout_of(L, max_tokens).total;
}

smoe_status smoe_moe_forward(const smoe_layer* L, const float* x, int n_tokens, float* out, void* scratch,
                             size_t scratch_bytes, const smoe_trace* trace, void* stream) {
    smoe_status st = check_layer(L);
    if (st != SMOE_OK) return st;
    if (n_tokens < 0) return fail(SMOE_INVALID_ARG, "moe_forward: negative token count");
    if (n_tokens == 0) return ok();
    if (!stream) return fail(SMOE_INVALID_ARG, "moe_forward: a non-null stream is required");
    if (!x || !out || !scratch || !aligned(scratch, 256) || !aligned(x, 16))
        return fail(SMOE_INVALID_ARG, "moe_forward: null buffer, x not 16-byte or scratch not 256-byte aligned");
    const Layout lo = layout_of(L, n_tokens);
    if (scratch_bytes < lo.total) return fail(SMOE_INVALID_ARG, "moe_forward: scratch is too small");
    cudaStream_t s = (cudaStream_t) stream;
    uint8_t* base = static_cast<uint8_t*>(scratch);
    const int T = n_tokens, H = L->n_embd, F = L->n_ff, E = L->n_expert, K = L->k;
    uint8_t* xq = base + lo.xq;
    float* logits = reinterpret_cast<float*>(base + lo.logits);
    float* sh_logit = reinterpret_cast<float*>(base + lo.sh_logit);
    int32_t* ids = reinterpret_cast<int32_t*>(base + lo.ids);
    float* w = reinterpret_cast<float*>(base + lo.w);
    int32_t* slot = reinterpret_cast<int32_t*>(base + lo.slot);
    int32_t* slot_tok = reinterpret_cast<int32_t*>(base + lo.slot_token);
    const GroupTables tabs = group_tables_at(base + lo.tables, E);
    const Sched sc = sched_at(base + lo.sched, E, T, K);
    const bool sh = L->has_shared != 0;
    const int rows = T * K + (sh ? T : 0);
    const KAct xa = ka_at(base + lo.xa, T, H / 32);
    const KAct xa2 = ka_at(base + lo.xa2, T, H / 32);
    const KAct ha = ka_at(base + lo.ha, rows, F / 32);
    float* gu = reinterpret_cast<float*>(base + lo.gu);
    float* parts = reinterpret_cast<float*>(base + lo.parts);

    if (use_decode(L, T)) {
        // one token: the whole block in one cooperative launch
        DecodeHost dh{};
        dh.layers = L;
        dh.n_layers = 1;
        dh.norm = 0;
        dh.x = x;
        dh.out = out;
        dh.scratch = base + lo.dec;
        if (trace) {
            dh.ids = trace->ids;
            dh.w = trace->weights;
            dh.xq = trace->xq;
            dh.parts = trace->parts;
            dh.shared_out = trace->shared;
        }
        cudaError_t e = launch_decode(dh, s);
        for (int st = 0; st < SMOE_STAGES && e == cudaSuccess; st++) e = mark(st, s);
        if (e != cudaSuccess) return cuda_fail(e, "moe_forward: fused single-token kernel");
        if (trace && trace->logits)
            e = cudaMemcpyAsync(trace->logits, base + lo.dec, (size_t) E * 4, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return cuda_fail(e, "moe_forward: trace");
        return ok();
    }

    // 2 to 64 tokens: the split-K router GEMM's partials are added by the top-k launch (two launches, not three)
    int splits = 0;
    cudaError_t e = launch_bf16_gemv(x, true, L->router, sh ? L->gate_inp_shexp : nullptr, logits, sh_logit, T, H,
                                     E, s, base + lo.rsplit, &splits);
    const RouterSplit rsplit{reinterpret_cast<const double*>(base + lo.rsplit), splits, logits, sh ? sh_logit : nullptr};
    if (e == cudaSuccess) e = mark(0, s);
    if (e != cudaSuccess) return cuda_fail(e, "moe_forward: router");
    if (any_format(L)) {
        // any block format (iqx.cu): the q8_1 blocks of x, grouping, gate/up rows, SwiGLU + q8_1 of h, down rows;
        // the shared expert in launches of its own (its types may differ from the routed ones)
        e = launch_router_topk(logits, T, E, K, ids, w, x, xq, H, s, nullptr, 0, &rsplit);
        if (e == cudaSuccess) e = mark(1, s);
        if (e != cudaSuccess) return cuda_fail(e, "moe_forward: top-k");
        e = launch_group(ids, T, K, E, tabs, slot, slot_tok, s, &sc, reinterpret_cast<int32_t*>(base + lo.chunk));
        if (e == cudaSuccess) e = mark(2, s);
        if (e != cudaSuccess) return cuda_fail(e, "moe_forward: dispatch");
        Work wk{};
        wk.sched = sc;
        wk.slot_token = slot_tok;
        wk.max_entries = sched_capacity(E, T, K);
        wk.shared_base = T * K;
        wk.shared_slots = sh ? T : 0;
        const int64_t gu_stride = (int64_t) F * (int64_t) row_bytes(L->gu_type, H);
        const int64_t d_stride = (int64_t) H * (int64_t) row_bytes(L->d_type, F);
        uint8_t* hq = base + lo.hq;
        e = launch_gx_gate_up(Matrix{L->gate, gu_stride, L->gu_type}, Matrix{L->up, gu_stride, L->gu_type}, wk, 0, xq,
                              gu, H, F, s);
        if (e == cudaSuccess && sh)
            e = launch_gx_gate_up(Matrix{L->sgate, 0, L->sg_type}, Matrix{L->sup, 0, L->su_type}, wk, 1, xq, gu, H, F, s);
        if (e == cudaSuccess) e = launch_gx_swiglu(gu, hq, rows, F, s);
        if (e == cudaSuccess) e = mark(3, s);
        if (e != cudaSuccess) return cuda_fail(e, "moe_forward: gate/up (any format)");
        e = launch_gx_down(Matrix{L->down, d_stride, L->d_type}, wk, 0, hq, parts, F, H, s);
        if (e == cudaSuccess && sh) e = launch_gx_down(Matrix{L->sdown, 0, L->sd_type}, wk, 1, hq, parts, F, H, s);
        if (e == cudaSuccess) e = mark(4, s);
        if (e != cudaSuccess) return cuda_fail(e, "moe_forward: down (any format)");
    } else {
    const bool tc = use_tc(L, T);
    // the q8_1 image of x in the reference's block format is only an output of the trace: the expert kernels
    // read their own layouts (xa for the SIMT kernels, xh for the tensor-core kernels)
    const bool want_xq = trace && trace->xq;
    e = launch_router_topk(logits, T, E, K, ids, w, x, want_xq ? xq : nullptr, H, s, tc ? nullptr : &xa,
                           L->gu_type == kQ2_0, &rsplit);
    __half* xh = reinterpret_cast<__half*>(base + lo.xh);
    if (e == cudaSuccess && tc) e = launch_quant_xh(x, T, H, xh, s);
    if (e == cudaSuccess) e = mark(1, s);
    if (e != cudaSuccess) return cuda_fail(e, "moe_forward: top-k");
    const Sched sct = tc ? sched_at(base + lo.sched_tc, E, T, K, kTcChunk) : sc;
    e = launch_group(ids, T, K, E, tabs, slot, slot_tok, s, &sct, reinterpret_cast<int32_t*>(base + lo.chunk));
    if (e == cudaSuccess) e = mark(2, s);
    if (e != cudaSuccess) return cuda_fail(e, "moe_forward: dispatch");

    Work wk{};
    wk.sched = sc;
    wk.slot_token = slot_tok;
    wk.max_entries = sched_capacity(E, T, K);
    wk.shared_base = T * K;
    const int64_t gu_stride = (int64_t) F * (int64_t) row_bytes(L->gu_type, H);
    const int64_t d_stride = (int64_t) H * (int64_t) row_bytes(L->d_type, F);
    const Matrix mg{L->gate, gu_stride, L->gu_type}, mu{L->up, gu_stride, L->gu_type}, md{L->down, d_stride, L->d_type};
    const Matrix sg{L->sgate, 0, L->sg_type}, su{L->sup, 0, L->su_type}, sd{L->sdown, 0, L->sd_type};

    if (tc) {
        // tensor-core path: every matrix is Q2_0, so the shared expert rides in the routed launches
        __half* hh = reinterpret_cast<__half*>(base + lo.hh);
        Work wt = wk;
        wt.sched = sct;
        wt.max_entries = sched_capacity(E, T, K, kTcChunk);
        wt.shared_slots = sh ? T : 0;
        e = launch_tc_gate_up(mg, mu, sg, su, wt, E, xh, T, hh, rows, H, F, s);
        if (e == cudaSuccess) e = mark(3, s);
        if (e != cudaSuccess) return cuda_fail(e, "moe_forward: gate/up (tensor cores)");
        e = launch_tc_down(md, sd, wt, E, hh, rows, parts, F, H, s);
        if (e == cudaSuccess) e = mark(4, s);
        if (e != cudaSuccess) return cuda_fail(e, "moe_forward: down (tensor cores)");
    } else if (use_tq(L, T)) {
        // int8 tensor cores (the q8_1 contract bit for bit): every matrix is Q2_0, the shared expert rides along
        Work wq = wk;
        wq.shared_slots = sh ? T : 0;
        e = launch_tq_gate_up(mg, mu, sg, su, wq, E, xa, ha, 1, H, F, s);
        if (e == cudaSuccess) e = mark(3, s);
        if (e != cudaSuccess) return cuda_fail(e, "moe_forward: gate/up (int8 tensor cores)");
        e = launch_tq_down(md, sd, wq, E, ha, parts, F, H, s);
        if (e == cudaSuccess) e = mark(4, s);
        if (e != cudaSuccess) return cuda_fail(e, "moe_forward: down (int8 tensor cores)");
    } else {
    // The shared expert rides in the routed launches when its types match; otherwise it gets its own.
    const bool gu_same = sh && L->sg_type == L->gu_type && L->su_type == L->gu_type;
    const bool d_same = sh && L->sd_type == L->d_type;
    Work w1 = wk;
    w1.shared_slots = gu_same ? T : 0;
    w1.counter = tabs.work + 0;
    e = launch_layer_gate_up(mg, mu, sg, su, w1, xa, gu, H, F, s);
    if (e != cudaSuccess) return cuda_fail(e, "moe_forward: gate/up");
    if (sh && !gu_same) {
        const bool same_layout = (L->sg_type == kQ2_0) == (L->gu_type == kQ2_0);
        if (!same_layout) {
            e = launch_quant_ka(x, T, H, xa2, L->sg_type == kQ2_0, s);
            if (e != cudaSuccess) return cuda_fail(e, "moe_forward: shared activation");
        }
        Work w2 = wk;
        w2.no_routed = 1;
        w2.shared_slots = T;
        w2.counter = tabs.work + 1;
        e = launch_layer_gate_up(sg, su, sg, su, w2, same_layout ? xa : xa2, gu, H, F, s);
        if (e != cudaSuccess) return cuda_fail(e, "moe_forward: shared gate/up");
    }
    // SwiGLU + q8_1 of h, each slot in its down matrix's activation layout
    const int routed_rows = T * K;
    e = launch_swiglu_ka(gu, ha, sh && L->sd_type == L->d_type ? rows : routed_rows, F, L->d_type == kQ2_0, s);
    if (e == cudaSuccess && sh && L->sd_type != L->d_type)
        e = launch_swiglu_ka(gu + (int64_t) routed_rows * 2 * F, KAct{ha.base + ka_bytes(routed_rows, F / 32)}, T, F,
                             L->sd_type == kQ2_0, s);
    if (e != cudaSuccess) return cuda_fail(e, "moe_forward: swiglu");
    e = mark(3, s);
    if (e != cudaSuccess) return cuda_fail(e, "moe_forward: stage event");
    Work w3 = wk;
    w3.shared_slots = d_same ? T : 0;
    w3.counter = tabs.work + 2;
    e = launch_layer_down(md, sd, w3, ha, parts, F, H, s);
    if (e != cudaSuccess) return cuda_fail(e, "moe_forward: down");
    if (sh && !d_same) {
        Work w4 = wk;
        w4.no_routed = 1;
        w4.shared_slots = T;
        w4.counter = tabs.work + 3;
        e = launch_layer_down(sd, sd, w4, ha, parts, F, H, s);
        if (e != cudaSuccess) return cuda_fail(e, "moe_forward: shared down");
    }
    e = mark(4, s);
    if (e != cudaSuccess) return cuda_fail(e, "moe_forward: stage event");
    }
    }
    e = launch_combine(parts, slot, w, sh ? parts + (int64_t) T * K * H : nullptr, sh ? sh_logit : nullptr, out,
                       trace ? trace->shared : nullptr, H, K, T, H, s);
    if (e == cudaSuccess) e = mark(5, s);
    if (e != cudaSuccess) return cuda_fail(e, "moe_forward: combine");

    if (trace) {
        if (trace->logits) e = cudaMemcpyAsync(trace->logits, logits, (size_t) T * E * 4, cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess && trace->ids)
            e = cudaMemcpyAsync(trace->ids, ids, (size_t) T * K * 4, cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess && trace->weights)
            e = cudaMemcpyAsync(trace->weights, w, (size_t) T * K * 4, cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess && trace->xq)
            e = cudaMemcpyAsync(trace->xq, xq, (size_t) T * (H / 32) * kQ8Block, cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess && trace->parts) e = launch_gather_parts(parts, slot, trace->parts, H, K, T, s);
        if (e != cudaSuccess) return cuda_fail(e, "moe_forward: trace");
    }
    return ok();
}

// ---- the batch-1 layer stack in one launch -------------------------------------------------------------------
static smoe_status check_stack(const smoe_layer* layers, int n_layers) {
    if (!layers || n_layers < 1) return fail(SMOE_INVALID_ARG, "stack_decode: no layers");
    const smoe_layer& L0 = layers[0];
    for (int l = 0; l < n_layers; l++) {
        const smoe_status st = check_layer(&layers[l]);
        if (st != SMOE_OK) return st;
        const smoe_layer& L = layers[l];
        if (L.n_embd != L0.n_embd || L.n_ff != L0.n_ff || L.n_expert != L0.n_expert || L.k != L0.k ||
            L.has_shared != L0.has_shared)
            return fail(SMOE_INVALID_ARG, "stack_decode: the layers differ in geometry");
        if (!decode_qualifies(L.n_embd, L.n_ff, L.n_expert, L.k, L.gu_type, L.d_type, L.has_shared, L.sg_type,
                              L.su_type, L.sd_type))
            return fail(SMOE_UNSUPPORTED, "stack_decode: a layer does not qualify for the fused single-token kernel "
                                          "(every matrix Q2_0, n_embd a multiple of 512, n_ff a multiple of 128)");
    }
    return SMOE_OK;
}

size_t smoe_stack_decode_scratch_bytes(const smoe_layer* L) {
    if (check_layer(L) != SMOE_OK) return 0;
    return decode_scratch_bytes(L->n_embd, L->n_ff, L->n_expert, L->k);
}

smoe_status smoe_stack_decode(const smoe_layer* layers, int n_layers, const float* const* norm_w, float eps,
                              const float* x, float* out, void* scratch, size_t scratch_bytes, void* stream) {
    smoe_status st = check_stack(layers, n_layers);
    if (st != SMOE_OK) return st;
    if (!(eps >= 0.f)) return fail(SMOE_INVALID_ARG, "stack_decode: eps must be >= 0");
    if (!stream) return fail(SMOE_INVALID_ARG, "stack_decode: a non-null stream is required");
    if (!x || !out || !scratch || !aligned(scratch, 256))
        return fail(SMOE_INVALID_ARG, "stack_decode: null buffer or scratch not 256-byte aligned");
    if (scratch_bytes < decode_scratch_bytes(layers[0].n_embd, layers[0].n_ff, layers[0].n_expert, layers[0].k))
        return fail(SMOE_INVALID_ARG, "stack_decode: scratch is too small");
    // launches of at most kDecodeMaxLayers layers; each after the first reads the previous one's output
    for (int l0 = 0; l0 < n_layers; l0 += kDecodeMaxLayers) {
        DecodeHost dh{};
        dh.layers = layers + l0;
        dh.n_layers = std::min(kDecodeMaxLayers, n_layers - l0);
        dh.norm_w = norm_w ? norm_w + l0 : nullptr;
        dh.norm = 1;
        dh.eps = eps;
        dh.x = l0 == 0 ? x : out;
        dh.out = out;
        dh.scratch = scratch;
        const cudaError_t e = launch_decode(dh, (cudaStream_t) stream);
        if (e != cudaSuccess) return cuda_fail(e, "stack_decode");
    }
    return ok();
}

// ---- the pack's planar S2 experts and the grouped / hit decode API ---------------------------------------------
static bool s2_geom_ok(int H, int F) { return H > 0 && F > 0 && H % 64 == 0 && F % 64 == 0 && H <= 16384 && F <= 16384; }

size_t smoe_s2_blob_bytes(int n_embd, int n_ff) { return s2_geom_ok(n_embd, n_ff) ? s2_blob_bytes(n_embd, n_ff) : 0; }

smoe_status smoe_s2_pack_expert(const uint8_t* gate, const uint8_t* up, const uint8_t* down, int n_embd, int n_ff,
                                uint8_t* blob, void* stream) {
    if (!s2_geom_ok(n_embd, n_ff)) return fail(SMOE_INVALID_ARG, "s2_pack_expert: n_embd and n_ff must be positive multiples of 64");
    if (!stream) return fail(SMOE_INVALID_ARG, "s2_pack_expert: a non-null stream is required");
    if (!gate || !up || !down || !blob || !aligned(blob, 16))
        return fail(SMOE_INVALID_ARG, "s2_pack_expert: null plane, or blob not 16-byte aligned");
    const cudaError_t e = launch_s2_pack(gate, up, down, n_embd, n_ff, blob, (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "s2_pack_expert");
}

smoe_status smoe_quantize_q8_0(const float* x, uint8_t* blocks, float* scales, int64_t n, void* stream) {
    if (n < 0) return fail(SMOE_INVALID_ARG, "quantize_q8_0: negative length");
    if (n == 0) return ok();
    if (n % 32) return fail(SMOE_INVALID_ARG, "quantize_q8_0: length must be a multiple of 32");
    if (!stream) return fail(SMOE_INVALID_ARG, "quantize_q8_0: a non-null stream is required");
    if (!x || !blocks || !aligned(blocks, 2)) return fail(SMOE_INVALID_ARG, "quantize_q8_0: null buffer or odd address");
    const cudaError_t e = launch_quant_q8_0(x, n, blocks, scales, (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "quantize_q8_0");
}

size_t smoe_moe_grouped_scratch_bytes(int64_t cap_entries, int64_t n_embd, int64_t n_ff) {
    if (cap_entries <= 0 || cap_entries > (1 << 20) || !s2_geom_ok((int) n_embd, (int) n_ff)) return 0;
    return s2_scratch_bytes(cap_entries, (int) n_embd, (int) n_ff);
}

static smoe_status s2_common(int H, int F, int64_t cap, const uint8_t* xq, void* scratch, float* out, void* stream,
                             const char* who) {
    if (!s2_geom_ok(H, F)) return fail(SMOE_INVALID_ARG, std::string(who) + ": n_embd and n_ff must be positive multiples of 64");
    if (cap > (1 << 20)) return fail(SMOE_INVALID_ARG, std::string(who) + ": capacity above 2^20");
    if (!stream) return fail(SMOE_INVALID_ARG, std::string(who) + ": a non-null stream is required");
    if (!xq || !scratch || !out || !aligned(xq, 2) || !aligned(scratch, 256))
        return fail(SMOE_INVALID_ARG, std::string(who) + ": null buffer, x not 2-byte or scratch not 256-byte aligned");
    return SMOE_OK;
}

smoe_status smoe_moe_grouped_s2(const unsigned long long* grp_ptr, const int32_t* grp_start, const int32_t* n_groups,
                                const int32_t* ent_dst, const int32_t* ent_tok, int64_t cap_groups, int64_t cap_entries,
                                int n_embd, int n_ff, const uint8_t* x_q8_0, const float* x_scales, void* scratch,
                                float* out, void* stream) {
    if (cap_groups < 0 || cap_entries < 0) return fail(SMOE_INVALID_ARG, "moe_grouped_s2: negative capacity");
    if (cap_groups == 0 || cap_entries == 0) return ok();
    smoe_status st = s2_common(n_embd, n_ff, std::max(cap_groups, cap_entries), x_q8_0, scratch, out, stream, "moe_grouped_s2");
    if (st != SMOE_OK) return st;
    if (!grp_ptr || !grp_start || !n_groups || !ent_dst || !ent_tok) return fail(SMOE_INVALID_ARG, "moe_grouped_s2: null list");
    const cudaError_t e = launch_s2_grouped(grp_ptr, grp_start, n_groups, ent_dst, ent_tok, (int) cap_groups,
                                            (int) cap_entries, n_embd, n_ff, x_q8_0, x_scales, scratch, out,
                                            (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "moe_grouped_s2");
}

smoe_status smoe_moe_group_resident(const int32_t* ids, int n, int k_per_tok, const uint8_t* base, int64_t blob_bytes,
                                    unsigned long long* grp_ptr, int32_t* grp_start, int32_t* counts, int32_t* ent_dst,
                                    int32_t* ent_tok, void* stream) {
    if (n < 0 || k_per_tok < 0 || blob_bytes < 0) return fail(SMOE_INVALID_ARG, "moe_group_resident: negative size");
    if (n > 1024) return fail(SMOE_INVALID_ARG, "moe_group_resident: at most 1024 routing entries");
    if (!stream) return fail(SMOE_INVALID_ARG, "moe_group_resident: a non-null stream is required");
    if (!ids && n > 0) return fail(SMOE_INVALID_ARG, "moe_group_resident: null ids");
    if (!base || !grp_ptr || !grp_start || !counts || !ent_dst || !ent_tok)
        return fail(SMOE_INVALID_ARG, "moe_group_resident: null output");
    const cudaError_t e = launch_s2_group_resident(ids, n, k_per_tok, base, blob_bytes, grp_ptr, grp_start, counts,
                                                   ent_dst, ent_tok, (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "moe_group_resident");
}

smoe_status smoe_moe_hit_select(const int32_t* ids, const int32_t* res_row, int n, int n_expert, int32_t* slot,
                                int32_t* dst, int32_t* count, void* stream) {
    if (n < 0 || n_expert < 0) return fail(SMOE_INVALID_ARG, "moe_hit_select: negative size");
    if (n > 1024) return fail(SMOE_INVALID_ARG, "moe_hit_select: at most 1024 routing entries");
    if (!stream) return fail(SMOE_INVALID_ARG, "moe_hit_select: a non-null stream is required");
    if ((!ids && n > 0) || !res_row || !slot || !dst || !count) return fail(SMOE_INVALID_ARG, "moe_hit_select: null buffer");
    const cudaError_t e = launch_s2_hit_select(ids, res_row, n, n_expert, slot, dst, count, (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "moe_hit_select");
}

smoe_status smoe_moe_hit_grouped_s2(const uint8_t* blob_base, const int32_t* slot_index, const int32_t* dst_index,
                                    const int32_t* d_count, int64_t cap, int64_t blob_bytes, int n_embd, int n_ff,
                                    const uint8_t* x_q8_0, const float* x_scales, int k_per_token, void* scratch,
                                    float* out, void* stream) {
    if (cap < 0 || k_per_token < 0) return fail(SMOE_INVALID_ARG, "moe_hit_grouped_s2: negative size");
    if (cap == 0) return ok();
    smoe_status st = s2_common(n_embd, n_ff, cap, x_q8_0, scratch, out, stream, "moe_hit_grouped_s2");
    if (st != SMOE_OK) return st;
    if (!blob_base || !slot_index || !dst_index || !d_count) return fail(SMOE_INVALID_ARG, "moe_hit_grouped_s2: null list");
    if (blob_bytes < (int64_t) s2_blob_bytes(n_embd, n_ff) || blob_bytes % 16 || !aligned(blob_base, 16))
        return fail(SMOE_INVALID_ARG, "moe_hit_grouped_s2: slots must hold a blob and be 16-byte aligned");
    const cudaError_t e = launch_s2_hits(blob_base, slot_index, dst_index, d_count, (int) cap, blob_bytes, n_embd, n_ff,
                                         x_q8_0, x_scales, k_per_token, scratch, out, (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "moe_hit_grouped_s2");
}

smoe_status smoe_moe_hit_add(float* parts, const float* hit_out, const int32_t* dst, const int32_t* count, int64_t cap,
                             int64_t n_embd, void* stream) {
    if (cap < 0 || n_embd < 0) return fail(SMOE_INVALID_ARG, "moe_hit_add: negative size");
    if (cap == 0 || n_embd == 0) return ok();
    if (!stream) return fail(SMOE_INVALID_ARG, "moe_hit_add: a non-null stream is required");
    if (!parts || !hit_out || !dst || !count) return fail(SMOE_INVALID_ARG, "moe_hit_add: null buffer");
    const cudaError_t e = launch_s2_hit_add(parts, hit_out, dst, count, (int) cap, n_embd, (cudaStream_t) stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "moe_hit_add");
}

size_t smoe_ep_area_bytes(const smoe_layer* L, int max_tokens, int world) {
    // geometry only (n_embd, k): the area does not depend on the planes
    if (!L || L->n_embd <= 0 || L->n_embd % 128 || L->k <= 0 || L->k > kMaxK || max_tokens < 1 || world < 1 ||
        world > SMOE_EP_MAX_WORLD)
        return 0;
    return ep_arena_bytes(L->n_embd, L->k, max_tokens, world);
}

smoe_status smoe_ep_area_alloc(size_t bytes, void** area, void* ipc_handle) {
    if (!area || bytes == 0) return fail(SMOE_INVALID_ARG, "ep_area_alloc: null result pointer or zero size");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess && ipc_handle) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return cuda_fail(e, "ep_area_alloc");
    }
    *area = p;
    return ok();
}

smoe_status smoe_ep_area_open(const void* ipc_handle, void** area) {
    if (!ipc_handle || !area) return fail(SMOE_INVALID_ARG, "ep_area_open: null argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof h);
    const cudaError_t e = cudaIpcOpenMemHandle(area, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? ok() : cuda_fail(e, "ep_area_open");
}

smoe_status smoe_ep_area_close(void* area) {
    const cudaError_t e = cudaIpcCloseMemHandle(area);
    return e == cudaSuccess ? ok() : cuda_fail(e, "ep_area_close");
}

smoe_status smoe_ep_area_free(void* area) {
    const cudaError_t e = cudaFree(area);
    return e == cudaSuccess ? ok() : cuda_fail(e, "ep_area_free");
}

smoe_status smoe_ep_init(const smoe_ep* ep, const smoe_layer* L) {
    const smoe_status st = check_ep(L, ep);
    if (st != SMOE_OK) return st;
    const cudaError_t e = ep_init(ep->areas[ep->rank], ep->areas, ep->rank, ep->world, L->n_embd, L->k, ep->max_tokens);
    return e == cudaSuccess ? ok() : cuda_fail(e, "ep_init");
}

size_t smoe_ep_scratch_bytes(const smoe_layer* L, const smoe_ep* ep) {
    if (check_ep(L, ep) != SMOE_OK) return 0;
    return ep_layout_of(L, ep).total;
}

smoe_status smoe_ep_forward(const smoe_layer* L, const smoe_ep* ep, const float* x, int n_tokens, float* out,
                            void* scratch, size_t scratch_bytes, const smoe_trace* trace, int phases, void* stream) {
    smoe_status st = check_ep(L, ep);
    if (st != SMOE_OK) return st;
    if (n_tokens < 0 || n_tokens > ep->max_tokens) return fail(SMOE_INVALID_ARG, "ep_forward: need 0 <= n_tokens <= max_tokens");
    if (phases < 1 || phases > 7) return fail(SMOE_INVALID_ARG, "ep_forward: phases must be 1..7");
    if (!stream) return fail(SMOE_INVALID_ARG, "ep_forward: a non-null stream is required");
    if (!scratch || !aligned(scratch, 256)) return fail(SMOE_INVALID_ARG, "ep_forward: scratch null or not 256-byte aligned");
    if (n_tokens > 0 && ((phases & 1) && (!x || !aligned(x, 16)))) return fail(SMOE_INVALID_ARG, "ep_forward: x null or unaligned");
    if (n_tokens > 0 && (phases & 4) && !out) return fail(SMOE_INVALID_ARG, "ep_forward: out is null");
    const EpLayout lo = ep_layout_of(L, ep);
    if (scratch_bytes < lo.total) return fail(SMOE_INVALID_ARG, "ep_forward: scratch is too small");
    cudaStream_t s = (cudaStream_t) stream;
    uint8_t* base = static_cast<uint8_t*>(scratch);
    void* area = ep->areas[ep->rank];
    const int T = n_tokens, H = L->n_embd, F = L->n_ff, E = L->n_expert, K = L->k;
    const int G = ep->world, Tm = ep->max_tokens, R = G * Tm, El = E / G;
    const bool sh = L->has_shared != 0;
    const int rows = R * K + (sh ? Tm : 0);
    uint8_t* xq = base + lo.xq;
    float* logits = reinterpret_cast<float*>(base + lo.logits);
    float* sh_logit = reinterpret_cast<float*>(base + lo.sh_logit);
    int32_t* ids = reinterpret_cast<int32_t*>(base + lo.ids);
    float* w = reinterpret_cast<float*>(base + lo.w);
    float* shared_rows = reinterpret_cast<float*>(base + lo.shared);
    const bool tc = use_tc(L, R);
    cudaError_t e = cudaSuccess;

    if (phases & 1) {
        if (T > 0) {
            int splits = 0;
            e = launch_bf16_gemv(x, true, L->router, sh ? L->gate_inp_shexp : nullptr, logits, sh_logit, T, H, E, s,
                                 base + lo.rsplit, &splits);
            const RouterSplit rsplit{reinterpret_cast<const double*>(base + lo.rsplit), splits, logits,
                                     sh ? sh_logit : nullptr};
            if (e == cudaSuccess) e = mark(0, s);
            if (e == cudaSuccess) e = launch_router_topk(logits, T, E, K, ids, w, x, xq, H, s, nullptr, 1, &rsplit);
            if (e == cudaSuccess) e = mark(1, s);
            if (e != cudaSuccess) return cuda_fail(e, "ep_forward: router");
        }
        e = launch_ep_dispatch(area, ids, xq, T, K, H, El, s);
        if (e == cudaSuccess) e = mark(2, s);
        if (e != cudaSuccess) return cuda_fail(e, "ep_forward: dispatch");
    }

    if (phases & 2) {
        int32_t* oids = reinterpret_cast<int32_t*>(base + lo.oids);
        int32_t* slot = reinterpret_cast<int32_t*>(base + lo.slot);
        int32_t* slot_tok = reinterpret_cast<int32_t*>(base + lo.slot_token);
        int32_t* slot_pair = reinterpret_cast<int32_t*>(base + lo.slot_pair);
        const GroupTables tabs = group_tables_at(base + lo.tables, El);
        const KAct xa = ka_at(base + lo.xa, R, H / 32);
        __half* xh = reinterpret_cast<__half*>(base + lo.xh);
        e = launch_ep_receive(area, K, H, ep->rank * El, El, oids, tc ? nullptr : &xa, L->gu_type == kQ2_0,
                              tc ? xh : nullptr, s, R);
        if (e != cudaSuccess) return cuda_fail(e, "ep_forward: receive");
        const Sched sc = tc ? sched_at(base + lo.sched_tc, El, R, K, kTcChunk) : sched_at(base + lo.sched, El, R, K);
        e = launch_group(oids, R, K, El, tabs, slot, slot_tok, s, &sc, reinterpret_cast<int32_t*>(base + lo.chunk), 1,
                         slot_pair);
        if (e != cudaSuccess) return cuda_fail(e, "ep_forward: grouping");
        Work wk{};
        wk.sched = sc;
        wk.slot_token = slot_tok;
        wk.max_entries = tc ? sched_capacity(El, R, K, kTcChunk) : sched_capacity(El, R, K);
        wk.shared_base = R * K;
        wk.shared_slots = sh ? T : 0;
        wk.slot_pair = slot_pair;
        wk.ep_out = ep_parts_table(area);
        wk.ep_shared = shared_rows;
        wk.ep_rows = Tm;
        wk.ep_k = K;
        const int64_t gu_stride = (int64_t) F * (int64_t) row_bytes(L->gu_type, H);
        const int64_t d_stride = (int64_t) H * (int64_t) row_bytes(L->d_type, F);
        const Matrix mg{L->gate, gu_stride, L->gu_type}, mu{L->up, gu_stride, L->gu_type}, md{L->down, d_stride, L->d_type};
        const Matrix sg{L->sgate, 0, L->sg_type}, su{L->sup, 0, L->su_type}, sd{L->sdown, 0, L->sd_type};
        EpDone done;
        done.counter = ep_done_counter(area);
        done.flags = ep_done_table(area);
        done.world = G;
        if (tc) {
            __half* hh = reinterpret_cast<__half*>(base + lo.hh);
            e = launch_tc_gate_up(mg, mu, sg, su, wk, El, xh, R, hh, rows, H, F, s);
            if (e == cudaSuccess) e = mark(3, s);
            if (e != cudaSuccess) return cuda_fail(e, "ep_forward: gate/up (tensor cores)");
            wk.ep_done = done;
            e = launch_tc_down(md, sd, wk, El, hh, rows, nullptr, F, H, s);
            if (e == cudaSuccess) e = mark(4, s);
            if (e != cudaSuccess) return cuda_fail(e, "ep_forward: down (tensor cores)");
        } else if (use_tq(L, R)) {
            const KAct ha = ka_at(base + lo.ha, rows, F / 32);
            e = launch_tq_gate_up(mg, mu, sg, su, wk, El, xa, ha, 1, H, F, s);
            if (e == cudaSuccess) e = mark(3, s);
            if (e != cudaSuccess) return cuda_fail(e, "ep_forward: gate/up (int8 tensor cores)");
            wk.ep_done = done;
            e = launch_tq_down(md, sd, wk, El, ha, nullptr, F, H, s);
            if (e == cudaSuccess) e = mark(4, s);
            if (e != cudaSuccess) return cuda_fail(e, "ep_forward: down (int8 tensor cores)");
        } else {
            float* gu = reinterpret_cast<float*>(base + lo.gu);
            const KAct ha = ka_at(base + lo.ha, rows, F / 32);
            Work w1 = wk;
            w1.counter = tabs.work + 0;
            e = launch_layer_gate_up(mg, mu, sg, su, w1, xa, gu, H, F, s);
            if (e == cudaSuccess) e = launch_swiglu_ka(gu, ha, rows, F, L->d_type == kQ2_0, s);
            if (e == cudaSuccess) e = mark(3, s);
            if (e != cudaSuccess) return cuda_fail(e, "ep_forward: gate/up");
            Work w3 = wk;
            w3.counter = tabs.work + 2;
            w3.ep_done = done;
            e = launch_layer_down(md, sd, w3, ha, nullptr, F, H, s);
            if (e == cudaSuccess) e = mark(4, s);
            if (e != cudaSuccess) return cuda_fail(e, "ep_forward: down");
        }
    }

    if (phases & 4) {
        e = launch_ep_wait_done(area, s);
        float* parts = ep_parts(area, H, K, Tm, G);
        if (e == cudaSuccess && T > 0)
            e = launch_combine(parts, nullptr, w, sh ? shared_rows : nullptr, sh ? sh_logit : nullptr, out,
                               trace ? trace->shared : nullptr, H, K, T, H, s);
        if (e == cudaSuccess) e = mark(5, s);
        if (e != cudaSuccess) return cuda_fail(e, "ep_forward: combine");
        if (trace && T > 0) {
            if (trace->logits) e = cudaMemcpyAsync(trace->logits, logits, (size_t) T * E * 4, cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess && trace->ids)
                e = cudaMemcpyAsync(trace->ids, ids, (size_t) T * K * 4, cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess && trace->weights)
                e = cudaMemcpyAsync(trace->weights, w, (size_t) T * K * 4, cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess && trace->xq)
                e = cudaMemcpyAsync(trace->xq, xq, (size_t) T * (H / 32) * kQ8Block, cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess && trace->parts)
                e = cudaMemcpyAsync(trace->parts, parts, (size_t) T * K * H * 4, cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) return cuda_fail(e, "ep_forward: trace");
        }
    }
    return ok();
}

}  // extern "C"
