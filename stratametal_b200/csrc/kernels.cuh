// kernels.cuh - launchers shared between the kernel files and the C ABI (api.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace smoe {

constexpr int kRouterTokTile = 16;  // tokens per CTA in the router GEMV (x staged as bf16: 16 x n_embd x 2 bytes)
constexpr int kMaxExperts = 1024;
constexpr int kMaxK = 64;

// ---- router.cu ----
cudaError_t launch_bf16_gemv(const void* x, bool f32_in, const uint16_t* w, const uint16_t* extra, float* y,
                             float* y_extra, int T, int H, int n_out, cudaStream_t s);
cudaError_t launch_router_topk(const float* logits, int T, int E, int k, int32_t* ids, float* w, const float* x,
                               uint8_t* xq, int H, cudaStream_t s);
cudaError_t launch_quant_q8_1(const float* x, int64_t n, uint8_t* y, cudaStream_t s);
cudaError_t launch_swiglu_q8(const float* g, const float* u, int64_t n, uint8_t* y, cudaStream_t s);
cudaError_t launch_f32_to_bf16(const float* x, uint16_t* y, int64_t n, cudaStream_t s);

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
cudaError_t launch_group(const int32_t* ids, int T, int k, int E, GroupTables g, int32_t* slot, int32_t* src,
                         cudaStream_t s);

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

// gate/up + SwiGLU + q8_1 of h for every slot of every expert in `g`:
// hq[slot][n_ff / 32 q8_1 blocks] from xq[token][n_embd / 32 blocks].
cudaError_t launch_expert_gate_up(Matrix gate, Matrix up, Matrix sgate, Matrix sup, GroupView g, const uint8_t* xq,
                                  uint8_t* hq, int n_embd, int n_ff, cudaStream_t s);
// y[slot][r] = down_e[r] . act[slot] for every slot, y row stride y_stride floats; act rows n_in / 32 blocks.
cudaError_t launch_expert_down(Matrix down, Matrix sdown, GroupView g, const uint8_t* act, int act_by_token,
                               float* y, int64_t y_stride, int n_in, int n_out, cudaStream_t s);

// ---- combine.cu ----
// out[t][j] = sum_i w[t][i] * parts[slot(t, i)][j] (+ shared[t][j] * sigmoid(gate_logit[t]) when shared)
// slot == nullptr means parts is [T][k][H] in router order; shared_scale == nullptr adds shared plain.
cudaError_t launch_combine(const float* parts, const int32_t* slot, const float* w, const float* shared,
                           const float* shared_logit, float* out, float* shared_out, int64_t H, int k, int T,
                           int64_t shared_stride, cudaStream_t s);
cudaError_t launch_gather_parts(const float* parts, const int32_t* slot, float* dst, int64_t H, int k, int T,
                                cudaStream_t s);

}  // namespace smoe
