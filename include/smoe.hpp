// smoe.hpp - C++ host API over the C ABI (smoe.h), shaped like the reference's layer walk.
//
//   smoe::FfnExec  - the MoE half of a layer: load(...) validates the weights and sizes the scratch arena (set-up,
//                    the only place that allocates); run(...) is one smoe_moe_forward on the exec's stream.
//                    Reference: FfnExec::load / FfnExec::run (metal/include/strata/metal/layer_exec.hpp:111-140,
//                    metal/src/layer_exec.cpp:369-563) between gr_read and gr_write.
//   smoe::Stack    - a Session-style walk over several layers, x = rms_norm(x + MoE_l(x)) per layer
//                    (Session::forward, metal/src/forward.cpp:554-565, with the MoE half only).
//   smoe::Error    - thrown for every non-OK status, as the reference throws MetalError (router.mm:33-37,
//                    iq.mm:150-158, moe_combine.mm:31-38); zero token counts return before any launch.
//
// Header-only; link libsmoe.so and the CUDA runtime.  Device pointers throughout: the caller owns the weights and
// the activations; the exec owns its scratch arena.
#ifndef SMOE_HPP
#define SMOE_HPP

#include "smoe.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace smoe {

class Error : public std::runtime_error {
public:
    Error(smoe_status s, const std::string& what) : std::runtime_error(what), status(s) {}
    smoe_status status;
};

inline void check(smoe_status s, const char* where) {
    if (s != SMOE_OK) throw Error(s, std::string(where) + ": " + smoe_last_error());
}

inline void check_cuda(cudaError_t e, const char* where) {
    if (e != cudaSuccess) throw Error(SMOE_CUDA_ERROR, std::string(where) + ": " + cudaGetErrorString(e));
}

// What one block produced, copied back to the host (the reference's FfnTrace fields of the MoE half:
// route = the router logits, ids / route_w = the chosen experts and weights, exq = the q8_1 image of x,
// edown = each routed slot's down row in router order, shared = the gated shared expert's output).
struct FfnTrace {
    std::vector<float> route, route_w, shared;
    std::vector<int> ids;
    std::vector<uint8_t> exq;
    std::vector<float> edown;  // [T][k][n_embd]
};

class FfnExec {
public:
    FfnExec() = default;
    FfnExec(const FfnExec&) = delete;
    FfnExec& operator=(const FfnExec&) = delete;
    FfnExec(FfnExec&& o) noexcept { *this = std::move(o); }
    FfnExec& operator=(FfnExec&& o) noexcept {
        if (this != &o) {
            release();
            layer_ = o.layer_;
            max_tokens_ = o.max_tokens_;
            stream_ = o.stream_;
            scratch_ = o.scratch_;
            scratch_bytes_ = o.scratch_bytes_;
            o.scratch_ = nullptr;
            o.scratch_bytes_ = 0;
        }
        return *this;
    }
    ~FfnExec() { release(); }

    // `layer` names the device planes (smoe_layer); `with_shared` false drops the shared expert.  Allocates the
    // scratch arena for up to max_tokens tokens (the set-up step: never on the token path).
    static FfnExec load(const smoe_layer& layer, int max_tokens, bool with_shared, cudaStream_t stream) {
        if (!stream) throw Error(SMOE_INVALID_ARG, "FfnExec::load: a non-null stream is required");
        if (max_tokens <= 0) throw Error(SMOE_INVALID_ARG, "FfnExec::load: max_tokens must be positive");
        FfnExec f;
        f.layer_ = layer;
        if (!with_shared) f.layer_.has_shared = 0;
        check(smoe_layer_check(&f.layer_), "FfnExec::load");
        f.max_tokens_ = max_tokens;
        f.stream_ = stream;
        f.scratch_bytes_ = smoe_moe_scratch_bytes(&f.layer_, max_tokens);
        if (f.scratch_bytes_ == 0) throw Error(SMOE_INVALID_ARG, "FfnExec::load: no scratch size for this layer");
        check_cuda(cudaMalloc(&f.scratch_, f.scratch_bytes_), "FfnExec::load");
        return f;
    }

    // combined[T][n_embd] = the MoE block of mixed[T][n_embd] (device pointers).  add_shared false leaves the
    // shared expert out of this call.  With a trace, waits for the stream and copies the stages back.
    void run(const float* mixed, float* combined, int n_tokens, bool add_shared = true, FfnTrace* trace = nullptr) {
        if (n_tokens < 0) throw Error(SMOE_INVALID_ARG, "FfnExec::run: negative token count");
        if (n_tokens > max_tokens_) throw Error(SMOE_INVALID_ARG, "FfnExec::run: more tokens than the arena holds");
        if (n_tokens == 0) return;
        smoe_layer L = layer_;
        if (!add_shared) L.has_shared = 0;
        if (!trace) {
            check(smoe_moe_forward(&L, mixed, n_tokens, combined, scratch_, scratch_bytes_, nullptr, stream_),
                  "FfnExec::run");
            return;
        }
        const size_t T = (size_t) n_tokens, H = (size_t) L.n_embd, K = (size_t) L.k, E = (size_t) L.n_expert;
        const size_t q8 = smoe_q8_1_bytes(L.n_embd);
        DeviceTrace d(T, H, K, E, q8);
        smoe_trace tr{d.logits, d.ids, d.weights, d.xq, d.parts, L.has_shared ? d.shared : nullptr};
        check(smoe_moe_forward(&L, mixed, n_tokens, combined, scratch_, scratch_bytes_, &tr, stream_), "FfnExec::run");
        check_cuda(cudaStreamSynchronize(stream_), "FfnExec::run");
        trace->route.resize(T * E);
        trace->ids.resize(T * K);
        trace->route_w.resize(T * K);
        trace->exq.resize(T * q8);
        trace->edown.resize(T * K * H);
        trace->shared.assign(L.has_shared ? T * H : 0, 0.f);
        d.copy(trace->route.data(), d.logits, T * E * 4);
        d.copy(trace->ids.data(), d.ids, T * K * 4);
        d.copy(trace->route_w.data(), d.weights, T * K * 4);
        d.copy(trace->exq.data(), d.xq, T * q8);
        d.copy(trace->edown.data(), d.parts, T * K * H * 4);
        if (L.has_shared) d.copy(trace->shared.data(), d.shared, T * H * 4);
    }

    const smoe_layer& layer() const { return layer_; }
    cudaStream_t stream() const { return stream_; }
    int max_tokens() const { return max_tokens_; }
    uint64_t gpu_bytes() const { return scratch_bytes_; }  // dense buffers this exec owns (the weights are the caller's)

private:
    // Device buffers of one traced call.  Each allocation is owned as soon as it succeeds, so a failure part way
    // through the constructor frees the ones already made (the destructor of a half-built object never runs).
    struct DeviceTrace {
        struct Free {
            void operator()(void* p) const { cudaFree(p); }
        };
        using Buf = std::unique_ptr<void, Free>;
        Buf bufs[6];
        float* logits = nullptr;
        int32_t* ids = nullptr;
        float* weights = nullptr;
        uint8_t* xq = nullptr;
        float* parts = nullptr;
        float* shared = nullptr;
        DeviceTrace(size_t T, size_t H, size_t K, size_t E, size_t q8) {
            const size_t bytes[6] = {T * E * 4, T * K * 4, T * K * 4, T * q8, T * K * H * 4, T * H * 4};
            void* p[6] = {};
            for (int i = 0; i < 6; i++) {
                check_cuda(cudaMalloc(&p[i], bytes[i]), "FfnTrace");
                bufs[i].reset(p[i]);
            }
            logits = static_cast<float*>(p[0]);
            ids = static_cast<int32_t*>(p[1]);
            weights = static_cast<float*>(p[2]);
            xq = static_cast<uint8_t*>(p[3]);
            parts = static_cast<float*>(p[4]);
            shared = static_cast<float*>(p[5]);
        }
        void copy(void* dst, const void* src, size_t bytes) {
            check_cuda(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost), "FfnTrace");
        }
    };

    void release() {
        if (scratch_) cudaFree(scratch_);
        scratch_ = nullptr;
    }

    smoe_layer layer_{};
    int max_tokens_ = 0;
    cudaStream_t stream_ = nullptr;
    void* scratch_ = nullptr;
    size_t scratch_bytes_ = 0;
};

// Several MoE layers walked in order: y_l = MoE_l(x), x = rms_norm(y_l + x) * norm_l (norm_l may be null: unit
// weight).  Two ping-pong buffers of max_tokens rows are owned by the stack.  Every layer must run on the same
// stream: layer l + 1 reads the buffer layer l wrote, and only stream order makes that read wait for the write.
class Stack {
public:
    Stack(std::vector<FfnExec> layers, std::vector<const float*> norms, float eps)
        : layers_(std::move(layers)), norms_(std::move(norms)), eps_(eps) {
        if (layers_.empty()) throw Error(SMOE_INVALID_ARG, "Stack: no layers");
        if (!norms_.empty() && norms_.size() != layers_.size())
            throw Error(SMOE_INVALID_ARG, "Stack: one norm weight (or none) per layer");
        const smoe_layer& L0 = layers_[0].layer();
        max_tokens_ = layers_[0].max_tokens();
        for (auto& l : layers_) {
            if (l.layer().n_embd != L0.n_embd) throw Error(SMOE_INVALID_ARG, "Stack: layers differ in n_embd");
            if (l.stream() != layers_[0].stream())
                throw Error(SMOE_INVALID_ARG, "Stack: every layer must be loaded on the same stream");
            if (l.max_tokens() < max_tokens_) max_tokens_ = l.max_tokens();
        }
        for (int i = 0; i < 2; i++) {
            void* p = nullptr;
            check_cuda(cudaMalloc(&p, (size_t) max_tokens_ * L0.n_embd * 4), "Stack");
            buf_[i].reset(static_cast<float*>(p));
        }
    }
    Stack(const Stack&) = delete;
    Stack& operator=(const Stack&) = delete;

    // x[T][n_embd] through every layer; returns the device buffer that holds the result (owned by the stack).
    const float* forward(const float* x, int n_tokens) {
        if (n_tokens < 0 || n_tokens > max_tokens_) throw Error(SMOE_INVALID_ARG, "Stack::forward: token count");
        const int H = layers_[0].layer().n_embd;
        const float* cur = x;
        for (size_t l = 0; l < layers_.size(); l++) {
            float* nxt = buf_[l & 1].get();
            layers_[l].run(cur, nxt, n_tokens);
            check(smoe_add_rms_norm(nxt, cur, norms_.empty() ? nullptr : norms_[l], n_tokens, H, eps_,
                                    layers_[l].stream()),
                  "Stack::forward");
            cur = nxt;
        }
        return cur;
    }

    int max_tokens() const { return max_tokens_; }  // the smallest arena among the layers

private:
    struct Free {
        void operator()(float* p) const { cudaFree(p); }
    };
    std::vector<FfnExec> layers_;
    std::vector<const float*> norms_;
    float eps_;
    int max_tokens_ = 0;
    std::unique_ptr<float, Free> buf_[2];
};

}  // namespace smoe

#endif
