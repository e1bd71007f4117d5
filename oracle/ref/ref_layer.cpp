// The MoE block on the host from the reference's OWN host references (TEST / BASELINE INFRASTRUCTURE ONLY).
//
// Arithmetic comes from StrataMetal's sources compiled unmodified in the sibling files: q8_1
// (quant_host_block), the expert chain gate/up -> SwiGLU -> q8_1 -> down (ref_expert, iq_parity.cpp:386-411),
// routing (router_parity.cpp:48-72) and the combine (moe_combine_parity.cpp:55-71).  Two pieces live only in
// pack_parity.cpp, which cannot be compiled here, and are restated: the double-accumulated bf16 router dot
// (pack_parity.cpp:3795-3799) and the shared expert's float sigmoid gate (:3646, :8604-8613).
//
// Work is spread over std::thread workers per (expert, tokens routed to it) group, the way the reference's
// expert pool splits its jobs (include/strata/kernels/cpu/pool.hpp:160-165).
#include "strata/kernels/bf16_bits.hpp"

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <thread>
#include <vector>

extern "C" {
void ref_quant_q8_1_block(const float* x, uint8_t* y);
void ref_expert_q8(int gu_type, int d_type, int n_embd, int n_ff, const uint8_t* blob, size_t blob_bytes,
                   const uint8_t* x_q8, int n_tok, float* y);
void ref_route(const float* logits, int n_expert, int k, int* ids, float* w);
void ref_combine(const float* parts, const float* w, const float* shared, float* y, int n_embd, int k,
                 int weight_routed, int weight_shared);
}

namespace {

size_t rowb(int t, int n) { return t == 42 ? (size_t) (n / 64) * 18 : (size_t) (n / 256) * 82; }

float bf16_dot(const float* x, const uint16_t* row, int n) {
    double acc = 0;
    for (int i = 0; i < n; ++i) acc += (double) x[i] * (double) strata::kernels::f32_from_bf16(row[i]);
    return (float) acc;
}

template <class F>
void parallel_for(int n, int threads, F&& fn) {
    std::atomic<int> next{0};
    auto work = [&] {
        for (int i; (i = next.fetch_add(1)) < n;) fn(i);
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < threads && t < n; ++t) pool.emplace_back(work);
    work();
    for (auto& th : pool) th.join();
}

}  // namespace

extern "C" int ref_moe_layer(int n_embd, int n_ff, int n_expert, int k, int gu_type, int d_type,
                             const uint16_t* router, const uint8_t* gate, const uint8_t* up, const uint8_t* down,
                             int has_shared, int sgu_type, int sd_type, const uint8_t* sgate, const uint8_t* sup,
                             const uint8_t* sdown, const uint16_t* ginp, const float* x, int T, float* out,
                             int threads) {
    const int H = n_embd, F = n_ff, E = n_expert, K = k;
    const size_t xqb = (size_t) (H / 32) * 36;
    std::vector<float> xr((size_t) T * H), logits((size_t) T * E), w((size_t) T * K), scale((size_t) T);
    std::vector<int> ids((size_t) T * K);
    std::vector<uint8_t> xq((size_t) T * xqb);
    parallel_for(T, threads, [&](int t) {
        const float* xt = x + (size_t) t * H;
        float* r = xr.data() + (size_t) t * H;
        for (int i = 0; i < H; ++i) r[i] = strata::kernels::f32_from_bf16(strata::kernels::bf16_from_f32(xt[i]));
        for (int e = 0; e < E; ++e) logits[(size_t) t * E + e] = bf16_dot(r, router + (size_t) e * H, H);
        ref_route(logits.data() + (size_t) t * E, E, K, ids.data() + (size_t) t * K, w.data() + (size_t) t * K);
        for (int b = 0; b < H / 32; ++b) ref_quant_q8_1_block(xt + b * 32, xq.data() + (size_t) t * xqb + b * 36);
        if (has_shared) scale[(size_t) t] = bf16_dot(r, ginp, H);
    });
    for (int v : ids)
        if (v < 0 || v >= E) return -1;
    // expert -> the (token, slot) pairs routed to it, in token order
    std::map<int, std::vector<int>> groups;
    for (int i = 0; i < T * K; ++i) groups[ids[(size_t) i]].push_back(i);
    std::vector<std::pair<int, std::vector<int>>> items(groups.begin(), groups.end());
    if (has_shared) {
        std::vector<int> all((size_t) T);
        for (int t = 0; t < T; ++t) all[(size_t) t] = -1 - t;
        items.emplace_back(-1, all);
    }
    const size_t gu_n = rowb(gu_type, H) * (size_t) F, d_n = rowb(d_type, F) * (size_t) H;
    const size_t sgu_n = has_shared ? rowb(sgu_type, H) * (size_t) F : 0, sd_n = has_shared ? rowb(sd_type, F) * (size_t) H : 0;
    std::vector<float> parts((size_t) T * K * H), shared((size_t) T * H);
    parallel_for((int) items.size(), threads, [&](int j) {
        const int e = items[(size_t) j].first;
        const std::vector<int>& pairs = items[(size_t) j].second;
        const bool sh = e < 0;
        const int gt = sh ? sgu_type : gu_type, dt = sh ? sd_type : d_type;
        const size_t g_n = sh ? sgu_n : gu_n, dn = sh ? sd_n : d_n;
        std::vector<uint8_t> blob(2 * g_n + dn);
        std::memcpy(blob.data(), sh ? sgate : gate + (size_t) e * g_n, g_n);
        std::memcpy(blob.data() + g_n, sh ? sup : up + (size_t) e * g_n, g_n);
        std::memcpy(blob.data() + 2 * g_n, sh ? sdown : down + (size_t) e * dn, dn);
        const int n = (int) pairs.size();
        std::vector<uint8_t> xs((size_t) n * xqb);
        for (int i = 0; i < n; ++i) {
            const int t = sh ? -1 - pairs[(size_t) i] : pairs[(size_t) i] / K;
            std::memcpy(xs.data() + (size_t) i * xqb, xq.data() + (size_t) t * xqb, xqb);
        }
        std::vector<float> y((size_t) n * H);
        ref_expert_q8(gt, dt, H, F, blob.data(), blob.size(), xs.data(), n, y.data());
        for (int i = 0; i < n; ++i) {
            float* dst = sh ? shared.data() + (size_t) (-1 - pairs[(size_t) i]) * H : parts.data() + (size_t) pairs[(size_t) i] * H;
            std::memcpy(dst, y.data() + (size_t) i * H, (size_t) H * 4);
        }
    });
    for (int t = 0; t < T; ++t) {
        const float* sh = nullptr;
        if (has_shared) {
            const float sig = 1.0f / (1.0f + std::exp(-scale[(size_t) t]));
            float* s = shared.data() + (size_t) t * H;
            for (int d = 0; d < H; ++d) s[d] = s[d] * sig;
            sh = s;
        }
        ref_combine(parts.data() + (size_t) t * K * H, w.data() + (size_t) t * K, sh, out + (size_t) t * H, H, K, 1, 0);
    }
    return 0;
}
