// ffn_exec_test.cpp - the C++ host API (include/smoe.hpp) against the C ABI.
//   mode "refusals" (no GPU needed): load() and run() throw smoe::Error for the reference's refused arguments
//       before any CUDA call; zero tokens return at once.
//   mode "run" (a GPU): FfnExec::run equals smoe_moe_forward bit for bit on one synthetic Q2_0 layer, with and
//       without the shared expert, and a two-layer Stack equals the same calls made by hand.
#include "smoe.hpp"

#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

static int fails = 0;
#define EXPECT(c)                                                       \
    do {                                                                \
        if (!(c)) {                                                     \
            std::fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #c); \
            fails++;                                                    \
        }                                                               \
    } while (0)

template <typename F>
static smoe_status throws(F f) {
    try {
        f();
    } catch (const smoe::Error& e) {
        return e.status;
    }
    return SMOE_OK;
}

static smoe_layer geometry(int H, int F, int E, int k) {
    smoe_layer L{};
    L.n_embd = H;
    L.n_ff = F;
    L.n_expert = E;
    L.k = k;
    L.gu_type = L.d_type = SMOE_Q2_0;
    return L;
}

static int refusals() {
    const auto fake = reinterpret_cast<const void*>(uintptr_t(4096));  // never dereferenced: refused before use
    smoe_layer L = geometry(512, 128, 16, 4);
    L.router = static_cast<const uint16_t*>(fake);
    L.gate = L.up = L.down = static_cast<const uint8_t*>(fake);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(uintptr_t(1));
    smoe_layer bad = L;
    bad.k = 65;  // k > 64
    EXPECT(throws([&] { smoe::FfnExec::load(bad, 8, false, s); }) == SMOE_INVALID_ARG);
    bad = L;
    bad.n_expert = 1025;  // more than 1024 experts
    EXPECT(throws([&] { smoe::FfnExec::load(bad, 8, false, s); }) == SMOE_INVALID_ARG);
    bad = L;
    bad.k = 17;  // k above n_expert
    EXPECT(throws([&] { smoe::FfnExec::load(bad, 8, false, s); }) == SMOE_INVALID_ARG);
    bad = L;
    bad.gu_type = 29;  // not Q2_0 / IQ2_S
    EXPECT(throws([&] { smoe::FfnExec::load(bad, 8, false, s); }) == SMOE_UNSUPPORTED);
    bad = L;
    bad.n_embd = 500;  // not whole blocks
    EXPECT(throws([&] { smoe::FfnExec::load(bad, 8, false, s); }) != SMOE_OK);
    EXPECT(throws([&] { smoe::FfnExec::load(L, 0, false, s); }) == SMOE_INVALID_ARG);
    EXPECT(throws([&] { smoe::FfnExec::load(L, 8, false, nullptr); }) == SMOE_INVALID_ARG);
    bad = L;
    bad.has_shared = 1;  // shared expert requested but its planes are null
    bad.sg_type = bad.su_type = bad.sd_type = SMOE_Q2_0;
    EXPECT(throws([&] { smoe::FfnExec::load(bad, 8, true, s); }) == SMOE_INVALID_ARG);
    smoe::FfnExec empty;  // a default exec holds no arena: zero tokens still return before any launch
    EXPECT(throws([&] { empty.run(nullptr, nullptr, 0); }) == SMOE_OK);
    EXPECT(throws([&] { empty.run(nullptr, nullptr, -1); }) == SMOE_INVALID_ARG);
    std::printf("refusals: %s\n", fails ? "FAIL" : "ok");
    return fails;
}

// Q2_0 bytes with sane fp16 scales: each 18-byte block starts with d = 2^-6 (0x2400) and 16 random code bytes.
static std::vector<uint8_t> q2_plane(size_t rows, int n, std::mt19937& g) {
    const size_t rb = (size_t) n / 64 * 18;
    std::vector<uint8_t> v(rows * rb);
    for (size_t i = 0; i < v.size(); i++) v[i] = (uint8_t) g();
    for (size_t r = 0; r < rows; r++)
        for (size_t b = 0; b < rb; b += 18) {
            v[r * rb + b] = 0x00;
            v[r * rb + b + 1] = 0x24;
        }
    return v;
}

template <typename T>
static T* upload(const std::vector<T>& h) {
    T* d = nullptr;
    smoe::check_cuda(cudaMalloc(&d, h.size() * sizeof(T)), "upload");
    smoe::check_cuda(cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice), "upload");
    return d;
}

static int run_gpu() {
    const int H = 512, F = 512, E = 32, K = 4, T = 9;
    std::mt19937 g(7);
    std::normal_distribution<float> nd(0.f, 1.f);
    std::vector<uint16_t> router((size_t) E * H), ginp(H);
    for (auto& v : router) v = (uint16_t) (0x3C00 ^ (g() & 0x80FF));  // bf16 around +-0.008
    for (auto& v : ginp) v = (uint16_t) (0x3C00 ^ (g() & 0x80FF));
    smoe_layer L = geometry(H, F, E, K);
    L.router = upload(router);
    L.gate = upload(q2_plane((size_t) E * F, H, g));
    L.up = upload(q2_plane((size_t) E * F, H, g));
    L.down = upload(q2_plane((size_t) E * H, F, g));
    L.has_shared = 1;
    L.sg_type = L.su_type = L.sd_type = SMOE_Q2_0;
    L.sgate = upload(q2_plane(F, H, g));
    L.sup = upload(q2_plane(F, H, g));
    L.sdown = upload(q2_plane(H, F, g));
    L.gate_inp_shexp = upload(ginp);
    std::vector<float> hx((size_t) T * H);
    for (auto& v : hx) v = nd(g);
    float* x = upload(hx);
    float *y1, *y2;
    smoe::check_cuda(cudaMalloc(&y1, hx.size() * 4), "y");
    smoe::check_cuda(cudaMalloc(&y2, hx.size() * 4), "y");
    cudaStream_t s;
    smoe::check_cuda(cudaStreamCreate(&s), "stream");
    std::vector<float> a(hx.size()), b(hx.size());
    for (int shared = 0; shared < 2; shared++) {
        auto f = smoe::FfnExec::load(L, 16, true, s);
        smoe::FfnTrace tr;
        f.run(x, y1, T, shared != 0, &tr);
        smoe_layer Lc = L;
        Lc.has_shared = shared;
        const size_t nb = smoe_moe_scratch_bytes(&Lc, T);
        void* scr;
        smoe::check_cuda(cudaMalloc(&scr, nb), "scratch");
        smoe::check(smoe_moe_forward(&Lc, x, T, y2, scr, nb, nullptr, s), "forward");
        smoe::check_cuda(cudaStreamSynchronize(s), "sync");
        cudaMemcpy(a.data(), y1, a.size() * 4, cudaMemcpyDeviceToHost);
        cudaMemcpy(b.data(), y2, b.size() * 4, cudaMemcpyDeviceToHost);
        EXPECT(std::memcmp(a.data(), b.data(), a.size() * 4) == 0);
        EXPECT(tr.ids.size() == (size_t) T * K && tr.route_w.size() == (size_t) T * K);
        for (int id : tr.ids) EXPECT(id >= 0 && id < E);
        EXPECT(tr.shared.size() == (shared ? (size_t) T * H : 0));
        cudaFree(scr);
    }
    // two layers through Stack == by hand
    std::vector<smoe::FfnExec> ls;
    ls.push_back(smoe::FfnExec::load(L, 16, true, s));
    ls.push_back(smoe::FfnExec::load(L, 16, true, s));
    smoe::Stack st(std::move(ls), {}, 1e-6f);
    const float* out = st.forward(x, T);
    auto f = smoe::FfnExec::load(L, 16, true, s);
    float *c1, *c2;
    cudaMalloc(&c1, hx.size() * 4);
    cudaMalloc(&c2, hx.size() * 4);
    f.run(x, c1, T);
    smoe::check(smoe_add_rms_norm(c1, x, nullptr, T, H, 1e-6f, s), "norm");
    f.run(c1, c2, T);
    smoe::check(smoe_add_rms_norm(c2, c1, nullptr, T, H, 1e-6f, s), "norm");
    smoe::check_cuda(cudaStreamSynchronize(s), "sync");
    cudaMemcpy(a.data(), out, a.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(b.data(), c2, b.size() * 4, cudaMemcpyDeviceToHost);
    EXPECT(std::memcmp(a.data(), b.data(), a.size() * 4) == 0);
    // layers on different streams would race on the stack's ping-pong buffers: refused
    cudaStream_t s2;
    smoe::check_cuda(cudaStreamCreate(&s2), "stream");
    {
        std::vector<smoe::FfnExec> mixed;
        mixed.push_back(smoe::FfnExec::load(L, 16, true, s));
        mixed.push_back(smoe::FfnExec::load(L, 16, true, s2));
        bool refused = false;
        try {
            smoe::Stack bad(std::move(mixed), {}, 1e-6f);
        } catch (const smoe::Error& e) {
            refused = e.status == SMOE_INVALID_ARG;
        }
        EXPECT(refused);
    }
    cudaStreamDestroy(s2);
    EXPECT(smoe_device_status(1) == 0);
    std::printf("run: %s\n", fails ? "FAIL" : "ok");
    return fails;
}

int main(int argc, char** argv) {
    const bool gpu = argc > 1 && std::strcmp(argv[1], "run") == 0;
    try {
        return gpu ? run_gpu() : refusals();
    } catch (const std::exception& e) {
        std::fprintf(stderr, "FAIL: %s\n", e.what());
        return 1;
    }
}
