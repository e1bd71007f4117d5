// smoe_gguf.hpp - the model boundary of the MoE block: one layer's planes read from a GGUF file by tensor name and
// uploaded to the device (host side, over the C ABI).
//
//   smoe::Gguf       - a GGUF v2/v3 file mapped read-only: the header, every metadata key (all value types, arrays
//                      included, kept as scalars or skipped), the tensor directory and the aligned data section
//                      (general.alignment, default 32).  find(name) -> type, shape, bytes and a host pointer.
//   smoe::GgufLayer  - MoE layer `layer` of such a file on the device, found by the names the reference's layer
//                      walk uses (blk.<L>.ffn_gate_inp / ffn_{gate,up,down}_exps / ffn_{gate,up,down}_shexp /
//                      ffn_gate_inp_shexp .weight; metal/src/layer_exec.cpp:109-123, 369-452, names
//                      layer_tensors.hpp:48) and checked the way expert_spans checks them: each expert plane holds
//                      exactly n_expert experts of whole rows.  Geometry comes from the shapes (gate ne = {n_embd,
//                      n_ff, n_expert}); k from <arch>.expert_used_count unless the caller gives it.  The router is
//                      BF16 (an F32 router is rounded to bf16 RNE, the contract's weight type).  desc() is the
//                      smoe_layer the block runs on.
//
// Header-only; link libsmoe.so and the CUDA runtime.  Throws smoe::Error like smoe.hpp.
#ifndef SMOE_GGUF_HPP
#define SMOE_GGUF_HPP

#include "smoe.hpp"

#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace smoe {

class Gguf {
public:
    enum : uint32_t { kF32 = 0, kF16 = 1, kBF16 = 30 };

    struct Tensor {
        std::string name;
        uint32_t type = 0;
        int n_dims = 0;
        int64_t ne[4] = {1, 1, 1, 1};
        uint64_t offset = 0, bytes = 0;
        const uint8_t* data = nullptr;
    };

    Gguf() = default;
    Gguf(const Gguf&) = delete;
    Gguf& operator=(const Gguf&) = delete;
    ~Gguf() { unmap(); }

    void open(const std::string& path) {
        unmap();
        fd_ = ::open(path.c_str(), O_RDONLY);
        if (fd_ < 0) throw Error(SMOE_INVALID_ARG, "GGUF: cannot open " + path);
        struct stat st;
        if (fstat(fd_, &st) != 0) throw Error(SMOE_INVALID_ARG, "GGUF: cannot stat " + path);
        size_ = (uint64_t) st.st_size;
        if (size_ < 24) throw Error(SMOE_INVALID_ARG, "GGUF: " + path + " is too short");
        void* p = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
        if (p == MAP_FAILED) throw Error(SMOE_INVALID_ARG, "GGUF: cannot map " + path);
        base_ = static_cast<const uint8_t*>(p);
        parse();
    }

    const Tensor* find(const std::string& name) const {
        auto it = index_.find(name);
        return it == index_.end() ? nullptr : &tensors_[it->second];
    }
    const Tensor& at(const std::string& name) const {
        const Tensor* t = find(name);
        if (!t) throw Error(SMOE_INVALID_ARG, "GGUF: tensor " + name + " is missing");
        return *t;
    }
    static std::string layer_name(int layer, const std::string& suffix) {
        return "blk." + std::to_string(layer) + "." + suffix;
    }
    // An unsigned-integer metadata value, or `dflt` when the key is absent or not an integer.
    uint64_t meta_u64(const std::string& key, uint64_t dflt) const {
        auto it = meta_u_.find(key);
        return it == meta_u_.end() ? dflt : it->second;
    }
    std::string meta_str(const std::string& key) const {
        auto it = meta_s_.find(key);
        return it == meta_s_.end() ? std::string() : it->second;
    }
    const std::vector<Tensor>& tensors() const { return tensors_; }
    uint32_t version() const { return version_; }

    // Bytes of a tensor of `type` and shape ne (0 for a type this reader cannot size).
    static uint64_t type_bytes(uint32_t type, const int64_t (&ne)[4]) {
        int64_t bv = 0, bb = 0;
        switch (type) {
            case kF32: bv = 1; bb = 4; break;
            case kF16: case kBF16: bv = 1; bb = 2; break;
            default: {
                const size_t rb = smoe_row_bytes((int) type, 256 * 64);  // any multiple of both block sizes
                if (rb == 0) return 0;
                bv = (type == SMOE_Q2_0) ? 64 : (type == SMOE_IQ4_NL) ? 32 : 256;
                bb = (int64_t) smoe_row_bytes((int) type, bv);
            }
        }
        if (ne[0] % bv) return 0;
        return (uint64_t) (ne[0] / bv) * (uint64_t) bb * (uint64_t) ne[1] * (uint64_t) ne[2] * (uint64_t) ne[3];
    }

private:
    template <typename T>
    T rd() {
        if (pos_ + sizeof(T) > size_) throw Error(SMOE_INVALID_ARG, "GGUF: truncated header");
        T v;
        std::memcpy(&v, base_ + pos_, sizeof(T));
        pos_ += sizeof(T);
        return v;
    }
    std::string rd_str() {
        const uint64_t n = rd<uint64_t>();
        if (n > size_ - pos_) throw Error(SMOE_INVALID_ARG, "GGUF: truncated string");
        std::string s(reinterpret_cast<const char*>(base_ + pos_), (size_t) n);
        pos_ += n;
        return s;
    }
    // Reads one value of type t; integer values are returned through u (when is_int), strings through s.
    void rd_value(uint32_t t, uint64_t& u, bool& is_int, std::string& s, int depth = 0) {
        is_int = false;
        switch (t) {
            case 0: u = rd<uint8_t>(); is_int = true; break;
            case 1: u = (uint64_t) rd<int8_t>(); is_int = true; break;
            case 2: u = rd<uint16_t>(); is_int = true; break;
            case 3: u = (uint64_t) rd<int16_t>(); is_int = true; break;
            case 4: u = rd<uint32_t>(); is_int = true; break;
            case 5: u = (uint64_t) rd<int32_t>(); is_int = true; break;
            case 6: rd<float>(); break;
            case 7: u = rd<uint8_t>(); break;
            case 8: s = rd_str(); break;
            case 9: {
                if (depth > 2) throw Error(SMOE_INVALID_ARG, "GGUF: nested arrays too deep");
                const uint32_t it = rd<uint32_t>();
                const uint64_t n = rd<uint64_t>();
                for (uint64_t i = 0; i < n; i++) {
                    uint64_t uu;
                    bool ii;
                    std::string ss;
                    rd_value(it, uu, ii, ss, depth + 1);
                }
                break;
            }
            case 10: u = rd<uint64_t>(); is_int = true; break;
            case 11: u = (uint64_t) rd<int64_t>(); is_int = true; break;
            case 12: rd<double>(); break;
            default: throw Error(SMOE_INVALID_ARG, "GGUF: unknown metadata value type " + std::to_string(t));
        }
    }

    void parse() {
        pos_ = 0;
        if (rd<uint32_t>() != 0x46554747u) throw Error(SMOE_INVALID_ARG, "GGUF: bad magic");
        version_ = rd<uint32_t>();
        if (version_ != 2 && version_ != 3) throw Error(SMOE_UNSUPPORTED, "GGUF: version " + std::to_string(version_));
        const uint64_t n_tensors = rd<uint64_t>(), n_kv = rd<uint64_t>();
        if (n_tensors > (1u << 24) || n_kv > (1u << 24)) throw Error(SMOE_INVALID_ARG, "GGUF: implausible counts");
        for (uint64_t i = 0; i < n_kv; i++) {
            const std::string key = rd_str();
            const uint32_t t = rd<uint32_t>();
            uint64_t u = 0;
            bool is_int = false;
            std::string s;
            rd_value(t, u, is_int, s);
            if (is_int) meta_u_[key] = u;
            if (t == 8) meta_s_[key] = s;
        }
        tensors_.resize((size_t) n_tensors);
        for (auto& t : tensors_) {
            t.name = rd_str();
            t.n_dims = (int) rd<uint32_t>();
            if (t.n_dims < 1 || t.n_dims > 4) throw Error(SMOE_INVALID_ARG, "GGUF: tensor " + t.name + " has bad rank");
            for (int d = 0; d < t.n_dims; d++) t.ne[d] = (int64_t) rd<uint64_t>();
            t.type = rd<uint32_t>();
            t.offset = rd<uint64_t>();
            if (!index_.emplace(t.name, (size_t) (&t - tensors_.data())).second)
                throw Error(SMOE_INVALID_ARG, "GGUF: tensor " + t.name + " is listed twice");
        }
        const uint64_t align = meta_u64("general.alignment", 32);
        if (align == 0 || (align & (align - 1))) throw Error(SMOE_INVALID_ARG, "GGUF: bad general.alignment");
        const uint64_t data = (pos_ + align - 1) / align * align;
        for (auto& t : tensors_) {
            t.bytes = type_bytes(t.type, t.ne);
            if (t.offset % align) throw Error(SMOE_INVALID_ARG, "GGUF: tensor " + t.name + " is not aligned");
            if (t.bytes && data + t.offset + t.bytes <= size_) t.data = base_ + data + t.offset;
            else if (t.bytes) throw Error(SMOE_INVALID_ARG, "GGUF: tensor " + t.name + " runs past the end of the file");
        }
    }

    void unmap() {
        if (base_) munmap(const_cast<uint8_t*>(base_), size_);
        if (fd_ >= 0) ::close(fd_);
        base_ = nullptr;
        fd_ = -1;
        tensors_.clear();
        index_.clear();
        meta_u_.clear();
        meta_s_.clear();
    }

    int fd_ = -1;
    const uint8_t* base_ = nullptr;
    uint64_t size_ = 0, pos_ = 0;
    uint32_t version_ = 0;
    std::vector<Tensor> tensors_;
    std::map<std::string, size_t> index_;
    std::map<std::string, uint64_t> meta_u_;
    std::map<std::string, std::string> meta_s_;
};

class GgufLayer {
public:
    GgufLayer() = default;
    GgufLayer(const GgufLayer&) = delete;
    GgufLayer& operator=(const GgufLayer&) = delete;

    // k <= 0: <general.architecture>.expert_used_count from the metadata.
    static std::unique_ptr<GgufLayer> load(const Gguf& m, int layer, bool with_shared, int k = 0) {
        std::unique_ptr<GgufLayer> g(new GgufLayer());
        const Gguf::Tensor& gate = m.at(Gguf::layer_name(layer, "ffn_gate_exps.weight"));
        const Gguf::Tensor& up = m.at(Gguf::layer_name(layer, "ffn_up_exps.weight"));
        const Gguf::Tensor& down = m.at(Gguf::layer_name(layer, "ffn_down_exps.weight"));
        const Gguf::Tensor& router = m.at(Gguf::layer_name(layer, "ffn_gate_inp.weight"));
        const int64_t H = gate.ne[0], F = gate.ne[1], E = gate.ne[2];
        if (gate.n_dims != 3 || up.n_dims != 3 || down.n_dims != 3 || up.ne[0] != H || up.ne[1] != F || up.ne[2] != E ||
            down.ne[0] != F || down.ne[1] != H || down.ne[2] != E)
            throw Error(SMOE_INVALID_ARG, "GGUF layer " + std::to_string(layer) + ": expert planes disagree in shape");
        // expert_spans (layer_exec.cpp:109-123): every plane holds exactly E experts of whole rows
        const size_t gn = smoe_row_bytes((int) gate.type, H) * (size_t) F, un = smoe_row_bytes((int) up.type, H) * (size_t) F;
        const size_t dn = smoe_row_bytes((int) down.type, F) * (size_t) H;
        if (!gn || !un || !dn || gate.bytes != gn * E || up.bytes != un * E || down.bytes != dn * E || !gate.data ||
            !up.data || !down.data)
            throw Error(SMOE_INVALID_ARG, "GGUF layer " + std::to_string(layer) + ": routed expert planes are missing");
        if (gate.type != up.type) throw Error(SMOE_UNSUPPORTED, "GGUF layer: gate and up types differ");
        if (router.ne[0] != H || router.ne[1] != E || (router.type != Gguf::kBF16 && router.type != Gguf::kF32))
            throw Error(SMOE_INVALID_ARG, "GGUF layer: ffn_gate_inp must be BF16 or F32 [n_expert][n_embd]");
        if (k <= 0) k = (int) m.meta_u64(m.meta_str("general.architecture") + ".expert_used_count", 0);
        if (k <= 0) throw Error(SMOE_INVALID_ARG, "GGUF: expert_used_count is missing; pass k");
        smoe_layer& L = g->L_;
        std::memset(&L, 0, sizeof L);
        L.n_embd = (int) H;
        L.n_ff = (int) F;
        L.n_expert = (int) E;
        L.k = k;
        L.gu_type = (int) gate.type;
        L.d_type = (int) down.type;
        L.router = static_cast<const uint16_t*>(g->upload_bf16(router));
        L.gate = static_cast<const uint8_t*>(g->upload(gate.data, gate.bytes));
        L.up = static_cast<const uint8_t*>(g->upload(up.data, up.bytes));
        L.down = static_cast<const uint8_t*>(g->upload(down.data, down.bytes));
        if (with_shared) {
            const Gguf::Tensor& sg = m.at(Gguf::layer_name(layer, "ffn_gate_shexp.weight"));
            const Gguf::Tensor& su = m.at(Gguf::layer_name(layer, "ffn_up_shexp.weight"));
            const Gguf::Tensor& sd = m.at(Gguf::layer_name(layer, "ffn_down_shexp.weight"));
            const Gguf::Tensor& gi = m.at(Gguf::layer_name(layer, "ffn_gate_inp_shexp.weight"));
            if (sg.ne[0] != H || su.ne[0] != H || sd.ne[0] != sg.ne[1] || sd.ne[1] != H || su.ne[1] != sg.ne[1] ||
                gi.ne[0] != H || (gi.type != Gguf::kBF16 && gi.type != Gguf::kF32) || !sg.data || !su.data || !sd.data)
                throw Error(SMOE_INVALID_ARG, "GGUF layer: shared expert planes disagree in shape");
            if (sg.ne[1] != F) throw Error(SMOE_UNSUPPORTED, "GGUF layer: the shared expert's width differs from n_ff");
            L.has_shared = 1;
            L.sg_type = (int) sg.type;
            L.su_type = (int) su.type;
            L.sd_type = (int) sd.type;
            L.sgate = static_cast<const uint8_t*>(g->upload(sg.data, sg.bytes));
            L.sup = static_cast<const uint8_t*>(g->upload(su.data, su.bytes));
            L.sdown = static_cast<const uint8_t*>(g->upload(sd.data, sd.bytes));
            L.gate_inp_shexp = static_cast<const uint16_t*>(g->upload_bf16(gi));
        }
        check(smoe_layer_check(&L), "GGUF layer");
        return g;
    }

    const smoe_layer& desc() const { return L_; }
    uint64_t gpu_bytes() const { return bytes_; }

private:
    struct Free {
        void operator()(void* p) const { cudaFree(p); }
    };

    void* upload(const void* host, uint64_t bytes) {
        void* p = nullptr;
        check_cuda(cudaMalloc(&p, (size_t) bytes), "GGUF layer upload");
        bufs_.emplace_back(p);
        check_cuda(cudaMemcpy(p, host, (size_t) bytes, cudaMemcpyHostToDevice), "GGUF layer upload");
        bytes_ += bytes;
        return p;
    }
    // BF16 as is; F32 rounded to bf16 (nearest even) on the host
    void* upload_bf16(const Gguf::Tensor& t) {
        if (t.type == Gguf::kBF16) return upload(t.data, t.bytes);
        const size_t n = (size_t) (t.bytes / 4);
        std::vector<uint16_t> b(n);
        for (size_t i = 0; i < n; i++) {
            uint32_t u;
            std::memcpy(&u, t.data + 4 * i, 4);
            if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) b[i] = (uint16_t) ((u >> 16) | 0x40u);  // NaN
            else b[i] = (uint16_t) ((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
        }
        return upload(b.data(), (uint64_t) n * 2);
    }

    smoe_layer L_{};
    std::vector<std::unique_ptr<void, Free>> bufs_;
    uint64_t bytes_ = 0;
};

// FfnExec::load(model, layer, geom, with_shared) (layer_exec.hpp:111-140) over a GGUF: the layer's planes on the
// device and the exec that runs the block on them, kept together (the planes outlive no exec that uses them).
struct GgufFfn {
    std::unique_ptr<GgufLayer> planes;
    FfnExec exec;

    static GgufFfn load(const Gguf& model, int layer, bool with_shared, int max_tokens, cudaStream_t stream, int k = 0) {
        GgufFfn f;
        f.planes = GgufLayer::load(model, layer, with_shared, k);
        f.exec = FfnExec::load(f.planes->desc(), max_tokens, with_shared, stream);
        return f;
    }
};

}  // namespace smoe

#endif
