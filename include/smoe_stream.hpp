// smoe_stream.hpp - streaming routed experts from the pack on disk into HBM (host side, over the C ABI).
//
//   smoe::NativeExperts  - the pack's expert file: native_experts.txt (one line per layer: layer, gate/up type, down
//                          type, byte offset, blob bytes; header "# strata native experts vN ... (n_expert E)")
//                          over experts.bin, whose layers follow each other and whose experts follow each other
//                          inside a layer.  pick(layer, expert) -> the blob's file offset and formats; blob() maps
//                          it.  Same file format, refusals and offsets as the reference's reader
//                          (metal/src/pack.cpp:367-416, used by run_routed_expert :840-860).
//   smoe::Residency      - the (layer, expert) -> slot table of the VRAM expert tier and its admission rule
//                          (include/strata/core/expert_cache.hpp:72-150): a slot is claimed once and never
//                          evicted; with per-layer admission layer l may only take slots [l q, (l + 1) q),
//                          q = slots / n_layers, the last layer taking the remainder.  Pure host code.
//   smoe::ExpertCache    - that table plus the device slot arena (n_slots x blob bytes, allocated once at open),
//                          its device copy of the table (int32 [n_layers][n_expert], the res_row of
//                          smoe_moe_hit_select), asynchronous fills from host blobs through a ring of pinned
//                          staging buffers, and a byte-for-byte verification of a slot.
//
// Header-only; link libsmoe.so and the CUDA runtime.  Throws smoe::Error like smoe.hpp.
#ifndef SMOE_STREAM_HPP
#define SMOE_STREAM_HPP

#include "smoe.hpp"

#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace smoe {

class NativeExperts {
public:
    struct Pick {
        int gu_type = 0, d_type = 0;
        uint64_t file_off = 0, blob_bytes = 0;
        int64_t n_expert = 0;
    };

    NativeExperts() = default;
    NativeExperts(const NativeExperts&) = delete;
    NativeExperts& operator=(const NativeExperts&) = delete;
    ~NativeExperts() { unmap(); }

    // Reads pack_dir/native_experts.txt and maps pack_dir/experts.bin read-only.  Throws on a malformed index.
    void open(const std::string& pack_dir) {
        parse(pack_dir + "/native_experts.txt");
        const std::string bin = pack_dir + "/experts.bin";
        fd_ = ::open(bin.c_str(), O_RDONLY);
        if (fd_ < 0) throw Error(SMOE_INVALID_ARG, "experts.bin is missing in " + pack_dir);
        struct stat st;
        if (fstat(fd_, &st) != 0) throw Error(SMOE_INVALID_ARG, "experts.bin: cannot stat");
        size_ = (uint64_t) st.st_size;
        if (size_ > 0) {
            void* p = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
            if (p == MAP_FAILED) throw Error(SMOE_INVALID_ARG, "experts.bin: cannot map");
            map_ = static_cast<const uint8_t*>(p);
        }
    }

    int64_t n_expert() const { return n_expert_; }
    int version() const { return version_; }

    // pick_native_expert (pack.cpp:368-416): the layer's line, its offset checked against the layers before it.
    Pick pick(int64_t layer, int64_t expert) const {
        if (expert < 0 || expert >= n_expert_)
            throw Error(SMOE_INVALID_ARG, "expert " + std::to_string(expert) + " is outside 0.." +
                                              std::to_string(n_expert_ - 1));
        const Line* row = find(layer);
        if (!row) throw Error(SMOE_INVALID_ARG, "native_experts.txt: layer " + std::to_string(layer) + " is missing or not contiguous");
        uint64_t at = 0;
        for (int64_t l = 0; l <= layer; ++l) {
            const Line* step = find(l);
            if (!step || step->offset != at)
                throw Error(SMOE_INVALID_ARG, "native_experts.txt: layer " + std::to_string(l) + " is missing or not contiguous");
            at += step->bytes * (uint64_t) n_expert_;
        }
        Pick p;
        p.gu_type = row->gu;
        p.d_type = row->d;
        p.file_off = row->offset + (uint64_t) expert * row->bytes;
        p.blob_bytes = row->bytes;
        p.n_expert = n_expert_;
        return p;
    }

    // The blob's bytes inside the mapped experts.bin (a pointer into the mapping, valid while this object lives).
    const uint8_t* blob(const Pick& p) const {
        if (!map_ || p.file_off + p.blob_bytes > size_)
            throw Error(SMOE_INVALID_ARG, "experts.bin is shorter than native_experts.txt says");
        return map_ + p.file_off;
    }

private:
    struct Line {
        int64_t layer;
        int gu, d;
        uint64_t offset, bytes;
    };

    const Line* find(int64_t layer) const {
        const Line* r = nullptr;
        for (const Line& l : lines_)
            if (l.layer == layer) r = &l;
        return r;
    }

    void parse(const std::string& path) {
        FILE* in = std::fopen(path.c_str(), "rb");
        if (!in) throw Error(SMOE_INVALID_ARG, "cannot open " + path);
        char buf[1024];
        std::string err;
        while (err.empty() && std::fgets(buf, sizeof buf, in)) {
            size_t len = std::strlen(buf);
            while (len > 0 && (buf[len - 1] == '\n' || buf[len - 1] == '\r')) buf[--len] = '\0';
            if (len == 0) continue;
            if (buf[0] == '#') {
                static const char tag[] = "# strata native experts v";
                if (std::strncmp(buf, tag, sizeof tag - 1) == 0) version_ = std::atoi(buf + (sizeof tag - 1));
                const char* at = std::strstr(buf, "(n_expert ");
                if (at) n_expert_ = std::atoll(at + 10);
                continue;
            }
            long long layer = -1;
            int gu = 0, d = 0;
            unsigned long long off = 0, bytes = 0;
            if (std::sscanf(buf, "%lld %d %d %llu %llu", &layer, &gu, &d, &off, &bytes) != 5 || layer < 0) {
                err = std::string("native_experts.txt: a malformed line: ") + buf;
                break;
            }
            if (find(layer)) {
                err = "native_experts.txt: layer " + std::to_string(layer) + " is repeated";
                break;
            }
            lines_.push_back(Line{(int64_t) layer, gu, d, (uint64_t) off, (uint64_t) bytes});
        }
        std::fclose(in);
        if (!err.empty()) throw Error(SMOE_INVALID_ARG, err);
        if (version_ > 4)
            throw Error(SMOE_UNSUPPORTED, "native_experts.txt is v" + std::to_string(version_) + "; this loader reads up to v4");
        if (n_expert_ <= 0) throw Error(SMOE_INVALID_ARG, "native_experts.txt does not say n_expert");
    }

    void unmap() {
        if (map_) munmap(const_cast<uint8_t*>(map_), size_);
        if (fd_ >= 0) ::close(fd_);
        map_ = nullptr;
        fd_ = -1;
    }

    std::vector<Line> lines_;
    int version_ = 0;
    int64_t n_expert_ = 0;
    int fd_ = -1;
    const uint8_t* map_ = nullptr;
    uint64_t size_ = 0;
};

// The residency table and the admission rule of the VRAM expert tier.
class Residency {
public:
    static constexpr int32_t kNotResident = -1;

    Residency() = default;
    Residency(int64_t n_slots, int64_t n_layers, int64_t n_expert) { reset(n_slots, n_layers, n_expert); }

    void reset(int64_t n_slots, int64_t n_layers, int64_t n_expert) {
        if (n_slots < 0 || n_layers <= 0 || n_expert <= 0) throw Error(SMOE_INVALID_ARG, "Residency: bad sizes");
        slots_ = n_slots;
        n_layers_ = n_layers;
        n_expert_ = n_expert;
        table_.assign((size_t) (n_layers * n_expert), kNotResident);
        taken_.assign((size_t) n_layers, 0);
        next_free_ = 0;
    }

    void set_per_layer_admission(bool on) { per_layer_ = on; }
    bool per_layer_admission() const { return per_layer_; }

    // expert_cache.hpp:130-131: bounds-checked; a bad layer or expert is not resident.
    int32_t slot_of(int64_t layer, int64_t expert) const {
        if (layer < 0 || layer >= n_layers_ || expert < 0 || expert >= n_expert_) return kNotResident;
        return table_[(size_t) (layer * n_expert_ + expert)];
    }

    // The slot range layer l may admit into under per-layer admission (expert_cache.hpp:157-165).
    void layer_slot_range(int64_t layer, int64_t& lo, int64_t& hi) const {
        const int64_t q = slots_ / n_layers_;
        lo = layer * q;
        hi = layer == n_layers_ - 1 ? slots_ : lo + q;
    }

    // expert_cache.hpp:133-137: claims the next free slot for (layer, expert), or kNotResident when the cache (or
    // the layer's range) is full.  Never evicts.  An expert already resident keeps its slot.
    int32_t admit(int64_t layer, int64_t expert) {
        if (layer < 0 || layer >= n_layers_ || expert < 0 || expert >= n_expert_) return kNotResident;
        int32_t& t = table_[(size_t) (layer * n_expert_ + expert)];
        if (t != kNotResident) return t;
        int64_t slot;
        if (per_layer_) {
            int64_t lo, hi;
            layer_slot_range(layer, lo, hi);
            if (lo + taken_[(size_t) layer] >= hi) return kNotResident;
            slot = lo + taken_[(size_t) layer]++;
        } else {
            if (next_free_ >= slots_) return kNotResident;
            slot = next_free_++;
        }
        t = (int32_t) slot;
        admitted_++;
        return t;
    }

    int64_t slots() const { return slots_; }
    int64_t resident() const { return admitted_; }
    int64_t n_layers() const { return n_layers_; }
    int64_t n_expert() const { return n_expert_; }
    const int32_t* table() const { return table_.data(); }

private:
    int64_t slots_ = 0, n_layers_ = 0, n_expert_ = 0, next_free_ = 0, admitted_ = 0;
    bool per_layer_ = false;
    std::vector<int32_t> table_;
    std::vector<int64_t> taken_;
};

// The device side: slot arena, device residency table, pinned staging ring.  Set-up (open) allocates; the fills
// and the table updates are stream-ordered and allocate nothing.
class ExpertCache {
public:
    ExpertCache() = default;
    ExpertCache(const ExpertCache&) = delete;
    ExpertCache& operator=(const ExpertCache&) = delete;
    ~ExpertCache() { close(); }

    // expert_cache.hpp:79-83: n_slots x blob_bytes of device memory, checked against what the device has free.
    void open(int64_t n_slots, int64_t n_layers, int64_t n_expert, int64_t blob_bytes, int staging = 4) {
        close();
        if (n_slots <= 0 || blob_bytes <= 0 || blob_bytes % 16 || staging <= 0)
            throw Error(SMOE_INVALID_ARG, "ExpertCache::open: bad sizes (blob bytes must be a positive multiple of 16)");
        res_.reset(n_slots, n_layers, n_expert);
        size_t free_b = 0, total_b = 0;
        check_cuda(cudaMemGetInfo(&free_b, &total_b), "ExpertCache::open");
        const uint64_t want = (uint64_t) n_slots * (uint64_t) blob_bytes;
        if (want > free_b)
            throw Error(SMOE_INVALID_ARG, "ExpertCache::open: " + std::to_string(want) + " B of slots but only " +
                                              std::to_string(free_b) + " B free on the device");
        blob_ = blob_bytes;
        void* p = nullptr;
        check_cuda(cudaMalloc(&p, want), "ExpertCache::open");
        arena_ = static_cast<uint8_t*>(p);
        check_cuda(cudaMalloc(&p, (size_t) n_layers * n_expert * 4), "ExpertCache::open");
        dtable_ = static_cast<int32_t*>(p);
        check_cuda(cudaMemset(dtable_, 0xFF, (size_t) n_layers * n_expert * 4), "ExpertCache::open");  // all -1
        stage_.resize((size_t) staging);
        for (auto& s : stage_) {
            check_cuda(cudaMallocHost(reinterpret_cast<void**>(&s.host), (size_t) blob_bytes), "ExpertCache::open");
            check_cuda(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming), "ExpertCache::open");
            s.used = false;
        }
        check_cuda(cudaMallocHost(reinterpret_cast<void**>(&entry_), (size_t) n_layers * n_expert * 4), "ExpertCache::open");
        check_cuda(cudaDeviceSynchronize(), "ExpertCache::open");
    }

    void close() {
        for (auto& s : stage_) {
            if (s.done) {
                cudaEventSynchronize(s.done);
                cudaEventDestroy(s.done);
            }
            if (s.host) cudaFreeHost(s.host);
        }
        stage_.clear();
        if (entry_) cudaFreeHost(entry_);
        if (dtable_) cudaFree(dtable_);
        if (arena_) cudaFree(arena_);
        entry_ = nullptr;
        dtable_ = nullptr;
        arena_ = nullptr;
    }

    bool valid() const { return arena_ != nullptr; }
    Residency& residency() { return res_; }
    const Residency& residency_const() const { return res_; }
    int64_t slots() const { return res_.slots(); }
    int64_t blob_bytes() const { return blob_; }
    uint8_t* arena() const { return arena_; }
    uint8_t* device_slot(int32_t slot) const {
        if (slot < 0 || slot >= res_.slots()) throw Error(SMOE_INVALID_ARG, "ExpertCache: slot out of range");
        return arena_ + (size_t) slot * (size_t) blob_;
    }
    // The device residency row of one layer: int32 [n_expert], slot or -1 (the res_row of smoe_moe_hit_select).
    const int32_t* device_row(int64_t layer) const { return dtable_ + (size_t) layer * (size_t) res_.n_expert(); }

    // Admits (layer, expert) if it is not resident and copies its blob (host memory, `bytes` <= blob_bytes) into
    // the new slot on `stream`, then publishes the slot in the device table on the same stream, so a kernel
    // queued after it on that stream sees both.  Returns the slot, or -1 when the cache is full (nothing is
    // queued).  The host bytes are copied into a pinned staging buffer first: the caller's memory (a mapped file)
    // may be reused as soon as this returns.
    int32_t ensure(int64_t layer, int64_t expert, const uint8_t* host_blob, int64_t bytes, cudaStream_t stream) {
        if (!valid()) throw Error(SMOE_INVALID_ARG, "ExpertCache: not open");
        if (!stream) throw Error(SMOE_INVALID_ARG, "ExpertCache::ensure: a non-null stream is required");
        if (bytes <= 0 || bytes > blob_) throw Error(SMOE_INVALID_ARG, "ExpertCache::ensure: blob larger than a slot");
        const int32_t have = res_.slot_of(layer, expert);
        if (have != Residency::kNotResident) return have;
        const int32_t slot = res_.admit(layer, expert);
        if (slot == Residency::kNotResident) return slot;
        Stage& s = stage_[next_stage_];
        next_stage_ = (next_stage_ + 1) % stage_.size();
        if (s.used) check_cuda(cudaEventSynchronize(s.done), "ExpertCache::ensure");  // its previous copy is done
        std::memcpy(s.host, host_blob, (size_t) bytes);
        check_cuda(cudaMemcpyAsync(device_slot(slot), s.host, (size_t) bytes, cudaMemcpyHostToDevice, stream),
                   "ExpertCache::ensure");
        const size_t idx = (size_t) (layer * res_.n_expert() + expert);
        entry_[idx] = slot;
        check_cuda(cudaMemcpyAsync(dtable_ + idx, entry_ + idx, 4, cudaMemcpyHostToDevice, stream), "ExpertCache::ensure");
        check_cuda(cudaEventRecord(s.done, stream), "ExpertCache::ensure");
        s.used = true;
        fills_++;
        return slot;
    }

    // expert_cache.hpp:187-190: reads the slot back and compares it with the host blob byte for byte.
    bool verify_slot(int32_t slot, const uint8_t* host_blob, int64_t bytes) const {
        std::vector<uint8_t> back((size_t) bytes);
        check_cuda(cudaDeviceSynchronize(), "ExpertCache::verify_slot");
        check_cuda(cudaMemcpy(back.data(), device_slot(slot), (size_t) bytes, cudaMemcpyDeviceToHost),
                   "ExpertCache::verify_slot");
        return std::memcmp(back.data(), host_blob, (size_t) bytes) == 0;
    }

    int64_t fills() const { return fills_; }

private:
    struct Stage {
        uint8_t* host = nullptr;
        cudaEvent_t done = nullptr;
        bool used = false;
    };
    Residency res_;
    int64_t blob_ = 0, fills_ = 0;
    uint8_t* arena_ = nullptr;
    int32_t* dtable_ = nullptr;
    int32_t* entry_ = nullptr;  // pinned host mirror of the table: the source of each published entry
    std::vector<Stage> stage_;
    size_t next_stage_ = 0;
};

}  // namespace smoe

#endif
