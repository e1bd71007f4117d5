// The admission rules of the VRAM expert tier (smoe::Residency, include/smoe_stream.hpp; the reference's contract
// include/strata/core/expert_cache.hpp:130-165): host only, no GPU.
#include "smoe_stream.hpp"

#include <cstdio>

static int fails = 0;
#define EXPECT(c)                                                   \
    do {                                                            \
        if (!(c)) {                                                 \
            std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #c); \
            fails++;                                                \
        }                                                           \
    } while (0)

int main() {
    // global admission: slots in arrival order, never evicted, full -> -1, a resident expert keeps its slot
    smoe::Residency r(4, 3, 8);
    EXPECT(r.admit(0, 5) == 0);
    EXPECT(r.admit(2, 1) == 1);
    EXPECT(r.admit(0, 5) == 0);
    EXPECT(r.admit(1, 7) == 2);
    EXPECT(r.admit(1, 6) == 3);
    EXPECT(r.admit(1, 0) == -1);
    EXPECT(r.slot_of(1, 0) == -1 && r.slot_of(2, 1) == 1);
    EXPECT(r.resident() == 4);
    // bounds: a bad layer or expert is not resident and is never admitted
    EXPECT(r.slot_of(-1, 0) == -1 && r.slot_of(3, 0) == -1 && r.slot_of(0, 8) == -1);
    EXPECT(r.admit(3, 0) == -1 && r.admit(0, -1) == -1);
    // per-layer admission: layer l takes [l q, (l + 1) q), q = slots / layers, the last layer the remainder
    smoe::Residency p(10, 3, 16);
    p.set_per_layer_admission(true);
    int64_t lo, hi;
    p.layer_slot_range(0, lo, hi);
    EXPECT(lo == 0 && hi == 3);
    p.layer_slot_range(2, lo, hi);
    EXPECT(lo == 6 && hi == 10);
    EXPECT(p.admit(1, 0) == 3 && p.admit(1, 1) == 4 && p.admit(1, 2) == 5);
    EXPECT(p.admit(1, 3) == -1);          // layer 1's range is full although other slots are free
    EXPECT(p.admit(0, 9) == 0);
    for (int e = 0; e < 4; e++) EXPECT(p.admit(2, e) == 6 + e);
    EXPECT(p.admit(2, 4) == -1);
    std::printf("residency: %s\n", fails ? "FAIL" : "ok");
    return fails;
}
