// Residency policy of the device expert tier (micro-vllm_b200/csrc/expert_tier.hpp),
// host only: built and run by tests/test_tier.py.  Prints TIER-POLICY-OK.
#include <cstdio>
#include <cstdlib>

#include "../micro-vllm_b200/csrc/expert_tier.hpp"

#define CHECK(c)                                                                       \
    do {                                                                               \
        if (!(c)) {                                                                    \
            std::printf("FAILED line %d: %s\n", __LINE__, #c);                         \
            std::exit(1);                                                              \
        }                                                                              \
    } while (0)

using mvb::TierEntry;
using mvb::TierPolicy;

static int use(TierPolicy &t, uintptr_t host, bool *copy) {
    TierEntry *e = t.find(host + 16, 32); // an array inside the blob
    CHECK(e != nullptr && e->host == host);
    return t.acquire(*e, copy);
}

int main() {
    TierPolicy t;
    t.configure(2, 1000);
    const uintptr_t A = 0x10000, B = 0x20000, C = 0x30000, D = 0x40000;
    CHECK(t.bind(A, 1000, 1) && t.bind(B, 1000, 1) && t.bind(C, 800, 1));
    CHECK(!t.bind(D, 5000, 1)); // larger than a slot: stays bound, never resident
    CHECK(t.find(A + 990, 20) == nullptr);  // crosses the blob's end
    CHECK(t.find(0x50000, 8) == nullptr);   // not bound

    bool copy = false;
    // call 1: A and B are cold -> both copied in
    t.begin_call();
    const int sa = use(t, A, &copy);
    CHECK(sa >= 0 && copy);
    CHECK(use(t, A, &copy) == sa && !copy); // same call, same blob: decided once
    const int sb = use(t, B, &copy);
    CHECK(sb >= 0 && sb != sa && copy);
    // C in the same call: both slots are used by this call -> overflow
    CHECK(use(t, C, &copy) == -1 && !copy);
    CHECK(use(t, D, &copy) == -1 && !copy);
    CHECK(t.stats().misses == 2 && t.stats().hits == 0 && t.stats().overflow == 2);
    CHECK(t.resident_bytes() == 2000);

    // call 2: B hit; C evicts A (least recently used, not used by this call)
    t.begin_call();
    CHECK(use(t, B, &copy) == sb && !copy);
    CHECK(use(t, C, &copy) == sa && copy);
    CHECK(t.stats().hits == 1 && t.stats().evictions == 1);
    CHECK(t.find(A, 8)->slot == -1);

    // call 3: A again -> evicts B (C used more recently)
    t.begin_call();
    CHECK(use(t, C, &copy) == sa && !copy);
    t.begin_call();
    CHECK(use(t, A, &copy) == sb && copy);
    CHECK(t.find(B, 8)->slot == -1 && t.find(C, 8)->slot == sa);

    // a refilled RAM slot (new generation) drops its device copy
    CHECK(t.bind(C, 800, 2));
    CHECK(t.find(C, 8)->slot == -1);
    t.begin_call();
    CHECK(use(t, C, &copy) >= 0 && copy);
    // the same generation again keeps it
    CHECK(t.bind(C, 800, 2));
    CHECK(t.find(C, 8)->slot >= 0);

    // an overlapping binding replaces the old one and frees its slot
    const int sc = t.find(C, 8)->slot;
    CHECK(t.bind(C + 400, 800, 1));
    CHECK(t.find(C, 8) == nullptr && t.find(C + 400, 8) != nullptr);
    t.begin_call();
    CHECK(use(t, C + 400, &copy) == sc && copy); // the freed slot, no eviction
    const uint64_t ev = t.stats().evictions;
    CHECK(ev == 2);

    // unbind frees the slot; reconfigure drops every residency
    CHECK(t.unbind(A) && !t.unbind(A));
    CHECK(t.resident_bytes() == 800);
    t.configure(3, 1000);
    CHECK(t.resident_bytes() == 0 && t.find(C + 400, 8)->slot == -1);
    std::printf("TIER-POLICY-OK\n");
    return 0;
}
