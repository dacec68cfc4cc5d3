// expert_tier.hpp -- residency policy of the device expert tier: a fixed
// number of equal VRAM slots holding copies of host expert blobs, least
// recently used out first.
//
// The tier is the device level above an ExpertStore (reference
// src/store/expert_store.hpp:71-175): the caller binds each RAM slot's blob
// (host start, bytes, generation -- the generation changes whenever the RAM
// slot is refilled, as on the REPIN events of src/store/expert_store.cpp:
// 306-316), and moe_block calls then find their weight arrays inside bound
// blobs.  A blob that is resident is read from its VRAM slot; one that is
// not is streamed into a slot (the least recently used blob that the current
// call does not use gives its slot up), overlapped with the compute of the
// call's resident experts.
//
// Host-only C++ (no CUDA): the library owns the slot arena and the copies;
// this class only decides.  tests/test_tier_policy.cpp drives it directly.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <vector>

namespace mvb {

struct TierEntry {
    uintptr_t host = 0;     // start of the bound host blob
    size_t bytes = 0;
    uint64_t generation = 0;
    int slot = -1;          // VRAM slot holding a current copy, or -1
    uint64_t last_use = 0;  // policy clock of the last call that used it
    uint64_t call = 0;      // id of the last call that used it
};

struct TierStats {
    uint64_t hits = 0, misses = 0, evictions = 0, bytes_in = 0, overflow = 0;
    uint64_t overflow_bytes = 0; // blobs uploaded for the call only
};

class TierPolicy {
  public:
    // nslots slots of slot_bytes each; drops every residency.
    void configure(int nslots, size_t slot_bytes) {
        slot_bytes_ = slot_bytes;
        owner_.assign(static_cast<size_t>(nslots > 0 ? nslots : 0), 0);
        for (auto &kv : entries_)
            kv.second.slot = -1;
    }
    int nslots() const { return static_cast<int>(owner_.size()); }
    size_t slot_bytes() const { return slot_bytes_; }

    // Binds (or re-binds) a blob.  A new generation or size drops the stale
    // copy.  Bound ranges do not overlap: an overlapping older binding is
    // removed.  Returns false for a blob that can never fit a slot (it stays
    // bound; its arrays are uploaded per call).
    bool bind(uintptr_t host, size_t bytes, uint64_t generation) {
        auto it = entries_.find(host);
        if (it != entries_.end() &&
            (it->second.bytes != bytes || it->second.generation != generation)) {
            drop(it->second);
            entries_.erase(it);
            it = entries_.end();
        }
        if (it == entries_.end()) {
            for (auto jt = entries_.begin(); jt != entries_.end();) {
                const uintptr_t s = jt->first, e = s + jt->second.bytes;
                if (s < host + bytes && host < e) {
                    drop(jt->second);
                    jt = entries_.erase(jt);
                } else {
                    ++jt;
                }
            }
            TierEntry t;
            t.host = host;
            t.bytes = bytes;
            t.generation = generation;
            entries_[host] = t;
        }
        return bytes <= slot_bytes_;
    }

    bool unbind(uintptr_t host) {
        auto it = entries_.find(host);
        if (it == entries_.end())
            return false;
        drop(it->second);
        entries_.erase(it);
        return true;
    }

    void clear() {
        entries_.clear();
        for (auto &o : owner_)
            o = 0;
    }

    // The bound blob containing [addr, addr + len), or nullptr.
    TierEntry *find(uintptr_t addr, size_t len) {
        auto it = entries_.upper_bound(addr);
        if (it == entries_.begin())
            return nullptr;
        --it;
        if (addr >= it->first && addr + len <= it->first + it->second.bytes)
            return &it->second;
        return nullptr;
    }

    // Starts a call: the blobs it acquires are kept until the next one.
    void begin_call() { call_ = ++clock_; }

    // Makes `e` resident for the current call.  Returns its slot, with
    // *copy = true when the blob must be copied into it first (only on the
    // call's first acquire of `e`), or -1 when every slot is held by a blob
    // this call already uses (or the blob is larger than a slot): the caller
    // then uploads it for this call only.
    int acquire(TierEntry &e, bool *copy) {
        *copy = false;
        if (e.call == call_)
            return e.slot; // decided earlier in this call
        e.call = call_;
        e.last_use = clock_;
        if (e.slot >= 0) {
            ++stats_.hits;
            return e.slot;
        }
        if (e.bytes > slot_bytes_ || owner_.empty()) {
            ++stats_.overflow;
            stats_.overflow_bytes += e.bytes;
            return -1;
        }
        int victim = -1;
        uint64_t oldest = ~uint64_t(0);
        for (size_t s = 0; s < owner_.size(); ++s) {
            if (owner_[s] == 0) {
                victim = static_cast<int>(s);
                break;
            }
            const TierEntry &o = entries_.at(owner_[s]);
            if (o.call == call_)
                continue; // in use by this call
            if (o.last_use < oldest) {
                oldest = o.last_use;
                victim = static_cast<int>(s);
            }
        }
        if (victim < 0) {
            ++stats_.overflow;
            stats_.overflow_bytes += e.bytes;
            return -1;
        }
        if (owner_[size_t(victim)] != 0) {
            entries_.at(owner_[size_t(victim)]).slot = -1;
            ++stats_.evictions;
        }
        owner_[size_t(victim)] = e.host;
        e.slot = victim;
        ++stats_.misses;
        stats_.bytes_in += e.bytes;
        *copy = true;
        return victim;
    }

    // A copy into `e`'s slot failed to be issued: forget the residency.
    void abandon(TierEntry &e) {
        drop(e);
    }

    const TierStats &stats() const { return stats_; }
    size_t resident_bytes() const {
        size_t b = 0;
        for (uintptr_t o : owner_)
            if (o)
                b += entries_.at(o).bytes;
        return b;
    }
    size_t bound() const { return entries_.size(); }

  private:
    void drop(TierEntry &e) {
        if (e.slot >= 0 && size_t(e.slot) < owner_.size() && owner_[size_t(e.slot)] == e.host)
            owner_[size_t(e.slot)] = 0;
        e.slot = -1;
    }

    std::map<uintptr_t, TierEntry> entries_;
    std::vector<uintptr_t> owner_; // host key of the blob in each slot, 0 = free
    size_t slot_bytes_ = 0;
    uint64_t clock_ = 0, call_ = ~uint64_t(0); // no call open
    TierStats stats_;
};

} // namespace mvb
