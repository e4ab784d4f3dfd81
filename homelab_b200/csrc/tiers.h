// tiers.h - expert records in a fixed pool of device slots over a pinned host
// arena: the two-phase fetch of ExpertSource (crates/oominf-core/src/
// experts.rs:12-41) and the replacement policies of the expert cache
// (crates/oominf-tiers/src/policy.rs:9-129), as TieredExperts uses them for
// its device tier (crates/oominf-tiers/src/tiered.rs:1105-1116, 1155-1421,
// 1494-1510).  Host code only: the copies are cudaMemcpyAsync on a copy queue
// (one per record), ordered against compute with events.
//
// A fetch for (layer, experts): every wanted record that is resident is a hit
// (its slot address, usable now); every other one takes a slot - a free one, or
// the policy's victim among the residents this fetch does not want - and its
// copy from the host arena is queued (address returned, not usable yet).  The
// copy queue first waits for the compute issued before the fetch (a kernel
// issued earlier may still read a victim's slot); finish_fetch makes the compute
// stream wait for the queued copies, so the work issued after it may read every
// record of the fetch.  Resident experts' work issued between begin_fetch and
// finish_fetch overlaps the copies.
#pragma once

#include <cmath>
#include <cstdint>
#include <map>
#include <set>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace oomb {

// Ranks resident keys (layer * experts + expert) for eviction.
class TierPolicy {
   public:
    virtual ~TierPolicy() = default;
    // `key` was accessed (a hit or a fresh insertion) at logical time `now`.
    virtual void touch(uint32_t key, uint64_t now) = 0;
    // `key` left the cache.
    virtual void remove(uint32_t key) = 0;
    // The best victim among resident keys for which pinned(key) is false, or -1.
    template <class Pinned>
    int64_t victim(const Pinned& pinned) const {
        for (const auto& e : order_)
            if (!pinned(e.second)) return e.second;
        return -1;
    }

   protected:
    std::set<std::pair<double, uint32_t>> order_;  // ascending: the first unpinned entry is the victim
};

// Least recently used: rank = time of the last access.
class LruPolicy : public TierPolicy {
   public:
    void touch(uint32_t key, uint64_t now) override {
        auto it = last_.find(key);
        if (it != last_.end()) order_.erase({it->second, key});
        last_[key] = static_cast<double>(now);
        order_.insert({static_cast<double>(now), key});
    }
    void remove(uint32_t key) override {
        auto it = last_.find(key);
        if (it == last_.end()) return;
        order_.erase({it->second, key});
        last_.erase(it);
    }

   private:
    std::unordered_map<uint32_t, double> last_;
};

// LRFU: an access at time `now` adds 2^(now / half_life) to a key's score (an
// access count with exponential decay of half-life `half_life` accesses: small
// half-lives act like LRU, large ones like LFU), kept as log2 so it never
// overflows: log2(2^a + 2^b) = max + log2(1 + 2^(min - max)).
class LrfuPolicy : public TierPolicy {
   public:
    explicit LrfuPolicy(double half_life) : half_life_(half_life) {}
    void touch(uint32_t key, uint64_t now) override {
        const double add = static_cast<double>(now) / half_life_;
        auto it = score_.find(key);
        double s = add;
        if (it != score_.end()) {
            order_.erase({it->second, key});
            const double hi = it->second > add ? it->second : add, lo = it->second > add ? add : it->second;
            s = hi + std::log2(1.0 + std::exp2(lo - hi));
        }
        score_[key] = s;
        order_.insert({s, key});
    }
    void remove(uint32_t key) override {
        auto it = score_.find(key);
        if (it == score_.end()) return;
        order_.erase({it->second, key});
        score_.erase(it);
    }

   private:
    double half_life_;
    std::unordered_map<uint32_t, double> score_;
};

// "lru", "lfu" (LRFU with a half-life of 1e12 accesses) or "lrfu:<half_life>";
// null for anything else.
inline TierPolicy* make_policy(const char* spec) {
    const std::string s = spec ? spec : "lru";
    if (s == "lru") return new LruPolicy();
    if (s == "lfu") return new LrfuPolicy(1e12);
    if (s.rfind("lrfu:", 0) == 0) {
        char* end = nullptr;
        const double h = std::strtod(s.c_str() + 5, &end);
        if (end && *end == '\0' && h > 0.0) return new LrfuPolicy(h);
    }
    return nullptr;
}

struct TierStats {
    uint64_t requests = 0, hits = 0, misses = 0, evictions = 0, bytes_copied = 0;
};

// The device tier of one model: `slots` records of `stride` bytes at
// `device_base`, filled from the pinned host arena (record (layer, e) at
// host_base + (layer * experts + e) * stride).
struct Tier {
    const uint8_t* host_base = nullptr;
    uint8_t* device_base = nullptr;
    size_t stride = 0;
    int layers = 0, experts = 0, slots = 0;
    TierPolicy* policy = nullptr;
    cudaStream_t queue = nullptr;
    cudaEvent_t compute_ev = nullptr, copies_ev = nullptr;
    std::unordered_map<uint32_t, int> slot_of;  // resident key -> slot
    std::vector<int64_t> key_of;                // slot -> key, or -1 (free)
    std::vector<int> free_slots;
    uint64_t now = 0;
    bool open = false;
    TierStats stats;
};

}  // namespace oomb
