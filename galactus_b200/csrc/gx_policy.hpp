// Per-layer slot policy and slot ledger (host side, no CUDA).
//
// Semantics follow the reference engine exactly, because slot ids are part of
// what the remap node hands to mul_mat_id and every hit/miss decides a
// host->HBM copy:
//   - quota = capacity / (one record of every layer), capped at the expert
//     count, at least 2 (src/h4/h4-expert-cache.cpp:68-135);
//   - two segments, probation then protected, promotion on the second access,
//     demotion of the protected LRU on overflow, eviction from probation
//     (src/h4/h4-expert-cache.cpp:340-396);
//   - segment split with the probation floor and the full-residency
//     short-circuit (src/h4/h4-expert-cache.cpp:32-60, 105-124);
//   - frequency victim: least frequent, oldest on ties, never a key touched in
//     the current micro-batch, frequencies halved every 4096 accesses of a
//     layer (src/h4/h4-expert-cache.cpp:230-273, h4-expert-cache.hpp:72);
//   - slots: per-layer LIFO free list, slot 0 handed out first, release before
//     allocation (src/h4/h4-expert-store.cpp:72-80, 119-150, 197-211).
// GX_POLICY_LRU adds a single-segment LRU that the reference does not have.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace gx {

struct PolicyError : std::runtime_error {
    int code;
    PolicyError(int c, const std::string & what) : std::runtime_error(what), code(c) {}
};

struct ServeOutcome {
    bool hit = false;
    int32_t evicted = -1;   // expert evicted by this access, -1 if none
};

class SlotPolicy {
public:
    static constexpr uint32_t kDecayPeriod = 4096;
    static constexpr uint32_t kKeyCapacity = 1024;

    SlotPolicy(uint32_t first_layer, uint32_t last_layer, uint32_t experts, uint32_t used,
               const std::vector<uint64_t> & record_bytes, uint64_t capacity_bytes, double protected_fraction,
               int policy, const uint32_t * plan_quotas);

    uint32_t first_layer() const { return first_; }
    uint32_t last_layer() const { return last_; }
    uint32_t layer_count() const { return last_ - first_ + 1; }
    uint32_t experts() const { return experts_; }
    uint32_t quota_uniform() const { return quota_; }
    uint32_t quota_of(uint32_t layer) const { return L(layer).quota; }
    uint32_t protected_of(uint32_t layer) const { return L(layer).protected_quota; }
    uint32_t probation_of(uint32_t layer) const { return L(layer).probation_quota; }
    bool frequency_victim() const { return frequency_victim_; }
    bool lru() const { return lru_; }

    // Micro-batch bound: distinct experts a batch may hold on this layer.
    uint32_t batch_bound(uint32_t layer) const;

    void begin_batch(uint32_t layer);
    ServeOutcome access(uint32_t layer, uint32_t expert);
    bool resident(uint32_t layer, uint32_t expert) const;

    // slot ledger
    int32_t slot_of(uint32_t layer, uint32_t expert) const { return L(layer).slot_of[expert]; }
    int32_t allocate_slot(uint32_t layer, uint32_t expert);
    void release_slot(uint32_t layer, uint32_t expert);

    uint64_t hits() const { return hits_; }
    uint64_t accesses() const { return accesses_; }
    uint64_t cold_bytes() const { return cold_bytes_; }

private:
    enum Seg : uint8_t { kAbsent = 0, kProbation = 1, kProtected = 2 };
    struct Layer {
        std::vector<int16_t> prev, next;
        std::vector<uint8_t> seg;
        std::vector<uint16_t> freq, epoch;
        int16_t head[3] = {-1, -1, -1}, tail[3] = {-1, -1, -1};
        uint32_t size[3] = {0, 0, 0};
        uint32_t quota = 0, protected_quota = 0, probation_quota = 0;
        uint16_t cur_epoch = 1;
        uint32_t since_decay = 0;
        std::vector<int32_t> slot_of;
        std::vector<int32_t> free_slots;
    };

    Layer & L(uint32_t layer) { return layers_[layer - first_]; }
    const Layer & L(uint32_t layer) const { return layers_[layer - first_]; }
    void unlink(Layer & l, int16_t i);
    void push_back(Layer & l, int16_t i, Seg into);
    int16_t pop_front(Layer & l, Seg from);
    int16_t take_victim(Layer & l);
    void note_access(Layer & l, int16_t i);
    static void split(uint32_t quota, double fraction, uint32_t experts, uint32_t floor, uint32_t & prot,
                      uint32_t & prob);

    uint32_t first_, last_, experts_, used_;
    std::vector<uint64_t> record_bytes_;
    uint32_t quota_ = 0, protected_quota_ = 0, probation_quota_ = 0;
    bool frequency_victim_ = false;
    bool lru_ = false;
    std::vector<Layer> layers_;
    uint64_t hits_ = 0, accesses_ = 0, cold_bytes_ = 0;
};

}  // namespace gx
