#include "gx_policy.hpp"

#include <algorithm>

#include "../../include/galactus_b200.h"

namespace gx {

namespace {
constexpr uint64_t kRecordAlign = 16384;
}

// Segment split of one layer (src/h4/h4-expert-cache.cpp:32-60): at full
// residency both segments equal the quota (no eviction can ever happen);
// otherwise protected = quota*fraction clamped to [1, quota-1], and the
// probation segment is raised to `floor` when asked.
void SlotPolicy::split(uint32_t quota, double fraction, uint32_t experts, uint32_t floor, uint32_t & prot,
                       uint32_t & prob) {
    if (quota >= experts) {
        prot = quota;
        prob = quota;
        return;
    }
    prot = static_cast<uint32_t>(static_cast<double>(quota) * fraction);
    if (prot < 1) prot = 1;
    if (prot > quota - 1) prot = quota - 1;
    prob = quota - prot;
    if (prob < floor) {
        prob = std::min(quota - 1, floor);
        prot = quota - prob;
    }
}

SlotPolicy::SlotPolicy(uint32_t first_layer, uint32_t last_layer, uint32_t experts, uint32_t used,
                       const std::vector<uint64_t> & record_bytes, uint64_t capacity_bytes, double protected_fraction,
                       int policy, const uint32_t * plan_quotas)
    : first_(first_layer), last_(last_layer), experts_(experts), used_(used), record_bytes_(record_bytes) {
    if (first_layer > last_layer) throw PolicyError(GX_ERR_INVALID, "profile: inverted layer range");
    if (experts == 0 || experts > kKeyCapacity) throw PolicyError(GX_ERR_INVALID, "profile: experts outside [1,1024]");
    if (used == 0 || used > experts) throw PolicyError(GX_ERR_INVALID, "profile: inconsistent experts used");
    if (record_bytes.size() != layer_count()) throw PolicyError(GX_ERR_INVALID, "profile: record table size");
    for (uint64_t r : record_bytes)
        if (r == 0 || r % kRecordAlign != 0) throw PolicyError(GX_ERR_INVALID, "profile: record not a multiple of 16 KiB");
    if (policy < GX_POLICY_AUTO || policy > GX_POLICY_LRU) throw PolicyError(GX_ERR_INVALID, "unknown policy");
    if (capacity_bytes == 0) throw PolicyError(GX_ERR_INVALID, "policy: zero-byte arena");
    lru_ = policy == GX_POLICY_LRU;
    if (!lru_ && (protected_fraction <= 0.0 || protected_fraction >= 1.0))
        throw PolicyError(GX_ERR_INVALID, "policy: protected share outside the open unit interval");

    uint64_t one_of_each = 0;
    for (uint64_t r : record_bytes) one_of_each += r;
    uint64_t q = capacity_bytes / one_of_each;
    if (q == 0) throw PolicyError(GX_ERR_INVALID, "policy: arena smaller than one record per layer");
    if (q > experts) q = experts;
    quota_ = static_cast<uint32_t>(q);
    if (quota_ < 2) throw PolicyError(GX_ERR_INVALID, "quota below 2 slots per layer");

    const bool sel_plan = policy == GX_POLICY_AUTO || policy == GX_POLICY_PLAN;
    const bool sel_freq = policy == GX_POLICY_AUTO || policy == GX_POLICY_FREQUENCY;
    layers_.resize(layer_count());
    if (lru_) {
        protected_quota_ = 0;
        probation_quota_ = quota_;
    } else {
        frequency_victim_ = sel_freq && quota_ < experts;
        split(quota_, protected_fraction, experts, 0, protected_quota_, probation_quota_);
        if ((sel_plan || sel_freq) && quota_ < experts && probation_quota_ < used) {
            split(quota_, protected_fraction, experts, std::min(quota_ - 1, used), protected_quota_, probation_quota_);
        }
    }
    for (auto & l : layers_) {
        l.quota = quota_;
        l.protected_quota = protected_quota_;
        l.probation_quota = probation_quota_;
    }
    // per-layer quotas from a cache plan, inside the budget the uniform quota
    // buys (src/h4/h4-expert-cache.cpp:137-202)
    if (plan_quotas != nullptr && sel_plan && !lru_ && quota_ < experts) {
        const uint64_t budget = static_cast<uint64_t>(quota_) * one_of_each;
        uint64_t spent = 0;
        for (uint32_t i = 0; i < layer_count(); ++i) {
            if (plan_quotas[i] < 2 || plan_quotas[i] > experts)
                throw PolicyError(GX_ERR_INVALID, "cache plan: a layer quota outside [2, experts]");
            spent += static_cast<uint64_t>(plan_quotas[i]) * record_bytes[i];
        }
        if (spent > budget) throw PolicyError(GX_ERR_INVALID, "cache plan: quotas exceed the arena budget");
        for (uint32_t i = 0; i < layer_count(); ++i) {
            Layer & l = layers_[i];
            l.quota = plan_quotas[i];
            split(l.quota, protected_fraction, experts, probation_quota_, l.protected_quota, l.probation_quota);
        }
    }
    for (auto & l : layers_) {
        l.prev.assign(experts, -1);
        l.next.assign(experts, -1);
        l.seg.assign(experts, kAbsent);
        l.freq.assign(experts, 0);
        l.epoch.assign(experts, 0);
        l.slot_of.assign(experts, -1);
        l.free_slots.clear();
        for (int32_t s = static_cast<int32_t>(l.quota) - 1; s >= 0; --s) l.free_slots.push_back(s);
    }
}

uint32_t SlotPolicy::batch_bound(uint32_t layer) const {
    const Layer & l = L(layer);
    return std::min(l.quota, l.probation_quota);
}

void SlotPolicy::unlink(Layer & l, int16_t i) {
    const uint8_t s = l.seg[i];
    if (l.prev[i] >= 0) l.next[l.prev[i]] = l.next[i]; else l.head[s] = l.next[i];
    if (l.next[i] >= 0) l.prev[l.next[i]] = l.prev[i]; else l.tail[s] = l.prev[i];
    l.prev[i] = l.next[i] = -1;
    l.seg[i] = kAbsent;
    --l.size[s];
}

void SlotPolicy::push_back(Layer & l, int16_t i, Seg into) {
    l.prev[i] = l.tail[into];
    l.next[i] = -1;
    l.seg[i] = into;
    if (l.tail[into] >= 0) l.next[l.tail[into]] = i; else l.head[into] = i;
    l.tail[into] = i;
    ++l.size[into];
}

int16_t SlotPolicy::pop_front(Layer & l, Seg from) {
    const int16_t i = l.head[from];
    if (i >= 0) unlink(l, i);
    return i;
}

void SlotPolicy::begin_batch(uint32_t layer) {
    if (layer < first_ || layer > last_) return;
    ++L(layer).cur_epoch;
}

void SlotPolicy::note_access(Layer & l, int16_t i) {
    if (!frequency_victim_) return;
    l.epoch[i] = l.cur_epoch;
    if (l.freq[i] < 0xFFFFu) ++l.freq[i];
    if (++l.since_decay >= kDecayPeriod) {
        l.since_decay = 0;
        for (auto & f : l.freq) f = static_cast<uint16_t>(f >> 1);
    }
}

int16_t SlotPolicy::take_victim(Layer & l) {
    if (!frequency_victim_) return pop_front(l, kProbation);
    int16_t worst = -1;
    uint16_t worst_f = 0;
    for (int16_t i = l.head[kProbation]; i >= 0; i = l.next[i]) {
        if (l.epoch[i] == l.cur_epoch) continue;
        if (worst < 0 || l.freq[i] < worst_f) {
            worst = i;
            worst_f = l.freq[i];
        }
    }
    if (worst < 0) return pop_front(l, kProbation);
    unlink(l, worst);
    return worst;
}

ServeOutcome SlotPolicy::access(uint32_t layer, uint32_t expert) {
    Layer & l = L(layer);
    const int16_t e = static_cast<int16_t>(expert);
    ServeOutcome out;
    ++accesses_;
    note_access(l, e);
    if (lru_) {
        if (l.seg[e] == kProbation) {
            unlink(l, e);
            push_back(l, e, kProbation);
            ++hits_;
            out.hit = true;
            return out;
        }
        cold_bytes_ += record_bytes_[layer - first_];
        push_back(l, e, kProbation);
        if (l.size[kProbation] > l.quota) {
            const int16_t d = pop_front(l, kProbation);
            if (d >= 0) out.evicted = d;
        }
        return out;
    }
    if (l.seg[e] == kProtected) {
        unlink(l, e);
        push_back(l, e, kProtected);
        ++hits_;
        out.hit = true;
        return out;
    }
    if (l.seg[e] == kProbation) {
        unlink(l, e);
        push_back(l, e, kProtected);
        if (l.size[kProtected] > l.protected_quota) {
            const int16_t demoted = pop_front(l, kProtected);
            if (demoted >= 0) {
                push_back(l, demoted, kProbation);
                if (l.size[kProbation] > l.probation_quota) {
                    const int16_t d = take_victim(l);
                    if (d >= 0) out.evicted = d;
                }
            }
        }
        ++hits_;
        out.hit = true;
        return out;
    }
    cold_bytes_ += record_bytes_[layer - first_];
    push_back(l, e, kProbation);
    if (l.size[kProbation] > l.probation_quota) {
        const int16_t d = take_victim(l);
        if (d >= 0) out.evicted = d;
    }
    return out;
}

bool SlotPolicy::resident(uint32_t layer, uint32_t expert) const {
    if (layer < first_ || layer > last_ || expert >= experts_) return false;
    return L(layer).seg[expert] != kAbsent;
}

int32_t SlotPolicy::allocate_slot(uint32_t layer, uint32_t expert) {
    Layer & l = L(layer);
    if (l.free_slots.empty())
        throw PolicyError(GX_ERR_SLOTS, "free list exhausted on layer " + std::to_string(layer) + " (slot leak)");
    const int32_t s = l.free_slots.back();
    l.free_slots.pop_back();
    l.slot_of[expert] = s;
    return s;
}

void SlotPolicy::release_slot(uint32_t layer, uint32_t expert) {
    Layer & l = L(layer);
    int32_t & s = l.slot_of[expert];
    if (s >= 0) {
        l.free_slots.push_back(s);
        s = -1;
    }
}

}  // namespace gx
