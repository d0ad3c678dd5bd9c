// Cache plan: per-layer slot quotas from measured miss curves (host only).
//
// A plan file (the reference's text format, src/h4/h4-cache-plan.cpp:31-86)
// holds, per layer, the misses a recorded route trace took at every quota
// 0..experts. The allocator (src/h4/h4-cache-plan.hpp:99-117, .cpp:146-223)
// spends a byte budget where a slot removes the most misses: every layer
// starts at `floor`; repeatedly, among the layers whose best step still fits
// the budget, the one with the steepest average fall of misses per byte
// (over any run of consecutive slots, i.e. along the concave envelope of its
// curve) takes that run; ties go to the lowest layer. The engine applies it
// with the budget the uniform quota buys and floor = uniform probation + 1
// (src/h4/h4-expert-cache.cpp:151-163), so a plan only moves slots between
// layers. The result must equal the reference's quota for quota, so the
// selection rule (strict comparison, lowest index first) is the reference's.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <new>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/galactus_b200.h"

struct gx_cache_plan {
    std::string arch, source;
    uint32_t first_layer = 0, last_layer = 0, experts = 0, used = 0;
    std::vector<std::vector<uint32_t>> curves;   // [layer][quota 0..experts] misses
};

namespace {

bool parse_plan(std::istream & in, gx_cache_plan & p, std::string & why) {
    std::string magic;
    int version = 0;
    if (!(in >> magic >> version) || magic != "galactus-cache-plan" || version != 1) {
        why = "unknown header";
        return false;
    }
    bool ended = false;
    std::string key;
    while (in >> key) {
        if (key == "arch") in >> p.arch;
        else if (key == "first_layer") in >> p.first_layer;
        else if (key == "last_layer") in >> p.last_layer;
        else if (key == "experts") in >> p.experts;
        else if (key == "used") in >> p.used;
        else if (key == "source") in >> p.source;
        else if (key == "tokens") {
            uint64_t t = 0;
            in >> t;
        } else if (key == "curve") {
            uint32_t layer = 0;
            in >> layer;
            if (layer != p.first_layer + (uint32_t)p.curves.size()) {
                why = "curves not contiguous";
                return false;
            }
            if (p.experts == 0) {
                why = "curve before the expert count";
                return false;
            }
            std::vector<uint32_t> row((size_t)p.experts + 1);
            for (auto & v : row) {
                if (!(in >> v)) {
                    why = "curve too short";
                    return false;
                }
            }
            p.curves.push_back(std::move(row));
        } else if (key == "end") {
            ended = true;
            break;
        } else {
            why = "unknown key " + key;
            return false;
        }
        if (!in) {
            why = "truncated";
            return false;
        }
    }
    if (!ended) {
        why = "no 'end'";
        return false;
    }
    if (p.first_layer > p.last_layer) {
        why = "inverted layer range";
        return false;
    }
    if (p.curves.size() != (size_t)(p.last_layer - p.first_layer + 1)) {
        why = "curve count does not match the layer range";
        return false;
    }
    return true;
}

// the best average fall per byte from quota `here`, over runs of 1..top-here slots
struct Step {
    double slope = 0.0;
    uint32_t take = 0;
};

Step best_run(const uint32_t * row, uint32_t len, uint32_t here, uint32_t ceiling, double cost) {
    Step s;
    const uint32_t top = ceiling < len - 1 ? ceiling : len - 1;
    if (here >= top) return s;
    for (uint32_t take = 1; take <= top - here; ++take) {
        const uint32_t a = row[here], b = row[here + take];
        if (b >= a) continue;   // a run whose end is not lower buys nothing
        const double slope = (double)(a - b) / ((double)take * cost);
        if (slope > s.slope) s = Step{slope, take};
    }
    return s;
}

}  // namespace

extern "C" {

int gx_cache_plan_load(const char * path, gx_cache_plan ** out) {
    if (path == nullptr || out == nullptr) return GX_ERR_INVALID;
    *out = nullptr;
    std::ifstream in(path);
    if (!in) return GX_ERR_INVALID;
    gx_cache_plan * p = new (std::nothrow) gx_cache_plan();
    if (p == nullptr) return GX_ERR_NOMEM;
    std::string why;
    if (!parse_plan(in, *p, why)) {
        std::fprintf(stderr, "galactus_b200: cache plan %s: %s\n", path, why.c_str());
        delete p;
        return GX_ERR_INVALID;
    }
    *out = p;
    return GX_OK;
}

void gx_cache_plan_destroy(gx_cache_plan * plan) { delete plan; }

int gx_cache_plan_info(const gx_cache_plan * p, uint32_t * first_layer, uint32_t * last_layer, uint32_t * experts,
                       uint32_t * used, char * arch, size_t arch_cap) {
    if (p == nullptr) return GX_ERR_INVALID;
    if (first_layer) *first_layer = p->first_layer;
    if (last_layer) *last_layer = p->last_layer;
    if (experts) *experts = p->experts;
    if (used) *used = p->used;
    if (arch && arch_cap > 0) {
        std::strncpy(arch, p->arch.c_str(), arch_cap - 1);
        arch[arch_cap - 1] = '\0';
    }
    return GX_OK;
}

int gx_cache_plan_curve(const gx_cache_plan * p, uint32_t layer, uint32_t * misses) {
    if (p == nullptr || misses == nullptr || layer < p->first_layer || layer > p->last_layer) return GX_ERR_INVALID;
    const auto & row = p->curves[layer - p->first_layer];
    std::memcpy(misses, row.data(), row.size() * sizeof(uint32_t));
    return GX_OK;
}

int gx_plan_layer_quotas(const uint32_t * curves, uint32_t n_layers, uint32_t curve_len, const uint64_t * record_bytes,
                         uint64_t budget, uint32_t floor, uint32_t ceiling, uint32_t * quotas) {
    if (curves == nullptr || record_bytes == nullptr || quotas == nullptr || n_layers == 0 || curve_len == 0 ||
        floor > ceiling)
        return GX_ERR_INVALID;
    uint64_t spent = 0;
    for (uint32_t i = 0; i < n_layers; ++i) {
        if (record_bytes[i] == 0) return GX_ERR_INVALID;
        quotas[i] = floor;
        spent += (uint64_t)floor * record_bytes[i];
    }
    if (spent > budget) return GX_ERR_INVALID;   // the floor alone exceeds the budget
    std::vector<Step> next(n_layers);
    for (uint32_t i = 0; i < n_layers; ++i)
        next[i] = best_run(curves + (size_t)i * curve_len, curve_len, quotas[i], ceiling, (double)record_bytes[i]);
    for (;;) {
        int pick = -1;
        double slope = 0.0;
        uint64_t cost = 0;
        for (uint32_t i = 0; i < n_layers; ++i) {
            if (next[i].take == 0) continue;
            const uint64_t c = (uint64_t)next[i].take * record_bytes[i];
            if (spent + c > budget) continue;
            if (pick < 0 || next[i].slope > slope) {   // strictly steeper: ties stay with the lower layer
                pick = (int)i;
                slope = next[i].slope;
                cost = c;
            }
        }
        if (pick < 0) break;
        quotas[pick] += next[pick].take;
        spent += cost;
        next[pick] = best_run(curves + (size_t)pick * curve_len, curve_len, quotas[pick], ceiling,
                              (double)record_bytes[pick]);
    }
    return GX_OK;
}

int gx_policy_plan_quotas(const gx_profile * profile, uint64_t capacity_bytes, double protected_fraction,
                          const gx_cache_plan * plan, uint32_t * quotas) {
    if (profile == nullptr || plan == nullptr || quotas == nullptr || profile->record_bytes == nullptr)
        return GX_ERR_INVALID;
    if (plan->first_layer != profile->first_layer || plan->last_layer != profile->last_layer ||
        plan->experts != profile->experts)
        return GX_ERR_STATE;   // a plan for another geometry: the uniform quota applies
    // the uniform engine's quota and probation segment
    gx_policy * uni = nullptr;
    int rc = gx_policy_create(profile, capacity_bytes, protected_fraction, GX_POLICY_FREQUENCY, nullptr, &uni);
    if (rc != GX_OK) return rc;
    uint32_t q = 0, prot = 0, prob = 0;
    rc = gx_policy_quota(uni, profile->first_layer, &q, &prot, &prob);
    gx_policy_destroy(uni);
    if (rc != GX_OK) return rc;
    if (q >= profile->experts) return GX_ERR_STATE;   // full residency: nothing to move
    const uint32_t n = profile->last_layer - profile->first_layer + 1;
    uint64_t one_of_each = 0;
    for (uint32_t i = 0; i < n; ++i) one_of_each += profile->record_bytes[i];
    const uint64_t budget = (uint64_t)q * one_of_each;
    const uint32_t floor = prob + 1;
    if (floor > profile->experts) return GX_ERR_STATE;
    std::vector<uint32_t> flat;
    flat.reserve((size_t)n * (plan->experts + 1));
    for (const auto & row : plan->curves) flat.insert(flat.end(), row.begin(), row.end());
    rc = gx_plan_layer_quotas(flat.data(), n, plan->experts + 1, profile->record_bytes, budget, floor, profile->experts,
                              quotas);
    if (rc != GX_OK) return rc;
    uint64_t spent = 0;
    for (uint32_t i = 0; i < n; ++i) {
        if (quotas[i] < 2) return GX_ERR_STATE;
        spent += (uint64_t)quotas[i] * profile->record_bytes[i];
    }
    return spent <= budget ? GX_OK : GX_ERR_STATE;
}

}  // extern "C"
