// C-ABI of galactus_b200: slot policy, HBM slot arena with its pinned host
// tier, the remap node, the expert kernels and the MoE layer entry point.
// No C++ exception crosses this boundary; every entry point returns GX_*.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <unordered_set>
#include <vector>

#include "../../include/galactus_b200.h"
#include "gx_formats.h"
#include "gx_kernels.h"
#include "gx_observer.hpp"
#include "gx_policy.hpp"

using gx::PolicyError;
using gx::SlotPolicy;

struct gx_policy {
    SlotPolicy impl;
    // geometry for the route observer's context lines
    uint64_t capacity = 0;
    double fraction = 0.0;
    uint32_t used = 0;
    std::vector<uint64_t> record;
    explicit gx_policy(SlotPolicy && p) : impl(std::move(p)) {}
};

namespace {

constexpr int kStageRing = 16;

struct CudaFail {
    cudaError_t err;
};

inline void ck(cudaError_t e) {
    if (e != cudaSuccess) throw CudaFail{e};
}

template <typename F>
int guarded(F && f) {
    try {
        return f();
    } catch (const PolicyError & e) {
        return e.code;
    } catch (const CudaFail & e) {
        std::fprintf(stderr, "galactus_b200: CUDA error: %s\n", cudaGetErrorString(e.err));
        return e.err == cudaErrorMemoryAllocation ? GX_ERR_NOMEM : GX_ERR_CUDA;
    } catch (const std::bad_alloc &) {
        return GX_ERR_NOMEM;
    } catch (...) {
        return GX_ERR_INVALID;
    }
}

SlotPolicy make_policy(const gx_profile & prof, uint64_t capacity, double fraction, int policy, const uint32_t * plan) {
    if (prof.record_bytes == nullptr) throw PolicyError(GX_ERR_INVALID, "profile without record table");
    if (prof.first_layer > prof.last_layer) throw PolicyError(GX_ERR_INVALID, "inverted layer range");
    const uint32_t n = prof.last_layer - prof.first_layer + 1;
    std::vector<uint64_t> rec(prof.record_bytes, prof.record_bytes + n);
    return SlotPolicy(prof.first_layer, prof.last_layer, prof.experts, prof.used, rec, capacity, fraction, policy, plan);
}

// Serve one micro-batch of one layer through the policy: the engine's
// micro-batch guard, begin_batch, one access per key in order (release of an
// evicted slot before any allocation), then the slot of every key.
// Misses are appended as (expert, slot).
int serve_policy(SlotPolicy & P, uint32_t layer, const int32_t * experts, uint32_t count, int32_t * slots,
                 uint8_t * hit_out, int32_t * evicted_out, std::vector<std::pair<int32_t, int32_t>> * misses,
                 gx_serve_stats * st) {
    if (layer < P.first_layer() || layer > P.last_layer()) return GX_ERR_INVALID;
    for (uint32_t i = 0; i < count; ++i)
        if (experts[i] < 0 || (uint32_t)experts[i] >= P.experts()) return GX_ERR_DOMAIN;
    thread_local std::vector<uint8_t> seen;
    seen.assign(P.experts(), 0);
    uint32_t distinct = 0;
    for (uint32_t i = 0; i < count; ++i)
        if (!seen[experts[i]]) { seen[experts[i]] = 1; ++distinct; }
    if (distinct > P.batch_bound(layer)) return GX_ERR_BATCH;
    gx_serve_stats local{};
    local.distinct = distinct;
    P.begin_batch(layer);
    for (uint32_t i = 0; i < count; ++i) {
        const gx::ServeOutcome o = P.access(layer, (uint32_t)experts[i]);
        if (evicted_out) evicted_out[i] = o.evicted;
        if (hit_out) hit_out[i] = o.hit ? 1 : 0;
        if (o.evicted >= 0) {
            P.release_slot(layer, (uint32_t)o.evicted);
            ++local.evictions;
        }
        if (o.hit) {
            ++local.hits;
            continue;
        }
        ++local.misses;
        const int32_t s = P.allocate_slot(layer, (uint32_t)experts[i]);
        if (misses) misses->emplace_back(experts[i], s);
    }
    for (uint32_t i = 0; i < count; ++i) {
        const int32_t s = P.slot_of(layer, (uint32_t)experts[i]);
        if (s < 0) return GX_ERR_SLOTS;  // a served key without a slot (scripts/derive-remap-strides.py:70)
        slots[i] = s;
    }
    if (st) *st = local;
    return GX_OK;
}

// The serve, with the route observer around it when a trace is open: the
// residency of every key sampled before the serve, the serve's clock, and the
// host->HBM bytes it issued (src/h4/h4-route-observer.hpp:84-128).
template <typename F>
int observed(const gx_policy * pol, uint32_t layer, const int32_t * experts, uint32_t count, uint32_t tokens,
             uint32_t k, F && serve) {
    uint64_t bytes = 0;
    if (!gx::observer_enabled()) return serve(bytes);
    const SlotPolicy & P = pol->impl;
    if ((uint64_t)tokens * k != count) {
        tokens = 1;
        k = count;
    }
    const uint64_t enter = gx::observer_now_ns();
    thread_local std::vector<uint8_t> resident;
    resident.assign(count, 0);
    const bool in_range = layer >= P.first_layer() && layer <= P.last_layer();
    for (uint32_t i = 0; i < count && in_range; ++i)
        resident[i] = experts[i] >= 0 && (uint32_t)experts[i] < P.experts() && P.slot_of(layer, (uint32_t)experts[i]) >= 0;
    const uint64_t start = gx::observer_now_ns();
    const int rc = serve(bytes);
    const uint64_t end = gx::observer_now_ns();
    if (rc == GX_OK) {
        gx::ObserverGeometry g{pol->capacity, pol->fraction, P.quota_uniform(), P.probation_of(P.first_layer()),
                               P.quota_uniform(), P.first_layer(), P.last_layer(), P.experts(), pol->used,
                               pol->record.data()};
        gx::observer_record(g, layer, tokens, k, experts, resident.data(), enter, start, end, bytes);
    }
    return rc;
}

gx_policy * make_gx_policy(const gx_profile & prof, uint64_t capacity, double fraction, int policy,
                           const uint32_t * plan) {
    gx_policy * p = new gx_policy(make_policy(prof, capacity, fraction, policy, plan));
    p->capacity = capacity;
    p->fraction = fraction;
    p->used = prof.used;
    p->record.assign(prof.record_bytes, prof.record_bytes + (prof.last_layer - prof.first_layer + 1));
    return p;
}

}  // namespace

struct gx_arena {
    gx_policy * policy = nullptr;
    int device = 0;
    std::vector<uint64_t> record, record_raw;
    std::vector<uint64_t> slab_base;    // device offset of each layer's slab
    std::vector<std::vector<uint32_t>> slot_gen;   // per layer and slot: fills so far (copies of a plan's slot mirror follow it)
    std::vector<uint64_t> host_base;    // host-tier offset of each layer's records
    uint8_t * d_arena = nullptr;
    uint64_t arena_bytes = 0;
    uint8_t * h_tier = nullptr;
    uint64_t tier_bytes = 0;
    cudaStream_t copy_stream = nullptr;
    std::vector<cudaEvent_t> ev_done, ev_copy;
    std::vector<cudaEvent_t> last_ev;   // last event after which nothing reads a layer's slab
    std::vector<int32_t> slot_scratch;  // slot ids of one micro-batch
    cudaEvent_t ev_snapshot = nullptr;
    // layer entry point scratch
    int64_t max_tokens = 0, hidden = 0, intermediate = 0;
    uint32_t used = 0;
    float * d_act = nullptr;            // [I, k, T] activations between gate/up and down
    uint8_t * d_xq = nullptr;           // quantized layer inputs, split layout, one row per token
    uint8_t * d_actq = nullptr;         // quantized activations of the down projection, one row per (token, slot)
    int32_t * d_cnt = nullptr;          // per (token, slot, Q8 block) completion counters, zero between calls
    // wave schedule (micro-batches whose distinct experts exceed the policy's
    // batch bound): per-pair inputs and outputs in wave order, outputs in pair
    // order, unit weights, gather/scatter indices (allocated on first use)
    float * d_wx = nullptr;             // [pairs, H] input row of each pair, wave order
    float * d_wy = nullptr;             // [pairs, H] down output of each pair, wave order
    float * d_wfull = nullptr;          // [pairs, H] the same in (token, slot) order
    float * d_ones = nullptr;           // [pairs] 1.0f
    float * d_shy = nullptr;            // [max_tokens, H] shared-expert output
    // tensor-core prefill: masked B tiles and block scales of every pair chunk
    uint8_t * d_mmab = nullptr;
    float * d_mmady = nullptr;
    size_t mmab_cap = 0;                // chunk-blocks the buffers hold
    int32_t * d_widx = nullptr;         // [2, pairs] token of each wave-order pair | its pair index
    int32_t * h_widx = nullptr;         // pinned staging of d_widx
    cudaEvent_t ev_widx = nullptr;
    // expert-grouped (prefill) path: per-pair outputs and the pair grouping
    float * d_y = nullptr;              // [pairs, H] down output of each (token, slot)
    int32_t * h_grp = nullptr;          // pinned staging of the grouping arrays
    int32_t * d_grp = nullptr;
    size_t grp_cap = 0;                 // ints
    cudaEvent_t ev_grp = nullptr;
    int32_t * d_ids = nullptr;          // kStageRing x (used * max_tokens) slot ids
    int32_t * h_ids = nullptr;          // pinned staging of the same
    cudaEvent_t ev_stage[kStageRing] = {};
    int stage_next = 0;
    gx_arena_stats stats{};
    bool own_tier = false;
    // kernel timing (gx_arena_timing)
    bool timing = false;
    std::vector<cudaEvent_t> tev;   // 3 per timed call
    size_t tev_used = 0;
    std::mutex mu;

    uint32_t L(uint32_t layer) const { return layer - policy->impl.first_layer(); }
};

extern "C" {

const char * gx_status_string(int status) {
    switch (status) {
        case GX_OK: return "ok";
        case GX_ERR_INVALID: return "invalid argument";
        case GX_ERR_TYPE: return "weight type without a bit-exact kernel";
        case GX_ERR_ALIGN: return "row length, base or stride not supported by the staged kernels";
        case GX_ERR_DOMAIN: return "expert id outside [0, n_expert)";
        case GX_ERR_BATCH: return "micro-batch holds more distinct experts than the probation segment";
        case GX_ERR_SLOTS: return "slot ledger exhausted or served key without a slot";
        case GX_ERR_CUDA: return "CUDA runtime error";
        case GX_ERR_TIMEOUT: return "bounded device wait ran out";
        case GX_ERR_NOMEM: return "out of memory";
        case GX_ERR_COPY: return "host->HBM copy failed";
        case GX_ERR_STATE: return "call out of order";
        case GX_ERR_DEVICE: return "a kernel reported an error";
        case GX_ERR_COMM: return "an NCCL call failed or NCCL could not be loaded";
        default: return "unknown status";
    }
}

const char * gx_version(void) { return "galactus_b200 0.1 sm_100a (bulk-TMA row tiles, dp4a integer partials)"; }

int gx_device_init(int device) {
    return guarded([&] {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return GX_ERR_CUDA;
        if (device < 0 || device >= n) return GX_ERR_INVALID;
        ck(cudaSetDevice(device));
        ck(cudaFree(nullptr));
        return GX_OK;
    });
}

int gx_device_error(int32_t * code_out) {
    return guarded([&] {
        int code = 0;
        ck(gx::read_and_clear_device_error(&code));
        if (code_out) *code_out = code;
        return GX_OK;
    });
}

// ------------------------------------------------------------------ policy

int gx_policy_create(const gx_profile * profile, uint64_t capacity_bytes, double protected_fraction, int policy,
                     const uint32_t * plan_quotas, gx_policy ** out) {
    if (profile == nullptr || out == nullptr) return GX_ERR_INVALID;
    return guarded([&] {
        *out = make_gx_policy(*profile, capacity_bytes, protected_fraction, policy, plan_quotas);
        return GX_OK;
    });
}

void gx_policy_destroy(gx_policy * policy) { delete policy; }

int gx_policy_quota(const gx_policy * policy, uint32_t layer, uint32_t * quota, uint32_t * protected_quota,
                    uint32_t * probation_quota) {
    if (policy == nullptr) return GX_ERR_INVALID;
    const SlotPolicy & P = policy->impl;
    if (layer < P.first_layer() || layer > P.last_layer()) return GX_ERR_INVALID;
    if (quota) *quota = P.quota_of(layer);
    if (protected_quota) *protected_quota = P.protected_of(layer);
    if (probation_quota) *probation_quota = P.probation_of(layer);
    return GX_OK;
}

int gx_policy_serve(gx_policy * policy, uint32_t layer, const int32_t * experts, uint32_t count, int32_t * slots_out,
                    uint8_t * hit_out, int32_t * evicted_out, gx_serve_stats * stats) {
    if (policy == nullptr || (count > 0 && (experts == nullptr || slots_out == nullptr))) return GX_ERR_INVALID;
    return guarded([&] {
        return observed(policy, layer, experts, count, 1, count, [&](uint64_t & bytes) {
            gx_serve_stats st{};
            const int rc = serve_policy(policy->impl, layer, experts, count, slots_out, hit_out, evicted_out, nullptr, &st);
            if (stats) *stats = st;
            // whole records per miss: what a reader of the backing tier would pull
            if (rc == GX_OK) bytes = (uint64_t)st.misses * policy->record[layer - policy->impl.first_layer()];
            return rc;
        });
    });
}

int32_t gx_policy_slot_of(const gx_policy * policy, uint32_t layer, uint32_t expert) {
    if (policy == nullptr) return -1;
    const SlotPolicy & P = policy->impl;
    if (layer < P.first_layer() || layer > P.last_layer() || expert >= P.experts()) return -1;
    return P.slot_of(layer, expert);
}

int gx_policy_counters(const gx_policy * policy, uint64_t * hits, uint64_t * accesses, uint64_t * cold_bytes) {
    if (policy == nullptr) return GX_ERR_INVALID;
    if (hits) *hits = policy->impl.hits();
    if (accesses) *accesses = policy->impl.accesses();
    if (cold_bytes) *cold_bytes = policy->impl.cold_bytes();
    return GX_OK;
}

// ------------------------------------------------------------------- arena

int gx_arena_destroy(gx_arena * a) {
    if (a == nullptr) return GX_OK;
    cudaSetDevice(a->device);
    if (a->copy_stream) cudaStreamSynchronize(a->copy_stream);
    for (auto e : a->ev_done) if (e) cudaEventDestroy(e);
    for (auto e : a->ev_copy) if (e) cudaEventDestroy(e);
    for (auto e : a->ev_stage) if (e) cudaEventDestroy(e);
    if (a->ev_snapshot) cudaEventDestroy(a->ev_snapshot);
    if (a->copy_stream) cudaStreamDestroy(a->copy_stream);
    if (a->d_arena) cudaFree(a->d_arena);
    if (a->d_act) cudaFree(a->d_act);
    if (a->d_ids) cudaFree(a->d_ids);
    if (a->d_xq) cudaFree(a->d_xq);
    if (a->d_actq) cudaFree(a->d_actq);
    if (a->d_cnt) cudaFree(a->d_cnt);
    if (a->d_y) cudaFree(a->d_y);
    if (a->ev_widx) cudaEventSynchronize(a->ev_widx);
    if (a->d_wx) cudaFree(a->d_wx);
    if (a->d_wy) cudaFree(a->d_wy);
    if (a->d_wfull) cudaFree(a->d_wfull);
    if (a->d_shy) cudaFree(a->d_shy);
    if (a->d_mmab) cudaFree(a->d_mmab);
    if (a->d_mmady) cudaFree(a->d_mmady);
    if (a->d_ones) cudaFree(a->d_ones);
    if (a->d_widx) cudaFree(a->d_widx);
    if (a->h_widx) cudaFreeHost(a->h_widx);
    if (a->ev_widx) cudaEventDestroy(a->ev_widx);
    if (a->d_grp) cudaFree(a->d_grp);
    if (a->h_grp) cudaFreeHost(a->h_grp);
    if (a->ev_grp) cudaEventDestroy(a->ev_grp);
    if (a->h_ids) cudaFreeHost(a->h_ids);
    for (auto e : a->tev) if (e) cudaEventDestroy(e);
    if (a->h_tier && a->own_tier) cudaFreeHost(a->h_tier);
    delete a->policy;
    delete a;
    return GX_OK;
}

int gx_arena_create(const gx_arena_config * c, gx_arena ** out) {
    if (c == nullptr || out == nullptr) return GX_ERR_INVALID;
    *out = nullptr;
    gx_arena * a = new (std::nothrow) gx_arena();
    if (a == nullptr) return GX_ERR_NOMEM;
    const int rc = guarded([&] {
        a->device = c->device;
        ck(cudaSetDevice(c->device));
        a->policy = make_gx_policy(c->profile, c->capacity_bytes, c->protected_fraction, c->policy, c->plan_quotas);
        const SlotPolicy & P = a->policy->impl;
        const uint32_t n = P.layer_count();
        a->record.assign(c->profile.record_bytes, c->profile.record_bytes + n);
        if (c->profile.record_bytes_raw)
            a->record_raw.assign(c->profile.record_bytes_raw, c->profile.record_bytes_raw + n);
        else
            a->record_raw = a->record;
        for (uint32_t i = 0; i < n; ++i)
            if (a->record_raw[i] == 0 || a->record_raw[i] > a->record[i]) return GX_ERR_INVALID;
        uint64_t off = 0, hoff = 0;
        for (uint32_t i = 0; i < n; ++i) {
            a->slab_base.push_back(off);
            a->slot_gen.emplace_back(P.quota_of(P.first_layer() + i), 0u);
            off += a->record[i] * P.quota_of(P.first_layer() + i);
            a->host_base.push_back(hoff);
            hoff += a->record[i] * P.experts();
        }
        a->arena_bytes = off;
        a->tier_bytes = hoff;
        ck(cudaMalloc(&a->d_arena, a->arena_bytes));
        if (c->host_tier) {
            if (c->host_tier_base != nullptr) {
                a->h_tier = static_cast<uint8_t *>(c->host_tier_base);
            } else {
                ck(cudaHostAlloc(&a->h_tier, a->tier_bytes, cudaHostAllocDefault));
                a->own_tier = true;
            }
        }
        ck(cudaStreamCreateWithFlags(&a->copy_stream, cudaStreamNonBlocking));
        a->ev_done.resize(n);
        a->ev_copy.resize(n);
        for (uint32_t i = 0; i < n; ++i) {
            ck(cudaEventCreateWithFlags(&a->ev_done[i], cudaEventDisableTiming));
            ck(cudaEventCreateWithFlags(&a->ev_copy[i], cudaEventDisableTiming));
        }
        ck(cudaEventCreateWithFlags(&a->ev_snapshot, cudaEventDisableTiming));
        a->last_ev = a->ev_done;
        a->slot_scratch.resize((size_t)std::max<int64_t>(1, (int64_t)c->profile.used * std::max<int64_t>(1, c->max_tokens)));
        a->max_tokens = c->max_tokens;
        a->used = c->profile.used;
        a->hidden = c->hidden;
        a->intermediate = c->intermediate;
        if (c->max_tokens > 0 && c->intermediate > 0) {
            const int64_t pairs = (int64_t)c->profile.used * c->max_tokens;
            ck(cudaMalloc(&a->d_act, (size_t)(pairs * c->intermediate * sizeof(float))));
            const int64_t px = std::max(gx::act_layout(gx::GX_T_Q8_0, (int)c->hidden).pitch,
                                        gx::act_layout(gx::GX_T_Q8_K, (int)c->hidden).pitch);
            const int64_t pa = std::max(gx::act_layout(gx::GX_T_Q8_0, (int)c->intermediate).pitch,
                                        gx::act_layout(gx::GX_T_Q8_K, (int)c->intermediate).pitch);
            ck(cudaMalloc(&a->d_xq, (size_t)(c->max_tokens * px)));
            ck(cudaMalloc(&a->d_actq, (size_t)(pairs * pa)));
            ck(cudaMalloc(&a->d_cnt, (size_t)(pairs * (c->intermediate / 32 + 1) * sizeof(int32_t))));
            ck(cudaMemset(a->d_cnt, 0, (size_t)(pairs * (c->intermediate / 32 + 1) * sizeof(int32_t))));
            ck(cudaMalloc(&a->d_ids, (size_t)(kStageRing * pairs * sizeof(int32_t))));
            ck(cudaHostAlloc(&a->h_ids, (size_t)(kStageRing * pairs * sizeof(int32_t)), cudaHostAllocDefault));
            for (int i = 0; i < kStageRing; ++i) ck(cudaEventCreateWithFlags(&a->ev_stage[i], cudaEventDisableTiming));
        }
        return GX_OK;
    });
    if (rc != GX_OK) {
        gx_arena_destroy(a);
        return rc;
    }
    *out = a;
    return GX_OK;
}

void * gx_arena_host_record(gx_arena * a, uint32_t layer, uint32_t expert) {
    if (a == nullptr || a->h_tier == nullptr) return nullptr;
    const SlotPolicy & P = a->policy->impl;
    if (layer < P.first_layer() || layer > P.last_layer() || expert >= P.experts()) return nullptr;
    const uint32_t i = a->L(layer);
    return a->h_tier + a->host_base[i] + (uint64_t)expert * a->record[i];
}

int gx_load_record(gx_arena * a, uint32_t layer, uint32_t expert, const void * src, uint64_t bytes) {
    void * dst = gx_arena_host_record(a, layer, expert);
    if (dst == nullptr || src == nullptr) return a && a->h_tier == nullptr ? GX_ERR_STATE : GX_ERR_INVALID;
    if (bytes > a->record[a->L(layer)]) return GX_ERR_INVALID;
    std::memcpy(dst, src, bytes);
    return GX_OK;
}

int gx_arena_layer_view(gx_arena * a, uint32_t layer, void ** base, uint64_t * record_bytes, uint32_t * slots) {
    if (a == nullptr) return GX_ERR_INVALID;
    const SlotPolicy & P = a->policy->impl;
    if (layer < P.first_layer() || layer > P.last_layer()) return GX_ERR_INVALID;
    const uint32_t i = a->L(layer);
    if (base) *base = a->d_arena + a->slab_base[i];
    if (record_bytes) *record_bytes = a->record[i];
    if (slots) *slots = P.quota_of(layer);
    return GX_OK;
}

gx_policy * gx_arena_policy(gx_arena * a) { return a ? a->policy : nullptr; }

int gx_stats(gx_arena * a, gx_arena_stats * s) {
    if (a == nullptr || s == nullptr) return GX_ERR_INVALID;
    *s = a->stats;
    return GX_OK;
}

int gx_arena_timing(gx_arena * a, int enable) {
    if (a == nullptr) return GX_ERR_INVALID;
    std::lock_guard<std::mutex> lock(a->mu);
    a->timing = enable != 0;
    a->tev_used = 0;
    return GX_OK;
}

int gx_arena_timing_read(gx_arena * a, double * gate_up_ms, double * down_ms, uint64_t * calls) {
    if (a == nullptr) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(a->mu);
        double gu = 0.0, dn = 0.0;
        if (a->tev_used > 0) ck(cudaEventSynchronize(a->tev[a->tev_used - 1]));
        for (size_t i = 0; i + 3 <= a->tev_used; i += 3) {
            float m1 = 0.f, m2 = 0.f;
            ck(cudaEventElapsedTime(&m1, a->tev[i], a->tev[i + 1]));
            ck(cudaEventElapsedTime(&m2, a->tev[i + 1], a->tev[i + 2]));
            gu += m1;
            dn += m2;
        }
        if (gate_up_ms) *gate_up_ms = gu;
        if (down_ms) *down_ms = dn;
        if (calls) *calls = a->tev_used / 3;
        a->tev_used = 0;
        return GX_OK;
    });
}

}  // extern "C"

namespace {

// Serve a micro-batch and issue one host->HBM copy per miss on the copy
// stream. The copies start after `after` (the last consumer of the layer's
// slots) and `consumer` waits for them.
int arena_serve_impl(gx_arena * a, uint32_t layer, const int32_t * experts, uint32_t count, int32_t * slots,
                     cudaEvent_t after, cudaStream_t consumer, gx_serve_stats * st_out);

// One micro-batch of one layer through the policy, miss copies issued on the
// copy stream; `tokens` x `k` is the micro-batch shape (for the route trace).
int arena_serve(gx_arena * a, uint32_t layer, const int32_t * experts, uint32_t count, int32_t * slots,
                cudaEvent_t after, cudaStream_t consumer, gx_serve_stats * st_out, uint32_t tokens, uint32_t k) {
    return observed(a->policy, layer, experts, count, tokens, k, [&](uint64_t & bytes) {
        gx_serve_stats st{};
        const int rc = arena_serve_impl(a, layer, experts, count, slots, after, consumer, &st);
        // the trace counts whole records per miss, the unit of the reference's reader
        if (rc == GX_OK) bytes = (uint64_t)st.misses * a->record[a->L(layer)];
        if (st_out) *st_out = st;
        return rc;
    });
}

int arena_serve_impl(gx_arena * a, uint32_t layer, const int32_t * experts, uint32_t count, int32_t * slots,
                     cudaEvent_t after, cudaStream_t consumer, gx_serve_stats * st_out) {
    thread_local std::vector<std::pair<int32_t, int32_t>> misses;
    misses.clear();
    gx_serve_stats st{};
    const int rc = serve_policy(a->policy->impl, layer, experts, count, slots, nullptr, nullptr, &misses, &st);
    if (rc != GX_OK) return rc;
    const uint32_t i = a->L(layer);
    if (!misses.empty()) {
        if (a->h_tier == nullptr) return GX_ERR_STATE;
        ck(cudaStreamWaitEvent(a->copy_stream, after, 0));
        for (const auto & m : misses) {
            uint8_t * dst = a->d_arena + a->slab_base[i] + (uint64_t)m.second * a->record[i];
            const uint8_t * src = a->h_tier + a->host_base[i] + (uint64_t)m.first * a->record[i];
            if (cudaMemcpyAsync(dst, src, a->record_raw[i], cudaMemcpyHostToDevice, a->copy_stream) != cudaSuccess)
                return GX_ERR_COPY;
            ++a->slot_gen[i][(size_t)m.second];
            st.bytes_copied += a->record_raw[i];
        }
        ck(cudaEventRecord(a->ev_copy[i], a->copy_stream));
        ck(cudaStreamWaitEvent(consumer, a->ev_copy[i], 0));
        a->stats.copies += misses.size();
    }
    a->stats.serves += 1;
    a->stats.hits += st.hits;
    a->stats.misses += st.misses;
    a->stats.evictions += st.evictions;
    a->stats.bytes_h2d += st.bytes_copied;
    if (st_out) *st_out = st;
    return GX_OK;
}

// Rows per expert tile: a divisor of ne01 whose byte span keeps the 16-byte
// alignment of bulk copies, whose shared memory fits, preferring enough CTAs
// to fill the 148 SMs several times over.
int pick_rows(int type, int mode, gx::RowsParams & p, int64_t ctas_per_tile, const int * cands, int ncand) {
    int best = 0;
    for (int ci = 0; ci < ncand; ++ci) {
        const int R = cands[ci];
        if (p.ne01 % R != 0) continue;
        if (((int64_t)R * p.nb01) % 16 != 0) continue;
        p.R = R;
        if (gx::rows_smem_layout(type, mode, p) == 0) continue;
        best = R;
        if ((int64_t)(p.ne01 / R) * ctas_per_tile >= 4 * 148) break;
    }
    p.R = best;
    return best;
}

bool aligned16(const void * p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int gx_remap_serve(gx_arena * a, uint32_t layer, const int32_t * ids, int64_t ne0, int64_t ne1, int64_t nb0, int64_t nb1,
                   int32_t * slots, int64_t dnb0, int64_t dnb1, void * stream, gx_serve_stats * stats) {
    if (a == nullptr || ids == nullptr || slots == nullptr || ne0 < 0 || ne1 < 0) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(a->mu);
        ck(cudaSetDevice(a->device));
        const int64_t n = ne0 * ne1;
        std::vector<int32_t> experts((size_t)n), sl((size_t)n);
        // strided read, token-major (scripts/derive-remap-strides.py:30-48)
        const char * src = reinterpret_cast<const char *>(ids);
        for (int64_t i1 = 0, f = 0; i1 < ne1; ++i1)
            for (int64_t i0 = 0; i0 < ne0; ++i0, ++f)
                experts[(size_t)f] = *reinterpret_cast<const int32_t *>(src + i1 * nb1 + i0 * nb0);
        cudaStream_t consumer = reinterpret_cast<cudaStream_t>(stream);
        // everything already queued on the consumer stream may read the slab
        ck(cudaEventRecord(a->ev_snapshot, consumer));
        const int rc = arena_serve(a, layer, experts.data(), (uint32_t)n, sl.data(), a->ev_snapshot, consumer, stats,
                                   (uint32_t)ne1, (uint32_t)ne0);
        if (rc != GX_OK) return rc;
        char * dst = reinterpret_cast<char *>(slots);
        for (int64_t i1 = 0, f = 0; i1 < ne1; ++i1)
            for (int64_t i0 = 0; i0 < ne0; ++i0, ++f)
                *reinterpret_cast<int32_t *>(dst + i1 * dnb1 + i0 * dnb0) = sl[(size_t)f];
        return GX_OK;
    });
}

int gx_arena_read_slot(gx_arena * a, uint32_t layer, uint32_t slot, void * dst, uint64_t bytes) {
    if (a == nullptr || dst == nullptr) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(a->mu);
        const SlotPolicy & P = a->policy->impl;
        if (layer < P.first_layer() || layer > P.last_layer() || slot >= P.quota_of(layer)) return GX_ERR_INVALID;
        const uint32_t i = a->L(layer);
        if (bytes > a->record[i]) return GX_ERR_INVALID;
        ck(cudaSetDevice(a->device));
        ck(cudaStreamSynchronize(a->copy_stream));
        ck(cudaMemcpy(dst, a->d_arena + a->slab_base[i] + (uint64_t)slot * a->record[i], bytes, cudaMemcpyDeviceToHost));
        return GX_OK;
    });
}

int gx_arena_warm_all(gx_arena * a, void * stream) {
    if (a == nullptr) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(a->mu);
        ck(cudaSetDevice(a->device));
        const SlotPolicy & P = a->policy->impl;
        cudaStream_t consumer = reinterpret_cast<cudaStream_t>(stream);
        for (uint32_t layer = P.first_layer(); layer <= P.last_layer(); ++layer) {
            const uint32_t bound = P.batch_bound(layer);
            for (uint32_t e0 = 0; e0 < P.experts(); e0 += bound) {
                const uint32_t cnt = std::min(bound, P.experts() - e0);
                std::vector<int32_t> ex(cnt), sl(cnt);
                for (uint32_t j = 0; j < cnt; ++j) ex[j] = (int32_t)(e0 + j);
                ck(cudaEventRecord(a->ev_snapshot, consumer));
                const int rc = arena_serve(a, layer, ex.data(), cnt, sl.data(), a->ev_snapshot, consumer, nullptr, 1, cnt);
                if (rc != GX_OK) return rc;
            }
        }
        return GX_OK;
    });
}

// ----------------------------------------------------------------- kernels

int gx_mul_mat_id(int type, const void * as, int64_t ne00, int64_t ne01, int64_t nb01, int64_t nb02, int64_t n_as,
                  const float * b, int64_t ne11, int64_t ne12, int64_t nb11, int64_t nb12, const int32_t * ids,
                  int64_t ne20, int64_t ne21, int64_t nbi1, float * dst, void * stream) {
    if (!gx::supported_weight_type(type)) return GX_ERR_TYPE;
    if (as == nullptr || b == nullptr || ids == nullptr || dst == nullptr) return GX_ERR_INVALID;
    if (ne00 <= 0 || ne01 <= 0 || n_as <= 0 || ne20 <= 0 || ne21 < 0 || ne12 != ne21) return GX_ERR_INVALID;
    if (ne11 != 1 && ne11 != ne20) return GX_ERR_INVALID;
    if (ne00 % gx::row_align(type) != 0) return GX_ERR_ALIGN;
    if (nb01 < gx::row_bytes(type, ne00) || (nb11 % 4) || (nb12 % 4) || (nbi1 % 4)) return GX_ERR_INVALID;
    if (!aligned16(as) || nb02 % 16 != 0) return GX_ERR_ALIGN;
    if (ne21 == 0) return GX_OK;
    if (ne20 * ne21 > 65535) return GX_ERR_INVALID;
    return guarded([&] {
        gx::RowsParams p{};
        p.w0 = static_cast<const uint8_t *>(as);
        p.nb01 = nb01; p.nb02 = nb02;
        p.ne00 = (int32_t)ne00; p.ne01 = (int32_t)ne01; p.n_as = (int32_t)n_as;
        p.src = b; p.nb11 = nb11; p.nb12 = nb12; p.ne11 = (int32_t)ne11;
        p.ids = ids; p.nbi1 = nbi1; p.k = (int32_t)ne20; p.T = (int32_t)ne21;
        p.dst = dst;
        static const int cands[] = {8, 4, 2, 1};
        if (pick_rows(type, gx::kModePlain, p, ne20 * ne21, cands, 4) == 0) return GX_ERR_ALIGN;
        const dim3 grid((unsigned)(ne01 / p.R), (unsigned)(ne20 * ne21));
        ck(gx::launch_rows(type, gx::kModePlain, p, grid, reinterpret_cast<cudaStream_t>(stream)));
        return GX_OK;
    });
}

int gx_quantize_rows(int vdt, const float * src, int64_t ne0, int64_t nrows, int64_t nb1, void * dst, int64_t dst_row_stride,
                     void * stream) {
    if (vdt != GX_TYPE_Q8_0 && vdt != GX_TYPE_Q8_K) return GX_ERR_TYPE;
    if (src == nullptr || dst == nullptr || ne0 <= 0 || nrows < 0 || nb1 % 4) return GX_ERR_INVALID;
    if (ne0 % (vdt == GX_TYPE_Q8_0 ? 32 : 256) != 0) return GX_ERR_ALIGN;
    if (dst_row_stride < gx::row_bytes(vdt, ne0)) return GX_ERR_INVALID;
    if (vdt == GX_TYPE_Q8_K && (dst_row_stride % 4 || !aligned16(dst))) return GX_ERR_ALIGN;
    return guarded([&] {
        ck(gx::launch_quantize_rows(vdt, src, (int)ne0, nrows, nb1, static_cast<uint8_t *>(dst), dst_row_stride,
                                    reinterpret_cast<cudaStream_t>(stream)));
        return GX_OK;
    });
}

int gx_swiglu(const float * g, const float * u, float * out, int64_t n, void * stream) {
    if (g == nullptr || u == nullptr || out == nullptr || n < 0) return GX_ERR_INVALID;
    return guarded([&] {
        ck(gx::launch_swiglu(g, u, out, n, reinterpret_cast<cudaStream_t>(stream)));
        return GX_OK;
    });
}

int gx_swiglu_oai(const float * g, const float * u, float * out, int64_t n, float alpha, float limit, void * stream) {
    if (g == nullptr || u == nullptr || out == nullptr || n < 0) return GX_ERR_INVALID;
    return guarded([&] {
        ck(gx::launch_swiglu_oai(g, u, out, n, alpha, limit, reinterpret_cast<cudaStream_t>(stream)));
        return GX_OK;
    });
}

int gx_combine(const float * y, const float * w, float * out, int64_t H, int64_t k, int64_t T, void * stream) {
    if (y == nullptr || w == nullptr || out == nullptr || H < 0 || k <= 0 || T < 0) return GX_ERR_INVALID;
    return guarded([&] {
        ck(gx::launch_combine(y, w, out, H, (int)k, T, reinterpret_cast<cudaStream_t>(stream)));
        return GX_OK;
    });
}

int gx_expf(const float * x, float * y, int64_t n, void * stream) {
    if (x == nullptr || y == nullptr || n < 0) return GX_ERR_INVALID;
    return guarded([&] {
        ck(gx::launch_expf(x, y, n, reinterpret_cast<cudaStream_t>(stream)));
        return GX_OK;
    });
}

// --------------------------------------------------------------- MoE layer

}  // extern "C"

namespace {

// Launch configuration of one routed-expert layer: everything the three
// kernels need except the per-call pointers and slot ids.
struct LayerPlan {
    uint32_t layer = 0, li = 0;
    int64_t H = 0, I = 0, k = 0, T = 0;
    int vdt_g = 0, vdt_d = 0;
    int type_gate = 0, type_down = 0;
    gx::DecodeParams g{}, dn{};
};

int plan_layer(gx_arena * a, uint32_t layer, const gx_layer_desc * d, int64_t k, int64_t T, LayerPlan & lp) {
    if (d == nullptr) return GX_ERR_INVALID;
    if (!gx::supported_weight_type(d->type_gate) || !gx::supported_weight_type(d->type_down)) return GX_ERR_TYPE;
    if (d->type_up != d->type_gate) return GX_ERR_TYPE;
    if (d->act != GX_ACT_SWIGLU && d->act != GX_ACT_SWIGLU_OAI) return GX_ERR_INVALID;
    if (T < 1 || k <= 0 || T > a->max_tokens || d->hidden != a->hidden || d->intermediate != a->intermediate)
        return GX_ERR_INVALID;
    if (k > (int64_t)a->used || k * T > 65535) return GX_ERR_INVALID;
    const int64_t H = d->hidden, I = d->intermediate;
    if (H % gx::row_align(d->type_gate) != 0 || I % gx::row_align(d->type_down) != 0) return GX_ERR_ALIGN;
    if (d->off_gate % 16 || d->off_up % 16) return GX_ERR_ALIGN;
    const SlotPolicy & P = a->policy->impl;
    if (layer < P.first_layer() || layer > P.last_layer()) return GX_ERR_INVALID;
    const uint32_t li = a->L(layer);
    if (d->off_up + gx::row_bytes(d->type_up, H) * I > a->record_raw[li] ||
        (uint64_t)gx::row_bytes(d->type_down, I) * H > d->off_gate)
        return GX_ERR_INVALID;
    lp.layer = layer;
    lp.li = li;
    lp.H = H;
    lp.I = I;
    lp.k = k;
    lp.T = T;
    lp.type_gate = d->type_gate;
    lp.type_down = d->type_down;
    lp.vdt_g = gx::vec_dot_type(d->type_gate);
    lp.vdt_d = gx::vec_dot_type(d->type_down);
    uint8_t * base = a->d_arena + a->slab_base[li];
    const int64_t n = k * T;

    gx::DecodeParams & g = lp.g;
    g = gx::DecodeParams{};
    g.w0 = base + d->off_gate;
    g.w1 = base + d->off_up;
    g.nb01 = gx::row_bytes(d->type_gate, H);
    g.nb02 = (int64_t)a->record[li];
    g.ne00 = (int32_t)H;
    g.ne01 = (int32_t)I;
    g.n_as = (int32_t)P.quota_of(layer);
    g.k = (int32_t)k;
    g.T = (int32_t)T;
    g.aq = a->d_xq;
    g.al = gx::act_layout(lp.vdt_g, (int)H);
    g.a_rows = 1;
    g.act_f32 = a->d_act;
    g.act_q = a->d_actq;
    g.al2 = gx::act_layout(lp.vdt_d, (int)I);
    g.vdt2 = lp.vdt_d;
    g.qblk = lp.vdt_d == gx::GX_T_Q8_0 ? 32 : 256;
    g.counters = a->d_cnt;
    g.act = d->act;
    g.alpha = d->alpha;
    g.limit = d->limit;
    {
        static const int cands[] = {8, 16, 4, 2, 1};
        int threads = 0;
        g.R = 0;
        for (int R : cands) {
            if (I % R || g.qblk % R) continue;
            gx::DecodeParams t = g;
            t.R = R;
            if (gx::decode_layout(1, t, threads) == 0) continue;
            g.R = R;
            break;
        }
        if (g.R == 0) return GX_ERR_ALIGN;
        g.n_units = (int32_t)(n * (I / g.R));
    }

    gx::DecodeParams & dn = lp.dn;
    dn = g;
    dn.w0 = base;
    dn.w1 = nullptr;
    dn.nb01 = gx::row_bytes(d->type_down, I);
    dn.ne00 = (int32_t)I;
    dn.ne01 = (int32_t)H;
    dn.aq = a->d_actq;
    dn.al = gx::act_layout(lp.vdt_d, (int)I);
    dn.a_rows = (int32_t)k;
    {
        // 32 rows per stage (128 threads, two rows each) when the tile keeps
        // 16-byte alignment, else larger or smaller tiles; R stays even
        const int base_r = (int)(32 / k) > 1 ? (int)(32 / k) : 2;
        const int cands[] = {base_r, 2 * base_r, base_r / 2, base_r / 4, 2};
        int threads = 0;
        dn.R = 0;
        for (int R : cands) {
            if (R < 1 || H % R) continue;
            gx::DecodeParams t = dn;
            t.R = R;
            if (gx::decode_layout(2, t, threads) == 0) continue;
            dn.R = R;
            break;
        }
        if (dn.R == 0) return GX_ERR_ALIGN;
        dn.n_units = (int32_t)(T * (H / dn.R));
    }
    return GX_OK;
}

// The layer plan of a shared expert: the routed plan's kernels on the
// caller's resident record (one "slot", index 0), k = 1, the arena's scratch.
int plan_shared(gx_arena * a, uint32_t layer, const gx_shared_expert * sh, int64_t T, LayerPlan & lp) {
    const gx_layer_desc & d = sh->desc;
    if (sh->record == nullptr) return GX_ERR_INVALID;
    if (!gx::supported_weight_type(d.type_gate) || !gx::supported_weight_type(d.type_down)) return GX_ERR_TYPE;
    if (d.type_up != d.type_gate) return GX_ERR_TYPE;
    if (d.act != GX_ACT_SWIGLU && d.act != GX_ACT_SWIGLU_OAI) return GX_ERR_INVALID;
    if (T < 1 || T > a->max_tokens || d.hidden != a->hidden || d.intermediate < 1 ||
        d.intermediate > (int64_t)a->used * a->intermediate)
        return GX_ERR_INVALID;
    const int64_t H = d.hidden, I = d.intermediate;
    if (H % gx::row_align(d.type_gate) != 0 || I % gx::row_align(d.type_down) != 0) return GX_ERR_ALIGN;
    if (d.off_gate % 16 || d.off_up % 16 || (reinterpret_cast<uintptr_t>(sh->record) & 15u) != 0) return GX_ERR_ALIGN;
    if ((uint64_t)gx::row_bytes(d.type_down, I) * H > d.off_gate ||
        d.off_gate + gx::row_bytes(d.type_gate, H) * I > d.off_up)
        return GX_ERR_INVALID;
    // the scratch of the routed plan, sized for k*max_tokens pairs of the routed I
    const int64_t pa_sh = std::max(gx::act_layout(gx::GX_T_Q8_0, (int)I).pitch, gx::act_layout(gx::GX_T_Q8_K, (int)I).pitch);
    const int64_t pa = std::max(gx::act_layout(gx::GX_T_Q8_0, (int)a->intermediate).pitch,
                                gx::act_layout(gx::GX_T_Q8_K, (int)a->intermediate).pitch);
    if (T * pa_sh > (int64_t)a->used * a->max_tokens * pa) return GX_ERR_INVALID;
    gx_layer_desc rd = d;
    // plan_layer checks the routed geometry; plan with the shared one by hand
    lp = LayerPlan{};
    lp.layer = layer;
    lp.li = a->L(layer);
    lp.H = H;
    lp.I = I;
    lp.k = 1;
    lp.T = T;
    lp.type_gate = rd.type_gate;
    lp.type_down = rd.type_down;
    lp.vdt_g = gx::vec_dot_type(rd.type_gate);
    lp.vdt_d = gx::vec_dot_type(rd.type_down);
    const uint8_t * base = static_cast<const uint8_t *>(sh->record);
    gx::DecodeParams & g = lp.g;
    g = gx::DecodeParams{};
    g.w0 = base + rd.off_gate;
    g.w1 = base + rd.off_up;
    g.nb01 = gx::row_bytes(rd.type_gate, H);
    g.nb02 = 0;
    g.ne00 = (int32_t)H;
    g.ne01 = (int32_t)I;
    g.n_as = 1;
    g.k = 1;
    g.T = (int32_t)T;
    g.aq = a->d_xq;
    g.al = gx::act_layout(lp.vdt_g, (int)H);
    g.a_rows = 1;
    g.act_f32 = a->d_act;
    g.act_q = a->d_actq;
    g.al2 = gx::act_layout(lp.vdt_d, (int)I);
    g.vdt2 = lp.vdt_d;
    g.qblk = lp.vdt_d == gx::GX_T_Q8_0 ? 32 : 256;
    g.counters = a->d_cnt;
    g.act = rd.act;
    g.alpha = rd.alpha;
    g.limit = rd.limit;
    {
        static const int cands[] = {8, 16, 4, 2, 1};
        int threads = 0;
        g.R = 0;
        for (int R : cands) {
            if (I % R || g.qblk % R) continue;
            gx::DecodeParams t = g;
            t.R = R;
            if (gx::decode_layout(1, t, threads) == 0) continue;
            g.R = R;
            break;
        }
        if (g.R == 0) return GX_ERR_ALIGN;
        g.n_units = (int32_t)(T * (I / g.R));
    }
    gx::DecodeParams & dn = lp.dn;
    dn = g;
    dn.w0 = base;
    dn.w1 = nullptr;
    dn.nb01 = gx::row_bytes(rd.type_down, I);
    dn.ne00 = (int32_t)I;
    dn.ne01 = (int32_t)H;
    dn.aq = a->d_actq;
    dn.al = gx::act_layout(lp.vdt_d, (int)I);
    dn.a_rows = 1;
    {
        static const int cands[] = {32, 64, 16, 8, 4, 2};
        int threads = 0;
        dn.R = 0;
        for (int R : cands) {
            if (H % R) continue;
            gx::DecodeParams t = dn;
            t.R = R;
            if (gx::decode_layout(2, t, threads) == 0) continue;
            dn.R = R;
            break;
        }
        if (dn.R == 0) return GX_ERR_ALIGN;
        dn.n_units = (int32_t)(T * (H / dn.R));
    }
    return GX_OK;
}

// Enqueue the three kernels of a planned layer. Slot ids come either inline
// (n <= kInlineIds) or from a device array [T, k].
void enqueue_layer(const LayerPlan & lp, const float * x, const float * w, float * out, const int32_t * ids_dev,
                   const int32_t * inline_slots, cudaStream_t s, bool pdl_first, bool pdl, cudaEvent_t tv[3]) {
    gx::DecodeParams g = lp.g, dn = lp.dn;
    const int64_t n = lp.k * lp.T;
    if (ids_dev == nullptr) {
        g.use_inline = dn.use_inline = 1;
        for (int64_t j = 0; j < n; ++j) g.inline_ids[j] = dn.inline_ids[j] = inline_slots[j];
    } else {
        g.use_inline = dn.use_inline = 0;
        g.ids = dn.ids = ids_dev;
    }
    dn.rw = w;
    dn.out = out;
    ck(gx::launch_quant_split(lp.vdt_g, x, (int)lp.H, lp.T, lp.H * 4, const_cast<uint8_t *>(g.aq), s, pdl_first));
    // external records: inside a stream capture they become event nodes of the graph
    if (tv && tv[0]) ck(cudaEventRecordWithFlags(tv[0], s, cudaEventRecordExternal));
    ck(gx::launch_decode(lp.type_gate, 1, g, s, pdl));
    if (tv && tv[1]) ck(cudaEventRecordWithFlags(tv[1], s, cudaEventRecordExternal));
    ck(gx::launch_decode(lp.type_down, 2, dn, s, pdl));
    if (tv && tv[2]) ck(cudaEventRecordWithFlags(tv[2], s, cudaEventRecordExternal));
}

// Micro-batches with many (token, slot) pairs run the expert-grouped kernels:
// every expert's rows are read once per layer instead of once per pair.
constexpr int64_t kGroupedPairs = 128;

// cuTensorMapEncodeTiled from the driver, resolved once through the runtime
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void * f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// Weight rows of every slot of a layer as a 3-D tensor of 16-bit words
// (x: word of a row, y: row, z: slot), boxes of 136 words (8 Q8_0 blocks)
// by box_rows rows.
bool encode_rows_map(CUtensorMap * map, const void * base, int64_t nb01, int64_t rows, int64_t slots, int64_t nb02,
                     uint32_t box_rows) {
    const auto enc = tensor_map_encoder();
    if (enc == nullptr || (reinterpret_cast<uintptr_t>(base) & 15u) != 0 || nb01 % 16 != 0 || nb02 % 16 != 0) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)(nb01 / 2), (cuuint64_t)rows, (cuuint64_t)slots};
    const cuuint64_t strides[2] = {(cuuint64_t)nb01, (cuuint64_t)nb02};
    const cuuint32_t box[3] = {136u, box_rows, 1u};
    const cuuint32_t elem[3] = {1u, 1u, 1u};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void *>(base), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The tensor-core prefill replaces the CUDA-core grouped kernels when the
// weights are Q8_0 and the micro-batch has at least this many pairs per
// touched expert on average (below it most of an MMA's 16-pair columns
// would be padding).
constexpr int64_t kMmaPairsPerExpert = 4;

bool use_mma(const LayerPlan & lp, int64_t pairs, int64_t experts_touched) {
    if (const char * env = std::getenv("GX_PREFILL_MMA")) {
        if (env[0] == '0') return false;
    }
    // the up rows must follow the gate rows in the record (one tensor for both)
    return gx::prefill_mma_supported(lp.type_gate, lp.type_down, lp.H, lp.I) &&
           lp.g.w1 == lp.g.w0 + lp.I * lp.g.nb01 && tensor_map_encoder() != nullptr &&
           pairs >= kMmaPairsPerExpert * std::max<int64_t>(1, experts_touched);
}

bool use_grouped(const LayerPlan & lp, int64_t pairs) {
    if (const char * env = std::getenv("GX_GROUPED")) {
        if (env[0] == '0') return false;
    }
    return pairs >= kGroupedPairs && lp.type_gate == gx::GX_T_Q8_0 && lp.type_down == gx::GX_T_Q8_0 && lp.H % 256 == 0 &&
           lp.I % 256 == 0;
}

// quantize x -> gate/up grouped -> quantize act -> down grouped -> combine
void prefill_layer(gx_arena * a, const LayerPlan & lp, const float * x, const int32_t * slots, const float * w, float * out,
                   cudaStream_t s) {
    const int64_t T = lp.T, k = lp.k, P = T * k, H = lp.H, I = lp.I;
    const int32_t n_as = lp.g.n_as;
    if (a->d_y == nullptr) ck(cudaMalloc(&a->d_y, (size_t)(a->used * a->max_tokens) * (size_t)a->hidden * sizeof(float)));
    if (a->ev_grp == nullptr) ck(cudaEventCreateWithFlags(&a->ev_grp, cudaEventDisableTiming));
    // grouping: counting sort of the pairs by slot
    const int64_t slots_used = std::min<int64_t>(P, n_as);
    const int64_t units_max = slots_used * (I / 8 + H / 16);
    const int64_t chunks_max = P / gx::kMmaTok + slots_used;
    const size_t need = (size_t)(n_as + 1) + 3 * (size_t)P + 4 * (size_t)units_max + 3 * (size_t)chunks_max;
    if (need > a->grp_cap) {
        if (a->h_grp) {
            ck(cudaEventSynchronize(a->ev_grp));
            cudaFreeHost(a->h_grp);
            a->h_grp = nullptr;
        }
        if (a->d_grp) cudaFree(a->d_grp);
        a->d_grp = nullptr;
        a->grp_cap = 0;
        ck(cudaHostAlloc(&a->h_grp, need * sizeof(int32_t), cudaHostAllocDefault));
        ck(cudaMalloc(&a->d_grp, need * sizeof(int32_t)));
        a->grp_cap = need;
    }
    ck(cudaEventSynchronize(a->ev_grp));   // the previous upload out of h_grp has run
    int32_t * seg = a->h_grp;
    int32_t * src_tok = seg + (n_as + 1);
    int32_t * src_pair = src_tok + P;
    int32_t * dst = src_pair + P;
    int32_t * u_slot_g = dst + P;
    int32_t * u_row_g = u_slot_g + units_max;
    int32_t * u_slot_d = u_row_g + units_max;
    int32_t * u_row_d = u_slot_d + units_max;
    for (int32_t e = 0; e <= n_as; ++e) seg[e] = 0;
    for (int64_t i = 0; i < P; ++i) {
        if (slots[i] < 0 || slots[i] >= n_as) throw PolicyError(GX_ERR_SLOTS, "slot id out of range");
        ++seg[slots[i] + 1];
    }
    for (int32_t e = 0; e < n_as; ++e) seg[e + 1] += seg[e];
    std::vector<int32_t> fill(seg, seg + n_as);
    for (int64_t i = 0; i < P; ++i) {
        const int32_t j = fill[(size_t)slots[i]]++;
        src_tok[j] = (int32_t)(i / k);
        src_pair[j] = (int32_t)i;
        dst[j] = (int32_t)i;
    }
    int32_t * c_slot = u_row_d + units_max;
    int32_t * c_first = c_slot + chunks_max;
    int32_t * c_count = c_first + chunks_max;
    int32_t nchunks = 0, touched = 0;
    for (int32_t e = 0; e < n_as; ++e) {
        if (seg[e + 1] > seg[e]) ++touched;
        for (int32_t f = seg[e]; f < seg[e + 1]; f += gx::kMmaTok) {
            c_slot[nchunks] = e;
            c_first[nchunks] = f;
            c_count[nchunks++] = std::min<int32_t>(gx::kMmaTok, seg[e + 1] - f);
        }
    }
    const bool mma = use_mma(lp, P, touched);
    int32_t ng = 0, nd = 0;
    for (int32_t e = 0; e < n_as && !mma; ++e) {
        if (seg[e + 1] == seg[e]) continue;
        for (int64_t r = 0; r < I; r += 8) {
            u_slot_g[ng] = e;
            u_row_g[ng++] = (int32_t)r;
        }
        for (int64_t r = 0; r < H; r += 16) {
            u_slot_d[nd] = e;
            u_row_d[nd++] = (int32_t)r;
        }
    }
    ck(cudaMemcpyAsync(a->d_grp, a->h_grp, need * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    ck(cudaEventRecord(a->ev_grp, s));
    const int32_t * dseg = a->d_grp;
    const int32_t * dtok = dseg + (n_as + 1);
    const int32_t * dpair = dtok + P;
    const int32_t * ddst = dpair + P;
    const int32_t * dusg = ddst + P;
    const int32_t * durg = dusg + units_max;
    const int32_t * dusd = durg + units_max;
    const int32_t * durd = dusd + units_max;
    const int32_t * dcs = durd + units_max;
    const int32_t * dcf = dcs + chunks_max;
    const int32_t * dcc = dcf + chunks_max;

    ck(gx::launch_quant_split(gx::GX_T_Q8_0, x, (int)H, T, H * 4, a->d_xq, s, false));
    if (mma) {
        // tensor cores: masked B tiles of the layer input per chunk, gate/up
        // units (64 gate + 64 up rows x 16 pairs), the activation quantized,
        // masked B tiles of it, down units (128 rows x 16 pairs), combine
        const int64_t nbh = H / 32, nbi = I / 32, nbmax = std::max(nbh, nbi);
        const size_t want = (size_t)chunks_max * (size_t)nbmax;
        if (want > a->mmab_cap) {
            if (a->d_mmab) cudaFree(a->d_mmab);
            if (a->d_mmady) cudaFree(a->d_mmady);
            a->d_mmab = nullptr;
            a->d_mmady = nullptr;
            a->mmab_cap = 0;
            ck(cudaMalloc(&a->d_mmab, want * (size_t)(gx::kMmaN * 32)));
            ck(cudaMalloc(&a->d_mmady, want * (size_t)gx::kMmaTok * sizeof(float)));
            a->mmab_cap = want;
        }
        gx::MmaPrepParams bp{};
        bp.chunk_first = dcf;
        bp.chunk_count = dcc;
        bp.pair_src = dtok;
        bp.aq = a->d_xq;
        bp.al = lp.g.al;
        bp.nblk = (int32_t)nbh;
        bp.btiles = a->d_mmab;
        bp.dyt = a->d_mmady;
        ck(gx::launch_mma_bprep(bp, nchunks, s));
        gx::MmaParams mp{};
        if (!encode_rows_map(&mp.tmap, lp.g.w0, lp.g.nb01, 2 * I, n_as, lp.g.nb02, 64u))
            throw PolicyError(GX_ERR_ALIGN, "gate/up tensor map");
        mp.up_row0 = (int32_t)I;
        mp.nb01 = lp.g.nb01;
        mp.nblk = (int32_t)nbh;
        mp.n_rt = (int32_t)(I / 64);
        mp.chunk_slot = dcs;
        mp.chunk_first = dcf;
        mp.chunk_count = dcc;
        mp.pair_dst = ddst;
        mp.btiles = a->d_mmab;
        mp.dyt = a->d_mmady;
        mp.out = a->d_act;
        mp.out_ld = I;
        mp.act = lp.g.act;
        mp.alpha = lp.g.alpha;
        mp.limit = lp.g.limit;
        ck(gx::launch_prefill_mma(0, mp, nchunks * mp.n_rt, s));
        ck(gx::launch_quant_split(gx::GX_T_Q8_0, a->d_act, (int)I, P, I * 4, a->d_actq, s, false));
        bp.pair_src = dpair;
        bp.aq = a->d_actq;
        bp.al = lp.dn.al;
        bp.nblk = (int32_t)nbi;
        ck(gx::launch_mma_bprep(bp, nchunks, s));
        if (!encode_rows_map(&mp.tmap, lp.dn.w0, lp.dn.nb01, H, n_as, lp.dn.nb02, (uint32_t)gx::kMmaRows))
            throw PolicyError(GX_ERR_ALIGN, "down tensor map");
        mp.up_row0 = 0;
        mp.nb01 = lp.dn.nb01;
        mp.nblk = (int32_t)nbi;
        mp.n_rt = (int32_t)(H / gx::kMmaRows);
        mp.out = a->d_y;
        mp.out_ld = H;
        ck(gx::launch_prefill_mma(1, mp, nchunks * mp.n_rt, s));
        ck(gx::launch_combine(a->d_y, w, out, H, (int)k, T, s));
        return;
    }
    gx::PrefillParams g{};
    g.w0 = lp.g.w0;
    g.w1 = lp.g.w1;
    g.nb01 = lp.g.nb01;
    g.nb02 = lp.g.nb02;
    g.K = (int32_t)H;
    g.n_as = n_as;
    g.n_units = ng;
    g.unit_slot = dusg;
    g.unit_row0 = durg;
    g.seg_start = dseg;
    g.pair_src = dtok;
    g.pair_dst = ddst;
    g.aq = a->d_xq;
    g.al = lp.g.al;
    g.out = a->d_act;
    g.out_ld = I;
    g.act = lp.g.act;
    g.alpha = lp.g.alpha;
    g.limit = lp.g.limit;
    const uint32_t smem_g = gx::prefill_layout(g);
    if (smem_g == 0) throw PolicyError(GX_ERR_ALIGN, "grouped gate/up layout");
    ck(gx::launch_prefill(0, g, smem_g, s));
    ck(gx::launch_quant_split(gx::GX_T_Q8_0, a->d_act, (int)I, P, I * 4, a->d_actq, s, false));
    gx::PrefillParams dn = g;
    dn.w0 = lp.dn.w0;
    dn.w1 = nullptr;
    dn.nb01 = lp.dn.nb01;
    dn.K = (int32_t)I;
    dn.n_units = nd;
    dn.unit_slot = dusd;
    dn.unit_row0 = durd;
    dn.pair_src = dpair;
    dn.aq = a->d_actq;
    dn.al = lp.dn.al;
    dn.out = a->d_y;
    dn.out_ld = H;
    const uint32_t smem_d = gx::prefill_layout(dn);
    if (smem_d == 0) throw PolicyError(GX_ERR_ALIGN, "grouped down layout");
    ck(gx::launch_prefill(1, dn, smem_d, s));
    ck(gx::launch_combine(a->d_y, w, out, H, (int)k, T, s));
}

int layer_forward_waves(gx_arena * a, const LayerPlan & lp, const gx_layer_desc * d, const float * x,
                        const int32_t * ids, const float * w, float * out, cudaStream_t s, gx_serve_stats * stats);

int layer_forward_locked(gx_arena * a, uint32_t layer, const gx_layer_desc * d, const float * x, const int32_t * ids,
                         const float * w, int64_t k, int64_t T, float * out, cudaStream_t s, gx_serve_stats * stats) {
    if (x == nullptr || ids == nullptr || w == nullptr || out == nullptr) return GX_ERR_INVALID;
    if (T == 0) return GX_OK;
    LayerPlan lp;
    int rc = plan_layer(a, layer, d, k, T, lp);
    if (rc != GX_OK) return rc;
    const int64_t n = k * T;
    {
        // more distinct experts than the policy serves in one batch: waves
        const SlotPolicy & P = a->policy->impl;
        thread_local std::vector<uint8_t> seen;
        seen.assign(P.experts(), 0);
        uint32_t distinct = 0;
        for (int64_t i = 0; i < n; ++i) {
            if (ids[i] < 0 || (uint32_t)ids[i] >= P.experts()) return GX_ERR_DOMAIN;
            if (!seen[(size_t)ids[i]]) {
                seen[(size_t)ids[i]] = 1;
                ++distinct;
            }
        }
        if (distinct > P.batch_bound(layer)) return layer_forward_waves(a, lp, d, x, ids, w, out, s, stats);
    }
    int32_t * slots = a->slot_scratch.data();
    gx_serve_stats sst{};
    rc = arena_serve(a, layer, ids, (uint32_t)n, slots, a->last_ev[lp.li], s, &sst, (uint32_t)T, (uint32_t)k);
    if (rc != GX_OK) return rc;
    if (stats) *stats = sst;

    if (use_grouped(lp, n)) {
        prefill_layer(a, lp, x, slots, w, out, s);
        ck(cudaEventRecord(a->ev_done[lp.li], s));
        a->last_ev[lp.li] = a->ev_done[lp.li];
        return GX_OK;
    }

    const int32_t * ids_dev = nullptr;
    if (n > gx::kInlineIds) {
        // stage the slot ids through a pinned ring; a ring entry is reused
        // only after the copy that read it has run
        const int st = a->stage_next;
        a->stage_next = (st + 1) % kStageRing;
        const int64_t stride = (int64_t)a->used * a->max_tokens;
        ck(cudaEventSynchronize(a->ev_stage[st]));
        int32_t * h = a->h_ids + (size_t)st * stride;
        int32_t * dd = a->d_ids + (size_t)st * stride;
        std::memcpy(h, slots, (size_t)n * sizeof(int32_t));
        ck(cudaMemcpyAsync(dd, h, (size_t)n * sizeof(int32_t), cudaMemcpyHostToDevice, s));
        ck(cudaEventRecord(a->ev_stage[st], s));
        ids_dev = dd;
    }
    cudaEvent_t tv[3] = {nullptr, nullptr, nullptr};
    if (a->timing) {
        while (a->tev.size() < a->tev_used + 3) {
            cudaEvent_t e;
            ck(cudaEventCreate(&e));
            a->tev.push_back(e);
        }
        for (int j = 0; j < 3; ++j) tv[j] = a->tev[a->tev_used + j];
        a->tev_used += 3;
    }
    // programmatic overlap between the kernels, except right after a miss
    // copy wait or while timing the kernels one by one
    const bool pdl = !a->timing;
    enqueue_layer(lp, x, w, out, ids_dev, slots, s, pdl && sst.misses == 0 && ids_dev == nullptr, pdl, tv);
    ck(cudaEventRecord(a->ev_done[lp.li], s));
    a->last_ev[lp.li] = a->ev_done[lp.li];
    return GX_OK;
}

// Expert-major waves for a micro-batch whose distinct experts exceed the
// policy's batch bound min(quota, probation) (the reference bounds its
// micro-batches by it: src/h4/h4-expert-cache.cpp:105-124). The distinct
// experts, in order of first appearance, are cut into waves of at most
// `bound`; the (token, slot) pairs are ordered by wave. Each wave is served
// and computed as micro-batches of one expert per pair with unit router
// weight, at most max_tokens pairs each (the result fl(1 * y) = y is the
// pair's down projection, bit for bit); a later wave's misses may evict a
// slot of an earlier wave only after the kernels that read it (the copy
// stream waits for the layer's last kernels). The per-pair outputs go back
// to (token, slot) order and the combine ((w0*y0 + w1*y1) + ...) runs in
// slot order: the same bits as the one-shot path, for any wave schedule.
int layer_forward_waves(gx_arena * a, const LayerPlan & lp, const gx_layer_desc * d, const float * x,
                        const int32_t * ids, const float * w, float * out, cudaStream_t s, gx_serve_stats * stats) {
    const SlotPolicy & P = a->policy->impl;
    const int64_t k = lp.k, T = lp.T, n = k * T, H = lp.H;
    const uint32_t bound = P.batch_bound(lp.layer);
    if (bound == 0) return GX_ERR_BATCH;
    const int64_t cap = (int64_t)a->used * a->max_tokens;   // pairs the scratch holds
    if (a->d_wx == nullptr) {
        ck(cudaMalloc(&a->d_wx, (size_t)cap * (size_t)a->hidden * sizeof(float)));
        ck(cudaMalloc(&a->d_wy, (size_t)cap * (size_t)a->hidden * sizeof(float)));
        ck(cudaMalloc(&a->d_wfull, (size_t)cap * (size_t)a->hidden * sizeof(float)));
        ck(cudaMalloc(&a->d_ones, (size_t)cap * sizeof(float)));
        ck(gx::launch_fill(a->d_ones, cap, 1.0f, s));
        ck(cudaStreamSynchronize(s));   // the unit weights are read on whatever stream calls next
        ck(cudaMalloc(&a->d_widx, (size_t)(2 * cap) * sizeof(int32_t)));
        ck(cudaHostAlloc(&a->h_widx, (size_t)(2 * cap) * sizeof(int32_t), cudaHostAllocDefault));
        ck(cudaEventCreateWithFlags(&a->ev_widx, cudaEventDisableTiming));
    }
    // wave of every distinct expert, in order of first appearance
    thread_local std::vector<int32_t> wave_of;
    wave_of.assign(P.experts(), -1);
    int32_t nd = 0;
    for (int64_t i = 0; i < n; ++i)
        if (wave_of[(size_t)ids[i]] < 0) wave_of[(size_t)ids[i]] = nd++ / (int32_t)bound;
    const int32_t nw = (nd + (int32_t)bound - 1) / (int32_t)bound;
    // pairs in wave order (stable inside a wave)
    thread_local std::vector<int32_t> start, order, wids;
    start.assign((size_t)nw + 1, 0);
    for (int64_t i = 0; i < n; ++i) ++start[(size_t)wave_of[(size_t)ids[i]] + 1];
    for (int32_t v = 0; v < nw; ++v) start[(size_t)v + 1] += start[(size_t)v];
    order.assign((size_t)n, 0);
    {
        std::vector<int32_t> fill(start.begin(), start.end() - 1);
        for (int64_t i = 0; i < n; ++i) order[(size_t)fill[(size_t)wave_of[(size_t)ids[i]]]++] = (int32_t)i;
    }
    wids.resize((size_t)n);
    for (int64_t j = 0; j < n; ++j) wids[(size_t)j] = ids[order[(size_t)j]];
    // gather the input row of every pair in wave order
    ck(cudaEventSynchronize(a->ev_widx));   // the previous upload out of h_widx has run
    for (int64_t j = 0; j < n; ++j) {
        a->h_widx[j] = order[(size_t)j] / (int32_t)k;
        a->h_widx[n + j] = order[(size_t)j];
    }
    ck(cudaMemcpyAsync(a->d_widx, a->h_widx, (size_t)(2 * n) * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    ck(cudaEventRecord(a->ev_widx, s));
    ck(gx::launch_move_rows(x, a->d_widx, n, H, a->d_wx, false, s));
    gx_serve_stats sum{};
    for (int32_t v = 0; v < nw; ++v) {
        for (int64_t b = start[(size_t)v]; b < start[(size_t)v + 1]; b += a->max_tokens) {
            const int64_t m = std::min<int64_t>(a->max_tokens, start[(size_t)v + 1] - b);
            gx_serve_stats st{};
            const int rc = layer_forward_locked(a, lp.layer, d, a->d_wx + b * H, wids.data() + b, a->d_ones, 1, m,
                                                a->d_wy + b * H, s, &st);
            if (rc != GX_OK) return rc;
            sum.hits += st.hits;
            sum.misses += st.misses;
            sum.evictions += st.evictions;
            sum.bytes_copied += st.bytes_copied;
        }
    }
    sum.distinct = (uint32_t)nd;
    ck(gx::launch_move_rows(a->d_wy, a->d_widx + n, n, H, a->d_wfull, true, s));
    ck(gx::launch_combine(a->d_wfull, w, out, H, (int)k, T, s));
    ck(cudaEventRecord(a->ev_done[lp.li], s));
    a->last_ev[lp.li] = a->ev_done[lp.li];
    if (stats) *stats = sum;
    return GX_OK;
}

}  // namespace

struct gx_stack_plan {
    gx_arena * a = nullptr;
    uint32_t first = 0, n = 0;
    int64_t k = 0, T = 0;
    gx_layer_desc desc{};
    std::vector<LayerPlan> lps;
    int32_t * d_slots = nullptr;
    int32_t * h_slots[2] = {nullptr, nullptr};
    cudaEvent_t ev_h[2] = {nullptr, nullptr};
    int cur = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaEvent_t ev_graph = nullptr;
    int timing = 0;
    std::vector<cudaEvent_t> tev;
    // persistent stack kernel
    bool stack = false;
    gx::StackParams sp{};
    int grid = 0, threads = 0, per_sm = 0;
    uint32_t smem = 0;
    int32_t * d_cnt = nullptr;          // q_done [n] | gu_done [n*T] | per-block counters [n*T*k*I/qblk]
    size_t cnt_bytes = 0;
    uint8_t * d_xq = nullptr;
    float * d_act = nullptr;
    uint8_t * d_actq = nullptr;
    // device routing (gx_stack_plan_run_routed)
    std::vector<const float *> wp;      // the plan's router weight pointers
    int32_t * d_table = nullptr;        // [n, experts] slot of every expert, built once the layers are pinned
    int32_t * d_ids = nullptr;          // [n, T, k] router ids when the caller keeps none
    // row mode 5: the layers' slots in the tensor-core record layout, kept in
    // step with the arena's fills, and the TMA maps over their codes
    uint8_t * d_shadow = nullptr;
    std::vector<uint64_t> shadow_base;             // per layer: offset of its slots in d_shadow
    std::vector<std::vector<uint32_t>> shadow_gen; // per layer and slot: the arena fill the copy follows
    CUtensorMap * d_maps = nullptr;                // [n][3]
    std::vector<int32_t> h_ids;         // ids read back for the route trace
};

namespace {

// Tiling of the stack kernel: 8 gate/up rows per gate/up job, 32/k output
// rows per down job, as many ring stages as the shared memory holds (at most
// kStackMaxConsumers; GX_STACK_STAGES caps it) and GX_STACK_WARPS consumer
// warps (default 8).
bool choose_stack_tiles(gx::StackParams & sp, int & threads, uint32_t & smem) {
    if (sp.k <= 0 || 32 % sp.k != 0) return false;
    // MXFP4 gate/up jobs hold 16 gate + 16 up rows (the stage is sized by the
    // 32-row down job anyway), computed by two warps of 8 + 8 rows each
    sp.Rg = sp.row_mode == 3 ? 16 : 8;
    int cap = gx::kStackMaxConsumers;
    if (const char * env = std::getenv("GX_STACK_STAGES")) {
        const int v = std::atoi(env);
        if (v >= 1 && v <= gx::kStackMaxConsumers) cap = v;
    }
    int wenv = 0;
    if (const char * env = std::getenv("GX_STACK_WARPS")) {
        const int v = std::atoi(env);
        if (v >= 1 && v <= gx::stack_max_warps(sp.row_mode)) wenv = v;
    }
    // the two-lane K-quant rows prefer 16-row down jobs (smaller stages, more
    // of them in flight) where 2 rows of an expert make whole 16-byte chunks
    for (int drows : {16, 32}) {
        if (drows == 16 && (sp.row_mode != 2 || 16 % sp.k != 0)) continue;
        sp.Rd = drows / sp.k;
        for (int C = cap; C >= 2; --C) {
            sp.C = C;
            // one consumer warp per stage (two for split jobs, four for MXFP4
            // jobs), at least 8
            const int per_stage = sp.row_mode == 3 ? 4 : (sp.row_mode == 1 || (sp.row_mode == 2 && drows == 32)) ? 2 : 1;
            sp.W = wenv ? wenv : std::min(std::max(8, per_stage * C), gx::stack_max_warps(sp.row_mode));
            smem = gx::stack_layout(sp, threads);
            if (smem != 0) return true;
        }
    }
    return false;
}

// MXFP4 jobs on the tensor cores (row mode 4): 16 + 16 gate/up rows, 8 rows
// of each of k = 4 experts per down job, the 12 role warps of the tensor-core
// jobs, three ring stages, the activations as e4m3 digit rows (per 32-element
// block: 2 K halves x k rows x 2 digits x 16 bytes, then the fp16 scales;
// the down inputs of a token's k slots interleaved in one row). On with
// GX_STACK_MMA=1 (opt-in: measured slower than the CUDA-core MXFP4 jobs,
// whose default it is not); on any shape it does not cover the CUDA-core
// MXFP4 jobs run.
bool choose_stack_tiles_tc(gx::StackParams & sp, int & threads, uint32_t & smem) {
    const char * env = std::getenv("GX_STACK_MMA");
    if (env == nullptr || std::strcmp(env, "1") != 0) return false;
    if (sp.k != 4 || sp.H % 64 != 0 || sp.I % 64 != 0) return false;
    const gx::StackParams keep = sp;
    const int nbh = sp.H / 32, nbi = sp.I / 32;
    sp.row_mode = 4;
    sp.Rg = 16;
    sp.Rd = 8;
    sp.W = 12;
    sp.alx.d_off = 64 * nbh;
    sp.alx.bs_off = sp.alx.d_off;
    // the N = 16 B tiles of the last block read up to 224 bytes past the digits
    sp.alx.pitch = gx::align16i((int64_t)sp.alx.d_off + std::max(2 * nbh, 256));
    const int64_t tok = 64ll * sp.k * nbi + std::max(2ll * sp.k * nbi, 256ll);   // a token's k digit rows and scales
    const int64_t tok_al = (tok + 16 * sp.k - 1) / (16 * sp.k) * (16 * sp.k);
    sp.ald.d_off = 64 * sp.k * nbi;
    sp.ald.bs_off = sp.ald.d_off;
    sp.ald.pitch = (int32_t)(tok_al / sp.k);
    for (int C = 3; C >= 2; --C) {
        sp.C = C;
        smem = gx::stack_layout(sp, threads);
        if (smem != 0) return true;
    }
    sp = keep;
    return false;
}

// MXFP4 jobs on the tensor cores fed by TMA (row mode 5, gx_stack_tma.cuh):
// 64 + 64 gate/up rows, 32 rows of each of k = 4 experts per down job, read
// from a copy of the slots in the tensor-core record layout. The default for
// such stacks; GX_STACK_MMA=0 keeps them on the CUDA cores (row mode 3) and
// GX_STACK_MMA=1 selects row mode 4.
bool choose_stack_tiles_t5(gx::StackParams & sp, int & threads, uint32_t & smem) {
    const char * env = std::getenv("GX_STACK_MMA");
    if (env != nullptr && std::strcmp(env, "2") != 0) return false;
    if (sp.k != 4 || sp.H % 64 != 0 || sp.I % 64 != 0 || tensor_map_encoder() == nullptr) return false;
    const gx::StackParams keep = sp;
    const int nbh = sp.H / 32, nbi = sp.I / 32;
    sp.row_mode = 5;
    sp.Rg = 64;
    sp.Rd = 32;
    sp.W = gx::kT5Warps - 4;   // warps 4..: epilogue, tails, more MMA issuers and producers
    sp.C = 1;
    sp.alx.d_off = 64 * nbh;
    sp.alx.bs_off = sp.alx.d_off;
    sp.alx.pitch = gx::align16i((int64_t)sp.alx.d_off + std::max(2 * nbh, 256));
    const int64_t tok = 64ll * sp.k * nbi + std::max(2ll * sp.k * nbi, 256ll);
    const int64_t tok_al = (tok + 16 * sp.k - 1) / (16 * sp.k) * (16 * sp.k);
    sp.ald.d_off = 64 * sp.k * nbi;
    sp.ald.bs_off = sp.ald.d_off;
    sp.ald.pitch = (int32_t)(tok_al / sp.k);
    smem = gx::stack_layout(sp, threads);
    if (smem != 0) return true;
    sp = keep;
    return false;
}

// The MXFP4 matrices of a layer's record: down (H rows of I), gate and up (I
// rows of H), and their places in the tensor-core record (32-byte aligned).
gx::Mxfp4TcMats mxfp4_mats(const LayerPlan & lp, int64_t * tc_record = nullptr) {
    const uint8_t * base = lp.dn.w0;
    gx::Mxfp4TcMats m{};
    m.off[0] = 0;
    m.off[1] = lp.g.w0 - base;
    m.off[2] = lp.g.w1 - base;
    m.rows[0] = (int32_t)lp.H;
    m.rows[1] = m.rows[2] = (int32_t)lp.I;
    m.nb[0] = (int32_t)(lp.I / 32);
    m.nb[1] = m.nb[2] = (int32_t)(lp.H / 32);
    m.trows[0] = 32;                 // down jobs: 32 rows of each expert
    m.trows[1] = m.trows[2] = 64;    // gate/up jobs: 64 gate + 64 up rows
    int64_t at = 0;
    for (int q = 0; q < 3; ++q) {
        m.doff[q] = at;
        at += ((int64_t)m.rows[q] * (gx::mxfp4_tc_cstride(m.nb[q]) + m.nb[q]) + 31) / 32 * 32;
    }
    if (tc_record) *tc_record = at;
    return m;
}

// The codes of one matrix of every slot of a layer in TMA-box order as a 5-D
// tensor of 4-bit values (x: 128 elements = 4 blocks of a row, y: row of a
// tile, z: chunk, w: tile, v: slot), unpacked by TMA into 16-byte groups of
// 16 with the 128-byte swizzle; a box (128 elements x trows rows) is one
// contiguous run.
bool encode_codes_map(CUtensorMap * map, const void * base, int64_t nch, int64_t trows, int64_t tiles, int64_t slots,
                      int64_t record) {
    const auto enc = tensor_map_encoder();
    if (enc == nullptr || (reinterpret_cast<uintptr_t>(base) & 31u) != 0 || record % 32 != 0) return false;
    // row length a multiple of 128 elements, strides of 32 bytes (16U4_ALIGN16B)
    const cuuint64_t dims[5] = {128u, (cuuint64_t)trows, (cuuint64_t)nch, (cuuint64_t)tiles, (cuuint64_t)slots};
    const cuuint64_t strides[4] = {64u, (cuuint64_t)(64 * trows), (cuuint64_t)(64 * trows * nch), (cuuint64_t)record};
    const cuuint32_t box[5] = {128u, (cuuint32_t)trows, 1u, 1u, 1u};
    const cuuint32_t elem[5] = {1u, 1u, 1u, 1u, 1u};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 5, const_cast<void *>(base), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Slot `slot` of plan layer i into the tensor-core layout copy, on stream s,
// when the arena has filled it since the copy was made.
void t5_follow_slot(gx_stack_plan * p, uint32_t i, int32_t slot, cudaStream_t s) {
    gx_arena * a = p->a;
    const uint32_t li = p->lps[i].li;
    uint32_t & gen = p->shadow_gen[i][(size_t)slot];
    if (gen == a->slot_gen[li][(size_t)slot]) return;
    int64_t trec = 0;
    const gx::Mxfp4TcMats m = mxfp4_mats(p->lps[i], &trec);
    ck(gx::launch_mxfp4_tc_layout(a->d_arena + a->slab_base[li] + (uint64_t)slot * a->record[li],
                                  p->d_shadow + p->shadow_base[i] + (uint64_t)slot * (uint64_t)trec, m, s));
    gen = a->slot_gen[li][(size_t)slot];
}

// Row mode 5: the slot copies in the tensor-core layout (every slot now),
// their tensor maps, and the layer table pointed at the copies.
int setup_t5(gx_stack_plan * p) {
    gx_arena * a = p->a;
    gx::StackParams & sp = p->sp;
    uint64_t total = 0;
    p->shadow_base.assign(p->n, 0);
    p->shadow_gen.assign(p->n, {});
    for (uint32_t i = 0; i < p->n; ++i) {
        int64_t trec = 0;
        mxfp4_mats(p->lps[i], &trec);
        p->shadow_base[i] = total;
        total += (uint64_t)trec * (uint64_t)p->lps[i].g.n_as;
        p->shadow_gen[i].assign((size_t)p->lps[i].g.n_as, ~0u);
    }
    ck(cudaMalloc(&p->d_shadow, (size_t)total));
    ck(cudaMemset(p->d_shadow, 0, (size_t)total));   // row padding reads as zero codes
    std::vector<CUtensorMap> maps((size_t)p->n * 3);
    for (uint32_t i = 0; i < p->n; ++i) {
        const LayerPlan & lp = p->lps[i];
        int64_t trec = 0;
        const gx::Mxfp4TcMats m = mxfp4_mats(lp, &trec);
        uint8_t * lb = p->d_shadow + p->shadow_base[i];
        bool okm = true;
        for (int q = 0; q < 3 && okm; ++q) {
            const int idx = q == 0 ? 2 : q - 1;   // maps: gate, up, down
            okm = m.rows[q] % m.trows[q] == 0 &&
                  encode_codes_map(&maps[3 * i + idx], lb + m.doff[q], gx::mxfp4_tc_cstride(m.nb[q]) / 64, m.trows[q],
                                   m.rows[q] / m.trows[q], lp.g.n_as, trec);
        }
        if (!okm) return GX_ERR_ALIGN;
        gx::StackLayer & L = sp.layers[i];
        L.wg = lb + m.doff[1];
        L.wu = lb + m.doff[2];
        L.wd = lb + m.doff[0];
        L.nb02 = trec;
    }
    ck(cudaMalloc(&p->d_maps, maps.size() * sizeof(CUtensorMap)));
    ck(cudaMemcpy(p->d_maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice));
    sp.t5_maps = p->d_maps;
    // every slot now (a copy of what it holds, once its fills have landed),
    // then in step with the arena's fills
    ck(cudaStreamSynchronize(a->copy_stream));
    for (uint32_t i = 0; i < p->n; ++i)
        for (int32_t slot = 0; slot < p->lps[i].g.n_as; ++slot) t5_follow_slot(p, i, slot, nullptr);
    ck(cudaDeviceSynchronize());
    return GX_OK;
}

// Device buffers and the layer table of the stack kernel.
int setup_stack(gx_stack_plan * p, const float * const * x, const float * const * w, float * const * out) {
    gx_arena * a = p->a;
    const LayerPlan & l0 = p->lps[0];
    if (!gx::stack_types_supported(l0.type_gate, l0.type_down)) return GX_ERR_TYPE;
    if (p->n > (uint32_t)gx::kStackMaxLayers) return GX_ERR_INVALID;
    gx::StackParams & sp = p->sp;
    sp = gx::StackParams{};
    sp.NL = (int32_t)p->n;
    sp.skew = p->n >= 2 ? 2 : 1;
    sp.k = (int32_t)p->k;
    sp.T = (int32_t)p->T;
    sp.H = (int32_t)l0.H;
    sp.I = (int32_t)l0.I;
    sp.nb01_g = l0.g.nb01;
    sp.nb01_d = l0.dn.nb01;
    sp.alx = l0.g.al;
    sp.ald = l0.g.al2;
    sp.qblk = l0.g.qblk;
    sp.act = l0.g.act;
    sp.alpha = l0.g.alpha;
    sp.limit = l0.g.limit;
    sp.row_mode = (l0.type_gate == gx::GX_T_Q8_0 && l0.type_down == gx::GX_T_Q8_0)     ? 0
                  : (l0.type_gate == gx::GX_T_Q4_K && l0.type_down == gx::GX_T_Q6_K)   ? 2
                  : (l0.type_gate == gx::GX_T_MXFP4 && l0.type_down == gx::GX_T_MXFP4) ? 3
                                                                                       : 1;
    sp.gu_copies = (sp.row_mode == 1 || sp.row_mode == 3) ? 2 : 4;
    sp.need_grid = (l0.type_gate == gx::GX_T_IQ1_S || l0.type_down == gx::GX_T_IQ1_S) ? 1 : 0;
    int threads = 0;
    uint32_t smem = 0;
    // row mode 5 where its copies of the slots fit in free device memory with
    // 1 GiB to spare (else the CUDA-core rows)
    bool t5_fits = false;
    if (sp.row_mode == 3) {
        uint64_t need = 1ull << 30;
        for (uint32_t i = 0; i < p->n; ++i) {
            int64_t trec = 0;
            mxfp4_mats(p->lps[i], &trec);
            need += (uint64_t)trec * (uint64_t)p->lps[i].g.n_as;
        }
        size_t free_b = 0, total_b = 0;
        t5_fits = cudaMemGetInfo(&free_b, &total_b) == cudaSuccess && need <= (uint64_t)free_b;
    }
    if (!(sp.row_mode == 3 && ((t5_fits && choose_stack_tiles_t5(sp, threads, smem)) ||
                               choose_stack_tiles_tc(sp, threads, smem))) &&
        !choose_stack_tiles(sp, threads, smem))
        return GX_ERR_ALIGN;
    sp.split = sp.row_mode == 3 ? 4 : (sp.row_mode == 1 || (sp.row_mode == 2 && sp.k * sp.Rd == 32)) ? 2 : 1;
    sp.n_gu = (int32_t)(p->T * p->k * (l0.I / sp.Rg));
    sp.n_d = (int32_t)(p->T * (l0.H / sp.Rd));
    int per_sm = 0;
    ck(gx::prepare_stack(l0.type_gate, l0.type_down, sp, threads, smem, per_sm));
    if (per_sm > 1) per_sm = 1;   // one CTA per SM: the ring holds the SM's shared memory
    const int64_t n = p->n, T = p->T, k = p->k;
    const int64_t nblk = l0.I / sp.qblk;
    p->cnt_bytes = (size_t)(n + n * T + n * T * k * nblk) * sizeof(int32_t);
    ck(cudaMalloc(&p->d_cnt, p->cnt_bytes));
    ck(cudaMemset(p->d_cnt, 0, p->cnt_bytes));
    ck(cudaMalloc(&p->d_xq, (size_t)(n * T) * sp.alx.pitch));
    ck(cudaMalloc(&p->d_act, (size_t)(n * T * k * l0.I) * sizeof(float)));
    ck(cudaMalloc(&p->d_actq, (size_t)(n * T * k) * sp.ald.pitch));
    for (int64_t i = 0; i < n; ++i) {
        const LayerPlan & lp = p->lps[(size_t)i];
        gx::StackLayer & L = sp.layers[i];
        L.wg = lp.g.w0;
        L.wu = lp.g.w1;
        L.wd = lp.dn.w0;
        L.x = x[i];
        L.rw = w[i];
        L.out = out[i];
        L.slots = p->d_slots + i * k * T;
        L.xq = p->d_xq + (size_t)(i * T) * sp.alx.pitch;
        L.act = p->d_act + (size_t)(i * T * k) * l0.I;
        L.actq = p->d_actq + (size_t)(i * T * k) * sp.ald.pitch;
        L.cnt = p->d_cnt + n + n * T + i * T * k * nblk;
        L.nb02 = lp.g.nb02;
        L.n_as = lp.g.n_as;
        L.pad = 0;
    }
    sp.q_done = p->d_cnt;
    sp.gu_done = p->d_cnt + n;
    if (sp.row_mode == 5) {
        const int rc = setup_t5(p);
        if (rc != GX_OK) return rc;
    }
    p->threads = threads;
    p->smem = smem;
    p->per_sm = per_sm;
    p->grid = per_sm * gx::device_sms();
    p->stack = true;
    (void)a;
    return GX_OK;
}

}  // namespace

extern "C" {

int gx_moe_layer_forward(gx_arena * a, uint32_t layer, const gx_layer_desc * d, const float * x, const int32_t * ids,
                         const float * w, int64_t k, int64_t T, float * out, void * stream, gx_serve_stats * stats) {
    if (a == nullptr) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(a->mu);
        ck(cudaSetDevice(a->device));
        return layer_forward_locked(a, layer, d, x, ids, w, k, T, out, reinterpret_cast<cudaStream_t>(stream), stats);
    });
}

int gx_moe_layer_forward_shared(gx_arena * a, uint32_t layer, const gx_layer_desc * d, const float * x,
                                const int32_t * ids, const float * w, int64_t k, int64_t T,
                                const gx_shared_expert * sh, float * out, void * stream, gx_serve_stats * stats) {
    if (a == nullptr || sh == nullptr || x == nullptr || out == nullptr) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(a->mu);
        ck(cudaSetDevice(a->device));
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        if (T == 0) return GX_OK;
        LayerPlan sp;
        int rc = plan_shared(a, layer, sh, T, sp);
        if (rc != GX_OK) return rc;
        // the routed experts, then the shared expert into its own buffer
        rc = layer_forward_locked(a, layer, d, x, ids, w, k, T, out, s, stats);
        if (rc != GX_OK) return rc;
        if (a->d_shy == nullptr) ck(cudaMalloc(&a->d_shy, (size_t)a->max_tokens * (size_t)a->hidden * sizeof(float)));
        if (a->d_ones == nullptr) {
            const int64_t cap = (int64_t)a->used * a->max_tokens;
            ck(cudaMalloc(&a->d_ones, (size_t)cap * sizeof(float)));
            ck(gx::launch_fill(a->d_ones, cap, 1.0f, s));
            ck(cudaStreamSynchronize(s));
        }
        static const int32_t zeros[gx::kInlineIds] = {};
        const int32_t * slot0 = zeros;
        const int32_t * ids_dev = nullptr;
        if (T > gx::kInlineIds) {
            // slot ids of more than kInlineIds tokens through the pinned ring
            const int st = a->stage_next;
            a->stage_next = (st + 1) % kStageRing;
            const int64_t stride = (int64_t)a->used * a->max_tokens;
            ck(cudaEventSynchronize(a->ev_stage[st]));
            int32_t * h = a->h_ids + (size_t)st * stride;
            int32_t * dd = a->d_ids + (size_t)st * stride;
            std::memset(h, 0, (size_t)T * sizeof(int32_t));
            ck(cudaMemcpyAsync(dd, h, (size_t)T * sizeof(int32_t), cudaMemcpyHostToDevice, s));
            ck(cudaEventRecord(a->ev_stage[st], s));
            ids_dev = dd;
        }
        enqueue_layer(sp, x, a->d_ones, a->d_shy, ids_dev, slot0, s, false, false, nullptr);
        // out = moe_out + shexp (ggml_add)
        ck(gx::launch_add_inplace(out, a->d_shy, T * a->hidden, s));
        ck(cudaEventRecord(a->ev_done[sp.li], s));
        a->last_ev[sp.li] = a->ev_done[sp.li];
        return GX_OK;
    });
}

int gx_moe_stack_forward(gx_arena * a, uint32_t first_layer, uint32_t n_layers, const gx_layer_desc * d,
                         const float * const * x, const int32_t * ids, const float * const * w, int64_t k, int64_t T,
                         float * const * out, void * stream, gx_serve_stats * stats) {
    if (a == nullptr || x == nullptr || ids == nullptr || w == nullptr || out == nullptr) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(a->mu);
        ck(cudaSetDevice(a->device));
        gx_serve_stats sum{};
        for (uint32_t i = 0; i < n_layers; ++i) {
            gx_serve_stats st{};
            const int rc = layer_forward_locked(a, first_layer + i, d, x[i], ids + (size_t)i * k * T, w[i], k, T, out[i],
                                                reinterpret_cast<cudaStream_t>(stream), &st);
            if (rc != GX_OK) return rc;
            sum.hits += st.hits;
            sum.misses += st.misses;
            sum.evictions += st.evictions;
            sum.distinct += st.distinct;
            sum.bytes_copied += st.bytes_copied;
        }
        if (stats) *stats = sum;
        return GX_OK;
    });
}

int gx_stack_plan_destroy(gx_stack_plan * p) {
    if (p == nullptr) return GX_OK;
    if (p->a) cudaSetDevice(p->a->device);
    if (p->ev_graph) cudaEventSynchronize(p->ev_graph);
    if (p->exec) cudaGraphExecDestroy(p->exec);
    if (p->graph) cudaGraphDestroy(p->graph);
    for (auto e : p->tev) if (e) cudaEventDestroy(e);
    for (auto e : p->ev_h) if (e) cudaEventDestroy(e);
    if (p->ev_graph) cudaEventDestroy(p->ev_graph);
    if (p->d_slots) cudaFree(p->d_slots);
    for (auto h : p->h_slots) if (h) cudaFreeHost(h);
    if (p->d_cnt) cudaFree(p->d_cnt);
    if (p->d_xq) cudaFree(p->d_xq);
    if (p->d_act) cudaFree(p->d_act);
    if (p->d_actq) cudaFree(p->d_actq);
    if (p->d_shadow) cudaFree(p->d_shadow);
    if (p->d_maps) cudaFree(p->d_maps);
    if (p->d_table) cudaFree(p->d_table);
    if (p->d_ids) cudaFree(p->d_ids);
    delete p;
    return GX_OK;
}

int gx_stack_plan_create(gx_arena * a, uint32_t first_layer, uint32_t n_layers, const gx_layer_desc * d,
                         const float * const * x, const float * const * w, float * const * out, int64_t k, int64_t T,
                         int flags, gx_stack_plan ** out_plan) {
    if (a == nullptr || d == nullptr || x == nullptr || w == nullptr || out == nullptr || out_plan == nullptr ||
        n_layers == 0 || (flags & ~(GX_PLAN_TIMING | GX_PLAN_LAYERWISE)) != 0)
        return GX_ERR_INVALID;
    *out_plan = nullptr;
    gx_stack_plan * p = new (std::nothrow) gx_stack_plan();
    if (p == nullptr) return GX_ERR_NOMEM;
    const int rc = guarded([&] {
        std::lock_guard<std::mutex> lock(a->mu);
        ck(cudaSetDevice(a->device));
        const bool timing = (flags & GX_PLAN_TIMING) != 0;
        p->a = a;
        p->first = first_layer;
        p->n = n_layers;
        p->k = k;
        p->T = T;
        p->desc = *d;
        p->timing = timing ? 1 : 0;
        p->wp.assign(w, w + n_layers);
        p->lps.resize(n_layers);
        for (uint32_t i = 0; i < n_layers; ++i) {
            const int r = plan_layer(a, first_layer + i, d, k, T, p->lps[i]);
            if (r != GX_OK) return r;
        }
        const size_t bytes = (size_t)n_layers * k * T * sizeof(int32_t);
        ck(cudaMalloc(&p->d_slots, bytes));
        ck(cudaMemset(p->d_slots, 0, bytes));
        for (int j = 0; j < 2; ++j) {
            ck(cudaHostAlloc(&p->h_slots[j], bytes, cudaHostAllocDefault));
            ck(cudaEventCreateWithFlags(&p->ev_h[j], cudaEventDisableTiming));
        }
        ck(cudaEventCreateWithFlags(&p->ev_graph, cudaEventDisableTiming));
        const bool want_stack = (flags & GX_PLAN_LAYERWISE) == 0 && k * T <= gx::kInlineIds &&
                                n_layers <= (uint32_t)gx::kStackMaxLayers &&
                                gx::stack_types_supported(p->lps[0].type_gate, p->lps[0].type_down);
        if (want_stack) {
            const int r = setup_stack(p, x, w, out);
            if (r != GX_OK) return r;
        }
        if (timing) {
            p->tev.resize(p->stack ? 2 : (size_t)3 * n_layers);
            for (auto & e : p->tev) ck(cudaEventCreate(&e));
        }
        // warm every kernel configuration (attributes, occupancy) outside the capture
        if (!p->stack) {
            for (uint32_t i = 0; i < n_layers; ++i) {
                ck(gx::prepare_decode(p->lps[i].type_gate, 1, p->lps[i].g));
                ck(gx::prepare_decode(p->lps[i].type_down, 2, p->lps[i].dn));
            }
        }
        cudaStream_t cap;
        ck(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
        ck(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal));
        if (p->stack) {
            ck(cudaMemsetAsync(p->d_cnt, 0, p->cnt_bytes, cap));
            if (timing) ck(cudaEventRecordWithFlags(p->tev[0], cap, cudaEventRecordExternal));
            ck(gx::launch_stack(p->lps[0].type_gate, p->lps[0].type_down, p->sp, p->grid, p->threads, p->smem, cap));
            if (timing) ck(cudaEventRecordWithFlags(p->tev[1], cap, cudaEventRecordExternal));
        } else {
            for (uint32_t i = 0; i < n_layers; ++i) {
                cudaEvent_t * tv = timing ? &p->tev[(size_t)3 * i] : nullptr;
                enqueue_layer(p->lps[i], x[i], w[i], out[i], p->d_slots + (size_t)i * k * T, nullptr, cap, !timing,
                              !timing, tv);
            }
        }
        cudaGraph_t graph = nullptr;
        const cudaError_t ce = cudaStreamEndCapture(cap, &graph);
        cudaStreamDestroy(cap);
        ck(ce);
        p->graph = graph;
        ck(cudaGraphInstantiate(&p->exec, p->graph, 0));
        return GX_OK;
    });
    if (rc != GX_OK) {
        gx_stack_plan_destroy(p);
        return rc;
    }
    *out_plan = p;
    return GX_OK;
}

int gx_stack_plan_run(gx_stack_plan * p, const int32_t * ids, void * stream, gx_serve_stats * stats) {
    if (p == nullptr || ids == nullptr) return GX_ERR_INVALID;
    gx_arena * a = p->a;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(a->mu);
        ck(cudaSetDevice(a->device));
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        const int64_t per = p->k * p->T;
        int32_t * h = p->h_slots[p->cur];
        ck(cudaEventSynchronize(p->ev_h[p->cur]));     // the previous copy out of this buffer has run
        gx_serve_stats sum{};
        for (uint32_t i = 0; i < p->n; ++i) {
            gx_serve_stats st{};
            const uint32_t li = p->lps[i].li;
            const int rc = arena_serve(a, p->first + i, ids + (size_t)i * per, (uint32_t)per, h + (size_t)i * per,
                                       a->last_ev[li], s, &st, (uint32_t)p->T, (uint32_t)p->k);
            if (rc != GX_OK) return rc;
            if (p->d_shadow)   // slots filled by this serve: their tensor-core copies, after the fill on s
                for (int64_t j = 0; j < per; ++j) t5_follow_slot(p, i, h[(size_t)i * per + j], s);
            sum.hits += st.hits;
            sum.misses += st.misses;
            sum.evictions += st.evictions;
            sum.distinct += st.distinct;
            sum.bytes_copied += st.bytes_copied;
        }
        ck(cudaMemcpyAsync(p->d_slots, h, (size_t)p->n * per * sizeof(int32_t), cudaMemcpyHostToDevice, s));
        ck(cudaEventRecord(p->ev_h[p->cur], s));
        p->cur ^= 1;
        ck(cudaGraphLaunch(p->exec, s));
        ck(cudaEventRecord(p->ev_graph, s));
        for (uint32_t i = 0; i < p->n; ++i) a->last_ev[p->lps[i].li] = p->ev_graph;
        if (stats) *stats = sum;
        return GX_OK;
    });
}

int gx_stack_plan_timing(gx_stack_plan * p, double * gate_up_ms, double * down_ms) {
    if (p == nullptr || !p->timing) return GX_ERR_STATE;
    return guarded([&] {
        ck(cudaEventSynchronize(p->ev_graph));
        double gu = 0.0, dn = 0.0;
        if (p->stack) {
            float m = 0.f;
            ck(cudaEventElapsedTime(&m, p->tev[0], p->tev[1]));
            gu = m;
        } else {
            for (uint32_t i = 0; i < p->n; ++i) {
                float m1 = 0.f, m2 = 0.f;
                ck(cudaEventElapsedTime(&m1, p->tev[3 * i], p->tev[3 * i + 1]));
                ck(cudaEventElapsedTime(&m2, p->tev[3 * i + 1], p->tev[3 * i + 2]));
                gu += m1;
                dn += m2;
            }
        }
        if (gate_up_ms) *gate_up_ms = gu;
        if (down_ms) *down_ms = dn;
        return GX_OK;
    });
}

int gx_stack_plan_info_get(const gx_stack_plan * p, gx_stack_plan_info * info) {
    if (p == nullptr || info == nullptr) return GX_ERR_INVALID;
    *info = gx_stack_plan_info{};
    info->stack_kernel = p->stack ? 1 : 0;
    if (p->stack) {
        info->grid = p->grid;
        info->threads = p->threads;
        info->ctas_per_sm = p->per_sm;
        info->stages = p->sp.row_mode == 5 ? p->sp.tc_na : p->sp.C;
        info->rows_gate_up = p->sp.Rg;
        info->rows_down = p->sp.Rd;
        info->smem_bytes = p->smem;
        info->tensor_cores = p->sp.row_mode == 4 ? 1 : p->sp.row_mode == 5 ? 2 : 0;
    }
    return GX_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- router

namespace {

bool router_valid(const gx_router_desc * d) {
    if (d == nullptr) return false;
    const int E = d->n_expert, k = d->n_expert_used;
    if (d->gating < GX_GATING_SOFTMAX || d->gating > GX_GATING_SOFTMAX_WEIGHT) return false;
    if (k < 1 || k > gx::kRouterMaxUsed || E < k || E > gx::kRouterMaxExperts) return false;
    if (d->n_groups > 1) {
        const int G = d->n_groups;
        if (G > gx::kRouterMaxGroups || E % G != 0 || E / G < 2) return false;
        if (d->n_group_used < 1 || d->n_group_used > G || d->n_group_used * (E / G) < k) return false;
    }
    return true;
}

gx::RouterLaunch router_launch(const gx_router_desc * d, const float * logits, int64_t ld, const float * bias,
                               int64_t T, int64_t n_layers, int32_t * ids, float * w, const int32_t * table,
                               int32_t * slots) {
    gx::RouterLaunch r{};
    r.logits = logits;
    r.ld = ld;
    r.bias = bias;
    r.table = table;
    r.ids = ids;
    r.w = w;
    r.slots = slots;
    r.T = T;
    r.n_layers = n_layers;
    r.E = d->n_expert;
    r.k = d->n_expert_used;
    r.gating = d->gating;
    r.groups = d->n_groups > 1 ? d->n_groups : 0;
    r.group_used = d->n_group_used;
    r.norm = d->norm_w ? 1 : 0;
    r.scale_on = d->scale_w ? 1 : 0;
    r.scale = d->w_scale;
    return r;
}

// the slot of every expert of layers [first, first + n) into host [n, experts];
// false when require_all and some expert has none
bool collect_slot_table(const SlotPolicy & P, uint32_t first, uint32_t n, bool require_all, std::vector<int32_t> & h) {
    const uint32_t E = P.experts();
    h.assign((size_t)n * E, -1);
    for (uint32_t i = 0; i < n; ++i)
        for (uint32_t e = 0; e < E; ++e) {
            const int32_t s = P.slot_of(first + i, e);
            if (s < 0 && require_all) return false;
            h[(size_t)i * E + e] = s;
        }
    return true;
}

}  // namespace

extern "C" {

int gx_router_forward(const gx_router_desc * d, const float * logits, int64_t ld, const float * bias, int64_t T,
                      int64_t n_layers, int32_t * ids, float * weights, const int32_t * slot_table, int32_t * slots,
                      void * stream) {
    if (!router_valid(d) || T < 0 || n_layers < 0) return GX_ERR_INVALID;
    if (T * n_layers == 0) return GX_OK;
    if (logits == nullptr || ids == nullptr || weights == nullptr || ld < d->n_expert) return GX_ERR_INVALID;
    if ((slot_table == nullptr) != (slots == nullptr)) return GX_ERR_INVALID;
    return guarded([&] {
        ck(gx::launch_router(router_launch(d, logits, ld, bias, T, n_layers, ids, weights, slot_table, slots),
                             reinterpret_cast<cudaStream_t>(stream)));
        return GX_OK;
    });
}

int gx_arena_slot_table(gx_arena * a, uint32_t first_layer, uint32_t n_layers, int32_t * table, int require_all,
                        void * stream) {
    if (a == nullptr || table == nullptr || n_layers == 0) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(a->mu);
        const SlotPolicy & P = a->policy->impl;
        if (first_layer < P.first_layer() || first_layer + n_layers - 1 > P.last_layer()) return GX_ERR_INVALID;
        std::vector<int32_t> h;
        if (!collect_slot_table(P, first_layer, n_layers, require_all != 0, h)) return GX_ERR_STATE;
        ck(cudaSetDevice(a->device));
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        ck(cudaMemcpyAsync(table, h.data(), h.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s));
        ck(cudaStreamSynchronize(s));
        return GX_OK;
    });
}

int gx_stack_plan_run_routed(gx_stack_plan * p, const gx_router_desc * d, const float * logits, int64_t ld,
                             const float * bias, int32_t * ids_out, void * stream, gx_serve_stats * stats) {
    if (p == nullptr || !router_valid(d) || logits == nullptr || ld < (d ? d->n_expert : 0)) return GX_ERR_INVALID;
    gx_arena * a = p->a;
    const SlotPolicy & P = a->policy->impl;
    if ((uint32_t)d->n_expert != P.experts() || d->n_expert_used != p->k) return GX_ERR_INVALID;
    const int64_t per = p->k * p->T;
    for (uint32_t i = 1; i < p->n; ++i)
        if (p->wp[i] != p->wp[0] + (size_t)i * per) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(a->mu);
        ck(cudaSetDevice(a->device));
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        if (p->d_table == nullptr) {
            // pinned layers keep every slot for good: the table is built once
            std::vector<int32_t> h;
            if (!collect_slot_table(P, p->first, p->n, true, h)) return GX_ERR_STATE;
            ck(cudaMalloc(&p->d_table, h.size() * sizeof(int32_t)));
            ck(cudaMemcpy(p->d_table, h.data(), h.size() * sizeof(int32_t), cudaMemcpyHostToDevice));
        }
        int32_t * ids = ids_out;
        if (ids == nullptr) {
            if (p->d_ids == nullptr) ck(cudaMalloc(&p->d_ids, (size_t)p->n * per * sizeof(int32_t)));
            ids = p->d_ids;
        }
        ck(gx::launch_router(router_launch(d, logits, ld, bias, p->T, p->n, ids, const_cast<float *>(p->wp[0]),
                                           p->d_table, p->d_slots),
                             s));
        ck(cudaGraphLaunch(p->exec, s));
        ck(cudaEventRecord(p->ev_graph, s));
        for (uint32_t i = 0; i < p->n; ++i) a->last_ev[p->lps[i].li] = p->ev_graph;
        const uint64_t hits = (uint64_t)p->n * per;
        a->stats.serves += p->n;
        a->stats.hits += hits;
        if (stats) {
            *stats = gx_serve_stats{};
            stats->hits = hits;
        }
        if (gx::observer_enabled()) {
            // the ids exist on the device only: read them back for the trace
            p->h_ids.resize((size_t)p->n * per);
            ck(cudaMemcpyAsync(p->h_ids.data(), ids, p->h_ids.size() * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
            ck(cudaStreamSynchronize(s));
            for (uint32_t i = 0; i < p->n; ++i)
                observed(a->policy, p->first + i, p->h_ids.data() + (size_t)i * per, (uint32_t)per, (uint32_t)p->T,
                         (uint32_t)p->k, [](uint64_t & bytes) {
                             bytes = 0;
                             return GX_OK;
                         });
        }
        return GX_OK;
    });
}

// --------------------------------------------------------------- synthetic

int gx_synth_normal(float * dst, int64_t n, uint64_t seed, uint64_t stream_id, float sigma, void * stream) {
    if (dst == nullptr || n < 0) return GX_ERR_INVALID;
    return guarded([&] {
        ck(gx::launch_synth_normal(dst, n, seed, stream_id, sigma, reinterpret_cast<cudaStream_t>(stream)));
        return GX_OK;
    });
}

int gx_synth_weights(int type, void * dst, int64_t ne00, int64_t n_rows, uint64_t seed, uint64_t stream_id, float sigma,
                     void * stream) {
    if (!gx::supported_weight_type(type)) return GX_ERR_TYPE;
    if (dst == nullptr || ne00 <= 0 || n_rows < 0) return GX_ERR_INVALID;
    if (ne00 % gx::block_elems(type) != 0) return GX_ERR_ALIGN;
    return guarded([&] {
        ck(gx::launch_synth_weights(type, dst, ne00, n_rows, seed, stream_id, sigma, reinterpret_cast<cudaStream_t>(stream)));
        return GX_OK;
    });
}

}  // extern "C"
