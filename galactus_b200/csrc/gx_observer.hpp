// Route observer hooks used by the serve paths (host only).
#pragma once

#include <cstdint>

namespace gx {

// The context line and geometry of the engine that records (first caller wins).
struct ObserverGeometry {
    uint64_t cache_bytes;
    double protected_fraction;
    uint32_t quota, probation, slots;
    uint32_t first_layer, last_layer, experts, used;
    const uint64_t * record_bytes;   // [last_layer - first_layer + 1]
};

uint64_t observer_now_ns();
// true when a trace file is open (GALACTUS_H4_ROUTES, checked at the first call)
bool observer_enabled();
// one served micro-batch: ids [tokens*k] token-major, resident [tokens*k]
// sampled before the serve
void observer_record(const ObserverGeometry & g, uint32_t layer, uint32_t tokens, uint32_t k, const int32_t * ids,
                     const uint8_t * resident, uint64_t enter_ns, uint64_t serve_start_ns, uint64_t serve_end_ns,
                     uint64_t bytes_read);

}  // namespace gx
