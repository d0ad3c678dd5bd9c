// TEST INFRASTRUCTURE ONLY -- drives the reference's own slot policy.
//
// Built by oracle/Makefile from the reference's src/h4 sources where they lie
// (never copied): ExpertCache (src/h4/h4-expert-cache.cpp) gives the per-access
// outcome (hit, eviction) and ExpertStore::warm (src/h4/h4-expert-store.cpp:
// 197-211) gives the slot each key occupies, with no I/O. The product's policy
// is checked against this binary, access by access and slot by slot.
//
// Input on stdin (text):
//   capacity_bytes protected_fraction n_batches
//   then per batch:  layer count expert_0 ... expert_{count-1}
// The model geometry comes from GALACTUS_PROFILE (a profile sidecar written by
// the test) and the policy from GALACTUS_H4_CACHE_POLICY, both read by the
// reference code itself.
//
// Output on stdout, per batch:
//   B <layer> <count>
//   A <hit> <evicted> <evicted_expert>        one line per access, in order
//   S <slot_0> ... <slot_{count-1}>            store slot of each key after the batch
//   R <expert ids resident in that layer after the batch, ascending>

#include "h4-core.hpp"
#include "h4-expert-cache.hpp"
#include "h4-expert-store.hpp"
#include "h4-profile.hpp"
#include "h4-reader.hpp"

#include <cstdio>
#include <cstdlib>
#include <fcntl.h>
#include <iostream>
#include <string>
#include <unistd.h>
#include <vector>

using namespace galactus::h4;

static std::string make_temp_file() {
    char pattern[] = "/tmp/h4ref-volume-XXXXXX";
    const int fd = mkstemp(pattern);
    if (fd < 0) throw std::runtime_error("mkstemp failed");
    // one 16 KiB block so that the reader can open and size the volume
    std::vector<char> block(record_alignment_bytes, 0);
    if (write(fd, block.data(), block.size()) != (ssize_t)block.size()) throw std::runtime_error("write failed");
    close(fd);
    return pattern;
}

int main() try {
    std::uint64_t capacity = 0;
    double fraction = 0.0;
    std::uint32_t n_batches = 0;
    if (!(std::cin >> capacity >> fraction >> n_batches)) {
        std::fprintf(stderr, "h4ref_replay: bad header\n");
        return 2;
    }
    const std::string internal_path = make_temp_file();
    const std::string external_path = make_temp_file();
    int rc = 0;
    {
        DualVolumeReader reader(internal_path, external_path, 1, record_alignment_bytes, 1ULL << 26, false);
        P0Layout layout(frozen_layer_record_bytes());
        ExpertCache cache(capacity, fraction);
        ExpertStore store(capacity, fraction, reader, layout);
        const auto & profile = ModelProfile::active();
        std::printf("Q");
        for (std::uint32_t layer = profile.first_layer; layer <= profile.last_layer; ++layer) {
            std::printf(" %u:%u:%u", cache.quota_of(layer), cache.protected_quota_of(layer),
                        cache.probation_quota_of(layer));
        }
        std::printf("\n");
        for (std::uint32_t b = 0; b < n_batches; ++b) {
            std::uint32_t layer = 0, count = 0;
            std::cin >> layer >> count;
            std::vector<std::uint32_t> keys(count);
            for (auto & key : keys) {
                std::uint32_t expert = 0;
                std::cin >> expert;
                key = (layer << key_expert_bits) | expert;
            }
            std::printf("B %u %u\n", layer, count);
            cache.begin_batch(layer);
            for (const auto key : keys) {
                const auto a = cache.access(key);
                std::printf("A %d %d %u\n", a.hit ? 1 : 0, a.evicted ? 1 : 0,
                            a.evicted ? (a.evicted_key & key_expert_mask) : 0U);
            }
            store.warm(keys);
            std::printf("S");
            for (const auto key : keys) std::printf(" %d", (int)store.slot_of(key));
            std::printf("\nR");
            for (std::uint32_t e = 0; e < profile.experts; ++e) {
                if (cache.resident((layer << key_expert_bits) | e)) std::printf(" %u", e);
            }
            std::printf("\n");
        }
    }
    unlink(internal_path.c_str());
    unlink(external_path.c_str());
    return rc;
} catch (const std::exception & error) {
    std::fprintf(stderr, "h4ref_replay: %s\n", error.what());
    return 1;
}
