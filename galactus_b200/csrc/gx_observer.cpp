// Route observer: what each served micro-batch asked for and what was already
// resident (host only, observational). Mirrors the reference's RouteObserver
// (src/h4/h4-route-observer.hpp:58-304): entries are buffered in memory during
// the run and written once, in its "galactus.route-observer.v1" text format,
// so the reference's replay tooling reads our traces. Switched on by
// GALACTUS_H4_ROUTES=<file> (read at the first serve) or gx_route_observer_open;
// it never touches a policy, an arena or a tensor.
#include "gx_observer.hpp"

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/galactus_b200.h"

namespace gx {

namespace {

struct Entry {
    uint32_t layer, tokens, k;
    uint64_t enter_ns, serve_start_ns, serve_end_ns, gap_ns, bytes_read;
    size_t id_offset;
};

struct Observer {
    std::mutex mu;
    std::FILE * file = nullptr;
    bool env_checked = false;
    std::string arch = "unknown";
    uint64_t cap = 4000000;
    bool truncated = false;
    uint64_t last_exit_ns = 0;
    // configuration line and geometry (from the first arena or policy that records)
    bool configured = false;
    uint64_t cache_bytes = 0;
    double protected_fraction = 0.0;
    uint32_t quota = 0, probation = 0, slots = 0;
    uint32_t first_layer = 0, last_layer = 0, experts = 0, used = 0;
    std::vector<uint64_t> record_bytes;
    std::vector<Entry> entries;
    std::vector<int32_t> ids;
    std::vector<uint8_t> resident;

    void write_and_close() {
        if (file == nullptr) return;
        std::FILE * f = file;
        std::fprintf(f, "# galactus.route-observer.v1\n");
        std::fprintf(f, "# arch %s\n", arch.c_str());
        std::fprintf(f, "# first_layer %u last_layer %u experts %u used %u\n", first_layer, last_layer, experts, used);
        std::fprintf(f, "# cache_bytes %llu protected %.2f quota %u probation %u slots %u\n",
                     (unsigned long long)cache_bytes, protected_fraction, quota, probation, slots);
        for (size_t i = 0; i < record_bytes.size(); ++i)
            std::fprintf(f, "# record %u %llu\n", first_layer + (uint32_t)i, (unsigned long long)record_bytes[i]);
        std::fprintf(f, "# entries %zu truncated %d\n", entries.size(), truncated ? 1 : 0);
        std::fprintf(f,
                     "# e <seq> <layer> <tokens> <k> <enter_ns> <serve_start_ns> <serve_end_ns> <gap_ns> "
                     "<bytes_read> then <id>:<resident>...\n");
        std::fprintf(f, "# r <seq> <ranks_per_token> then <id>...\n");
        for (size_t e = 0; e < entries.size(); ++e) {
            const Entry & x = entries[e];
            std::fprintf(f, "e %zu %u %u %u %llu %llu %llu %llu %llu", e, x.layer, x.tokens, x.k,
                         (unsigned long long)x.enter_ns, (unsigned long long)x.serve_start_ns,
                         (unsigned long long)x.serve_end_ns, (unsigned long long)x.gap_ns,
                         (unsigned long long)x.bytes_read);
            const size_t n = (size_t)x.tokens * x.k;
            for (size_t i = 0; i < n; ++i)
                std::fprintf(f, " %d:%u", ids[x.id_offset + i], (unsigned)resident[x.id_offset + i]);
            std::fputc('\n', f);
        }
        std::fflush(f);
        std::fclose(f);
        file = nullptr;
        entries.clear();
        ids.clear();
        resident.clear();
        configured = false;
        truncated = false;
        last_exit_ns = 0;
    }
};

Observer & obs() {
    // leaked on purpose: the atexit writer must find it alive
    static Observer * o = new Observer();
    return *o;
}

bool open_locked(Observer & o, const char * path, const char * arch, uint64_t cap) {
    if (o.file) o.write_and_close();
    o.file = std::fopen(path, "w");
    if (o.file == nullptr) return false;
    o.arch = arch && arch[0] ? arch : "unknown";
    o.cap = cap ? cap : 4000000;   // the reference's default entry cap
    static bool registered = false;
    if (!registered) {
        registered = true;
        std::atexit([] {
            Observer & ob = obs();
            std::lock_guard<std::mutex> lock(ob.mu);
            ob.write_and_close();
        });
    }
    return true;
}

}  // namespace

uint64_t observer_now_ns() {
    return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

bool observer_enabled() {
    Observer & o = obs();
    std::lock_guard<std::mutex> lock(o.mu);
    if (!o.env_checked) {
        o.env_checked = true;
        const char * path = std::getenv("GALACTUS_H4_ROUTES");
        if (path && path[0] && o.file == nullptr) {
            const char * cap = std::getenv("GALACTUS_H4_ROUTES_CAP");
            if (!open_locked(o, path, nullptr, cap && cap[0] ? std::strtoull(cap, nullptr, 10) : 0))
                std::fprintf(stderr, "galactus_b200: cannot open %s, route observation is off\n", path);
        }
    }
    return o.file != nullptr;
}

void observer_record(const ObserverGeometry & g, uint32_t layer, uint32_t tokens, uint32_t k, const int32_t * ids,
                     const uint8_t * resident, uint64_t enter_ns, uint64_t serve_start_ns, uint64_t serve_end_ns,
                     uint64_t bytes_read) {
    Observer & o = obs();
    std::lock_guard<std::mutex> lock(o.mu);
    if (o.file == nullptr) return;
    if (!o.configured) {
        o.configured = true;
        o.cache_bytes = g.cache_bytes;
        o.protected_fraction = g.protected_fraction;
        o.quota = g.quota;
        o.probation = g.probation;
        o.slots = g.slots;
        o.first_layer = g.first_layer;
        o.last_layer = g.last_layer;
        o.experts = g.experts;
        o.used = g.used;
        o.record_bytes.assign(g.record_bytes, g.record_bytes + (g.last_layer - g.first_layer + 1));
    }
    if (o.entries.size() >= o.cap) {
        o.truncated = true;
        return;
    }
    Entry e{};
    e.layer = layer;
    e.tokens = tokens;
    e.k = k;
    e.enter_ns = enter_ns;
    e.serve_start_ns = serve_start_ns;
    e.serve_end_ns = serve_end_ns;
    e.gap_ns = o.last_exit_ns == 0 ? 0 : enter_ns - o.last_exit_ns;
    e.bytes_read = bytes_read;
    e.id_offset = o.ids.size();
    const size_t n = (size_t)tokens * k;
    o.ids.insert(o.ids.end(), ids, ids + n);
    o.resident.insert(o.resident.end(), resident, resident + n);
    o.entries.push_back(e);
    o.last_exit_ns = observer_now_ns();
}

}  // namespace gx

extern "C" {

int gx_route_observer_open(const char * path, const char * arch, uint64_t entry_cap) {
    if (path == nullptr) return GX_ERR_INVALID;
    gx::Observer & o = gx::obs();
    std::lock_guard<std::mutex> lock(o.mu);
    o.env_checked = true;
    return gx::open_locked(o, path, arch, entry_cap) ? GX_OK : GX_ERR_INVALID;
}

int gx_route_observer_close(void) {
    gx::Observer & o = gx::obs();
    std::lock_guard<std::mutex> lock(o.mu);
    o.write_and_close();
    return GX_OK;
}

}  // extern "C"
