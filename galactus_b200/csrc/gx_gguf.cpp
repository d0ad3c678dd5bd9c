// GGUF routed-expert reader: fills an arena's pinned host tier from a GGUF
// checkpoint, record by record (host only).
//
// A routed MoE layer L holds its experts in three 3-D tensors
// blk.L.ffn_{down,gate,up}_exps.weight of shape [ne0, ne1, n_expert]; expert
// e's rows of a role are the contiguous bytes [e*per_expert, (e+1)*per_expert).
// The record of (L, e) is the concatenation down | gate | up of those slices,
// padded to 16 KiB, the layout of the reference's packs and profile
// (scripts/moe-profile.py:116-211); the tier is layer-major, expert-minor.
// GGUF container (version 2 and 3): magic, version, tensor and key/value
// counts, key/value pairs, tensor infos (name, dims, ggml type, offset in the
// data section), data section at general.alignment (default 32).
// FNV-1a 64 (offset 14695981039346656037, prime 1099511628211) is the record
// fingerprint the reference's paranoia check compares
// (scripts/verify-paranoia-trace.py:8-20).
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <new>
#include <string>
#include <vector>

#include "../../include/galactus_b200.h"

namespace {

struct TensorInfo {
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0;   // absolute file offset of the data
};

struct GgufFile {
    std::string arch;
    std::map<std::string, uint64_t> ints;   // integer metadata
    std::map<std::string, TensorInfo> tensors;
};

struct Reader {
    std::ifstream in;
    bool ok = true;
    template <typename T>
    T get() {
        T v{};
        in.read(reinterpret_cast<char *>(&v), sizeof(T));
        if (!in) ok = false;
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (1u << 24)) {
            ok = false;
            return {};
        }
        std::string s(n, '\0');
        in.read(&s[0], (std::streamsize)n);
        if (!in) ok = false;
        return s;
    }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;   // u8 i8 bool
        case 2: case 3: return 2;           // u16 i16
        case 4: case 5: case 6: return 4;   // u32 i32 f32
        case 10: case 11: case 12: return 8;   // u64 i64 f64
        default: return 0;
    }
}

bool read_int(Reader & r, uint32_t t, uint64_t & v) {
    switch (t) {
        case 0: v = r.get<uint8_t>(); return true;
        case 1: v = (uint64_t)(int64_t)r.get<int8_t>(); return true;
        case 2: v = r.get<uint16_t>(); return true;
        case 3: v = (uint64_t)(int64_t)r.get<int16_t>(); return true;
        case 4: v = r.get<uint32_t>(); return true;
        case 5: v = (uint64_t)(int64_t)r.get<int32_t>(); return true;
        case 10: v = r.get<uint64_t>(); return true;
        case 11: v = (uint64_t)r.get<int64_t>(); return true;
        default: return false;
    }
}

bool skip_value(Reader & r, uint32_t t) {
    if (t == 8) {
        r.str();
        return r.ok;
    }
    if (t == 9) {
        const uint32_t et = r.get<uint32_t>();
        const uint64_t n = r.get<uint64_t>();
        if (!r.ok) return false;
        if (et == 8) {
            for (uint64_t i = 0; i < n && r.ok; ++i) r.str();
            return r.ok;
        }
        const size_t sz = scalar_size(et);
        if (sz == 0) return false;
        r.in.seekg((std::streamoff)(n * sz), std::ios::cur);
        return (bool)r.in;
    }
    const size_t sz = scalar_size(t);
    if (sz == 0) return false;
    r.in.seekg((std::streamoff)sz, std::ios::cur);
    return (bool)r.in;
}

int parse(const char * path, GgufFile & g, std::string & why) {
    Reader r;
    r.in.open(path, std::ios::binary);
    if (!r.in) {
        why = "cannot open";
        return GX_ERR_INVALID;
    }
    char magic[4];
    r.in.read(magic, 4);
    if (!r.in || std::memcmp(magic, "GGUF", 4) != 0) {
        why = "not a GGUF file";
        return GX_ERR_INVALID;
    }
    const uint32_t version = r.get<uint32_t>();
    if (version < 2 || version > 3) {
        why = "unsupported GGUF version";
        return GX_ERR_INVALID;
    }
    const uint64_t n_tensors = r.get<uint64_t>();
    const uint64_t n_kv = r.get<uint64_t>();
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        const std::string key = r.str();
        const uint32_t t = r.get<uint32_t>();
        if (!r.ok) break;
        uint64_t v = 0;
        if (t == 8 && key == "general.architecture") {
            g.arch = r.str();
        } else if (read_int(r, t, v)) {
            g.ints[key] = v;
            if (key == "general.alignment") alignment = v;
        } else if (!skip_value(r, t)) {
            r.ok = false;
        }
    }
    std::vector<std::pair<std::string, TensorInfo>> infos;
    for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
        std::string name = r.str();
        TensorInfo ti;
        const uint32_t nd = r.get<uint32_t>();
        if (nd > 4) r.ok = false;
        for (uint32_t d = 0; d < nd && r.ok; ++d) ti.dims.push_back(r.get<uint64_t>());
        ti.type = r.get<uint32_t>();
        ti.offset = r.get<uint64_t>();
        infos.emplace_back(std::move(name), std::move(ti));
    }
    if (!r.ok) {
        why = "truncated header";
        return GX_ERR_INVALID;
    }
    if (alignment == 0 || (alignment & (alignment - 1)) != 0) {
        why = "bad alignment";
        return GX_ERR_INVALID;
    }
    const uint64_t pos = (uint64_t)r.in.tellg();
    const uint64_t data = (pos + alignment - 1) / alignment * alignment;
    for (auto & [name, ti] : infos) {
        ti.offset += data;
        g.tensors[name] = ti;
    }
    return GX_OK;
}

uint64_t row_bytes_of(uint32_t type, uint64_t ne0) {
    switch (type) {
        case GX_TYPE_Q8_0: return ne0 / 32 * 34;
        case GX_TYPE_Q4_K: return ne0 / 256 * 144;
        case GX_TYPE_Q6_K: return ne0 / 256 * 210;
        case GX_TYPE_IQ1_S: return ne0 / 256 * 50;
        case GX_TYPE_MXFP4: return ne0 / 32 * 17;
        default: return 0;
    }
}

}  // namespace

extern "C" {

uint64_t gx_fnv1a64(const void * data, uint64_t n) {
    const uint8_t * p = static_cast<const uint8_t *>(data);
    uint64_t h = 14695981039346656037ull;
    for (uint64_t i = 0; i < n; ++i) h = (h ^ p[i]) * 1099511628211ull;
    return h;
}

int gx_gguf_moe_info(const char * path, gx_gguf_moe * info) {
    if (path == nullptr || info == nullptr) return GX_ERR_INVALID;
    GgufFile g;
    std::string why;
    const int rc = parse(path, g, why);
    if (rc != GX_OK) {
        std::fprintf(stderr, "galactus_b200: %s: %s\n", path, why.c_str());
        return rc;
    }
    *info = gx_gguf_moe{};
    std::strncpy(info->arch, g.arch.c_str(), sizeof(info->arch) - 1);
    auto meta = [&](const char * suffix) -> uint64_t {
        auto it = g.ints.find(g.arch + "." + suffix);
        return it == g.ints.end() ? 0 : it->second;
    };
    info->experts = (uint32_t)meta("expert_count");
    info->used = (uint32_t)meta("expert_used_count");
    info->block_count = (uint32_t)meta("block_count");
    uint32_t first = UINT32_MAX, last = 0, n = 0;
    for (uint32_t L = 0; L < info->block_count || (info->block_count == 0 && L < 4096); ++L) {
        const std::string pre = "blk." + std::to_string(L) + ".ffn_";
        if (g.tensors.count(pre + "down_exps.weight") == 0) continue;
        first = std::min(first, L);
        last = std::max(last, L);
        ++n;
        const TensorInfo & d = g.tensors[pre + "down_exps.weight"];
        auto gi = g.tensors.find(pre + "gate_exps.weight");
        auto ui = g.tensors.find(pre + "up_exps.weight");
        if (gi == g.tensors.end() || ui == g.tensors.end() || d.dims.size() != 3) return GX_ERR_INVALID;
        if (n == 1) {
            info->type_down = d.type;
            info->type_gate = gi->second.type;
            info->type_up = ui->second.type;
            info->hidden = d.dims[1];
            info->intermediate = d.dims[0];
        }
    }
    if (n == 0) return GX_ERR_INVALID;   // no routed-expert tensors: a dense model
    if (n != last - first + 1) return GX_ERR_INVALID;   // routed layers must be contiguous
    info->first_layer = first;
    info->last_layer = last;
    const uint64_t raw = row_bytes_of(info->type_down, info->intermediate) * info->hidden +
                         row_bytes_of(info->type_gate, info->hidden) * info->intermediate +
                         row_bytes_of(info->type_up, info->hidden) * info->intermediate;
    info->record_bytes_raw = raw;
    info->record_bytes = (raw + 16383) / 16384 * 16384;
    return GX_OK;
}

int gx_arena_load_gguf(gx_arena * arena, const char * path, uint32_t * records_loaded) {
    if (arena == nullptr || path == nullptr) return GX_ERR_INVALID;
    GgufFile g;
    std::string why;
    int rc = parse(path, g, why);
    if (rc != GX_OK) {
        std::fprintf(stderr, "galactus_b200: %s: %s\n", path, why.c_str());
        return rc;
    }
    std::ifstream in(path, std::ios::binary);
    if (!in) return GX_ERR_INVALID;
    gx_policy * pol = gx_arena_policy(arena);
    uint32_t loaded = 0;
    std::vector<uint8_t> rec;
    for (uint32_t L = 0;; ++L) {
        uint32_t q = 0, pq = 0, bq = 0;
        if (gx_policy_quota(pol, L, &q, &pq, &bq) != GX_OK) {
            if (loaded > 0) break;   // past the arena's last layer
            if (L > 4096) return GX_ERR_INVALID;
            continue;                // before its first layer
        }
        const std::string pre = "blk." + std::to_string(L) + ".ffn_";
        const char * roles[3] = {"down", "gate", "up"};
        const TensorInfo * t[3];
        for (int r = 0; r < 3; ++r) {
            auto it = g.tensors.find(pre + roles[r] + "_exps.weight");
            if (it == g.tensors.end() || it->second.dims.size() != 3) return GX_ERR_INVALID;
            t[r] = &it->second;
        }
        const uint64_t E = t[0]->dims[2];
        uint64_t per[3];
        uint64_t raw = 0;
        for (int r = 0; r < 3; ++r) {
            if (t[r]->dims[2] != E) return GX_ERR_INVALID;
            const uint64_t rb = row_bytes_of(t[r]->type, t[r]->dims[0]);
            if (rb == 0) return GX_ERR_TYPE;
            per[r] = rb * t[r]->dims[1];
            raw += per[r];
        }
        rec.assign(raw, 0);
        for (uint64_t e = 0; e < E; ++e) {
            uint64_t off = 0;
            for (int r = 0; r < 3; ++r) {
                in.seekg((std::streamoff)(t[r]->offset + e * per[r]));
                in.read(reinterpret_cast<char *>(rec.data() + off), (std::streamsize)per[r]);
                if (!in) return GX_ERR_INVALID;
                off += per[r];
            }
            rc = gx_load_record(arena, L, (uint32_t)e, rec.data(), raw);
            if (rc != GX_OK) return rc;
            ++loaded;
        }
    }
    if (records_loaded) *records_loaded = loaded;
    return loaded > 0 ? GX_OK : GX_ERR_INVALID;
}

}  // extern "C"
