// One routed-expert FFN layer for callers that cannot allocate device memory.
//
// Who needs this: code that runs where cudaMalloc is off limits -- inside a
// host framework that owns every device allocation through its own pool and
// forbids others, inside a plugin loaded into such a process, or on a path
// whose latency budget cannot absorb an allocation (and the implicit device
// synchronization cudaFree brings). gx_moe_layer_forward needs an arena
// (created once with cudaMalloc'd scratch); this entry point needs nothing
// but the caller's buffers.
//
// Its scratch -- the quantized layer inputs, the f32 activation, the quantized
// activation and the per-block completion counters of the fused kernels --
// lives in one file-scope __device__ array of kNoAllocScratchBytes. Every GPU
// that loads this library holds that array until the process exits. The array
// is shared by every call on a device: calls whose kernels overlap on the GPU
// (two streams, or two host threads) race on it and must be serialized by the
// caller. Each call clears the counters it needs before its kernels run; the
// other regions are fully rewritten by each call.
//
// Each call outside a stream capture resolves the array's device address with
// cudaGetSymbolAddress (with its device current) and caches it; a call during
// a capture uses the cached address, so make one call on the device before
// capturing (a context reset between them needs another call outside a
// capture).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/galactus_b200.h"
#include "gx_formats.h"
#include "gx_kernels.h"

namespace {

constexpr uint64_t kNoAllocScratchBytes = (uint64_t)GX_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_addr_mu;
uint8_t * g_addr[kMaxDevices] = {nullptr};

// device address of the scratch array on the current device (host code only
// sees a host-side stand-in under the array's name). Outside a stream capture
// the address is looked up on every call, so a context that was reset and
// reloaded the module is picked up; during a capture the address cached by
// the last call outside one is used (a capture cannot look it up).
cudaError_t scratch_address(cudaStream_t stream, uint8_t ** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(stream, &cap);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(g_addr_mu);
    if (cap == cudaStreamCaptureStatusNone) {
        void * p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_addr[dev] = static_cast<uint8_t *>(p);
    } else if (g_addr[dev] == nullptr) {
        return cudaErrorStreamCaptureUnsupported;
    }
    *out = g_addr[dev];
    return cudaSuccess;
}

uint64_t up256(uint64_t v) { return (v + 255) / 256 * 256; }

}  // namespace

extern "C" int gx_moe_ffn_noalloc(const gx_layer_desc * d, const void * slot0_record, uint64_t record_bytes,
                                  uint32_t n_slots, const float * x, const int32_t * slots, const float * w, int64_t k,
                                  int64_t T, float * out, void * stream) {
    if (d == nullptr || slot0_record == nullptr || x == nullptr || slots == nullptr || w == nullptr || out == nullptr)
        return GX_ERR_INVALID;
    if (!gx::supported_weight_type(d->type_gate) || !gx::supported_weight_type(d->type_down)) return GX_ERR_TYPE;
    if (d->type_up != d->type_gate) return GX_ERR_TYPE;
    if (d->act != GX_ACT_SWIGLU && d->act != GX_ACT_SWIGLU_OAI) return GX_ERR_INVALID;
    const int64_t H = d->hidden, I = d->intermediate;
    if (k <= 0 || T < 0 || n_slots == 0) return GX_ERR_INVALID;
    if (T == 0) return GX_OK;
    // the array's fixed size bounds the call
    if (k * T > GX_NOALLOC_MAX_PAIRS || H > GX_NOALLOC_MAX_HIDDEN || I > GX_NOALLOC_MAX_INTERMEDIATE)
        return GX_ERR_INVALID;
    if (H % gx::row_align(d->type_gate) != 0 || I % gx::row_align(d->type_down) != 0) return GX_ERR_ALIGN;
    if ((reinterpret_cast<uintptr_t>(slot0_record) & 15u) || record_bytes % 16 || d->off_gate % 16 || d->off_up % 16)
        return GX_ERR_ALIGN;
    if (d->off_up + (uint64_t)gx::row_bytes(d->type_up, H) * I > record_bytes ||
        (uint64_t)gx::row_bytes(d->type_down, I) * H > d->off_gate)
        return GX_ERR_INVALID;
    const int64_t n = k * T;
    for (int64_t j = 0; j < n; ++j)
        if (slots[j] < 0 || (uint32_t)slots[j] >= n_slots) return GX_ERR_DOMAIN;

    uint8_t * base = nullptr;
    if (scratch_address(reinterpret_cast<cudaStream_t>(stream), &base) != cudaSuccess) return GX_ERR_CUDA;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int vdt_g = gx::vec_dot_type(d->type_gate), vdt_d = gx::vec_dot_type(d->type_down);
    const gx::ActLayout al_x = gx::act_layout(vdt_g, (int)H), al_a = gx::act_layout(vdt_d, (int)I);
    const int qblk = vdt_d == gx::GX_T_Q8_0 ? 32 : 256;

    // carve the array: inputs, f32 activation, quantized activation, counters
    uint64_t off = 0;
    uint8_t * xq = base + off;
    off = up256(off + (uint64_t)T * al_x.pitch);
    float * act = reinterpret_cast<float *>(base + off);
    off = up256(off + (uint64_t)n * I * sizeof(float));
    uint8_t * actq = base + off;
    off = up256(off + (uint64_t)n * al_a.pitch);
    int32_t * cnt = reinterpret_cast<int32_t *>(base + off);
    const uint64_t cnt_bytes = (uint64_t)n * (I / qblk) * sizeof(int32_t);
    off = up256(off + cnt_bytes);
    if (off > kNoAllocScratchBytes) return GX_ERR_INVALID;

    const uint8_t * rec = static_cast<const uint8_t *>(slot0_record);
    gx::DecodeParams g{};
    g.w0 = rec + d->off_gate;
    g.w1 = rec + d->off_up;
    g.nb01 = gx::row_bytes(d->type_gate, H);
    g.nb02 = (int64_t)record_bytes;
    g.ne00 = (int32_t)H;
    g.ne01 = (int32_t)I;
    g.n_as = (int32_t)n_slots;
    g.k = (int32_t)k;
    g.T = (int32_t)T;
    g.use_inline = 1;
    for (int64_t j = 0; j < n; ++j) g.inline_ids[j] = slots[j];
    g.aq = xq;
    g.al = al_x;
    g.a_rows = 1;
    g.act_f32 = act;
    g.act_q = actq;
    g.al2 = al_a;
    g.vdt2 = vdt_d;
    g.qblk = qblk;
    g.counters = cnt;
    g.act = d->act;
    g.alpha = d->alpha;
    g.limit = d->limit;
    {
        static const int cands[] = {8, 16, 4, 2, 1};
        int threads = 0;
        for (int R : cands) {
            if (I % R || qblk % R) continue;
            gx::DecodeParams t = g;
            t.R = R;
            if (gx::decode_layout(1, t, threads) == 0) continue;
            g.R = R;
            break;
        }
        if (g.R == 0) return GX_ERR_ALIGN;
        g.n_units = (int32_t)(n * (I / g.R));
    }
    gx::DecodeParams dn = g;
    dn.w0 = rec;
    dn.w1 = nullptr;
    dn.nb01 = gx::row_bytes(d->type_down, I);
    dn.ne00 = (int32_t)I;
    dn.ne01 = (int32_t)H;
    dn.aq = actq;
    dn.al = al_a;
    dn.a_rows = (int32_t)k;
    dn.rw = w;
    dn.out = out;
    {
        const int base_r = (int)(16 / k) > 0 ? (int)(16 / k) : 1;
        const int cands[] = {base_r, 2 * base_r, base_r / 2, base_r / 4, 1};
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

    // counters must start at zero; a call cut short could have left some set
    if (cudaMemsetAsync(cnt, 0, cnt_bytes, s) != cudaSuccess) return GX_ERR_CUDA;
    if (gx::launch_quant_split(vdt_g, x, (int)H, T, H * 4, xq, s, false) != cudaSuccess) return GX_ERR_CUDA;
    if (gx::launch_decode(d->type_gate, 1, g, s, false) != cudaSuccess) return GX_ERR_CUDA;
    if (gx::launch_decode(d->type_down, 2, dn, s, false) != cudaSuccess) return GX_ERR_CUDA;
    return GX_OK;
}
