// Expert parallelism over G ranks (one process per GPU): the routed pairs of
// a rank's tokens are dispatched to the ranks that own their experts, computed
// there on the local slot arena, and combined at home in slot order.
//
// The exchanges use NCCL point-to-point calls grouped into one all-to-all per
// phase (ncclGroupStart/ncclSend/ncclRecv/ncclGroupEnd), on the caller's
// communicator. The entry points are resolved at run time from the NCCL
// library already loaded in the process (the one that created the caller's
// communicator), else from libnccl.so.2 or $GX_NCCL_LIB, so the library does
// not pin an NCCL version of its own.
//
// One step covers n consecutive layers whose routes are known (one layer for
// gx_ep_layer_forward / gx_ep_dispatch):
//   1. shape all-to-all: 8 ints per peer [status, n, k, T, first layer, H,
//      world, experts]; one stream synchronization. Every rank sees every
//      rank's status and shape, so a call that one rank rejects (bad ids,
//      mismatched layers or widths) ends with the same error on all ranks
//      before any payload moves; T may differ between ranks;
//   2. id all-to-all: per peer n counts and the local expert ids of the pairs
//      (sized by the sender's own T); one stream synchronization: the owner's
//      slot policy runs on its host;
//   3. row all-to-all: each pair's input row x_L[t] (H f32), all layers in one
//      exchange, rows grouped by peer then layer;
//   4. owner compute, per layer with no host synchronization: the received
//      rows of the layer as a micro-batch of one expert each with unit router
//      weight (gx_moe_layer_forward, k = 1, expert-major waves when the slot
//      cache cannot hold them at once): fl(1 * y) = y, the pair's down output;
//   5. result all-to-all back, scatter to [n, T, k, H] by pair, and the
//      combine ((w0*y0 + w1*y1) + ...) of the single-GPU path, per layer.
// A failure on an owner after the exchanges began (a miss copy that fails)
// does not stop the exchange: its result rows are NaN, the peers complete
// their calls, and the owner returns the error.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "../../include/galactus_b200.h"
#include "gx_kernels.h"

namespace {

// ---------------------------------------------------------------- NCCL API
// The handful of NCCL entry points used here, by their public signatures.
typedef int (*nccl_group_fn)(void);
typedef int (*nccl_p2p_send_fn)(const void *, size_t, int, int, void *, cudaStream_t);
typedef int (*nccl_p2p_recv_fn)(void *, size_t, int, int, void *, cudaStream_t);
constexpr int kNcclInt32 = 2;     // ncclInt32
constexpr int kNcclFloat32 = 7;   // ncclFloat32

struct NcclApi {
    nccl_group_fn group_start = nullptr, group_end = nullptr;
    nccl_p2p_send_fn send = nullptr;
    nccl_p2p_recv_fn recv = nullptr;
    bool ok = false;
};

NcclApi load_nccl() {
    NcclApi api;
    void * h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (h == nullptr) {
        const char * env = std::getenv("GX_NCCL_LIB");
        h = dlopen(env ? env : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    }
    if (h == nullptr) return api;
    api.group_start = reinterpret_cast<nccl_group_fn>(dlsym(h, "ncclGroupStart"));
    api.group_end = reinterpret_cast<nccl_group_fn>(dlsym(h, "ncclGroupEnd"));
    api.send = reinterpret_cast<nccl_p2p_send_fn>(dlsym(h, "ncclSend"));
    api.recv = reinterpret_cast<nccl_p2p_recv_fn>(dlsym(h, "ncclRecv"));
    api.ok = api.group_start && api.group_end && api.send && api.recv;
    return api;
}

const NcclApi & nccl() {
    static NcclApi api = load_nccl();
    return api;
}

struct CommFail {};
struct CudaFail {
    cudaError_t err;
};
struct Invalid {
    int code;
};

inline void ck(cudaError_t e) {
    if (e != cudaSuccess) throw CudaFail{e};
}
inline void nk(int r) {
    if (r != 0) throw CommFail{};
}

template <typename F>
int guarded(F && f) {
    try {
        return f();
    } catch (const Invalid & e) {
        return e.code;
    } catch (const CommFail &) {
        return GX_ERR_COMM;
    } catch (const CudaFail & e) {
        std::fprintf(stderr, "galactus_b200: CUDA error: %s\n", cudaGetErrorString(e.err));
        return e.err == cudaErrorMemoryAllocation ? GX_ERR_NOMEM : GX_ERR_CUDA;
    } catch (const std::bad_alloc &) {
        return GX_ERR_NOMEM;
    } catch (...) {
        return GX_ERR_INVALID;
    }
}

int owner_of(int32_t placement, uint32_t E, int32_t G, int32_t e, int32_t & rank, int32_t & local) {
    if (G <= 0 || e < 0 || (uint32_t)e >= E) return GX_ERR_DOMAIN;
    if (placement == GX_EP_MODULO) {
        rank = e % G;
        local = e / G;
    } else if (placement == GX_EP_BLOCK) {
        const int32_t block = (int32_t)((E + (uint32_t)G - 1) / (uint32_t)G);
        rank = e / block;
        local = e - rank * block;
    } else {
        return GX_ERR_INVALID;
    }
    return GX_OK;
}

template <typename T>
struct DevBuf {
    T * p = nullptr;
    size_t n = 0;
    void reserve(size_t want) {
        if (want <= n) return;
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
        ck(cudaMalloc(&p, std::max<size_t>(want, 1) * sizeof(T)));
        n = want;
    }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
};

template <typename T>
struct HostBuf {
    T * p = nullptr;
    size_t n = 0;
    void reserve(size_t want) {
        if (want <= n) return;
        if (p) cudaFreeHost(p);
        p = nullptr;
        n = 0;
        ck(cudaHostAlloc(&p, std::max<size_t>(want, 1) * sizeof(T), cudaHostAllocDefault));
        n = want;
    }
    ~HostBuf() {
        if (p) cudaFreeHost(p);
    }
};

constexpr int kShapeInts = 8;   // [status, n, k, T, first, H, world, experts]

}  // namespace

struct gx_ep {
    gx_arena * arena = nullptr;
    void * comm = nullptr;
    int32_t rank = 0, world = 1, placement = GX_EP_MODULO;
    uint32_t E = 0;
    int device = 0;
    std::mutex mu;
    // the step in progress (0 idle, 1 dispatched, 2 computed)
    int state = 0;
    uint32_t first = 0, n = 0;
    int64_t k = 0, T = 0, H = 0;
    int err = GX_OK;                       // a failure on this owner during the step
    std::vector<int32_t> peerT;            // T of each rank
    // home side: the pairs sent to each peer, in send order (peer, layer, pair)
    std::vector<int32_t> scount, soff;     // rows per peer, first row
    std::vector<int32_t> send_L, send_pair;
    // owner side: received rows, peer-major (peer, layer, in the sender's order)
    std::vector<int32_t> rcount, roff;
    std::vector<int32_t> recv_local;       // local expert id of each received row
    std::vector<int32_t> lay_cnt, lay_off; // layer-major layout of the received rows
    int64_t n_recv = 0;
    // headers and index staging
    HostBuf<int32_t> h_shape_s, h_shape_r, h_hdr_s, h_hdr_r, h_idx;
    DevBuf<int32_t> d_shape_s, d_shape_r, d_hdr_s, d_hdr_r, d_idx;
    HostBuf<const float *> h_ptrs;
    DevBuf<const float *> d_ptrs;
    // rows: sent inputs (peer-major), received inputs (peer-major), the same
    // layer-major, owner outputs layer-major and peer-major, results back home
    // (peer-major) and in [n, T, k, H] pair order
    DevBuf<float> d_send, d_recv, d_xl, d_yl, d_yback, d_back, d_full, d_ones;
    cudaEvent_t ev = nullptr;              // the last upload out of the pinned staging has run
    gx_serve_stats st{};
};

namespace {

// One grouped exchange: per peer r, send `scnt[r]` elements from src + soff[r]
// and receive `rcnt[r]` into dst + roff[r] (elements of `width` values each).
// The rank's own share is a device copy.
template <typename V>
void exchange(gx_ep * ep, const V * src, const std::vector<int32_t> & scnt, const std::vector<int32_t> & soff, V * dst,
              const std::vector<int32_t> & rcnt, const std::vector<int32_t> & roff, int64_t width, int dtype,
              cudaStream_t s) {
    const int32_t G = ep->world, me = ep->rank;
    if (scnt[(size_t)me] != rcnt[(size_t)me]) throw Invalid{GX_ERR_STATE};
    if (scnt[(size_t)me] > 0)
        ck(cudaMemcpyAsync(dst + (size_t)roff[(size_t)me] * (size_t)width, src + (size_t)soff[(size_t)me] * (size_t)width,
                           (size_t)scnt[(size_t)me] * (size_t)width * sizeof(V), cudaMemcpyDeviceToDevice, s));
    if (G == 1) return;
    const NcclApi & n = nccl();
    nk(n.group_start());
    for (int32_t r = 0; r < G; ++r) {
        if (r == me) continue;
        if (scnt[(size_t)r] > 0)
            nk(n.send(src + (size_t)soff[(size_t)r] * (size_t)width, (size_t)scnt[(size_t)r] * (size_t)width, dtype, r,
                      ep->comm, s));
        if (rcnt[(size_t)r] > 0)
            nk(n.recv(dst + (size_t)roff[(size_t)r] * (size_t)width, (size_t)rcnt[(size_t)r] * (size_t)width, dtype, r,
                      ep->comm, s));
    }
    nk(n.group_end());
}

// device -> pinned host copy, then wait for it (the host reads the result)
void fetch(gx_ep * ep, int32_t * h, const int32_t * d, size_t count, cudaStream_t s) {
    ck(cudaMemcpyAsync(h, d, count * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    ck(cudaEventRecord(ep->ev, s));
    ck(cudaEventSynchronize(ep->ev));
}

// Steps 1-3 for n layers: shapes, ids, input rows. Every rank runs both
// header exchanges, also when its own call is invalid (status != 0), and all
// ranks return the same status.
int ep_dispatch(gx_ep * ep, uint32_t first, uint32_t n, const float * const * x, const int32_t * ids, int64_t k,
                int64_t T, int64_t H, cudaStream_t s) {
    const int32_t G = ep->world, me = ep->rank;
    ep->state = 0;
    ep->err = GX_OK;
    ep->st = gx_serve_stats{};
    // local validation: the plan of every pair
    int status = GX_OK;
    if (n == 0 || k <= 0 || T < 0 || H <= 0 || x == nullptr || (T > 0 && ids == nullptr)) status = GX_ERR_INVALID;
    const int64_t P = k * T;
    std::vector<int32_t> dest, local;
    if (status == GX_OK) {
        dest.resize((size_t)(n * P));
        local.resize((size_t)(n * P));
        for (int64_t i = 0; i < (int64_t)n * P && status == GX_OK; ++i)
            status = owner_of(ep->placement, ep->E, G, ids[i], dest[(size_t)i], local[(size_t)i]);
    }
    // 1. shapes
    ep->h_shape_s.reserve((size_t)kShapeInts);
    ep->h_shape_r.reserve((size_t)(G * kShapeInts));
    ep->d_shape_s.reserve((size_t)(G * kShapeInts));
    ep->d_shape_r.reserve((size_t)(G * kShapeInts));
    const int32_t shape[kShapeInts] = {status, (int32_t)n, (int32_t)k, (int32_t)T, (int32_t)first, (int32_t)H, G,
                                       (int32_t)ep->E};
    ck(cudaEventSynchronize(ep->ev));   // the pinned staging is free
    std::memcpy(ep->h_shape_s.p, shape, sizeof(shape));
    ck(cudaMemcpyAsync(ep->d_shape_s.p, ep->h_shape_s.p, sizeof(shape), cudaMemcpyHostToDevice, s));
    {
        std::vector<int32_t> one((size_t)G, 1), zero((size_t)G, 0), offs((size_t)G, 0);
        for (int32_t r = 0; r < G; ++r) offs[(size_t)r] = r;
        // every peer gets the same 8 ints: send from offset 0, receive into slot r
        exchange<int32_t>(ep, ep->d_shape_s.p, one, zero, ep->d_shape_r.p, one, offs, kShapeInts, kNcclInt32, s);
    }
    fetch(ep, ep->h_shape_r.p, ep->d_shape_r.p, (size_t)(G * kShapeInts), s);
    ep->peerT.assign((size_t)G, 0);
    int agreed = GX_OK;
    for (int32_t r = 0; r < G; ++r) {
        const int32_t * h = ep->h_shape_r.p + (size_t)r * kShapeInts;
        if (h[0] != GX_OK && agreed == GX_OK) agreed = h[0];
        if (h[1] != (int32_t)n || h[2] != (int32_t)k || h[4] != (int32_t)first || h[5] != (int32_t)H || h[6] != G ||
            h[7] != (int32_t)ep->E || h[3] < 0)
            if (agreed == GX_OK) agreed = GX_ERR_INVALID;
        ep->peerT[(size_t)r] = h[3];
    }
    if (agreed != GX_OK) return agreed;

    // 2. ids: per peer [n counts][local ids, layer by layer]
    ep->first = first;
    ep->n = n;
    ep->k = k;
    ep->T = T;
    ep->H = H;
    ep->scount.assign((size_t)G, 0);
    std::vector<int32_t> cnt((size_t)G * n, 0);   // [peer][layer]
    for (uint32_t L = 0; L < n; ++L)
        for (int64_t i = 0; i < P; ++i) ++cnt[(size_t)dest[(size_t)(L * P + i)] * n + L];
    for (int32_t r = 0; r < G; ++r)
        for (uint32_t L = 0; L < n; ++L) ep->scount[(size_t)r] += cnt[(size_t)r * n + L];
    ep->soff.assign((size_t)G, 0);
    for (int32_t r = 1; r < G; ++r) ep->soff[(size_t)r] = ep->soff[(size_t)r - 1] + ep->scount[(size_t)r - 1];
    // send order: peer, layer, pair
    ep->send_L.assign((size_t)(n * P), 0);
    ep->send_pair.assign((size_t)(n * P), 0);
    const int64_t hs = (int64_t)n * (1 + P);         // ints this rank sends to each peer
    std::vector<int64_t> hoff((size_t)G + 1, 0);     // ints received from each peer
    for (int32_t r = 0; r < G; ++r) hoff[(size_t)r + 1] = hoff[(size_t)r] + (int64_t)n * (1 + k * ep->peerT[(size_t)r]);
    ep->h_hdr_s.reserve((size_t)(G * hs));
    ep->h_hdr_r.reserve((size_t)hoff[(size_t)G]);
    ep->d_hdr_s.reserve((size_t)(G * hs));
    ep->d_hdr_r.reserve((size_t)hoff[(size_t)G]);
    {
        std::vector<int32_t> fill(ep->soff);
        for (int32_t r = 0; r < G; ++r) {
            int32_t * h = ep->h_hdr_s.p + (size_t)r * hs;
            int32_t * idp = h + n;
            for (uint32_t L = 0; L < n; ++L) h[L] = cnt[(size_t)r * n + L];
            for (uint32_t L = 0; L < n; ++L)
                for (int64_t i = 0; i < P; ++i) {
                    const size_t j = (size_t)(L * P + i);
                    if (dest[j] != r) continue;
                    *idp++ = local[j];
                    ep->send_L[(size_t)fill[(size_t)r]] = (int32_t)L;
                    ep->send_pair[(size_t)fill[(size_t)r]++] = (int32_t)i;
                }
        }
    }
    ck(cudaMemcpyAsync(ep->d_hdr_s.p, ep->h_hdr_s.p, (size_t)(G * hs) * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    {
        std::vector<int32_t> sc((size_t)G, (int32_t)hs), so((size_t)G), rc((size_t)G), ro((size_t)G);
        for (int32_t r = 0; r < G; ++r) {
            so[(size_t)r] = (int32_t)(r * hs);
            rc[(size_t)r] = (int32_t)(hoff[(size_t)r + 1] - hoff[(size_t)r]);
            ro[(size_t)r] = (int32_t)hoff[(size_t)r];
        }
        exchange<int32_t>(ep, ep->d_hdr_s.p, sc, so, ep->d_hdr_r.p, rc, ro, 1, kNcclInt32, s);
    }
    fetch(ep, ep->h_hdr_r.p, ep->d_hdr_r.p, (size_t)hoff[(size_t)G], s);
    // received rows: peer-major, layer, sender's order
    ep->rcount.assign((size_t)G, 0);
    ep->roff.assign((size_t)G, 0);
    ep->recv_local.clear();
    ep->lay_cnt.assign(n, 0);
    std::vector<int32_t> rl;   // layer of each received row
    for (int32_t r = 0; r < G; ++r) {
        const int32_t * h = ep->h_hdr_r.p + hoff[(size_t)r];
        const int32_t * idp = h + n;
        ep->roff[(size_t)r] = (int32_t)ep->recv_local.size();
        for (uint32_t L = 0; L < n; ++L) {
            if (h[L] < 0 || h[L] > k * ep->peerT[(size_t)r]) throw Invalid{GX_ERR_STATE};
            for (int32_t i = 0; i < h[L]; ++i) {
                ep->recv_local.push_back(*idp++);
                rl.push_back((int32_t)L);
            }
            ep->lay_cnt[L] += h[L];
            ep->rcount[(size_t)r] += h[L];
        }
    }
    ep->n_recv = (int64_t)ep->recv_local.size();
    ep->lay_off.assign(n, 0);
    for (uint32_t L = 1; L < n; ++L) ep->lay_off[L] = ep->lay_off[L - 1] + ep->lay_cnt[L - 1];

    // 3. input rows: gather x_L[t] of every sent pair, exchange
    const int64_t S = n * P, R = ep->n_recv;
    ep->h_idx.reserve((size_t)(3 * S + R));
    ep->d_idx.reserve((size_t)(3 * S + R));
    ep->h_ptrs.reserve(n);
    ep->d_ptrs.reserve(n);
    int32_t * hL = ep->h_idx.p;             // [S] layer of each sent row
    int32_t * hR = hL + S;                  // [S] token of each sent row
    int32_t * hlm = hR + S;                 // [R] layer-major position of each received row
    int32_t * hfull = hlm + R;              // [S] pair position in [n, T, k] of each sent row (results)
    for (int64_t j = 0; j < S; ++j) {
        hL[j] = ep->send_L[(size_t)j];
        hR[j] = ep->send_pair[(size_t)j] / (int32_t)k;
    }
    {
        std::vector<int32_t> lf(ep->lay_off);
        for (int64_t j = 0; j < R; ++j) hlm[j] = lf[(size_t)rl[(size_t)j]]++;
    }
    for (int64_t j = 0; j < S; ++j) hfull[j] = (int32_t)(ep->send_L[(size_t)j] * P + ep->send_pair[(size_t)j]);
    for (uint32_t L = 0; L < n; ++L) ep->h_ptrs.p[L] = x[L];
    ck(cudaMemcpyAsync(ep->d_idx.p, ep->h_idx.p, (size_t)(3 * S + R) * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    ck(cudaMemcpyAsync(ep->d_ptrs.p, ep->h_ptrs.p, (size_t)n * sizeof(const float *), cudaMemcpyHostToDevice, s));
    ck(cudaEventRecord(ep->ev, s));   // the staging is rewritten by the next step only after these uploads
    ep->d_send.reserve((size_t)std::max<int64_t>(S, 1) * (size_t)H);
    ep->d_recv.reserve((size_t)std::max<int64_t>(R, 1) * (size_t)H);
    ck(gx::launch_gather_ptrs(ep->d_ptrs.p, ep->d_idx.p, ep->d_idx.p + S, S, H, ep->d_send.p, s));
    exchange<float>(ep, ep->d_send.p, ep->scount, ep->soff, ep->d_recv.p, ep->rcount, ep->roff, H, kNcclFloat32, s);
    ep->state = 1;
    (void)me;
    return GX_OK;
}

// Step 4: the received rows of every layer on the local arena. A failure is
// recorded (ep->err) and leaves that layer's result rows NaN.
void ep_compute(gx_ep * ep, const gx_layer_desc * desc, cudaStream_t s) {
    const int64_t R = ep->n_recv, H = ep->H, S = (int64_t)ep->n * ep->k * ep->T;
    ep->d_xl.reserve((size_t)std::max<int64_t>(R, 1) * (size_t)H);
    ep->d_yl.reserve((size_t)std::max<int64_t>(R, 1) * (size_t)H);
    ep->d_yback.reserve((size_t)std::max<int64_t>(R, 1) * (size_t)H);
    const int32_t * dlm = ep->d_idx.p + 2 * S;   // layer-major position of each received row
    if (R > 0) {
        ck(gx::launch_move_rows(ep->d_recv.p, dlm, R, H, ep->d_xl.p, true, s));
        int64_t mx = 0;
        for (uint32_t L = 0; L < ep->n; ++L) mx = std::max<int64_t>(mx, ep->lay_cnt[L]);
        if ((int64_t)ep->d_ones.n < mx) {
            ep->d_ones.reserve((size_t)mx);
            ck(gx::launch_fill(ep->d_ones.p, mx, 1.0f, s));
        }
        // local ids in layer-major order (rows arrive peer-major, layers in
        // order inside each peer; hlm is the layer-major position of each)
        std::vector<int32_t> lids((size_t)R);
        const int32_t * hlm = ep->h_idx.p + 2 * S;
        for (int64_t j = 0; j < R; ++j) lids[(size_t)hlm[j]] = ep->recv_local[(size_t)j];
        for (uint32_t L = 0; L < ep->n; ++L) {
            const int64_t c = ep->lay_cnt[L];
            if (c == 0) continue;
            gx_serve_stats st{};
            const int64_t o = ep->lay_off[L];
            const int rc = gx_moe_layer_forward(ep->arena, ep->first + L, desc, ep->d_xl.p + o * H, lids.data() + o,
                                                ep->d_ones.p, 1, c, ep->d_yl.p + o * H, s, &st);
            if (rc != GX_OK) {
                if (ep->err == GX_OK) ep->err = rc;
                ck(cudaMemsetAsync(ep->d_yl.p + o * H, 0xff, (size_t)(c * H) * sizeof(float), s));
                continue;
            }
            ep->st.hits += st.hits;
            ep->st.misses += st.misses;
            ep->st.evictions += st.evictions;
            ep->st.distinct += st.distinct;
            ep->st.bytes_copied += st.bytes_copied;
        }
        // back to peer-major order for the results exchange
        ck(gx::launch_move_rows(ep->d_yl.p, dlm, R, H, ep->d_yback.p, false, s));
    }
    ep->state = 2;
}

// Step 5: results home, scattered to pair order, combined per layer.
void ep_combine(gx_ep * ep, const float * const * w, float * const * out, cudaStream_t s) {
    const int64_t P = ep->k * ep->T, S = (int64_t)ep->n * P, H = ep->H;
    ep->d_back.reserve((size_t)std::max<int64_t>(S, 1) * (size_t)H);
    ep->d_full.reserve((size_t)std::max<int64_t>(S, 1) * (size_t)H);
    exchange<float>(ep, ep->d_yback.p, ep->rcount, ep->roff, ep->d_back.p, ep->scount, ep->soff, H, kNcclFloat32, s);
    const int32_t * dfull = ep->d_idx.p + 2 * S + ep->n_recv;   // pair positions, after the layer-major positions
    if (S > 0) ck(gx::launch_move_rows(ep->d_back.p, dfull, S, H, ep->d_full.p, true, s));
    for (uint32_t L = 0; L < ep->n; ++L)
        if (ep->T > 0) ck(gx::launch_combine(ep->d_full.p + (size_t)L * P * H, w[L], out[L], H, (int)ep->k, ep->T, s));
    ep->state = 0;
}

}  // namespace

extern "C" {

int gx_ep_owner(int32_t placement, uint32_t n_expert, int32_t world, int32_t expert, int32_t * rank, int32_t * local_id) {
    if (rank == nullptr || local_id == nullptr) return GX_ERR_INVALID;
    return owner_of(placement, n_expert, world, expert, *rank, *local_id);
}

int gx_ep_plan(int32_t placement, uint32_t n_expert, int32_t world, const int32_t * ids, int64_t k, int64_t T,
               int32_t * send_counts, int32_t * send_pairs) {
    if (ids == nullptr || send_counts == nullptr || send_pairs == nullptr || world <= 0 || k <= 0 || T < 0)
        return GX_ERR_INVALID;
    std::vector<int32_t> dest((size_t)(k * T));
    for (int32_t r = 0; r < world; ++r) send_counts[r] = 0;
    for (int64_t i = 0; i < k * T; ++i) {
        int32_t r = 0, l = 0;
        const int rc = owner_of(placement, n_expert, world, ids[i], r, l);
        if (rc != GX_OK) return rc;
        dest[(size_t)i] = r;
        ++send_counts[r];
    }
    // pairs grouped by destination, (token, slot) order inside a group
    std::vector<int32_t> off((size_t)world, 0);
    for (int32_t r = 1; r < world; ++r) off[(size_t)r] = off[(size_t)r - 1] + send_counts[r - 1];
    for (int64_t i = 0; i < k * T; ++i) send_pairs[off[(size_t)dest[(size_t)i]]++] = (int32_t)i;
    return GX_OK;
}

int gx_ep_init(gx_arena * local_arena, void * nccl_comm, int32_t rank, int32_t world, uint32_t n_expert,
               int32_t placement, gx_ep ** out) {
    if (local_arena == nullptr || out == nullptr || world <= 0 || rank < 0 || rank >= world || n_expert == 0 ||
        (placement != GX_EP_MODULO && placement != GX_EP_BLOCK))
        return GX_ERR_INVALID;
    if (world > 1 && nccl_comm == nullptr) return GX_ERR_INVALID;
    if (world > 1 && !nccl().ok) return GX_ERR_COMM;
    *out = nullptr;
    gx_ep * ep = new (std::nothrow) gx_ep();
    if (ep == nullptr) return GX_ERR_NOMEM;
    const int rc = guarded([&] {
        ep->arena = local_arena;
        ep->comm = nccl_comm;
        ep->rank = rank;
        ep->world = world;
        ep->E = n_expert;
        ep->placement = placement;
        ck(cudaGetDevice(&ep->device));
        ck(cudaEventCreateWithFlags(&ep->ev, cudaEventDisableTiming));
        return GX_OK;
    });
    if (rc != GX_OK) {
        gx_ep_destroy(ep);
        return rc;
    }
    *out = ep;
    return GX_OK;
}

int gx_ep_destroy(gx_ep * ep) {
    if (ep == nullptr) return GX_OK;
    cudaSetDevice(ep->device);
    cudaDeviceSynchronize();
    if (ep->ev) cudaEventDestroy(ep->ev);
    delete ep;
    return GX_OK;
}

int gx_ep_dispatch(gx_ep * ep, uint32_t layer, const float * x, const int32_t * ids, int64_t k, int64_t T, int64_t H,
                   void * stream) {
    if (ep == nullptr) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(ep->mu);
        ck(cudaSetDevice(ep->device));
        const float * xs[1] = {x};
        return ep_dispatch(ep, layer, 1, xs, ids, k, T, H, reinterpret_cast<cudaStream_t>(stream));
    });
}

int gx_ep_compute(gx_ep * ep, const gx_layer_desc * desc, void * stream, gx_serve_stats * stats) {
    if (ep == nullptr || desc == nullptr) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(ep->mu);
        if (ep->state != 1) throw Invalid{GX_ERR_STATE};
        if (desc->hidden != ep->H) throw Invalid{GX_ERR_INVALID};
        ck(cudaSetDevice(ep->device));
        ep_compute(ep, desc, reinterpret_cast<cudaStream_t>(stream));
        if (stats) *stats = ep->st;
        return GX_OK;
    });
}

int gx_ep_combine(gx_ep * ep, const float * w, float * out, void * stream) {
    if (ep == nullptr || w == nullptr || out == nullptr) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(ep->mu);
        if (ep->state != 2) throw Invalid{GX_ERR_STATE};
        ck(cudaSetDevice(ep->device));
        const float * ws[1] = {w};
        float * os[1] = {out};
        ep_combine(ep, ws, os, reinterpret_cast<cudaStream_t>(stream));
        const int e = ep->err;
        ep->err = GX_OK;
        return e;
    });
}

int gx_ep_stack_forward(gx_ep * ep, uint32_t first_layer, uint32_t n_layers, const gx_layer_desc * desc,
                        const float * const * x, const int32_t * ids, const float * const * w, int64_t k, int64_t T,
                        float * const * out, void * stream, gx_serve_stats * stats) {
    if (ep == nullptr || desc == nullptr || w == nullptr || out == nullptr) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(ep->mu);
        ck(cudaSetDevice(ep->device));
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        const int rc = ep_dispatch(ep, first_layer, n_layers, x, ids, k, T, desc->hidden, s);
        if (rc != GX_OK) return rc;
        ep_compute(ep, desc, s);
        ep_combine(ep, w, out, s);
        if (stats) *stats = ep->st;
        const int e = ep->err;
        ep->err = GX_OK;
        return e;
    });
}

int gx_ep_layer_forward(gx_ep * ep, uint32_t layer, const gx_layer_desc * desc, const float * x, const int32_t * ids,
                        const float * w, int64_t k, int64_t T, float * out, void * stream, gx_serve_stats * stats) {
    const float * xs[1] = {x};
    const float * ws[1] = {w};
    float * os[1] = {out};
    return gx_ep_stack_forward(ep, layer, 1, desc, xs, ids, ws, k, T, os, stream, stats);
}

}  // extern "C"
