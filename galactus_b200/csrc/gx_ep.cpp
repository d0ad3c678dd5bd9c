// Expert parallelism over G ranks (one process per GPU): the routed pairs of
// a rank's tokens are dispatched to the ranks that own their experts, computed
// there on the local slot arena, and combined at home in slot order.
//
// The exchange uses NCCL point-to-point calls grouped into one all-to-all per
// phase (ncclGroupStart/ncclSend/ncclRecv/ncclGroupEnd), on the caller's
// communicator. The entry points are resolved at run time from the NCCL
// library already loaded in the process (the one that created the caller's
// communicator), else from libnccl.so.2 or $GX_NCCL_LIB, so the library does
// not pin an NCCL version of its own.
//
// Per layer step:
//   1. plan (host): pairs (t, s) grouped by the owner of ids[t, s];
//   2. header all-to-all: per peer [count, expert ids...] (fixed size
//      1 + max_pairs ints), then one stream synchronization: the host needs
//      the received expert ids for the slot policy;
//   3. row all-to-all: each pair's input row x[t] (H f32);
//   4. local compute: the received pairs as a micro-batch of one slot each
//      with unit router weight (gx_moe_layer_forward, k = 1), which leaves
//      exactly the down projection of each pair: fl(1 * y) = y;
//   5. row all-to-all back, scatter into [T, k, H] by pair, and the combine
//      ((w0*y0 + w1*y1) + ...) of the single-GPU path.
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
        ck(cudaMalloc(&p, want * sizeof(T)));
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
        ck(cudaHostAlloc(&p, want * sizeof(T), cudaHostAllocDefault));
        n = want;
    }
    ~HostBuf() {
        if (p) cudaFreeHost(p);
    }
};

}  // namespace

struct gx_ep {
    gx_arena * arena = nullptr;
    void * comm = nullptr;
    int32_t rank = 0, world = 1, placement = GX_EP_MODULO;
    uint32_t E = 0;
    int device = 0;
    std::mutex mu;
    // the last dispatch
    bool dispatched = false, computed = false;
    uint32_t layer = 0;
    int64_t k = 0, T = 0, H = 0, hdr = 0;   // hdr: ints per peer header
    std::vector<int32_t> send_counts, recv_counts, send_off, recv_off;
    std::vector<int32_t> send_pairs;        // pair index t*k+s, grouped by destination
    std::vector<int32_t> recv_local;        // local expert id of each received pair
    int64_t n_recv = 0;
    HostBuf<int32_t> h_hdr_send, h_hdr_recv, h_idx;
    DevBuf<int32_t> d_hdr_send, d_hdr_recv, d_idx;
    DevBuf<float> d_send, d_recv, d_recv_y, d_back, d_full, d_ones;
    cudaEvent_t ev_hdr = nullptr;
};

namespace {

// rows of the sent pairs: gather x[t] for each pair in send order, then one
// grouped all-to-all of H-float rows
void exchange_rows(gx_ep * ep, const float * src_rows, const std::vector<int32_t> & sc, const std::vector<int32_t> & so,
                   float * dst_rows, const std::vector<int32_t> & rcnt, const std::vector<int32_t> & ro, int64_t H,
                   cudaStream_t s) {
    const int32_t G = ep->world;
    if (G == 1) {
        if (sc[0] > 0)
            ck(cudaMemcpyAsync(dst_rows, src_rows, (size_t)sc[0] * (size_t)H * sizeof(float), cudaMemcpyDeviceToDevice, s));
        return;
    }
    const NcclApi & n = nccl();
    nk(n.group_start());
    for (int32_t r = 0; r < G; ++r) {
        if (sc[(size_t)r] > 0)
            nk(n.send(src_rows + (size_t)so[(size_t)r] * (size_t)H, (size_t)sc[(size_t)r] * (size_t)H, kNcclFloat32, r, ep->comm, s));
        if (rcnt[(size_t)r] > 0)
            nk(n.recv(dst_rows + (size_t)ro[(size_t)r] * (size_t)H, (size_t)rcnt[(size_t)r] * (size_t)H, kNcclFloat32, r, ep->comm, s));
    }
    nk(n.group_end());
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
        ck(cudaEventCreateWithFlags(&ep->ev_hdr, cudaEventDisableTiming));
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
    if (ep->ev_hdr) cudaEventDestroy(ep->ev_hdr);
    delete ep;
    return GX_OK;
}

int gx_ep_dispatch(gx_ep * ep, uint32_t layer, const float * x, const int32_t * ids, int64_t k, int64_t T, int64_t H,
                   void * stream) {
    if (ep == nullptr || x == nullptr || ids == nullptr || k <= 0 || T <= 0 || H <= 0) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(ep->mu);
        ck(cudaSetDevice(ep->device));
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        const int32_t G = ep->world;
        const int64_t P = k * T;
        ep->dispatched = ep->computed = false;
        ep->layer = layer;
        ep->k = k;
        ep->T = T;
        ep->send_counts.assign((size_t)G, 0);
        ep->send_pairs.assign((size_t)P, 0);
        int rc = gx_ep_plan(ep->placement, ep->E, G, ids, k, T, ep->send_counts.data(), ep->send_pairs.data());
        if (rc != GX_OK) throw Invalid{rc};
        ep->send_off.assign((size_t)G, 0);
        for (int32_t r = 1; r < G; ++r) ep->send_off[(size_t)r] = ep->send_off[(size_t)r - 1] + ep->send_counts[(size_t)r - 1];

        // 2. headers: [count, global expert ids of the pairs] per peer
        ep->hdr = 1 + P;
        ep->h_hdr_send.reserve((size_t)(G * ep->hdr));
        ep->h_hdr_recv.reserve((size_t)(G * ep->hdr));
        ep->d_hdr_send.reserve((size_t)(G * ep->hdr));
        ep->d_hdr_recv.reserve((size_t)(G * ep->hdr));
        for (int32_t r = 0; r < G; ++r) {
            int32_t * h = ep->h_hdr_send.p + (size_t)r * ep->hdr;
            h[0] = ep->send_counts[(size_t)r];
            for (int32_t i = 0; i < ep->send_counts[(size_t)r]; ++i) h[1 + i] = ids[ep->send_pairs[(size_t)(ep->send_off[(size_t)r] + i)]];
        }
        ck(cudaMemcpyAsync(ep->d_hdr_send.p, ep->h_hdr_send.p, (size_t)(G * ep->hdr) * sizeof(int32_t),
                           cudaMemcpyHostToDevice, s));
        if (G > 1) {
            const NcclApi & n = nccl();
            nk(n.group_start());
            for (int32_t r = 0; r < G; ++r) {
                nk(n.send(ep->d_hdr_send.p + (size_t)r * ep->hdr, (size_t)ep->hdr, kNcclInt32, r, ep->comm, s));
                nk(n.recv(ep->d_hdr_recv.p + (size_t)r * ep->hdr, (size_t)ep->hdr, kNcclInt32, r, ep->comm, s));
            }
            nk(n.group_end());
        } else {
            ck(cudaMemcpyAsync(ep->d_hdr_recv.p, ep->d_hdr_send.p, (size_t)ep->hdr * sizeof(int32_t),
                               cudaMemcpyDeviceToDevice, s));
        }
        ck(cudaMemcpyAsync(ep->h_hdr_recv.p, ep->d_hdr_recv.p, (size_t)(G * ep->hdr) * sizeof(int32_t),
                           cudaMemcpyDeviceToHost, s));
        ck(cudaEventRecord(ep->ev_hdr, s));
        ck(cudaEventSynchronize(ep->ev_hdr));
        ep->recv_counts.assign((size_t)G, 0);
        ep->recv_off.assign((size_t)G, 0);
        ep->recv_local.clear();
        for (int32_t r = 0; r < G; ++r) {
            const int32_t * h = ep->h_hdr_recv.p + (size_t)r * ep->hdr;
            if (h[0] < 0 || h[0] > P) throw Invalid{GX_ERR_INVALID};
            ep->recv_counts[(size_t)r] = h[0];
            ep->recv_off[(size_t)r] = (int32_t)ep->recv_local.size();
            for (int32_t i = 0; i < h[0]; ++i) {
                int32_t owner = 0, local = 0;
                rc = owner_of(ep->placement, ep->E, G, h[1 + i], owner, local);
                if (rc != GX_OK || owner != ep->rank) throw Invalid{rc != GX_OK ? rc : GX_ERR_DOMAIN};
                ep->recv_local.push_back(local);
            }
        }
        ep->n_recv = (int64_t)ep->recv_local.size();

        // 3. the input row of every sent pair, then one grouped all-to-all
        ep->H = H;
        ep->h_idx.reserve((size_t)P);
        ep->d_idx.reserve((size_t)P);
        for (int64_t i = 0; i < P; ++i) ep->h_idx.p[i] = ep->send_pairs[(size_t)i] / (int32_t)k;
        ck(cudaMemcpyAsync(ep->d_idx.p, ep->h_idx.p, (size_t)P * sizeof(int32_t), cudaMemcpyHostToDevice, s));
        ep->d_send.reserve((size_t)(P * H));
        ck(gx::launch_move_rows(x, ep->d_idx.p, P, H, ep->d_send.p, false, s));
        ep->d_recv.reserve((size_t)std::max<int64_t>(ep->n_recv, 1) * (size_t)H);
        exchange_rows(ep, ep->d_send.p, ep->send_counts, ep->send_off, ep->d_recv.p, ep->recv_counts, ep->recv_off, H, s);
        // the pinned index buffer is rewritten by combine only after this copy ran
        ck(cudaEventRecord(ep->ev_hdr, s));
        ep->dispatched = true;
        return GX_OK;
    });
}

}  // extern "C"


extern "C" {

int gx_ep_compute(gx_ep * ep, const gx_layer_desc * desc, void * stream, gx_serve_stats * stats) {
    if (ep == nullptr || desc == nullptr) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(ep->mu);
        if (!ep->dispatched) throw Invalid{GX_ERR_STATE};
        if (desc->hidden != ep->H) throw Invalid{GX_ERR_INVALID};
        ck(cudaSetDevice(ep->device));
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        const int64_t R = ep->n_recv, H = ep->H;
        // 4. the received pairs as a micro-batch of one slot each, unit weight
        ep->d_recv_y.reserve((size_t)std::max<int64_t>(R, 1) * (size_t)H);
        gx_serve_stats st{};
        if (R > 0) {
            ep->d_ones.reserve((size_t)R);
            ck(gx::launch_fill(ep->d_ones.p, R, 1.0f, s));
            const int rc = gx_moe_layer_forward(ep->arena, ep->layer, desc, ep->d_recv.p, ep->recv_local.data(),
                                                ep->d_ones.p, 1, R, ep->d_recv_y.p, stream, &st);
            if (rc != GX_OK) throw Invalid{rc};
        }
        if (stats) *stats = st;
        ep->dispatched = false;
        ep->computed = true;
        return GX_OK;
    });
}

int gx_ep_combine(gx_ep * ep, const float * w, float * out, void * stream) {
    if (ep == nullptr || w == nullptr || out == nullptr) return GX_ERR_INVALID;
    return guarded([&] {
        std::lock_guard<std::mutex> lock(ep->mu);
        if (!ep->computed) throw Invalid{GX_ERR_STATE};
        ck(cudaSetDevice(ep->device));
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        const int64_t P = ep->k * ep->T, H = ep->H;
        // 5. outputs back to their home ranks, in the order the pairs were sent
        ep->d_back.reserve((size_t)P * (size_t)H);
        exchange_rows(ep, ep->d_recv_y.p, ep->recv_counts, ep->recv_off, ep->d_back.p, ep->send_counts, ep->send_off, H, s);
        // scatter to [T, k, H] by pair index, then the slot-order combine
        ep->d_full.reserve((size_t)P * (size_t)H);
        ck(cudaEventSynchronize(ep->ev_hdr));   // the dispatch's index copy has run
        for (int64_t i = 0; i < P; ++i) ep->h_idx.p[i] = ep->send_pairs[(size_t)i];
        ck(cudaMemcpyAsync(ep->d_idx.p, ep->h_idx.p, (size_t)P * sizeof(int32_t), cudaMemcpyHostToDevice, s));
        ck(gx::launch_move_rows(ep->d_back.p, ep->d_idx.p, P, H, ep->d_full.p, true, s));
        ck(gx::launch_combine(ep->d_full.p, w, out, H, (int)ep->k, ep->T, s));
        // the pinned index buffer is rewritten by the next call only after this copy ran
        ck(cudaEventRecord(ep->ev_hdr, s));
        ck(cudaEventSynchronize(ep->ev_hdr));
        ep->computed = false;
        return GX_OK;
    });
}

int gx_ep_layer_forward(gx_ep * ep, uint32_t layer, const gx_layer_desc * desc, const float * x, const int32_t * ids,
                        const float * w, int64_t k, int64_t T, float * out, void * stream, gx_serve_stats * stats) {
    if (desc == nullptr) return GX_ERR_INVALID;
    int rc = gx_ep_dispatch(ep, layer, x, ids, k, T, desc->hidden, stream);
    if (rc != GX_OK) return rc;
    rc = gx_ep_compute(ep, desc, stream, stats);
    if (rc != GX_OK) return rc;
    return gx_ep_combine(ep, w, out, stream);
}

}  // extern "C"
