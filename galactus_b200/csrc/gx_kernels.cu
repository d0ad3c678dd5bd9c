// CUDA kernels of the routed-expert FFN (sm_100a).
//
// The expert contraction runs on row tiles: one CTA stages R consecutive rows
// of an expert matrix (a contiguous byte range of the slot arena) into shared
// memory with one bulk TMA copy (cp.async.bulk, completion on an mbarrier),
// quantizes its activation row(s) to Q8_0/Q8_K while the copy is in flight,
// then computes every output of the tile in two phases: exact integer partial
// sums per 64-element unit (all threads, any order), then the float tail of
// the reference's CPU loop, serially per row and chain, in unit order.
//
// Three modes share that core:
//   PLAIN         ggml_mul_mat_id: one (token, slot) pair, R rows -> dst
//   GATE_UP       gate and up tiles of one (token, slot), then SwiGLU / SWIGLU_OAI
//   DOWN_COMBINE  the k down tiles of one token, then the weighted sum in slot order
#include <cstdint>
#include <cstdio>
#include <map>
#include <mutex>
#include <cuda_runtime.h>

#include "gx_device.cuh"
#include "gx_kernels.h"
#include "gx_moe.cuh"
#include "gx_stack.cuh"
#include "gx_prefill.cuh"
#include "gx_router.cuh"
#include "gx_mma.cuh"

namespace gx {


// ------------------------------------------------------------ row kernel

enum { MODE_PLAIN = 0, MODE_GATE_UP = 1, MODE_DOWN_COMBINE = 2 };

__device__ __forceinline__ int32_t get_id(const RowsParams & p, int t, int s) {
    if (p.use_inline) return p.inline_ids[t * p.k + s];
    return *reinterpret_cast<const int32_t *>(reinterpret_cast<const char *>(p.ids) + (int64_t)t * p.nbi1 + 4 * s);
}

template <int TYPE, int MODE>
__global__ void __launch_bounds__(kRowsThreads) k_rows(const RowsParams p) {
    using D = Dot<TYPE>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t * bar = reinterpret_cast<uint64_t *>(smem + p.bar_off);
    uint8_t * tile = smem + p.tile_off;
    uint8_t * act = smem + p.act_off;
    uint32_t * terms = reinterpret_cast<uint32_t *>(smem + p.terms_off);
    float * dots = reinterpret_cast<float *>(smem + p.dots_off);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps = kRowsThreads / 32;
    const int R = p.R;
    const int r0 = blockIdx.x * R;
    const int n_exp = MODE == MODE_DOWN_COMBINE ? p.k : 1;
    const int NR = MODE == MODE_GATE_UP ? 2 * R : n_exp * R;
    const int U = p.ne00 / 64;
    const uint32_t tile_bytes = (uint32_t)(R * p.nb01);

    int t, s0;
    if (MODE == MODE_DOWN_COMBINE) { t = blockIdx.y; s0 = 0; }
    else { t = blockIdx.y / p.k; s0 = blockIdx.y % p.k; }

    // expert ids of this CTA, checked before any load
    bool bad = false;
    for (int i = 0; i < n_exp; ++i) {
        const int32_t e = get_id(p, t, s0 + i);
        if (e < 0 || e >= p.n_as) bad = true;
    }
    if (bad) {
        if (tid == 0) record_error(GX_DEVERR_DOMAIN);
        for (int r = tid; r < R; r += blockDim.x) {
            const float nanv = __int_as_float(0x7fc00000);
            if (MODE == MODE_DOWN_COMBINE) p.dst[(int64_t)t * p.ne01 + r0 + r] = nanv;
            else p.dst[((int64_t)t * p.k + s0) * p.ne01 + r0 + r] = nanv;
        }
        return;
    }

    if (tid == 0) {
        mbar_init(bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0) {
        const uint32_t total = tile_bytes * (uint32_t)(MODE == MODE_GATE_UP ? 2 : n_exp);
        mbar_arrive_expect_tx(bar, total);
        if (MODE == MODE_GATE_UP) {
            const int32_t e = get_id(p, t, s0);
            bulk_g2s(tile, p.w0 + (int64_t)e * p.nb02 + (int64_t)r0 * p.nb01, tile_bytes, bar);
            bulk_g2s(tile + tile_bytes, p.w1 + (int64_t)e * p.nb02 + (int64_t)r0 * p.nb01, tile_bytes, bar);
        } else {
            for (int i = 0; i < n_exp; ++i) {
                const int32_t e = get_id(p, t, s0 + i);
                bulk_g2s(tile + (uint32_t)i * tile_bytes, p.w0 + (int64_t)e * p.nb02 + (int64_t)r0 * p.nb01, tile_bytes, bar);
            }
        }
    }

    // quantize the activation row(s) while the weights are in flight
    for (int a = 0; a < p.n_act; ++a) {
        int s_row;
        if (MODE == MODE_DOWN_COMBINE) s_row = a;
        else if (MODE == MODE_PLAIN) s_row = s0 % p.ne11;
        else s_row = 0;
        const float * x = reinterpret_cast<const float *>(reinterpret_cast<const char *>(p.src) + (int64_t)t * p.nb12 +
                                                          (int64_t)s_row * p.nb11);
        quantize_row_cta<D::VDT>(x, p.ne00, act + a * p.act_pitch, warp, nwarps, lane);
    }
    __syncthreads();

    if (!mbar_wait_bounded(bar, 0)) {
        if (tid == 0) record_error(GX_DEVERR_TIMEOUT);
        mbar_wait_bounded(bar, 0);  // give copies in flight one more bounded chance
        return;
    }

    // phase 1: integer partial sums and block scales of every (row, unit)
    const int items = NR * U;
    for (int it = tid; it < items; it += kRowsThreads) {
        const int r = it / U, u = it - r * U;
        const uint8_t * arow = act + (MODE == MODE_DOWN_COMBINE ? (r / R) * p.act_pitch : 0);
        D::unit(tile, r * (int)p.nb01, arow, u, terms + ((size_t)r * U + u) * D::TERMS);
    }
    __syncthreads();

    // phase 2: the serial float tail, one thread per (row, chain)
    const int chains = NR * D::CHAINS;
    for (int base = 0; base < chains; base += kRowsThreads) {
        const int it = base + tid;
        const bool ok = it < chains;
        const int r = it / D::CHAINS, c = it % D::CHAINS;
        float v = ok ? D::chain(terms + (size_t)r * U * D::TERMS, U, c) : 0.0f;
        if (D::CHAINS == 8) {
            // ((e0+e1)+(e2+e3)) + ((o0+o1)+(o2+o3)) on lane c == 0 of each group of 8
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
        }
        if (ok && c == 0) dots[r] = v;
    }
    __syncthreads();

    // epilogue
    for (int r = tid; r < R; r += kRowsThreads) {
        if (MODE == MODE_PLAIN) {
            p.dst[((int64_t)t * p.k + s0) * p.ne01 + r0 + r] = dots[r];
        } else if (MODE == MODE_GATE_UP) {
            const float g = dots[r], u = dots[R + r];
            const float a = p.act == 1 ? act_swiglu_oai(g, u, p.alpha, p.limit) : act_swiglu(g, u);
            p.dst[((int64_t)t * p.k + s0) * p.ne01 + r0 + r] = a;
        } else {
            const float * w = p.rw + (int64_t)t * p.k;
            float acc = __fmul_rn(dots[r], w[0]);
            for (int s = 1; s < p.k; ++s) acc = __fadd_rn(acc, __fmul_rn(dots[s * R + r], w[s]));
            p.dst[(int64_t)t * p.ne01 + r0 + r] = acc;
        }
    }
}

// ------------------------------------------------------- small kernels

template <int VDT>
__global__ void k_quantize_rows(const float * src, int ne0, int64_t nb1, uint8_t * dst, int64_t pitch, int nblocks) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int ib = blockIdx.y * (blockDim.x / 32) + w;
    if (ib >= nblocks) return;
    const float * x = reinterpret_cast<const float *>(reinterpret_cast<const char *>(src) + (int64_t)blockIdx.x * nb1);
    uint8_t * row = dst + (int64_t)blockIdx.x * pitch;
    if (VDT == GX_T_Q8_0) {
        quantize_q8_0_block_warp(x[ib * 32 + lane], row + ib * 34, lane);
    } else {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = x[ib * 256 + 8 * lane + j];
        quantize_q8_K_block_warp(v, row + ib * 292, lane);
    }
}

__global__ void k_swiglu(const float * g, const float * u, float * out, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = act_swiglu(g[i], u[i]);
}

__global__ void k_swiglu_oai(const float * g, const float * u, float * out, int64_t n, float alpha, float limit) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = act_swiglu_oai(g[i], u[i], alpha, limit);
}

__global__ void k_expf(const float * x, float * y, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = gx_expf(x[i]);
}

__global__ void k_combine(const float * y, const float * w, float * out, int64_t H, int k, int64_t T) {
    const int64_t n = H * T;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / H, h = i - t * H;
        const float * wt = w + t * k;
        float acc = __fmul_rn(y[(t * k) * H + h], wt[0]);
        for (int s = 1; s < k; ++s) acc = __fadd_rn(acc, __fmul_rn(y[(t * k + s) * H + h], wt[s]));
        out[i] = acc;
    }
}

// ------------------------------------------------------- row gather/scatter
// dst[i] = src[idx[i]] (gather) or dst[idx[i]] = src[i] (scatter), rows of
// H floats, 16-byte vectors when H % 4 == 0 (expert-parallel dispatch and
// combine staging).
__global__ void k_move_rows(const float * src, const int32_t * idx, int64_t n, int64_t H, float * dst, int scatter) {
    const int64_t per = (H % 4 == 0) ? H / 4 : H;
    const int64_t total = n * per;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / per, c = i - r * per;
        const int64_t sr = scatter ? r : idx[r], dr = scatter ? idx[r] : r;
        if (H % 4 == 0) {
            reinterpret_cast<float4 *>(dst + dr * H)[c] = reinterpret_cast<const float4 *>(src + sr * H)[c];
        } else {
            dst[dr * H + c] = src[sr * H + c];
        }
    }
}

__global__ void k_gather_ptrs(const float * const * ptrs, const int32_t * layers, const int32_t * rows, int64_t n,
                              int64_t H, float * dst) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n * H; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i / H, c = i - j * H;
        dst[i] = ptrs[layers[j]][(int64_t)rows[j] * H + c];
    }
}

__global__ void k_add_inplace(float * out, const float * b, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(out[i], b[i]);
}

__global__ void k_fill(float * dst, int64_t n, float v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) dst[i] = v;
}

// ----------------------------------------------------------- synthetic data
// Counter-based generator (splitmix64 finaliser of Steele, Lea & Flood 2014),
// N(0,1) approximated by the standardised sum of four 16-bit uniforms
// (Irwin-Hall, n = 4). Restated identically in the oracle.

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t synth_bits(uint64_t key, uint64_t i) { return splitmix64(key + i * 0xD1B54A32D192ED03ull); }

__device__ __forceinline__ float synth_normal(uint64_t key, uint64_t i, float sigma) {
    const uint64_t b = synth_bits(key, i);
    const int S = (int)(b & 0xffff) + (int)((b >> 16) & 0xffff) + (int)((b >> 32) & 0xffff) + (int)((b >> 48) & 0xffff);
    const float z = __fmul_rn((float)(S - 131070), 2.642899744e-05f);
    return __fmul_rn(z, sigma);
}

__global__ void k_synth_normal(float * dst, int64_t n, uint64_t key, float sigma) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = synth_normal(key, (uint64_t)i, sigma);
}

__device__ __forceinline__ float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

// one thread per block / superblock
__global__ void k_synth_weights(int type, uint8_t * dst, int64_t ne00, int64_t n_rows, uint64_t key, float sigma) {
    const int be = block_elems(type), bb = block_bytes(type);
    const int64_t bpr = ne00 / be;
    const int64_t nblk = bpr * n_rows;
    for (int64_t bi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; bi < nblk; bi += (int64_t)gridDim.x * blockDim.x) {
        uint8_t * o = dst + bi * bb;
        const int64_t row = bi / bpr, col = bi - row * bpr;
        const uint64_t e0 = (uint64_t)(row * ne00 + col * be);
        if (type == GX_T_Q8_0) {
            float x[32];
            float amax = 0.0f;
            for (int j = 0; j < 32; ++j) {
                x[j] = synth_normal(key, e0 + j, sigma);
                const float a = fabsf(x[j]);
                if (a > amax) amax = a;
            }
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            const uint16_t h = f2h(d);
            o[0] = (uint8_t)(h & 0xff);
            o[1] = (uint8_t)(h >> 8);
            for (int j = 0; j < 32; ++j) o[2 + j] = (uint8_t)(int8_t)__float2int_rn(__fmul_rn(x[j], id));
        } else if (type == GX_T_Q4_K) {
            float x[256];
            for (int j = 0; j < 256; ++j) x[j] = synth_normal(key, e0 + j, sigma);
            float scf[8], mnf[8];
            for (int sb = 0; sb < 8; ++sb) {
                float mn = x[32 * sb], mx = mn;
                for (int j = 1; j < 32; ++j) {
                    const float v = x[32 * sb + j];
                    if (v < mn) mn = v;
                    if (v > mx) mx = v;
                }
                if (mn > 0.0f) mn = 0.0f;
                scf[sb] = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
                mnf[sb] = -mn;
            }
            float maxsc = 0.0f, maxmn = 0.0f;
            for (int sb = 0; sb < 8; ++sb) {
                if (scf[sb] > maxsc) maxsc = scf[sb];
                if (mnf[sb] > maxmn) maxmn = mnf[sb];
            }
            const uint16_t d16 = f2h(__fdiv_rn(maxsc, 63.0f)), dm16 = f2h(__fdiv_rn(maxmn, 63.0f));
            const float df = h2f(d16), dmf = h2f(dm16);
            int sc[8], mq[8];
            uint8_t q[256];
            for (int sb = 0; sb < 8; ++sb) {
                sc[sb] = df > 0.0f ? __float2int_rn(clampf(__fdiv_rn(scf[sb], df), 0.0f, 63.0f)) : 0;
                mq[sb] = dmf > 0.0f ? __float2int_rn(clampf(__fdiv_rn(mnf[sb], dmf), 0.0f, 63.0f)) : 0;
                const float ds = __fmul_rn(df, (float)sc[sb]), dm = __fmul_rn(dmf, (float)mq[sb]);
                for (int j = 0; j < 32; ++j) {
                    q[32 * sb + j] = ds > 0.0f ? (uint8_t)__float2int_rn(clampf(__fdiv_rn(__fadd_rn(x[32 * sb + j], dm), ds), 0.0f, 15.0f)) : 0;
                }
            }
            o[0] = (uint8_t)(d16 & 0xff); o[1] = (uint8_t)(d16 >> 8);
            o[2] = (uint8_t)(dm16 & 0xff); o[3] = (uint8_t)(dm16 >> 8);
            uint8_t * s = o + 4;
            for (int j = 0; j < 4; ++j) {
                s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
                s[j + 4] = (uint8_t)((mq[j] & 63) | ((mq[j + 4] >> 4) << 6));
                s[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mq[j + 4] & 15) << 4));
            }
            for (int j = 0; j < 4; ++j)
                for (int m = 0; m < 32; ++m) o[16 + 32 * j + m] = (uint8_t)(q[64 * j + m] | (q[64 * j + 32 + m] << 4));
        } else if (type == GX_T_Q6_K) {
            float x[256];
            for (int j = 0; j < 256; ++j) x[j] = synth_normal(key, e0 + j, sigma);
            float scf[16];
            float maxs = 0.0f;
            for (int g = 0; g < 16; ++g) {
                float amax = 0.0f;
                for (int j = 0; j < 16; ++j) {
                    const float a = fabsf(x[16 * g + j]);
                    if (a > amax) amax = a;
                }
                scf[g] = __fdiv_rn(amax, 31.0f);
                if (scf[g] > maxs) maxs = scf[g];
            }
            const uint16_t d16 = f2h(__fdiv_rn(maxs, 127.0f));
            const float df = h2f(d16);
            for (int j = 0; j < 208; ++j) o[j] = 0;
            for (int g = 0; g < 16; ++g) {
                const int sc = df > 0.0f ? __float2int_rn(clampf(__fdiv_rn(scf[g], df), 0.0f, 127.0f)) : 0;
                o[192 + g] = (uint8_t)(int8_t)sc;
                const float ds = __fmul_rn(df, (float)sc);
                for (int j = 0; j < 16; ++j) {
                    const int e = 16 * g + j;
                    const int qv = ds > 0.0f ? __float2int_rn(clampf(__fdiv_rn(x[e], ds), -32.0f, 31.0f)) : 0;
                    const int code = qv + 32;
                    const int hh = e / 128, r = e % 128;
                    o[64 * hh + (r % 64)] |= (uint8_t)((code & 15) << (r < 64 ? 0 : 4));
                    o[128 + 32 * hh + (r % 32)] |= (uint8_t)((code >> 4) << (2 * (r / 32)));
                }
            }
            o[208] = (uint8_t)(d16 & 0xff);
            o[209] = (uint8_t)(d16 >> 8);
        } else if (type == GX_T_MXFP4) {
            const uint64_t w0 = synth_bits(key, 3 * (uint64_t)bi), w1 = synth_bits(key, 3 * (uint64_t)bi + 1),
                           w2 = synth_bits(key, 3 * (uint64_t)bi + 2);
            o[0] = (uint8_t)(118 + (w0 & 7));
            for (int j = 0; j < 8; ++j) { o[1 + j] = (uint8_t)(w1 >> (8 * j)); o[9 + j] = (uint8_t)(w2 >> (8 * j)); }
        } else if (type == GX_T_IQ1_S) {
            uint64_t w[7];
            for (int j = 0; j < 7; ++j) w[j] = synth_bits(key, 8 * (uint64_t)bi + j);
            const uint16_t d16 = (uint16_t)(0x1400u | (w[0] & 0x3ffu));
            o[0] = (uint8_t)(d16 & 0xff); o[1] = (uint8_t)(d16 >> 8);
            for (int j = 0; j < 32; ++j) o[2 + j] = (uint8_t)(w[1 + j / 8] >> (8 * (j % 8)));
            for (int j = 0; j < 16; ++j) o[34 + j] = (uint8_t)(w[5 + j / 8] >> (8 * (j % 8)));
        }
    }
}

// -------------------------------------------------------------- launchers

static int grid_1d(int64_t n, int threads) {
    int64_t b = (n + threads - 1) / threads;
    if (b > 148 * 32) b = 148 * 32;
    if (b < 1) b = 1;
    return (int)b;
}

uint64_t synth_key(uint64_t seed, uint64_t stream_id) {
    auto sm = [](uint64_t z) {
        z += 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    return sm(seed ^ sm(stream_id + 0x632BE59BD9B4E019ull));
}

template <int TYPE, int MODE>
static cudaError_t launch_rows_t(const RowsParams & p, dim3 grid, uint32_t smem, cudaStream_t stream) {
    static int configured_smem = 0;  // per instantiation, single device process
    if ((int)smem > configured_smem) {
        cudaError_t e = cudaFuncSetAttribute(k_rows<TYPE, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured_smem = (int)smem;
    }
    k_rows<TYPE, MODE><<<grid, kRowsThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

template <int MODE>
static cudaError_t launch_rows_mode(int type, const RowsParams & p, dim3 grid, uint32_t smem, cudaStream_t stream) {
    switch (type) {
        case GX_T_Q8_0: return launch_rows_t<GX_T_Q8_0, MODE>(p, grid, smem, stream);
        case GX_T_MXFP4: return launch_rows_t<GX_T_MXFP4, MODE>(p, grid, smem, stream);
        case GX_T_Q4_K: return launch_rows_t<GX_T_Q4_K, MODE>(p, grid, smem, stream);
        case GX_T_Q6_K: return launch_rows_t<GX_T_Q6_K, MODE>(p, grid, smem, stream);
        case GX_T_IQ1_S: return launch_rows_t<GX_T_IQ1_S, MODE>(p, grid, smem, stream);
        default: return cudaErrorInvalidValue;
    }
}

static int terms_per_unit(int type) {
    switch (type) {
        case GX_T_Q8_0: return Dot<GX_T_Q8_0>::TERMS;
        case GX_T_MXFP4: return Dot<GX_T_MXFP4>::TERMS;
        case GX_T_Q4_K: return Dot<GX_T_Q4_K>::TERMS;
        case GX_T_Q6_K: return Dot<GX_T_Q6_K>::TERMS;
        case GX_T_IQ1_S: return Dot<GX_T_IQ1_S>::TERMS;
        default: return 0;
    }
}

static uint32_t align_up(uint64_t v, uint64_t a) { return (uint32_t)((v + a - 1) / a * a); }

// Lay out shared memory for a tile of NR rows and n_act activation rows.
// Returns the byte count, or 0 when it does not fit.
uint32_t rows_smem_layout(int type, int mode, RowsParams & p) {
    const int n_exp = mode == MODE_DOWN_COMBINE ? p.k : 1;
    const int NR = mode == MODE_GATE_UP ? 2 * p.R : n_exp * p.R;
    const int vdt = vec_dot_type(type);
    const int U = p.ne00 / 64;
    p.act_pitch = (int32_t)align_up((uint64_t)row_bytes(vdt, p.ne00), 16);
    p.n_act = mode == MODE_DOWN_COMBINE ? p.k : 1;
    uint64_t off = 0;
    p.bar_off = 0;
    off = 128;
    p.tile_off = (uint32_t)off;
    off = align_up(off + (uint64_t)NR * p.nb01 + 16, 128);
    p.act_off = (uint32_t)off;
    off = align_up(off + (uint64_t)p.n_act * p.act_pitch + 16, 128);
    p.terms_off = (uint32_t)off;
    off = align_up(off + (uint64_t)NR * U * terms_per_unit(type) * 4, 128);
    p.dots_off = (uint32_t)off;
    off = align_up(off + (uint64_t)NR * 4, 128);
    if (off > kMaxSmem) return 0;
    return (uint32_t)off;
}

cudaError_t launch_rows(int type, int mode, RowsParams & p, dim3 grid, cudaStream_t stream) {
    const uint32_t smem = rows_smem_layout(type, mode, p);
    if (smem == 0) return cudaErrorInvalidConfiguration;
    switch (mode) {
        case MODE_PLAIN: return launch_rows_mode<MODE_PLAIN>(type, p, grid, smem, stream);
        case MODE_GATE_UP: return launch_rows_mode<MODE_GATE_UP>(type, p, grid, smem, stream);
        case MODE_DOWN_COMBINE: return launch_rows_mode<MODE_DOWN_COMBINE>(type, p, grid, smem, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_quantize_rows(int vdt, const float * src, int ne0, int64_t nrows, int64_t nb1, uint8_t * dst, int64_t pitch,
                                 cudaStream_t stream) {
    if (nrows <= 0) return cudaSuccess;
    const int nblocks = vdt == GX_T_Q8_0 ? ne0 / 32 : ne0 / 256;
    const dim3 grid((unsigned)nrows, (unsigned)((nblocks + 3) / 4));
    if (vdt == GX_T_Q8_0) k_quantize_rows<GX_T_Q8_0><<<grid, 128, 0, stream>>>(src, ne0, nb1, dst, pitch, nblocks);
    else k_quantize_rows<GX_T_Q8_K><<<grid, 128, 0, stream>>>(src, ne0, nb1, dst, pitch, nblocks);
    return cudaGetLastError();
}

cudaError_t launch_swiglu(const float * g, const float * u, float * out, int64_t n, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    k_swiglu<<<grid_1d(n, 256), 256, 0, stream>>>(g, u, out, n);
    return cudaGetLastError();
}

cudaError_t launch_swiglu_oai(const float * g, const float * u, float * out, int64_t n, float alpha, float limit,
                              cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    k_swiglu_oai<<<grid_1d(n, 256), 256, 0, stream>>>(g, u, out, n, alpha, limit);
    return cudaGetLastError();
}

cudaError_t launch_expf(const float * x, float * y, int64_t n, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    k_expf<<<grid_1d(n, 256), 256, 0, stream>>>(x, y, n);
    return cudaGetLastError();
}

cudaError_t launch_combine(const float * y, const float * w, float * out, int64_t H, int k, int64_t T, cudaStream_t stream) {
    if (H * T <= 0) return cudaSuccess;
    k_combine<<<grid_1d(H * T, 256), 256, 0, stream>>>(y, w, out, H, k, T);
    return cudaGetLastError();
}

cudaError_t launch_move_rows(const float * src, const int32_t * idx, int64_t n, int64_t H, float * dst, bool scatter,
                             cudaStream_t stream) {
    if (n <= 0 || H <= 0) return cudaSuccess;
    const int64_t per = (H % 4 == 0) ? H / 4 : H;
    k_move_rows<<<grid_1d(n * per, 256), 256, 0, stream>>>(src, idx, n, H, dst, scatter ? 1 : 0);
    return cudaGetLastError();
}

cudaError_t launch_gather_ptrs(const float * const * ptrs, const int32_t * layers, const int32_t * rows, int64_t n,
                               int64_t H, float * dst, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    k_gather_ptrs<<<grid_1d(n * H, 256), 256, 0, stream>>>(ptrs, layers, rows, n, H, dst);
    return cudaGetLastError();
}

cudaError_t launch_add_inplace(float * out, const float * b, int64_t n, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    k_add_inplace<<<grid_1d(n, 256), 256, 0, stream>>>(out, b, n);
    return cudaGetLastError();
}

// MXFP4 matrices of one record into the tensor-core record layout
// (Mxfp4TcMats). One thread per (row, block): byte reads of the 17-byte
// block, one 16-byte store of its codes, one byte store of its scale.
__global__ void k_mxfp4_tc_layout(const uint8_t * src, uint8_t * dst, Mxfp4TcMats m) {
    int64_t n[3], tot = 0;
    for (int q = 0; q < 3; ++q) {
        n[q] = (int64_t)m.rows[q] * m.nb[q];
        tot += n[q];
    }
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < tot; i += (int64_t)gridDim.x * blockDim.x) {
        int q = 0;
        int64_t j = i;
        while (j >= n[q]) j -= n[q++];
        const int nb = m.nb[q];
        const int64_t r = j / nb, bb = j - r * nb;
        const uint8_t * blk = src + m.off[q] + r * (int64_t)(17 * nb) + 17 * bb;
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            w[k] = (uint32_t)blk[1 + 4 * k] | ((uint32_t)blk[2 + 4 * k] << 8) | ((uint32_t)blk[3 + 4 * k] << 16) |
                   ((uint32_t)blk[4 + 4 * k] << 24);
        const int64_t cs = mxfp4_tc_cstride(nb), nch = cs / 64, tr = m.trows[q];
        const int64_t tile = r / tr, ri = r - tile * tr, c = bb / 4;
        uint8_t * d = dst + m.doff[q];
        *reinterpret_cast<uint4 *>(d + ((tile * nch + c) * tr + ri) * 64 + 16 * (bb - 4 * c)) = make_uint4(w[0], w[1], w[2], w[3]);
        d[(int64_t)m.rows[q] * cs + r * nb + bb] = blk[0];
    }
}

cudaError_t launch_mxfp4_tc_layout(const uint8_t * src, uint8_t * dst, const Mxfp4TcMats & m, cudaStream_t stream) {
    k_mxfp4_tc_layout<<<1184, 256, 0, stream>>>(src, dst, m);   // 8 CTAs per SM of a B200, grid-stride
    return cudaGetLastError();
}

cudaError_t launch_fill(float * dst, int64_t n, float v, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    k_fill<<<grid_1d(n, 256), 256, 0, stream>>>(dst, n, v);
    return cudaGetLastError();
}

cudaError_t launch_router(const RouterLaunch & r, cudaStream_t stream) {
    const int64_t rows = r.T * r.n_layers;
    if (rows <= 0) return cudaSuccess;
    RouterParams p{};
    p.logits = r.logits;
    p.ld = r.ld;
    p.bias = r.bias;
    p.table = r.table;
    p.ids = r.ids;
    p.w = r.w;
    p.slots = r.slots;
    p.rows = rows;
    p.T = r.T;
    p.E = r.E;
    p.k = r.k;
    p.gating = r.gating;
    p.groups = r.groups;
    p.group_used = r.group_used;
    p.norm = r.norm;
    p.scale_on = r.scale_on;
    p.scale = r.scale;
    const size_t smem = (size_t)kRouterWarps * router_smem_floats(r.E) * sizeof(float);
    const unsigned grid = (unsigned)((rows + kRouterWarps - 1) / kRouterWarps);
    k_router<<<grid, 32 * kRouterWarps, smem, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_synth_normal(float * dst, int64_t n, uint64_t seed, uint64_t stream_id, float sigma, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    k_synth_normal<<<grid_1d(n, 256), 256, 0, stream>>>(dst, n, synth_key(seed, stream_id), sigma);
    return cudaGetLastError();
}

cudaError_t launch_synth_weights(int type, void * dst, int64_t ne00, int64_t n_rows, uint64_t seed, uint64_t stream_id,
                                 float sigma, cudaStream_t stream) {
    const int64_t nblk = (ne00 / block_elems(type)) * n_rows;
    if (nblk <= 0) return cudaSuccess;
    const int threads = (type == GX_T_Q4_K || type == GX_T_Q6_K) ? 64 : 256;
    k_synth_weights<<<grid_1d(nblk, threads), threads, 0, stream>>>(type, (uint8_t *)dst, ne00, n_rows,
                                                                     synth_key(seed, stream_id), sigma);
    return cudaGetLastError();
}

// ------------------------------------------------------- decode launchers

static int device_sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
        cached[dev] = sms;
    }
    return cached[dev];
}

// Resident CTAs per SM of one kernel configuration, computed once (the
// occupancy query and the shared-memory attribute stay off the launch path).
template <typename K>
static cudaError_t resident_per_sm(K kernel, int threads, uint32_t smem, int & per_sm) {
    // keyed by the kernel's address: every instantiation has its own
    // shared-memory attribute and occupancy
    static std::mutex mu;
    static std::map<std::pair<const void *, uint64_t>, int> cache;
    static std::map<const void *, int> configured;
    const void * fn = reinterpret_cast<const void *>(kernel);
    const auto key = std::make_pair(fn, ((uint64_t)threads << 32) | smem);
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        per_sm = it->second;
        return cudaSuccess;
    }
    int & conf = configured[fn];
    if ((int)smem > conf) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        conf = (int)smem;
    }
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    cache[key] = per_sm;
    return cudaSuccess;
}

template <int TYPE, int MODE>
static cudaError_t launch_decode_t(DecodeParams & p, int threads, uint32_t smem, cudaStream_t stream, bool pdl) {
    int per_sm = 0;
    cudaError_t e = resident_per_sm(k_decode<TYPE, MODE>, threads, smem, per_sm);
    if (e != cudaSuccess) return e;
    const int cap = per_sm * device_sm_count();
    // one unit per CTA (S = 1) launches every unit; persistent grids are capped
    const int grid = (p.S == 1 || p.n_units < cap) ? p.n_units : cap;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_decode<TYPE, MODE>, p);
}

// Shared-memory layout and tiling of a decode launch; 0 when it cannot fit.
uint32_t decode_layout(int mode, DecodeParams & p, int & threads) {
    const int nexp = mode == 1 ? 2 : p.k;
    if (mode == 2 && (p.R & 1)) return 0;   // row pairs stay inside one expert tile
    threads = 4 * nexp * p.R;               // eight lanes per pair of rows
    if (threads > kDecodeMaxThreads || threads < 32 || threads % 32 != 0) return 0;
    if (p.nb01 % 16 == 0) {
        p.row_copy = 1;
        p.pitch_w = (int32_t)(p.nb01 % 128 == 0 ? p.nb01 + 16 : p.nb01);
    } else {
        if ((p.R * p.nb01) % 16 != 0) return 0;
        p.row_copy = 0;
        p.pitch_w = (int32_t)p.nb01;
    }
    p.stage_bytes = (int32_t)align_up((uint64_t)nexp * p.R * p.pitch_w + 16, 128);
    const uint32_t act_bytes = align_up((uint64_t)p.a_rows * p.al.pitch + 16, 128);
    const uint32_t fixed = 128 + act_bytes + 128 + 128;
    int S = p.S;
    if (S <= 0) {
        const uint32_t budget = 72 * 1024;   // three CTAs per SM
        S = (int)((budget > fixed ? budget - fixed : 0) / (uint32_t)p.stage_bytes);
        if (S > 4) S = 4;
        if (S < 2) S = 2;
    }
    p.S = S;
    p.act_off = 128;
    p.stage_off = p.act_off + act_bytes;
    p.dots_off = p.stage_off + (uint32_t)S * p.stage_bytes;
    p.flag_off = p.dots_off + (uint32_t)kDecodeMaxThreads / 8 * 2 * 4;
    const uint32_t total = p.flag_off + 128;
    if (total > kMaxSmem) return 0;
    return total;
}

template <int MODE>
static cudaError_t launch_decode_mode(int type, DecodeParams & p, int threads, uint32_t smem, cudaStream_t stream, bool pdl) {
    switch (type) {
        case GX_T_Q8_0: return launch_decode_t<GX_T_Q8_0, MODE>(p, threads, smem, stream, pdl);
        case GX_T_MXFP4: return launch_decode_t<GX_T_MXFP4, MODE>(p, threads, smem, stream, pdl);
        case GX_T_Q4_K: return launch_decode_t<GX_T_Q4_K, MODE>(p, threads, smem, stream, pdl);
        case GX_T_Q6_K: return launch_decode_t<GX_T_Q6_K, MODE>(p, threads, smem, stream, pdl);
        case GX_T_IQ1_S: return launch_decode_t<GX_T_IQ1_S, MODE>(p, threads, smem, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

static void choose_stages(int mode, DecodeParams & p);

template <int MODE>
static cudaError_t prepare_decode_mode(int type, int threads, uint32_t smem) {
    int per_sm = 0;
    switch (type) {
        case GX_T_Q8_0: return resident_per_sm(k_decode<GX_T_Q8_0, MODE>, threads, smem, per_sm);
        case GX_T_MXFP4: return resident_per_sm(k_decode<GX_T_MXFP4, MODE>, threads, smem, per_sm);
        case GX_T_Q4_K: return resident_per_sm(k_decode<GX_T_Q4_K, MODE>, threads, smem, per_sm);
        case GX_T_Q6_K: return resident_per_sm(k_decode<GX_T_Q6_K, MODE>, threads, smem, per_sm);
        case GX_T_IQ1_S: return resident_per_sm(k_decode<GX_T_IQ1_S, MODE>, threads, smem, per_sm);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t prepare_decode(int type, int mode, DecodeParams p) {
    int threads = 0;
    if (p.S == 0) choose_stages(mode, p);
    const uint32_t smem = decode_layout(mode, p, threads);
    if (smem == 0) return cudaErrorInvalidConfiguration;
    return mode == 1 ? prepare_decode_mode<1>(type, threads, smem) : prepare_decode_mode<2>(type, threads, smem);
}

// Decode-sized launches (a few units per SM) run one unit per CTA with one
// stage: half the shared memory per CTA, twice the resident warps, every
// weight byte requested at once. Larger launches use persistent CTAs with a
// multi-stage pipeline.
static void choose_stages(int mode, DecodeParams & p) {
    DecodeParams one = p;
    one.S = 1;
    int threads = 0;
    const uint32_t smem1 = decode_layout(mode, one, threads);
    if (smem1 == 0) { p.S = 0; return; }
    const uint32_t per_sm_smem = 227u * 1024u;
    const int per_sm = (int)(per_sm_smem / (smem1 + 1024u)) > 0 ? (int)(per_sm_smem / (smem1 + 1024u)) : 1;
    p.S = p.n_units <= 2 * per_sm * device_sm_count() ? 1 : 0;
}

cudaError_t launch_decode(int type, int mode, DecodeParams & p, cudaStream_t stream, bool pdl) {
    int threads = 0;
    if (p.S == 0) choose_stages(mode, p);
    const uint32_t smem = decode_layout(mode, p, threads);
    if (smem == 0) return cudaErrorInvalidConfiguration;
    return mode == 1 ? launch_decode_mode<1>(type, p, threads, smem, stream, pdl)
                     : launch_decode_mode<2>(type, p, threads, smem, stream, pdl);
}

cudaError_t launch_quant_split(int vdt, const float * src, int ne0, int64_t nrows, int64_t nb1, uint8_t * dst,
                               cudaStream_t stream, bool pdl) {
    const ActLayout L = act_layout(vdt, ne0);
    const int64_t warps = nrows * (ne0 / (vdt == GX_T_Q8_0 ? 32 : 256));
    if (warps <= 0) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((warps + 3) / 4));
    cfg.blockDim = dim3(128);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (vdt == GX_T_Q8_0) return cudaLaunchKernelEx(&cfg, k_quant_split<GX_T_Q8_0>, src, ne0, nrows, nb1, dst, L);
    return cudaLaunchKernelEx(&cfg, k_quant_split<GX_T_Q8_K>, src, ne0, nrows, nb1, dst, L);
}

// ------------------------------------------------------- stack launcher

int device_sms() { return device_sm_count(); }

bool stack_types_supported(int type_gate, int type_down) {
    return (type_gate == GX_T_Q8_0 && type_down == GX_T_Q8_0) || (type_gate == GX_T_Q4_K && type_down == GX_T_Q6_K) ||
           (type_gate == GX_T_MXFP4 && type_down == GX_T_MXFP4) || (type_gate == GX_T_IQ1_S && type_down == GX_T_IQ1_S);
}

// Bulk-copy mode of one role: rows of a multiple of 128 bytes get 16 bytes of
// padding against bank conflicts and one copy per row; other rows are copied
// as one tile of R rows per expert (R rows must make whole 16-byte chunks).
static bool stack_copy_mode(int64_t nb01, int R, int32_t & row_copy, int32_t & pitch) {
    if ((R * nb01) % 16 != 0) return false;
    row_copy = nb01 % 128 == 0 ? 1 : 0;
    pitch = (int32_t)(row_copy ? nb01 + 16 : nb01);
    return true;
}

// Shared-memory layout of the stack kernel; 0 when the shape is not covered.
// Jobs: 8 gate + 8 up rows, or k*Rd = 32 down rows. Row modes: 0 two-lane
// Q8_0 rows, 2 two-lane Q4_K gate/up and Q6_K down rows (both in 4 staggered
// gate/up tiles and rows of K % 256 == 0), 1 octet rows (any whole number
// of their type's 64- or 256-element units, checked per layer; 2 gate/up copies).
// Row mode 5 (gx_stack_tma.cuh): 64 + 64 gate/up rows, 32 rows of each of 4
// experts per down job, 4 epilogue warps, no weight stage of the generic
// layout (its ring is the region at tc_off: as many 16 KB chunk stages as fit).
static uint32_t stack_layout_t5(StackParams & p, int & threads) {
    if (p.Rg != 64 || p.Rd != 32 || p.k != 4 || p.W != kT5Warps - 4 || p.C != 1) return 0;
    if (p.H % 64 || p.I % 64 || p.H / 32 > kTcMaxBlocks || p.I / 32 > kTcMaxBlocks) return 0;
    if (p.NL < 1 || p.NL > kStackMaxLayers) return 0;
    if (p.alx.d_off != 64 * (p.H / 32) || p.ald.d_off != 64 * p.k * (p.I / 32) || p.alx.pitch < p.alx.d_off + 256 ||
        p.alx.pitch < p.alx.d_off + 2 * (p.H / 32) || (int64_t)p.k * p.ald.pitch < p.ald.d_off + 256 ||
        (int64_t)p.k * p.ald.pitch < p.ald.d_off + 2 * p.k * (p.I / 32))
        return 0;
    threads = 32 * (kStackProducers + 2) + 32 * p.W;
    p.stage_bytes = 0;
    p.row_copy_d = 0;
    p.pitch_d = (int32_t)p.nb01_d;
    p.bar_off = 0;
    p.meta_off = (uint32_t)align_up(8ull * (3 * kStackMaxConsumers + 2 * kStackBufs), 128);
    p.stage_off = p.meta_off + (uint32_t)align_up(4ull * (3 * kStackMaxConsumers + 2 * kStackBufs + 1), 128);
    p.tc_off = p.stage_off;
    const int nbmax = (p.H > p.I ? p.H : p.I) / 32;
    // the most stages that fit, a multiple of kT5StageStep (gx_stack_tma.cuh),
    // with two down-input buffers where they fit (a down job's inputs then
    // load during the job before), else one
    const auto rest = [&](int nbd) {
        return align_up((uint64_t)kStackBufs * p.alx.pitch, 128) + align_up((uint64_t)nbd * p.k * p.ald.pitch, 128) +
               (uint64_t)p.NL * 32u + (uint64_t)p.C * 32u * 4u + align_up((uint64_t)p.NL * p.T * p.k * 4u, 16);
    };
    int stages = kT5StagesMax / kT5StageStep * kT5StageStep, nbd = 2;
    while (stages >= kT5StagesMin && p.tc_off + align_up(t5_bytes(nbmax, stages), 128) + rest(nbd) > kMaxSmem) {
        if (nbd == 2) {
            nbd = 1;
        } else {
            nbd = 2;
            stages -= kT5StageStep;
        }
    }
    if (stages < kT5StagesMin || stages % kT5StageStep != 0) return 0;
    p.tc_na = stages;
    p.nbuf_d = nbd;
    p.xbuf_off = p.tc_off + (uint32_t)align_up(t5_bytes(nbmax, stages), 128);
    p.dbuf_off = p.xbuf_off + (uint32_t)align_up((uint64_t)kStackBufs * p.alx.pitch, 128);
    p.wt_off = p.dbuf_off + (uint32_t)align_up((uint64_t)nbd * p.k * p.ald.pitch, 128);
    p.dots_off = p.wt_off + (uint32_t)p.NL * 32u;
    p.slots_off = p.dots_off + (uint32_t)p.C * 32u * 4u;
    p.grid_off = p.slots_off + (uint32_t)align_up((uint64_t)p.NL * p.T * p.k * 4u, 16);
    // the job table: every job of a CTA of a 148-CTA grid, or what the rest holds
    const int64_t nj = (int64_t)p.NL * p.T * ((int64_t)p.k * (p.I / p.Rg) + p.H / p.Rd);
    const int64_t want = (nj + 147) / 148;
    p.t5_jobs_off = p.grid_off;
    const int64_t room = p.grid_off <= kMaxSmem ? (int64_t)(kMaxSmem - p.grid_off) / 8 : 0;
    p.t5_jobs = (int32_t)(want < room ? want : room);
    p.grid_off += (uint32_t)(8 * p.t5_jobs);
    return p.grid_off <= kMaxSmem ? p.grid_off : 0;
}

uint32_t stack_layout(StackParams & p, int & threads) {
    if (p.row_mode == 5) return stack_layout_t5(p, threads);
    const bool mx = p.row_mode == 3 || p.row_mode == 4;
    if (!(p.Rg == 8 || (p.Rg == 16 && mx)) || p.Rd < 1 || (p.k * p.Rd != 32 && !(p.row_mode == 2 && p.k * p.Rd == 16)))
        return 0;
    // tensor-core MXFP4 jobs: 16 + 16 gate/up rows, 8 rows of each of 4 experts,
    // the 12 role warps of gx_stack_tc.cuh, rows of at most kTcMaxBlocks blocks
    if (p.row_mode == 4 && (p.Rg != 16 || p.k != 4 || p.W != 12 || p.H / 32 > kTcMaxBlocks || p.I / 32 > kTcMaxBlocks))
        return 0;
    const bool tiles8 = p.row_mode == 1 || mx;   // gate/up as 2 copies of Rg rows
    if (p.row_mode < 0 || p.row_mode > 4 || p.gu_copies != (tiles8 ? 2 : 4)) return 0;
    const int ra = tiles8 ? 64 : 256;
    if (p.H % ra || p.I % ra || p.I % p.Rg || p.qblk % p.Rg || p.H % p.Rd) return 0;
    if (p.C < 1 || p.C > kStackMaxConsumers || p.NL < 1 || p.NL > kStackMaxLayers) return 0;
    // every stage belongs to one weight producer (stage s gets jobs s, s+C, ...,
    // all of producer s % P): that producer issued the stage's previous job, so
    // the stage's "empty" barrier is at most one phase behind when it waits on
    // it and the parity wait is unambiguous. With C not a multiple of P two
    // producers would share a stage and one could wait on a barrier two phases
    // behind, read the older phase as complete and refill a stage in use.
    if (p.C % (p.row_mode == 4 ? 1 : kStackProducers) != 0) return 0;
    if (p.W < 1 || p.W > stack_max_warps(p.row_mode)) return 0;
    if (p.row_mode == 1 && (p.Rd & 1)) return 0;   // octet row pairs stay inside one expert
    threads = 32 * (kStackProducers + 2) + 32 * p.W;
    // the digit rows of row mode 4 (per block: 2 K halves x k rows x 2 digits x 16 bytes, then fp16 scales)
    // (and room for the MMA's N = 16 B tiles of the last block, which read up to 256 bytes past the digits)
    if (p.row_mode == 4 && (p.alx.d_off != 64 * (p.H / 32) || p.ald.d_off != 64 * p.k * (p.I / 32) ||
                            p.alx.pitch < p.alx.d_off + 256 || p.alx.pitch < p.alx.d_off + 2 * (p.H / 32) ||
                            (int64_t)p.k * p.ald.pitch < p.ald.d_off + 256 ||
                            (int64_t)p.k * p.ald.pitch < p.ald.d_off + 2 * p.k * (p.I / 32)))
        return 0;
    if (!stack_copy_mode(p.nb01_d, p.Rd, p.row_copy_d, p.pitch_d)) return 0;
    uint64_t gw;
    if (p.gu_copies == 4) {
        // gate/up tiles: tile t starts at a 16-byte chunk index xs[t] mod 8; a
        // quarter warp reads one row of each tile at both lane halves. Q8_0
        // halves are 32 bytes apart: xs = {0, 1, 4, 5} gives chunk groups
        // {0,2}, {1,3}, {4,6}, {5,7}; Q4_K halves are 16 bytes apart:
        // xs = {0, 2, 4, 6} gives {0,1}, {2,3}, {4,5}, {6,7}
        if (p.nb01_g % 16 != 0) return 0;
        static const int xs0[4] = {0, 1, 4, 5}, xs2[4] = {0, 2, 4, 6};
        const int * xs = p.row_mode == 2 ? xs2 : xs0;
        const uint64_t tile = 4ull * (uint64_t)p.nb01_g;
        p.gu_tile[0] = 0;
        for (int t = 1; t < 4; ++t) {
            uint64_t c = (p.gu_tile[t - 1] + tile + 15) / 16;
            while (c % 8 != (uint64_t)xs[t]) ++c;
            p.gu_tile[t] = (int32_t)(c * 16);
        }
        gw = (uint64_t)p.gu_tile[3] + 4ull * (uint64_t)p.nb01_g;
    } else {
        // octet and MXFP4 rows: the Rg gate rows, then the Rg up rows, one copy each
        const uint64_t tile = (uint64_t)p.Rg * (uint64_t)p.nb01_g;
        if (tile % 16 != 0) return 0;
        p.gu_tile[0] = 0;
        p.gu_tile[1] = (int32_t)tile;
        p.gu_tile[2] = p.gu_tile[3] = 0;
        gw = 2 * tile + 16;   // ld_words may read one word past a row
    }
    // the unaligned row readers (octet rows, Q6_K) may read one word past the last row
    const uint64_t dw = (uint64_t)p.k * p.Rd * (uint64_t)p.pitch_d + (p.row_mode != 0 ? 16 : 0);
    p.stage_bytes = (int32_t)align_up(gw > dw ? gw : dw, 128);
    p.bar_off = 0;      // 3*C + 2*kStackBufs mbarriers
    p.meta_off = (uint32_t)align_up(8ull * (3 * kStackMaxConsumers + 2 * kStackBufs), 128);
    // fill words, buffer counters, release counter per stage, next task, finished parts per stage
    p.stage_off = p.meta_off + (uint32_t)align_up(4ull * (3 * kStackMaxConsumers + 2 * kStackBufs + 1), 128);
    // row mode 4: the A tiles, scales, pair terms, dots and barriers of the roles
    p.tc_off = p.stage_off + (uint32_t)p.C * (uint32_t)p.stage_bytes;
    const int nbmax = (p.H > p.I ? p.H : p.I) / 32;
    p.tc_na = kTcAmax;
    p.xbuf_off = p.tc_off + (p.row_mode == 4 ? (uint32_t)align_up(tc_bytes(nbmax, p.tc_na), 128) : 0u);
    p.dbuf_off = p.xbuf_off + align_up((uint64_t)kStackBufs * p.alx.pitch, 128);
    p.nbuf_d = p.row_mode == 4 ? 1 : kStackBufs;
    p.wt_off = p.dbuf_off + align_up((uint64_t)p.nbuf_d * p.k * p.ald.pitch, 128);
    p.dots_off = p.wt_off + (uint32_t)p.NL * 32u;    // per-layer weight bases
    p.slots_off = p.dots_off + (uint32_t)p.C * 32u * 4u;   // 32 down-row dots per stage
    p.grid_off = p.slots_off + (uint32_t)align_up((uint64_t)p.NL * p.T * p.k * 4u, 16);
    // row mode 4: the B tiles of the last MMA steps read up to 2 KB past the input rows
    const uint32_t total = p.grid_off + (p.need_grid ? 2048u * 8u : 0u) + (p.row_mode == 4 ? 2048u : 0u);
    if (p.row_mode == 4 && total > kMaxSmem) {
        // fewer A slots (MMA steps in flight), down to kTcAmin
        const uint32_t over = total - kMaxSmem;
        const int drop = (int)((over + 4095) / 4096);
        if (p.tc_na - drop < kTcAmin) return 0;
        p.tc_na -= drop;
        const uint32_t shift = (uint32_t)align_up(tc_bytes(nbmax, kTcAmax), 128) - (uint32_t)align_up(tc_bytes(nbmax, p.tc_na), 128);
        p.xbuf_off -= shift;
        p.dbuf_off -= shift;
        p.wt_off -= shift;
        p.dots_off -= shift;
        p.slots_off -= shift;
        p.grid_off -= shift;
        return total - shift <= kMaxSmem ? total - shift : 0;
    }
    return total <= kMaxSmem ? total : 0;
}

template <int TG, int TD, int TC = 0>
static cudaError_t stack_dispatch(const StackParams * p, int grid, int threads, uint32_t smem, cudaStream_t stream,
                                  int * per_sm) {
    if (per_sm) return resident_per_sm(k_stack<TG, TD, TC>, threads, smem, *per_sm);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    // all CTAs must be resident at once: units wait on units of other CTAs
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_stack<TG, TD, TC>, *p);
}

static cudaError_t stack_switch(int tg, int td, const StackParams * p, int grid, int threads, uint32_t smem,
                                cudaStream_t stream, int * per_sm) {
    if (tg == GX_T_Q8_0 && td == GX_T_Q8_0) return stack_dispatch<GX_T_Q8_0, GX_T_Q8_0>(p, grid, threads, smem, stream, per_sm);
    if (tg == GX_T_Q4_K && td == GX_T_Q6_K) return stack_dispatch<GX_T_Q4_K, GX_T_Q6_K>(p, grid, threads, smem, stream, per_sm);
    if (tg == GX_T_MXFP4 && td == GX_T_MXFP4)
        return p->row_mode == 4   ? stack_dispatch<GX_T_MXFP4, GX_T_MXFP4, 4>(p, grid, threads, smem, stream, per_sm)
               : p->row_mode == 5 ? stack_dispatch<GX_T_MXFP4, GX_T_MXFP4, 5>(p, grid, threads, smem, stream, per_sm)
                                  : stack_dispatch<GX_T_MXFP4, GX_T_MXFP4>(p, grid, threads, smem, stream, per_sm);
    if (tg == GX_T_IQ1_S && td == GX_T_IQ1_S)
        return stack_dispatch<GX_T_IQ1_S, GX_T_IQ1_S>(p, grid, threads, smem, stream, per_sm);
    return cudaErrorInvalidValue;
}

cudaError_t prepare_stack(int type_gate, int type_down, const StackParams & p, int threads, uint32_t smem, int & per_sm) {
    per_sm = 0;
    return stack_switch(type_gate, type_down, &p, 0, threads, smem, nullptr, &per_sm);
}

cudaError_t launch_stack(int type_gate, int type_down, const StackParams & p, int grid, int threads, uint32_t smem,
                         cudaStream_t stream) {
    return stack_switch(type_gate, type_down, &p, grid, threads, smem, stream, nullptr);
}

// ------------------------------------------------------ prefill launchers

// Shared-memory layout of a prefill CTA: barriers, the four staggered weight
// tiles (gx_stack's bank-group offsets), two activation chunks.
uint32_t prefill_layout(PrefillParams & p) {
    if (p.K % 256 != 0 || p.nb01 % 16 != 0 || p.al.pitch % 16 != 0) return 0;
    static const int xs[4] = {0, 1, 4, 5};
    const uint64_t tile = 4ull * (uint64_t)p.nb01;
    p.tile[0] = 0;
    for (int t = 1; t < 4; ++t) {
        uint64_t c = (p.tile[t - 1] + tile + 15) / 16;
        while (c % 8 != (uint64_t)xs[t]) ++c;
        p.tile[t] = (int32_t)(c * 16);
    }
    const uint64_t wbytes = (uint64_t)p.tile[3] + tile;
    p.act_off = align_up(128 + wbytes, 128);
    const uint64_t total = (uint64_t)p.act_off + 2ull * kPrefillChunk * (uint64_t)p.al.pitch;
    return total <= kMaxSmem ? (uint32_t)total : 0;
}

template <int MODE>
static cudaError_t launch_prefill_t(const PrefillParams & p, uint32_t smem, cudaStream_t stream) {
    static int configured = 0;   // per instantiation
    if ((int)smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(k_prefill<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured = (int)smem;
    }
    if (p.n_units <= 0) return cudaSuccess;
    k_prefill<MODE><<<p.n_units, 32 * kPrefillWarps, smem, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_mma_bprep(const MmaPrepParams & p, int n_chunks, cudaStream_t stream) {
    if (n_chunks <= 0) return cudaSuccess;
    k_mma_bprep<<<dim3((unsigned)p.nblk, (unsigned)n_chunks), kMmaN, 0, stream>>>(p);
    return cudaGetLastError();
}

template <int MODE>
static cudaError_t launch_prefill_mma_t(const MmaParams & p, int n_units, cudaStream_t stream) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [] {
        attr_err = cudaFuncSetAttribute(k_prefill_mma<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)MmaSmem::total);
    });
    if (attr_err != cudaSuccess) return attr_err;
    k_prefill_mma<MODE><<<(unsigned)n_units, kMmaThreads, MmaSmem::total, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_prefill_mma(int mode, const MmaParams & p, int n_units, cudaStream_t stream) {
    if (n_units <= 0) return cudaSuccess;
    return mode == 0 ? launch_prefill_mma_t<0>(p, n_units, stream) : launch_prefill_mma_t<1>(p, n_units, stream);
}

bool prefill_mma_supported(int type_gate, int type_down, int64_t H, int64_t I) {
    return type_gate == GX_T_Q8_0 && type_down == GX_T_Q8_0 && H % 256 == 0 && I % 256 == 0 && H <= 32 * kMmaMaxBlocks &&
           I <= 32 * kMmaMaxBlocks && I % 64 == 0 && H % kMmaRows == 0;
}

cudaError_t launch_prefill(int mode, const PrefillParams & p, uint32_t smem, cudaStream_t stream) {
    return mode == 0 ? launch_prefill_t<0>(p, smem, stream) : launch_prefill_t<1>(p, smem, stream);
}

ActLayout act_layout_host(int vdt, int n) { return act_layout(vdt, n); }

cudaError_t read_and_clear_device_error(int * code) {
    int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(code, g_dev_error, sizeof(int));
    if (e != cudaSuccess) return e;
    return cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(int));
}

}  // namespace gx
