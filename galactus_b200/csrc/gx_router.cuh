// Router on the device: logits -> selected expert ids, weights (and slots).
//
// Upstream llama.cpp's build_moe_ffn computes, per token, probs from the
// router logits (softmax, sigmoid, or the logits themselves for gpt-oss's
// softmax-over-selected), adds the selection bias, optionally keeps the best
// expert groups, takes the first k of the descending argsort, gathers the
// weights and normalises or scales them (the reference's remap node consumes
// that selection, patches/galactus-h4-llamacpp.diff:2124-2150). One warp per
// (layer, token) row; the row lives in shared memory. Every float operation
// is an explicit IEEE intrinsic in the oracle's order (oracle/gx_oracle.cpp,
// orc_router), so ids and weights agree bit for bit:
//   soft_max  e = exp(x - max) with the library's expf; float sums of four
//             consecutive e's ((e0+e1)+(e2+e3)); those sums and the tail
//             accumulated in double, in order, by lane 0 (a sequential sum is
//             the arithmetic being matched; the row is at most 1024 values);
//             every e times (float)(1.0/sum);
//   top-k     k rounds of a warp arg-max under one total order (score
//             descending, lower id first), so the butterfly reduction agrees
//             with the oracle's linear scan;
//   groups    per group the two best scores by a warp merge of (best,
//             second) pairs, summed once; the best groups by the same arg-max.
// Memory: reads E floats of logits per row, writes 2k-3k words; the kernel
// is latency-bound (a few microseconds for a 48-layer decode step).
#pragma once

#include <cstdint>

#include "gx_device.cuh"
#include "gx_kernels.h"

namespace gx {

struct RouterParams {
    const float * logits;
    int64_t ld;
    const float * bias;      // [n_layers, E] or null
    const int32_t * table;   // [n_layers, E] or null
    int32_t * ids;
    float * w;
    int32_t * slots;
    int64_t rows, T;
    int E, k, gating, groups, group_used, norm, scale_on;
    float scale;
};

// shared floats per warp: probs[E], sel[E], chunk sums[E/4], weights[32]
__host__ __device__ inline int router_smem_floats(int E) { return 2 * E + E / 4 + kRouterMaxUsed; }

__device__ __forceinline__ bool rt_better(float a, int ia, float b, int ib) { return a > b || (a == b && ia < ib); }

// arg-max of (v, i) over the warp under rt_better; i < 0 marks "none"
__device__ __forceinline__ void rt_warp_argmax(float & v, int & i) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, off);
        const int oi = __shfl_xor_sync(0xffffffffu, i, off);
        if (oi >= 0 && (i < 0 || rt_better(ov, oi, v, i))) {
            v = ov;
            i = oi;
        }
    }
}

// soft_max of n values x -> y (may alias) in shared memory, one warp
__device__ __forceinline__ void rt_soft_max(const float * x, float * y, float * csum, int n, int lane) {
    float m = -__int_as_float(0x7f800000);
    for (int j = lane; j < n; j += 32) m = fmaxf(m, x[j]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    for (int j = lane; j < n; j += 32) y[j] = gx_expf(__fsub_rn(x[j], m));
    __syncwarp();
    const int nc = n >> 2;
    for (int c = lane; c < nc; c += 32)
        csum[c] = __fadd_rn(__fadd_rn(y[4 * c], y[4 * c + 1]), __fadd_rn(y[4 * c + 2], y[4 * c + 3]));
    __syncwarp();
    float inv = 0.0f;
    if (lane == 0) {
        double s = 0.0;
        for (int c = 0; c < nc; ++c) s = __dadd_rn(s, (double)csum[c]);
        for (int j = 4 * nc; j < n; ++j) s = __dadd_rn(s, (double)y[j]);
        inv = __double2float_rn(__ddiv_rn(1.0, s));
    }
    inv = __shfl_sync(0xffffffffu, inv, 0);
    for (int j = lane; j < n; j += 32) y[j] = __fmul_rn(y[j], inv);
    __syncwarp();
}

__global__ void __launch_bounds__(32 * kRouterWarps) k_router(const RouterParams p) {
    extern __shared__ float rt_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kRouterWarps + warp;
    if (row >= p.rows) return;
    const int E = p.E, k = p.k;
    float * probs = rt_smem + (size_t)warp * router_smem_floats(E);
    float * sel = probs + E;
    float * csum = sel + E;
    float * wbuf = csum + E / 4;
    const int64_t layer = row / p.T;
    const float * x = p.logits + row * p.ld;

    for (int j = lane; j < E; j += 32) {
        const float v = x[j];
        probs[j] = p.gating == 1 ? __fdiv_rn(1.0f, __fadd_rn(1.0f, gx_expf(-v))) : v;
    }
    __syncwarp();
    if (p.gating == 0) rt_soft_max(probs, probs, csum, E, lane);
    const float * b = p.bias ? p.bias + layer * E : nullptr;
    for (int j = lane; j < E; j += 32) sel[j] = b ? __fadd_rn(probs[j], b[j]) : probs[j];
    __syncwarp();

    if (p.groups > 1) {
        const int G = p.groups, gs = E / G;
        float gscore = 0.0f;   // lane g holds group g's score
        for (int g = 0; g < G; ++g) {
            float t1 = -__int_as_float(0x7f800000), t2 = t1;
            for (int j = lane; j < gs; j += 32) {
                const float v = sel[g * gs + j];
                if (v > t1) {
                    t2 = t1;
                    t1 = v;
                } else if (v > t2) {
                    t2 = v;
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const float o1 = __shfl_xor_sync(0xffffffffu, t1, off);
                const float o2 = __shfl_xor_sync(0xffffffffu, t2, off);
                const float n1 = fmaxf(t1, o1);
                t2 = fmaxf(fminf(t1, o1), fmaxf(t2, o2));
                t1 = n1;
            }
            if (lane == g) gscore = __fadd_rn(t1, t2);
        }
        bool keep = false;
        for (int r = 0; r < p.group_used; ++r) {
            float v = gscore;
            int i = (lane < G && !keep) ? lane : -1;
            rt_warp_argmax(v, i);
            if (lane == i) keep = true;
        }
        const uint32_t kept = __ballot_sync(0xffffffffu, keep);
        for (int j = lane; j < E; j += 32)
            if (!((kept >> (j / gs)) & 1u)) sel[j] = -__int_as_float(0x7f800000);
        __syncwarp();
    }

    uint32_t taken = 0;   // bit i: element lane + 32 i
    int my_id = -1;
    for (int r = 0; r < k; ++r) {
        float v = 0.0f;
        int i = -1;
        for (int s = 0, j = lane; j < E; ++s, j += 32) {
            if ((taken >> s) & 1u) continue;
            const float c = sel[j];
            if (i < 0 || rt_better(c, j, v, i)) {
                v = c;
                i = j;
            }
        }
        rt_warp_argmax(v, i);
        if ((i & 31) == lane) taken |= 1u << (i >> 5);
        if (lane == r) my_id = i;
    }
    if (lane < k) wbuf[lane] = probs[my_id];
    __syncwarp();
    if (p.gating == 2) rt_soft_max(wbuf, wbuf, csum, k, lane);
    float wv = lane < k ? wbuf[lane] : 0.0f;
    if (p.norm) {
        float sf = 0.0f;
        if (lane == 0) {
            double s = 0.0;
            for (int r = 0; r < k; ++r) s = __dadd_rn(s, (double)wbuf[r]);
            sf = __double2float_rn(s);
            sf = sf > 6.103515625e-5f ? sf : 6.103515625e-5f;
        }
        sf = __shfl_sync(0xffffffffu, sf, 0);
        wv = __fdiv_rn(wv, sf);
    }
    if (p.scale_on) wv = __fmul_rn(wv, p.scale);
    if (lane < k) {
        const int64_t o = row * k + lane;
        p.ids[o] = my_id;
        p.w[o] = wv;
        if (p.table) {
            const int32_t s = p.table[layer * E + my_id];
            if (s < 0) record_error(GX_DEVERR_DOMAIN);
            p.slots[o] = s;
        }
    }
}

}  // namespace gx
