// Expert-grouped kernels for micro-batches with many tokens per expert
// (prefill), Q8_0 weights and activations (sm_100a).
//
// The host sorts the micro-batch's (token, slot) pairs by slot. A CTA takes
// one (slot, row tile): it stages the tile's weight rows in shared memory once
// (four bulk copies of four rows, at the staggered offsets of the stack
// kernel, so 16-byte loads of a quarter warp hit distinct bank groups) and
// then streams the slot's activation rows through a double-buffered chunk of
// 16 rows (one bulk copy per row, gathered by index). Each warp takes four
// activation rows of a chunk; each lane owns one weight row at one block
// parity and keeps the four NEON accumulator chains of every one of its four
// rows in registers, so a weight block is loaded and realigned once and used
// for four rows. The float tail is the decode kernels' (diff:1049-1054 chain
// order), so results are bit-identical to them and to the oracle.
//   MODE 0 (gate/up): 8 gate + 8 up rows per tile; output act f32 [pair, I]
//                     (SwiGLU / SWIGLU_OAI of the gate/up pair).
//   MODE 1 (down):    16 down rows per tile; output y f32 [pair, H].
#pragma once

#include <cstdint>

#include "gx_stack.cuh"

namespace gx {

constexpr int kPrefillNT = 4;        // activation rows per warp per chunk
constexpr int kPrefillWarps = 4;
constexpr int kPrefillChunk = kPrefillNT * kPrefillWarps;

template <int MODE>
__global__ void __launch_bounds__(32 * kPrefillWarps) k_prefill(const PrefillParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t * wbar = reinterpret_cast<uint64_t *>(smem);
    uint64_t * abar = wbar + 1;   // two chunk buffers
    uint8_t * wst = smem + 128;
    uint8_t * abuf = smem + p.act_off;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int u = blockIdx.x;
    if (u >= p.n_units) return;
    const int slot = p.unit_slot[u], r0 = p.unit_row0[u];
    const int s0 = p.seg_start[slot], ns = p.seg_start[slot + 1] - s0;
    const int nchunks = (ns + kPrefillChunk - 1) / kPrefillChunk;
    const int apitch = p.al.pitch;

    if (tid == 0) {
        for (int i = 0; i < 3; ++i) mbar_init(wbar + i, 1);
        mbar_fence_init();
    }
    __syncthreads();
    // slot id checked before any load
    if (slot < 0 || slot >= p.n_as) {
        if (tid == 0) record_error(GX_DEVERR_DOMAIN);
        return;
    }
    auto issue_chunk = [&](int c) {
        const int base = c * kPrefillChunk;
        const int n = ns - base < kPrefillChunk ? ns - base : kPrefillChunk;
        uint8_t * dst = abuf + (c & 1) * kPrefillChunk * apitch;
        tma_expect(abar + (c & 1), (uint32_t)(n * apitch));
        for (int i = 0; i < n; ++i)
            tma_load(dst + i * apitch, p.aq + (int64_t)p.pair_src[s0 + base + i] * apitch, (uint32_t)apitch, abar + (c & 1));
    };
    if (tid == 0) {
        // 4 tiles of 4 rows: MODE 0 gate rows r0..r0+7 then up rows, MODE 1
        // down rows r0..r0+15
        const int64_t base = (int64_t)slot * p.nb02 + (int64_t)r0 * p.nb01;
        const uint32_t tile = (uint32_t)(4 * p.nb01);
        tma_expect(wbar, 4u * tile);
        for (int t = 0; t < 4; ++t) {
            const uint8_t * src = MODE == 0 ? (t < 2 ? p.w0 : p.w1) + base + (int64_t)(t & 1) * tile
                                            : p.w0 + base + (int64_t)t * tile;
            tma_load(wst + p.tile[t], src, tile, wbar);
        }
        if (nchunks > 0) issue_chunk(0);
        if (nchunks > 1) issue_chunk(1);
    }
    if (__syncthreads_or(!mbar_wait_bounded(wbar, 0))) {
        if (tid == 0) record_error(GX_DEVERR_TIMEOUT);
        return;
    }
    // lane = qr*8 + tl*2 + gp: row qr of tile tl, block parity gp
    const int qr = lane >> 3, tl = (lane >> 1) & 3, gp = lane & 1;
    const uint8_t * wrow = wst + p.tile[tl] + qr * (int)p.nb01 + 32 * gp;
    const uint32_t sh = 16u + 16u * (uint32_t)gp, dsh = 16u * (uint32_t)gp;
    const int nu = p.K / 64;

    for (int c = 0; c < nchunks; ++c) {
        if (__syncthreads_or(!mbar_wait_bounded(abar + (c & 1), (uint32_t)((c >> 1) & 1)))) {
            if (tid == 0) record_error(GX_DEVERR_TIMEOUT);
            return;
        }
        const int first = c * kPrefillChunk + warp * kPrefillNT;   // this warp's rows in the segment
        const int nrows = ns - first < kPrefillNT ? (ns - first > 0 ? ns - first : 0) : kPrefillNT;
        if (nrows > 0) {
            const uint8_t * ab = abuf + (c & 1) * kPrefillChunk * apitch + (warp * kPrefillNT) * apitch;
            float acc[kPrefillNT][4];
#pragma unroll
            for (int n = 0; n < kPrefillNT; ++n)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[n][j] = 0.0f;
            for (int u0 = 0; u0 < nu; u0 += 4) {
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    const int uu = u0 + cc;
                    const uint8_t * wb = wrow + 68 * u0 + 64 * cc;
                    const uint4 c0 = lds128(wb), c1 = lds128(wb + 16), c2 = lds128(wb + 32);
                    const uint32_t W[12] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w, c2.x, c2.y, c2.z, c2.w};
                    const float dx = h2f((uint16_t)((W[cc] >> dsh) & 0xffffu));
                    uint32_t q[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) q[i] = __funnelshift_rc(W[cc + i], W[cc + i + 1], sh);
#pragma unroll
                    for (int n = 0; n < kPrefillNT; ++n) {
                        if (n < nrows) {
                            const uint8_t * ar = ab + n * apitch;
                            const uint4 ya = lds128(ar + 32 * gp + 64 * uu), yb = lds128(ar + 32 * gp + 64 * uu + 16);
                            const uint32_t y[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
                            const float dy = h2f((uint16_t)((lds32(ar + p.al.d_off + 4 * uu) >> dsh) & 0xffffu));
                            const float dd = __fmul_rn(dx, dy);
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const int pj = dp4a(q[4 + j], y[4 + j], dp4a(q[j], y[j], 0));
                                acc[n][j] = __fmaf_rn((float)pj, dd, acc[n][j]);
                            }
                        }
                    }
                }
            }
#pragma unroll
            for (int n = 0; n < kPrefillNT; ++n) {
                const float dot = q8_0_finish_x1(acc[n]);
                if (n < nrows) {
                    const int64_t orow = p.pair_dst[s0 + first + n];
                    if (MODE == 0) {
                        const float up = __shfl_down_sync(0xffffffffu, dot, 4);
                        if (gp == 0 && tl < 2) {
                            const float a = p.act == 1 ? act_swiglu_oai(dot, up, p.alpha, p.limit) : act_swiglu(dot, up);
                            p.out[orow * p.out_ld + r0 + 4 * tl + qr] = a;
                        }
                    } else if (gp == 0) {
                        p.out[orow * p.out_ld + r0 + 4 * tl + qr] = dot;
                    }
                } else if (MODE == 0) {
                    (void)__shfl_down_sync(0xffffffffu, dot, 4);
                }
            }
        }
        __syncthreads();
        if (tid == 0 && c + 2 < nchunks) issue_chunk(c + 2);
    }
}

}  // namespace gx
