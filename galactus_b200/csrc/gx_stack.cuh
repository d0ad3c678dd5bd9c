// Persistent, warp-specialized decode kernel for a stack of routed-expert
// layers (sm_100a).
//
// One cooperative launch (one CTA per SM) runs every layer of a micro-batch
// whose slot ids are all known when it starts. The jobs of the stack form one
// global list in which the down jobs of layer L follow the gate/up jobs of
// layer L+skew:
//   [GU(0)] .. [GU(skew-1)] [GU(skew)] [D(0)] [GU(skew+1)] [D(1)] ... [D(NL-1)]
// and CTA b takes jobs b, b+G, b+2G, ... ; its j-th job uses ring stage j % C.
// Inside a CTA:
//   warps 0, 1    weight producers (even and odd jobs of the CTA, so that the
//                 per-job issue work of one thread is not the limit): as soon
//                 as a stage is released, bulk-TMA
//                 copies the expert rows of the CTA's next job into it (one
//                 lane per copy). Weights
//                 never depend on earlier jobs, so the HBM stream runs ahead
//                 across job, half-layer and layer boundaries;
//   warp 2        gate/up input producer: once per (layer, token) that the
//                 CTA's jobs need, waits until x_L is quantized and copies the
//                 row into buffer (L*T + t) % 2 (see stack_input_producer);
//   warp 3        down input producer: the same for the k activation rows of
//                 a token, once every Q8 block of them has been quantized;
//   warps 4..     consumers: warp c computes the jobs of stage c, releases the
//                 stage and the input buffer, then runs the job's epilogue
//                 (activation and its Q8 quantization, or the combine).
// The x_L quantization runs first, in the consumer warps of CTA L mod G. The
// layer table travels in the kernel parameters (constant bank), the slot ids
// are copied to shared memory at the start. After set-up there is no
// CTA-wide barrier: roles synchronize through mbarriers and counters.
//
// Deadlock freedom: a job waits only on jobs of an earlier half-layer; every
// CTA issues and computes its jobs in increasing order and all CTAs are
// resident (cooperative launch), so the smallest unfinished job can always
// run. Every wait is bounded, gives up as soon as any CTA has recorded an
// error, and on giving up records GX_DEVERR_TIMEOUT; producers then let their
// copies in flight land (bounded) before the CTA exits.
//
// IQ1_S rows use the octet row dots of the per-layer kernels (eight lanes per
// row, two rows per lane, gx_moe.cuh): a gate/up job is two passes over gate
// row i and up row i together (octet g takes i = 4*pass + g), a down job four
// passes over row pairs (2g, 2g+1) of one expert; the down dots go through a
// per-warp scratch to the combine. Their activations are Q8_K.
//
// MXFP4 rows (gpt-oss-shaped models): a job is 32 rows (16 gate + 16 up, or
// 32/k rows of each of the k experts), four warps per job. Lane r of each
// warp takes row r; warp `sub` computes the pair terms t_u of the pairs
// u = sub, sub+4, ... (every integer dot exact, each term in the reference's
// float order) and parks each term in a word of the stage that only its pair
// occupies; the job's last warp folds every row's terms in pair order,
// releases the stage and runs the epilogue. The Q8_0 activation rows these
// jobs read are stored in the codes' byte order.
//
// Q8_0 rows (the gate/up/down type of Q8_0 models): two lanes per weight row,
// one per block parity. Lane p owns the four NEON accumulator chains of the
// blocks 2u+p (diff:1049-1054: per-lane int32 partial of words j and 4+j,
// acc_j = fma((float)partial_j, dx*dy, acc_j)); a row's dot is
// ((e0+e1)+(e2+e3)) + ((o0+o1)+(o2+o3)), the faddp order. Each block is read
// as three aligned 16-byte shared loads and realigned with clamped funnel
// shifts, the same instruction sequence for both parities.
#pragma once

#include <cstdint>

#include "gx_moe.cuh"

namespace gx {

// generic-proxy global writes -> later bulk-TMA (async-proxy) reads
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint4 lds128(const uint8_t * p) { return *reinterpret_cast<const uint4 *>(p); }

// Release/acquire at GPU scope: orders this thread's (and, after a warp or
// CTA barrier, its peers') earlier accesses before its later ones. The
// publish/consume protocol of the kernel needs nothing stronger.
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Bounded wait until *p reaches target (the counters only grow).
__device__ __forceinline__ bool stack_wait(const int32_t * p, int32_t target) {
    for (uint32_t i = 0; i < (1u << 23); ++i) {
        if (*reinterpret_cast<const volatile int32_t *>(p) >= target) return true;
        if ((i & 15u) == 15u && *reinterpret_cast<volatile int *>(&g_dev_error) != 0) return false;
        if (i >= 8) __nanosleep(64);
    }
    return false;
}

// Bounded mbarrier wait that also stops once another CTA recorded an error.
// Each poll sleeps in the barrier for up to 0.5 us (it wakes when the phase
// completes), so waiting warps leave the issue slots to the working ones; the
// bound is 2^20 polls (about half a second).
__device__ __forceinline__ bool stack_mbar_wait(uint64_t * bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 20); ++i) {
        if (mbar_try_wait_sleep(bar, parity, 500u)) return true;
        if ((i & 63u) == 63u && *reinterpret_cast<volatile int *>(&g_dev_error) != 0) return false;
    }
    return false;
}

// One decoded job of the global list.
struct StackJob {
    int L, gu, t, r0, pair;
};

// Job-list geometry, copied once into registers by every role.
struct StackGeom {
    int NL, n_gu, n_d, skew, tiles_g, tiles_d, Rg, Rd, k;
};

__device__ __forceinline__ StackGeom stack_geom(const StackParams & p) {
    StackGeom g;
    g.NL = p.NL;
    g.n_gu = p.n_gu;
    g.n_d = p.n_d;
    g.skew = p.skew;
    g.tiles_g = p.I / p.Rg;
    g.tiles_d = p.H / p.Rd;
    g.Rg = p.Rg;
    g.Rd = p.Rd;
    g.k = p.k;
    return g;
}

__device__ __forceinline__ StackJob stack_job(const StackGeom & p, int j) {
    StackJob J;
    int w;
    const int d = p.skew;
    const int seg = p.n_gu + p.n_d;
    if (j < d * p.n_gu) {
        J.L = j / p.n_gu;
        J.gu = 1;
        w = j - J.L * p.n_gu;
    } else {
        const int jj = j - d * p.n_gu;
        const int full = p.NL - d;   // blocks [GU(B+d)][D(B)]
        if (jj < full * seg) {
            const int B = jj / seg;
            w = jj - B * seg;
            J.gu = w < p.n_gu;
            J.L = J.gu ? B + d : B;
            if (!J.gu) w -= p.n_gu;
        } else {
            const int jr = jj - full * seg;
            const int B = jr / p.n_d;
            J.L = full + B;
            J.gu = 0;
            w = jr - B * p.n_d;
        }
    }
    if (J.gu) {
        J.pair = w / p.tiles_g;
        J.r0 = (w - J.pair * p.tiles_g) * p.Rg;
        J.t = J.pair / p.k;
    } else {
        J.t = w / p.tiles_d;
        J.r0 = (w - J.t * p.tiles_d) * p.Rd;
        J.pair = J.t * p.k;
    }
    return J;
}

// Weight bases of one layer, kept in shared memory for the weight producer.
struct StackWeights {
    const uint8_t * wg;
    const uint8_t * wu;
    const uint8_t * wd;
    int64_t nb02;
};

// Row-copy geometry of the weight producer (registers).
struct StackCopy {
    int64_t nb01_g, nb01_d;
    int pitch_d, row_copy_d, T, k, Rg, Rd, gu_copies;
    int tile[4];
};

// The weight producer's walk over jobs b, b+G, b+2G, ... without divisions
// by the segment lengths: segments are GU(0) .. GU(skew-1), then
// [GU(B+skew)][D(B)] for B < NL-skew, then D(NL-skew) .. D(NL-1).
struct StackWalk {
    int seg, w;   // current segment and index inside it
    __device__ __forceinline__ void kind(const StackGeom & g, int & L, int & gu) const {
        const int d = g.skew, mid = 2 * (g.NL - d);
        if (seg < d) {
            L = seg;
            gu = 1;
        } else if (seg < d + mid) {
            const int k = seg - d;
            gu = (k & 1) == 0;
            L = gu ? (k >> 1) + d : (k >> 1);
        } else {
            L = g.NL - d + (seg - d - mid);
            gu = 0;
        }
    }
    __device__ __forceinline__ int len(const StackGeom & g) const {
        int L, gu;
        kind(g, L, gu);
        return gu ? g.n_gu : g.n_d;
    }
    __device__ __forceinline__ void advance(const StackGeom & g, int step) {
        w += step;
        for (int l = len(g); w >= l; l = len(g)) {
            w -= l;
            ++seg;
            if (seg >= g.skew + 2 * (g.NL - g.skew) + g.skew) break;
        }
    }
    __device__ __forceinline__ StackJob job(const StackGeom & g) const {
        StackJob J;
        kind(g, J.L, J.gu);
        if (J.gu) {
            J.pair = w / g.tiles_g;
            J.r0 = (w - J.pair * g.tiles_g) * g.Rg;
            J.t = J.pair / g.k;
        } else {
            J.t = w / g.tiles_d;
            J.r0 = (w - J.t * g.tiles_d) * g.Rd;
            J.pair = J.t * g.k;
        }
        return J;
    }
};

// Q8_0 x Q8_0 rows of one parity: NR rows, row r against activation row r,
// K/64 units (a multiple of four). rb[r] = row base + 32*p, ab[r] =
// activation quants + 32*p, ad[r] = activation scales.
template <int NR>
__device__ __forceinline__ void q8_0_rows(const uint8_t * const (&rb)[NR], const uint8_t * const (&ab)[NR],
                                          const uint8_t * const (&ad)[NR], int p, int nu, float (&acc)[NR][4]) {
    const uint32_t sh = 16u + 16u * (uint32_t)p;   // quants at +2 (even block) or word-aligned (odd block)
    const uint32_t dsh = 16u * (uint32_t)p;        // scale: low or high half of word c
    for (int u0 = 0; u0 < nu; u0 += 4) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int u = u0 + c;
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const uint4 ya = lds128(ab[r] + 64 * u), yb = lds128(ab[r] + 64 * u + 16);
                const uint32_t y[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
                const float dy = h2f((uint16_t)((lds32(ad[r] + 4 * u) >> dsh) & 0xffffu));
                // 16-byte aligned: 68u - 4c is a multiple of 16 for u = c mod 4
                const uint8_t * base = rb[r] + 68 * u0 + 64 * c;
                const uint4 c0 = lds128(base), c1 = lds128(base + 16), c2 = lds128(base + 32);
                const uint32_t W[12] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w, c2.x, c2.y, c2.z, c2.w};
                const float dx = h2f((uint16_t)((W[c] >> dsh) & 0xffffu));
                const float dd = __fmul_rn(dx, dy);
                uint32_t q[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) q[i] = __funnelshift_rc(W[c + i], W[c + i + 1], sh);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int pj = dp4a(q[4 + j], y[4 + j], dp4a(q[j], y[j], 0));
                    acc[r][j] = __fmaf_rn((float)pj, dd, acc[r][j]);
                }
            }
        }
    }
}

// the row's dot from the two parity lanes (lane and lane ^ 16)
__device__ __forceinline__ float q8_0_finish(const float (&a)[4]) {
    const float s = __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
    return __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 16));
}

// the same with the parity lanes adjacent (lane and lane ^ 1)
__device__ __forceinline__ float q8_0_finish_x1(const float (&a)[4]) {
    const float s = __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
    return __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));
}

// Weight copies of job J into a stage, issued by the 32 lanes of the weight
// producer warp: lane 0 arms the stage barrier with the job's bytes, then one
// lane per copy issues it (the copies of a job go out together). Slot ids and
// the layer's weight bases come from shared memory.
__device__ __forceinline__ void stack_issue_weights(const StackCopy & q, const StackJob & J, const int32_t * slots,
                                                    const StackWeights * wt, uint8_t * stage, uint64_t * bar, int lane) {
    const StackWeights ly = wt[J.L];
    const int32_t * sl = slots + J.L * q.T * q.k;
    if (J.gu) {
        const int64_t off = (int64_t)sl[J.pair] * ly.nb02 + (int64_t)J.r0 * q.nb01_g;
        if (q.gu_copies == 4) {
            // 4 tiles of 4 rows: gate rows r0..r0+3, r0+4..r0+7, then up rows
            const uint32_t tile = (uint32_t)(4 * q.nb01_g);
            if (lane == 0) tma_expect(bar, 4u * tile);
            __syncwarp();
            if (lane < 4)
                tma_load(stage + q.tile[lane], (lane < 2 ? ly.wg : ly.wu) + off + (int64_t)(lane & 1) * tile, tile, bar);
        } else {
            // gate rows r0..r0+Rg-1, then up rows r0..r0+Rg-1
            const uint32_t tile = (uint32_t)(q.Rg * q.nb01_g);
            if (lane == 0) tma_expect(bar, 2u * tile);
            __syncwarp();
            if (lane < 2) tma_load(stage + q.tile[lane], (lane == 0 ? ly.wg : ly.wu) + off, tile, bar);
        }
    } else {
        const uint32_t bytes = (uint32_t)(q.Rd * q.nb01_d);
        if (lane == 0) tma_expect(bar, (uint32_t)q.k * bytes);
        __syncwarp();
        if (q.row_copy_d) {
            for (int i = lane; i < q.k * q.Rd; i += 32) {
                const int m = i / q.Rd, r = i - m * q.Rd;
                tma_load(stage + (m * q.Rd + r) * q.pitch_d,
                         ly.wd + (int64_t)sl[J.pair + m] * ly.nb02 + (int64_t)(J.r0 + r) * q.nb01_d, (uint32_t)q.nb01_d, bar);
            }
        } else if (lane < q.k) {
            tma_load(stage + lane * q.Rd * q.pitch_d, ly.wd + (int64_t)sl[J.pair + lane] * ly.nb02 + (int64_t)J.r0 * q.nb01_d,
                     bytes, bar);
        }
    }
}

// unsigned-by-signed byte dot: a holds four unsigned bytes, b four signed
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// two signed 16-bit halves of a times bytes 0,1 (LO) or 2,3 (HI) of b, plus c
__device__ __forceinline__ int dp2a_lo(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// prmt in its generic mode: each selector nibble's low three bits pick a byte
// of {b:a}, its high bit replaces that byte by copies of the byte's sign bit
__device__ __forceinline__ uint32_t prmt_sx(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// e2m1 magnitudes of codes 0..7, doubled (0, 0.5, 1, 1.5, 2, 3, 4, 6 -> 0..12):
// bytes 0-3 and 4-7 of the prmt source pair
constexpr uint32_t kE2m1Lo = 0x03020100u, kE2m1Hi = 0x0c080604u;

// Exact dot of the 16 code bytes at words W0.. of w, shifted right by cs bits
// (a clamped funnel shift: cs = 32 takes the next word whole; code byte j
// holds elements j and j+16), with its Q8_0 activation block stored in code
// order (quant_block_split<..., PERM>: word 2t = elements 4t, 4t+16, 4t+1,
// 4t+17, word 2t+1 = 4t+2, 4t+18, 4t+3, 4t+19). prmt in its default mode
// takes a selector nibble's low three bits as the byte index and its high bit
// as "replace the byte by copies of its sign bit"; the table bytes are
// non-negative, so prmt(table, q) gives the magnitudes of the positive codes
// and zero for the negative ones, and prmt(table, q ^ 0x8888...) the
// reverse. dot = dp4a(positive mags, a) - dp4a(negative mags, a), exact.
template <int W0>
__device__ __forceinline__ int mxfp4_codes_dot(const uint32_t (&w)[9], uint32_t cs, const uint4 & a0, const uint4 & a1) {
    const uint32_t aw[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    int pp0 = 0, pp1 = 0, pn0 = 0, pn1 = 0;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint32_t q = __funnelshift_rc(w[W0 + t], w[W0 + t + 1], cs);
        const uint32_t qx = q ^ 0x88888888u;
        pp0 = dp4a(prmt_sx(kE2m1Lo, kE2m1Hi, q), aw[2 * t], pp0);
        pn0 = dp4a(prmt_sx(kE2m1Lo, kE2m1Hi, qx), aw[2 * t], pn0);
        pp1 = dp4a(prmt_sx(kE2m1Lo, kE2m1Hi, q >> 16), aw[2 * t + 1], pp1);
        pn1 = dp4a(prmt_sx(kE2m1Lo, kE2m1Hi, qx >> 16), aw[2 * t + 1], pn1);
    }
    return (pp0 + pp1) - (pn0 + pn1);
}

// The term of block pair u of one MXFP4 row (ggml_vec_dot_mxfp4_q8_0's
// t = fma(sc_e, p_e, sc_o*p_o), diff:1209-1240), computed by one lane from the
// pair's 34 bytes at `pr` (an even byte offset: row pitches and pair sizes are
// even), read as nine aligned words, against the activation pair at `ap`
// (64 quants in code order) and its two fp16 scales in word `dw`.
__device__ __forceinline__ float mxfp4_pair_term(const uint8_t * pr, const uint8_t * ap, uint32_t dw) {
    const uintptr_t P = reinterpret_cast<uintptr_t>(pr);
    const uint8_t * wp = reinterpret_cast<const uint8_t *>(P & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(P & 3) * 8u;   // 0 or 16
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = lds32(wp + 4 * i);
    const uint4 a0 = lds128(ap), a1 = lds128(ap + 16), a2 = lds128(ap + 32), a3 = lds128(ap + 48);
    // even block: scale at byte sh/8, codes from byte sh/8 + 1; odd block:
    // scale at byte 17 + sh/8 (word 4), codes from byte 18 + sh/8
    const int pe = mxfp4_codes_dot<0>(w, sh + 8u, a0, a1);
    const int po = mxfp4_codes_dot<4>(w, sh + 16u, a2, a3);
    const float sce = __fmul_rn(h2f((uint16_t)(dw & 0xffffu)), e8m0_half((w[0] >> sh) & 0xffu));
    const float sco = __fmul_rn(h2f((uint16_t)(dw >> 16)), e8m0_half((w[4] >> (sh + 8u)) & 0xffu));
    return __fmaf_rn(sce, (float)pe, __fmul_rn(sco, (float)po));
}

// Where a lane parks the term of pair u: a word strictly inside the pair's
// own bytes that no other pair's nine-word window touches (windows reach at
// most two bytes past their pair), so the stage holds the terms once the
// pair has been read.
__device__ __forceinline__ float * mxfp4_term_slot(const uint8_t * pr) {
    const uintptr_t P = reinterpret_cast<uintptr_t>(pr);
    return reinterpret_cast<float *>(((P + 3) & ~(uintptr_t)3) + 4);
}

// Part `sub` of a 32-row MXFP4 job (`split` parts): lane r takes row r
// (base row_r) and the pairs u = sub, sub + split, ... of it, and parks each
// pair's term in the stage. act(r) is the row's activation row.
__device__ __forceinline__ void mxfp4_rows_part(const uint8_t * row_r, const uint8_t * act_r, const ActLayout & al,
                                                int npairs, int sub, int split) {
    const uint8_t * ad = act_r + al.d_off;
#pragma unroll 2
    for (int u = sub; u < npairs; u += split) {
        const float t = mxfp4_pair_term(row_r + 34 * u, act_r + 64 * u, lds32(ad + 4 * u));
        *mxfp4_term_slot(row_r + 34 * u) = t;
    }
}

// The row's dot: its pair terms folded in pair order (the reference chain sumf += t).
__device__ __forceinline__ float mxfp4_rows_fold(const uint8_t * row_r, int npairs) {
    float sumf = 0.0f;
    int u = 0;
    for (; u + 8 <= npairs; u += 8) {   // eight loads in flight, then the chain
        float t[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) t[i] = *mxfp4_term_slot(row_r + 34 * (u + i));
#pragma unroll
        for (int i = 0; i < 8; ++i) sumf = __fadd_rn(sumf, t[i]);
    }
    for (; u < npairs; ++u) sumf = __fadd_rn(sumf, *mxfp4_term_slot(row_r + 34 * u));
    return sumf;
}

// async-proxy (bulk copy) writes after generic-proxy accesses of shared memory
__device__ __forceinline__ void fence_proxy_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Superblocks whose integer parts a lane computes before their exchanges and
// float chain (Q4_K rows), and whether Q6_K rows go by superblock pairs.
constexpr int kQ4kGroup = 1;
constexpr bool kQ6kPairs = true;

// the exact integer parts of one Q4_K superblock half (see q4k_row2)
__device__ __forceinline__ void q4k_half(const uint8_t * xb, const uint8_t * aq, const uint8_t * bsp, uint32_t sel,
                                         int p, int & sumi, int & prod, uint32_t & dm) {
    const uint4 hdr = lds128(xb);   // d | dmin, scale bytes 0-3, 4-7, 8-11
    dm = hdr.x;
    const uint32_t sc_lo = hdr.y & 0x3f3f3f3fu;
    const uint32_t sc_hi = (hdr.w & 0x0f0f0f0fu) | ((hdr.y >> 2) & 0x30303030u);
    const uint32_t mn_lo = hdr.z & 0x3f3f3f3fu;
    const uint32_t mn_hi = ((hdr.w >> 4) & 0x0f0f0f0fu) | ((hdr.z >> 2) & 0x30303030u);
    int si = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint4 q = lds128(xb + 16 + 32 * j + 16 * p);
        const uint4 lo = lds128(aq + 64 * j);
        const uint4 hi = lds128(aq + 64 * j + 32);
        int p1 = dp4a(q.x & 0x0f0f0f0fu, lo.x, 0);
        p1 = dp4a(q.y & 0x0f0f0f0fu, lo.y, p1);
        p1 = dp4a(q.z & 0x0f0f0f0fu, lo.z, p1);
        p1 = dp4a(q.w & 0x0f0f0f0fu, lo.w, p1);
        int p2 = dp4a_us(q.x & 0xf0f0f0f0u, hi.x, 0);
        p2 = dp4a_us(q.y & 0xf0f0f0f0u, hi.y, p2);
        p2 = dp4a_us(q.z & 0xf0f0f0f0u, hi.z, p2);
        p2 = dp4a_us(q.w & 0xf0f0f0f0u, hi.w, p2);
        p2 >>= 4;
        const uint32_t sw = j < 2 ? sc_lo : sc_hi;
        const int s0 = (int)((sw >> (16 * (j & 1))) & 0xffu), s1 = (int)((sw >> (16 * (j & 1) + 8)) & 0xffu);
        si += p1 * s0 + p2 * s1;
    }
    uint32_t bw[8];
#pragma unroll
    for (int o = 0; o < 8; ++o) bw[o] = lds32(bsp + 4 * o);
    int pr = dp2a_lo(__byte_perm(bw[0], bw[1], sel), mn_lo, 0);
    pr = dp2a_hi(__byte_perm(bw[2], bw[3], sel), mn_lo, pr);
    pr = dp2a_lo(__byte_perm(bw[4], bw[5], sel), mn_hi, pr);
    pr = dp2a_hi(__byte_perm(bw[6], bw[7], sel), mn_hi, pr);
    sumi = si;
    prod = pr;
}

// Q4_K row x Q8_K activation row (split layout), two lanes per row
// (ggml_vec_dot_q4_K_q8_K, diff:1254-1259, 1300-1357). Lane half p takes
// bytes 16p..16p+15 of every 32-byte quant group j, i.e. the 16-element runs
// 64j+16p.. (low nibbles, sub-block 2j) and 64j+32+16p.. (high nibbles,
// sub-block 2j+1), and the block sums bs[2o+p] of the mins. The high nibbles
// are dotted in place (byte & 0xf0, unsigned) and the sum shifted down by 4,
// exact since every term is a multiple of 16. The six-bit scales and mins of
// the 12-byte packing are unpacked four at a time; the mins meet the 16-bit
// block sums in dp2a. The exact integer parts of a superblock are summed with
// the partner lane (lane ^ xm), then both lanes run the superblock chain:
//   sumf = fma(-(yd*fp16(dmin)), prod, sumf); sumf = fma(yd*fp16(d), sumi, sumf).
__device__ __forceinline__ float q4k_row2(const uint8_t * row, const uint8_t * act, const ActLayout & al, int p, int nsb,
                                          int xm) {
    float sumf = 0.0f;
    const uint8_t * aq = act + 16 * p;
    const uint32_t sel = p ? 0x7632u : 0x5410u;   // half p of two block-sum words
    int i = 0;
    // kQ4kGroup superblocks' integer parts first (independent), then their
    // exchanges, then the chain in superblock order
    constexpr int NG = kQ4kGroup;
    for (; NG > 1 && i + NG <= nsb; i += NG) {
        int si[NG], pr[NG];
        uint32_t dm[NG];
#pragma unroll
        for (int k = 0; k < NG; ++k)
            q4k_half(row + 144 * (i + k), aq + 256 * (i + k), act + al.bs_off + 32 * (i + k), sel, p, si[k], pr[k], dm[k]);
#pragma unroll
        for (int k = 0; k < NG; ++k) {
            si[k] += __shfl_xor_sync(0xffffffffu, si[k], xm);
            pr[k] += __shfl_xor_sync(0xffffffffu, pr[k], xm);
        }
#pragma unroll
        for (int k = 0; k < NG; ++k) {
            const float yd = __uint_as_float(lds32(act + al.d_off + 4 * (i + k)));
            sumf = __fmaf_rn(-__fmul_rn(yd, h2f((uint16_t)(dm[k] >> 16))), (float)pr[k], sumf);
            sumf = __fmaf_rn(__fmul_rn(yd, h2f((uint16_t)(dm[k] & 0xffffu))), (float)si[k], sumf);
        }
    }
    for (; i < nsb; ++i) {
        int si, pr;
        uint32_t dm;
        q4k_half(row + 144 * i, aq + 256 * i, act + al.bs_off + 32 * i, sel, p, si, pr, dm);
        si += __shfl_xor_sync(0xffffffffu, si, xm);
        pr += __shfl_xor_sync(0xffffffffu, pr, xm);
        const float yd = __uint_as_float(lds32(act + al.d_off + 4 * i));
        sumf = __fmaf_rn(-__fmul_rn(yd, h2f((uint16_t)(dm >> 16))), (float)pr, sumf);
        sumf = __fmaf_rn(__fmul_rn(yd, h2f((uint16_t)(dm & 0xffffu))), (float)si, sumf);
    }
    return sumf;
}

// N consecutive words at wb + off (wb 4-byte aligned) shifted right by SH bits
template <int N, int SH>
__device__ __forceinline__ void lds_words(const uint8_t * wb, int off, uint32_t (&out)[N]) {
    if constexpr (SH == 0) {
#pragma unroll
        for (int k = 0; k < N; ++k) out[k] = lds32(wb + off + 4 * k);
    } else {
        uint32_t w0 = lds32(wb + off);
#pragma unroll
        for (int k = 0; k < N; ++k) {
            const uint32_t w1 = lds32(wb + off + 4 * (k + 1));
            out[k] = __funnelshift_r(w0, w1, SH);
            w0 = w1;
        }
    }
}

// One Q6_K superblock half of one row (see q6k_rows2); SH = 0 for a
// word-aligned superblock, 16 for one two bytes off.
template <int SH>
__device__ __forceinline__ void q6k_half(const uint8_t * wb, const uint8_t * aq, const uint8_t * bsp, int p,
                                         int & isum, int & mins, uint32_t & dw) {
    uint32_t sc4[4], dd[1];
    lds_words<4, SH>(wb, 192, sc4);
    lds_words<1, SH>(wb, 208, dd);
    dw = dd[0];
    isum = 0;
    mins = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        uint32_t ql[8], qh[8];
        lds_words<8, SH>(wb, 64 * h + 32 * p, ql);
        lds_words<8, SH>(wb, 128 + 32 * h, qh);
        uint32_t aw[2][8];
#pragma unroll
        for (int odd = 0; odd < 2; ++odd) {
            const uint8_t * ap = aq + 64 * (2 * h + odd);
            const uint4 a0 = lds128(ap), a1 = lds128(ap + 16);
            aw[odd][0] = a0.x; aw[odd][1] = a0.y; aw[odd][2] = a0.z; aw[odd][3] = a0.w;
            aw[odd][4] = a1.x; aw[odd][5] = a1.y; aw[odd][6] = a1.z; aw[odd][7] = a1.w;
        }
        int pg[2][2] = {{0, 0}, {0, 0}};
#pragma unroll
        for (int ww = 0; ww < 8; ++ww) {
            const uint32_t hp = qh[ww] >> (2 * p);   // the two bits of half p at 0-1 (odd 0) and 4-5 (odd 1)
            const uint32_t q0 = (ql[ww] & 0x0f0f0f0fu) | ((hp << 4) & 0x30303030u);
            const uint32_t q1 = ((ql[ww] >> 4) & 0x0f0f0f0fu) | (hp & 0x30303030u);
            pg[0][ww >> 2] = dp4a(q0, aw[0][ww], pg[0][ww >> 2]);
            pg[1][ww >> 2] = dp4a(q1, aw[1][ww], pg[1][ww >> 2]);
        }
#pragma unroll
        for (int odd = 0; odd < 2; ++odd) {
            const int j = 2 * h + odd;
            // groups 4j+2p and 4j+2p+1: scale bytes 4j+2p, 4j+2p+1
            const uint32_t sw = sc4[j] >> (16 * p);
            const int s0 = (int)(int8_t)(sw & 0xffu), s1 = (int)(int8_t)((sw >> 8) & 0xffu);
            const uint32_t bw = lds32(bsp + 8 * j + 4 * p);
            isum += pg[odd][0] * s0 + pg[odd][1] * s1;
            mins += (int)(int16_t)(bw & 0xffffu) * s0 + (int)(int16_t)(bw >> 16) * s1;
        }
    }
}

// Two Q6_K rows x their Q8_K activation rows (split layout), two lanes per
// row (ggml_vec_dot_q6_K_q8_K, diff:1366-1370, 1393-1446). Lane half p takes
// the 32-element half p of every 64-element quarter j: groups 4j+2p and
// 4j+2p+1, quants ql bytes 64(j/2)+32p.. (nibble 4*(j&1)) with qh bytes
// 128+32(j/2).. (bits 4*(j&1)+2p). Superblocks are 210 bytes, so the odd ones
// sit two bytes off a word and are realigned with funnel shifts. isum and mins
// are summed with the partner lane (lane ^ xm), then per superblock
// sumf = fma(yd*fp16(d), isum - 32*mins, sumf). The two rows run in one loop.
template <int NR>
__device__ __forceinline__ void q6k_rows2(const uint8_t * row0, const uint8_t * row1, const uint8_t * act0,
                                          const uint8_t * act1, const ActLayout & al, int p, int nsb, int xm,
                                          float & d0, float & d1) {
    const uint8_t * rows[2] = {row0, row1};
    const uint8_t * acts[2] = {act0, act1};
    float sums[2] = {0.0f, 0.0f};
    int i = 0;
    if constexpr (!kQ6kPairs) {
        for (; i < nsb; ++i) {
            const int off = (210 * i) & ~3;
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                int is, mn;
                uint32_t dw;
                if (i & 1)
                    q6k_half<16>(rows[r] + off, acts[r] + 256 * i + 32 * p, acts[r] + al.bs_off + 32 * i, p, is, mn, dw);
                else
                    q6k_half<0>(rows[r] + off, acts[r] + 256 * i + 32 * p, acts[r] + al.bs_off + 32 * i, p, is, mn, dw);
                is += __shfl_xor_sync(0xffffffffu, is, xm);
                mn += __shfl_xor_sync(0xffffffffu, mn, xm);
                const float yd = __uint_as_float(lds32(acts[r] + al.d_off + 4 * i));
                sums[r] = __fmaf_rn(__fmul_rn(yd, h2f((uint16_t)(dw & 0xffffu))), (float)(is - 32 * mn), sums[r]);
            }
        }
    }
    // superblock pairs: the even one is word-aligned, the odd one two bytes off
    for (; i + 2 <= nsb; i += 2) {
        int is[2][2], mn[2][2];
        uint32_t dw[2][2];
        const int off0 = 210 * i, off1 = (210 * (i + 1)) & ~3;
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            q6k_half<0>(rows[r] + off0, acts[r] + 256 * i + 32 * p, acts[r] + al.bs_off + 32 * i, p, is[r][0], mn[r][0],
                        dw[r][0]);
            q6k_half<16>(rows[r] + off1, acts[r] + 256 * (i + 1) + 32 * p, acts[r] + al.bs_off + 32 * (i + 1), p,
                         is[r][1], mn[r][1], dw[r][1]);
        }
#pragma unroll
        for (int r = 0; r < NR; ++r)
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                is[r][k] += __shfl_xor_sync(0xffffffffu, is[r][k], xm);
                mn[r][k] += __shfl_xor_sync(0xffffffffu, mn[r][k], xm);
            }
#pragma unroll
        for (int r = 0; r < NR; ++r)
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const float yd = __uint_as_float(lds32(acts[r] + al.d_off + 4 * (i + k)));
                sums[r] = __fmaf_rn(__fmul_rn(yd, h2f((uint16_t)(dw[r][k] & 0xffffu))), (float)(is[r][k] - 32 * mn[r][k]),
                                    sums[r]);
            }
    }
    if (i < nsb) {   // a last even superblock
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            int is, mn;
            uint32_t dw;
            q6k_half<0>(rows[r] + 210 * i, acts[r] + 256 * i + 32 * p, acts[r] + al.bs_off + 32 * i, p, is, mn, dw);
            is += __shfl_xor_sync(0xffffffffu, is, xm);
            mn += __shfl_xor_sync(0xffffffffu, mn, xm);
            const float yd = __uint_as_float(lds32(acts[r] + al.d_off + 4 * i));
            sums[r] = __fmaf_rn(__fmul_rn(yd, h2f((uint16_t)(dw & 0xffffu))), (float)(is - 32 * mn), sums[r]);
        }
    }
    d0 = sums[0];
    d1 = sums[1];
}

// Octet gate/up job: gate row i and up row i (octet g, i = 4*pass + g)
// against the token's activation row; every lane of octet g ends with the
// two dots of row 4*pass + g. Passes ps0, ps0 + pstep, ... (a split job's
// warps take every pstep-th pass).
template <int TYPE>
__device__ __forceinline__ typename Oct<TYPE>::A oct_act(const uint8_t * ar, const ActLayout & L, int o,
                                                        const uint2 * grid) {
    if constexpr (TYPE == GX_T_IQ1_S) return Oct<TYPE>::inita(ar, L, o, grid);
    else return Oct<TYPE>::inita(ar, L, o);
}

template <int TYPE>
__device__ __forceinline__ void stack_gu_oct(const StackParams & p, const uint8_t * st, const uint8_t * xa, int lane,
                                             float (&gd)[2], float (&ud)[2], int ps0, int pstep, const uint2 * grid) {
    using Q = Oct<TYPE>;
    const int o = lane & 7, g = lane >> 3;
    const int U = p.H / Q::UNIT;
    const typename Q::A al = oct_act<TYPE>(xa, p.alx, o, grid);
    for (int ps = ps0; ps < 2; ps += pstep) {
        const int row = 4 * ps + g;
        typename Q::St acc[2];
        const typename Q::W wl[2] = {Q::initw(st, p.gu_tile[0] + row * (int)p.nb01_g, o),
                                     Q::initw(st, p.gu_tile[1] + row * (int)p.nb01_g, o)};
        int v = 0;
        for (; v + 1 < U; v += 2) {
            Q::template unit<0>(wl, al, v, acc);
            Q::template unit<1>(wl, al, v + 1, acc);
        }
        if (v < U) Q::template unit<0>(wl, al, v, acc);
        gd[ps] = Q::finish(acc[0]);
        ud[ps] = Q::finish(acc[1]);
    }
}

// Octet down job: k*Rd rows in passes of eight; octet g takes rows
// 8*pass + 2g and 8*pass + 2g + 1 (one expert, Rd even) against that
// expert's activation row; lane 8g writes both dots to dots[row].
template <int TYPE>
__device__ __forceinline__ void stack_d_oct(const StackParams & p, const uint8_t * st, const uint8_t * da, int lane,
                                            float * dots, int ps0, int pstep, const uint2 * grid) {
    using Q = Oct<TYPE>;
    const int o = lane & 7, g = lane >> 3;
    const int U = p.I / Q::UNIT;
    const int passes = p.k * p.Rd / 8;
    for (int ps = ps0; ps < passes; ps += pstep) {
        const int row = 8 * ps + 2 * g;
        const typename Q::A al = oct_act<TYPE>(da + (row / p.Rd) * p.ald.pitch, p.ald, o, grid);
        typename Q::St acc[2];
        const typename Q::W wl[2] = {Q::initw(st, row * p.pitch_d, o), Q::initw(st, (row + 1) * p.pitch_d, o)};
        int v = 0;
        for (; v + 1 < U; v += 2) {
            Q::template unit<0>(wl, al, v, acc);
            Q::template unit<1>(wl, al, v + 1, acc);
        }
        if (v < U) Q::template unit<0>(wl, al, v, acc);
        const float d0 = Q::finish(acc[0]);
        const float d1 = Q::finish(acc[1]);
        if (o == 0) {
            dots[row] = d0;
            dots[row + 1] = d1;
        }
    }
}

// Input producer of one kind (0: gate/up inputs x_L, 1: down inputs).
// The input rows of key K = L*T + t (a layer's token) go to buffer
// K % (kStackBufs, or nbuf_d for down inputs). Walking the CTA's jobs of its kind in order (their keys
// never decrease), the producer counts the jobs of each buffer; at each new
// key it waits until every job of the buffer's previous key is done, waits
// for the rows to exist (x_L quantized: q_done[L] reaches q_target, or every
// Q8 block of the token's activations), copies them in and publishes the fill word (K << 1 | phase
// parity). A consumer spins until its buffer's fill word names its key, then
// waits on the buffer barrier with that parity: the fill of K is issued only
// after every job of the buffer's previous key has finished, so the barrier
// is never two phases behind a waiting consumer and its parity is unambiguous.
__device__ __forceinline__ void stack_input_producer(const StackParams & p, int kind, int mine, int b, int G,
                                                     uint64_t * bbar, volatile int * fillw, volatile int * bufdone,
                                                     uint8_t * buf, int buf_bytes, int q_target) {
    const StackGeom g = stack_geom(p);
    const int blocks_per_token = p.k * (p.I / p.qblk);   // quantized down-input blocks of a token
    const int nb = kind == 1 ? p.nbuf_d : kStackBufs;       // buffers of this kind
    int iss[kStackBufs], fills[kStackBufs];
#pragma unroll
    for (int i = 0; i < kStackBufs; ++i) {
        iss[i] = 0;
        fills[i] = 0;
    }
    int cur = -1;
    StackWalk walk{0, 0};
    walk.advance(g, b);
    for (int jl = 0; jl < mine; ++jl, walk.advance(g, G)) {
        int jL, jgu;
        walk.kind(g, jL, jgu);
        if (jgu != (kind == 0 ? 1 : 0)) continue;
        const StackJob J = walk.job(g);
        const int K = J.L * p.T + J.t, bi = K % nb;
        if (K != cur) {
            // every job that used the buffer before is done with it
            bool ok = false;
            for (uint32_t i = 0; i < (1u << 23) && !ok; ++i) {
                ok = bufdone[bi] >= iss[bi];
                if (!ok && (i & 63u) == 63u && *reinterpret_cast<volatile int *>(&g_dev_error) != 0) break;
                if (!ok && i >= 16) __nanosleep(64);
            }
            if (ok) ok = kind == 0 ? stack_wait(p.q_done + J.L, q_target) : stack_wait(p.gu_done + K, blocks_per_token);
            if (!ok) {
                record_error(GX_DEVERR_TIMEOUT);
                break;
            }
            fence_acq_rel_gpu();
            fence_proxy_async_global();
            const StackLayer & ly = p.layers[J.L];
            uint8_t * dst = buf + bi * buf_bytes;
            if (kind == 0) {
                tma_expect(bbar + bi, (uint32_t)p.alx.pitch);
                tma_load(dst, ly.xq + (int64_t)J.t * p.alx.pitch, (uint32_t)p.alx.pitch, bbar + bi);
            } else {
                const uint32_t bytes = (uint32_t)(p.k * p.ald.pitch);
                tma_expect(bbar + bi, bytes);
                tma_load(dst, ly.actq + (int64_t)J.t * p.k * p.ald.pitch, bytes, bbar + bi);
            }
            ++fills[bi];
            fillw[bi] = (K << 1) | ((fills[bi] - 1) & 1);
            cur = K;
        }
        ++iss[bi];
    }
    // copies in flight land before the CTA can exit
#pragma unroll
    for (int i = 0; i < kStackBufs; ++i)
        if (fills[i] > 0) stack_mbar_wait(bbar + i, (uint32_t)((fills[i] - 1) & 1));
}

}  // namespace gx

#include "gx_stack_tc.cuh"
#include "gx_stack_tma.cuh"

namespace gx {

// TCM: MXFP4 jobs on the tensor cores, row mode 4 (one weight producer, the
// roles of gx_stack_tc.cuh on warps 1 and 4-15) or row mode 5 (the roles of
// gx_stack_tma.cuh on warps 0, 1 and 4-13); 0 for the CUDA-core row modes
template <int TG, int TD, int TCM = 0>
__global__ void __launch_bounds__(TCM == 4 ? kTcThreads : TCM == 5 ? kT5Threads
                                  : 32 * (kStackProducers + 2) + 32 * stack_max_warps(TG == GX_T_MXFP4 ? 3 : 0), 1)
    k_stack(const __grid_constant__ StackParams p) {
    // row mode: 0 two-lane Q8_0 rows, 2 two-lane Q4_K gate/up + Q6_K down rows, 1 octet rows,
    // 3 MXFP4 rows on the CUDA cores, 4 MXFP4 rows on the tensor cores
    constexpr bool TC = TCM != 0;
    constexpr int kMode = TC ? TCM
                          : (TG == GX_T_Q8_0 && TD == GX_T_Q8_0) ? 0
                          : (TG == GX_T_Q4_K && TD == GX_T_Q6_K) ? 2
                          : (TG == GX_T_MXFP4 && TD == GX_T_MXFP4) ? 3
                                                                  : 1;
    static_assert(!TC || (TG == GX_T_MXFP4 && TD == GX_T_MXFP4), "tensor-core stack jobs are MXFP4 rows");
    constexpr int P = TC ? 1 : kStackProducers;   // weight producer warps
    constexpr int VG = Oct<TG>::VDT, VD = Oct<TD>::VDT;       // activation types of gate/up and down
    // warps per job (p.split): octet jobs are compute-bound and two warps
    // share each (passes split between them); so do the 32-row down jobs of
    // the two-lane K-quant rows (row q | row q + 16 of each lane pair), whose
    // gate/up jobs stay whole (their second part only counts itself)
    extern __shared__ __align__(128) uint8_t smem[];
    const int C = p.C;
    uint64_t * wfull = reinterpret_cast<uint64_t *>(smem + p.bar_off);
    uint64_t * empty = wfull + C;
    uint64_t * xbar = empty + C;            // kStackBufs input-buffer barriers per kind
    uint64_t * dbar = xbar + kStackBufs;
    int * fillw = reinterpret_cast<int *>(smem + p.meta_off);   // [2][kStackBufs] fill words
    int * bufdone = fillw + kStackMaxConsumers;      // [2][kStackBufs]
    int * rel = bufdone + 2 * kStackBufs;             // [C] releases per stage
    uint8_t * stages = smem + p.stage_off;
    uint8_t * xbuf = smem + p.xbuf_off;
    uint8_t * dbuf = smem + p.dbuf_off;
    const int xbytes = p.alx.pitch, dbytes = p.k * p.ald.pitch;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, b = blockIdx.x;
    const int NJ = p.NL * (p.n_gu + p.n_d);
    const int mine = b < NJ ? (NJ - b + G - 1) / G : 0;   // jobs of this CTA

    // every slot id of the launch is checked before any load and kept in
    // shared memory for the weight producer
    int32_t * slots = reinterpret_cast<int32_t *>(smem + p.slots_off);
    StackWeights * wt = reinterpret_cast<StackWeights *>(smem + p.wt_off);
    {
        int bad = 0;
        const int per = p.T * p.k;
        for (int j = tid; j < p.NL * per; j += blockDim.x) {
            const int L = j / per;
            const int32_t e = p.layers[L].slots[j - L * per];
            if (e < 0 || e >= p.layers[L].n_as) bad = 1;
            slots[j] = e;
        }
        for (int L = tid; L < p.NL; L += blockDim.x) {
            StackWeights w;
            w.wg = p.layers[L].wg;
            w.wu = p.layers[L].wu;
            w.wd = p.layers[L].wd;
            w.nb02 = p.layers[L].nb02;
            wt[L] = w;
        }
        // bufdone, rel, next task, per-stage finished-part counters
        if (tid < 2 * kStackBufs + 2 * kStackMaxConsumers + 1) bufdone[tid] = 0;
        if (tid < 2 * kStackBufs) fillw[tid] = -1;                                // no key filled yet
        if (__syncthreads_or(bad)) {
            if (tid == 0) record_error(GX_DEVERR_DOMAIN);
            return;
        }
    }
    if (tid == 0) {
        for (int s = 0; s < 2 * C + 2 * kStackBufs; ++s) mbar_init(wfull + s, 1);
        if constexpr (TCM == 4) tc_init_bars(tc_team(smem, p.tc_off, (p.H > p.I ? p.H : p.I) / 32, p.tc_na));
        if constexpr (TCM == 5) t5_init_bars(t5_team(smem, p.tc_off, (p.H > p.I ? p.H : p.I) / 32, p.tc_na));
        mbar_fence_init();
    }
    if constexpr (TCM == 5) {
        // row mode 5: the CTA's jobs, decoded once
        const StackGeom g = stack_geom(p);
        uint2 * jobs = reinterpret_cast<uint2 *>(smem + p.t5_jobs_off);
        for (int jl = tid; jl < mine && jl < p.t5_jobs; jl += blockDim.x) jobs[jl] = t5_pack(stack_job(g, b + jl * G));
    }
    __syncthreads();

    if constexpr (TCM == 5) {
        // row mode 5: the TMA producer (warp 0) and the MMA issuer (warp 1)
        if (warp < kStackProducers) {
            stack_t5(p, smem, warp, lane, b, G, mine, slots, wt, xbar, dbar, fillw, bufdone, smem + p.xbuf_off,
                     smem + p.dbuf_off);
            return;
        }
    }
    if (TCM == 4 && warp > 0 && warp < kStackProducers) {
        // one weight producer; warp 1 issues the MMAs
        stack_tc(p, smem, warp, lane, b, G, mine, wfull, empty, xbar, dbar, fillw, bufdone, rel, smem + p.stage_off,
                 smem + p.xbuf_off, smem + p.dbuf_off);
        return;
    }
    if (warp < P) {
        // ------------------------------------------------ weight producers
        // producer warp w issues the jobs jl = w, w + P, ... (P producers)
        const StackGeom g = stack_geom(p);
        StackCopy q;
        q.nb01_g = p.nb01_g;
        q.nb01_d = p.nb01_d;
        q.pitch_d = p.pitch_d;
        q.row_copy_d = p.row_copy_d;
        q.T = p.T;
        q.k = p.k;
        q.Rg = p.Rg;
        q.Rd = p.Rd;
        q.gu_copies = (kMode == 1 || kMode >= 3) ? 2 : 4;
        for (int t = 0; t < 4; ++t) q.tile[t] = p.gu_tile[t];
        const int stage_bytes = p.stage_bytes;
        StackWalk walk{0, 0};
        walk.advance(g, b + warp * G);
        int last = -1;   // the last job this warp issued
        bool aborted = false;
        for (int jl = warp; jl < mine; jl += P) {
            const int s = jl % C, n = jl / C;
            int okw = 1;
            if (n > 0) {
                if (lane == 0) okw = stack_mbar_wait(empty + s, (uint32_t)((n - 1) & 1)) ? 1 : 0;
                okw = __shfl_sync(0xffffffffu, okw, 0);
            }
            if (!okw) {
                if (lane == 0) record_error(GX_DEVERR_TIMEOUT);
                aborted = true;
                break;
            }
            stack_issue_weights(q, walk.job(g), slots, wt, stages + s * stage_bytes, wfull + s, lane);
            last = jl;
            walk.advance(g, P * G);
        }
        // Let the copies of this warp that no later job consumed land before
        // the CTA can exit: a stage's final job (jl + C >= mine); a job with a
        // successor on its stage was consumed before the successor was issued.
        // After an abort, every recent copy (bounded waits).
        if (lane == 0)
            for (int jl = last; jl >= 0 && jl > last - C; jl -= P)
                if (aborted || jl + C >= mine) stack_mbar_wait(wfull + jl % C, (uint32_t)((jl / C) & 1));
        return;
    }
    if (warp == kStackProducers || warp == kStackProducers + 1) {
        // -------------------------------------------------- input producers
        if (lane != 0) return;
        const int kind = warp - kStackProducers;
        // row mode 5 counts x blocks quantized anywhere in the grid; the
        // others flag a layer once its owner CTA quantized all of it
        const int q_target = TCM == 5 ? p.T * (p.H / 32) : 1;
        stack_input_producer(p, kind, mine, b, G, kind == 0 ? xbar : dbar, fillw + kind * kStackBufs,
                             bufdone + kind * kStackBufs, kind == 0 ? xbuf : dbuf, kind == 0 ? xbytes : dbytes,
                             q_target);
        return;
    }

    if constexpr (TCM == 4) {
        // ------------------------------------------ tensor-core roles
        stack_tc(p, smem, warp, lane, b, G, mine, wfull, empty, xbar, dbar, fillw, bufdone, rel, stages, xbuf, dbuf);
        return;
    }
    if constexpr (TCM == 5) {
        // ------------------------------------------ epilogue warps of row mode 5
        stack_t5(p, smem, warp, lane, b, G, mine, slots, wt, xbar, dbar, fillw, bufdone, xbuf, dbuf);
        return;
    }
    // ------------------------------------------------------------ consumers
    // W consumer warps take the CTA's jobs dynamically (a shared counter), so
    // a warp busy with an epilogue never leaves a loaded stage idle; job jl
    // still uses stage jl % C, and each stage is consumed in job order: the
    // warp that takes job jl first waits until job jl - C was released.
    const int W = p.W;
    const int c = warp - kStackProducers - 2;
    if (c >= W) return;
    if constexpr (TG == GX_T_IQ1_S || TD == GX_T_IQ1_S) {
        uint2 * g2 = reinterpret_cast<uint2 *>(smem + p.grid_off);
        for (int i = c * 32 + lane; i < 2048; i += 32 * W) g2[i] = g_iq1s_grid[i];
        named_barrier(2, 32 * W);
    }
    // quantize the inputs of layers L = b, b+G, ... (one warp per Q8 block)
    {
        const int nblk = p.H / (VG == GX_T_Q8_0 ? 32 : 256);
        bool any = false;
        for (int L = b; L < p.NL; L += G) {
            const StackLayer & ly = p.layers[L];
            for (int wi = c; wi < p.T * nblk; wi += W) {
                const int t = wi / nblk, ib = wi - t * nblk;
                quant_block_split<VG, false, kMode >= 3>(ly.x + (int64_t)t * p.H, ly.xq + (int64_t)t * p.alx.pitch, p.alx,
                                                         ib, lane);
            }
            any = true;
        }
        if (any) {
            fence_proxy_async_global();
            named_barrier(1, 32 * W);
            if (c == 0 && lane == 0) {
                fence_acq_rel_gpu();
                for (int L = b; L < p.NL; L += G) atomicExch(p.q_done + L, 1);
            }
        }
    }
    const StackGeom g = stack_geom(p);
    const int par = lane >> 4;   // block parity of this lane
    int * next_job = rel + kStackMaxConsumers;
    int * parts = next_job + 1;                        // [C] finished parts of the stage's current job
    float * sdots = reinterpret_cast<float *>(smem + p.dots_off);   // [C][32] down-row dots per stage
    // IQ1_S: the codebook in shared memory (copied by the consumers before the
    // input quantization barrier below, i.e. before their first job)
    const uint2 * sgrid = reinterpret_cast<const uint2 *>(smem + p.grid_off);
    for (;;) {
        int task = 0;
        if (lane == 0) task = atomicAdd(next_job, 1);
        task = __shfl_sync(0xffffffffu, task, 0);
        const int split = kMode == 0 ? 1 : p.split;
        const int jl = task / split, sub = task - jl * split;
        if (jl >= mine) break;
        const int cs = jl % C, n = jl / C;
        const uint32_t ph = (uint32_t)(n & 1);
        // the previous job of this stage was released: its phases completed
        bool ok = true;
        if (lane == 0) {
            ok = n == 0;
            for (uint32_t i = 0; i < (1u << 23) && !ok; ++i) {
                ok = *reinterpret_cast<volatile int *>(rel + cs) >= n;
                if (!ok && (i & 63u) == 63u && *reinterpret_cast<volatile int *>(&g_dev_error) != 0) break;
                if (!ok && i >= 16) __nanosleep(32);
            }
        }
        ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
        ok = ok && stack_mbar_wait(wfull + cs, ph);
        const StackJob J = stack_job(g, b + jl * G);
        // the job's input buffer: its fill word must name the job's key
        const int key = J.L * p.T + J.t, bi = key % kStackBufs;
        int fpar = 0;
        if (lane == 0 && ok) {
            const volatile int * fw = fillw + (J.gu ? 0 : kStackBufs) + bi;
            bool got = false;
            for (uint32_t i = 0; i < (1u << 23) && !got; ++i) {
                const int v = *fw;
                got = (v >> 1) == key;
                fpar = v & 1;
                if (!got && (i & 63u) == 63u && *reinterpret_cast<volatile int *>(&g_dev_error) != 0) break;
                if (!got && i >= 16) __nanosleep(32);
            }
            ok = got;
        }
        ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
        fpar = __shfl_sync(0xffffffffu, fpar, 0);
        uint64_t * ibar = (J.gu ? xbar : dbar) + bi;
        ok = ok && stack_mbar_wait(ibar, (uint32_t)fpar);
        if (__any_sync(0xffffffffu, !ok)) {
            if (lane == 0) record_error(GX_DEVERR_TIMEOUT);
            break;
        }
        const StackLayer & ly = p.layers[J.L];
        const uint8_t * st = stages + cs * p.stage_bytes;
        int * done = bufdone + (J.gu ? 0 : kStackBufs) + bi;
        if (J.gu) {
            const uint8_t * xa = xbuf + bi * xbytes;
            if constexpr (kMode >= 3) {
                // 16 gate rows (tile 0) + 16 up rows (tile 1): lane r takes row r;
                // part `sub` computes pairs sub, sub + split, ... and parks their terms
                const uint8_t * row = st + p.gu_tile[lane >> 4] + (lane & 15) * (int)p.nb01_g;
                mxfp4_rows_part(row, xa, p.alx, p.H / 64, sub, split);
                __syncwarp();
                int lastp = 0;
                if (lane == 0) {
                    __threadfence_block();
                    lastp = atomicAdd(parts + cs, 1) == split - 1;
                    if (lastp) __threadfence_block();
                }
                if (!__shfl_sync(0xffffffffu, lastp, 0)) continue;   // the last part folds and runs the epilogue
                const float dot = mxfp4_rows_fold(row, p.H / 64);
                fence_proxy_async_shared();   // terms written into the stage before its refill
                __syncwarp();
                if (lane == 0) {
                    parts[cs] = 0;
                    __threadfence_block();
                    atomicAdd(done, 1);
                    atomicAdd(rel + cs, 1);
                    mbar_arrive(empty + cs);
                }
                // gate row r (lane r < 16) pairs with up row r (lane r + 16)
                const float up = __shfl_down_sync(0xffffffffu, dot, 16);
                if (lane < 16) {
                    const float a = p.act == 1 ? act_swiglu_oai(dot, up, p.alpha, p.limit) : act_swiglu(dot, up);
                    ly.act[(int64_t)J.pair * p.I + J.r0 + lane] = a;
                }
            } else if constexpr (kMode != 1) {
                // lane = qr*8 + tile*2 + gp: row qr of tile `tile` (gate rows 4*tile+qr
                // for tiles 0, 1; up rows 4*(tile-2)+qr for tiles 2, 3), lane half gp
                const int qr = lane >> 3, tl = (lane >> 1) & 3, gp = lane & 1;
                float dot;
                if constexpr (kMode == 0) {
                    const uint8_t * rb[1] = {st + p.gu_tile[tl] + qr * (int)p.nb01_g + 32 * gp};
                    const uint8_t * ab[1] = {xa + 32 * gp};
                    const uint8_t * ad[1] = {xa + p.alx.d_off};
                    float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
                    q8_0_rows<1>(rb, ab, ad, gp, p.H / 64, acc);
                    __syncwarp();
                    if (lane == 0) {
                        __threadfence_block();
                        atomicAdd(done, 1);
                        atomicAdd(rel + cs, 1);
                        mbar_arrive(empty + cs);   // stage and input buffer are free
                    }
                    dot = q8_0_finish_x1(acc[0]);
                } else {
                    if (sub == 0) dot = q4k_row2(st + p.gu_tile[tl] + qr * (int)p.nb01_g, xa, p.alx, gp, p.H / 256, 1);
                    __syncwarp();
                    if (lane == 0) {
                        // the job's last part frees the stage and the input buffer
                        __threadfence_block();
                        if (split == 1 || atomicAdd(parts + cs, 1) == split - 1) {
                            if (split > 1) {
                                parts[cs] = 0;
                                __threadfence_block();
                            }
                            atomicAdd(done, 1);
                            atomicAdd(rel + cs, 1);
                            mbar_arrive(empty + cs);
                        }
                    }
                    if (sub != 0) continue;   // a whole gate/up job's second part only counts itself
                }
                // gate row i = 4*tl + qr (tl < 2) pairs with up row i in tile tl + 2 (lane + 4)
                const float up = __shfl_down_sync(0xffffffffu, dot, 4);
                if (gp == 0 && tl < 2) {
                    const float a = p.act == 1 ? act_swiglu_oai(dot, up, p.alpha, p.limit) : act_swiglu(dot, up);
                    ly.act[(int64_t)J.pair * p.I + J.r0 + 4 * tl + qr] = a;
                }
            } else {
                float gd[2], ud[2];
                stack_gu_oct<TG>(p, st, xa, lane, gd, ud, sub, split, sgrid);
                __syncwarp();
                if (lane == 0) {
                    // the job's last part frees the stage and the input buffer
                    __threadfence_block();
                    if (atomicAdd(parts + cs, 1) == split - 1) {
                        parts[cs] = 0;
                        __threadfence_block();
                        atomicAdd(done, 1);
                        atomicAdd(rel + cs, 1);
                        mbar_arrive(empty + cs);
                    }
                }
                if ((lane & 7) == 0) {
                    for (int ps = sub; ps < 2; ps += split) {
                        const float a = p.act == 1 ? act_swiglu_oai(gd[ps], ud[ps], p.alpha, p.limit)
                                                   : act_swiglu(gd[ps], ud[ps]);
                        ly.act[(int64_t)J.pair * p.I + J.r0 + 4 * ps + (lane >> 3)] = a;
                    }
                }
            }
            const int nblk = p.I / p.qblk, blk = J.r0 / p.qblk;
            __syncwarp();
            // release this job's activation values, then count it into its
            // Q8 block; the block's last arriver acquires everyone's values
            int last = 0;
            if (lane == 0) {
                fence_acq_rel_gpu();
                last = atomicAdd(ly.cnt + J.pair * nblk + blk, 1) ==
                       (kMode == 1 ? split : 1) * (p.qblk / p.Rg) - 1;
            }
            if (__shfl_sync(0xffffffffu, last, 0)) {
                // this job finished the Q8 block last: quantize it and count the
                // block into its token (the down inputs wait for k*I/qblk blocks)
                fence_acq_rel_gpu();
                quant_block_split<VD, true, kMode >= 3>(ly.act + (int64_t)J.pair * p.I,
                                                         ly.actq + (int64_t)J.pair * p.ald.pitch, p.ald, blk, lane);
                fence_proxy_async_global();
                __syncwarp();
                if (lane == 0) {
                    fence_acq_rel_gpu();
                    atomicAdd(p.gu_done + J.L * p.T + J.t, 1);
                }
            }
        } else if constexpr (kMode == 1) {
            float * dts = sdots + cs * 32;
            stack_d_oct<TD>(p, st, dbuf + bi * dbytes, lane, dts, sub, split, sgrid);
            __syncwarp();
            int lastp = 0;
            if (lane == 0) {
                __threadfence_block();
                lastp = atomicAdd(parts + cs, 1) == split - 1;
                if (lastp) __threadfence_block();
            }
            if (__shfl_sync(0xffffffffu, lastp, 0)) {
                // the job's last part: every row dot is in the stage's scratch;
                // output row rr = lane < Rd: sum over slots m of w[m] * dot(m*Rd + rr), in slot order
                if (lane < p.Rd) {
                    const float * wr = ly.rw + (int64_t)J.t * p.k;
                    float accf = __fmul_rn(dts[lane], wr[0]);
                    for (int mm = 1; mm < p.k; ++mm) accf = __fadd_rn(accf, __fmul_rn(dts[mm * p.Rd + lane], wr[mm]));
                    ly.out[(int64_t)J.t * p.H + J.r0 + lane] = accf;
                }
                __syncwarp();
                if (lane == 0) {
                    parts[cs] = 0;
                    __threadfence_block();
                    atomicAdd(done, 1);
                    atomicAdd(rel + cs, 1);
                    mbar_arrive(empty + cs);
                }
            }
            __syncwarp();
        } else if constexpr (kMode >= 3) {
            // k*Rd = 32 weight rows (row r: row r % Rd of expert r / Rd): lane r
            // takes row r against its expert's activation row
            const uint8_t * da = dbuf + bi * dbytes;
            const uint8_t * row = st + lane * p.pitch_d;
            mxfp4_rows_part(row, da + (lane / p.Rd) * p.ald.pitch, p.ald, p.I / 64, sub, split);
            __syncwarp();
            int lastp = 0;
            if (lane == 0) {
                __threadfence_block();
                lastp = atomicAdd(parts + cs, 1) == split - 1;
                if (lastp) __threadfence_block();
            }
            if (!__shfl_sync(0xffffffffu, lastp, 0)) continue;
            const float dot = mxfp4_rows_fold(row, p.I / 64);
            fence_proxy_async_shared();
            __syncwarp();
            if (lane == 0) {
                parts[cs] = 0;
                __threadfence_block();
                atomicAdd(done, 1);
                atomicAdd(rel + cs, 1);
                mbar_arrive(empty + cs);
            }
            // output row rr = lane < Rd: sum over slots m of w[m] * dot(m*Rd + rr), in slot order
            const float * wr = ly.rw + (int64_t)J.t * p.k;
            float accf = 0.0f;
            for (int mm = 0; mm < p.k; ++mm) {
                const float v = __shfl_sync(0xffffffffu, dot, (mm * p.Rd + lane) & 31);
                const float prod = __fmul_rn(v, lane < p.Rd ? wr[mm] : 0.0f);
                accf = mm == 0 ? prod : __fadd_rn(accf, prod);
            }
            if (lane < p.Rd) ly.out[(int64_t)J.t * p.H + J.r0 + lane] = accf;
        } else {
            // lane = par*16 + q: weight rows q and q+16 of the job's k*Rd rows
            // (row R is row R % Rd of expert R / Rd); eight consecutive lanes
            // read eight consecutive rows, so the 16-byte loads of a quarter
            // warp fall in distinct bank groups
            const int q = lane & 15;
            const int m0 = q / p.Rd, m1 = (q + 16) / p.Rd;
            const uint8_t * da = dbuf + bi * dbytes;
            const uint8_t * a0 = da + m0 * p.ald.pitch;
            const uint8_t * a1 = da + m1 * p.ald.pitch;
            float d0, d1;
            if constexpr (kMode == 0) {
                const uint8_t * rb[2] = {st + q * p.pitch_d + 32 * par, st + (q + 16) * p.pitch_d + 32 * par};
                const uint8_t * ab[2] = {a0 + 32 * par, a1 + 32 * par};
                const uint8_t * ad[2] = {a0 + p.ald.d_off, a1 + p.ald.d_off};
                float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                q8_0_rows<2>(rb, ab, ad, par, p.I / 64, acc);
                __syncwarp();
                if (lane == 0) {
                    __threadfence_block();
                    atomicAdd(done, 1);
                    atomicAdd(rel + cs, 1);
                    mbar_arrive(empty + cs);
                }
                d0 = q8_0_finish(acc[0]);
                d1 = q8_0_finish(acc[1]);
            } else {
                if (split == 2) {
                    // part sub: row R = q + 16*sub of each lane pair, into the stage's dot scratch
                    const int R = q + 16 * sub;
                    const uint8_t * ar = da + (R / p.Rd) * p.ald.pitch;
                    float dd, unused;
                    q6k_rows2<1>(st + R * p.pitch_d, st, ar, ar, p.ald, par, p.I / 256, 16, dd, unused);
                    float * dts = sdots + cs * 32;
                    if (par == 0) dts[R] = dd;
                    __syncwarp();
                    int lastp = 0;
                    if (lane == 0) {
                        __threadfence_block();
                        lastp = atomicAdd(parts + cs, 1) == split - 1;
                        if (lastp) __threadfence_block();
                    }
                    if (__shfl_sync(0xffffffffu, lastp, 0)) {
                        // the last part: output row rr = lane < Rd, slots in order
                        if (lane < p.Rd) {
                            const float * wr = ly.rw + (int64_t)J.t * p.k;
                            float accf = __fmul_rn(dts[lane], wr[0]);
                            for (int mm = 1; mm < p.k; ++mm)
                                accf = __fadd_rn(accf, __fmul_rn(dts[mm * p.Rd + lane], wr[mm]));
                            ly.out[(int64_t)J.t * p.H + J.r0 + lane] = accf;
                        }
                        __syncwarp();
                        if (lane == 0) {
                            parts[cs] = 0;
                            __threadfence_block();
                            atomicAdd(done, 1);
                            atomicAdd(rel + cs, 1);
                            mbar_arrive(empty + cs);
                        }
                    }
                    __syncwarp();
                    continue;
                }
                if (p.k * p.Rd == 16)   // one row per lane
                    q6k_rows2<1>(st + q * p.pitch_d, st, a0, a0, p.ald, par, p.I / 256, 16, d0, d1);
                else
                    q6k_rows2<2>(st + q * p.pitch_d, st + (q + 16) * p.pitch_d, a0, a1, p.ald, par, p.I / 256, 16, d0, d1);
                __syncwarp();
                if (lane == 0) {
                    __threadfence_block();
                    atomicAdd(done, 1);
                    atomicAdd(rel + cs, 1);
                    mbar_arrive(empty + cs);
                }
            }
            // output row rr = lane < Rd: weight row R = m*Rd + rr of expert m
            // is d0 of lane R (R < 16) or d1 of lane R - 16
            const float * wr = ly.rw + (int64_t)J.t * p.k;
            float accf = 0.0f;
            for (int mm = 0; mm < p.k; ++mm) {
                const int R = mm * p.Rd + (lane < p.Rd ? lane : 0);
                const float v0 = __shfl_sync(0xffffffffu, d0, R & 15);
                const float v1 = __shfl_sync(0xffffffffu, d1, R & 15);
                const float prod = __fmul_rn(R < 16 ? v0 : v1, lane < p.Rd ? wr[mm] : 0.0f);
                accf = mm == 0 ? prod : __fadd_rn(accf, prod);
            }
            if (lane < p.Rd) ly.out[(int64_t)J.t * p.H + J.r0 + lane] = accf;
        }
    }
}

}  // namespace gx
