// Device building blocks of the routed-expert FFN for sm_100a.
//
// Everything here is exact integer work or IEEE single-precision arithmetic
// written with explicit rounding intrinsics (__fmul_rn, __fadd_rn, __fmaf_rn,
// __fdiv_rn), so that no compiler contraction or approximation can change a
// bit: the float operations and their order are the ones the reference
// certifies for ggml's arm64-NEON CPU functions
// (patches/galactus-h4-llamacpp.diff, cited per function below).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "gx_formats.h"

namespace gx {

// ---------------------------------------------------------------- helpers

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
// binary32 -> binary16 with round to nearest even, written out on the bits
// (IEEE 754 narrowing, the same definition as the oracle's orc_fp32_to_fp16)
__device__ __forceinline__ uint16_t f2h(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u | ((ax >> 13) & 0x3ffu) : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    if (ax < 0x38800000u) {
        if (ax < 0x33000000u) return (uint16_t)sign;
        const uint32_t e = ax >> 23;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e;
        const uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        const uint32_t r = q + ((rem > half || (rem == half && (q & 1u))) ? 1u : 0u);
        return (uint16_t)(sign | r);
    }
    uint32_t h = (ax >> 13) - (112u << 10);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

__device__ __forceinline__ uint32_t lds32(const uint8_t * p) { return *reinterpret_cast<const uint32_t *>(p); }

// N consecutive 32-bit words starting at any byte offset of a shared-memory
// buffer (the buffer is padded so that reading one word past the end is in
// bounds). Block formats of 17, 34, 50 and 210 bytes do not keep 4-byte
// alignment, so their fields are re-aligned with funnel shifts.
template <int N>
__device__ __forceinline__ void ld_words(const uint8_t * base, int off, uint32_t (&out)[N]) {
    const uint8_t * p = base + (off & ~3);
    const uint32_t sh = (uint32_t)(off & 3) * 8u;
    uint32_t w0 = lds32(p);
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const uint32_t w1 = lds32(p + 4 * (i + 1));
        out[i] = __funnelshift_r(w0, w1, sh);
        w0 = w1;
    }
}

__device__ __forceinline__ uint16_t ld_u16(const uint8_t * base, int off) {
    return (uint16_t)base[off] | ((uint16_t)base[off + 1] << 8);
}

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

// ------------------------------------------------------------------- expf
// The one exp of the library, shared bit for bit with the oracle's orc_expf
// (same constants, same operations). Method: n = RNE(x*log2 e) by the
// 1.5*2^23 rounding constant; r = x - n*ln2 with ln2 split into a 15-bit head
// (exact products for |n| <= 256) and a tail (Cody & Waite, 1980); e^r by the
// degree-7 Taylor polynomial in Horner form with fused multiply-adds; 2^n
// applied through the exponent field, in two steps (the first exact) when the
// result is subnormal.
__device__ __forceinline__ float gx_expf(float x) {
    if (x != x) return __fadd_rn(x, x);
    if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
    if (x < -103.972084045410156f) return 0.0f;
    const float t = __fmaf_rn(x, 1.44269502162933349609375f, 12582912.0f);
    const float n = __fsub_rn(t, 12582912.0f);
    float r = __fmaf_rn(-n, 0.693145751953125f, x);
    r = __fmaf_rn(-n, 1.428606765330187045e-06f, r);
    float p = __fmaf_rn(r, 1.98412701138295233249664306640625e-04f, 1.3888889225199818611145019531250e-03f);
    p = __fmaf_rn(p, r, 8.3333337679505348205566406250000e-03f);
    p = __fmaf_rn(p, r, 4.1666667908430099487304687500000e-02f);
    p = __fmaf_rn(p, r, 1.6666667163372039794921875000000e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = (int)n;
    if (ni >= -125) {
        if (ni > 127) return __fmul_rn(__fmul_rn(p, 2.0f), __int_as_float((ni - 1 + 127) << 23));
        return __fmul_rn(p, __int_as_float((ni + 127) << 23));
    }
    return __fmul_rn(__fmul_rn(p, __int_as_float((ni + 64 + 127) << 23)), __int_as_float((-64 + 127) << 23));
}

// ggml's scalar SiLU times the up projection: g / (1 + exp(-g)) * u
__device__ __forceinline__ float act_swiglu(float g, float u) {
    const float s = __fdiv_rn(g, __fadd_rn(1.0f, gx_expf(-g)));
    return __fmul_rn(s, u);
}

// SWIGLU_OAI (diff:1461-1465, 1911-1918): ordered-comparison min/clamp,
// IEEE divide, then (y + 1)
__device__ __forceinline__ float act_swiglu_oai(float g, float u, float alpha, float limit) {
    const float x = limit < g ? limit : g;
    const float y = u < -limit ? -limit : (limit < u ? limit : u);
    const float glu = __fdiv_rn(x, __fadd_rn(1.0f, gx_expf(__fmul_rn(alpha, -x))));
    return __fmul_rn(glu, __fadd_rn(y, 1.0f));
}

// ------------------------------------------------- activation quantizers

// One Q8_0 block by one warp, lane = element (quantize_row_q8_0 NEON order,
// diff:1000-1007): amax is a max (order-free), d = amax/127, id = d ? 1/d : 0,
// q = RNE(x*id) narrowed to int8, d stored as binary16 RNE.
__device__ __forceinline__ void quantize_q8_0_block_warp(float v, uint8_t * blk, int lane) {
    float a = fabsf(v);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
    const float d = __fdiv_rn(a, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const int q = __float2int_rn(__fmul_rn(v, id));
    blk[2 + lane] = (uint8_t)(int8_t)q;
    if (lane == 0) {
        const uint16_t h = f2h(d);
        blk[0] = (uint8_t)(h & 0xff);
        blk[1] = (uint8_t)(h >> 8);
    }
}

// One Q8_K superblock by one warp, lane = elements 8*lane .. 8*lane+7
// (quantize_row_q8_K, diff:348-427): first strict max of |x| wins and ties
// keep the smaller index, iscale = -127/max, q = min(127, RNE(iscale*x)),
// bsums per 16, d = 1/iscale. An all-zero superblock is d = 0, zeros.
__device__ __forceinline__ void quantize_q8_K_block_warp(const float (&v)[8], uint8_t * blk, int lane) {
    float amax = 0.0f, vmax = 0.0f;
    int imax = 8 * lane;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float av = fabsf(v[j]);
        if (av > amax) { amax = av; vmax = v[j]; imax = 8 * lane + j; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, off);
        const float ov = __shfl_xor_sync(0xffffffffu, vmax, off);
        const int oi = __shfl_xor_sync(0xffffffffu, imax, off);
        if (oa > amax || (oa == amax && oi < imax)) { amax = oa; vmax = ov; imax = oi; }
    }
    int8_t * qs = reinterpret_cast<int8_t *>(blk + 4);
    int16_t * bsums = reinterpret_cast<int16_t *>(blk + 260);
    if (amax == 0.0f) {
#pragma unroll
        for (int j = 0; j < 8; ++j) qs[8 * lane + j] = 0;
        if (lane < 16) bsums[lane] = 0;
        if (lane == 0) *reinterpret_cast<float *>(blk) = 0.0f;
        return;
    }
    const float iscale = __fdiv_rn(-127.0f, vmax);
    int lsum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int q = min(127, __float2int_rn(__fmul_rn(iscale, v[j])));
        qs[8 * lane + j] = (int8_t)q;
        lsum += q;
    }
    const int pair = lsum + __shfl_xor_sync(0xffffffffu, lsum, 1);
    if ((lane & 1) == 0) bsums[lane >> 1] = (int16_t)pair;
    if (lane == 0) *reinterpret_cast<float *>(blk) = __fdiv_rn(1.0f, iscale);
}

// Quantize one f32 row (global memory) into a row of blocks in shared or
// global memory, with the warps of the calling CTA (nwarps, warp id w).
template <int VDT>
__device__ __forceinline__ void quantize_row_cta(const float * __restrict__ x, int ne0, uint8_t * dst, int w, int nwarps, int lane) {
    if (VDT == GX_T_Q8_0) {
        for (int ib = w; ib < ne0 / 32; ib += nwarps) {
            const float v = __ldg(x + ib * 32 + lane);
            quantize_q8_0_block_warp(v, dst + ib * 34, lane);
        }
    } else {
        for (int ib = w; ib < ne0 / 256; ib += nwarps) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __ldg(x + ib * 256 + 8 * lane + j);
            quantize_q8_K_block_warp(v, dst + ib * 292, lane);
        }
    }
}

// --------------------------------------------------- per-type dot pieces
//
// A row of ne00 weights is cut into units of 64 elements (a pair of 32-element
// blocks, or a quarter of a 256-element superblock). Phase 1 computes each
// unit's exact integer partial sums and per-block float scales, in any order
// and in parallel; phase 2 runs the reference's float tail serially, unit
// after unit in row order, exactly as the CPU loop does. Terms are 32-bit
// words in shared memory, TERMS of them per unit.

template <int TYPE> struct Dot;

__device__ __forceinline__ uint32_t mxfp4_lut(uint32_t idx4) {
    // four 4-bit codes (one per byte, 0..15) -> four int8 values of
    // kvalues_mxfp4 {0,1,2,3,4,6,8,12, 0,-1,-2,-3,-4,-6,-8,-12}
    const uint32_t x = idx4 & 0x07070707u;
    const uint32_t y = x | (x >> 4);
    const uint32_t sel = (y & 0xffu) | ((y >> 8) & 0xff00u);
    const uint32_t lo = __byte_perm(0x03020100u, 0x0c080604u, sel);
    const uint32_t hi = __byte_perm(0xfdfeff00u, 0xf4f8fafcu, sel);
    const uint32_t m = ((idx4 >> 3) & 0x01010101u) * 0xffu;
    return (lo & ~m) | (hi & m);
}

// Q8_0 x Q8_0 (ggml_vec_dot_q8_0_q8_0, diff:1049-1054, 1074-1163).
// Unit = block pair p. Terms: 8 partials as float (exact, |p| < 2^24) and the
// two block scales fp16(x.d)*fp16(y.d). Eight chains per row:
// acc[c] = fma(part[c], scale, acc[c]); result ((a0+a1)+(a2+a3))+((a4+a5)+(a6+a7)).
template <> struct Dot<GX_T_Q8_0> {
    static constexpr int TERMS = 10;
    static constexpr int CHAINS = 8;
    static constexpr int VDT = GX_T_Q8_0;
    __device__ __forceinline__ static void unit(const uint8_t * wb, int wo, const uint8_t * arow, int u, uint32_t * t) {
        const int o = 68 * u;
        uint32_t xe[8], ye[8], xo[8], yo[8];
        ld_words<8>(wb, wo + o + 2, xe);
        ld_words<8>(arow, o + 2, ye);
        ld_words<8>(wb, wo + o + 36, xo);
        ld_words<8>(arow, o + 36, yo);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const int pe = dp4a(xe[4 + l], ye[4 + l], dp4a(xe[l], ye[l], 0));
            const int po = dp4a(xo[4 + l], yo[4 + l], dp4a(xo[l], yo[l], 0));
            t[l] = __float_as_uint((float)pe);
            t[4 + l] = __float_as_uint((float)po);
        }
        const uint32_t wy0 = lds32(arow + o), wy8 = lds32(arow + o + 32);
        t[8] = __float_as_uint(__fmul_rn(h2f(ld_u16(wb, wo + o)), h2f((uint16_t)(wy0 & 0xffff))));
        t[9] = __float_as_uint(__fmul_rn(h2f(ld_u16(wb, wo + o + 34)), h2f((uint16_t)(wy8 >> 16))));
    }
    // chain c of a row over units [0, U)
    __device__ __forceinline__ static float chain(const uint32_t * terms_row, int U, int c) {
        float acc = 0.0f;
        const int si = c < 4 ? 8 : 9;
        for (int u = 0; u < U; ++u) {
            const uint32_t * t = terms_row + u * TERMS;
            acc = __fmaf_rn(__uint_as_float(t[c]), __uint_as_float(t[si]), acc);
        }
        return acc;
    }
};

// MXFP4 x Q8_0 (ggml_vec_dot_mxfp4_q8_0, diff:1167-1174, 1209-1240).
// Unit = block pair p; the pair's term t = fma(sc_e, p_e, sc_o*p_o) depends
// only on the pair, so it is computed in phase 1. One chain: sumf = sumf + t.
__device__ __forceinline__ float e8m0_half(uint32_t e) {
    const uint32_t bits = e < 2 ? (0x00200000u << e) : ((e - 1) << 23);
    return __uint_as_float(bits);
}

template <> struct Dot<GX_T_MXFP4> {
    static constexpr int TERMS = 1;
    static constexpr int CHAINS = 1;
    static constexpr int VDT = GX_T_Q8_0;
    __device__ __forceinline__ static void unit(const uint8_t * wb, int wo, const uint8_t * arow, int u, uint32_t * t) {
        const int ow = wo + 34 * u, oa = 68 * u;
        uint32_t qe[4], qo[4], ye[8], yo[8];
        ld_words<4>(wb, ow + 1, qe);
        ld_words<4>(wb, ow + 18, qo);
        ld_words<8>(arow, oa + 2, ye);
        ld_words<8>(arow, oa + 36, yo);
        int pe = 0, po = 0;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            pe = dp4a(mxfp4_lut(qe[w] & 0x0f0f0f0fu), ye[w], pe);
            pe = dp4a(mxfp4_lut((qe[w] >> 4) & 0x0f0f0f0fu), ye[4 + w], pe);
            po = dp4a(mxfp4_lut(qo[w] & 0x0f0f0f0fu), yo[w], po);
            po = dp4a(mxfp4_lut((qo[w] >> 4) & 0x0f0f0f0fu), yo[4 + w], po);
        }
        const uint32_t wy0 = lds32(arow + oa), wy8 = lds32(arow + oa + 32);
        const float sce = __fmul_rn(h2f((uint16_t)(wy0 & 0xffff)), e8m0_half(wb[ow]));
        const float sco = __fmul_rn(h2f((uint16_t)(wy8 >> 16)), e8m0_half(wb[ow + 17]));
        t[0] = __float_as_uint(__fmaf_rn(sce, (float)pe, __fmul_rn(sco, (float)po)));
    }
    __device__ __forceinline__ static float chain(const uint32_t * terms_row, int U, int) {
        float sumf = 0.0f;
        for (int u = 0; u < U; ++u) sumf = __fadd_rn(sumf, __uint_as_float(terms_row[u]));
        return sumf;
    }
};

// Q4_K x Q8_K (ggml_vec_dot_q4_K_q8_K, diff:1254-1259, 1300-1357).
// Unit = quarter j of superblock i (elements 64j..64j+63). Terms: the quarter's
// share of sumi = p1*sc[2j] + p2*sc[2j+1] and of prod = sum q8sums*mins, and
// the superblock's d = y.d*fp16(x.d) and dmin = -(y.d*fp16(x.dmin)).
// One chain: per superblock sumf = fma(dmin, prod, sumf); sumf = fma(d, sumi, sumf).
template <> struct Dot<GX_T_Q4_K> {
    static constexpr int TERMS = 4;
    static constexpr int CHAINS = 1;
    static constexpr int VDT = GX_T_Q8_K;
    __device__ __forceinline__ static void unit(const uint8_t * wb, int wo, const uint8_t * arow, int u, uint32_t * t) {
        const int i = u >> 2, j = u & 3;
        const int xo = wo + 144 * i;
        const uint8_t * yb = arow + 292 * i;
        uint32_t q[8], a[16];
        ld_words<8>(wb, xo + 16 + 32 * j, q);
        ld_words<16>(yb, 4 + 64 * j, a);
        int p1 = 0, p2 = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            p1 = dp4a(q[w] & 0x0f0f0f0fu, a[w], p1);
            p2 = dp4a((q[w] >> 4) & 0x0f0f0f0fu, a[8 + w], p2);
        }
        // 6-bit scales and mins of sub-blocks 2j and 2j+1 (the 12-byte packing)
        const uint8_t * s = wb + xo + 4;
        int sc0, sc1, m0, m1;
        {
            const int a0 = 2 * j, a1 = 2 * j + 1;
            sc0 = a0 < 4 ? (s[a0] & 63) : ((s[a0 + 4] & 0x0f) | ((s[a0 - 4] >> 6) << 4));
            m0 = a0 < 4 ? (s[a0 + 4] & 63) : ((s[a0 + 4] >> 4) | ((s[a0] >> 6) << 4));
            sc1 = a1 < 4 ? (s[a1] & 63) : ((s[a1 + 4] & 0x0f) | ((s[a1 - 4] >> 6) << 4));
            m1 = a1 < 4 ? (s[a1 + 4] & 63) : ((s[a1 + 4] >> 4) | ((s[a1] >> 6) << 4));
        }
        const int16_t * bs = reinterpret_cast<const int16_t *>(yb + 260);
        const int q8s0 = (int16_t)(bs[4 * j] + bs[4 * j + 1]);
        const int q8s1 = (int16_t)(bs[4 * j + 2] + bs[4 * j + 3]);
        const float yd = __uint_as_float(lds32(yb));
        t[0] = (uint32_t)(p1 * sc0 + p2 * sc1);
        t[1] = (uint32_t)(q8s0 * m0 + q8s1 * m1);
        t[2] = __float_as_uint(__fmul_rn(yd, h2f(ld_u16(wb, xo))));
        t[3] = __float_as_uint(-__fmul_rn(yd, h2f(ld_u16(wb, xo + 2))));
    }
    __device__ __forceinline__ static float chain(const uint32_t * terms_row, int U, int) {
        float sumf = 0.0f;
        for (int u0 = 0; u0 < U; u0 += 4) {
            const uint32_t * t = terms_row + u0 * TERMS;
            const int sumi = (int)t[0] + (int)t[4] + (int)t[8] + (int)t[12];
            const int prod = (int)t[1] + (int)t[5] + (int)t[9] + (int)t[13];
            sumf = __fmaf_rn(__uint_as_float(t[3]), (float)prod, sumf);
            sumf = __fmaf_rn(__uint_as_float(t[2]), (float)sumi, sumf);
        }
        return sumf;
    }
};

// Q6_K x Q8_K (ggml_vec_dot_q6_K_q8_K, diff:1366-1370, 1393-1446).
// Unit = quarter j of superblock i (16-element groups 4j..4j+3). Terms: the
// quarter's share of isum = sum sc[g]*dot_g and of isum_mins = sum bsums[g]*sc[g],
// and d = y.d*fp16(x.d). One chain: sumf = fma(d, isum - 32*isum_mins, sumf).
template <> struct Dot<GX_T_Q6_K> {
    static constexpr int TERMS = 3;
    static constexpr int CHAINS = 1;
    static constexpr int VDT = GX_T_Q8_K;
    __device__ __forceinline__ static void unit(const uint8_t * wrow, int wo, const uint8_t * arow, int u, uint32_t * t) {
        const int i = u >> 2, j = u & 3;
        const int xo = wo + 210 * i;
        const uint8_t * yb = arow + 292 * i;
        const int h = j >> 1, odd = j & 1;
        uint32_t ql[16], qh[8], a[16];
        ld_words<16>(wrow, xo + 64 * h, ql);
        ld_words<8>(wrow, xo + 128 + 32 * h, qh);
        ld_words<16>(yb, 4 + 64 * j, a);
        uint32_t scw[1];
        ld_words<1>(wrow, xo + 192 + 4 * j, scw);       // int8 scales of groups 4j..4j+3
        const int16_t * bs = reinterpret_cast<const int16_t *>(yb + 260);
        int isum = 0, mins = 0;
#pragma unroll
        for (int gg = 0; gg < 4; ++gg) {
            int pg = 0;
#pragma unroll
            for (int ww = 0; ww < 4; ++ww) {
                const int w = 4 * gg + ww;            // word of the 64-element quarter
                const uint32_t nib = (odd ? (ql[w] >> 4) : ql[w]) & 0x0f0f0f0fu;
                const uint32_t sh = 4u * (uint32_t)odd + (w >= 8 ? 2u : 0u);
                const uint32_t hb = (qh[w & 7] >> sh) & 0x03030303u;
                pg = dp4a(nib | (hb << 4), a[w], pg);
            }
            const int g = 4 * j + gg;
            const int scg = (int)(int8_t)(scw[0] >> (8 * gg));
            isum += pg * scg;
            mins += (int)bs[g] * scg;
        }
        const float yd = __uint_as_float(lds32(yb));
        t[0] = (uint32_t)isum;
        t[1] = (uint32_t)mins;
        t[2] = __float_as_uint(__fmul_rn(yd, h2f(ld_u16(wrow, xo + 208))));
    }
    __device__ __forceinline__ static float chain(const uint32_t * terms_row, int U, int) {
        float sumf = 0.0f;
        for (int u0 = 0; u0 < U; u0 += 4) {
            const uint32_t * t = terms_row + u0 * TERMS;
            const int isum = (int)t[0] + (int)t[3] + (int)t[6] + (int)t[9];
            const int mins = (int)t[1] + (int)t[4] + (int)t[7] + (int)t[10];
            sumf = __fmaf_rn(__uint_as_float(t[2]), (float)(isum - 32 * mins), sumf);
        }
        return sumf;
    }
};

// IQ1_S x Q8_K (ggml_vec_dot_iq1_s_q8_K, diff:335-345, 458-510).
// Unit = sub-block pair (2j, 2j+1) of superblock i. Terms: shares of
// sumi1, sumi2, sumi3 and d = y.d*fp16(x.d). One chain per superblock:
// expr = fma((float)sumi3, 0.125, (float)(sumi1+sumi2)); sumf = fma(d, expr, sumf).
// iq1s grid: 2048 entries of 8 ternary int8 values, two words per entry,
// generated at build time from the gguf-py table (never retyped). This header
// is compiled into exactly one translation unit.
__device__ uint2 g_iq1s_grid[2048] = {
#include "_gen/iq1s_grid.inc"
};

template <> struct Dot<GX_T_IQ1_S> {
    static constexpr int TERMS = 4;
    static constexpr int CHAINS = 1;
    static constexpr int VDT = GX_T_Q8_K;
    __device__ __forceinline__ static void unit(const uint8_t * wrow, int wo, const uint8_t * arow, int u, uint32_t * t) {
        const int i = u >> 2, j = u & 3;
        const int xo = wo + 50 * i;
        const uint8_t * yb = arow + 292 * i;
        uint32_t qsw[2];
        ld_words<2>(wrow, xo + 2 + 8 * j, qsw);          // qs of sub-blocks 2j, 2j+1
        uint32_t qhw[1];
        ld_words<1>(wrow, xo + 34 + 4 * j, qhw);         // qh[2j], qh[2j+1]
        uint32_t a[16];
        ld_words<16>(yb, 4 + 64 * j, a);
        const int16_t * bs = reinterpret_cast<const int16_t *>(yb + 260);
        int p[2] = {0, 0};
        int ls[2];
        int sg[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const uint32_t qh = (qhw[0] >> (16 * hh)) & 0xffffu;
            const uint32_t qs4 = qsw[hh];
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const uint32_t gi = ((qs4 >> (8 * l)) & 0xffu) | (((qh >> (3 * l)) & 7u) << 8);
                const uint2 g = g_iq1s_grid[gi];
                p[hh] = dp4a(g.x, a[8 * hh + 2 * l], p[hh]);
                p[hh] = dp4a(g.y, a[8 * hh + 2 * l + 1], p[hh]);
            }
            ls[hh] = 2 * (int)((qh >> 12) & 7u) + 1;
            sg[hh] = (qh & 0x8000u) ? -1 : 1;
        }
        t[0] = (uint32_t)(p[0] * ls[0]);
        t[1] = (uint32_t)(p[1] * ls[1]);
        t[2] = (uint32_t)(((int)bs[4 * j] + (int)bs[4 * j + 1]) * ls[0] * sg[0]
                        + ((int)bs[4 * j + 2] + (int)bs[4 * j + 3]) * ls[1] * sg[1]);
        const float yd = __uint_as_float(lds32(yb));
        t[3] = __float_as_uint(__fmul_rn(yd, h2f(ld_u16(wrow, xo))));
    }
    __device__ __forceinline__ static float chain(const uint32_t * terms_row, int U, int) {
        float sumf = 0.0f;
        for (int u0 = 0; u0 < U; u0 += 4) {
            const uint32_t * t = terms_row + u0 * TERMS;
            const int s1 = (int)t[0] + (int)t[4] + (int)t[8] + (int)t[12];
            const int s2 = (int)t[1] + (int)t[5] + (int)t[9] + (int)t[13];
            const int s3 = (int)t[2] + (int)t[6] + (int)t[10] + (int)t[14];
            const float expr = __fmaf_rn((float)s3, 0.125f, (float)(s1 + s2));
            sumf = __fmaf_rn(__uint_as_float(t[3]), expr, sumf);
        }
        return sumf;
    }
};

// ---------------------------------------------------- errors, mbarriers

__device__ int g_dev_error = 0;

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_dev_error, 0, code); }

// --------------------------------------------------------- TMA / mbarrier

__device__ __forceinline__ uint32_t smem_u32(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// bulk copy global -> shared of this CTA, completion counted on the mbarrier
__device__ __forceinline__ void bulk_g2s(void * dst_smem, const void * src_gmem, uint32_t bytes, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// The same with a suspend-time hint: a waiting thread sleeps in the barrier
// until the phase completes or about `ns` nanoseconds pass, instead of
// returning at once and spinning in the caller's loop.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t * bar, uint32_t parity, uint32_t ns) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Every wait is bounded: after the limit the kernel records a timeout and
// gives up instead of spinning forever.
constexpr uint32_t kWaitLimit = 1u << 24;

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t * bar, uint32_t parity) {
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    return false;
}

}  // namespace gx
