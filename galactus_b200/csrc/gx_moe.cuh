// Decode-path kernels of the routed-expert FFN (sm_100a): persistent CTAs,
// multi-stage bulk-TMA pipelines, four lanes per weight row.
//
// Activations are quantized once into an internal "split" layout (all int8
// quants of a row contiguous, then the block scales, then the Q8_K block
// sums), so the dot loops read them with aligned 32-bit loads. The values are
// exactly those of ggml's Q8_0 / Q8_K blocks; only the byte layout differs.
//
// A weight row is processed by eight lanes: lane o owns one eighth of every
// 64- or 256-element unit. Integer partial sums are exact, so the lanes add
// them with shuffles in any order; the float tail is then evaluated in the
// reference's order (diff:1049-1054, 1167-1174, 1254-1259, 1366-1370,
// 335-345) in registers, identically in the eight lanes (or, for Q8_0, as the
// NEON loop's per-lane accumulator chains, reduced by its faddp trees).
#pragma once

#include <cstdint>

#include "gx_device.cuh"
#include "gx_kernels.h"

namespace gx {

// position of element e of a 32-element Q8_0 block in "code order", the byte
// order of an MXFP4 block's codes (code byte j holds elements j and j+16):
// word t of the block holds elements 4(t/2) + 2(t%2) + {0, 16, 1, 17}
__device__ __forceinline__ int mxfp4_code_pos(int e) { return 8 * ((e & 15) >> 2) + 2 * (e & 3) + (e >> 4); }

// quantize block ib of an f32 row into the split layout, one warp; PERM
// stores a Q8_0 block's quants in code order (same values and scale)
template <int VDT, bool COHERENT, bool PERM = false>
__device__ __forceinline__ void quant_block_split(const float * x, uint8_t * row, const ActLayout & L, int ib, int lane) {
    if (VDT == GX_T_Q8_0) {
        const float v = COHERENT ? __ldcg(x + 32 * ib + lane) : __ldg(x + 32 * ib + lane);
        float a = fabsf(v);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
        const float d = __fdiv_rn(a, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        row[32 * ib + (PERM ? mxfp4_code_pos(lane) : lane)] = (uint8_t)(int8_t)__float2int_rn(__fmul_rn(v, id));
        if (lane == 0) *reinterpret_cast<uint16_t *>(row + L.d_off + 2 * ib) = f2h(d);
    } else {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = COHERENT ? __ldcg(x + 256 * ib + 8 * lane + j) : __ldg(x + 256 * ib + 8 * lane + j);
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
        int8_t * qs = reinterpret_cast<int8_t *>(row + 256 * ib);
        int16_t * bs = reinterpret_cast<int16_t *>(row + L.bs_off) + 16 * ib;
        float * dp = reinterpret_cast<float *>(row + L.d_off) + ib;
        if (amax == 0.0f) {
#pragma unroll
            for (int j = 0; j < 8; ++j) qs[8 * lane + j] = 0;
            if (lane < 16) bs[lane] = 0;
            if (lane == 0) *dp = 0.0f;
            return;
        }
        const float iscale = __fdiv_rn(-127.0f, vmax);
        int lsum = 0;
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int q = min(127, __float2int_rn(__fmul_rn(iscale, v[j])));
            lsum += q;
            if (j < 4) w0 |= ((uint32_t)(q & 0xff)) << (8 * j); else w1 |= ((uint32_t)(q & 0xff)) << (8 * (j - 4));
        }
        *reinterpret_cast<uint2 *>(qs + 8 * lane) = make_uint2(w0, w1);
        const int pair = lsum + __shfl_xor_sync(0xffffffffu, lsum, 1);
        if ((lane & 1) == 0) bs[lane >> 1] = (int16_t)pair;
        if (lane == 0) *dp = __fdiv_rn(1.0f, iscale);
    }
}

// ---------------------------------------------------------- octet dots
//
// Eight lanes per weight row; lane o owns one eighth of every unit (one
// 32-element block of a Q8_0/MXFP4 pair split in quarters, or one 32-element
// sub-block of a 256-element superblock).

__device__ __forceinline__ int oct_sum(int v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    return v;
}

__device__ __forceinline__ int quad_sum(int v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    return v;
}

// 16-bit value at an even byte offset of a shared-memory buffer whose base is 4-byte aligned
__device__ __forceinline__ uint32_t lds_u16_even(const uint8_t * base, int off) {
    return (lds32(base + (off & ~3)) >> ((off & 2) * 8)) & 0xffffu;
}

// Each lane prepares its lane-constant shared-memory offsets once per row
// (Lane), then walks the units with immediate offsets. Block sizes of 17, 50
// and 210 bytes make the byte alignment alternate between even and odd units,
// so units are processed in (even, odd) pairs, each with its own precomputed
// shift, in row order.

template <int TYPE> struct Oct;

__device__ __forceinline__ uint32_t bfe16(uint32_t w, uint32_t sh) { return (w >> sh) & 0xffffu; }

// A thread computes two weight rows against one activation row: the
// activation words and scales are loaded once for both. W is the per-row
// lane context, A the shared activation context.

template <> struct Oct<GX_T_Q8_0> {
    static constexpr int VDT = GX_T_Q8_0;
    static constexpr int UNIT = 64;
    struct St { float a = 0.0f; };
    struct W { const uint8_t * wq; const uint8_t * wd; uint32_t sh, dsh; };
    struct A { const uint8_t * aq; const uint8_t * ad; uint32_t ash; };
    __device__ __forceinline__ static W initw(const uint8_t * wb, int wo, int o) {
        const int b = o >> 2, l = o & 3;
        const int q = wo + 34 * b + 2 + 4 * l, d = wo + 34 * b;
        W w;
        w.wq = wb + (q & ~3);
        w.sh = (uint32_t)(q & 3) * 8u;
        w.wd = wb + (d & ~3);
        w.dsh = (uint32_t)(d & 2) * 8u;
        return w;
    }
    __device__ __forceinline__ static A inita(const uint8_t * ar, const ActLayout & L, int o) {
        const int b = o >> 2, l = o & 3;
        A a;
        a.aq = ar + 32 * b + 4 * l;
        a.ad = ar + L.d_off;
        a.ash = 16u * (uint32_t)b;
        return a;
    }
    template <int PAR>
    __device__ __forceinline__ static void unit(const W (&w)[2], const A & a, int u, St (&st)[2]) {
        const uint8_t * ap = a.aq + 64 * u;
        const uint32_t y0 = lds32(ap), y1 = lds32(ap + 16);
        const float dy = h2f((uint16_t)bfe16(lds32(a.ad + 4 * u), a.ash));
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint8_t * q = w[r].wq + 68 * u;
            const uint32_t x0 = __funnelshift_r(lds32(q), lds32(q + 4), w[r].sh);
            const uint32_t x1 = __funnelshift_r(lds32(q + 16), lds32(q + 20), w[r].sh);
            const float dx = h2f((uint16_t)bfe16(lds32(w[r].wd + 68 * u), w[r].dsh));
            const int ip = dp4a(x1, y1, dp4a(x0, y0, 0));
            st[r].a = __fmaf_rn((float)ip, __fmul_rn(dx, dy), st[r].a);
        }
    }
    // ((e0+e1)+(e2+e3)) + ((o0+o1)+(o2+o3)), the NEON faddp trees
    __device__ __forceinline__ static float finish(St & st) {
        float v = st.a;
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
        return __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
    }
};

// MXFP4: lane o -> block b = o>>2, quant word l = o&3 of its 16 bytes;
// t = fma(sc_e, p_e, sc_o*p_o) per pair, sumf = sumf + t.
template <> struct Oct<GX_T_MXFP4> {
    static constexpr int VDT = GX_T_Q8_0;
    static constexpr int UNIT = 64;
    struct St { float s = 0.0f; };
    struct W { const uint8_t * wq[2]; uint32_t sh[2]; const uint8_t * we; };
    struct A { const uint8_t * aq; const uint8_t * ad; int b; };
    __device__ __forceinline__ static W initw(const uint8_t * wb, int wo, int o) {
        const int b = o >> 2, l = o & 3;
        W w;
        for (int par = 0; par < 2; ++par) {
            const int q = wo + 34 * par + 17 * b + 1 + 4 * l;
            w.wq[par] = wb + (q & ~3) - 34 * par;   // unit u of parity par reads wq[par] + 34*u
            w.sh[par] = (uint32_t)(q & 3) * 8u;
        }
        w.we = wb + wo;
        return w;
    }
    __device__ __forceinline__ static A inita(const uint8_t * ar, const ActLayout & L, int o) {
        A a;
        a.b = o >> 2;
        a.aq = ar + 32 * a.b + 4 * (o & 3);
        a.ad = ar + L.d_off;
        return a;
    }
    template <int PAR>
    __device__ __forceinline__ static void unit(const W (&w)[2], const A & a, int u, St (&st)[2]) {
        const uint8_t * ap = a.aq + 64 * u;
        const uint32_t ylo = lds32(ap), yhi = lds32(ap + 16);
        const uint32_t dd = lds32(a.ad + 4 * u);
        const float dye = h2f((uint16_t)(dd & 0xffffu)), dyo = h2f((uint16_t)(dd >> 16));
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint8_t * q = w[r].wq[PAR] + 34 * u;
            const uint32_t qq = __funnelshift_r(lds32(q), lds32(q + 4), w[r].sh[PAR]);
            int ip = dp4a(mxfp4_lut(qq & 0x0f0f0f0fu), ylo, 0);
            ip = dp4a(mxfp4_lut((qq >> 4) & 0x0f0f0f0fu), yhi, ip);
            ip = quad_sum(ip);
            const int other = __shfl_xor_sync(0xffffffffu, ip, 4);
            const int pe = a.b ? other : ip, po = a.b ? ip : other;
            const float sce = __fmul_rn(dye, e8m0_half(w[r].we[34 * u]));
            const float sco = __fmul_rn(dyo, e8m0_half(w[r].we[34 * u + 17]));
            st[r].s = __fadd_rn(st[r].s, __fmaf_rn(sce, (float)pe, __fmul_rn(sco, (float)po)));
        }
    }
    __device__ __forceinline__ static float finish(St & st) { return st.s; }
};

// Q4_K: lane o -> sub-block o (32 elements: nibble o&1 of quant bytes 32(o>>1)..);
// rows and superblocks are 16-byte aligned, so quants load 16 bytes at a time.
template <> struct Oct<GX_T_Q4_K> {
    static constexpr int VDT = GX_T_Q8_K;
    static constexpr int UNIT = 256;
    struct St { float s = 0.0f; };
    struct W { const uint8_t * wb; };
    struct A { const uint8_t * aq; const uint8_t * ar; ActLayout L; int o; };
    __device__ __forceinline__ static W initw(const uint8_t * wb, int wo, int) { return W{wb + wo}; }
    __device__ __forceinline__ static A inita(const uint8_t * ar, const ActLayout & L, int o) {
        A a;
        a.aq = ar + 32 * o;
        a.ar = ar;
        a.L = L;
        a.o = o;
        return a;
    }
    template <int PAR>
    __device__ __forceinline__ static void unit(const W (&w)[2], const A & a, int i, St (&st)[2]) {
        const int o = a.o, m = o >> 1;
        const uint32_t shn = 4u * (uint32_t)(o & 1);
        const uint8_t * ap = a.aq + 256 * i;
        const uint4 a0 = *reinterpret_cast<const uint4 *>(ap);
        const uint4 a1 = *reinterpret_cast<const uint4 *>(ap + 16);
        const uint32_t aw[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const uint32_t bw = lds32(a.ar + a.L.bs_off + 32 * i + 4 * o);
        const int q8s = (int16_t)((int16_t)(bw & 0xffff) + (int16_t)(bw >> 16));
        const float yd = __uint_as_float(lds32(a.ar + a.L.d_off + 4 * i));
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint8_t * xb = w[r].wb + 144 * i;
            const uint4 q0 = *reinterpret_cast<const uint4 *>(xb + 16 + 32 * m);
            const uint4 q1 = *reinterpret_cast<const uint4 *>(xb + 32 + 32 * m);
            const uint4 hdr = *reinterpret_cast<const uint4 *>(xb);
            const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            int p = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) p = dp4a((qw[k] >> shn) & 0x0f0f0f0fu, aw[k], p);
            int sc, mn;
            if (o < 4) {
                sc = (hdr.y >> (8 * o)) & 63;
                mn = (hdr.z >> (8 * o)) & 63;
            } else {
                const int b = o - 4;
                sc = ((hdr.w >> (8 * b)) & 0x0f) | (((hdr.y >> (8 * b + 6)) & 3) << 4);
                mn = ((hdr.w >> (8 * b + 4)) & 0x0f) | (((hdr.z >> (8 * b + 6)) & 3) << 4);
            }
            const int sumi = oct_sum(p * sc);
            const int prod = oct_sum(q8s * mn);
            st[r].s = __fmaf_rn(-__fmul_rn(yd, h2f((uint16_t)(hdr.x >> 16))), (float)prod, st[r].s);
            st[r].s = __fmaf_rn(__fmul_rn(yd, h2f((uint16_t)(hdr.x & 0xffffu))), (float)sumi, st[r].s);
        }
    }
    __device__ __forceinline__ static float finish(St & st) { return st.s; }
};

// Q6_K: lane o -> 16-element groups 2o and 2o+1 (elements 32o..32o+31)
template <> struct Oct<GX_T_Q6_K> {
    static constexpr int VDT = GX_T_Q8_K;
    static constexpr int UNIT = 256;
    struct St { float s = 0.0f; };
    struct W { const uint8_t * wb; int wo; };
    struct A { const uint8_t * aq; const uint8_t * ar; ActLayout L; int o; };
    __device__ __forceinline__ static W initw(const uint8_t * wb, int wo, int) { return W{wb, wo}; }
    __device__ __forceinline__ static A inita(const uint8_t * ar, const ActLayout & L, int o) {
        A a;
        a.aq = ar + 32 * o;
        a.ar = ar;
        a.L = L;
        a.o = o;
        return a;
    }
    template <int PAR>
    __device__ __forceinline__ static void unit(const W (&w)[2], const A & a, int i, St (&st)[2]) {
        const int o = a.o;
        const int j = o >> 1, ho = o & 1, h = j >> 1, odd = j & 1;
        const uint8_t * ap = a.aq + 256 * i;
        const uint4 a0 = *reinterpret_cast<const uint4 *>(ap);
        const uint4 a1 = *reinterpret_cast<const uint4 *>(ap + 16);
        const uint32_t aw[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const uint32_t sh = 4u * (uint32_t)odd + 2u * (uint32_t)ho;
        const uint32_t nsh = 4u * (uint32_t)odd;
        const uint32_t bw = lds32(a.ar + a.L.bs_off + 32 * i + 4 * o);
        const int bs0 = (int)(int16_t)(bw & 0xffff), bs1 = (int)(int16_t)(bw >> 16);
        const float yd = __uint_as_float(lds32(a.ar + a.L.d_off + 4 * i));
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int xo = w[r].wo + 210 * i;
            uint32_t ql[8], qh[8], scw[1];
            ld_words<8>(w[r].wb, xo + 64 * h + 32 * ho, ql);
            ld_words<8>(w[r].wb, xo + 128 + 32 * h, qh);
            ld_words<1>(w[r].wb, xo + 192 + 2 * o, scw);
            int pg[2] = {0, 0};
#pragma unroll
            for (int ww = 0; ww < 8; ++ww) {
                const uint32_t nib = (ql[ww] >> nsh) & 0x0f0f0f0fu;
                const uint32_t hb = (qh[ww] >> sh) & 0x03030303u;
                pg[ww >> 2] = dp4a(nib | (hb << 4), aw[ww], pg[ww >> 2]);
            }
            const int sc0 = (int)(int8_t)(scw[0] & 0xff), sc1 = (int)(int8_t)((scw[0] >> 8) & 0xff);
            const int isum = oct_sum(pg[0] * sc0 + pg[1] * sc1);
            const int mins = oct_sum(bs0 * sc0 + bs1 * sc1);
            st[r].s = __fmaf_rn(__fmul_rn(yd, h2f(ld_u16(w[r].wb, xo + 208))), (float)(isum - 32 * mins), st[r].s);
        }
    }
    __device__ __forceinline__ static float finish(St & st) { return st.s; }
};

// IQ1_S: lane o -> sub-block o; sumi1 + sumi2 is the integer sum over all eight
template <> struct Oct<GX_T_IQ1_S> {
    static constexpr int VDT = GX_T_Q8_K;
    static constexpr int UNIT = 256;
    struct St { float s = 0.0f; };
    struct W { const uint8_t * wb; int wo; };
    // grid: the codebook, in global memory or a shared-memory copy
    struct A { const uint8_t * aq; const uint8_t * ar; ActLayout L; int o; const uint2 * grid; };
    __device__ __forceinline__ static W initw(const uint8_t * wb, int wo, int) { return W{wb, wo}; }
    __device__ __forceinline__ static A inita(const uint8_t * ar, const ActLayout & L, int o,
                                              const uint2 * grid = g_iq1s_grid) {
        A a;
        a.aq = ar + 32 * o;
        a.ar = ar;
        a.L = L;
        a.o = o;
        a.grid = grid;
        return a;
    }
    template <int PAR>
    __device__ __forceinline__ static void unit(const W (&w)[2], const A & a, int i, St (&st)[2]) {
        const int o = a.o;
        const uint8_t * ap = a.aq + 256 * i;
        const uint4 a0 = *reinterpret_cast<const uint4 *>(ap);
        const uint4 a1 = *reinterpret_cast<const uint4 *>(ap + 16);
        const uint32_t aw[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const uint32_t bw = lds32(a.ar + a.L.bs_off + 32 * i + 4 * o);
        const int bsum = (int)(int16_t)(bw & 0xffff) + (int)(int16_t)(bw >> 16);
        const float yd = __uint_as_float(lds32(a.ar + a.L.d_off + 4 * i));
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int xo = w[r].wo + 50 * i;
            uint32_t qsw[1], qhw[1];
            ld_words<1>(w[r].wb, xo + 2 + 4 * o, qsw);
            ld_words<1>(w[r].wb, xo + 34 + 2 * o, qhw);
            const uint32_t qh = qhw[0] & 0xffffu;
            int p = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t gi = ((qsw[0] >> (8 * j)) & 0xffu) | (((qh >> (3 * j)) & 7u) << 8);
                const uint2 g = a.grid[gi];
                p = dp4a(g.x, aw[2 * j], p);
                p = dp4a(g.y, aw[2 * j + 1], p);
            }
            const int ls = 2 * (int)((qh >> 12) & 7u) + 1;
            const int sg = (qh & 0x8000u) ? -1 : 1;
            const int s12 = oct_sum(p * ls);
            const int s3 = oct_sum(bsum * ls * sg);
            const float expr = __fmaf_rn((float)s3, 0.125f, (float)s12);
            st[r].s = __fmaf_rn(__fmul_rn(yd, h2f(ld_u16(w[r].wb, xo))), expr, st[r].s);
        }
    }
    __device__ __forceinline__ static float finish(St & st) { return st.s; }
};

// --------------------------------------------------------- PDL and TMA

__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------ decode kernels

__device__ __forceinline__ int32_t dec_id(const DecodeParams & p, int t, int s) {
    return p.use_inline ? p.inline_ids[t * p.k + s] : p.ids[t * p.k + s];
}

__device__ __forceinline__ bool mbar_wait_limit(uint64_t * bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 24); ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"((uint32_t)__cvta_generic_to_shared(bar)), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void tma_expect(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void tma_load(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            (uint32_t)__cvta_generic_to_shared(dst)),
        "l"(src), "r"(bytes), "r"((uint32_t)__cvta_generic_to_shared(bar))
        : "memory");
}

// Issue the weight copies of one unit into a stage. GATE_UP: R gate rows then
// R up rows of the pair's expert; DOWN: R rows of each of the token's k experts.
template <int MODE>
__device__ __forceinline__ void issue_unit(const DecodeParams & p, int u, uint8_t * stage, uint64_t * bar) {
    const int tiles = p.ne01 / p.R;
    const int r0 = (u % tiles) * p.R;
    const int nexp = MODE == 1 ? 2 : p.k;
    tma_expect(bar, (uint32_t)(nexp * p.R) * (uint32_t)p.nb01);
    for (int m = 0; m < nexp; ++m) {
        const uint8_t * src;
        if (MODE == 1) {
            const int pair = u / tiles;
            const int32_t e = dec_id(p, pair / p.k, pair % p.k);
            src = (m == 0 ? p.w0 : p.w1) + (int64_t)e * p.nb02 + (int64_t)r0 * p.nb01;
        } else {
            const int t = u / tiles;
            src = p.w0 + (int64_t)dec_id(p, t, m) * p.nb02 + (int64_t)r0 * p.nb01;
        }
        uint8_t * dst = stage + m * p.R * p.pitch_w;
        if (p.row_copy) {
            for (int r = 0; r < p.R; ++r) tma_load(dst + r * p.pitch_w, src + (int64_t)r * p.nb01, (uint32_t)p.nb01, bar);
        } else {
            tma_load(dst, src, (uint32_t)(p.R * p.nb01), bar);
        }
    }
}

// MODE 1: gate/up + activation, one (token, slot) pair per unit, then the
//         quantization of each completed Q8 block of the activation row by the
//         last CTA that contributed to it (no CTA ever waits for another).
// MODE 2: down + weighted combine, one token per unit (all k slots).
template <int TYPE, int MODE>
__global__ void __launch_bounds__(kDecodeMaxThreads, 1) k_decode(const DecodeParams p) {
    using Q = Oct<TYPE>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t * full = reinterpret_cast<uint64_t *>(smem);   // S stage barriers, then the activation barrier
    uint64_t * abar = full + p.S;
    uint8_t * act = smem + p.act_off;
    uint8_t * stages = smem + p.stage_off;
    float * dots = reinterpret_cast<float *>(smem + p.dots_off);
    int * flag = reinterpret_cast<int *>(smem + p.flag_off);
    const int tid = threadIdx.x, lane = tid & 31, l = tid & 7, grp = tid >> 3;
    // the two rows of this thread: gate row and up row (MODE 1), or two
    // adjacent rows of one expert tile (MODE 2); both use the same activation
    const int row0 = MODE == 1 ? grp : 2 * grp;
    const int row1 = MODE == 1 ? grp + p.R : 2 * grp + 1;
    const int G = gridDim.x;
    const int tiles = p.ne01 / p.R;
    const int U = p.ne00 / Q::UNIT;

    // every slot id of the call is checked before any load
    {
        int bad = 0;
        for (int j = tid; j < p.T * p.k; j += blockDim.x) {
            const int32_t e = p.use_inline ? p.inline_ids[j] : p.ids[j];
            if (e < 0 || e >= p.n_as) bad = 1;
        }
        if (__syncthreads_or(bad)) {
            if (tid == 0) record_error(GX_DEVERR_DOMAIN);
            return;
        }
    }

    if (tid == 0) {
        for (int s = 0; s <= p.S; ++s) mbar_init(full + s, 1);
        mbar_fence_init();
    }
    __syncthreads();
    // weights do not depend on the previous kernel: start streaming them now
    if (tid == 0) {
        for (int i = 0; i < p.S; ++i) {
            const int u = blockIdx.x + i * G;
            if (u < p.n_units) issue_unit<MODE>(p, u, stages + i * p.stage_bytes, full + i);
        }
    }
    griddep_launch_dependents();
    griddep_wait();   // the quantized activations come from the previous kernel

    int cur_t = -1;
    uint32_t aphase = 0;
    for (int i = 0;; ++i) {
        const int u = blockIdx.x + i * G;
        if (u >= p.n_units) break;
        const int s = i % p.S;
        const int t = MODE == 1 ? (u / tiles) / p.k : u / tiles;
        const int r0 = (u % tiles) * p.R;
        if (t != cur_t) {
            if (tid == 0) {
                tma_expect(abar, (uint32_t)(p.a_rows * p.al.pitch));
                const int arow0 = MODE == 1 ? t : t * p.k;
                tma_load(act, p.aq + (int64_t)arow0 * p.al.pitch, (uint32_t)(p.a_rows * p.al.pitch), abar);
            }
            if (!mbar_wait_limit(abar, aphase)) {
                if (tid == 0) record_error(GX_DEVERR_TIMEOUT);
                mbar_wait_limit(abar, aphase);
                return;
            }
            aphase ^= 1u;
            cur_t = t;
        }
        if (!mbar_wait_limit(full + s, (uint32_t)((i / p.S) & 1))) {
            if (tid == 0) record_error(GX_DEVERR_TIMEOUT);
            mbar_wait_limit(full + s, (uint32_t)((i / p.S) & 1));
            return;
        }
        const uint8_t * st_base = stages + s * p.stage_bytes;
        const uint8_t * arow = MODE == 1 ? act : act + (row0 / p.R) * p.al.pitch;
        typename Q::St acc[2];
        const typename Q::W wl[2] = {Q::initw(st_base, row0 * p.pitch_w, l), Q::initw(st_base, row1 * p.pitch_w, l)};
        const typename Q::A al = Q::inita(arow, p.al, l);
        int v = 0;
#pragma unroll 2
        for (; v + 1 < U; v += 2) {
            Q::template unit<0>(wl, al, v, acc);
            Q::template unit<1>(wl, al, v + 1, acc);
        }
        if (v < U) Q::template unit<0>(wl, al, v, acc);
        const float dot0 = Q::finish(acc[0]);
        const float dot1 = Q::finish(acc[1]);
        if (l == 0) {
            dots[row0] = dot0;
            dots[row1] = dot1;
        }
        __syncthreads();
        // the stage is free: stream the unit S steps ahead into it
        if (tid == 0) {
            const int un = u + p.S * G;
            if (un < p.n_units) issue_unit<MODE>(p, un, stages + s * p.stage_bytes, full + s);
        }
        if (MODE == 1) {
            const int pair = u / tiles;
            if (tid < p.R) {
                const float g = dots[tid], up = dots[p.R + tid];
                const float a = p.act == 1 ? act_swiglu_oai(g, up, p.alpha, p.limit) : act_swiglu(g, up);
                p.act_f32[(int64_t)pair * p.ne01 + r0 + tid] = a;
                __threadfence();
            }
            __syncthreads();
            const int nblk = p.ne01 / p.qblk;
            const int blk = r0 / p.qblk;
            if (tid == 0) {
                const int old = atomicAdd(p.counters + pair * nblk + blk, 1);
                *flag = old == p.qblk / p.R - 1;
            }
            __syncthreads();
            if (*flag && tid < 32) {
                __threadfence();
                const float * src = p.act_f32 + (int64_t)pair * p.ne01;
                uint8_t * dst = p.act_q + (int64_t)pair * p.al2.pitch;
                if (p.vdt2 == GX_T_Q8_0) quant_block_split<GX_T_Q8_0, true>(src, dst, p.al2, blk, lane);
                else quant_block_split<GX_T_Q8_K, true>(src, dst, p.al2, blk, lane);
                if (lane == 0) atomicExch(p.counters + pair * nblk + blk, 0);
            }
        } else {
            if (tid < p.R) {
                const float * w = p.rw + (int64_t)t * p.k;
                float accf = __fmul_rn(dots[tid], w[0]);
                for (int m = 1; m < p.k; ++m) accf = __fadd_rn(accf, __fmul_rn(dots[m * p.R + tid], w[m]));
                p.out[(int64_t)t * p.ne01 + r0 + tid] = accf;
            }
        }
        __syncthreads();
    }
}

// f32 rows -> split-layout Q8 rows, one warp per block
template <int VDT>
__global__ void k_quant_split(const float * src, int ne0, int64_t nrows, int64_t nb1, uint8_t * dst, ActLayout L) {
    griddep_launch_dependents();
    griddep_wait();
    const int nblk = ne0 / (VDT == GX_T_Q8_0 ? 32 : 256);
    const int64_t wid = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (wid >= nrows * nblk) return;
    const int64_t r = wid / nblk;
    const int ib = (int)(wid - r * nblk);
    const float * x = reinterpret_cast<const float *>(reinterpret_cast<const char *>(src) + r * nb1);
    quant_block_split<VDT, false>(x, dst + r * L.pitch, L, ib, threadIdx.x & 31);
}

}  // namespace gx
