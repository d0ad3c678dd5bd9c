// TEST INFRASTRUCTURE ONLY -- the CPU oracle of the routed-expert FFN.
//
// This file is the checker, never the product. Only tests/, the smoke entry
// point and bench.py's CPU-baseline leg may load it. The product path
// (galactus_b200/) never links, loads or falls back to it.
//
// What it restates. The reference certifies bit-identity of its GPU kernels
// against ggml's arm64-NEON CPU functions; the operation order of every one of
// those functions is written down, step by step, in the reference's Metal
// restatement (patches/galactus-h4-llamacpp.diff). Each function below cites
// the diff lines it follows. The arithmetic is plain IEEE single precision:
// this file is compiled with -ffp-contract=off and no fast-math, and every
// fused multiply-add that the reference says the CPU executes is an explicit
// std::fma. Integer partial sums are exact and therefore order-free.
//
// Parity status. ggml itself (llama.cpp commit da5b4486, the third-party module
// that owns this arithmetic) is not vendored with the reference and cannot be
// built here, so "identical to ggml's CPU bits" is UNPINNED: what is pinned is
//   - block layouts and element decoding, against the installed gguf-py 0.19.0
//     dequantizers (golden fixtures under tests/golden/, made by
//     tests/golden/make_golden.py);
//   - the operation orders, by citation of the diff lines below;
//   - the slot policy, against the reference's own src/h4 C++ compiled into
//     oracle/_ref (see oracle/Makefile).
//
// SiLU: the reference has no bit-exact SiLU (its Metal SWIGLU_OAI reproduces a
// closed vendor libm). Here both the oracle and the device use ONE expf,
// written from the textbook method (Cody-Waite reduction by ln2 in two parts,
// degree-7 Taylor polynomial in Horner form with fused multiply-adds, exact
// power-of-two scaling), so that the oracle and the device agree bit for bit by
// construction. Its distance to the host libm expf is measured by the tests.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include <atomic>
#include <thread>

extern "C" {

// ------------------------------------------------------------------ formats
// ggml block layouts (ggml-common.h of the pinned llama.cpp; the same byte
// layout is used by scripts/moe-profile.py:25-37 for its size table).

enum {
    ORC_Q8_0 = 8,
    ORC_Q8_K = 15,
    ORC_Q4_K = 12,
    ORC_Q6_K = 14,
    ORC_IQ1_S = 19,
    ORC_MXFP4 = 39,
};

#pragma pack(push, 1)
struct orc_block_q8_0 { uint16_t d; int8_t qs[32]; };                       // 34 B
struct orc_block_q8_K { float d; int8_t qs[256]; int16_t bsums[16]; };      // 292 B
struct orc_block_q4_K { uint16_t d; uint16_t dmin; uint8_t scales[12]; uint8_t qs[128]; };  // 144 B
struct orc_block_q6_K { uint8_t ql[128]; uint8_t qh[64]; int8_t scales[16]; uint16_t d; };  // 210 B
struct orc_block_mxfp4 { uint8_t e; uint8_t qs[16]; };                      // 17 B
struct orc_block_iq1_s { uint16_t d; uint8_t qs[32]; uint16_t qh[8]; };     // 50 B
#pragma pack(pop)

static_assert(sizeof(orc_block_q8_0) == 34, "q8_0");
static_assert(sizeof(orc_block_q8_K) == 292, "q8_K");
static_assert(sizeof(orc_block_q4_K) == 144, "q4_K");
static_assert(sizeof(orc_block_q6_K) == 210, "q6_K");
static_assert(sizeof(orc_block_mxfp4) == 17, "mxfp4");
static_assert(sizeof(orc_block_iq1_s) == 50, "iq1_s");

int orc_block_bytes(int type) {
    switch (type) {
        case ORC_Q8_0: return 34;
        case ORC_Q8_K: return 292;
        case ORC_Q4_K: return 144;
        case ORC_Q6_K: return 210;
        case ORC_MXFP4: return 17;
        case ORC_IQ1_S: return 50;
        default: return 0;
    }
}

int orc_block_elems(int type) {
    switch (type) {
        case ORC_Q8_0: case ORC_MXFP4: return 32;
        case ORC_Q8_K: case ORC_Q4_K: case ORC_Q6_K: case ORC_IQ1_S: return 256;
        default: return 0;
    }
}

// activation type of the CPU path for a weight type (type_traits_cpu
// vec_dot_type; the reference's map is diff:166-178)
int orc_vec_dot_type(int type) {
    switch (type) {
        case ORC_Q8_0: case ORC_MXFP4: return ORC_Q8_0;
        default: return ORC_Q8_K;
    }
}

// ------------------------------------------------------------- conversions

static inline uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// binary16 -> binary32, exact (IEEE 754 widening)
float orc_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ffu;
    if (exp == 0x1f) return u2f(sign | 0x7f800000u | (man << 13));
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        // subnormal half: value = man * 2^-24, exact in binary32
        int e = -1;
        do { ++e; man <<= 1; } while ((man & 0x400u) == 0);
        man &= 0x3ffu;
        return u2f(sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13));
    }
    return u2f(sign | ((exp + 112) << 23) | (man << 13));
}

// binary32 -> binary16, round to nearest even (IEEE 754 narrowing; this is
// what the NEON fcvt and the reference's "(half) d" do, diff:1008, 1035)
uint16_t orc_fp32_to_fp16(float f) {
    const uint32_t x = f2u(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {  // inf or nan
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u | ((ax >> 13) & 0x3ffu) : 0));
    }
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to >= 65520 -> inf
    if (ax < 0x38800000u) {  // below the smallest normal half (2^-14): subnormal or zero
        if (ax < 0x33000000u) return (uint16_t)sign;  // < 2^-25: rounds to zero (ties at 2^-25 -> even 0)
        const uint32_t e = ax >> 23;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126 - e;  // value = m * 2^(e-150); half ulp 2^-24 -> m >> (126-e) ... see below
        // result in units of 2^-24: m * 2^(e-150+24) = m >> (126 - e)
        const uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        uint32_t r = q;
        if (rem > half || (rem == half && (q & 1u))) ++r;
        return (uint16_t)(sign | r);
    }
    // normal range
    uint32_t h = ((ax >> 13) - (112u << 10));
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

// round to nearest even for |v| < 2^22, the way ggml's nearest_int and NEON's
// fcvtns agree in range (diff:399-401, 1005)
static inline int rne_int(float v) {
    const float t = v + 12582912.0f;  // 1.5 * 2^23
    return (int)(f2u(t) & 0x007fffffu) - 0x00400000;
}

// ------------------------------------------------- activation quantizers

// quantize_row_q8_0, NEON order (diff:1000-1007): amax over the 32 elements
// (order-free), d = amax/127 (IEEE divide), id = d ? 1/d : 0, q = RNE(x*id)
// narrowed to int8, d stored as binary16 RNE.
void orc_quantize_q8_0(const float * x, int64_t n, void * vy) {
    orc_block_q8_0 * y = (orc_block_q8_0 *)vy;
    for (int64_t ib = 0; ib < n / 32; ++ib) {
        const float * xb = x + ib * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float a = std::fabs(xb[j]);
            if (a > amax) amax = a;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float p = xb[j] * id;
            y[ib].qs[j] = (int8_t)rne_int(p);
        }
        y[ib].d = orc_fp32_to_fp16(d);
    }
}

// quantize_row_q8_K (diff:335-345, 364-427): first strict max of |x| wins
// (ties keep the smaller index), iscale = -127/max (IEEE divide),
// q = min(127, RNE(iscale*x)), bsums over groups of 16, d = 1/iscale.
// An all-zero superblock stores d = 0, zero quants and zero sums.
void orc_quantize_q8_K(const float * x, int64_t n, void * vy) {
    orc_block_q8_K * y = (orc_block_q8_K *)vy;
    for (int64_t ib = 0; ib < n / 256; ++ib) {
        const float * xb = x + ib * 256;
        float amax = 0.0f, vmax = 0.0f;
        for (int j = 0; j < 256; ++j) {
            const float a = std::fabs(xb[j]);
            if (a > amax) { amax = a; vmax = xb[j]; }
        }
        if (amax == 0.0f) {
            y[ib].d = 0.0f;
            std::memset(y[ib].qs, 0, 256);
            std::memset(y[ib].bsums, 0, sizeof(y[ib].bsums));
            continue;
        }
        const float iscale = -127.0f / vmax;
        for (int j = 0; j < 256; ++j) {
            const int v = rne_int(iscale * xb[j]);
            y[ib].qs[j] = (int8_t)std::min(127, v);
        }
        for (int g = 0; g < 16; ++g) {
            int s = 0;
            for (int j = 0; j < 16; ++j) s += y[ib].qs[16 * g + j];
            y[ib].bsums[g] = (int16_t)s;
        }
        y[ib].d = 1.0f / iscale;
    }
}

// ------------------------------------------------------------ dot products

// ggml_vec_dot_q8_0_q8_0, NEON nrc=1 order (diff:1049-1054, 1074-1163):
// blocks in pairs; per block four 8-element integer partials
// p[l] = sum_m x[4l+m]y[4l+m] + x[16+4l+m]y[16+4l+m]; per block
// scale = fp16(x.d)*fp16(y.d); acc[l] = fma((float)p[l], scale, acc[l]) with
// separate even/odd accumulators; final ((e0+e1)+(e2+e3)) + ((o0+o1)+(o2+o3)).
static float dot_q8_0(int64_t n, const void * vx, const void * vy) {
    const orc_block_q8_0 * x = (const orc_block_q8_0 *)vx;
    const orc_block_q8_0 * y = (const orc_block_q8_0 *)vy;
    const int64_t nb = n / 32;
    float ae[4] = {0, 0, 0, 0}, ao[4] = {0, 0, 0, 0};
    for (int64_t ib = 0; ib + 1 < nb; ib += 2) {
        for (int half = 0; half < 2; ++half) {
            const orc_block_q8_0 & xb = x[ib + half];
            const orc_block_q8_0 & yb = y[ib + half];
            const float s = orc_fp16_to_fp32(xb.d) * orc_fp16_to_fp32(yb.d);
            float * acc = half == 0 ? ae : ao;
            for (int l = 0; l < 4; ++l) {
                int p = 0;
                for (int m = 0; m < 4; ++m) {
                    p += (int)xb.qs[4 * l + m] * (int)yb.qs[4 * l + m];
                    p += (int)xb.qs[16 + 4 * l + m] * (int)yb.qs[16 + 4 * l + m];
                }
                acc[l] = std::fma((float)p, s, acc[l]);
            }
        }
    }
    const float se = (ae[0] + ae[1]) + (ae[2] + ae[3]);
    const float so = (ao[0] + ao[1]) + (ao[2] + ao[3]);
    return se + so;
}

// GGML_E8M0_TO_FP32_HALF: 2^(e-128) from bits, subnormal for e < 2 (diff:1176-1180)
static inline float e8m0_half(uint8_t e) {
    const uint32_t bits = e < 2 ? (0x00200000u << e) : ((uint32_t)(e - 1) << 23);
    return u2f(bits);
}

static const int8_t kvalues_mxfp4[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

// ggml_vec_dot_mxfp4_q8_0, NEON order (diff:1167-1174, 1209-1240): pairs;
// sc = fp16(y.d) * e8m0_half(x.e); t = fma(sc_e, (float)p_e, sc_o*(float)p_o);
// sumf = sumf + t.
static float dot_mxfp4(int64_t n, const void * vx, const void * vy) {
    const orc_block_mxfp4 * x = (const orc_block_mxfp4 *)vx;
    const orc_block_q8_0 * y = (const orc_block_q8_0 *)vy;
    const int64_t nb = n / 32;
    float sumf = 0.0f;
    for (int64_t ib = 0; ib + 1 < nb; ib += 2) {
        int p[2] = {0, 0};
        float sc[2];
        for (int half = 0; half < 2; ++half) {
            const orc_block_mxfp4 & xb = x[ib + half];
            const orc_block_q8_0 & yb = y[ib + half];
            int s = 0;
            for (int j = 0; j < 16; ++j) {
                s += (int)yb.qs[j] * (int)kvalues_mxfp4[xb.qs[j] & 0xf];
                s += (int)yb.qs[j + 16] * (int)kvalues_mxfp4[xb.qs[j] >> 4];
            }
            p[half] = s;
            sc[half] = orc_fp16_to_fp32(yb.d) * e8m0_half(xb.e);
        }
        const float t = std::fma(sc[0], (float)p[0], sc[1] * (float)p[1]);
        sumf = sumf + t;
    }
    return sumf;
}

// ggml_vec_dot_q4_K_q8_K, NEON nrc=1 order (diff:1254-1259, 1300-1357):
// q8sums[j] = bsums[2j]+bsums[2j+1] (int16); prod = sum_j q8sums[j]*min[j];
// sumi = sum_j p1_j*sc[2j] + p2_j*sc[2j+1]; per superblock
// sumf = fma(-(y.d*fp16(x.dmin)), prod, sumf); sumf = fma(y.d*fp16(x.d), sumi, sumf).
static void q4k_scales_mins(const uint8_t * s, int sc[8], int mn[8]) {
    for (int j = 0; j < 4; ++j) {
        sc[j] = s[j] & 63;
        mn[j] = s[j + 4] & 63;
        sc[j + 4] = (s[j + 8] & 0x0f) | ((s[j] >> 6) << 4);
        mn[j + 4] = (s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4);
    }
}

static float dot_q4_K(int64_t n, const void * vx, const void * vy) {
    const orc_block_q4_K * x = (const orc_block_q4_K *)vx;
    const orc_block_q8_K * y = (const orc_block_q8_K *)vy;
    float sumf = 0.0f;
    for (int64_t i = 0; i < n / 256; ++i) {
        int sc[8], mn[8];
        q4k_scales_mins(x[i].scales, sc, mn);
        int prod = 0;
        for (int j = 0; j < 8; ++j) {
            const int q8s = (int16_t)(y[i].bsums[2 * j] + y[i].bsums[2 * j + 1]);
            prod += q8s * mn[j];
        }
        int sumi1 = 0, sumi2 = 0;
        for (int j = 0; j < 4; ++j) {
            int p1 = 0, p2 = 0;
            for (int m = 0; m < 32; ++m) {
                p1 += (int)(x[i].qs[32 * j + m] & 0xf) * (int)y[i].qs[64 * j + m];
                p2 += (int)(x[i].qs[32 * j + m] >> 4) * (int)y[i].qs[64 * j + 32 + m];
            }
            sumi1 += p1 * sc[2 * j];
            sumi2 += p2 * sc[2 * j + 1];
        }
        const float dmin = -(y[i].d * orc_fp16_to_fp32(x[i].dmin));
        const float d = y[i].d * orc_fp16_to_fp32(x[i].d);
        sumf = std::fma(dmin, (float)prod, sumf);
        sumf = std::fma(d, (float)(sumi1 + sumi2), sumf);
    }
    return sumf;
}

// element e (0..255) of a q6_K superblock as its unsigned 6-bit code
// (layout per gguf-py Q6_K.dequantize_blocks and diff:1411-1424)
static inline int q6k_code(const orc_block_q6_K & b, int e) {
    const int h = e / 128, r = e % 128;
    const int lo = r < 64 ? (b.ql[64 * h + r] & 0xf) : (b.ql[64 * h + r - 64] >> 4);
    const int hi = (b.qh[32 * h + (r % 32)] >> (2 * (r / 32))) & 3;
    return lo | (hi << 4);
}

// ggml_vec_dot_q6_K_q8_K, NEON nrc=1 order (diff:1366-1370, 1393-1446):
// isum_mins = sum_g bsums[g]*sc[g]; isum = sum_g sc[g] * sum_m code*q8;
// sumf = fma(y.d*fp16(x.d), (float)(isum - 32*isum_mins), sumf).
static float dot_q6_K(int64_t n, const void * vx, const void * vy) {
    const orc_block_q6_K * x = (const orc_block_q6_K *)vx;
    const orc_block_q8_K * y = (const orc_block_q8_K *)vy;
    float sumf = 0.0f;
    for (int64_t i = 0; i < n / 256; ++i) {
        int isum_mins = 0;
        for (int g = 0; g < 16; ++g) isum_mins += (int)y[i].bsums[g] * (int)x[i].scales[g];
        int isum = 0;
        for (int g = 0; g < 16; ++g) {
            int pg = 0;
            for (int m = 0; m < 16; ++m) pg += q6k_code(x[i], 16 * g + m) * (int)y[i].qs[16 * g + m];
            isum += pg * (int)x[i].scales[g];
        }
        const float d = y[i].d * orc_fp16_to_fp32(x[i].d);
        sumf = std::fma(d, (float)(isum - 32 * isum_mins), sumf);
    }
    return sumf;
}

// iq1s grid: 2048 entries of 8 ternary values, installed by the test harness
// from the gguf-py table (orc_set_iq1s_grid); the oracle never retypes it.
static int8_t g_iq1s_grid[2048][8];
static int g_iq1s_grid_set = 0;

void orc_set_iq1s_grid(const int8_t * grid /* 2048*8 */) {
    std::memcpy(g_iq1s_grid, grid, sizeof(g_iq1s_grid));
    g_iq1s_grid_set = 1;
}

int orc_iq1s_grid_ready(void) { return g_iq1s_grid_set; }

// ggml_vec_dot_iq1_s_q8_K, NEON order (diff:335-345, 458-510):
// per 32-element sub-block: grid index = qs | ((qh >> 3l) & 7) << 8 per group
// of 8, ls = 2*((qh>>12)&7)+1, delta sign from qh bit 15;
// sumi1/sumi2 = sum p*ls; sumi3 = sum (bsum pair)*ls*sign;
// expr = fma((float)sumi3, 0.125, (float)(sumi1+sumi2));
// sumf = fma(y.d*fp16(x.d), expr, sumf).
static float dot_iq1_s(int64_t n, const void * vx, const void * vy) {
    const orc_block_iq1_s * x = (const orc_block_iq1_s *)vx;
    const orc_block_q8_K * y = (const orc_block_q8_K *)vy;
    float sumf = 0.0f;
    for (int64_t i = 0; i < n / 256; ++i) {
        int sumi1 = 0, sumi2 = 0, sumi3 = 0;
        for (int ib = 0; ib < 8; ib += 2) {
            int p[2] = {0, 0};
            for (int h = 0; h < 2; ++h) {
                const int sb = ib + h;
                const uint16_t qh = x[i].qh[sb];
                for (int l = 0; l < 4; ++l) {
                    const int gi = x[i].qs[4 * sb + l] | (((qh >> (3 * l)) & 7) << 8);
                    for (int m = 0; m < 8; ++m) p[h] += (int)g_iq1s_grid[gi][m] * (int)y[i].qs[32 * sb + 8 * l + m];
                }
            }
            const int ls1 = 2 * ((x[i].qh[ib] >> 12) & 7) + 1;
            const int ls2 = 2 * ((x[i].qh[ib + 1] >> 12) & 7) + 1;
            sumi1 += p[0] * ls1;
            sumi2 += p[1] * ls2;
            sumi3 += ((int)y[i].bsums[2 * ib] + (int)y[i].bsums[2 * ib + 1]) * ls1 * ((x[i].qh[ib] & 0x8000) ? -1 : 1)
                   + ((int)y[i].bsums[2 * ib + 2] + (int)y[i].bsums[2 * ib + 3]) * ls2 * ((x[i].qh[ib + 1] & 0x8000) ? -1 : 1);
        }
        const float d = y[i].d * orc_fp16_to_fp32(x[i].d);
        const float expr = std::fma((float)sumi3, 0.125f, (float)(sumi1 + sumi2));
        sumf = std::fma(d, expr, sumf);
    }
    return sumf;
}

// one row of weights (type) against one quantized activation row
float orc_vec_dot(int type, int64_t n, const void * x, const void * y) {
    switch (type) {
        case ORC_Q8_0: return dot_q8_0(n, x, y);
        case ORC_MXFP4: return dot_mxfp4(n, x, y);
        case ORC_Q4_K: return dot_q4_K(n, x, y);
        case ORC_Q6_K: return dot_q6_K(n, x, y);
        case ORC_IQ1_S: return dot_iq1_s(n, x, y);
        default: return std::nanf("");
    }
}

// ----------------------------------------------------------------- dequant
// float dequantization of one row (used only to pin block decoding against
// the gguf-py dequantizers; the arithmetic path never dequantizes)
void orc_dequantize_row(int type, const void * vx, float * out, int64_t n) {
    const int64_t nb = n / orc_block_elems(type);
    for (int64_t i = 0; i < nb; ++i) {
        float * o = out + i * orc_block_elems(type);
        switch (type) {
            case ORC_Q8_0: {
                const orc_block_q8_0 & b = ((const orc_block_q8_0 *)vx)[i];
                const float d = orc_fp16_to_fp32(b.d);
                for (int j = 0; j < 32; ++j) o[j] = (float)b.qs[j] * d;
            } break;
            case ORC_MXFP4: {
                const orc_block_mxfp4 & b = ((const orc_block_mxfp4 *)vx)[i];
                const float d = e8m0_half(b.e);
                for (int j = 0; j < 16; ++j) {
                    o[j] = d * (float)kvalues_mxfp4[b.qs[j] & 0xf];
                    o[j + 16] = d * (float)kvalues_mxfp4[b.qs[j] >> 4];
                }
            } break;
            case ORC_Q4_K: {
                const orc_block_q4_K & b = ((const orc_block_q4_K *)vx)[i];
                int sc[8], mn[8];
                q4k_scales_mins(b.scales, sc, mn);
                const float d = orc_fp16_to_fp32(b.d), dm = orc_fp16_to_fp32(b.dmin);
                for (int j = 0; j < 4; ++j) {
                    const float d1 = d * (float)sc[2 * j], m1 = dm * (float)mn[2 * j];
                    const float d2 = d * (float)sc[2 * j + 1], m2 = dm * (float)mn[2 * j + 1];
                    for (int m = 0; m < 32; ++m) {
                        o[64 * j + m] = d1 * (float)(b.qs[32 * j + m] & 0xf) - m1;
                        o[64 * j + 32 + m] = d2 * (float)(b.qs[32 * j + m] >> 4) - m2;
                    }
                }
            } break;
            case ORC_Q6_K: {
                const orc_block_q6_K & b = ((const orc_block_q6_K *)vx)[i];
                const float d = orc_fp16_to_fp32(b.d);
                for (int e = 0; e < 256; ++e) {
                    o[e] = (d * (float)b.scales[e / 16]) * (float)(q6k_code(b, e) - 32);
                }
            } break;
            case ORC_IQ1_S: {
                const orc_block_iq1_s & b = ((const orc_block_iq1_s *)vx)[i];
                const float d = orc_fp16_to_fp32(b.d);
                for (int sb = 0; sb < 8; ++sb) {
                    const float dl = d * (float)(2 * ((b.qh[sb] >> 12) & 7) + 1);
                    const float delta = (b.qh[sb] & 0x8000) ? -0.125f : 0.125f;
                    for (int l = 0; l < 4; ++l) {
                        const int gi = b.qs[4 * sb + l] | (((b.qh[sb] >> (3 * l)) & 7) << 8);
                        for (int m = 0; m < 8; ++m) o[32 * sb + 8 * l + m] = dl * ((float)g_iq1s_grid[gi][m] + delta);
                    }
                }
            } break;
            default: break;
        }
    }
}

// -------------------------------------------------------------------- expf
// One expf shared by the oracle and the device (restated identically in the
// CUDA sources). Method: n = RNE(x*log2(e)); r = x - n*ln2 with ln2 split into
// a 16-bit head (exact products for |n| <= 256) and a tail (Cody & Waite,
// "Software Manual for the Elementary Functions", 1980); e^r by the degree-7
// Taylor polynomial in Horner form with fused multiply-adds; scaling by 2^n
// through the exponent field, in two exact steps when the result is
// subnormal. Saturates to +inf above 88.72283935546875 and to +0 below
// -103.97208; NaN propagates.
static const float EXPF_LOG2E = 1.44269502162933349609375f;   // RN(log2 e)
static const float EXPF_LN2_HI = 0.693145751953125f;          // 0x3f317200, 15 significant bits
static const float EXPF_LN2_LO = 1.428606765330187045e-06f;   // RN(ln2 - LN2_HI)

float orc_expf(float x) {
    if (x != x) return x + x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.972084045410156f) return 0.0f;
    const float t = std::fma(x, EXPF_LOG2E, 12582912.0f);
    const float n = t - 12582912.0f;
    float r = std::fma(-n, EXPF_LN2_HI, x);
    r = std::fma(-n, EXPF_LN2_LO, r);
    // 1/k! rounded to binary32, k = 7..2
    float p = std::fma(r, 1.98412701138295233249664306640625e-04f, 1.3888889225199818611145019531250e-03f);
    p = std::fma(p, r, 8.3333337679505348205566406250000e-03f);
    p = std::fma(p, r, 4.1666667908430099487304687500000e-02f);
    p = std::fma(p, r, 1.6666667163372039794921875000000e-01f);
    p = std::fma(p, r, 0.5f);
    p = std::fma(p, r, 1.0f);
    p = std::fma(p, r, 1.0f);
    const int ni = (int)n;
    if (ni >= -125) {
        if (ni > 127) {  // p < 2 and result finite: split 2^ni = 2 * 2^(ni-1)
            return (p * 2.0f) * u2f((uint32_t)(ni - 1 + 127) << 23);
        }
        return p * u2f((uint32_t)(ni + 127) << 23);
    }
    // subnormal range: two scalings, the first exact
    return (p * u2f((uint32_t)(ni + 64 + 127) << 23)) * u2f((uint32_t)(-64 + 127) << 23);
}

void orc_expf_many(const float * x, float * y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = orc_expf(x[i]);
}

// ------------------------------------------------------------ activations

// The exp inside the activations: this library's orc_expf (the default, the
// one the device shares) or the host C library's expf (orc_act_exp_libm(1)),
// for measuring how far layer outputs move when the exp is swapped.
static std::atomic<int> g_act_exp_libm{0};
void orc_act_exp_libm(int on) { g_act_exp_libm.store(on ? 1 : 0); }
static inline float act_exp(float x) { return g_act_exp_libm.load(std::memory_order_relaxed) ? std::exp(x) : orc_expf(x); }

// SwiGLU as ggml's scalar CPU form: silu(g) * u with silu(g) = g / (1 + exp(-g))
void orc_swiglu(const float * g, const float * u, float * out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        const float s = g[i] / (1.0f + act_exp(-g[i]));
        out[i] = s * u[i];
    }
}

// SWIGLU_OAI semantics (diff:1461-1465, 1911-1918): x = min(g, limit) with
// std::min's ordered comparison, y = clamp(u, -limit, limit),
// out = x / (1 + exp(alpha * -x)) * (y + 1)
void orc_swiglu_oai(const float * g, const float * u, float * out, int64_t n, float alpha, float limit) {
    for (int64_t i = 0; i < n; ++i) {
        const float x = limit < g[i] ? limit : g[i];
        const float y = u[i] < -limit ? -limit : (limit < u[i] ? limit : u[i]);
        const float glu = x / (1.0f + act_exp(alpha * (-x)));
        out[i] = glu * (y + 1.0f);
    }
}

// weighted combine of build_moe_ffn: each expert output scaled by its router
// weight (ggml_mul, one rounding), then summed in slot order 0..k-1 by a chain
// of ggml_add (one rounding each). y is [H, k, T], w is [k, T], out is [H, T].
void orc_combine(const float * y, const float * w, float * out, int64_t H, int64_t k, int64_t T) {
    for (int64_t t = 0; t < T; ++t) {
        for (int64_t h = 0; h < H; ++h) {
            float acc = y[(t * k + 0) * H + h] * w[t * k + 0];
            for (int64_t s = 1; s < k; ++s) {
                const float p = y[(t * k + s) * H + h] * w[t * k + s];
                acc = acc + p;
            }
            out[t * H + h] = acc;
        }
    }
}

// ------------------------------------------------------------ mul_mat_id
// ggml_mul_mat_id on the CPU: src1 rows are first quantized to the weight
// type's vec_dot_type, then every output element is one vec_dot (nrc = 1).
//   as   : expert weights, row r of expert e at as + e*nb02 + r*nb01
//   b    : f32 [ne10, ne11, ne12] with byte strides nb11, nb12 (ne11 is 1 or k)
//   ids  : i32 [k, T] with byte stride nbi1 between tokens
//   dst  : f32 [ne01, k, T], contiguous
// Output element (r, s, t) = vec_dot(row r of expert ids[s,t], q(b[:, s % ne11, t])).
int orc_mul_mat_id(int type, const void * as, int64_t ne00, int64_t ne01, int64_t nb01, int64_t nb02, int64_t n_as,
                   const float * b, int64_t ne11, int64_t ne12, int64_t nb11, int64_t nb12,
                   const int32_t * ids, int64_t k, int64_t nbi1,
                   float * dst, int nthreads) {
    const int vdt = orc_vec_dot_type(type);
    const int64_t qrow = (ne00 / orc_block_elems(vdt)) * orc_block_bytes(vdt);
    std::vector<uint8_t> q((size_t)(qrow * ne11 * ne12));
    for (int64_t t = 0; t < ne12; ++t) {
        for (int64_t i = 0; i < ne11; ++i) {
            const float * src = (const float *)((const char *)b + t * nb12 + i * nb11);
            void * yq = q.data() + (t * ne11 + i) * qrow;
            if (vdt == ORC_Q8_0) orc_quantize_q8_0(src, ne00, yq); else orc_quantize_q8_K(src, ne00, yq);
        }
    }
    for (int64_t t = 0; t < ne12; ++t) {
        for (int64_t s = 0; s < k; ++s) {
            const int32_t e = *(const int32_t *)((const char *)ids + t * nbi1 + s * 4);
            if (e < 0 || e >= n_as) return -1;
        }
    }
    // every output element is computed independently, so splitting rows over
    // threads cannot change a bit
    const int64_t total = ne12 * k * ne01;
    std::atomic<int64_t> next{0};
    auto worker = [&]() {
        const int64_t chunk = 64;
        for (;;) {
            const int64_t begin = next.fetch_add(chunk);
            if (begin >= total) break;
            const int64_t end = std::min(total, begin + chunk);
            for (int64_t idx = begin; idx < end; ++idx) {
                const int64_t pr = idx / ne01, r = idx % ne01;
                const int64_t t = pr / k, s = pr % k;
                const int32_t e = *(const int32_t *)((const char *)ids + t * nbi1 + s * 4);
                const uint8_t * yq = q.data() + (t * ne11 + (s % ne11)) * qrow;
                dst[pr * ne01 + r] = orc_vec_dot(type, ne00, (const char *)as + e * nb02 + r * nb01, yq);
            }
        }
    };
    const int nt = nthreads > 1 ? nthreads : 1;
    std::vector<std::thread> pool;
    for (int i = 1; i < nt; ++i) pool.emplace_back(worker);
    worker();
    for (auto & th : pool) th.join();
    return 0;
}

// ------------------------------------------------------------- MoE layer
// One routed-expert FFN layer as the patched llama.cpp graph runs it
// (diff:2140-2191): gate = mul_mat_id(gate_exps, x, ids), up = likewise,
// act = swiglu(gate, up) (or SWIGLU_OAI), down = mul_mat_id(down_exps, act, ids)
// with ne11 = k, then the weighted combine in slot order.
// Expert e's record starts at records + e*record_bytes and holds
// down | gate | up (src/h4/h4-metal-arena-probe.cpp:143-145).
struct orc_layer_desc {
    int32_t type_gate, type_up, type_down;
    int32_t act;          // 0 = SwiGLU, 1 = SWIGLU_OAI
    float alpha, limit;   // SWIGLU_OAI parameters
    int64_t H, I;         // hidden, expert intermediate
    int64_t off_gate, off_up;  // byte offsets inside a record (down at 0)
    int64_t record_bytes;
    int64_t n_experts;
};

static int64_t row_bytes(int type, int64_t n) { return (n / orc_block_elems(type)) * orc_block_bytes(type); }

int orc_moe_layer(const orc_layer_desc * L, const void * records,
                  const float * x /* [H, T] */, const int32_t * ids /* [k, T] */, const float * w /* [k, T] */,
                  int64_t k, int64_t T, float * out /* [H, T] */, int nthreads) {
    const int64_t H = L->H, I = L->I;
    std::vector<float> g((size_t)(I * k * T)), u((size_t)(I * k * T)), a((size_t)(I * k * T)), d((size_t)(H * k * T));
    const char * base = (const char *)records;
    int rc = orc_mul_mat_id(L->type_gate, base + L->off_gate, H, I, row_bytes(L->type_gate, H), L->record_bytes, L->n_experts,
                            x, 1, T, H * 4, H * 4, ids, k, k * 4, g.data(), nthreads);
    if (rc) return rc;
    rc = orc_mul_mat_id(L->type_up, base + L->off_up, H, I, row_bytes(L->type_up, H), L->record_bytes, L->n_experts,
                        x, 1, T, H * 4, H * 4, ids, k, k * 4, u.data(), nthreads);
    if (rc) return rc;
    if (L->act == 1) orc_swiglu_oai(g.data(), u.data(), a.data(), I * k * T, L->alpha, L->limit);
    else orc_swiglu(g.data(), u.data(), a.data(), I * k * T);
    rc = orc_mul_mat_id(L->type_down, base, I, H, row_bytes(L->type_down, I), L->record_bytes, L->n_experts,
                        a.data(), k, T, I * 4, I * k * 4, ids, k, k * 4, d.data(), nthreads);
    if (rc) return rc;
    orc_combine(d.data(), w, out, H, k, T);
    return 0;
}

// ------------------------------------------------------------ synthetic data
// Restatement of the product's seeded generator (gx_synth_normal,
// gx_synth_weights): splitmix64 counters (Steele, Lea & Flood 2014), N(0,1)
// as the standardised sum of four 16-bit uniforms (Irwin-Hall, n = 4), and the
// synthetic weight quantizers. Parity tests check that the device writes the
// same bytes.
static inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t orc_synth_key(uint64_t seed, uint64_t stream_id) {
    return splitmix64(seed ^ splitmix64(stream_id + 0x632BE59BD9B4E019ull));
}

static inline uint64_t synth_bits(uint64_t key, uint64_t i) { return splitmix64(key + i * 0xD1B54A32D192ED03ull); }

static inline float synth_normal(uint64_t key, uint64_t i, float sigma) {
    const uint64_t b = synth_bits(key, i);
    const int S = (int)(b & 0xffff) + (int)((b >> 16) & 0xffff) + (int)((b >> 32) & 0xffff) + (int)((b >> 48) & 0xffff);
    const float z = (float)(S - 131070) * 2.642899744e-05f;
    return z * sigma;
}

void orc_synth_normal(float * dst, int64_t n, uint64_t seed, uint64_t stream_id, float sigma) {
    const uint64_t key = orc_synth_key(seed, stream_id);
    for (int64_t i = 0; i < n; ++i) dst[i] = synth_normal(key, (uint64_t)i, sigma);
}

static inline float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

int orc_synth_weights(int type, void * vdst, int64_t ne00, int64_t n_rows, uint64_t seed, uint64_t stream_id, float sigma) {
    const int be = orc_block_elems(type), bb = orc_block_bytes(type);
    if (be == 0 || ne00 % be) return -1;
    const uint64_t key = orc_synth_key(seed, stream_id);
    const int64_t bpr = ne00 / be, nblk = bpr * n_rows;
    uint8_t * dst = (uint8_t *)vdst;
    for (int64_t bi = 0; bi < nblk; ++bi) {
        uint8_t * o = dst + bi * bb;
        const int64_t row = bi / bpr, col = bi % bpr;
        const uint64_t e0 = (uint64_t)(row * ne00 + col * be);
        if (type == ORC_Q8_0) {
            float x[32];
            for (int j = 0; j < 32; ++j) x[j] = synth_normal(key, e0 + j, sigma);
            orc_quantize_q8_0(x, 32, o);
        } else if (type == ORC_Q4_K) {
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
                scf[sb] = (mx - mn) / 15.0f;
                mnf[sb] = -mn;
            }
            float maxsc = 0.0f, maxmn = 0.0f;
            for (int sb = 0; sb < 8; ++sb) {
                if (scf[sb] > maxsc) maxsc = scf[sb];
                if (mnf[sb] > maxmn) maxmn = mnf[sb];
            }
            const uint16_t d16 = orc_fp32_to_fp16(maxsc / 63.0f), dm16 = orc_fp32_to_fp16(maxmn / 63.0f);
            const float df = orc_fp16_to_fp32(d16), dmf = orc_fp16_to_fp32(dm16);
            int sc[8], mq[8];
            uint8_t q[256];
            for (int sb = 0; sb < 8; ++sb) {
                sc[sb] = df > 0.0f ? rne_int(clampf(scf[sb] / df, 0.0f, 63.0f)) : 0;
                mq[sb] = dmf > 0.0f ? rne_int(clampf(mnf[sb] / dmf, 0.0f, 63.0f)) : 0;
                const float ds = df * (float)sc[sb], dm = dmf * (float)mq[sb];
                for (int j = 0; j < 32; ++j)
                    q[32 * sb + j] = ds > 0.0f ? (uint8_t)rne_int(clampf((x[32 * sb + j] + dm) / ds, 0.0f, 15.0f)) : 0;
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
        } else if (type == ORC_Q6_K) {
            float x[256];
            for (int j = 0; j < 256; ++j) x[j] = synth_normal(key, e0 + j, sigma);
            float scf[16], maxs = 0.0f;
            for (int g = 0; g < 16; ++g) {
                float amax = 0.0f;
                for (int j = 0; j < 16; ++j) {
                    const float a = std::fabs(x[16 * g + j]);
                    if (a > amax) amax = a;
                }
                scf[g] = amax / 31.0f;
                if (scf[g] > maxs) maxs = scf[g];
            }
            const uint16_t d16 = orc_fp32_to_fp16(maxs / 127.0f);
            const float df = orc_fp16_to_fp32(d16);
            std::memset(o, 0, 208);
            for (int g = 0; g < 16; ++g) {
                const int sc = df > 0.0f ? rne_int(clampf(scf[g] / df, 0.0f, 127.0f)) : 0;
                o[192 + g] = (uint8_t)(int8_t)sc;
                const float ds = df * (float)sc;
                for (int j = 0; j < 16; ++j) {
                    const int e = 16 * g + j;
                    const int qv = ds > 0.0f ? rne_int(clampf(x[e] / ds, -32.0f, 31.0f)) : 0;
                    const int code = qv + 32;
                    const int hh = e / 128, r = e % 128;
                    o[64 * hh + (r % 64)] |= (uint8_t)((code & 15) << (r < 64 ? 0 : 4));
                    o[128 + 32 * hh + (r % 32)] |= (uint8_t)((code >> 4) << (2 * (r / 32)));
                }
            }
            o[208] = (uint8_t)(d16 & 0xff);
            o[209] = (uint8_t)(d16 >> 8);
        } else if (type == ORC_MXFP4) {
            const uint64_t w0 = synth_bits(key, 3 * (uint64_t)bi), w1 = synth_bits(key, 3 * (uint64_t)bi + 1),
                           w2 = synth_bits(key, 3 * (uint64_t)bi + 2);
            o[0] = (uint8_t)(118 + (w0 & 7));
            for (int j = 0; j < 8; ++j) { o[1 + j] = (uint8_t)(w1 >> (8 * j)); o[9 + j] = (uint8_t)(w2 >> (8 * j)); }
        } else if (type == ORC_IQ1_S) {
            uint64_t w[7];
            for (int j = 0; j < 7; ++j) w[j] = synth_bits(key, 8 * (uint64_t)bi + j);
            const uint16_t d16 = (uint16_t)(0x1400u | (w[0] & 0x3ffu));
            o[0] = (uint8_t)(d16 & 0xff); o[1] = (uint8_t)(d16 >> 8);
            for (int j = 0; j < 32; ++j) o[2 + j] = (uint8_t)(w[1 + j / 8] >> (8 * (j % 8)));
            for (int j = 0; j < 16; ++j) o[34 + j] = (uint8_t)(w[5 + j / 8] >> (8 * (j % 8)));
        } else {
            return -1;
        }
    }
    return 0;
}


// ------------------------------------------------------------------ router
// The router step of upstream llama.cpp's build_moe_ffn (third-party; the
// reference pins commit da5b4486 in patches/UPSTREAM-COMMIT.txt and patches
// the function right after it, patches/galactus-h4-llamacpp.diff:2124-2150).
// Restated from the published graph of that function:
//   probs = soft_max(logits) | sigmoid(logits) | logits (SOFTMAX_WEIGHT);
//   selection = probs + exp_probs_b (when a bias is given);
//   group-limited selection: score of a group = sum of its two best
//     selection values, the n_group_used best groups kept, others -inf;
//   selected = the first k of the descending argsort of selection (the view
//     the remap node reads, docs/STUDY.md:74); ties go to the lower id (the
//     argsort's comparator leaves them unordered, so this is our choice);
//   weights = probs at the selected ids; SOFTMAX_WEIGHT: soft_max over the k;
//     norm_w: divided by clamp(sum_rows, 6.103515625e-5, inf); scale_w: times
//     w_scale.
// soft_max is ggml's arm64 CPU order: max, e = exp(x - max) (the library's
// expf above, in place of ggml's vector exp), float sums of four consecutive
// e's as ((e0+e1)+(e2+e3)) (vaddvq_f32) accumulated in double in order, the
// tail one by one, then every e times (float)(1.0/sum). sum_rows accumulates
// in double in order (the non-Accelerate form); sigmoid is 1/(1+exp(-x)).
struct orc_router_desc {
    int32_t gating, n_expert, n_expert_used, n_groups, n_group_used, norm_w, scale_w;
    float w_scale;
};

static void router_soft_max(const float * x, float * y, int n) {
    float m = -INFINITY;
    for (int i = 0; i < n; ++i) m = x[i] > m ? x[i] : m;
    double sum = 0.0;
    int i = 0;
    for (; i + 3 < n; i += 4) {
        float v[4];
        for (int j = 0; j < 4; ++j) v[j] = orc_expf(x[i + j] - m);
        for (int j = 0; j < 4; ++j) y[i + j] = v[j];
        sum += (double)((v[0] + v[1]) + (v[2] + v[3]));
    }
    for (; i < n; ++i) {
        const float v = orc_expf(x[i] - m);
        y[i] = v;
        sum += (double)v;
    }
    const float inv = (float)(1.0 / sum);
    for (i = 0; i < n; ++i) y[i] = y[i] * inv;
}

static inline bool router_better(float a, int ia, float b, int ib) { return a > b || (a == b && ia < ib); }

int orc_router_valid(const orc_router_desc * d) {
    if (d == nullptr) return 0;
    const int E = d->n_expert, k = d->n_expert_used;
    if (d->gating < 0 || d->gating > 2) return 0;
    if (k < 1 || k > 32 || E < k || E > 1024) return 0;
    if (d->n_groups > 1) {
        const int G = d->n_groups;
        if (G > 32 || E % G != 0 || E / G < 2) return 0;
        if (d->n_group_used < 1 || d->n_group_used > G || d->n_group_used * (E / G) < k) return 0;
    }
    return 1;
}

int orc_router(const orc_router_desc * d, const float * logits, int64_t ld, const float * bias, int64_t T,
               int64_t n_layers, int32_t * ids, float * weights) {
    if (!orc_router_valid(d) || T < 0 || n_layers < 0) return -1;
    const int E = d->n_expert, k = d->n_expert_used;
    std::vector<float> probs(E), sel(E), w(k);
    std::vector<char> taken(E);
    for (int64_t row = 0; row < T * n_layers; ++row) {
        const float * x = logits + row * ld;
        const int64_t layer = row / (T > 0 ? T : 1);
        if (d->gating == 1) {
            for (int j = 0; j < E; ++j) probs[j] = 1.0f / (1.0f + orc_expf(-x[j]));
        } else {
            for (int j = 0; j < E; ++j) probs[j] = x[j];
            if (d->gating == 0) router_soft_max(probs.data(), probs.data(), E);
        }
        for (int j = 0; j < E; ++j) sel[j] = bias ? probs[j] + bias[layer * E + j] : probs[j];
        if (d->n_groups > 1) {
            const int G = d->n_groups, gs = E / G;
            std::vector<float> score(G);
            for (int g = 0; g < G; ++g) {
                float t1 = -INFINITY, t2 = -INFINITY;
                for (int j = 0; j < gs; ++j) {
                    const float v = sel[g * gs + j];
                    if (v > t1) {
                        t2 = t1;
                        t1 = v;
                    } else if (v > t2) {
                        t2 = v;
                    }
                }
                score[g] = t1 + t2;
            }
            std::vector<char> keep(G, 0);
            for (int r = 0; r < d->n_group_used; ++r) {
                int best = -1;
                for (int g = 0; g < G; ++g)
                    if (!keep[g] && (best < 0 || router_better(score[g], g, score[best], best))) best = g;
                keep[best] = 1;
            }
            for (int j = 0; j < E; ++j)
                if (!keep[j / gs]) sel[j] = -INFINITY;
        }
        std::fill(taken.begin(), taken.end(), 0);
        for (int r = 0; r < k; ++r) {
            int best = -1;
            for (int j = 0; j < E; ++j)
                if (!taken[j] && (best < 0 || router_better(sel[j], j, sel[best], best))) best = j;
            taken[best] = 1;
            ids[row * k + r] = best;
            w[r] = probs[best];
        }
        if (d->gating == 2) router_soft_max(w.data(), w.data(), k);
        if (d->norm_w) {
            double s = 0.0;
            for (int r = 0; r < k; ++r) s += (double)w[r];
            float sf = (float)s;
            sf = sf > 6.103515625e-5f ? sf : 6.103515625e-5f;
            for (int r = 0; r < k; ++r) w[r] = w[r] / sf;
        }
        if (d->scale_w)
            for (int r = 0; r < k; ++r) w[r] = w[r] * d->w_scale;
        for (int r = 0; r < k; ++r) weights[row * k + r] = w[r];
    }
    return 0;
}

}  // extern "C"
