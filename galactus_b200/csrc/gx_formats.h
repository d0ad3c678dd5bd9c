// GGUF block-quant formats the routed-expert FFN computes on, and the status
// codes shared by host and device code. Byte layouts are ggml's (the same
// sizes as scripts/moe-profile.py:25-37 of the reference):
//   Q8_0   { fp16 d; int8 qs[32]; }                               34 B / 32
//   Q8_K   { f32 d; int8 qs[256]; int16 bsums[16]; }               292 B / 256
//   Q4_K   { fp16 d; fp16 dmin; u8 scales[12]; u8 qs[128]; }       144 B / 256
//   Q6_K   { u8 ql[128]; u8 qh[64]; int8 scales[16]; fp16 d; }     210 B / 256
//   MXFP4  { u8 e (e8m0); u8 qs[16]; }                             17 B / 32
//   IQ1_S  { fp16 d; u8 qs[32]; u16 qh[8]; }                       50 B / 256
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define GX_HD __host__ __device__ __forceinline__
#else
#define GX_HD inline
#endif

namespace gx {

enum : int {
    GX_T_Q8_0 = 8,
    GX_T_Q4_K = 12,
    GX_T_Q6_K = 14,
    GX_T_Q8_K = 15,
    GX_T_IQ1_S = 19,
    GX_T_MXFP4 = 39,
};

GX_HD int block_bytes(int type) {
    switch (type) {
        case GX_T_Q8_0: return 34;
        case GX_T_Q8_K: return 292;
        case GX_T_Q4_K: return 144;
        case GX_T_Q6_K: return 210;
        case GX_T_MXFP4: return 17;
        case GX_T_IQ1_S: return 50;
        default: return 0;
    }
}

GX_HD int block_elems(int type) {
    switch (type) {
        case GX_T_Q8_0: case GX_T_MXFP4: return 32;
        case GX_T_Q8_K: case GX_T_Q4_K: case GX_T_Q6_K: case GX_T_IQ1_S: return 256;
        default: return 0;
    }
}

// activation type of the CPU path (type_traits_cpu vec_dot_type; diff:166-178)
GX_HD int vec_dot_type(int type) {
    return (type == GX_T_Q8_0 || type == GX_T_MXFP4) ? GX_T_Q8_0 : GX_T_Q8_K;
}

GX_HD bool supported_weight_type(int type) {
    return type == GX_T_Q8_0 || type == GX_T_Q4_K || type == GX_T_Q6_K || type == GX_T_MXFP4 || type == GX_T_IQ1_S;
}

// ne00 granularity of the bit-exact path: the Q8_0-activation kernels work on
// block pairs (64), the Q8_K ones on whole superblocks (256) (diff:181-187)
GX_HD int row_align(int type) { return vec_dot_type(type) == GX_T_Q8_0 ? 64 : 256; }

GX_HD int64_t row_bytes(int type, int64_t n) { return (n / block_elems(type)) * block_bytes(type); }

// device error codes recorded by kernels (first one wins)
enum : int {
    GX_DEVERR_NONE = 0,
    GX_DEVERR_DOMAIN = 1,    // expert id outside [0, n_as)
    GX_DEVERR_TIMEOUT = 2,   // a bounded mbarrier wait ran out
};

}  // namespace gx
