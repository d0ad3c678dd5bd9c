// Tensor-core MXFP4 jobs of the stack kernel (row mode 4, sm_100a).
//
// A job holds the same 32 weight rows as in row mode 3 (16 gate + 16 up rows
// of one (token, slot) pair, or 8 rows of each of the k = 4 experts of a
// token's down projection), but its integer block dots run on the tensor
// cores: tcgen05.mma kind::f8f6f4 with the weight codes as A (e2m1 in the
// 16U4_ALIGN16B shared layout: 16 codes in the first 8 bytes of every 16)
// and the activation as B (e4m3). An activation quant q (int8) is split into
// the digits q = 16*hi + lo, hi = q >> 4 in [-8, 7], lo = q & 15, both exact
// in e4m3, two B columns (hi, lo) per activation row; D_hi = sum w*hi and
// D_lo = sum w*lo with w the e2m1 value (the reference's kvalue / 2). Every
// product is a multiple of 1/2 of magnitude <= 90 and every partial sum a
// multiple of 1/2 below 2^12: exact in any accumulation order. The block's
// integer dot is sumi = 2*(16*D_hi + D_lo), exact in f32, and the rest is the
// reference's float order (ggml_vec_dot_mxfp4_q8_0, diff:1209-1240): per
// block pair u, t_u = fma(sc_e, sumi_e, sc_o*sumi_o), sc = fp16(d_y) *
// e8m0_half(e), and the row's dot is the chain sumf += t_u in pair order.
//
// One MMA instruction costs about as much to issue as an M=128 x N=64 tile
// computes, so every MMA carries 128 real rows: the job's K range is split
// into 4 segments of S blocks (S even, 4S >= blocks per row) and MMA step b
// (M=128, N=32, K=32) takes row r's block s*S + b as A row 32s + r. B's four
// 8-column groups (SBO apart) are the activation blocks s*S + b: the k = 4
// rows' (hi, lo) columns of a down job, or (hi, lo) and six columns never
// read back of a gate/up job. TMEM lane 32s + r then holds segment s of row r,
// in the sub-partition of warp 4 + s.
//
// The 16 code bytes of a block (byte j: element j in the low nibble, element
// j + 16 in the high nibble) are copied as they are: bytes 0-7 fill the first
// 16-element K half (K order e0, e16, e1, e17, ..., e7, e23), bytes 8-15 the
// second (e8, e24, ..., e15, e31). The quantizer writes the activation digits
// in the same K order (the code order of the Q8_0 quants), per block as
// [K half][activation row][digit][16 bytes]: B core matrices in place.
//
// Warps of a CTA in row mode 4 (512 threads):
//   0       weight producer;  1 (lane 0) MMA issuer;  2, 3 input producers;
//   4-7     epilogue warp s = segment s: per step it loads its 8 columns,
//           frees the TMEM and scale slot, forms sumi and the pair terms of
//           its segment and stores them for the chain;
//   8-11    repack warp s: per step, block s*S + b of the job's 32 rows (lane
//           = row) into the A slot (core matrices of 8 rows x 16 bytes) and
//           the (row, block) scales sc into the scale slot;
//   12      chain: per job, the row dots from the pair terms in pair order;
//   13-15   tails: activation, its digit quantization and the down-input
//           count (gate/up jobs), or the combine (down jobs).
// A slots (3 to 8, as the shared memory allows) are freed by the MMA's
// completion, TMEM and scale slots (8) by
// the epilogue, pair-term buffers (2) by the chain, dot slots (3) by the
// tails. Hand-offs inside the pipeline spin on mbarriers; every wait is
// bounded; TMEM is freed after the MMAs in flight land.
//
// Opt-in (GX_STACK_MMA=1): bit-identical to the CUDA-core MXFP4 jobs but
// slower on B200. Every (row, block) still passes through the CUDA cores:
// about 45 instructions of repack (unaligned block reads, the code copy into
// the K-major layout, the scale) and 15 of epilogue, against about 75 for the
// CUDA-core decode of the same block, and the hand-offs between the roles
// serialize the MMA steps (~1,100 cycles per 4 KB step, 9 % of the copy
// bandwidth). Records laid
// out for TMA (codes apart from scales, 16-byte rows) would let TMA build the
// A tiles and remove the repack.
#pragma once

#include <cstdint>

#include "gx_tc.cuh"

namespace gx {

constexpr int kTcSeg = 4;                   // K segments = TMEM sub-partitions
constexpr int kTcAmin = 3, kTcAmax = 8;     // A slots (one MMA step each): as many as the shared memory holds
constexpr int kTcT = 8;                     // TMEM and scale slots (one MMA step each)
constexpr int kTcN = 32;                    // MMA N: 4 segment groups of 8 columns
constexpr int kTcCols = 256;                // TMEM columns: kTcT x kTcN
static_assert(kTcT * kTcN == kTcCols, "TMEM slots");
constexpr int kTcTails = 3;                 // tail warps (and dot slots)
constexpr int kTcMaxBlocks = 128;           // MXFP4 blocks per row (K <= 4096)
constexpr int kTcThreads = 512;
constexpr int kTcBarThreads = 9 * 32;           // warps 1 and 4-11: TMEM users
constexpr uint32_t kTcScBytes = kTcT * 128 * 4;              // 128 (row, segment) scales per slot
constexpr uint32_t kTcDotBytes = kTcTails * 32 * 4;
constexpr uint32_t kTcBars = kTcAmax + 2 * kTcT + 4 + 2 * kTcTails + 1;
// a_full[Amax], d_full[T], d_empty[T], terms_full[2], terms_free[2], dots_full[3], dots_free[3], fin

// pair-term buffers for rows of nbmax blocks
__host__ __device__ constexpr uint32_t tc_terms_bytes(int nbmax) { return 2u * (uint32_t)(nbmax / 2) * 32u * 4u; }
__host__ __device__ constexpr uint32_t tc_bytes(int nbmax, int na) {
    return 4096u * (uint32_t)na + kTcScBytes + tc_terms_bytes(nbmax) + kTcDotBytes + kTcBars * 8 + 16;
}
// MMA steps of a job with nb blocks per row: 4 segments, an even step count
__host__ __device__ constexpr int tc_steps(int nb) { return ((nb + 7) >> 3) << 1; }

// e4m3 bits of a small integer n, |n| <= 15 (exact)
__device__ __forceinline__ uint32_t e4m3_small(int n) {
    const uint32_t a = (uint32_t)(n < 0 ? -n : n);
    if (a == 0) return 0u;
    const int e = 31 - __clz((int)a);                 // 0..3
    const uint32_t m = (a << (3 - e)) & 7u;
    return (n < 0 ? 0x80u : 0u) | ((uint32_t)(e + 7) << 3) | m;
}

// Q8_0 block ib of an f32 row (one warp, lane = element), the same quants and
// fp16 scale as quant_block_split, stored as e4m3 digits for activation row m
// of a k-row digit set: quant q of element e sits at code position
// c = mxfp4_code_pos(e), K half u = c / 16; digit hi at
// dst + 64k*ib + 32k*u + 32m + (c % 16), digit lo 16 bytes further; the
// scale at dst + d_off + 2*(m*nblk + ib).
template <bool COHERENT>
__device__ __forceinline__ void quant_block_digits(const float * x, uint8_t * dst, int m, int k, int nblk, int d_off,
                                                   int ib, int lane) {
    const float v = COHERENT ? __ldcg(x + 32 * ib + lane) : __ldg(x + 32 * ib + lane);
    float a = fabsf(v);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
    const float d = __fdiv_rn(a, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const int q = (int)(int8_t)__float2int_rn(__fmul_rn(v, id));
    const int c = mxfp4_code_pos(lane);
    uint8_t * base = dst + (int64_t)64 * k * ib + 32 * k * (c >> 4) + 32 * m + (c & 15);
    base[0] = (uint8_t)e4m3_small(q >> 4);
    base[16] = (uint8_t)e4m3_small(q & 15);
    if (lane == 0) *reinterpret_cast<uint16_t *>(dst + d_off + 2 * (m * nblk + ib)) = f2h(d);
}

// Shared state of the row-mode-4 roles.
struct TcTeam {
    uint8_t * abuf;        // [na][4096] A tiles (128 x 32-byte K-major)
    float * sc;            // [kTcT][128] scales of the step's (segment, row) pairs
    float * terms;         // [2][nbmax/2][32] pair terms of a job
    float * dots;          // [kTcTails][32] row dots of a job
    uint64_t * a_full;     // [na]     the 4 repack warps
    uint64_t * d_full;     // [kTcT]   the MMA commit
    uint64_t * d_empty;    // [kTcT]   the 4 epilogue warps
    uint64_t * terms_full; // [2]      the 4 epilogue warps
    uint64_t * terms_free; // [2]      the chain
    uint64_t * dots_full;  // [kTcTails] the chain
    uint64_t * dots_free;  // [kTcTails] the tail
    uint64_t * fin;        // the issuer's final commit
    uint32_t * tslot;      // TMEM base address
};

__device__ __forceinline__ TcTeam tc_team(uint8_t * smem, uint32_t off, int nbmax, int na) {
    TcTeam t;
    uint8_t * q = smem + off;
    const uint32_t ab = 4096u * (uint32_t)na;
    t.abuf = q;
    t.sc = reinterpret_cast<float *>(q + ab);
    t.terms = reinterpret_cast<float *>(q + ab + kTcScBytes);
    t.dots = reinterpret_cast<float *>(q + ab + kTcScBytes + tc_terms_bytes(nbmax));
    t.a_full = reinterpret_cast<uint64_t *>(q + ab + kTcScBytes + tc_terms_bytes(nbmax) + kTcDotBytes);
    t.d_full = t.a_full + kTcAmax;
    t.d_empty = t.d_full + kTcT;
    t.terms_full = t.d_empty + kTcT;
    t.terms_free = t.terms_full + 2;
    t.dots_full = t.terms_free + 2;
    t.dots_free = t.dots_full + kTcTails;
    t.fin = t.dots_free + kTcTails;
    t.tslot = reinterpret_cast<uint32_t *>(t.fin + 1);
    return t;
}

// mbarrier counts, in TcTeam order
__device__ __forceinline__ void tc_init_bars(const TcTeam & t) {
    for (int i = 0; i < kTcAmax; ++i) mbar_init(t.a_full + i, kTcSeg);
    for (int i = 0; i < kTcT; ++i) mbar_init(t.d_full + i, 1);
    for (int i = 0; i < kTcT; ++i) mbar_init(t.d_empty + i, kTcSeg);
    for (int i = 0; i < 2; ++i) mbar_init(t.terms_full + i, kTcSeg);
    for (int i = 0; i < 2; ++i) mbar_init(t.terms_free + i, 1);
    for (int i = 0; i < kTcTails; ++i) mbar_init(t.dots_full + i, 1);
    for (int i = 0; i < kTcTails; ++i) mbar_init(t.dots_free + i, 1);
    mbar_init(t.fin, 1);
}

// Bounded spin by lane 0, the outcome broadcast to the warp.
__device__ __forceinline__ bool tc_warp_wait(uint64_t * bar, uint32_t parity, int lane) {
    int ok = 1;
    if (lane == 0) ok = mbar_spin(bar, parity) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// parity of use c of a barrier that completes once per use, n slots round robin
__device__ __forceinline__ uint32_t tc_par(uint32_t c, uint32_t n) { return (c / n) & 1u; }

// The job's input buffer of key `key` (nb buffers): spin until its fill word
// names the key, then wait on its barrier with the published parity (lane 0).
__device__ __forceinline__ bool tc_wait_input(const volatile int * fw, uint64_t * ibars, int key, int nb, int lane) {
    int ok = 0;
    if (lane == 0) {
        const int bi = key % nb;
        int fpar = 0;
        bool got = false;
        for (uint32_t i = 0; i < (1u << 23) && !got; ++i) {
            const int v = fw[bi];
            got = (v >> 1) == key;
            fpar = v & 1;
            if (!got && (i & 63u) == 63u && *reinterpret_cast<volatile int *>(&g_dev_error) != 0) break;
            if (!got && i >= 16) __nanosleep(32);
        }
        ok = got && mbar_spin(ibars + bi, (uint32_t)fpar) ? 1 : 0;
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// What every role needs to know of job jl.
struct TcJob {
    StackJob J;
    int cs, n;             // stage and its use count
    int key, bi;           // input key and buffer
    int kk;                // activation rows of the job's B (1, or k for down jobs)
    int NB, S;             // blocks per row, MMA steps
    const uint8_t * inb;   // input buffer (digit rows, then fp16 scales at in_doff)
    int in_doff;
};

__device__ __forceinline__ TcJob tc_job(const StackParams & p, const StackGeom & g, int b, int G, int jl,
                                        const uint8_t * xbuf, const uint8_t * dbuf) {
    TcJob q;
    q.J = stack_job(g, b + jl * G);
    q.cs = jl % p.C;
    q.n = jl / p.C;
    q.key = q.J.L * p.T + q.J.t;
    q.bi = q.key % (q.J.gu ? kStackBufs : p.nbuf_d);
    q.kk = q.J.gu ? 1 : p.k;
    q.NB = (q.J.gu ? p.H : p.I) / 32;
    q.S = tc_steps(q.NB);
    q.inb = q.J.gu ? xbuf + q.bi * p.alx.pitch : dbuf + q.bi * p.k * p.ald.pitch;
    q.in_doff = q.J.gu ? p.alx.d_off : p.ald.d_off;
    return q;
}

// ------------------------------------------------------------------ roles

// TMEM address of lane group s (bits 31-16: lane) and column c
__device__ __forceinline__ uint32_t tc_taddr(uint32_t tbase, int s, int c) {
    return tbase + ((uint32_t)(32 * s) << 16) + (uint32_t)c;
}

// Warp 1 lane 0: per MMA step of every job, wait for the A slot, one MMA,
// one commit; after a job's last step frees its stage.
__device__ __forceinline__ void tc_issuer(const StackParams & p, const TcTeam & tm, uint32_t tbase, int b, int G,
                                          int mine, const uint8_t * xbuf, const uint8_t * dbuf, int * rel,
                                          uint64_t * empty) {
    const StackGeom g = stack_geom(p);
    const uint32_t na = (uint32_t)p.tc_na;
    const uint32_t idesc = umma_idesc_e2m1_e4m3(128, kTcN);
    const uint64_t ad0 = umma_desc(tm.abuf, 128, 256);   // slot sa: start address + 4096*sa
    uint32_t gs = 0;
    bool ok = true;
    for (int jl = 0; jl < mine && ok; ++jl) {
        const TcJob q = tc_job(p, g, b, G, jl, xbuf, dbuf);
        const uint32_t lbo = 32u * (uint32_t)q.kk, sbo = 64u * (uint32_t)q.kk * (uint32_t)q.S;
        const uint64_t bd0 = umma_desc(q.inb, lbo, sbo);       // step st: start address + 64*kk*st
        const uint64_t bstep = (uint64_t)(4 * q.kk);           // 64*kk bytes in 16-byte units
        uint32_t sa = gs % na, slot = gs % kTcT;
        for (int st = 0; st < q.S; ++st, ++gs) {
            if (!mbar_spin(tm.a_full + sa, tc_par(gs, na))) {
                ok = false;
                break;
            }
            tc_fence_after();
            mma_f8f6f4(tbase + (uint32_t)kTcN * slot, ad0 + (uint64_t)(256u * sa), bd0 + bstep * (uint64_t)st, idesc, 0u);
            mma_commit(tm.d_full + slot);
            sa = sa + 1 == na ? 0 : sa + 1;
            slot = (slot + 1) & (kTcT - 1);
        }
        if (!ok) break;
        // the repack warps have read the job's rows: free the stage
        __threadfence_block();
        atomicAdd(rel + q.cs, 1);
        mbar_arrive(empty + q.cs);
    }
    if (!ok) record_error(GX_DEVERR_TIMEOUT);
    // the MMAs in flight land before TMEM is freed
    mma_commit(tm.fin);
    mbar_spin(tm.fin, 0u);
}

// Repack warp s: block s*S + b of the job's 32 rows per step b.
__device__ __forceinline__ void tc_repack(const StackParams & p, const TcTeam & tm, int s, int lane, int b, int G,
                                          int mine, uint64_t * wfull, uint64_t * xbar, uint64_t * dbar,
                                          const int * fillw, const int * rel, const uint8_t * stages,
                                          const uint8_t * xbuf, const uint8_t * dbuf) {
    const StackGeom g = stack_geom(p);
    const uint32_t na = (uint32_t)p.tc_na;
    uint32_t gs = 0;
    bool ok = true;
    for (int jl = 0; jl < mine && ok; ++jl) {
        const TcJob q = tc_job(p, g, b, G, jl, xbuf, dbuf);
        const uint8_t * st = stages + q.cs * p.stage_bytes;
        const int nbr = q.J.gu ? (int)p.nb01_g : p.pitch_d;   // stage row pitch (up rows follow the gate rows)
        // the stage's previous job was released, its rows landed, the inputs are in
        int okr = 1;
        if (lane == 0) {
            bool r = q.n == 0;
            for (uint32_t i = 0; i < (1u << 23) && !r; ++i) {
                r = *reinterpret_cast<const volatile int *>(rel + q.cs) >= q.n;
                if (!r && (i & 63u) == 63u && *reinterpret_cast<volatile int *>(&g_dev_error) != 0) break;
                if (!r && i >= 16) __nanosleep(32);
            }
            okr = r ? 1 : 0;
        }
        ok = __shfl_sync(0xffffffffu, okr, 0) != 0;
        ok = ok && tc_warp_wait(wfull + q.cs, (uint32_t)(q.n & 1), lane);
        ok = ok && tc_wait_input(fillw + (q.J.gu ? 0 : kStackBufs), q.J.gu ? xbar : dbar, q.key,
                                 q.J.gu ? kStackBufs : p.nbuf_d, lane);
        if (!ok) break;
        const int m = q.J.gu ? 0 : lane / p.Rd;
        const uint8_t * row = st + lane * nbr;
        for (int stp = 0; stp < q.S; ++stp, ++gs) {
            const uint32_t sa = gs % na, slot = gs % kTcT;
            // the A slot went through its MMA, the scale slot was read back
            if (gs >= na && !tc_warp_wait(tm.d_full + (gs - na) % kTcT, tc_par(gs - na, kTcT), lane)) {
                ok = false;
                break;
            }
            if (gs >= (uint32_t)kTcT && !tc_warp_wait(tm.d_empty + slot, tc_par(gs - kTcT, kTcT), lane)) {
                ok = false;
                break;
            }
            const int j = s * q.S + stp;
            if (j < q.NB) {
                const uintptr_t P = reinterpret_cast<uintptr_t>(row + 17 * j);
                const uint8_t * wp = reinterpret_cast<const uint8_t *>(P & ~(uintptr_t)3);
                const uint32_t sh = (uint32_t)(P & 3) * 8u;
                uint32_t w[5];
#pragma unroll
                for (int i = 0; i < 5; ++i) w[i] = lds32(wp + 4 * i);
                const uint32_t e = (w[0] >> sh) & 0xffu;
                uint32_t c4[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) c4[i] = __funnelshift_rc(w[i], w[i + 1], sh + 8u);
                // A row 32s + lane: group 4s + lane/8, row lane%8 of its core matrices
                uint8_t * dst = tm.abuf + sa * 4096u + (4 * s + (lane >> 3)) * 256 + (lane & 7) * 16;
                *reinterpret_cast<uint2 *>(dst) = make_uint2(c4[0], c4[1]);
                *reinterpret_cast<uint2 *>(dst + 128) = make_uint2(c4[2], c4[3]);
                const uint16_t dyh = *reinterpret_cast<const uint16_t *>(q.inb + q.in_doff + 2 * (m * q.NB + j));
                tm.sc[slot * 128 + 32 * s + lane] = __fmul_rn(h2f(dyh), e8m0_half(e));
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(tm.a_full + sa);
        }
    }
    if (!ok && lane == 0) record_error(GX_DEVERR_TIMEOUT);
}

// Epilogue warp s (TMEM lanes 32s..32s+31): segment s of every row, per step
// its 8 columns; the pair terms of the segment into the job's term buffer.
__device__ __forceinline__ void tc_epilogue(const StackParams & p, const TcTeam & tm, uint32_t tbase, int s, int lane,
                                            int b, int G, int mine, const uint8_t * xbuf, const uint8_t * dbuf,
                                            int nbmax) {
    const StackGeom g = stack_geom(p);
    uint32_t gs = 0;
    bool ok = true;
    for (int jl = 0; jl < mine && ok; ++jl) {
        const TcJob q = tc_job(p, g, b, G, jl, xbuf, dbuf);
        const int p2 = jl & 1;
        // the chain has read this buffer's previous job (jl - 2)
        if (jl >= 2 && !tc_warp_wait(tm.terms_free + p2, (uint32_t)(((jl >> 1) - 1) & 1), lane)) {
            ok = false;
            break;
        }
        float * tb = tm.terms + p2 * (nbmax / 2) * 32;
        const int m = q.J.gu ? 0 : lane / p.Rd;
        const bool m1 = (m & 1) != 0, m2 = (m & 2) != 0;
        float sce = 0.0f, sie = 0.0f;
        for (int stp = 0; stp < q.S; ++stp, ++gs) {
            const uint32_t slot = gs % kTcT;
            if (!tc_warp_wait(tm.d_full + slot, tc_par(gs, kTcT), lane)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t v[8];
            tmem_ld8(tc_taddr(tbase, s, kTcN * (int)slot + 8 * s), v);
            tmem_wait_ld();
            const float scv = tm.sc[slot * 128 + 32 * s + lane];
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tm.d_empty + slot);
            const int j = s * q.S + stp;
            if (j < q.NB) {
                uint32_t h, l;
                if (q.J.gu) {
                    h = v[0];
                    l = v[1];
                } else {
                    const uint32_t h01 = m1 ? v[2] : v[0], h23 = m1 ? v[6] : v[4];
                    const uint32_t l01 = m1 ? v[3] : v[1], l23 = m1 ? v[7] : v[5];
                    h = m2 ? h23 : h01;
                    l = m2 ? l23 : l01;
                }
                const float x = __fmaf_rn(16.0f, __uint_as_float(h), __uint_as_float(l));
                const float si = __fadd_rn(x, x);   // the block's integer dot, exact
                if ((stp & 1) == 0) {
                    sce = scv;
                    sie = si;
                } else {
                    tb[(j >> 1) * 32 + lane] = __fmaf_rn(sce, sie, __fmul_rn(scv, si));
                }
            }
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(tm.terms_full + p2);
    }
    if (!ok && lane == 0) record_error(GX_DEVERR_TIMEOUT);
}

// Chain warp: the row dots in pair order; frees the term buffer and the
// job's input buffer, hands the dots to the job's tail warp.
__device__ __forceinline__ void tc_chain(const StackParams & p, const TcTeam & tm, int lane, int b, int G, int mine,
                                         const uint8_t * xbuf, const uint8_t * dbuf, int * bufdone, int nbmax) {
    const StackGeom g = stack_geom(p);
    bool ok = true;
    for (int jl = 0; jl < mine && ok; ++jl) {
        const TcJob q = tc_job(p, g, b, G, jl, xbuf, dbuf);
        const int p2 = jl & 1;
        if (!tc_warp_wait(tm.terms_full + p2, (uint32_t)((jl >> 1) & 1), lane)) {
            ok = false;
            break;
        }
        const float * tb = tm.terms + p2 * (nbmax / 2) * 32;
        float sumf = 0.0f;
        const int np = q.NB / 2;
        int u = 0;
        for (; u + 8 <= np; u += 8) {   // eight loads in flight, then the chain
            float t[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) t[i] = tb[(u + i) * 32 + lane];
#pragma unroll
            for (int i = 0; i < 8; ++i) sumf = __fadd_rn(sumf, t[i]);
        }
        for (; u < np; ++u) sumf = __fadd_rn(sumf, tb[u * 32 + lane]);
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(tm.terms_free + p2);
            // the MMAs and the scales have read the job's inputs: free the buffer
            __threadfence_block();
            atomicAdd(bufdone + (q.J.gu ? 0 : kStackBufs) + q.bi, 1);
        }
        const int tq = jl % kTcTails;
        if (jl >= kTcTails && !tc_warp_wait(tm.dots_free + tq, tc_par(jl - kTcTails, kTcTails), lane)) {
            ok = false;
            break;
        }
        tm.dots[tq * 32 + lane] = sumf;
        __syncwarp();
        if (lane == 0) mbar_arrive(tm.dots_full + tq);
    }
    if (!ok && lane == 0) record_error(GX_DEVERR_TIMEOUT);
}

// Tail warp tq: jobs tq, tq + 3, ...: SwiGLU and the digit quantization of
// the down inputs (gate/up jobs), or the weighted combine (down jobs).
__device__ __forceinline__ void tc_tail(const StackParams & p, const TcTeam & tm, int tq, int lane, int b, int G,
                                        int mine, const uint8_t * xbuf, const uint8_t * dbuf) {
    const StackGeom g = stack_geom(p);
    bool ok = true;
    for (int jl = tq; jl < mine && ok; jl += kTcTails) {
        const TcJob q = tc_job(p, g, b, G, jl, xbuf, dbuf);
        const StackJob & J = q.J;
        if (!tc_warp_wait(tm.dots_full + tq, tc_par((uint32_t)jl, kTcTails), lane)) {
            ok = false;
            break;
        }
        const float dot = tm.dots[tq * 32 + lane];
        __syncwarp();
        if (lane == 0) mbar_arrive(tm.dots_free + tq);
        const StackLayer & ly = p.layers[J.L];
        if (J.gu) {
            // gate row r (lane r < 16) pairs with up row r (lane r + 16)
            const float up = __shfl_down_sync(0xffffffffu, dot, 16);
            if (lane < 16) {
                const float a = p.act == 1 ? act_swiglu_oai(dot, up, p.alpha, p.limit) : act_swiglu(dot, up);
                ly.act[(int64_t)J.pair * p.I + J.r0 + lane] = a;
            }
            const int nblk = p.I / p.qblk, blk = J.r0 / p.qblk;
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                fence_acq_rel_gpu();
                last = atomicAdd(ly.cnt + J.pair * nblk + blk, 1) == (p.qblk / p.Rg) - 1;
            }
            if (__shfl_sync(0xffffffffu, last, 0)) {
                // this job finished the Q8 block last: its digits into the token's down inputs
                fence_acq_rel_gpu();
                const int mm = J.pair - J.t * p.k;
                quant_block_digits<true>(ly.act + (int64_t)J.pair * p.I, ly.actq + (int64_t)J.t * p.k * p.ald.pitch, mm,
                                         p.k, nblk, p.ald.d_off, blk, lane);
                fence_proxy_async_global();
                __syncwarp();
                if (lane == 0) {
                    fence_acq_rel_gpu();
                    atomicAdd(p.gu_done + J.L * p.T + J.t, 1);
                }
            }
        } else {
            // output row rr = lane < Rd: sum over slots mm of w[mm] * dot(mm*Rd + rr), in slot order
            const float * wr = ly.rw + (int64_t)J.t * p.k;
            float accf = 0.0f;
            for (int mm = 0; mm < p.k; ++mm) {
                const float vv = __shfl_sync(0xffffffffu, dot, (mm * p.Rd + lane) & 31);
                const float prod = __fmul_rn(vv, lane < p.Rd ? wr[mm] : 0.0f);
                accf = mm == 0 ? prod : __fadd_rn(accf, prod);
            }
            if (lane < p.Rd) ly.out[(int64_t)J.t * p.H + J.r0 + lane] = accf;
        }
    }
    if (!ok && lane == 0) record_error(GX_DEVERR_TIMEOUT);
}

// Row mode 4 from warp 1 on: TMEM, the layer inputs' digit rows, the roles,
// and TMEM freed once the MMAs have landed.
__device__ __forceinline__ void stack_tc(const StackParams & p, uint8_t * smem, int warp, int lane, int b, int G,
                                         int mine, uint64_t * wfull, uint64_t * empty, uint64_t * xbar, uint64_t * dbar,
                                         const int * fillw, int * bufdone, int * rel, const uint8_t * stages,
                                         const uint8_t * xbuf, const uint8_t * dbuf) {
    const int nbmax = (p.H > p.I ? p.H : p.I) / 32;
    const TcTeam tm = tc_team(smem, p.tc_off, nbmax, p.tc_na);
    if (warp >= 12) {
        // chain and tails: no TMEM
        if (warp == 12) tc_chain(p, tm, lane, b, G, mine, xbuf, dbuf, bufdone, nbmax);
        else tc_tail(p, tm, warp - 13, lane, b, G, mine, xbuf, dbuf);
        return;
    }
    // warps 1 and 4-11 from here on (kTcBarThreads)
    if (warp == 4) {
        tmem_alloc(tm.tslot, kTcCols);
        tmem_relinquish();
    }
    bool any = false;
    if (warp >= 4) {
        // the inputs of layers L = b, b+G, ... as digit rows (one warp per block)
        const int nblk = p.H / 32;
        for (int L = b; L < p.NL; L += G) {
            const StackLayer & ly = p.layers[L];
            for (int wi = warp - 4; wi < p.T * nblk; wi += 8) {
                const int t = wi / nblk, ib = wi - t * nblk;
                quant_block_digits<false>(ly.x + (int64_t)t * p.H, ly.xq + (int64_t)t * p.alx.pitch, 0, 1, nblk,
                                          p.alx.d_off, ib, lane);
            }
            any = true;
        }
        if (any) fence_proxy_async_global();
    }
    tc_fence_before();
    named_barrier(3, kTcBarThreads);
    tc_fence_after();
    if (any && warp == 4 && lane == 0) {
        fence_acq_rel_gpu();
        for (int L = b; L < p.NL; L += G) atomicExch(p.q_done + L, 1);
    }
    const uint32_t tbase = *reinterpret_cast<volatile uint32_t *>(tm.tslot);
    if (warp == 1) {
        if (lane == 0) tc_issuer(p, tm, tbase, b, G, mine, xbuf, dbuf, rel, empty);
        __syncwarp();
    } else if (warp < 8) {
        tc_epilogue(p, tm, tbase, warp - 4, lane, b, G, mine, xbuf, dbuf, nbmax);
    } else {
        tc_repack(p, tm, warp - 8, lane, b, G, mine, wfull, xbar, dbar, fillw, rel, stages, xbuf, dbuf);
    }
    tc_fence_before();
    named_barrier(4, kTcBarThreads);
    tc_fence_after();
    if (warp == 4) tmem_dealloc(tbase, kTcCols);
}

}  // namespace gx
