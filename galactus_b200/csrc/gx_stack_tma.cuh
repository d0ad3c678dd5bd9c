// TMA-fed tensor-core MXFP4 jobs of the stack kernel (row mode 5, sm_100a).
//
// The rows come from a copy of the layer's slots in the tensor-core record
// layout (Mxfp4TcMats): per matrix, the 16 code bytes of every block of a row
// side by side in TMA-box order (tile, group of 4 blocks, row: each box one
// contiguous run of 64 bytes per row), then the block scale bytes
// ([rows][nb]). TMA loads the codes with data type 16U4_ALIGN16B, which
// writes each 16 codes (8 bytes) into 16 bytes of shared memory, the
// unpacked e2m1 operand of tcgen05.mma kind::f8f6f4, and with the 128-byte
// swizzle the UMMA descriptor reads: no CUDA core touches a weight byte. A
// job is 128 rows (64 gate + 64 up rows of one (token, slot) pair, or 32
// rows of each of the k = 4 experts of a token's down projection); a chunk
// is 4 blocks (128 K elements, a 16 KB tile), and each
// block is one M=128 x N=16 x K=32 MMA against the activation's e4m3 digit
// columns (hi, lo; q = 16*hi + lo, exact) in TMEM columns of its own.
//
// The arithmetic is that of ggml_vec_dot_mxfp4_q8_0 (diff:1209-1240): the
// block's integer dot sumi = 2*(16*D_hi + D_lo) (exact: every partial is a
// multiple of 1/2 below 2^12), sc = fp16(d_y) * e8m0_half(e), per block pair
// t = fma(sc_e, sumi_e, sc_o*sumi_o) and the chain sumf += t in pair order,
// each row in its own lane from the first chunk to the last.
//
// Warps (kT5Warps, 32 * (11 + kT5Issuers) threads):
//   0, 13   chunk producers (lane 0): producer i takes the chunks gc = i
//           (mod 2), the TMA tiles (2 boxes of 64 rows, or 4 of 32 rows, one
//           per expert slot) into the ring;
//   12      scale producer (lane 0): per job the scale bytes of its rows (one
//           bulk copy per 64 or 32 rows), a job ahead of the epilogue;
//   1, 10, 11, 14..  MMA issuers: issuer i takes the chunks gc = i (mod
//           kT5Issuers) of the CTA's chunk sequence, so that one chunk's waits
//           and commits overlap other chunks' MMAs; the whole warp walks the
//           chunks (its descriptors stay warp-uniform), lane 0 issues per
//           chunk 4 MMAs and 2 commits (TMEM slot full, ring stage empty);
//   2, 3    input producers (the digit rows of x and of the down inputs);
//   4-7     epilogue warp s, TMEM lanes 32s..32s+31 = rows 32s..32s+31 of the
//           job: the pair terms and the chain of its rows (the next chunk's
//           scales loaded before its MMAs are waited for), into one of two
//           128-float exchanges;
//   8, 9    tails: SwiGLU and the digit quantization of the down inputs (gate
//           rows 32s.. with up rows 64+32s.., gate/up jobs), or the combine
//           (down jobs, warp 8), while the epilogue runs the next job.
// Before the roles start, warps 4-9 of every CTA quantize the layers' x into
// digit rows, the blocks of all layers spread over the grid; a layer's inputs
// are ready once its q_done counter reaches T * H / 32.
// Ring stages, TMEM slots (8 chunks of 4 x 16 columns), the two job scale
// buffers and the two exchanges are each freed by their consumer through an
// mbarrier; every wait is bounded; TMEM is freed after the MMAs in flight land.
#pragma once

#include <cstdint>

#include "gx_stack_tc.cuh"

namespace gx {

constexpr int kT5Chunk = 4;                    // MXFP4 blocks per chunk (128 K elements)
constexpr int kT5Sub = 4;                      // blocks per TMA box (one 128-byte swizzled row of 128 codes)
constexpr int kT5Subs = kT5Chunk / kT5Sub;     // sub-tiles per chunk
constexpr uint32_t kT5SubTile = 128u * 128u;   // 128 rows x 128 swizzled bytes: 4 blocks of the job's rows
constexpr uint32_t kT5Tile = kT5Subs * kT5SubTile;
constexpr int kT5StagesMin = 4, kT5StagesMax = 12;   // (a multiple of kT5StageStep, below)
constexpr int kT5TSlots = 8;                   // TMEM slots (chunks)
constexpr int kT5N = 16;                       // MMA N (digit columns: 2 per activation row, k = 4 rows)
constexpr int kT5Cols = kT5TSlots * kT5Chunk * kT5N;   // 512
constexpr int kT5Producers = 2;                // warps 0, 13
constexpr int kT5Threads = 32 * kT5Warps;
// Every wait names the barrier's phase by its parity, which is unambiguous
// only while the waiter is at most one phase ahead of the barrier. A role
// that takes every n-th chunk could otherwise run a whole ring ahead of
// another role's chunk on the same stage and read an older, still incomplete
// phase as complete. So the ring's stage count is a multiple of both the
// issuer and the producer counts, and the TMEM slot count a multiple of the
// issuer count: the previous use of every stage and slot a role waits on was
// that role's own chunk, which it has already waited for.
constexpr int t5_gcd(int a, int b) { return b == 0 ? a : t5_gcd(b, a % b); }
constexpr int kT5StageStep = kT5Issuers / t5_gcd(kT5Issuers, kT5Producers) * kT5Producers;
static_assert(kT5TSlots % kT5Issuers == 0, "TMEM slots: a multiple of the issuer count");

// issuer index of warp w (-1: not an issuer)
__host__ __device__ constexpr int t5_issuer_index(int w) {
    return w == 1 ? 0 : (w == 10 || w == 11) ? w - 9 : (w >= 14 && w < kT5Warps) ? w - 11 : -1;
}
constexpr uint32_t kT5Bars = 2 * kT5StagesMax + 2 * kT5TSlots + 8 + 1;
// full[S], empty[S], tfull[8], tempty[8], sfull[2], sfree[2], xfull[2], xfree[2], fin

// bytes of the row-mode-5 region (from its start; the ring starts at the
// first 1024-byte boundary of shared memory inside it)
__host__ __device__ constexpr uint32_t t5_scale_bytes(int nbmax) { return 2u * ((128u * (uint32_t)nbmax + 127u) / 128u * 128u); }
__host__ __device__ constexpr uint32_t t5_bytes(int nbmax, int stages) {
    return 1024u + (uint32_t)stages * kT5Tile + t5_scale_bytes(nbmax) + 2u * 128u * 4u + kT5Bars * 8u + 16u;
}

// Shared state of row mode 5.
struct T5Team {
    uint8_t * ring;        // [stages][16 KB], 1024-byte aligned
    uint8_t * sbuf;        // [2][128 rows][nb] scale bytes of a job (nb: blocks per row of the job)
    float * xchg;          // [2][128] a job's row dots, epilogue to tails
    uint64_t * full;       // [stages] TMA tiles landed
    uint64_t * empty;      // [stages] the MMAs have read the stage
    uint64_t * tfull;      // [8] a chunk's MMAs are done
    uint64_t * tempty;     // [8] the 4 epilogue warps have read the TMEM slot
    uint64_t * sfull;      // [2] a job's scales landed
    uint64_t * sfree;      // [2] the 4 epilogue warps are done with them
    uint64_t * xfull;      // [2] the 4 epilogue warps wrote the exchange
    uint64_t * xfree;      // [2] the 2 tail warps read it
    uint64_t * fin;
    uint32_t * tslot;
    uint32_t sbuf_stride;  // bytes between the two job buffers
};

__device__ __forceinline__ T5Team t5_team(uint8_t * smem, uint32_t off, int nbmax, int stages) {
    T5Team t;
    uint8_t * q = smem + off;
    const uint32_t a = smem_u32(q);
    uint8_t * ring = q + ((1024u - (a & 1023u)) & 1023u);
    t.ring = ring;
    t.sbuf_stride = t5_scale_bytes(nbmax) / 2u;
    uint8_t * r = q + 1024u + (uint32_t)stages * kT5Tile;
    t.sbuf = r;
    r += t5_scale_bytes(nbmax);
    t.xchg = reinterpret_cast<float *>(r);
    r += 2u * 128u * 4u;
    t.full = reinterpret_cast<uint64_t *>(r);
    t.empty = t.full + kT5StagesMax;
    t.tfull = t.empty + kT5StagesMax;
    t.tempty = t.tfull + kT5TSlots;
    t.sfull = t.tempty + kT5TSlots;
    t.sfree = t.sfull + 2;
    t.xfull = t.sfree + 2;
    t.xfree = t.xfull + 2;
    t.fin = t.xfree + 2;
    t.tslot = reinterpret_cast<uint32_t *>(t.fin + 1);
    return t;
}

__device__ __forceinline__ void t5_init_bars(const T5Team & t) {
    for (int i = 0; i < kT5StagesMax; ++i) {
        mbar_init(t.full + i, 1);
        mbar_init(t.empty + i, 1);
    }
    for (int i = 0; i < kT5TSlots; ++i) {
        mbar_init(t.tfull + i, 1);
        mbar_init(t.tempty + i, 4);
    }
    for (int i = 0; i < 2; ++i) {
        mbar_init(t.sfull + i, 1);
        mbar_init(t.sfree + i, 4);
        mbar_init(t.xfull + i, 4);
        mbar_init(t.xfree + i, 2);
    }
    mbar_init(t.fin, kT5Issuers);
}

// A job of row mode 5 in 8 bytes: L | gu << 8 | t << 9, r0 | pair << 16
// (L < 128 layers, r0 and pair below 2^16).
__device__ __forceinline__ uint2 t5_pack(const StackJob & J) {
    return make_uint2((uint32_t)J.L | ((uint32_t)J.gu << 8) | ((uint32_t)J.t << 9),
                      (uint32_t)J.r0 | ((uint32_t)J.pair << 16));
}

// Job jl of this CTA: from the table the prologue filled, else decoded here.
__device__ __forceinline__ StackJob t5_job(const StackParams & p, const StackGeom & g, int b, int G, int jl) {
    if (jl < p.t5_jobs) {
        extern __shared__ __align__(128) uint8_t smem[];
        const uint2 v = reinterpret_cast<const uint2 *>(smem + p.t5_jobs_off)[jl];
        StackJob J;
        J.L = (int)(v.x & 0xffu);
        J.gu = (int)((v.x >> 8) & 1u);
        J.t = (int)(v.x >> 9);
        J.r0 = (int)(v.y & 0xffffu);
        J.pair = (int)(v.y >> 16);
        return J;
    }
    return stack_job(g, b + jl * G);
}

// tc_job over the job table: the key and buffer of the job's inputs, its
// blocks per row and its B rows (buffer counts are 1 or 2).
__device__ __forceinline__ TcJob t5_tcjob(const StackParams & p, const StackGeom & g, int b, int G, int jl,
                                          const uint8_t * xbuf, const uint8_t * dbuf) {
    TcJob q;
    q.J = t5_job(p, g, b, G, jl);
    q.cs = 0;
    q.n = jl;
    q.key = q.J.L * p.T + q.J.t;
    q.bi = q.J.gu ? (q.key & (kStackBufs - 1)) : (p.nbuf_d == 2 ? (q.key & 1) : 0);
    q.kk = q.J.gu ? 1 : p.k;
    q.NB = (q.J.gu ? p.H : p.I) >> 5;
    q.S = 0;
    q.inb = q.J.gu ? xbuf + q.bi * p.alx.pitch : dbuf + q.bi * p.k * p.ald.pitch;
    q.in_doff = q.J.gu ? p.alx.d_off : p.ald.d_off;
    return q;
}

// Q8_0 quantization of one 32-element block held by a warp (lane = element),
// the same quants and fp16 scale as quant_block_split, stored as e4m3 digits
// (quant_block_digits' layout).
__device__ __forceinline__ void quant_value_digits(float v, uint8_t * dst, int m, int k, int nblk, int d_off, int ib,
                                                   int lane) {
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

// The scale bytes of job jn's 128 rows into scale buffer jn & 1 (one bulk
// copy per 64 gate/up rows or per expert's 32 down rows).
__device__ __forceinline__ void t5_issue_scales(const StackParams & p, const T5Team & tm, const StackGeom & g, int b,
                                                int G, int jn, const int32_t * slots, const StackWeights * wt) {
    const StackJob J = t5_job(p, g, b, G, jn);
    const StackWeights w = wt[J.L];
    const int32_t * sl = slots + J.L * p.T * p.k;
    const int NB = (J.gu ? p.H : p.I) / 32;
    const int64_t soff = (int64_t)(J.gu ? p.I : p.H) * mxfp4_tc_cstride(NB);   // the scales follow the codes
    uint8_t * sb = tm.sbuf + (jn & 1) * tm.sbuf_stride;
    uint64_t * bar = tm.sfull + (jn & 1);
    if (J.gu) {
        const int64_t off = (int64_t)sl[J.pair] * w.nb02 + soff + (int64_t)J.r0 * NB;
        const uint32_t bytes = 64u * (uint32_t)NB;
        tma_expect(bar, 2u * bytes);
        tma_load(sb, w.wg + off, bytes, bar);
        tma_load(sb + bytes, w.wu + off, bytes, bar);
    } else {
        const uint32_t bytes = 32u * (uint32_t)NB;
        tma_expect(bar, (uint32_t)p.k * bytes);
        for (int m = 0; m < p.k; ++m)
            tma_load(sb + m * bytes, w.wd + (int64_t)sl[J.pair + m] * w.nb02 + soff + (int64_t)J.r0 * NB, bytes, bar);
    }
}

// Chunk producer ii (lane 0 of warps 0 and 13): the chunks gc = ii (mod
// kT5Producers) of the CTA's chunk sequence, the codes of their 128 rows as
// TMA tiles into ring stage gc mod S once the MMAs of chunk gc - S have read it.
__device__ __forceinline__ void t5_producer(const StackParams & p, const T5Team & tm, int b, int G, int mine,
                                            const int32_t * slots, int ii) {
    const StackGeom g = stack_geom(p);
    const uint32_t S = (uint32_t)p.tc_na;
    uint32_t st = 0, sph = 0;   // ring stage of chunk gc and the parity of its use
    uint32_t gc = 0;
    bool ok = true;
    for (int jl = 0; jl < mine && ok; ++jl) {
        const StackJob J = t5_job(p, g, b, G, jl);
        const int32_t * sl = slots + J.L * p.T * p.k + J.pair;
        const int NB = (J.gu ? p.H : p.I) / 32, nch = (NB + kT5Chunk - 1) / kT5Chunk;
        const int nsub_all = (NB + kT5Sub - 1) / kT5Sub;   // boxes along the row
        const CUtensorMap * mp = p.t5_maps + 3 * J.L;
        const int tile_y = J.gu ? J.r0 / 64 : J.r0 / 32;
        int sk[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) sk[m] = (J.gu && m > 0) || m >= p.k ? 0 : sl[m];
        for (int c = 0; c < nch; ++c, ++gc) {
            if (gc % kT5Producers == (uint32_t)ii) {
                if (gc >= S && !mbar_spin(tm.empty + st, sph ^ 1u)) {
                    ok = false;
                    break;
                }
                uint8_t * tile = tm.ring + st * kT5Tile;
                const int nsub = min(kT5Subs, nsub_all - kT5Subs * c);
                // the transaction bytes of 16U4_ALIGN16B boxes count the packed 4-bit
                // values (half the 16 KB each sub-tile fills in shared memory)
                tma_expect(tm.full + st, (uint32_t)nsub * (kT5SubTile / 2));
                // box (4-block group kT5Subs*c + u, tile of the job's rows, slot): one contiguous run
                for (int u = 0; u < nsub; ++u) {
                    uint8_t * sub = tile + u * kT5SubTile;
                    if (J.gu) {
                        tma_load_5d(sub, mp + 0, 0, 0, kT5Subs * c + u, tile_y, sk[0], tm.full + st);
                        tma_load_5d(sub + kT5SubTile / 2, mp + 1, 0, 0, kT5Subs * c + u, tile_y, sk[0], tm.full + st);
                    } else {
#pragma unroll
                        for (int m = 0; m < 4; ++m)
                            tma_load_5d(sub + (kT5SubTile / 4) * m, mp + 2, 0, 0, kT5Subs * c + u, tile_y, sk[m], tm.full + st);
                    }
                }
            }
            if (++st == S) {
                st = 0;
                sph ^= 1u;
            }
        }
    }
    if (!ok) record_error(GX_DEVERR_TIMEOUT);
    // this producer's copies in flight land before the CTA can exit (bounded waits)
    for (uint32_t c = gc > S ? gc - S : 0; c < gc; ++c)
        if (c % kT5Producers == (uint32_t)ii) mbar_spin(tm.full + c % S, tc_par(c, S));
}

// Scale producer (warp 12 lane 0): job jn's scales into buffer jn & 1 once the
// epilogue is done with job jn - 2's, i.e. up to a job ahead of the epilogue.
__device__ __forceinline__ void t5_scale_producer(const StackParams & p, const T5Team & tm, int b, int G, int mine,
                                                  const int32_t * slots, const StackWeights * wt) {
    const StackGeom g = stack_geom(p);
    int jn = 0;
    for (; jn < mine; ++jn) {
        if (jn >= 2 && !mbar_spin(tm.sfree + (jn & 1), (uint32_t)(((jn >> 1) - 1) & 1))) {
            record_error(GX_DEVERR_TIMEOUT);
            break;
        }
        t5_issue_scales(p, tm, g, b, G, jn, slots, wt);
    }
    for (int j = jn > 2 ? jn - 2 : 0; j < jn; ++j) mbar_spin(tm.sfull + (j & 1), (uint32_t)((j >> 1) & 1));
}

// One thread: the job's input buffer holds its key and its copy has landed
// (fill word, then the buffer's barrier with the published parity).
__device__ __forceinline__ bool t5_wait_input(const TcJob & q, const int * fillw, uint64_t * xbar, uint64_t * dbar) {
    const volatile int * fw = fillw + (q.J.gu ? 0 : kStackBufs);
    bool got = false;
    int fpar = 0;
    for (uint32_t i = 0; i < (1u << 23) && !got; ++i) {
        const int v = fw[q.bi];
        got = (v >> 1) == q.key;
        fpar = v & 1;
        if (!got && (i & 63u) == 63u && *reinterpret_cast<volatile int *>(&g_dev_error) != 0) break;
        if (!got && i >= 16) __nanosleep(32);
    }
    return got && mbar_spin((q.J.gu ? xbar : dbar) + q.bi, (uint32_t)fpar);
}

// Issuer ii: per chunk gc = ii (mod kT5Issuers), once its tiles landed and
// its TMEM slot is free, lane 0 issues one MMA per block into columns
// 64*slot + 16*j, then the commits (each commit covers this thread's own
// MMAs, i.e. its chunk). The whole warp runs the loop so that the stage, slot
// and descriptors are the same in every lane.
__device__ __forceinline__ void t5_issuer(const StackParams & p, const T5Team & tm, uint32_t tbase, int b, int G,
                                          int mine, uint64_t * xbar, uint64_t * dbar, const int * fillw,
                                          const uint8_t * xbuf, const uint8_t * dbuf, int lane, int ii) {
    const StackGeom g = stack_geom(p);
    const uint32_t S = (uint32_t)p.tc_na;
    const uint32_t idesc = umma_idesc_e2m1_e4m3(128, kT5N);
    const uint64_t ring0 = umma_desc_sw128(tm.ring, 1024u);
    uint32_t st = 0, sph = 0;   // ring stage of the chunk and the parity of its fill
    uint32_t ts = 0, tph = 0;   // TMEM slot and the parity of its use
    uint32_t gc = 0;            // chunks so far
    bool ok = true;
    for (int jl = 0; jl < mine && ok; ++jl) {
        const TcJob q = t5_tcjob(p, g, b, G, jl, xbuf, dbuf);
        // the job's inputs (B digits) are in
        int okin = 1;
        if (lane == 0) okin = t5_wait_input(q, fillw, xbar, dbar) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, okin, 0)) {
            ok = false;
            break;
        }
        const int nch = (q.NB + kT5Chunk - 1) / kT5Chunk;
        uint64_t bd = umma_desc(q.inb, 32u * (uint32_t)q.kk, 128u);
        const uint64_t bstep = (uint64_t)(4 * q.kk);   // one block of digits (64*kk bytes) in 16-byte units
        for (int c = 0; c < nch; ++c, ++gc) {
            if (gc % kT5Issuers == (uint32_t)ii) {
                if (!tc_warp_wait(tm.full + st, sph, lane) ||
                    (gc >= (uint32_t)kT5TSlots && !tc_warp_wait(tm.tempty + ts, tph ^ 1u, lane))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t ad = ring0 + (uint64_t)((st * kT5Tile) >> 4);
                const uint32_t dt = tbase + (uint32_t)(kT5Chunk * kT5N) * ts;
                const int nbc = min(kT5Chunk, q.NB - kT5Chunk * c);
                if (lane == 0) {
                    mma_f8f6f4(dt, ad, bd, idesc, 0u);
#pragma unroll
                    for (int j = 1; j < kT5Chunk; ++j)
                        if (j < nbc)
                            mma_f8f6f4(dt + (uint32_t)(kT5N * j),
                                       ad + (uint64_t)((j / kT5Sub) * (kT5SubTile >> 4) + 2 * (j % kT5Sub)),
                                       bd + bstep * (uint64_t)j, idesc, 0u);
                    mma_commit(tm.tfull + ts);
                    mma_commit(tm.empty + st);
                }
                __syncwarp();
            }
            bd += bstep * (uint64_t)kT5Chunk;
            if (++st == S) {
                st = 0;
                sph ^= 1u;
            }
            if (++ts == (uint32_t)kT5TSlots) {
                ts = 0;
                tph ^= 1u;
            }
        }
    }
    if (!ok && lane == 0) record_error(GX_DEVERR_TIMEOUT);
    if (lane == 0) mma_commit(tm.fin);
    __syncwarp();
    tc_warp_wait(tm.fin, 0u, lane);
}

// the raw block scales of blocks c0..c0+3 of one row (the last block's past nb)
__device__ __forceinline__ void t5_scales(const uint8_t * sb, const uint8_t * dyp, int c0, int nb, uint16_t (&dy)[kT5Chunk],
                                          uint8_t (&e)[kT5Chunk]) {
#pragma unroll
    for (int j = 0; j < kT5Chunk; ++j) {
        const int bb = min(c0 + j, nb - 1);
        dy[j] = *reinterpret_cast<const uint16_t *>(dyp + 2 * bb);
        e[j] = sb[bb];
    }
}

// Epilogue warp sp (TMEM lanes 32sp.., rows 32sp.. of every job).
__device__ __forceinline__ void t5_epilogue(const StackParams & p, const T5Team & tm, uint32_t tbase, int sp, int lane,
                                            int b, int G, int mine, const int * fillw, uint64_t * xbar, uint64_t * dbar,
                                            const uint8_t * xbuf, const uint8_t * dbuf) {
    const StackGeom g = stack_geom(p);
    const int row = 32 * sp + lane;
    uint32_t ts = 0, tph = 0;   // TMEM slot and the parity of its use
    bool ok = true;
    for (int jl = 0; jl < mine && ok; ++jl) {
        const TcJob q = t5_tcjob(p, g, b, G, jl, xbuf, dbuf);
        const StackJob & J = q.J;
        const int p2 = jl & 1, NB = q.NB, nch = (NB + kT5Chunk - 1) / kT5Chunk;
        // the job's scales landed; its input buffer (the activation scales read here) holds its key
        int okin = 1;
        if (lane == 0) okin = t5_wait_input(q, fillw, xbar, dbar) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, okin, 0) || !tc_warp_wait(tm.sfull + p2, (uint32_t)((jl >> 1) & 1), lane)) {
            ok = false;
            break;
        }
        const uint8_t * sb = tm.sbuf + p2 * tm.sbuf_stride + row * NB;   // this row's block scales
        const uint8_t * dyp = q.inb + q.in_doff + 2 * (J.gu ? 0 : sp) * NB;   // its activation row's scales
        const int col = J.gu ? 0 : 2 * sp;                                  // its activation row's digit columns
        float sumf = 0.0f, sce = 0.0f, sie = 0.0f;
        uint16_t dy[kT5Chunk];
        uint8_t e8[kT5Chunk];
        t5_scales(sb, dyp, 0, NB, dy, e8);
        for (int c = 0; c < nch; ++c) {
            float scv[kT5Chunk];
#pragma unroll
            for (int j = 0; j < kT5Chunk; ++j) scv[j] = __fmul_rn(h2f(dy[j]), e8m0_half(e8[j]));
            // the next chunk's scales load while this chunk's MMAs are awaited
            t5_scales(sb, dyp, kT5Chunk * (c + 1), NB, dy, e8);
            if (!tc_warp_wait(tm.tfull + ts, tph, lane)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t v[kT5Chunk][2];
#pragma unroll
            for (int j = 0; j < kT5Chunk; ++j)
                tmem_ld2(tc_taddr(tbase, sp, (kT5Chunk * kT5N) * (int)ts + kT5N * j + col), v[j]);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tm.tempty + ts);
            if (++ts == (uint32_t)kT5TSlots) {
                ts = 0;
                tph ^= 1u;
            }
            const int nbc = min(kT5Chunk, NB - kT5Chunk * c);
#pragma unroll
            for (int j = 0; j < kT5Chunk; ++j) {
                if (j < nbc) {
                    const float x = __fmaf_rn(16.0f, __uint_as_float(v[j][0]), __uint_as_float(v[j][1]));
                    const float si = __fadd_rn(x, x);   // the block's integer dot, exact
                    if ((j & 1) == 0) {
                        sce = scv[j];
                        sie = si;
                    } else {
                        sumf = __fadd_rn(sumf, __fmaf_rn(sce, sie, __fmul_rn(scv[j], si)));
                    }
                }
            }
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(tm.sfree + p2);
        // the row's dot to the tails, once they have read job jl - 2's
        if (jl >= 2 && !tc_warp_wait(tm.xfree + p2, (uint32_t)(((jl >> 1) - 1) & 1), lane)) {
            ok = false;
            break;
        }
        tm.xchg[128 * p2 + row] = sumf;
        __syncwarp();
        if (lane == 0) mbar_arrive(tm.xfull + p2);
    }
    if (!ok && lane == 0) record_error(GX_DEVERR_TIMEOUT);
}

// Tail warp s (0, 1): per job, once the epilogue wrote its row dots, the
// input buffer is released (every MMA of the job is done and every epilogue
// warp has read its scales), then SwiGLU of gate row 32s + lane with up row
// 64 + 32s + lane and the digit quantization of that block of the down
// inputs (gate/up jobs), or the combine of the k experts' rows (down jobs,
// s = 0).
__device__ __forceinline__ void t5_tail(const StackParams & p, const T5Team & tm, int s, int lane, int b, int G,
                                        int mine, const uint8_t * xbuf, const uint8_t * dbuf, int * bufdone) {
    const StackGeom g = stack_geom(p);
    bool ok = true;
    for (int jl = 0; jl < mine && ok; ++jl) {
        const TcJob q = t5_tcjob(p, g, b, G, jl, xbuf, dbuf);
        const StackJob & J = q.J;
        const int p2 = jl & 1;
        if (!tc_warp_wait(tm.xfull + p2, (uint32_t)((jl >> 1) & 1), lane)) {
            ok = false;
            break;
        }
        if (s == 0 && lane == 0) {
            __threadfence_block();
            atomicAdd(bufdone + (J.gu ? 0 : kStackBufs) + q.bi, 1);
        }
        const float * xc = tm.xchg + 128 * p2;
        float d[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) d[i] = xc[32 * i + lane];
        __syncwarp();
        if (lane == 0) mbar_arrive(tm.xfree + p2);
        const StackLayer & ly = p.layers[J.L];
        if (J.gu) {
            const float gate = d[s], up = d[2 + s];
            const float a = p.act == 1 ? act_swiglu_oai(gate, up, p.alpha, p.limit) : act_swiglu(gate, up);
            quant_value_digits(a, ly.actq + (int64_t)J.t * p.k * p.ald.pitch, J.pair - J.t * p.k, p.k, p.I / 32,
                               p.ald.d_off, J.r0 / 32 + s, lane);
            fence_proxy_async_global();
            __syncwarp();
            if (lane == 0) {
                fence_acq_rel_gpu();
                atomicAdd(p.gu_done + J.L * p.T + J.t, 1);
            }
        } else if (s == 0) {
            // output row r0 + lane: sum over slots mm of w[mm] * dot(expert mm, row), in slot order
            const float * wr = ly.rw + (int64_t)J.t * p.k;
            float accf = 0.0f;
#pragma unroll
            for (int mm = 0; mm < 4; ++mm) {
                const float prod = __fmul_rn(d[mm], wr[mm]);
                accf = mm == 0 ? prod : __fadd_rn(accf, prod);
            }
            ly.out[(int64_t)J.t * p.H + J.r0 + lane] = accf;
        }
    }
    if (!ok && lane == 0) record_error(GX_DEVERR_TIMEOUT);
}

// Publishes cnt quantized x blocks of layer L written by this warp (their
// digit rows visible to the TMA loads of every CTA first).
__device__ __forceinline__ void t5_count_blocks(int32_t * q_done, int L, int cnt, int lane) {
    if (cnt == 0) return;
    fence_proxy_async_global();
    __syncwarp();
    if (lane == 0) {
        fence_acq_rel_gpu();
        atomicAdd(q_done + L, cnt);
    }
}

// Row mode 5 on warps 0, 1 and 4-13: TMEM, the layer inputs' digit rows, the
// roles, and TMEM freed once the MMAs have landed.
__device__ __forceinline__ void stack_t5(const StackParams & p, uint8_t * smem, int warp, int lane, int b, int G,
                                         int mine, const int32_t * slots, const StackWeights * wt, uint64_t * xbar,
                                         uint64_t * dbar, const int * fillw, int * bufdone, const uint8_t * xbuf,
                                         const uint8_t * dbuf) {
    const int nbmax = (p.H > p.I ? p.H : p.I) / 32;
    const T5Team tm = t5_team(smem, p.tc_off, nbmax, p.tc_na);
    if (warp == 0 || warp == 13) {
        if (lane == 0) t5_producer(p, tm, b, G, mine, slots, warp == 0 ? 0 : 1);
        return;
    }
    if (warp == 12) {
        if (lane == 0) t5_scale_producer(p, tm, b, G, mine, slots, wt);
        return;
    }
    // warps 1 and 4-11 from here on
    constexpr int kBar = 32 * (4 + kT5Issuers);   // the epilogue warps 4-7 and the issuers (the TMEM users)
    if (warp == 4) {
        tmem_alloc(tm.tslot, kT5Cols);
        tmem_relinquish();
    }
    if (warp >= 4 && warp < 10) {
        // x of every layer as digit rows, block i of layer L (i < T*H/32) on
        // warp (L*T*H/32 + i) mod 6G of the grid; each warp counts its blocks
        // of a layer into q_done[L] once they are visible
        const int nblk = p.H / 32, per = p.T * nblk;
        const int nw = 6 * G;
        int cur = -1, cnt = 0;
        for (int i = 6 * b + (warp - 4); i < p.NL * per; i += nw) {
            const int L = i / per;
            if (L != cur) {
                t5_count_blocks(p.q_done, cur, cnt, lane);
                cur = L;
                cnt = 0;
            }
            const int r = i - L * per, t = r / nblk, ib = r - t * nblk;
            const StackLayer & ly = p.layers[L];
            quant_block_digits<false>(ly.x + (int64_t)t * p.H, ly.xq + (int64_t)t * p.alx.pitch, 0, 1, nblk, p.alx.d_off,
                                      ib, lane);
            ++cnt;
        }
        t5_count_blocks(p.q_done, cur, cnt, lane);
    }
    if (warp == 8 || warp == 9) {
        t5_tail(p, tm, warp - 8, lane, b, G, mine, xbuf, dbuf, bufdone);
        return;
    }
    tc_fence_before();
    named_barrier(3, kBar);
    tc_fence_after();
    const uint32_t tbase = *reinterpret_cast<volatile uint32_t *>(tm.tslot);
    if (t5_issuer_index(warp) >= 0)
        t5_issuer(p, tm, tbase, b, G, mine, xbar, dbar, fillw, xbuf, dbuf, lane, t5_issuer_index(warp));
    else
        t5_epilogue(p, tm, tbase, warp - 4, lane, b, G, mine, fillw, xbar, dbar, xbuf, dbuf);
    tc_fence_before();
    named_barrier(4, kBar);
    tc_fence_after();
    if (warp == 4) tmem_dealloc(tbase, kT5Cols);
}

}  // namespace gx
