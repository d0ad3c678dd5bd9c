// Expert-grouped prefill on the 5th-generation tensor cores (sm_100a):
// tcgen05.mma kind::i8 with operands staged in shared memory by bulk copies,
// int32 accumulators in tensor memory, and the reference's float tail on the
// CUDA cores.
//
// Q8_0 x Q8_0 (ggml_vec_dot_q8_0_q8_0, NEON order, diff:1049-1054,
// 1074-1163): per 32-element block b the four integer partials
//   p_l = sum_m x[4l+m] y[4l+m] + x[16+4l+m] y[16+4l+m]      (l = 0..3)
// each enter their own float chain acc_l = fma((float)p_l, dx*dy, acc_l),
// one set of chains for even blocks and one for odd blocks, and the row's
// dot is ((e0+e1)+(e2+e3)) + ((o0+o1)+(o2+o3)). The tensor core computes the
// partials exactly: the B operand holds, for each token n, four copies of
// its activation block, copy l keeping only the eight bytes of lane l (the
// others zero), so one M=128 x N=64 x K=32 MMA per block writes p_l(m, n) to
// TMEM column 4n + l of row m. Each block's tile accumulates onto the
// integer 0x4B400000 (1.5 * 2^23 as f32), so the epilogue reads the partials
// as floats offset by 12582912 and one exact subtract recovers them; eight
// tiles of 64 columns rotate through the 512 TMEM columns while the epilogue
// warps read them (tcgen05.ld 32x32b), store the constant back (tcgen05.st)
// and run the chains in block order (packed f32x2 subtract and fma).
//
// A unit is (chunk of <= 16 (token, slot) pairs of one expert, tile of 128
// weight rows): gate/up units take gate rows r0..r0+63 and up rows
// r0..r0+63 of the expert (the SwiGLU pairs gate row i with up row i);
// down units take 128 rows of the down matrix. One CTA per unit, 20 warps:
//   warp 0        producer: per chunk of 8 blocks, the unit's weight rows
//                 as TMA tensor tiles (box 136 16-bit words x 64 or 128
//                 rows of a 3-D map over the slots) into a raw stage, and the
//                 chunk's 8 prepared B tiles (one bulk copy)
//   warp 1        TMEM allocation; lane 0 issues the MMAs and commits
//   warps 2-3     repack: thread q moves rows q and q+64's eight Q8_0 blocks
//                 from the raw stage into the UMMA K-major layout (core
//                 matrices of 8 rows x 16 bytes) and keeps each block's scale dx
//   warps 4-19    epilogue: warp w reads TMEM lanes 32*(w%4).. (its rows)
//                 and the 16 columns of tokens 4q..4q+3, q = (w-4)/4
// Every wait is bounded and gives up (recording GX_DEVERR_TIMEOUT) once any
// CTA has recorded an error; TMEM is freed after the MMAs in flight land.
#pragma once

#include <cstdint>

#include "gx_device.cuh"
#include "gx_kernels.h"
#include "gx_tc.cuh"

namespace gx {

// ---------------------------------------------------------------- layout

constexpr int kMmaKb = 8;              // Q8_0 blocks per stage
constexpr int kMmaBufs = 8;            // TMEM tiles of kMmaN columns
constexpr int kMmaRawPitch = 272;      // bytes per weight row in the raw stage (one box row)
constexpr int kMmaThreads = 20 * 32;   // 5 warps per SM sub-partition: up to 96 registers a thread
constexpr int kMmaEpiWarps = 16;       // 4 TMEM lane groups x 4 token quarters

struct MmaSmem {
    static constexpr uint32_t raw = 0;                                              // [2][128][272]
    static constexpr uint32_t atile = raw + 2 * kMmaRows * kMmaRawPitch;            // [2][8][128 x 32]
    static constexpr uint32_t btile = atile + 2 * kMmaKb * kMmaRows * 32;           // [2][8][64 x 32]
    static constexpr uint32_t dx = btile + 2 * kMmaKb * kMmaN * 32;                 // [64][128] f32
    static constexpr uint32_t dy = dx + kMmaMaxBlocks * kMmaRows * 4;               // [64][16] f32
    static constexpr uint32_t xch = dy + kMmaMaxBlocks * kMmaTok * 4;               // [16][64] f32 up dots
    static constexpr uint32_t bars = xch + kMmaTok * 64 * 4;                        // mbarriers
    static constexpr uint32_t nbars = 2 + 2 + 2 + 2 * kMmaBufs + kMmaMaxBlocks / kMmaKb + 1;
    static constexpr uint32_t tmem_slot = bars + nbars * 8;
    static constexpr uint32_t total = tmem_slot + 16;
};
static_assert(MmaSmem::total <= kMaxSmem, "prefill MMA shared memory");

// offset of row r, K-half c of a K-major tile in core-matrix order
__device__ __forceinline__ uint32_t core_off(int r, int c) { return (uint32_t)((r >> 3) * 256 + c * 128 + (r & 7) * 16); }

// ------------------------------------------------------ B operand prep
// For chunk c and block b: 64 rows (pair n = row / 4, lane l = row % 4) of
// 32 bytes, row (n, l) = the pair's activation block with every byte outside
// lane l's eight (4l..4l+3, 16+4l..16+4l+3) zeroed, in core-matrix order;
// and the pair's block scale as f32. Pairs past the chunk's count are zero.
__global__ void k_mma_bprep(MmaPrepParams p) {
    const int c = blockIdx.y;
    const int b = blockIdx.x;
    const int row = threadIdx.x;   // 0..63
    const int n = row >> 2, l = row & 3;
    const int cnt = p.chunk_count[c];
    uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
    float d = 0.0f;
    if (n < cnt) {
        const int src = p.pair_src[p.chunk_first[c] + n];
        const uint8_t * q = p.aq + (int64_t)src * p.al.pitch;
        const uint32_t wlo = *reinterpret_cast<const uint32_t *>(q + 32 * b + 4 * l);
        const uint32_t whi = *reinterpret_cast<const uint32_t *>(q + 32 * b + 16 + 4 * l);
        uint32_t * plo = reinterpret_cast<uint32_t *>(&lo);
        uint32_t * phi = reinterpret_cast<uint32_t *>(&hi);
        plo[l] = wlo;
        phi[l] = whi;
        d = h2f(*reinterpret_cast<const uint16_t *>(q + p.al.d_off + 2 * b));
    }
    uint8_t * t = p.btiles + ((int64_t)c * p.nblk + b) * (kMmaN * 32);
    *reinterpret_cast<uint4 *>(t + core_off(row, 0)) = lo;
    *reinterpret_cast<uint4 *>(t + core_off(row, 1)) = hi;
    if (l == 0) p.dyt[((int64_t)c * p.nblk + b) * kMmaTok + n] = d;
}

// ---------------------------------------------------------------- kernel

template <int MODE>
__global__ void __launch_bounds__(kMmaThreads, 1) k_prefill_mma(const __grid_constant__ MmaParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t * bars = reinterpret_cast<uint64_t *>(smem + MmaSmem::bars);
    uint64_t * raw_full = bars;                  // [2] producer -> repack, MMA
    uint64_t * a_ready = bars + 2;               // [2] repack -> MMA (128 arrivals)
    uint64_t * slot_free = bars + 4;             // [2] MMA commit -> producer
    uint64_t * tm_full = bars + 6;               // [8] MMA commit -> epilogue
    uint64_t * tm_empty = tm_full + kMmaBufs;    // [8] epilogue (8 warps) -> MMA
    uint64_t * dx_full = tm_empty + kMmaBufs;    // [chunks] repack (128) -> epilogue
    uint64_t * dy_full = dx_full + kMmaMaxBlocks / kMmaKb;
    uint32_t * tslot = reinterpret_cast<uint32_t *>(smem + MmaSmem::tmem_slot);
    float * dx = reinterpret_cast<float *>(smem + MmaSmem::dx);
    float * dy = reinterpret_cast<float *>(smem + MmaSmem::dy);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int unit = blockIdx.x;
    const int c = unit / p.n_rt, rt = unit - c * p.n_rt;
    const int nblk = p.nblk, nch = nblk / kMmaKb;
    const int slot = p.chunk_slot[c];
    const int first = p.chunk_first[c], cnt = p.chunk_count[c];
    const int r0 = rt * (MODE == 0 ? 64 : kMmaRows);

    if (tid == 0) {
        mbar_init(raw_full + 0, 1);
        mbar_init(raw_full + 1, 1);
        mbar_init(a_ready + 0, 64);
        mbar_init(a_ready + 1, 64);
        mbar_init(slot_free + 0, 1);
        mbar_init(slot_free + 1, 1);
        for (int i = 0; i < kMmaBufs; ++i) {
            mbar_init(tm_full + i, 1);
            mbar_init(tm_empty + i, kMmaEpiWarps);
        }
        for (int i = 0; i < nch; ++i) mbar_init(dx_full + i, 64);
        mbar_init(dy_full, 1);
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(tslot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    if (warp == 0) {
        // ---------------------------------------------------- producer
        if (lane == 0) {
            tma_expect(dy_full, (uint32_t)(nblk * kMmaTok * 4));
            tma_load(dy, p.dyt + (int64_t)c * nblk * kMmaTok, (uint32_t)(nblk * kMmaTok * 4), dy_full);
        }
        for (int j = 0; j < nch; ++j) {
            const int s = j & 1;
            int ok = 1;
            if (j >= 2 && lane == 0) ok = mma_wait(slot_free + s, (uint32_t)(((j >> 1) - 1) & 1)) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) record_error(GX_DEVERR_TIMEOUT);
                break;
            }
            uint8_t * rawp = smem + MmaSmem::raw + s * kMmaRows * kMmaRawPitch;
            const uint32_t chunk_bytes = (uint32_t)(kMmaKb * 34);   // 272 = 136 16-bit words
            if (lane == 0) {
                tma_expect(raw_full + s, (uint32_t)kMmaRows * chunk_bytes + (uint32_t)(kMmaKb * kMmaN * 32));
                const int x = j * (int)(chunk_bytes / 2);
                if (MODE == 0) {
                    tma_load_3d(rawp, &p.tmap, x, r0, slot, raw_full + s);                                  // gate rows
                    tma_load_3d(rawp + 64 * kMmaRawPitch, &p.tmap, x, p.up_row0 + r0, slot, raw_full + s);   // up rows
                } else {
                    tma_load_3d(rawp, &p.tmap, x, r0, slot, raw_full + s);
                }
                tma_load(smem + MmaSmem::btile + s * (kMmaKb * kMmaN * 32),
                         p.btiles + ((int64_t)c * nblk + (int64_t)j * kMmaKb) * (kMmaN * 32), (uint32_t)(kMmaKb * kMmaN * 32),
                         raw_full + s);
            }
        }
        // the last two stages' copies land before the CTA can exit
        if (lane == 0)
            for (int j = nch - 2 < 0 ? 0 : nch - 2; j < nch; ++j) mma_wait(raw_full + (j & 1), (uint32_t)((j >> 1) & 1));
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_i8(kMmaRows, kMmaN);
            bool ok = true;
            int issued = 0;
            for (int j = 0; j < nch && ok; ++j) {
                const int s = j & 1;
                ok = mma_wait(raw_full + s, (uint32_t)((j >> 1) & 1)) && mma_wait(a_ready + s, (uint32_t)((j >> 1) & 1));
                if (!ok) break;
                tc_fence_after();
                const uint8_t * at = smem + MmaSmem::atile + s * (kMmaKb * kMmaRows * 32);
                const uint8_t * bt = smem + MmaSmem::btile + s * (kMmaKb * kMmaN * 32);
                for (int i = 0; i < kMmaKb; ++i) {
                    const int bidx = j * kMmaKb + i, buf = bidx % kMmaBufs;
                    // the buffer holds the magic constant again (epilogue)
                    ok = mma_wait(tm_empty + buf, (uint32_t)((bidx / kMmaBufs) & 1));
                    if (!ok) break;
                    tc_fence_after();
                    mma_i8(tbase + (uint32_t)(buf * kMmaN), umma_desc(at + i * kMmaRows * 32, 128, 256),
                           umma_desc(bt + i * kMmaN * 32, 128, 256), idesc, 1u);
                    mma_commit(tm_full + buf);
                    ++issued;
                }
                mma_commit(slot_free + s);   // the chunk's operands are no longer read
            }
            if (!ok) record_error(GX_DEVERR_TIMEOUT);
            // every MMA issued has landed before TMEM is freed
            if (issued > 0) {
                const int last = issued - 1;
                mma_wait(tm_full + last % kMmaBufs, (uint32_t)((last / kMmaBufs) & 1));
            }
        }
    } else if (warp < 4) {
        // ------------------------------------------------------ repack
        // thread q (0..63) takes weight rows q and q + 64
        for (int j = 0; j < nch; ++j) {
            const int s = j & 1;
            if (!mma_wait(raw_full + s, (uint32_t)((j >> 1) & 1))) {
                record_error(GX_DEVERR_TIMEOUT);
                break;
            }
            uint8_t * at = smem + MmaSmem::atile + s * (kMmaKb * kMmaRows * 32);
            for (int m = tid - 64; m < kMmaRows; m += 64) {
            const uint8_t * rr = smem + MmaSmem::raw + s * kMmaRows * kMmaRawPitch + m * kMmaRawPitch;
#pragma unroll
            for (int i = 0; i < kMmaKb; ++i) {
                // block i: fp16 d at 34i, quants at 34i+2 (34i is 0 or 2 mod 4)
                const uint8_t * bp = rr + ((34 * i) & ~3);
                uint32_t W[9];
#pragma unroll
                for (int k = 0; k < 9; ++k) W[k] = lds32(bp + 4 * k);
                uint32_t q[8];
                uint16_t d;
                if ((i & 1) == 0) {
#pragma unroll
                    for (int k = 0; k < 8; ++k) q[k] = __funnelshift_r(W[k], W[k + 1], 16);
                    d = (uint16_t)(W[0] & 0xffffu);
                } else {
#pragma unroll
                    for (int k = 0; k < 8; ++k) q[k] = W[k + 1];
                    d = (uint16_t)(W[0] >> 16);
                }
                uint8_t * t = at + i * kMmaRows * 32;
                *reinterpret_cast<uint4 *>(t + core_off(m, 0)) = make_uint4(q[0], q[1], q[2], q[3]);
                *reinterpret_cast<uint4 *>(t + core_off(m, 1)) = make_uint4(q[4], q[5], q[6], q[7]);
                dx[(j * kMmaKb + i) * kMmaRows + m] = h2f(d);
            }
            }
            fence_async_smem();   // generic writes -> tensor-core reads
            mbar_arrive(a_ready + s);
            mbar_arrive(dx_full + j);
            // the slot's next fill waits for the MMAs, which wait for a_ready
        }
    } else {
        // ---------------------------------------------------- epilogue
        const int lg = warp & 3;                 // TMEM lane group: rows 32*lg..
        const int qt = (warp - 4) >> 2;          // token quarter: tokens 4*qt..4*qt+3
        const int m = 32 * lg + lane;
        // chains of 4 tokens: acc2[parity][t] = pairs (l0, l1), (l2, l3)
        uint64_t acc2[2][4][2];
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int t = 0; t < 4; ++t) acc2[a][t][0] = acc2[a][t][1] = 0ull;
        const uint64_t magic2 = f2pack(kMagic, kMagic);
        const uint32_t tl = tbase + ((uint32_t)(32 * lg) << 16) + (uint32_t)(16 * qt);
        // every buffer starts at the magic constant (its first phase of "empty")
        for (int buf = 0; buf < kMmaBufs; ++buf) tmem_st16_const(tl + (uint32_t)(buf * kMmaN), kMagicBits);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int buf = 0; buf < kMmaBufs; ++buf) mbar_arrive(tm_empty + buf);
        // one block: read its 16 columns, restore the constant (the store
        // overlaps the chains), run the chains, free the buffer
        auto block = [&](int b, uint64_t (&ac)[4][2]) -> bool {
            const int u = b % kMmaBufs;
            if (!mma_wait(tm_full + u, (uint32_t)((b / kMmaBufs) & 1))) return false;
            tc_fence_after();
            uint32_t v[16];
            tmem_ld16(tl + (uint32_t)(u * kMmaN), v);
            tmem_wait_ld();
            tmem_st16_const(tl + (uint32_t)(u * kMmaN), kMagicBits);
            const float dxm = dx[b * kMmaRows + m];
            const float4 dq = *reinterpret_cast<const float4 *>(dy + b * kMmaTok + 4 * qt);
            const float dyv[4] = {dq.x, dq.y, dq.z, dq.w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float sc = __fmul_rn(dxm, dyv[t]);
                const uint64_t sc2 = f2pack(sc, sc);
                ac[t][0] = fma_x2(sub_x2(u2pack(v[4 * t], v[4 * t + 1]), magic2), sc2, ac[t][0]);
                ac[t][1] = fma_x2(sub_x2(u2pack(v[4 * t + 2], v[4 * t + 3]), magic2), sc2, ac[t][1]);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tm_empty + u);
            return true;
        };
        bool ok = mma_wait(dy_full, 0);
        for (int j = 0; j < nch && ok; ++j) {
            ok = mma_wait(dx_full + j, 0);
            // blocks in (even, odd) pairs: the chunk size is even
            for (int i = 0; i < kMmaKb && ok; i += 2) {
                ok = block(j * kMmaKb + i, acc2[0]);
                if (ok) ok = block(j * kMmaKb + i + 1, acc2[1]);
            }
        }
        if (!ok) record_error(GX_DEVERR_TIMEOUT);
        float dot[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            float e0, e1, e2, e3, o0, o1, o2, o3;
            f2unpack(acc2[0][t][0], e0, e1);
            f2unpack(acc2[0][t][1], e2, e3);
            f2unpack(acc2[1][t][0], o0, o1);
            f2unpack(acc2[1][t][1], o2, o3);
            const float se = __fadd_rn(__fadd_rn(e0, e1), __fadd_rn(e2, e3));
            const float so = __fadd_rn(__fadd_rn(o0, o1), __fadd_rn(o2, o3));
            dot[t] = __fadd_rn(se, so);
        }
        if constexpr (MODE == 0) {
            // rows 64..127 are the up rows: hand them to the gate rows
            float * xch = reinterpret_cast<float *>(smem + MmaSmem::xch);
            if (m >= 64)
#pragma unroll
                for (int t = 0; t < 4; ++t) xch[(4 * qt + t) * 64 + (m - 64)] = dot[t];
            named_barrier(1, 32 * kMmaEpiWarps);
            if (m < 64 && ok) {
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int n = 4 * qt + t;
                    if (n < cnt) {
                        const float up = xch[n * 64 + m];
                        const float a = p.act == 1 ? act_swiglu_oai(dot[t], up, p.alpha, p.limit) : act_swiglu(dot[t], up);
                        p.out[(int64_t)p.pair_dst[first + n] * p.out_ld + r0 + m] = a;
                    }
                }
            }
        } else {
            if (ok)
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int n = 4 * qt + t;
                    if (n < cnt) p.out[(int64_t)p.pair_dst[first + n] * p.out_ld + r0 + m] = dot[t];
                }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tbase, 512);
}

}  // namespace gx
