// Persistent, warp-specialized decode kernel for a stack of routed-expert
// layers (sm_100a).
//
// One cooperative launch (one CTA per SM) runs every layer of a micro-batch
// whose slot ids are all known when it starts. The jobs of the stack form one
// global list,
//   [gate/up jobs of layer 0][gate/up jobs of layer 1][down jobs of layer 0]
//   [gate/up jobs of layer 2][down jobs of layer 1] ... [down jobs of layer NL-1]
// and CTA b takes jobs b, b+G, b+2G, ... ; its j-th job uses ring stage j % C.
// Inside a CTA:
//   warp 0        weight producer: as soon as a stage is released, bulk-TMA
//                 copies the expert rows of the CTA's next job into it. Weights
//                 never depend on earlier jobs, so the HBM stream runs ahead
//                 across job, half-layer and layer boundaries;
//   warp 1        activation producer: waits until the job's input exists
//                 (x_L quantized; every gate/up job of token t finished) and
//                 copies the input rows into the same stage;
//   warps 2..C+1  consumers: warp c computes the jobs of stage c, releases the
//                 stage, then runs the job's epilogue (activation and its Q8
//                 quantization, or the weighted combine).
// The x_L quantization runs first, in the consumer warps of CTA L mod G.
// There is no CTA-wide barrier after set-up: roles synchronize only through
// mbarriers (full/empty per stage) and the global counters.
//
// Deadlock freedom: a job waits only on jobs of an earlier half-layer; every
// CTA issues and computes its jobs in increasing order and all CTAs are
// resident (cooperative launch), so the smallest unfinished job can always
// run. Every wait is bounded, gives up as soon as any CTA has recorded an
// error, and on giving up records GX_DEVERR_TIMEOUT; producers then let their
// copies in flight land (bounded) before the CTA exits.
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

// Bounded wait until *p reaches target (the counters only grow).
__device__ __forceinline__ bool stack_wait(const int32_t * p, int32_t target) {
    for (uint32_t i = 0; i < (1u << 23); ++i) {
        if (*reinterpret_cast<const volatile int32_t *>(p) >= target) return true;
        if (*reinterpret_cast<volatile int *>(&g_dev_error) != 0) return false;
        if (i >= 64) __nanosleep(64);
    }
    return false;
}

// Bounded mbarrier wait that also stops once another CTA recorded an error.
__device__ __forceinline__ bool stack_mbar_wait(uint64_t * bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 22); ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && *reinterpret_cast<volatile int *>(&g_dev_error) != 0) return false;
    }
    return false;
}

// One decoded job of the global list.
struct StackJob {
    int L, gu, t, r0, pair;
};

// Job order: [GU(0)] then, for B = 0..NL-1, [GU(B+1)] [D(B)]. The down jobs
// of a layer come after the gate/up jobs of the next one, so a CTA reaches
// them a whole gate/up phase after the jobs they wait on were issued.
__device__ __forceinline__ StackJob stack_job(const StackParams & p, int j) {
    StackJob J;
    int w;
    if (j < p.n_gu) {
        J.L = 0;
        J.gu = 1;
        w = j;
    } else {
        const int seg = p.n_gu + p.n_d;
        const int jj = j - p.n_gu;
        const int B = jj / seg;
        w = jj - B * seg;
        if (B + 1 < p.NL && w < p.n_gu) {
            J.L = B + 1;
            J.gu = 1;
        } else {
            J.L = B;
            J.gu = 0;
            if (B + 1 < p.NL) w -= p.n_gu;
        }
    }
    if (J.gu) {
        const int tiles = p.I / p.Rg;
        J.pair = w / tiles;
        J.r0 = (w - J.pair * tiles) * p.Rg;
        J.t = J.pair / p.k;
    } else {
        const int tiles = p.H / p.Rd;
        J.t = w / tiles;
        J.r0 = (w - J.t * tiles) * p.Rd;
        J.pair = J.t * p.k;
    }
    return J;
}

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

// Weight copies of job J into a stage, issued by the 32 lanes of the producer
// warp in parallel (one copy per lane); slot ids come from shared memory.
__device__ __forceinline__ void stack_issue_weights(const StackParams & p, const StackJob & J, const int32_t * slots,
                                                    uint8_t * stage, uint64_t * bar, int lane) {
    const StackLayer & ly = p.layers[J.L];
    const int32_t * sl = slots + J.L * p.T * p.k;
    if (J.gu) {
        const int64_t off = (int64_t)sl[J.pair] * ly.nb02 + (int64_t)J.r0 * p.nb01_g;
        const uint32_t bytes = (uint32_t)(p.Rg * p.nb01_g);
        if (lane == 0) tma_expect(bar, 2u * bytes);
        __syncwarp();
        if (p.row_copy_g) {
            // copy i: role i / Rg, row i % Rg
            for (int i = lane; i < 2 * p.Rg; i += 32) {
                const int m = i / p.Rg, r = i - m * p.Rg;
                tma_load(stage + i * p.pitch_g, (m == 0 ? ly.wg : ly.wu) + off + (int64_t)r * p.nb01_g,
                         (uint32_t)p.nb01_g, bar);
            }
        } else if (lane < 2) {
            tma_load(stage + lane * p.Rg * p.pitch_g, (lane == 0 ? ly.wg : ly.wu) + off, bytes, bar);
        }
    } else {
        const uint32_t bytes = (uint32_t)(p.Rd * p.nb01_d);
        if (lane == 0) tma_expect(bar, (uint32_t)p.k * bytes);
        __syncwarp();
        if (p.row_copy_d) {
            for (int i = lane; i < p.k * p.Rd; i += 32) {
                const int m = i / p.Rd, r = i - m * p.Rd;
                tma_load(stage + i * p.pitch_d,
                         ly.wd + (int64_t)sl[J.pair + m] * ly.nb02 + (int64_t)(J.r0 + r) * p.nb01_d, (uint32_t)p.nb01_d,
                         bar);
            }
        } else {
            for (int m = lane; m < p.k; m += 32)
                tma_load(stage + m * p.Rd * p.pitch_d, ly.wd + (int64_t)sl[J.pair + m] * ly.nb02 + (int64_t)J.r0 * p.nb01_d,
                         bytes, bar);
        }
    }
}

template <int TG, int TD>
__global__ void __launch_bounds__(64 + 32 * kStackMaxConsumers, 1) k_stack(const StackParams p) {
    static_assert(TG == GX_T_Q8_0 && TD == GX_T_Q8_0, "stack kernel rows: Q8_0");
    extern __shared__ __align__(128) uint8_t smem[];
    const int C = p.C;
    uint64_t * wfull = reinterpret_cast<uint64_t *>(smem + p.bar_off);
    uint64_t * afull = wfull + C;
    uint64_t * empty = afull + C;
    uint8_t * stages = smem + p.stage_off;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, b = blockIdx.x;
    const int NJ = p.NL * (p.n_gu + p.n_d);
    const int mine = b < NJ ? (NJ - b + G - 1) / G : 0;   // jobs of this CTA
    const int gu_per_token = p.k * (p.I / p.Rg);

    // every slot id of the launch is checked before any load and kept in
    // shared memory for the producer
    int32_t * slots = reinterpret_cast<int32_t *>(smem + p.slots_off);
    {
        int bad = 0;
        const int per = p.T * p.k;
        for (int j = tid; j < p.NL * per; j += blockDim.x) {
            const int L = j / per;
            const int32_t e = p.layers[L].slots[j - L * per];
            if (e < 0 || e >= p.layers[L].n_as) bad = 1;
            slots[j] = e;
        }
        if (__syncthreads_or(bad)) {
            if (tid == 0) record_error(GX_DEVERR_DOMAIN);
            return;
        }
    }
    if (tid == 0) {
        for (int s = 0; s < 3 * C; ++s) mbar_init(wfull + s, 1);
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == 0) {
        // ------------------------------------------------ weight producer
        int issued = 0;
        for (int jl = 0; jl < mine; ++jl) {
            const int s = jl % C, n = jl / C;
            bool ok = true;
            if (n > 0 && lane == 0) ok = stack_mbar_wait(empty + s, (uint32_t)((n - 1) & 1));
            if (!__shfl_sync(0xffffffffu, (int)ok, 0)) {
                if (lane == 0) record_error(GX_DEVERR_TIMEOUT);
                break;
            }
            stack_issue_weights(p, stack_job(p, b + jl * G), slots, stages + s * p.stage_bytes, wfull + s, lane);
            ++issued;
        }
        // let the last copy of every stage land before the CTA can exit
        if (lane == 0)
            for (int jl = issued - C > 0 ? issued - C : 0; jl < issued; ++jl)
                stack_mbar_wait(wfull + jl % C, (uint32_t)((jl / C) & 1));
        return;
    }
    if (warp == 1) {
        // -------------------------------------------- activation producer
        if (lane != 0) return;
        int issued = 0;
        for (int jl = 0; jl < mine; ++jl) {
            const int s = jl % C, n = jl / C;
            if (n > 0 && !stack_mbar_wait(empty + s, (uint32_t)((n - 1) & 1))) {
                record_error(GX_DEVERR_TIMEOUT);
                break;
            }
            const StackJob J = stack_job(p, b + jl * G);
            const StackLayer & ly = p.layers[J.L];
            const bool ok = J.gu ? stack_wait(p.q_done + J.L, 1) : stack_wait(p.gu_done + J.L * p.T + J.t, gu_per_token);
            if (!ok) {
                record_error(GX_DEVERR_TIMEOUT);
                break;
            }
            __threadfence();
            fence_proxy_async_global();
            uint8_t * st = stages + s * p.stage_bytes;
            if (J.gu) {
                tma_expect(afull + s, (uint32_t)p.alx.pitch);
                tma_load(st + p.act_off_g, ly.xq + (int64_t)J.t * p.alx.pitch, (uint32_t)p.alx.pitch, afull + s);
            } else {
                const uint32_t bytes = (uint32_t)(p.k * p.ald.pitch);
                tma_expect(afull + s, bytes);
                tma_load(st + p.act_off_d, ly.actq + (int64_t)J.t * p.k * p.ald.pitch, bytes, afull + s);
            }
            ++issued;
        }
        for (int jl = issued - C > 0 ? issued - C : 0; jl < issued; ++jl)
            stack_mbar_wait(afull + jl % C, (uint32_t)((jl / C) & 1));
        return;
    }

    // ------------------------------------------------------------ consumers
    const int c = warp - 2;
    if (c >= C) return;
    // quantize the inputs of layers L = b, b+G, ... (one warp per Q8 block)
    {
        const int nblk = p.H / 32;
        bool any = false;
        for (int L = b; L < p.NL; L += G) {
            const StackLayer & ly = p.layers[L];
            for (int wi = c; wi < p.T * nblk; wi += C) {
                const int t = wi / nblk, ib = wi - t * nblk;
                quant_block_split<GX_T_Q8_0, false>(ly.x + (int64_t)t * p.H, ly.xq + (int64_t)t * p.alx.pitch, p.alx, ib,
                                                    lane);
            }
            any = true;
        }
        if (any) {
            fence_proxy_async_global();
            named_barrier(1, 32 * C);
            if (c == 0 && lane == 0) {
                __threadfence();
                for (int L = b; L < p.NL; L += G) atomicExch(p.q_done + L, 1);
            }
        }
    }
    float * scratch = reinterpret_cast<float *>(smem + p.scratch_off) + c * 64;
    const int par = lane >> 4;   // block parity of this lane
    for (int jl = c; jl < mine; jl += C) {
        const int n = jl / C;
        const uint32_t ph = (uint32_t)(n & 1);
        const bool ok = stack_mbar_wait(wfull + c, ph) && stack_mbar_wait(afull + c, ph);
        if (__any_sync(0xffffffffu, !ok)) {
            if (lane == 0) record_error(GX_DEVERR_TIMEOUT);
            break;
        }
        const StackJob J = stack_job(p, b + jl * G);
        const StackLayer & ly = p.layers[J.L];
        const uint8_t * st = stages + c * p.stage_bytes;
        if (J.gu) {
            // lane = par*16 + role*8 + i: gate (role 0) or up (role 1) row i
            const int row = lane & 15;
            const uint8_t * rb[1] = {st + row * p.pitch_g + 32 * par};
            const uint8_t * ab[1] = {st + p.act_off_g + 32 * par};
            const uint8_t * ad[1] = {st + p.act_off_g + p.alx.d_off};
            float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
            q8_0_rows<1>(rb, ab, ad, par, p.H / 64, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + c);   // the stage is free
            const float dot = q8_0_finish(acc[0]);
            const float up = __shfl_down_sync(0xffffffffu, dot, 8);
            const int nblk = p.I / p.qblk, blk = J.r0 / p.qblk;
            if (lane < p.Rg) {
                const float a = p.act == 1 ? act_swiglu_oai(dot, up, p.alpha, p.limit) : act_swiglu(dot, up);
                ly.act[(int64_t)J.pair * p.I + J.r0 + lane] = a;
            }
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                __threadfence();
                last = atomicAdd(ly.cnt + J.pair * nblk + blk, 1) == p.qblk / p.Rg - 1;
            }
            if (__shfl_sync(0xffffffffu, last, 0)) {
                // this job finished the Q8 block last: quantize it
                __threadfence();
                quant_block_split<GX_T_Q8_0, true>(ly.act + (int64_t)J.pair * p.I, ly.actq + (int64_t)J.pair * p.ald.pitch,
                                                   p.ald, blk, lane);
                fence_proxy_async_global();
                __syncwarp();
            }
            if (lane == 0) {
                __threadfence();
                atomicAdd(p.gu_done + J.L * p.T + J.t, 1);
            }
        } else {
            // lane = par*16 + q: weight rows q and q+16 of the job's k*Rd rows
            // (row R is row R % Rd of expert R / Rd); eight consecutive lanes
            // read eight consecutive rows, so the 16-byte loads of a quarter
            // warp fall in distinct bank groups
            const int q = lane & 15;
            const int m0 = q / p.Rd, m1 = (q + 16) / p.Rd;
            const uint8_t * rb[2] = {st + q * p.pitch_d + 32 * par, st + (q + 16) * p.pitch_d + 32 * par};
            const uint8_t * a0 = st + p.act_off_d + m0 * p.ald.pitch;
            const uint8_t * a1 = st + p.act_off_d + m1 * p.ald.pitch;
            const uint8_t * ab[2] = {a0 + 32 * par, a1 + 32 * par};
            const uint8_t * ad[2] = {a0 + p.ald.d_off, a1 + p.ald.d_off};
            float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            q8_0_rows<2>(rb, ab, ad, par, p.I / 64, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + c);
            const float d0 = q8_0_finish(acc[0]);
            const float d1 = q8_0_finish(acc[1]);
            if (lane < 16) {
                scratch[q] = d0;
                scratch[q + 16] = d1;
            }
            __syncwarp();
            if (lane < p.Rd) {
                const float * wr = ly.rw + (int64_t)J.t * p.k;
                float accf = __fmul_rn(scratch[lane], wr[0]);
                for (int mm = 1; mm < p.k; ++mm) accf = __fadd_rn(accf, __fmul_rn(scratch[mm * p.Rd + lane], wr[mm]));
                ly.out[(int64_t)J.t * p.H + J.r0 + lane] = accf;
            }
            __syncwarp();
        }
    }
}

}  // namespace gx
