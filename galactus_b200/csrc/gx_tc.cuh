// 5th-generation tensor-core (tcgen05) and tensor-memory helpers shared by
// the tensor-core prefill and the tensor-core MXFP4 stack kernel (sm_100a):
// TMEM allocation, MMA issue and commit, TMEM loads and stores, shared-memory
// matrix and instruction descriptors, packed f32x2 arithmetic and a bounded
// mbarrier wait.
#pragma once

#include <cstdint>

#include <cuda.h>

#include "gx_device.cuh"

namespace gx {

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ void tmem_alloc(uint32_t * dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D[tmem] = A x B^T (int8 x int8 -> int32), both K-major, one thread
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
        : "memory");
}
// D[tmem] = A x B^T in kind::f8f6f4 (A e2m1 in the 16U4_ALIGN16B shared
// layout, B e4m3, f32 accumulators), both K-major, one thread
__device__ __forceinline__ void mma_f8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
        : "memory");
}
// the mbarrier arrives once every MMA this thread issued before has completed
__device__ __forceinline__ void mma_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// A 3-D tile of the tensor map into shared memory (no multicast: the
// weights are this GPU's own memory)
__device__ __forceinline__ void tma_load_3d(void * dst, const CUtensorMap * map, int x, int y, int z, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// A 5-D tile of the tensor map into shared memory (no multicast: the
// weights are this GPU's own memory)
__device__ __forceinline__ void tma_load_5d(void * dst, const CUtensorMap * map, int x0, int x1, int x2, int x3, int x4,
                                            uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x0), "r"(x1), "r"(x2), "r"(x3), "r"(x4), "r"(smem_u32(bar))
        : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major operand without swizzling:
// core matrices of 8 rows x 16 bytes stored as 128 contiguous bytes, the
// two 16-byte halves of a 32-byte K step lbo bytes apart, consecutive
// 8-row groups sbo bytes apart (version 1, base offset 0, layout type 0).
__device__ __forceinline__ uint64_t umma_desc(const void * smem, uint32_t lbo, uint32_t sbo) {
    const uint32_t a = smem_u32(smem);
    return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Shared-memory matrix descriptor of a K-major operand in the 128-byte
// swizzled layout that TMA writes with CU_TENSOR_MAP_SWIZZLE_128B: rows of
// 128 bytes, the 16-byte chunks of row r XOR-ed with r % 8, 8-row atoms of
// 1024 bytes sbo apart (atoms 1024-byte aligned, base offset 0); a K step
// inside the row advances the start address (version 1, layout type 2).
__device__ __forceinline__ uint64_t umma_desc_sw128(const void * smem, uint32_t sbo) {
    const uint32_t a = smem_u32(smem);
    return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) |
           (1ull << 46) | (2ull << 61);
}

// instruction descriptor: s32 accumulator, signed int8 A and B, both K-major
__host__ __device__ constexpr uint32_t umma_idesc_i8(uint32_t M, uint32_t N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// instruction descriptor of kind::f8f6f4: f32 accumulator, A e2m1 (format 5),
// B e4m3 (format 0), both K-major
__host__ __device__ constexpr uint32_t umma_idesc_e2m1_e4m3(uint32_t M, uint32_t N) {
    return (1u << 4) | (5u << 7) | (0u << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// 2 and 8 consecutive 32-bit columns of this thread's TMEM lane (no wait)
__device__ __forceinline__ void tmem_ld2(uint32_t taddr, uint32_t (&v)[2]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(v[0]), "=r"(v[1]) : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}

// 16 consecutive 32-bit columns of this thread's TMEM lane (no wait)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 consecutive columns of this thread's TMEM lane set to v
__device__ __forceinline__ void tmem_st32_const(uint32_t taddr, uint32_t v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
        "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
        "r"(v)
        : "memory");
}
__device__ __forceinline__ void tmem_st16_const(uint32_t taddr, uint32_t v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
        "%1};" ::"r"(taddr),
        "r"(v)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// The accumulators start at the integer 0x4B400000, the bits of 1.5 * 2^23:
// a partial |p| < 2^22 added to it (exactly, in int32) lands in the mantissa,
// so the tile read as f32 is 12582912 + p and one exact float subtract gives
// (float)p (no conversion instruction)
constexpr uint32_t kMagicBits = 0x4B400000u;
constexpr float kMagic = 12582912.0f;

// f32 pairs in 64-bit registers: two IEEE operations per instruction
// (f32x2, round to nearest, no flush)
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ uint64_t u2pack(uint32_t a, uint32_t b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float & a, float & b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t sub_x2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t fma_x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// non-blocking test of an mbarrier phase
__device__ __forceinline__ bool mbar_test_wait(uint64_t * bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait on an mbarrier phase for the hand-offs between warps of one
// pipeline: a first non-blocking test, then try_wait polls that suspend the
// thread (it issues nothing while suspended) until the phase completes or a
// system-dependent time limit passes; gives up after 2^20 polls or once any
// CTA has recorded an error.
__device__ __forceinline__ bool mbar_spin(uint64_t * bar, uint32_t parity) {
    if (mbar_test_wait(bar, parity)) return true;
    for (uint32_t i = 0; i < (1u << 20); ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u && *reinterpret_cast<volatile int *>(&g_dev_error) != 0) return false;
    }
    return false;
}

__device__ __forceinline__ bool mma_wait(uint64_t * bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 20); ++i) {
        if (mbar_try_wait_sleep(bar, parity, 500u)) return true;
        if ((i & 63u) == 63u && *reinterpret_cast<volatile int *>(&g_dev_error) != 0) return false;
    }
    return false;
}

}  // namespace gx
