// Inline-PTX building blocks shared by the sm_100a tensor-core kernels:
// mbarriers with bounded waits, 2D TMA loads, shared-memory matrix descriptors,
// tcgen05 MMA / commit / TMEM loads and warpgroup register reallocation.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mf {
namespace tg {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// First 1024-byte-aligned byte of the dynamic shared-memory window (SWIZZLE
// atoms and UMMA descriptors want that alignment).  It is computed by pointer
// arithmetic on the __shared__ array itself, so the compiler keeps the state
// space and every access through the result is a shared-memory load or store;
// rounding the address as an integer would leave generic loads (4% of the packed
// kernel's time at 4096^3).
__device__ __forceinline__ uint8_t* smem_align1024(uint8_t* raw) {
    return raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
}

// ------------------------------------------------------------------ mbarriers
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete sleeps
// until the phase completes or about `ns` nanoseconds pass, instead of spinning
// on issue slots that the compute warps of the CTA need.
__device__ __forceinline__ bool mbar_try_suspend(uint64_t* bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

// Longest single suspension of a waiting thread; it also bounds how late a role
// notices that another role has aborted.
constexpr uint32_t kSuspendNs = 20000;

// Upper bound of every wait, in SM clock cycles (about 2 s at 1.965 GHz).
constexpr long long kWaitCycles = 4000000000LL;

// Bounded wait for phase `parity`.  Gives up when another role of the CTA has
// set *abort, or after `budget` cycles (kWaitCycles unless a launch asks for a
// shorter one); in the latter case it records `code` in the device error word
// and sets *abort so that every other role stops too.
__device__ __forceinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, int* abort, unsigned* error,
                                               unsigned code, long long budget = kWaitCycles) {
    const long long start = clock64();
    while (true) {
        if (mbar_try_suspend(bar, parity, kSuspendNs)) return true;
        if (*(volatile int*)abort) return false;
        if (clock64() - start > budget) {
            atomicCAS(error, 0u, code);
            *(volatile int*)abort = 1;
            return false;
        }
    }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* abort, unsigned* error,
                                          unsigned code, long long budget = kWaitCycles) {
    if (mbar_try(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, abort, error, code, budget);
}

// Bounded wait that ignores the abort flag: used to drain a role's own
// asynchronous work (TMA loads, MMAs) before the CTA exits.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    const long long start = clock64();
    while (!mbar_try(bar, parity)) {
        if (clock64() - start > kWaitCycles) return;
        __nanosleep(256);
    }
}

// ------------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ------------------------------------------------------------- MMA operands
// K-major operand tile with rows of 32 bytes and the 32-byte swizzle (the
// layout TMA writes for a box of 32 bytes x rows with CU_TENSOR_MAP_SWIZZLE_32B):
// 8-row atoms of 256 bytes (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t desc_sw32(const void* tile) {
    const uint64_t addr = smem_u32(tile);
    uint64_t d = 0;
    d |= (addr >> 4) & 0x3FFFull;            // start address
    d |= (uint64_t)1 << 16;                  // leading byte offset (unused when swizzled)
    d |= (uint64_t)(256 >> 4) << 32;         // stride byte offset: 8 rows x 32 B
    d |= (uint64_t)1 << 46;                  // descriptor version (sm_100)
    d |= (uint64_t)6 << 61;                  // SWIZZLE_32B
    return d;
}

// Instruction descriptors for dense K-major A and B.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n, bool a_signed, bool b_signed) {
    return (2u << 4)                       // D = S32
           | ((a_signed ? 1u : 0u) << 7)   // A = s8 / u8
           | ((b_signed ? 1u : 0u) << 10)  // B = s8 / u8
           | ((uint32_t)(n >> 3) << 17)    // N
           | ((uint32_t)(m >> 4) << 24);   // M
}
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
    return (1u << 4)                       // D = F32
           | (0u << 7) | (0u << 10)        // A = B = F16
           | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_e4m3(int m, int n) {
    return (1u << 4)                       // D = F32
           | (0u << 7) | (0u << 10)        // A = B = E4M3
           | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D (+)= A * B; `accumulate` = 0 overwrites the TMEM columns.
__device__ __forceinline__ void mma_i8(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_f8(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// The same with A taken from TMEM: `a_tmem` addresses row 0 / first column of a
// K-major A tile, row m in lane m and 4 consecutive 8-bit K elements per column.
__device__ __forceinline__ void mma_i8_ts(uint32_t tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate));
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far is complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// --------------------------------------------------------------------- TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t columns) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(columns));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t tmem, uint32_t columns) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(columns));
}

// Consecutive TMEM columns of this thread's lane (32x32b shape).  The values are
// only valid after tmem_wait(), which takes the registers as operands so that no
// use can be scheduled ahead of the wait.
__device__ __forceinline__ void tmem_ld(uint32_t addr, uint32_t (&r)[1]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r[0]) : "r"(addr));
}

__device__ __forceinline__ void tmem_ld(uint32_t addr, uint32_t (&r)[2]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}

__device__ __forceinline__ void tmem_ld(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void tmem_ld(uint32_t addr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(addr));
}

__device__ __forceinline__ void tmem_ld(uint32_t addr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(addr));
}

__device__ __forceinline__ void tmem_wait(uint32_t (&r)[8]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7])
                 :
                 : "memory");
}

__device__ __forceinline__ void tmem_wait(uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.wait::ld.sync.aligned;"
        : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
          "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
        :
        : "memory");
}

// Eight consecutive 32-bit TMEM columns of this thread's lane from registers;
// complete once tmem_wait_st() returns.
__device__ __forceinline__ void tmem_st(uint32_t addr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(addr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ------------------------------------------------------ register reallocation
template <int N>
__device__ __forceinline__ void set_maxnreg_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
__device__ __forceinline__ void set_maxnreg_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }

}  // namespace tg
}  // namespace mf
