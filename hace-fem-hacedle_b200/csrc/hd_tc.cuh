// hd_tc.cuh -- shared helpers of the tcgen05 kernels: mbarriers with bounded
// waits, tensor-memory fences and loads, SWIZZLE_128B shared-memory
// descriptors and stores, instruction descriptors.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>

#include "hd_internal.cuh"

namespace {

constexpr long long SPIN_LIMIT = 2000000000; // clock64 cycles (~1 s)

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: true when the phase completed, false on expiry (which sets
// the flag) or once another thread has set the flag.  The flag and the clock
// are looked at every 64th try, so that waiting threads do not flood the
// memory pipeline with loads of the flag.  Roles off the critical path pass
// sleep_ns > 0 and back off between tries, leaving issue slots to the warps
// that convert weights and issue MMAs.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int *flag, unsigned sleep_ns = 0) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    for (unsigned it = 1;; it++) {
        if (sleep_ns) __nanosleep(sleep_ns);
        if (mbar_try(bar, parity)) return true;
        if ((it & 63) == 0) {
            if (*(volatile int *)flag) return false;
            if (clock64() - t0 > SPIN_LIMIT) {
                atomicExch(flag, HD_E_TIMEOUT);
                return false;
            }
        }
    }
}
// Bounded by time only: for waits on the CTA's own asynchronous work (copies,
// MMAs) that must end before the CTA exits, also after an error.
__device__ __forceinline__ void mbar_wait_quiet(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try(bar, parity))
        if (clock64() - t0 > SPIN_LIMIT) return;
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, SWIZZLE_128B, 8-row groups 1024 B
// apart (SBO), version 1 (sm_100), base offset 0 (stage bases are 1024-aligned).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    uint64_t d = (uint64_t)((addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor: fp32 accumulate, bf16 A and B, both K-major, M=128, N=BT.
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// Same with fp16 A and B (formats 0): the exact-product mode.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

// Writes 32 bf16 values as 4 16-byte chunks (chunk index c0..c0+3) of row r
// of a SWIZZLE_128B K-major tile.
__device__ __forceinline__ void store_sw128(uint8_t *tile, int r, int c0, const float (&v)[32]) {
#pragma unroll
    for (int c = 0; c < 4; c++) {
        uint4 q;
        q.x = pack_bf16(v[8 * c + 0], v[8 * c + 1]);
        q.y = pack_bf16(v[8 * c + 2], v[8 * c + 3]);
        q.z = pack_bf16(v[8 * c + 4], v[8 * c + 5]);
        q.w = pack_bf16(v[8 * c + 6], v[8 * c + 7]);
        int chunk = (c0 + c) ^ (r & 7);
        *(uint4 *)(tile + r * 128 + chunk * 16) = q;
    }
}

// 16 consecutive fp32 columns of this warp's 32 TMEM lanes (one per thread);
// the registers are valid after tmem_wait_ld.
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Orders the uses of r after a preceding tmem_wait_ld (an empty statement
// that the compiler must assume rewrites r).
__device__ __forceinline__ void tmem_regs_ready(uint32_t (&r)[16]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

}  // namespace
