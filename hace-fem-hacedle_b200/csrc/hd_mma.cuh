// hd_mma.cuh -- helpers of the mma.sync decode Q-GEMV kernels: cp.async
// copies, ldmatrix, the m16n8k16 fp16 MMA, the exact fp16 unpacking of quant
// words into A fragments, and thread-block-cluster barriers and stores.
#pragma once
#include <cuda_fp16.h>

#include "hd_internal.cuh"

namespace {

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void cp16(uint32_t s, const void *g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(g) : "memory");
}
__device__ __forceinline__ void cp8(uint32_t s, const void *g) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(g) : "memory");
}
__device__ __forceinline__ void cp4(uint32_t s, const void *g) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// cp.async.wait_group with a run-time count (0..8; larger counts wait for all).
__device__ __forceinline__ void cp_wait_dyn(int n) {
    switch (n) {
    case 1: cp_wait<1>(); break;
    case 2: cp_wait<2>(); break;
    case 3: cp_wait<3>(); break;
    case 4: cp_wait<4>(); break;
    case 5: cp_wait<5>(); break;
    case 6: cp_wait<6>(); break;
    case 7: cp_wait<7>(); break;
    case 8: cp_wait<8>(); break;
    default: cp_wait<0>(); break;
    }
}
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// d = a b + c, m16n8k16, fp16 operands, fp32 accumulators.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1, const float (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %11, %12, %13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}
__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&a), *reinterpret_cast<const __half2 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
    __half2 r = __hfma2(*reinterpret_cast<const __half2 *>(&a), *reinterpret_cast<const __half2 *>(&b),
                        *reinterpret_cast<const __half2 *>(&c));
    return *reinterpret_cast<uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// Magic fp16 pairs.  A nibble q under exponent 0x64 is 1024 + q; a nibble
// kept in bits 4..7 is 1024 + 16 q.  Both are exact, and so are the fixups.
constexpr uint32_t H_MAGIC = 0x64006400u;   // (1024, 1024)
constexpr uint32_t H_SIXTEENTH = 0x2C002C00u;  // (1/16, 1/16)

// One 32-bit word of a row's unit -> the four A pairs (values (4t, 4t+2),
// (4t+1, 4t+3) of the low half and the same of the high half) as exact fp16
// quants with the type's offset removed.  ext: the row's extra bits already
// shifted for this thread (Q5_0: qh' >> t; Q6_K: high-bit words >> 2t).
template <int TYPE>
__device__ __forceinline__ void unpack_word(uint32_t w, uint32_t ex0, uint32_t ex1, uint32_t (&o)[4]) {
    const uint32_t w8 = w >> 8;
    if constexpr (TYPE == HD_TYPE_Q8_0) {
        // signed bytes: (byte ^ 0x80) under the exponent is 1152 + value
        const uint32_t lo02 = (w & 0x00FF00FFu) ^ 0x64806480u, lo13 = (w8 & 0x00FF00FFu) ^ 0x64806480u;
        o[0] = hsub2u(lo02, 0x64806480u);  // (1152, 1152)
        o[1] = hsub2u(lo13, 0x64806480u);
        (void)ex0;
        (void)ex1;
    } else {
        uint32_t lo02 = (w & 0x000F000Fu) | H_MAGIC, lo13 = (w8 & 0x000F000Fu) | H_MAGIC;
        uint32_t hi02 = (w & 0x00F000F0u) | H_MAGIC, hi13 = (w8 & 0x00F000F0u) | H_MAGIC;
        uint32_t lsub, hadd;
        if constexpr (TYPE == HD_TYPE_Q4_K) {
            lsub = 0x64006400u;  // 1024
            hadd = 0xD400D400u;  // -64
            (void)ex0;
            (void)ex1;
        } else if constexpr (TYPE == HD_TYPE_Q5_0) {
            // ex0 = qh' >> t: low value c's fifth bit at 8c + 4, high value c's at 8c
            lo02 |= ex0 & 0x00100010u;
            lo13 |= (ex0 >> 8) & 0x00100010u;
            hi02 |= (ex0 << 8) & 0x01000100u;
            hi13 |= ex0 & 0x01000100u;
            lsub = 0x64106410u;  // 1040
            hadd = 0xD500D500u;  // -80
            (void)ex1;
        } else {  // Q6_K: ex0 / ex1 = high-bit words of the low / high half >> 2t (bits 8c, 8c+1)
            lo02 |= (ex0 << 4) & 0x00300030u;
            lo13 |= (ex0 >> 4) & 0x00300030u;
            hi02 |= (ex1 << 8) & 0x03000300u;
            hi13 |= ex1 & 0x03000300u;
            lsub = 0x64206420u;  // 1056
            hadd = 0xD600D600u;  // -96
        }
        o[0] = hsub2u(lo02, lsub);
        o[1] = hsub2u(lo13, lsub);
        o[2] = hfma2u(hi02, H_SIXTEENTH, hadd);
        o[3] = hfma2u(hi13, H_SIXTEENTH, hadd);
    }
}

// Thread-block clusters: rank in the cluster, the split arrive/wait barrier
// (arrive early, wait before the first remote access), and stores into
// another CTA's shared memory.
__device__ __forceinline__ uint32_t mm_cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void mm_cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void mm_cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void mm_cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ uint32_t mm_mapa(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void mm_st_cluster(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

}  // namespace
