// hd_gemm_tc.cu -- prefill Q-GEMM on the 5th-generation tensor cores.
//
// Y[t][n] = sum_k X[t][k] W[n][k] with W a quantized GGUF weight and X fp32.
// Two kernels: the persistent, streamed v3 kernel (described at its
// definition) for weights with rows % 128 == 0, and the v1 kernel below for
// any shape.  In v1 one CTA computes a 128 (weight rows) x BT (tokens) tile with
// tcgen05.mma.cta_group::1.kind::f16 (bf16 operands, fp32 accumulator in
// TMEM: 128 lanes = weight rows, BT columns = tokens).
//
// Warp roles (9 warps):
//   warps 0-3  A producers: thread r dequantizes weight row n0+r, two 32-value
//              units per 64-wide K stage, straight from the unit-major layout
//              (one coalesced 16-byte load per unit per row), rounds to bf16
//              and writes its 128-byte row of the stage in the SWIZZLE_128B
//              K-major layout the MMA reads;
//   warps 4-7  B producers: convert the fp32 activation tile to bf16 into the
//              same swizzled layout;
//   warp 8     allocates TMEM, and one lane issues 4 MMAs (K = 16 each) per
//              stage, then tcgen05.commit to release the stage and, after the
//              last stage, to signal the accumulator.
// After the main loop warps 0-7 read the accumulator with tcgen05.ld (warp w
// reads TMEM lanes 32*(w%4).. and half of the columns) and store Y with
// lanes on consecutive weight rows (coalesced).
//
// Every mbarrier wait is bounded (about one second of clock64 time): on
// expiry the thread records HD_E_TIMEOUT in the context's flag word and stops
// waiting; the MMA warp always commits the accumulator barrier so that the
// epilogue's wait also covers any MMAs still in flight, and TMEM is freed
// before exit on every path.
#include <cstdlib>
#include <cuda.h>

#include "hd_internal.cuh"
#include "hd_tc.cuh"

namespace {

constexpr int STAGES = 4;
constexpr int BK = 64;                       // K per stage (one 128-byte swizzle row of bf16)
constexpr int A_BYTES = 128 * BK * 2;        // 16 KB

// 32 dequantized values of unit u of row r (fp32, weight semantics of the
// oracle up to rounding order), zeros outside the tensor.
template <int TYPE>
__device__ __forceinline__ void unit_values(const WView &w, int64_t r, int u, bool ok, float (&v)[32]) {
    if (!ok) {
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = 0.f;
        return;
    }
    const int64_t ur = (int64_t)u * w.rows + r;
    if constexpr (TYPE == HD_TYPE_Q8_0) {
        const uint4 *p = (const uint4 *)(w.q + ur * 32);
        uint4 a = __ldg(p), b = __ldg(p + 1);
        float d = h2f(__ldg((const unsigned short *)w.meta + ur));
        uint32_t wd[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            uint32_t x = wd[i] ^ 0x80808080u;
#pragma unroll
            for (int c = 0; c < 4; c++) v[4 * i + c] = (mag(x, c) - 8388736.0f) * d;
        }
    } else if constexpr (TYPE == HD_TYPE_Q5_0) {
        uint4 a = __ldg((const uint4 *)(w.q + ur * 16));
        uint32_t qh = __ldg((const unsigned int *)w.aux + ur);
        float d = h2f(__ldg((const unsigned short *)w.meta + ur));
        uint32_t wd[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t lo = (wd[i] & 0x0F0F0F0Fu) | ((qh >> i) & 0x10101010u);
            uint32_t hi = ((wd[i] >> 4) & 0x0F0F0F0Fu) | ((qh << (4 - i)) & 0x10101010u);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                v[4 * i + c] = (mag(lo, c) - 8388624.0f) * d;
                v[16 + 4 * i + c] = (mag(hi, c) - 8388624.0f) * d;
            }
        }
    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
        uint4 a = __ldg((const uint4 *)(w.q + ur * 16));
        uint4 m = __ldg((const uint4 *)(w.meta + ((int64_t)(u >> 3) * w.rows + r) * 16));
        int sc, mn;
        q4k_sm_regs(u & 7, m.y, m.z, m.w, sc, mn);
        float d1 = h2f((uint16_t)(m.x & 0xFFFF)) * (float)sc, m1 = h2f((uint16_t)(m.x >> 16)) * (float)mn;
        uint32_t wd[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t lo = wd[i] & 0x0F0F0F0Fu, hi = (wd[i] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                v[4 * i + c] = (mag(lo, c) - 8388608.0f) * d1 - m1;
                v[16 + 4 * i + c] = (mag(hi, c) - 8388608.0f) * d1 - m1;
            }
        }
    } else {
        const int64_t sr = (int64_t)(u >> 3) * w.rows + r;
        uint4 a = __ldg((const uint4 *)(w.q + ur * 16));
        uint2 h = __ldg((const uint2 *)w.aux + ur);
        const int8_t *scp = (const int8_t *)(w.meta + sr * 16);
        float d = h2f(__ldg(w.dsb + sr));
        int s0 = 2 * (u & 7);
        float dl = d * (float)scp[s0], dh = d * (float)scp[s0 + 1];
        uint32_t wd[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int sh = 4 - 2 * i;
            uint32_t hx = sh >= 0 ? (h.x << sh) : (h.x >> -sh), hy = sh >= 0 ? (h.y << sh) : (h.y >> -sh);
            uint32_t lo = (wd[i] & 0x0F0F0F0Fu) | (hx & 0x30303030u);
            uint32_t hi = ((wd[i] >> 4) & 0x0F0F0F0Fu) | (hy & 0x30303030u);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                v[4 * i + c] = (mag(lo, c) - 8388640.0f) * dl;
                v[16 + 4 * i + c] = (mag(hi, c) - 8388640.0f) * dh;
            }
        }
    }
}


template <int TYPE, int BT>
__global__ void __launch_bounds__(288, 1) k_qgemm_tc(WView w, const float *__restrict__ X, float *__restrict__ Y,
                                                    int T, int N, int K, int *flag) {
    extern __shared__ uint8_t smem_raw[];
    constexpr int B_BYTES = BT * BK * 2;
    __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES], acc_bar;
    __shared__ uint32_t tmem_base_sh;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * 128, t0 = blockIdx.y * BT;
    const int ksteps = (w.units + 1) / 2;
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *A = base;                                  // [STAGES][128 x 128 B]
    uint8_t *Bm = base + STAGES * A_BYTES;              // [STAGES][BT x 128 B]

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(smem_u32(&full_bar[s]), 256);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        mbar_init(smem_u32(&acc_bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 8) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                     "r"(BT));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    pdl_wait();
    pdl_trigger();

    if (warp < 4) {
        // ---- A producers: weight rows
        const int r = threadIdx.x;
        const int64_t row = n0 + r;
        const bool rok = row < N;
        for (int ks = 0; ks < ksteps; ks++) {
            const int s = ks % STAGES, round = ks / STAGES;
            float v0[32], v1[32];
            unit_values<TYPE>(w, row, 2 * ks, rok, v0);
            unit_values<TYPE>(w, row, 2 * ks + 1, rok && (2 * ks + 1 < w.units), v1);
            if (!mbar_wait(smem_u32(&empty_bar[s]), (round & 1) ^ 1, flag)) break;
            uint8_t *tile = A + s * A_BYTES;
            store_sw128(tile, r, 0, v0);
            store_sw128(tile, r, 4, v1);
            fence_async_smem();
            mbar_arrive(smem_u32(&full_bar[s]));
        }
    } else if (warp < 8) {
        // ---- B producers: fp32 activations -> bf16
        const int tid = threadIdx.x - 128;
        for (int ks = 0; ks < ksteps; ks++) {
            const int s = ks % STAGES, round = ks / STAGES;
            if (!mbar_wait(smem_u32(&empty_bar[s]), (round & 1) ^ 1, flag)) break;
            uint8_t *tile = Bm + s * B_BYTES;
            for (int c = tid; c < BT * 8; c += 128) {
                const int rr = c >> 3, ch = c & 7;
                const int t = t0 + rr, k = ks * BK + ch * 8;
                float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
                if (t < T && k < K) {
                    const float4 *p = (const float4 *)(X + (int64_t)t * K + k);
                    a = __ldg(p);
                    b = __ldg(p + 1);
                }
                uint4 q;
                q.x = pack_bf16(a.x, a.y);
                q.y = pack_bf16(a.z, a.w);
                q.z = pack_bf16(b.x, b.y);
                q.w = pack_bf16(b.z, b.w);
                *(uint4 *)(tile + rr * 128 + ((ch ^ (rr & 7)) * 16)) = q;
            }
            fence_async_smem();
            mbar_arrive(smem_u32(&full_bar[s]));
        }
    } else {
        // ---- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(BT);
            for (int ks = 0; ks < ksteps; ks++) {
                const int s = ks % STAGES, round = ks / STAGES;
                if (!mbar_wait(smem_u32(&full_bar[s]), round & 1, flag)) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(A + s * A_BYTES), b0 = smem_u32(Bm + s * B_BYTES);
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++) {
                    uint64_t ad = sw128_desc(a0 + kk * 32), bd = sw128_desc(b0 + kk * 32);
                    uint32_t acc = (ks > 0 || kk > 0) ? 1u : 0u;
                    asm volatile(
                        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
                        "l"(ad), "l"(bd), "r"(idesc), "r"(acc));
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_u32(&empty_bar[s]))
                             : "memory");
            }
            // Always signal the accumulator: its completion implies every MMA
            // issued above has finished (also on a timeout path).
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&acc_bar))
                         : "memory");
        }
        __syncwarp();
    }

    // ---- epilogue: warps 0-7
    if (warp < 8) {
        const bool ok = mbar_wait(smem_u32(&acc_bar), 0, flag);
        tc_fence_after();
        const int q = warp & 3, half = warp >> 2;
        const int64_t n = n0 + 32 * q + lane;
        for (int c0 = half * (BT / 2); c0 < (half + 1) * (BT / 2); c0 += 16) {
            uint32_t r[16];
            const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0;
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                "[%16];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                  "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                  "=r"(r[15])
                : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (ok && n < N) {
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int t = t0 + c0 + j;
                    if (t < T) Y[(int64_t)t * N + n] = __uint_as_float(r[j]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BT));
    }
}

template <int TYPE, int BT>
cudaError_t launch_tc(hd_ctx *ctx, const hd_weight *w, const float *X, float *Y, int T) {
    constexpr size_t smem = (size_t)STAGES * (A_BYTES + BT * BK * 2) + 1024;
    cudaError_t e = cudaFuncSetAttribute(k_qgemm_tc<TYPE, BT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)((w->rows + 127) / 128), (unsigned)((T + BT - 1) / BT));
    return hd_launch(ctx, k_qgemm_tc<TYPE, BT>, grid, dim3(288), smem, wview(w), X, Y, T, (int)w->rows,
                     (int)w->cols, ctx->flag);
}


// ------------------------------------------------------------------- v3
// Persistent and streamed.  Each SM runs one CTA that walks work items
// (128 weight rows x BT tokens, optionally one of two K halves) with three
// concurrent pipelines:
//   weights: the dequantizer threads copy their own raw quant bytes from
//     global memory with coalesced cp.async, PD K-steps ahead of use, into
//     per-thread shared slots, convert them to bf16 and store them with
//     tcgen05.st into one of AS weight stages in tensor memory;
//   activations: the bf16 tile of each K-step arrives by one TMA copy
//     (SWIZZLE_128B K-major) into the X ring (XS stages); NXW copy warps take
//     the steps in turn;
//   MMA: one thread issues 4 tcgen05.mma (K = 16, A from tensor memory, B
//     from shared memory) per step into one of two TMEM accumulators and
//     releases weight and X stages by tcgen05.commit.
// Why this shape.  (1) Shared-memory bandwidth (~128 B per cycle per SM) is
// the scarce resource: the MMA alone reads its shared operands at ~96 B per
// cycle at full rate, so bf16 weights written to and read from shared memory
// (32 KB per 64-deep step) and an epilogue transposed through it held a
// 64-deep step near 1000 cycles against 512 of MMA.  Weights in tensor memory
// and an epilogue straight from registers leave the activations as the only
// large shared-memory stream.  (2) The bulk-copy (TMA) operations that one
// warp issues are processed one after another at ~500-700 cycles each
// whatever their size, while those of different warps overlap; hence one
// whole activation tile per operation and several copy warps.
// Tensor memory (512 columns) holds two BT-column accumulators and the
// weight stages, so BT is at most 208 (2 x 208 + 3 x 32 = 512).
// Warps: 0-15 dequantize (thread = weight row x unit of the step x value
// half), 16-18 activation copies, 19 TMEM + MMA, 20-23 epilogue.  Requires rows % 128 == 0;
// other shapes use the v1 kernel above.

__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap *tm, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"((uint64_t)tm), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Raw words of one unit of one row (decoded into bf16 by dq_store).
struct DqRaw {
    uint4 q0, q1;  // packed quants (q1: bytes 16-31, Q8_0 only)
    uint4 m;       // Q4_K: d, dmin, 12 scale bytes; Q6_K: 16 int8 sub-scales
    uint2 hb;      // Q6_K high bit pairs
    uint32_t qh;   // Q5_0 fifth bits
    uint32_t d;    // Q8_0 / Q5_0 block scale, Q6_K super-block scale (fp16 bits in the low half)
};

// Per-thread raw slots of the dequantizers, structure of arrays over the 256
// threads of the role: region Q (16 B each), M (16 B: Q8_0 quant bytes 16-31,
// Q4_K/Q6_K scales), HB (8 B, Q6_K high bits), W0 (4 B: Q5_0 fifth bits) and
// W1 (4 B: the aligned 32-bit word holding the fp16 scale).
template <int TYPE>
struct RawSlot {
    static constexpr int Q = 0, M = 16 * 256;
    static constexpr bool HAS_M = TYPE != HD_TYPE_Q5_0;
    static constexpr int HB = M + (HAS_M ? 16 * 256 : 0);
    static constexpr bool HAS_HB = TYPE == HD_TYPE_Q6_K;
    static constexpr int W0 = HB + (HAS_HB ? 8 * 256 : 0);
    static constexpr bool HAS_W0 = TYPE == HD_TYPE_Q5_0;
    static constexpr int W1 = W0 + (HAS_W0 ? 4 * 256 : 0);
    static constexpr bool HAS_W1 = TYPE != HD_TYPE_Q4_K;
    static constexpr int BYTES = W1 + (HAS_W1 ? 4 * 256 : 0);
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Starts the asynchronous copies of the raw bytes of unit u of weight row
// `row` into entry e of a raw slot (global -> shared, no registers held).
// The two threads of an entry share the work: part 0 copies the 16 quant
// bytes (Q8_0: bytes 0-15), part 1 the rest (Q8_0: bytes 16-31 and scale).
template <int TYPE>
__device__ __forceinline__ void dq_fetch(const WView &w, int64_t row, int u, uint8_t *slot, int e, int part) {
    using RS = RawSlot<TYPE>;
    const int64_t ur = (int64_t)u * w.rows + row;
    const uint32_t sb = smem_u32(slot);
    if (part == 0) {
        cp_async16(sb + RS::Q + 16 * e, w.q + ur * (TYPE == HD_TYPE_Q8_0 ? 32 : 16));
        return;
    }
    if constexpr (TYPE == HD_TYPE_Q8_0) {
        cp_async16(sb + RS::M + 16 * e, w.q + ur * 32 + 16);
        cp_async4(sb + RS::W1 + 4 * e, (const unsigned short *)w.meta + (ur & ~(int64_t)1));
    } else if constexpr (TYPE == HD_TYPE_Q5_0) {
        cp_async4(sb + RS::W0 + 4 * e, (const unsigned int *)w.aux + ur);
        cp_async4(sb + RS::W1 + 4 * e, (const unsigned short *)w.meta + (ur & ~(int64_t)1));
    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
        cp_async16(sb + RS::M + 16 * e, w.meta + ((int64_t)(u >> 3) * w.rows + row) * 16);
    } else {
        const int64_t sr = (int64_t)(u >> 3) * w.rows + row;
        cp_async8(sb + RS::HB + 8 * e, (const uint2 *)w.aux + ur);
        cp_async16(sb + RS::M + 16 * e, w.meta + sr * 16);
        cp_async4(sb + RS::W1 + 4 * e, w.dsb + (sr & ~(int64_t)1));
    }
}

// Reads back what value half `part` of entry e needs; `odd` selects the fp16
// half of the 32-bit scale word (the parity of the element's index).
template <int TYPE>
__device__ __forceinline__ void dq_read(const uint8_t *slot, int e, int part, bool odd, DqRaw &g) {
    using RS = RawSlot<TYPE>;
    g.q0 = *(const uint4 *)(slot + ((TYPE == HD_TYPE_Q8_0 && part) ? RS::M : RS::Q) + 16 * e);
    if constexpr (TYPE == HD_TYPE_Q4_K || TYPE == HD_TYPE_Q6_K) g.m = *(const uint4 *)(slot + RS::M + 16 * e);
    if constexpr (RS::HAS_HB) g.hb = *(const uint2 *)(slot + RS::HB + 8 * e);
    if constexpr (RS::HAS_W0) g.qh = *(const uint32_t *)(slot + RS::W0 + 4 * e);
    if constexpr (RS::HAS_W1) g.d = (*(const uint32_t *)(slot + RS::W1 + 4 * e)) >> (odd ? 16 : 0);
}

// bf16x2 pairs straight from quant bytes (Q5_0, Q4_K, Q6_K: q < 128).  One
// byte_perm places two bytes under the bf16 exponent byte 0x43, giving the
// exact values 128 + q; one __hsub2 removes 128 + offset exactly; the scale is
// applied in bf16 (for the bf16 tensor-core path only).
__device__ __forceinline__ __nv_bfloat162 pair_bf16(uint32_t v, uint32_t sel) {
    uint32_t b = __byte_perm(v, 0x43434343u, sel);
    return *reinterpret_cast<__nv_bfloat162 *>(&b);
}
__device__ __forceinline__ uint32_t bits2(__nv_bfloat162 x) { return *reinterpret_cast<uint32_t *>(&x); }

// Values 16*part .. 16*part+15 of unit u (zeros when !valid) as 8 packed
// bf16 pairs, word j = values (16*part + 2j, +1), the lower K index in the
// low half.  For Q8_0, g.q0 holds the 16 quant bytes of that half.
template <int TYPE>
__device__ __forceinline__ void dq_words(int u, int part, bool valid, const DqRaw &g, uint32_t (&o)[8]) {
    if (!valid) {
#pragma unroll
        for (int j = 0; j < 8; j++) o[j] = 0u;
    } else if constexpr (TYPE == HD_TYPE_Q8_0) {
        const float d = h2f((uint16_t)g.d);
        const uint32_t wd[4] = {g.q0.x, g.q0.y, g.q0.z, g.q0.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t x = wd[i] ^ 0x80808080u;
            o[2 * i] = pack_bf16((mag(x, 0) - 8388736.0f) * d, (mag(x, 1) - 8388736.0f) * d);
            o[2 * i + 1] = pack_bf16((mag(x, 2) - 8388736.0f) * d, (mag(x, 3) - 8388736.0f) * d);
        }
    } else {
        float sc, mn = 0.f;
        if constexpr (TYPE == HD_TYPE_Q5_0) {
            sc = h2f((uint16_t)g.d);
        } else if constexpr (TYPE == HD_TYPE_Q4_K) {
            int s6, m6;
            q4k_sm_regs(u & 7, g.m.y, g.m.z, g.m.w, s6, m6);
            sc = h2f((uint16_t)(g.m.x & 0xFFFF)) * (float)s6;
            mn = -h2f((uint16_t)(g.m.x >> 16)) * (float)m6;
        } else {
            // sub-scale 2(u&7) + part: byte 2(u&1) + part of word (u&7)/2
            const uint32_t sw = (u & 4) ? ((u & 2) ? g.m.w : g.m.z) : ((u & 2) ? g.m.y : g.m.x);
            sc = h2f((uint16_t)g.d) * (float)(int8_t)((sw >> (8 * (2 * (u & 1) + part))) & 0xFF);
        }
        const uint32_t wd[4] = {g.q0.x, g.q0.y, g.q0.z, g.q0.w};
        const __nv_bfloat162 off =
            __float2bfloat162_rn(TYPE == HD_TYPE_Q5_0 ? 144.f : TYPE == HD_TYPE_Q4_K ? 128.f : 160.f);
        const __nv_bfloat162 mlo = __float2bfloat162_rn(mn), s2 = __float2bfloat162_rn(sc);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t b;
            if constexpr (TYPE == HD_TYPE_Q5_0) {
                b = part ? (((wd[i] >> 4) & 0x0F0F0F0Fu) | ((g.qh << (4 - i)) & 0x10101010u))
                         : ((wd[i] & 0x0F0F0F0Fu) | ((g.qh >> i) & 0x10101010u));
            } else if constexpr (TYPE == HD_TYPE_Q4_K) {
                b = (wd[i] >> (4 * part)) & 0x0F0F0F0Fu;
            } else {
                const int sh = 4 - 2 * i;
                const uint32_t hsel = part ? g.hb.y : g.hb.x;
                const uint32_t hx = sh >= 0 ? (hsel << sh) : (hsel >> -sh);
                b = ((wd[i] >> (4 * part)) & 0x0F0F0F0Fu) | (hx & 0x30303030u);
            }
            o[2 * i] = bits2(__hfma2(__hsub2(pair_bf16(b, 0x5140u), off), s2, mlo));
            o[2 * i + 1] = bits2(__hfma2(__hsub2(pair_bf16(b, 0x7362u), off), s2, mlo));
        }
    }
}

// Stores 8 words per thread into 8 consecutive TMEM columns of the thread's
// lane (warp w reaches lanes 32*(w%4)..), and waits for the store.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&o)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(o[0]),
                 "r"(o[1]), "r"(o[2]), "r"(o[3]), "r"(o[4]), "r"(o[5]), "r"(o[6]), "r"(o[7])
                 : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Exact-product mode: values 16*part .. 16*part+15 of unit u as exact fp32
// (the fp32 path's dequantization), times 2^shift (exact), split into fp16
// halves: v = hi + lo + r with |r| <= 2^-22 |v| (zeros when !valid).
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}
template <int TYPE>
__device__ __forceinline__ void dq_words_exact(int u, int part, bool valid, const DqRaw &g, float scale,
                                               uint32_t (&hi)[8], uint32_t (&lo)[8]) {
    if (!valid) {
#pragma unroll
        for (int j = 0; j < 8; j++) hi[j] = lo[j] = 0u;
        return;
    }
    float v[16];
    const uint32_t wd[4] = {g.q0.x, g.q0.y, g.q0.z, g.q0.w};
    if constexpr (TYPE == HD_TYPE_Q8_0) {
        const float d = h2f((uint16_t)g.d);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t x = wd[i] ^ 0x80808080u;
#pragma unroll
            for (int c = 0; c < 4; c++) v[4 * i + c] = __fmul_rn(mag(x, c) - 8388736.0f, d);
        }
    } else if constexpr (TYPE == HD_TYPE_Q5_0) {
        const float d = h2f((uint16_t)g.d);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t b = part ? (((wd[i] >> 4) & 0x0F0F0F0Fu) | ((g.qh << (4 - i)) & 0x10101010u))
                                    : ((wd[i] & 0x0F0F0F0Fu) | ((g.qh >> i) & 0x10101010u));
#pragma unroll
            for (int c = 0; c < 4; c++) v[4 * i + c] = __fmul_rn(mag(b, c) - 8388624.0f, d);
        }
    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
        int s6, m6;
        q4k_sm_regs(u & 7, g.m.y, g.m.z, g.m.w, s6, m6);
        const float d1 = __fmul_rn(h2f((uint16_t)(g.m.x & 0xFFFF)), (float)s6);
        const float m1 = __fmul_rn(h2f((uint16_t)(g.m.x >> 16)), (float)m6);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t b = (wd[i] >> (4 * part)) & 0x0F0F0F0Fu;
#pragma unroll
            for (int c = 0; c < 4; c++) v[4 * i + c] = __fsub_rn(__fmul_rn(mag(b, c) - 8388608.0f, d1), m1);
        }
    } else {
        const uint32_t sw = (u & 4) ? ((u & 2) ? g.m.w : g.m.z) : ((u & 2) ? g.m.y : g.m.x);
        const float dd =
            __fmul_rn(h2f((uint16_t)g.d), (float)(int8_t)((sw >> (8 * (2 * (u & 1) + part))) & 0xFF));
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int sh = 4 - 2 * i;
            const uint32_t hsel = part ? g.hb.y : g.hb.x;
            const uint32_t hx = sh >= 0 ? (hsel << sh) : (hsel >> -sh);
            const uint32_t b = ((wd[i] >> (4 * part)) & 0x0F0F0F0Fu) | (hx & 0x30303030u);
#pragma unroll
            for (int c = 0; c < 4; c++) v[4 * i + c] = __fmul_rn(mag(b, c) - 8388640.0f, dd);
        }
    }
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float a = v[2 * j] * scale, b = v[2 * j + 1] * scale;
        const __half2 h = __floats2half2_rn(a, b);
        hi[j] = *reinterpret_cast<const uint32_t *>(&h);
        lo[j] = pack_h2(a - __low2float(h), b - __high2float(h));
    }
}

constexpr int DQ_WARPS = 16, DQ_THREADS = DQ_WARPS * 32;
constexpr int NXW = 3;                                  // activation copy warps
constexpr int W_X = DQ_WARPS, W_MMA = W_X + NXW, W_EPI = W_MMA + 1;
constexpr int TC3_THREADS = (W_EPI + 4) * 32;

// Shared memory: XS activation stages (EX: an fp16 hi and an fp16 lo tile
// each) and PD raw slots for the dequantizers (the weight bytes of PD
// K-steps in flight).  Tensor memory (512 columns): two fp32 accumulators of
// BT columns, then AS weight stages of 32 columns (128 rows x 64 K values,
// two per column; EX: 64 columns, hi then lo) that the MMA reads as A.
template <int TYPE, int BT, int EX>
struct TC3 {
    static constexpr int XB = BT * BK * 2;
    static constexpr int XT = EX ? 2 : 1;
    static constexpr int RB = RawSlot<TYPE>::BYTES;
    static constexpr int ASC = EX ? 64 : 32;
    static constexpr int AS = (512 - 2 * BT) / ASC > 4 ? 4 : (512 - 2 * BT) / ASC;
    static constexpr int A_COL = 2 * BT;
    static_assert(AS >= 2, "tensor memory plan");
    static constexpr int XS = EX ? (BT >= 128 ? 4 : 6) : (BT >= 192 ? 6 : 8);
    static constexpr int R_OFF = XS * XT * XB;
    static constexpr int FREE = 227 * 1024 - 1024 - 512 - R_OFF;
    static constexpr int PD = FREE / RB > 6 ? 6 : FREE / RB;
    static_assert(PD >= 2, "shared memory plan");
    static constexpr size_t SMEM = (size_t)R_OFF + PD * RB + 1024;
};

// The (item, K-step) sequence of this CTA: items blockIdx.x, +gridDim.x, ...;
// item = tile + ntiles * (K part); steps k0..k1-1 of its K part.  row0 is
// the first weight row of the item's tile (divisions once per item).
struct StepCursor {
    int item, ks, k1, row0;
    __device__ __forceinline__ void range(int ntiles, int ntm, int kper, int ksteps) {
        ks = (item / ntiles) * kper;
        k1 = min(ksteps, ks + kper);
        row0 = ((item % ntiles) % ntm) * 128;
    }
    __device__ __forceinline__ void start(int nitems, int ntiles, int ntm, int kper, int ksteps) {
        item = blockIdx.x;
        if (item < nitems) range(ntiles, ntm, kper, ksteps);
    }
    __device__ __forceinline__ void next(int nitems, int ntiles, int ntm, int kper, int ksteps) {
        if (++ks < k1) return;
        item += gridDim.x;
        if (item < nitems) range(ntiles, ntm, kper, ksteps);
    }
};

// Persistent: an item is a tile (row tile fastest, so CTAs running at the
// same time share an activation tile in L2) and, when the tiles alone would
// leave SMs idle, one of two K halves (KS = 2: both halves add into Y, zeroed
// beforehand; two addends onto zero commute, so the sum is order-independent).
template <int TYPE, int BT, int EX>
__global__ void __launch_bounds__(TC3_THREADS, 1)
    k_qgemm_tc3(WView w, const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmx_lo,
                float *__restrict__ Y, int T, int N, int ntm, int ntiles, int KS, int wshift,
                const int *__restrict__ rowshift, int *flag) {
    using C = TC3<TYPE, BT, EX>;
    constexpr int XS = C::XS, AS = C::AS, PD = C::PD;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t x_full[XS], x_empty[XS], a_full[AS], a_empty[AS];
    __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], fin_bar;
    __shared__ uint32_t tmem_base_sh;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = w.units, ksteps = (units + 1) / 2;
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);

    if (threadIdx.x == 0) {
        for (int s = 0; s < XS; s++) {
            mbar_init(smem_u32(&x_full[s]), 1);
            mbar_init(smem_u32(&x_empty[s]), 1);
        }
        for (int s = 0; s < AS; s++) {
            mbar_init(smem_u32(&a_full[s]), DQ_THREADS);
            mbar_init(smem_u32(&a_empty[s]), 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(smem_u32(&acc_full[i]), 1);
            mbar_init(smem_u32(&acc_empty[i]), 128);
        }
        mbar_init(smem_u32(&fin_bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmx) : "memory");
        if (EX) asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmx_lo) : "memory");
    }
    if (warp == W_MMA) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    pdl_wait();
    pdl_trigger();

    const int kper = (ksteps + KS - 1) / KS, nitems = ntiles * KS;
    if (warp < DQ_WARPS) {
        // ---- dequantizers: thread (weight row r, unit h of the step, value
        // half part).  The two threads of a (row, unit) entry copy its raw
        // bytes (cp.async) into a raw slot PD - 1 steps ahead; a named barrier
        // over the role makes every copy of step g visible before any thread
        // reads it, and also tells that every thread is done with step g - 1,
        // whose slot is then refilled.
        const int e = threadIdx.x & 255, r = e & 127, h = e >> 7, part = threadIdx.x >> 8;
        uint8_t *slots = base + C::R_OFF;
        const float wscale = __int_as_float((127 + wshift) << 23);  // 2^wshift, |wshift| <= 60
        StepCursor cl, cc;  // fetch cursor PD - 1 steps ahead of the compute cursor
        bool alive = true;
        cl.start(nitems, ntiles, ntm, kper, ksteps);
        cc = cl;
        for (int j = 0; j < PD - 1; j++) {
            if (cl.item < nitems) {
                const int u = 2 * cl.ks + h;
                if (u < units) dq_fetch<TYPE>(w, (int64_t)(cl.row0 + r), u, slots + j * C::RB, e, part);
                cl.next(nitems, ntiles, ntm, kper, ksteps);
            }
            cp_async_commit();
        }
        for (int g = 0; cc.item < nitems; g++) {
            const int as = g % AS;
            cp_async_wait<PD - 2>();   // this thread's copies of step g have landed
            asm volatile("bar.sync 1, %0;" ::"n"(DQ_THREADS) : "memory");
            if (cl.item < nitems) {
                const int ul = 2 * cl.ks + h;
                if (ul < units)
                    dq_fetch<TYPE>(w, (int64_t)(cl.row0 + r), ul, slots + ((g + PD - 1) % PD) * C::RB, e, part);
                cl.next(nitems, ntiles, ntm, kper, ksteps);
            }
            cp_async_commit();
            const int u = 2 * cc.ks + h;
            DqRaw rg;
            if (u < units) dq_read<TYPE>(slots + (g % PD) * C::RB, e, part, r & 1, rg);
            uint32_t o[8], ol[8];
            if constexpr (EX) dq_words_exact<TYPE>(u, part, u < units, rg, wscale, o, ol);
            else dq_words<TYPE>(u, part, u < units, rg, o);
            // After a failed wait the thread stops storing but keeps its place
            // in the loop, so that every thread takes the named barrier
            // equally often.
            alive = alive && mbar_wait(smem_u32(&a_empty[as]), ((g / AS) & 1) ^ 1, flag);
            if (alive) {
                tc_fence_after();
                const uint32_t ta = tmem + ((uint32_t)(32 * (warp & 3)) << 16) +
                                    (uint32_t)(C::A_COL + C::ASC * as + 16 * h + 8 * part);
                tmem_st8(ta, o);
                if constexpr (EX) tmem_st8(ta + 32, ol);
                tc_fence_before();
            }
            mbar_arrive(smem_u32(&a_full[as]));
            cc.next(nitems, ntiles, ntm, kper, ksteps);
        }
        cp_async_wait<0>();
    } else if (warp < W_MMA) {
        // ---- activation copies: warp j issues the steps g with g % NXW == j
        if (lane == 0) {
            const int j = warp - W_X;
            int g = 0, last[XS];
            for (int s = 0; s < XS; s++) last[s] = -1;
            bool alive = true;
            for (int item = blockIdx.x; item < nitems && alive; item += gridDim.x) {
                const int t0 = ((item % ntiles) / ntm) * BT;
                const int k0 = (item / ntiles) * kper, k1 = min(ksteps, k0 + kper);
                for (int ks = k0; ks < k1; ks++, g++) {
                    if (g % NXW != j) continue;
                    const int s = g % XS;
                    if (!mbar_wait(smem_u32(&x_empty[s]), ((g / XS) & 1) ^ 1, flag, 64)) { alive = false; break; }
                    const uint32_t bar = smem_u32(&x_full[s]);
                    mbar_expect_tx(bar, C::XT * C::XB);
                    tma_2d(smem_u32(base + s * C::XT * C::XB), &tmx, ks * BK, t0, bar);
                    if (EX) tma_2d(smem_u32(base + (s * C::XT + 1) * C::XB), &tmx_lo, ks * BK, t0, bar);
                    last[s] = g;
                }
            }
            // On an early exit, this warp's copies still in flight land before
            // the CTA does (on a normal exit the MMA has consumed them all).
            if (!alive)
                for (int s = 0; s < XS; s++)
                    if (last[s] >= 0) mbar_wait_quiet(smem_u32(&x_full[s]), (last[s] / XS) & 1);
        }
        __syncwarp();
    } else if (warp == W_MMA) {
        // ---- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = EX ? idesc_f16(BT) : idesc_bf16(BT);
            int g = 0, li = 0;
            bool alive = true;
            for (int item = blockIdx.x; item < nitems && alive; item += gridDim.x, li++) {
                const int buf = li & 1;
                const int k0 = (item / ntiles) * kper, k1 = min(ksteps, k0 + kper);
                if (!mbar_wait(smem_u32(&acc_empty[buf]), ((li >> 1) & 1) ^ 1, flag)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * BT);
                for (int ks = k0; ks < k1; ks++, g++) {
                    const int xs = g % XS, as = g % AS;
                    if (!mbar_wait(smem_u32(&x_full[xs]), (g / XS) & 1, flag) ||
                        !mbar_wait(smem_u32(&a_full[as]), (g / AS) & 1, flag)) {
                        alive = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = tmem + (uint32_t)(C::A_COL + C::ASC * as);
                    const uint32_t b0 = smem_u32(base + xs * C::XT * C::XB);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++) {
                        const uint64_t bd = sw128_desc(b0 + kk * 32);
                        const uint32_t acc = (ks > k0 || kk > 0) ? 1u : 0u;
                        asm volatile(
                            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                            " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
                            "r"(a0 + 8 * kk), "l"(bd), "r"(idesc), "r"(acc));
                        if constexpr (EX) {
                            // + w_hi x_lo + w_lo x_hi (w_lo x_lo is below 2^-22)
                            const uint64_t bdl = sw128_desc(b0 + C::XB + kk * 32);
                            asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, 1;" ::"r"(d),
                                         "r"(a0 + 8 * kk), "l"(bdl), "r"(idesc));
                            asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, 1;" ::"r"(d),
                                         "r"(a0 + 32 + 8 * kk), "l"(bd), "r"(idesc));
                        }
                    }
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                     smem_u32(&x_empty[xs]))
                                 : "memory");
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                     smem_u32(&a_empty[as]))
                                 : "memory");
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_u32(&acc_full[buf]))
                             : "memory");
            }
            // Completion of this commit covers every MMA issued above; it is
            // awaited also after a timeout, before TMEM is freed.
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&fin_bar))
                         : "memory");
            mbar_wait_quiet(smem_u32(&fin_bar), 0);
        }
        __syncwarp();
    } else {
        // ---- epilogue: warp quarter q reads TMEM lanes 32q.. (weight rows),
        // 16 token columns at a time; each store instruction writes 32
        // consecutive weight rows of one token (128 contiguous bytes of Y).
        const int q = warp & 3;
        int li = 0;
        for (int item = blockIdx.x; item < nitems; item += gridDim.x, li++) {
            const int buf = li & 1, tile = item % ntiles;
            const int64_t n = (int64_t)(tile % ntm) * 128 + 32 * q + lane;
            const int t0 = (tile / ntm) * BT;
            const bool ok = mbar_wait(smem_u32(&acc_full[buf]), (li >> 1) & 1, flag, 128);
            tc_fence_after();
            for (int c0 = 0; ok && c0 < BT && t0 + c0 < T; c0 += 16) {
                uint32_t rr[16];
                const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * BT + c0);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                    "[%16];"
                    : "=r"(rr[0]), "=r"(rr[1]), "=r"(rr[2]), "=r"(rr[3]), "=r"(rr[4]), "=r"(rr[5]), "=r"(rr[6]),
                      "=r"(rr[7]), "=r"(rr[8]), "=r"(rr[9]), "=r"(rr[10]), "=r"(rr[11]), "=r"(rr[12]), "=r"(rr[13]),
                      "=r"(rr[14]), "=r"(rr[15])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int t = t0 + c0 + j;
                    if (t < T) {
                        float v = __uint_as_float(rr[j]);
                        // EX: undo 2^(wshift + rowshift[t]) (exact power of two)
                        if (EX) v *= __int_as_float((127 - wshift - __ldg(rowshift + t)) << 23);
                        float *dst = Y + (int64_t)t * N + n;
                        if (KS == 1) *dst = v;
                        else atomicAdd(dst, v);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&acc_empty[buf]));
            if (!ok) break;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// Exact-product mode: row t of x times 2^rowshift[t] (largest magnitude near
// 2^14), split into fp16 halves hi + lo (|x - hi - lo| <= 2^-22 |x|), by the
// whole CTA; K % 8 == 0.
__device__ __forceinline__ void f16_split_row(const float *__restrict__ x, int K, __half *__restrict__ hi,
                                              __half *__restrict__ lo, int *__restrict__ rowshift, int64_t t,
                                              float *red) {
    const float4 *xr = (const float4 *)(x + t * K);
    float m = 0.f;
    for (int k = threadIdx.x; k < K / 4; k += blockDim.x) {
        const float4 v = xr[k];
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) m = fmaxf(m, red[i]);
    int sh = 0;
    if (m > 0.f && m < INFINITY) {
        int ex;
        frexpf(16384.f / m, &ex);
        sh = ex - 1;
        sh = sh < -60 ? -60 : sh > 60 ? 60 : sh;
    }
    const float sc = __int_as_float((127 + sh) << 23);
    for (int k = threadIdx.x; k < K / 4; k += blockDim.x) {
        const float4 v = xr[k];
        const float a0 = v.x * sc, a1 = v.y * sc, a2 = v.z * sc, a3 = v.w * sc;
        const __half2 h01 = __floats2half2_rn(a0, a1), h23 = __floats2half2_rn(a2, a3);
        const __half2 l01 = __floats2half2_rn(a0 - __low2float(h01), a1 - __high2float(h01));
        const __half2 l23 = __floats2half2_rn(a2 - __low2float(h23), a3 - __high2float(h23));
        __half2 *ph = (__half2 *)(hi + t * K) + 2 * k, *pl = (__half2 *)(lo + t * K) + 2 * k;
        ph[0] = h01;
        ph[1] = h23;
        pl[0] = l01;
        pl[1] = l23;
    }
    if (threadIdx.x == 0) rowshift[t] = sh;
}

// One CTA per row.
__global__ void k_to_f16_split(const float *__restrict__ x, int K, __half *__restrict__ hi, __half *__restrict__ lo,
                               int *__restrict__ rowshift) {
    __shared__ float red[32];
    pdl_wait();
    pdl_trigger();
    f16_split_row(x, K, hi, lo, rowshift, blockIdx.x, red);
}

__global__ void k_to_bf16(const float *__restrict__ x, __nv_bfloat16 *__restrict__ y, int64_t n) {
    pdl_wait();
    pdl_trigger();
    int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i + 3 < n) {
        float4 v = *(const float4 *)(x + i);
        __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
        *(__nv_bfloat162 *)(y + i) = a;
        *(__nv_bfloat162 *)(y + i + 2) = b;
    } else {
        for (; i < n; i++) y[i] = __float2bfloat16_rn(x[i]);
    }
}

// cuTensorMapEncodeTiled, looked up through the runtime so the library does
// not link the driver library (it still loads on machines without a GPU).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

// ------------------------------------------------------------------- v4
// Two passes, for prompts long enough that one dequantization of the weight
// is cheap next to the products (the weight is re-read by every token tile):
//   k_prep writes the weight once as 16-bit rows [N][K] (bf16, or in the
//     exact-product mode fp16 hi and lo planes of 2^wshift * w), into a
//     workspace that stays in L2 for the layer sizes of a 0.5B-7B model, and
//     in the same launch converts the activations as for v3;
//   k_gemm_tc4 is then a persistent tcgen05 GEMM whose operands both arrive by
//     TMA (SWIZZLE_128B K-major) into a ring of STG stages of 128 weight rows
//     and BT tokens x 64 K values each.
// Without dequantizer warps on the critical path a K-step costs what its
// shared-memory traffic costs (each stage is written once by TMA and read
// once by the MMA), against 2*BT cycles of MMA.  BT (a multiple of 16, at most
// 256) is a runtime argument, chosen by the host against wave quantization.
// Warps: 0-3 TMA producers (warp j issues the steps g with g % 4 == j, since
// one warp's bulk copies are processed one after another; with fewer than 4
// stages, as many warps as stages), 4 TMEM + MMA,
// 5-8 epilogue (as in v3: straight from TMEM registers to Y, 128 contiguous
// bytes per store instruction).  Any row count: rows past N arrive as zeros
// from the TMA and are not stored.

// Both operand preparations in one launch (256 threads per CTA).  CTAs
// [0, nw) dequantize blocks of 32 weight rows x 8 units: thread (row r, unit
// u) makes one coalesced load of its unit from the unit-major layout (a warp
// reads 32 consecutive rows), decodes 32 values and stages the 16-bit values
// in shared memory, after which every warp store writes 512 contiguous bytes
// of one row.  The exact mode stores fp16 hi and lo planes of 2^wshift * w
// from the exact (oracle-order) dequantization.  The remaining CTAs convert
// the activations: bf16, 8 values per thread; exact mode, one CTA per row
// (f16_split_row).
constexpr int PREP_RS = 32 * 16 + 16;  // staged row stride in bytes (conflict-free)

constexpr int PREP_XV = 4;   // bf16 mode: groups of 8 activations per thread, at most
// From this many groups on, one group per thread (more blocks in flight);
// below, PREP_XV (fewer blocks to launch).  Measured on B200, prep + GEMM:
// Q5_0 4864 x 896 T = 128 / 512 +9 % / +4 % with 4, T = 2048 +2 % with 1.
constexpr int64_t PREP_XV_BIG = 131072;
template <int TYPE, int EX>
__global__ void __launch_bounds__(256) k_prep(WView w, uint16_t *__restrict__ whi, uint16_t *__restrict__ wlo,
                                              int wshift, int nrb, int nw, const float *__restrict__ X, int T,
                                              uint16_t *__restrict__ xhi, uint16_t *__restrict__ xlo,
                                              int *__restrict__ rowshift) {
    __shared__ __align__(16) uint8_t tile[EX ? 2 : 1][32 * PREP_RS];
    __shared__ float red[32];
    pdl_wait();
    pdl_trigger();
    const int64_t K = (int64_t)w.units * 32;
    if ((int)blockIdx.x < nw) {
        const int rb = blockIdx.x % nrb, ub = blockIdx.x / nrb;
        const int r = threadIdx.x & 31, wp = threadIdx.x >> 5;
        const int64_t row = (int64_t)rb * 32 + r;
        const int u = ub * 8 + wp;
        if (row < w.rows && u < w.units) {
            float v[32];
            if constexpr (EX) decode_unit_exact<TYPE>(w, row, u, v);
            else unit_values<TYPE>(w, row, u, true, v);
            uint8_t *dh = tile[0] + r * PREP_RS + wp * 64;
            if constexpr (EX) {
                uint8_t *dl = tile[EX ? 1 : 0] + r * PREP_RS + wp * 64;
                const float sc = __int_as_float((127 + wshift) << 23);  // 2^wshift, |wshift| <= 60
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    uint32_t h[4], l[4];
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const float a = v[8 * c + 2 * j] * sc, b = v[8 * c + 2 * j + 1] * sc;
                        const __half2 hh = __floats2half2_rn(a, b);
                        const __half2 ll = __floats2half2_rn(a - __low2float(hh), b - __high2float(hh));
                        h[j] = *reinterpret_cast<const uint32_t *>(&hh);
                        l[j] = *reinterpret_cast<const uint32_t *>(&ll);
                    }
                    *(uint4 *)(dh + 16 * c) = make_uint4(h[0], h[1], h[2], h[3]);
                    *(uint4 *)(dl + 16 * c) = make_uint4(l[0], l[1], l[2], l[3]);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 4; c++)
                    *(uint4 *)(dh + 16 * c) =
                        make_uint4(pack_bf16(v[8 * c], v[8 * c + 1]), pack_bf16(v[8 * c + 2], v[8 * c + 3]),
                                   pack_bf16(v[8 * c + 4], v[8 * c + 5]), pack_bf16(v[8 * c + 6], v[8 * c + 7]));
            }
        }
        __syncthreads();
        // lane l writes bytes 16l.. of the block's 512-byte row segment
        const int l = threadIdx.x & 31;
        if (ub * 8 + (l >> 2) < w.units) {
            for (int rr = wp; rr < 32; rr += 8) {
                const int64_t grow = (int64_t)rb * 32 + rr;
                if (grow >= w.rows) break;
                const int64_t o = (grow * K + (int64_t)ub * 256) * 2 + 16 * l;
                *(uint4 *)((uint8_t *)whi + o) = *(const uint4 *)(tile[0] + rr * PREP_RS + 16 * l);
                if constexpr (EX) *(uint4 *)((uint8_t *)wlo + o) = *(const uint4 *)(tile[EX ? 1 : 0] + rr * PREP_RS + 16 * l);
            }
        }
        return;
    }
    const int xb = blockIdx.x - nw;
    if constexpr (EX) {
        f16_split_row(X, (int)K, (__half *)xhi, (__half *)xlo, rowshift, xb, red);
    } else {
        // xv (1 or PREP_XV) groups of 8 values per thread, a block's groups
        // 8 x 256 apart (coalesced), every load issued before the first store
        const int64_t n8 = (int64_t)T * K / 8;
        const int xv = n8 >= PREP_XV_BIG ? 1 : PREP_XV;
        float4 a[PREP_XV], b[PREP_XV];
#pragma unroll
        for (int r = 0; r < PREP_XV; r++) {
            const int64_t gi = ((int64_t)xb * xv + r) * 256 + threadIdx.x;
            if (r < xv && gi < n8) {
                a[r] = __ldcs((const float4 *)(X + 8 * gi));
                b[r] = __ldcs((const float4 *)(X + 8 * gi + 4));
            }
        }
#pragma unroll
        for (int r = 0; r < PREP_XV; r++) {
            const int64_t gi = ((int64_t)xb * xv + r) * 256 + threadIdx.x;
            if (r < xv && gi < n8)
                *(uint4 *)(xhi + 8 * gi) = make_uint4(pack_bf16(a[r].x, a[r].y), pack_bf16(a[r].z, a[r].w),
                                                      pack_bf16(b[r].x, b[r].y), pack_bf16(b[r].z, b[r].w));
        }
    }
}

constexpr int TC4_PW = 4;                       // TMA producer warps
constexpr int TC4_MMA = TC4_PW, TC4_EPI = TC4_PW + 1;
constexpr int TC4_THREADS = (TC4_EPI + 4) * 32;
constexpr int TC4_MAX_STG = 10;
constexpr int TC4_SMEM_MAX = 227 * 1024;
constexpr int TC4_ECH = 16;                              // token columns per output chunk
constexpr int TC4_EPI_BYTES = 2 * TC4_ECH * 128 * 4;     // two fp32 chunks [16 tokens][128 rows]

// Shared memory: STG stages [A hi 16 KB][A lo 16 KB, EX][B hi BT*128][B lo
// BT*128, EX], then the two output chunks of the epilogue.
__host__ __device__ inline int tc4_stage_bytes(int bt, int ex) { return (ex ? 2 : 1) * (128 + bt) * BK * 2; }
__host__ __device__ inline int tc4_stages(int bt, int ex) {
    const int n = (TC4_SMEM_MAX - 2048 - TC4_EPI_BYTES) / tc4_stage_bytes(bt, ex);
    return n > TC4_MAX_STG ? TC4_MAX_STG : n;
}

// Bounded wait by a whole warp, with a warp-uniform result.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, int *flag, unsigned sleep_ns = 0) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, flag, sleep_ns));
}

// The 128 epilogue threads: named barrier 1, and a vote that makes a flag
// uniform over them (so that all take the same barriers).
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ bool epi_all(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, 128, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *tm, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"((uint64_t)tm),
                 "r"(src), "r"(x), "r"(y)
                 : "memory");
}
// The same tile added element-wise to global memory (fp32, in L2).
__device__ __forceinline__ void tma_add_2d(const CUtensorMap *tm, uint32_t src, int x, int y) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     (uint64_t)tm),
                 "r"(src), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

template <int EX>
__global__ void __launch_bounds__(TC4_THREADS, 1)
    k_gemm_tc4(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmw_lo,
               const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmx_lo,
               const __grid_constant__ CUtensorMap tmy, float *__restrict__ Y, int T, int N, int BT, int ntm,
               int ntiles, int ksteps, int wshift, const int *__restrict__ rowshift, int ytma, int *flag) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full[TC4_MAX_STG], empty[TC4_MAX_STG];
    __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], fin_bar;
    __shared__ uint32_t tmem_base_sh;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int SB = tc4_stage_bytes(BT, EX), STG = tc4_stages(BT, EX);
    const int AB = 128 * BK * 2, BB = BT * BK * 2;
    const int A_LO = AB, B_HI = (EX ? 2 : 1) * AB, B_LO = B_HI + BB;
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STG; s++) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(smem_u32(&acc_full[i]), 1);
            mbar_init(smem_u32(&acc_empty[i]), 128);
        }
        mbar_init(smem_u32(&fin_bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmw) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmx) : "memory");
        if (ytma) asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmy) : "memory");
        if (EX) {
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmw_lo) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmx_lo) : "memory");
        }
    }
    if (warp == TC4_MMA) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    pdl_wait();
    pdl_trigger();

    // The producer and MMA loops run on whole warps (one lane issues), so that
    // no lane waits at a reconvergence point while another spins.
    if (warp < TC4_PW) {
        // ---- TMA producers: warp j < npw issues the steps g with g % npw == j.
        // npw <= STG keeps every parity wait on empty[s] at most one phase
        // ahead: before its step g a warp has seen step g - npw - STG consumed
        // (its previous wait), so the phase of step g - 2 STG is complete.
        const int npw = STG < TC4_PW ? STG : TC4_PW;
        if (warp < npw) {
            int g = 0, s = 0, turn = 0, last[TC4_MAX_STG];
            uint32_t ph = 0;  // phase parity of stage s at step g
            for (int i = 0; i < STG; i++) last[i] = -1;
            bool alive = true;
            for (int item = blockIdx.x; item < ntiles && alive; item += gridDim.x) {
                const int row0 = (item % ntm) * 128, t0 = (item / ntm) * BT;
                for (int ks = 0; ks < ksteps; ks++) {
                    if (turn == warp) {
                        if (!mbar_wait_warp(smem_u32(&empty[s]), ph ^ 1, flag, 64)) { alive = false; break; }
                        if (lane == 0) {
                            const uint32_t bar = smem_u32(&full[s]), st = smem_u32(base + s * SB);
                            mbar_expect_tx(bar, SB);
                            tma_2d(st, &tmw, ks * BK, row0, bar);
                            tma_2d(st + B_HI, &tmx, ks * BK, t0, bar);
                            if (EX) {
                                tma_2d(st + A_LO, &tmw_lo, ks * BK, row0, bar);
                                tma_2d(st + B_LO, &tmx_lo, ks * BK, t0, bar);
                            }
                        }
                        __syncwarp();
                        last[s] = g;
                    }
                    g++;
                    if (++s == STG) { s = 0; ph ^= 1; }
                    if (++turn == npw) turn = 0;
                }
            }
            // On an early exit, this warp's copies still in flight land before
            // the CTA does (on a normal exit the MMA has consumed them all).
            if (!alive)
                for (int i = 0; i < STG; i++)
                    if (last[i] >= 0) mbar_wait_quiet(smem_u32(&full[i]), (last[i] / STG) & 1);
        }
    } else if (warp == TC4_MMA) {
        // ---- MMA issuer
        const uint32_t idesc = EX ? idesc_f16(BT) : idesc_bf16(BT);
        int s = 0, li = 0;
        uint32_t ph = 0;
        bool alive = true;
        for (int item = blockIdx.x; item < ntiles && alive; item += gridDim.x, li++) {
            const int buf = li & 1;
            if (!mbar_wait_warp(smem_u32(&acc_empty[buf]), ((li >> 1) & 1) ^ 1, flag)) break;
            tc_fence_after();
            const uint32_t d = tmem + (uint32_t)(buf * BT);
            // With four or more stages, two K-steps per round: their waits,
            // MMAs and commits back to back, so that the fixed per-round cost
            // of the issuing thread (barrier waits, commits) is paid once per
            // 8 MMAs.  The MMAs read shared memory that TMA wrote; the
            // mbarrier completion orders those writes, no tcgen05 fence is
            // needed here.
            for (int ks = 0; ks < ksteps;) {
                const bool two = STG >= 4 && ks + 1 < ksteps;
                const int s1 = s + 1 == STG ? 0 : s + 1;
                const uint32_t ph1 = s + 1 == STG ? ph ^ 1 : ph;
                bool ok = mbar_wait(smem_u32(&full[s]), ph, flag);
                if (two) ok = ok && mbar_wait(smem_u32(&full[s1]), ph1, flag);
                if (!__all_sync(0xffffffffu, ok)) { alive = false; break; }
                if (lane == 0) {
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        if (h == 1 && !two) break;
                        const uint32_t a0 = smem_u32(base + (h ? s1 : s) * SB), b0 = a0 + B_HI;
#pragma unroll
                        for (int kk = 0; kk < BK / 16; kk++) {
                            const uint64_t ad = sw128_desc(a0 + kk * 32), bd = sw128_desc(b0 + kk * 32);
                            const uint32_t acc = (ks > 0 || h > 0 || kk > 0) ? 1u : 0u;
                            asm volatile(
                                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                                " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
                                "l"(ad), "l"(bd), "r"(idesc), "r"(acc));
                            if (EX) {
                                // + w_hi x_lo + w_lo x_hi (w_lo x_lo is below 2^-22)
                                const uint64_t bdl = sw128_desc(a0 + B_LO + kk * 32);
                                const uint64_t adl = sw128_desc(a0 + A_LO + kk * 32);
                                asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 1;" ::"r"(d),
                                             "l"(ad), "l"(bdl), "r"(idesc));
                                asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 1;" ::"r"(d),
                                             "l"(adl), "l"(bd), "r"(idesc));
                            }
                        }
                    }
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                     smem_u32(&empty[s]))
                                 : "memory");
                    if (two)
                        asm volatile(
                            "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                smem_u32(&empty[s1]))
                            : "memory");
                }
                __syncwarp();
                if (two) {
                    s = s1 + 1 == STG ? 0 : s1 + 1;
                    ph = s1 + 1 == STG ? ph1 ^ 1 : ph1;
                } else {
                    s = s1;
                    ph = ph1;
                }
                ks += two ? 2 : 1;
            }
            if (alive && lane == 0)
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_u32(&acc_full[buf]))
                             : "memory");
            __syncwarp();
        }
        // Completion of this commit covers every MMA issued above; it is
        // awaited also after a timeout, before TMEM is freed.
        if (lane == 0)
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&fin_bar))
                         : "memory");
        __syncwarp();
        mbar_wait_quiet(smem_u32(&fin_bar), 0);
    } else {
        // ---- epilogue: warp quarter q reads TMEM lanes 32q.. (weight rows),
        // 16 token columns at a time.  With ytma the chunk goes through shared
        // memory ([16 tokens][128 rows], two buffers) and leaves by one TMA
        // store, which clips rows past N and tokens past T; otherwise each
        // store instruction writes 32 consecutive weight rows of one token.
        const int q = warp & 3, et = threadIdx.x - TC4_EPI * 32;
        float *ebuf = (float *)(base + STG * SB);
        int li = 0, ch = 0;
        for (int item = blockIdx.x; item < ntiles; item += gridDim.x, li++) {
            const int buf = li & 1;
            const int row0 = (item % ntm) * 128;
            const int64_t n = (int64_t)row0 + 32 * q + lane;
            const int t0 = (item / ntm) * BT;
            const bool ok = epi_all(mbar_wait(smem_u32(&acc_full[buf]), (li >> 1) & 1, flag, 128));
            tc_fence_after();
            for (int c0 = 0; ok && c0 < BT && t0 + c0 < T; c0 += TC4_ECH, ch++) {
                uint32_t rr[16];
                const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * BT + c0);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                    "[%16];"
                    : "=r"(rr[0]), "=r"(rr[1]), "=r"(rr[2]), "=r"(rr[3]), "=r"(rr[4]), "=r"(rr[5]), "=r"(rr[6]),
                      "=r"(rr[7]), "=r"(rr[8]), "=r"(rr[9]), "=r"(rr[10]), "=r"(rr[11]), "=r"(rr[12]), "=r"(rr[13]),
                      "=r"(rr[14]), "=r"(rr[15])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    v[j] = __uint_as_float(rr[j]);
                    // EX: undo 2^(wshift + rowshift[t]) (exact power of two)
                    if (EX) {
                        const int t = min(t0 + c0 + j, T - 1);
                        v[j] *= __int_as_float((127 - wshift - __ldg(rowshift + t)) << 23);
                    }
                }
                if (ytma) {
                    float *sb = ebuf + (ch & 1) * (TC4_ECH * 128);
                    if (et == 0) bulk_wait_read1();  // the store issued from this buffer two chunks ago has read it
                    epi_sync();
#pragma unroll
                    for (int j = 0; j < 16; j++) sb[j * 128 + 32 * q + lane] = v[j];
                    fence_async_smem();
                    epi_sync();
                    if (et == 0) {
                        tma_store_2d(&tmy, smem_u32(sb), row0, t0 + c0);
                        bulk_commit();
                    }
                } else if (n < N) {
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (t0 + c0 + j < T) Y[(int64_t)(t0 + c0 + j) * N + n] = v[j];
                }
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&acc_empty[buf]));
            if (!ok) break;
        }
        if (et == 0) bulk_wait_all();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == TC4_MMA) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// ------------------------------------------------------------------- v5
// The two-pass GEMM with each MMA across an SM pair (bf16 mode):
// tcgen05.mma.cta_group::2 with M = 256.  A CTA pair (a cluster of two) owns
// a tile of 256 weight rows x BT tokens: CTA r of the pair loads weight rows
// 128 r .. 128 r + 127 of the tile and tokens BT/2 r .. BT/2 r + BT/2 - 1
// into the same shared-memory offsets, and the leader's (rank 0) single MMA
// thread issues MMAs that read both CTAs' halves; each CTA's tensor memory
// receives its 128 rows x BT tokens of the product.
// Why.  In the one-SM kernel each 64-deep K-step moves (128 + BT) x 128 bytes
// through an SM's shared memory twice (TMA write, MMA read): at BT = 192,
// 80 KB against 384 cycles of MMA, so shared memory (~128 B per cycle), not
// the tensor pipe, set the pace.  Split across the pair, an SM moves
// (128 + BT/2) x 128 bytes per step for the same 2 BT cycles of MMA per SM:
// at BT = 256, 64 KB against 512 cycles.
// Protocol (per stage s): each CTA's producer waits for its own empty[s]
// (released by the leader's tcgen05.commit multicast to both CTAs), the
// leader's producer posts the transaction bytes of both halves on the
// leader's full[s], and both CTAs' TMA loads (cta_group::2, no multicast)
// complete on the leader's full[s]; the leader's MMA thread waits for
// full[s].  The accumulators: acc_full[b] in both CTAs (multicast commit),
// acc_empty[b] in the leader with 256 arrivals (the 128 epilogue threads of
// each CTA, the peer's arriving remotely).  Tensor memory is allocated and
// freed by warp 4 of both CTAs (cta_group::2).  Cluster barriers after the
// barrier initialisation and before the end keep either CTA from signalling
// or reading a partner that has not started or has already left.  Waits are
// bounded as in v4.
// The issuing thread sets the pace: a tcgen05.mma costs it ~100 cycles to
// issue whatever its N (clock64 traces of the leader's MMA thread), and a
// barrier wait ~190 cycles even when the stage has landed.  So stages go in
// pairs with one (full, empty) barrier pair per two K-steps, one wait and
// one commit per 8 MMAs, and the thread's loop is lean: descriptors are one
// add from per-kernel bases.  Measured (prep + GEMM, B200): Q5_0 4864 x 896
// at T = 2048 26.2 us (682 TFLOP/s; one-SM kernel 28.0), Q4_K 3584 x 3584
// 57.8 us (911; 65.6), Q4_K 18944 x 3584 at T = 512 96.5 us (721; 112.9).
constexpr int TC5_MAX_STG = 12;
constexpr int TC5_EPI_WARPS = 8;                          // two per TMEM lane quarter, each half the columns
constexpr int TC5_THREADS = (TC4_EPI + TC5_EPI_WARPS) * 32;
constexpr int TC5_EPI_BYTES = 2 * TC4_EPI_BYTES;          // two output chunk buffers per column half
__host__ __device__ inline int tc5_stage_bytes(int bt) { return (128 + bt / 2) * BK * 2; }
__host__ __device__ inline int tc5_stages(int bt) {
    const int n = (TC4_SMEM_MAX - 2048 - TC5_EPI_BYTES) / tc5_stage_bytes(bt);
    return n > TC5_MAX_STG ? TC5_MAX_STG : n;
}
// Named barrier 1 + h of the 128 epilogue threads of column half h, and a
// vote over them.
__device__ __forceinline__ void epi5_sync(int h) { asm volatile("bar.sync %0, 128;" ::"r"(1 + h) : "memory"); }
__device__ __forceinline__ bool epi5_all(int h, bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, 128, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(1 + h)
        : "memory");
    return r != 0;
}
// Instruction descriptor: fp32 accumulate, bf16 A and B, both K-major, M = 256 (the pair), N = bt.
__host__ __device__ constexpr uint32_t idesc_bf16_pair(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}
__device__ __forceinline__ uint32_t tc5_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void tc5_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t tc5_mapa(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// A 2D tile load of one CTA of the pair, completing on the barrier at the
// cluster address bar (the leader's).
__device__ __forceinline__ void tma_2d_pair(uint32_t dst, const CUtensorMap *tm, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3}], [%4];" ::"r"(dst),
        "l"((uint64_t)tm), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Completion of the leader's MMAs issued so far, as one arrival on the
// barrier at this offset in both CTAs of the pair.
__device__ __forceinline__ void commit_pair(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"((uint16_t)3)
        : "memory");
}

__global__ void __launch_bounds__(TC5_THREADS, 1)
    k_gemm_tc5(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
               const __grid_constant__ CUtensorMap tmy, float *__restrict__ Y, int T, int N, int BT, int ntm2,
               int ntiles, int ksteps, int ytma, int ksplit, int *flag) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full[TC5_MAX_STG], empty[TC5_MAX_STG];
    __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], fin_bar;
    __shared__ uint32_t tmem_base_sh;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = tc5_rank();   // 0: the leader, which issues the MMAs
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int SB = tc5_stage_bytes(BT), STG = tc5_stages(BT) & ~1, NP = STG / 2;   // stage pairs
    const int AB = 128 * BK * 2, HB = BT / 2, kpairs = (ksteps + 1) / 2;
    // Items: ksplit parts of K (contiguous runs of step pairs) of every tile,
    // part-major; with ksplit = 2 each part adds its sums into Y (zeroed
    // before the launch): two addends onto zero give the same bits in either
    // order.
    const int nitems = ntiles * ksplit;
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);

    if (threadIdx.x == 0) {
        for (int s = 0; s < NP; s++) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(smem_u32(&acc_full[i]), 1);
            mbar_init(smem_u32(&acc_empty[i]), 2 * TC5_EPI_WARPS * 32);
        }
        mbar_init(smem_u32(&fin_bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmw) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmx) : "memory");
        if (ytma) asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmy) : "memory");
    }
    if (warp == TC4_MMA) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc5_cluster_sync();   // both CTAs' barriers initialised before any remote arrival
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    pdl_wait();
    pdl_trigger();

    if (warp < TC4_PW) {
        // ---- TMA producers (both CTAs).  Stages go in pairs: one barrier
        // pair (full, empty) per two K-steps, so that the MMA thread waits and
        // commits once per 8 MMAs.  Pairs of steps are dealt to the warps in
        // turn as the steps are in v4.
        const int npw = NP < TC4_PW ? NP : TC4_PW;
        if (warp < npw) {
            const uint32_t full0 = tc5_mapa(smem_u32(&full[0]), 0);   // the leader's full[0]
            int g = 0, sp = 0, turn = 0;
            uint32_t ph = 0;
            bool alive = true;
            for (int item = pair; item < nitems && alive; item += npairs) {
                const int tile = item % ntiles, part = item / ntiles;
                const int row0 = (tile % ntm2) * 256 + (int)rank * 128, t0 = (tile / ntm2) * BT + (int)rank * HB;
                const int kp0 = part * kpairs / ksplit, kp1 = (part + 1) * kpairs / ksplit;
                for (int kp = kp0; kp < kp1; kp++) {
                    if (turn == warp) {
                        if (!mbar_wait_warp(smem_u32(&empty[sp]), ph ^ 1, flag, 64)) { alive = false; break; }
                        if (lane == 0) {
                            const int nst = 2 * kp + 1 < ksteps ? 2 : 1;
                            const uint32_t bar = full0 + 8u * (uint32_t)sp;
                            if (rank == 0) mbar_expect_tx(smem_u32(&full[sp]), 2 * nst * SB);
                            for (int j = 0; j < nst; j++) {
                                const uint32_t st = smem_u32(base + (2 * sp + j) * SB);
                                const int ks = 2 * kp + j;
                                tma_2d_pair(st, &tmw, ks * BK, row0, bar);
                                tma_2d_pair(st + AB, &tmx, ks * BK, t0, bar);
                            }
                        }
                        __syncwarp();
                    }
                    g++;
                    if (++sp == NP) { sp = 0; ph ^= 1; }
                    if (++turn == npw) turn = 0;
                }
            }
            // After a timeout the loads in flight complete on the leader's
            // barrier; give them time to land in this CTA's stages.
            if (!alive) __nanosleep(100000);
        }
    } else if (warp == TC4_MMA) {
        if (rank == 0 && lane == 0) {
            // ---- MMA issuer: the leader's lane 0 alone (the rest of the warp
            // waits below).  The issuing thread's own instructions set the
            // pace of short MMAs, so its loop is lean: descriptors are one
            // add from per-kernel bases (stages are contiguous, a descriptor
            // holds the address / 16), and the waits are its own.
            const uint32_t idesc = idesc_bf16_pair(BT);
            const uint64_t adesc0 = sw128_desc(smem_u32(base)), bdesc0 = sw128_desc(smem_u32(base) + AB);
            const uint32_t sstep = (uint32_t)(SB >> 4);
            int sp = 0, li = 0;
            uint32_t ph = 0;
            bool alive = true;
            for (int item = pair; item < nitems && alive; item += npairs, li++) {
                const int buf = li & 1, part = item / ntiles;
                const int kp0 = part * kpairs / ksplit, kp1 = (part + 1) * kpairs / ksplit;
                if (!mbar_wait(smem_u32(&acc_empty[buf]), ((li >> 1) & 1) ^ 1, flag)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * BT);
                for (int kp = kp0; kp < kp1; kp++) {
                    if (!mbar_wait(smem_u32(&full[sp]), ph, flag)) { alive = false; break; }
                    const int nst = 2 * kp + 1 < ksteps ? 2 : 1;
                    for (int j = 0; j < nst; j++) {
                        const uint32_t off = (uint32_t)(2 * sp + j) * sstep;
                        const uint64_t ad = adesc0 + off, bd = bdesc0 + off;
#pragma unroll
                        for (int kk = 0; kk < BK / 16; kk++) {
                            const uint32_t acc = (kp > kp0 || j > 0 || kk > 0) ? 1u : 0u;
                            asm volatile(
                                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                                " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
                                "l"(ad + 2 * kk), "l"(bd + 2 * kk), "r"(idesc), "r"(acc));
                        }
                    }
                    commit_pair(smem_u32(&empty[sp]));
                    if (++sp == NP) { sp = 0; ph ^= 1; }
                }
                if (alive) commit_pair(smem_u32(&acc_full[buf]));
            }
            // Completion of this commit covers every MMA issued above (in both
            // CTAs' tensor memory); awaited also after a timeout.
            commit_pair(smem_u32(&fin_bar));
        }
        __syncwarp();
        mbar_wait_quiet(smem_u32(&fin_bar), 0);
    } else {
        // ---- epilogue (both CTAs): this CTA's 128 rows of the tile; warp
        // w reads TMEM lanes 32 (w % 4).. (rows) and column half h of the
        // tile's BT token columns, 16 columns at a time.
        const int ew = warp - TC4_EPI, q = warp & 3, h = ew >> 2, et = threadIdx.x - (TC4_EPI + 4 * h) * 32;
        float *ebuf = (float *)(base + STG * SB) + h * (2 * TC4_ECH * 128);
        const uint32_t ae0 = tc5_mapa(smem_u32(&acc_empty[0]), 0);   // the leader's acc_empty[0]
        const int c_lo = h * (BT / 2), c_hi = c_lo + BT / 2;
        int li = 0, ch = 0;
        for (int item = pair; item < nitems; item += npairs, li++) {
            const int buf = li & 1, tile = item % ntiles;
            const int row0 = (tile % ntm2) * 256 + (int)rank * 128;
            const int64_t n = (int64_t)row0 + 32 * q + lane;
            const int t0 = (tile / ntm2) * BT;
            const bool ok = epi5_all(h, mbar_wait(smem_u32(&acc_full[buf]), (li >> 1) & 1, flag, 128));
            tc_fence_after();
            // (the peer's rows of the last tile may all lie past N: nothing to store)
            for (int c0 = c_lo; ok && row0 < N && c0 < c_hi && t0 + c0 < T; c0 += TC4_ECH, ch++) {
                uint32_t rr[16];
                const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * BT + c0);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                    "[%16];"
                    : "=r"(rr[0]), "=r"(rr[1]), "=r"(rr[2]), "=r"(rr[3]), "=r"(rr[4]), "=r"(rr[5]), "=r"(rr[6]),
                      "=r"(rr[7]), "=r"(rr[8]), "=r"(rr[9]), "=r"(rr[10]), "=r"(rr[11]), "=r"(rr[12]), "=r"(rr[13]),
                      "=r"(rr[14]), "=r"(rr[15])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; j++) v[j] = __uint_as_float(rr[j]);
                if (ytma) {
                    float *sb = ebuf + (ch & 1) * (TC4_ECH * 128);
                    if (et == 0) bulk_wait_read1();
                    epi5_sync(h);
#pragma unroll
                    for (int j = 0; j < 16; j++) sb[j * 128 + 32 * q + lane] = v[j];
                    fence_async_smem();
                    epi5_sync(h);
                    if (et == 0) {
                        if (ksplit > 1)
                            tma_add_2d(&tmy, smem_u32(sb), row0, t0 + c0);
                        else
                            tma_store_2d(&tmy, smem_u32(sb), row0, t0 + c0);
                        bulk_commit();
                    }
                } else if (n < N) {
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (t0 + c0 + j < T) Y[(int64_t)(t0 + c0 + j) * N + n] = v[j];
                }
            }
            tc_fence_before();
            mbar_arrive_cluster(ae0 + 8u * (uint32_t)buf);
            if (!ok) break;
        }
        if (et == 0) bulk_wait_all();
    }
    tc_fence_before();
    __syncthreads();
    tc5_cluster_sync();   // neither CTA leaves while its partner may still signal it or read its stages
    if (warp == TC4_MMA) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// Token tile (a multiple of 32, 64..256) and K parts (1 or 2) of the pair
// GEMM, minimising rounds of items per pair x (K-steps per item x cycles per
// step + ~1000 cycles of tile turnover); a step costs the larger of its MMA
// time (2 BT per SM) and the shared-memory traffic of one SM's halves
// (written once, read once, ~128 B per cycle).  Two K parts add ~3e-3 cycles
// per output element (Y zeroed, then two additions in L2): worth it when the
// tiles alone leave pairs idle (896 x 4864 at T = 2048: 44 tiles, 74 pairs).
int tc5_pick(int64_t mt2, int T, int pairs, int ksteps, int64_t N, bool can_split, int *ks_out) {
    int best_bt = 64, best_ks = 1;
    double best = 1e30;
    const int kpairs = (ksteps + 1) / 2;
    for (int ks = 1; ks <= (can_split && kpairs >= 2 ? 2 : 1); ks++) {
        for (int bt = 64; bt <= 256; bt += 32) {
            if (bt > 64 && T <= bt - 32) break;
            if (tc5_stages(bt) < 4) continue;   // two stage pairs at least
            const int64_t items = mt2 * ((T + bt - 1) / bt) * ks;
            const double rounds = (double)((items + pairs - 1) / pairs);
            const double mma = 2.0 * bt, smem = 2.0 * tc5_stage_bytes(bt) / 128.0;
            const double steps = 2.0 * ((kpairs + ks - 1) / ks);
            double cost = rounds * (steps * ((mma > smem ? mma : smem) + 64.0) + 1000.0);
            if (ks > 1) cost += 3e-3 * (double)T * (double)N;
            if (cost < best - 1e-9) { best = cost; best_bt = bt; best_ks = ks; }
        }
    }
    *ks_out = best_ks;
    return best_bt;
}

template <int TYPE, int BT, int EX>
cudaError_t launch_tc3(hd_ctx *ctx, const hd_weight *w, const CUtensorMap &tmx, const CUtensorMap &tmx_lo, float *Y,
                       int T, int ks, const int *rowshift) {
    constexpr size_t smem = TC3<TYPE, BT, EX>::SMEM;
    cudaError_t e =
        cudaFuncSetAttribute(k_qgemm_tc3<TYPE, BT, EX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int ntm = (int)(w->rows / 128), ntiles = ntm * ((T + BT - 1) / BT);
    if (ks == 2) {
        e = cudaMemsetAsync(Y, 0, (size_t)T * w->rows * sizeof(float), ctx->stream);
        if (e != cudaSuccess) return e;
    }
    const int nitems = ntiles * ks;
    const int grid = nitems < ctx->sm_count ? nitems : ctx->sm_count;
    return hd_launch(ctx, k_qgemm_tc3<TYPE, BT, EX>, dim3(grid), dim3(TC3_THREADS), smem, wview(w), tmx, tmx_lo, Y, T,
                     (int)w->rows, ntm, ntiles, ks, w->f16_shift, rowshift, ctx->flag);
}

// Token tile of the two-pass GEMM: the multiple of 16 (64..256; exact mode
// up to 160, three stages of hi and lo tiles) minimising rounds of tiles per
// SM x cycles per K-step, a step costing the larger of its MMA time (2*BT per
// product) and its shared-memory traffic at ~128 B per cycle (stage written
// once, read once; exact mode: hi tiles read twice).
int tc4_pick_bt(int64_t mt, int T, int sms, int ex) {
    int best_bt = 64;
    double best = 1e30;
    for (int bt = 64; bt <= (ex ? 160 : 256); bt += 16) {
        if (bt > 64 && T <= bt - 16) break;
        if (tc4_stages(bt, ex) < 3) continue;
        const int64_t tiles = mt * ((T + bt - 1) / bt);
        const double rounds = (double)((tiles + sms - 1) / sms);
        const double sb = tc4_stage_bytes(bt, ex);
        const double mma = (ex ? 3.0 : 1.0) * 2.0 * bt, smem = (ex ? 2.5 : 2.0) * sb / 128.0;
        const double cost = rounds * ((mma > smem ? mma : smem) + 64.0);
        if (cost < best - 1e-9) { best = cost; best_bt = bt; }
    }
    return best_bt;
}

// The pair GEMM (k_gemm_tc5) on the prepared bf16 operands wb [N][K] and
// xb [T][K]: clusters of two CTAs, one pair per two SMs.
int launch_tc5(hd_ctx *ctx, const uint8_t *wb, const uint8_t *xb, int64_t N, int64_t K, int T, float *Y, int ksteps) {
    const int64_t mt2 = (N + 255) / 256;
    const int pairs_max = ctx->sm_count / 2;
    const bool ytma_ok = N % 4 == 0 && getenv("HACEDLE_TC4_DIRECT_STORE") == nullptr;
    int ks = 1;
    int bt = tc5_pick(mt2, T, pairs_max, ksteps, N, ytma_ok, &ks);
    if (const char *env = getenv("HACEDLE_TC_BT")) {
        const int b = atoi(env);
        if (b >= 64 && b <= 256 && b % 32 == 0) bt = b;
    }
    if (const char *env = getenv("HACEDLE_TC5_KS")) {   // K parts: 1, or 2 where the output goes by TMA
        const int k = atoi(env);
        if (k == 1 || (k == 2 && ytma_ok && ksteps >= 3)) ks = k;
    }
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm: cuTensorMapEncodeTiled is not available");
    auto make = [&](CUtensorMap *m, const void *ptr, int64_t rows, int box_rows) {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
        cuuint64_t strides[1] = {(cuuint64_t)K * 2};
        cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
        cuuint32_t estr[2] = {1, 1};
        return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    };
    CUtensorMap tw, tx, ty;
    CUresult cr = make(&tw, wb, N, 128);
    if (cr == CUDA_SUCCESS) cr = make(&tx, xb, T, bt / 2);
    int ytma = 0;
    if (cr == CUDA_SUCCESS && ytma_ok) {
        cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)T};
        cuuint64_t strides[1] = {(cuuint64_t)N * 4};
        cuuint32_t box[2] = {128, (cuuint32_t)TC4_ECH};
        cuuint32_t estr[2] = {1, 1};
        cr = enc(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, Y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                 CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        ytma = 1;
    } else {
        ty = tx;
    }
    if (cr != CUDA_SUCCESS) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm: cuTensorMapEncodeTiled failed (%d)", (int)cr);
    const size_t smem = (size_t)tc5_stages(bt) * tc5_stage_bytes(bt) + TC5_EPI_BYTES + 1024;
    const int ntm2 = (int)mt2, ntiles = ntm2 * ((T + bt - 1) / bt);
    const int pairs = ntiles * ks < pairs_max ? ntiles * ks : pairs_max;
    cudaError_t e = cudaSuccess;
    if (ks > 1) e = cudaMemsetAsync(Y, 0, (size_t)T * (size_t)N * sizeof(float), ctx->stream);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_gemm_tc5, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
        e = hd_launch_cluster(ctx, k_gemm_tc5, dim3(2 * pairs), dim3(TC5_THREADS), smem, 2, tw, tx, ty, Y, T, (int)N, bt,
                              ntm2, ntiles, ksteps, ytma, ks, ctx->flag);
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm (tcgen05 pair GEMM): %s", cudaGetErrorString(e));
    return HD_OK;
}

// The two-pass path (see k_gemm_tc4).  Activations as for v3; the weight is
// dequantized into ctx->wbf first.  The bf16 mode runs the pair GEMM
// (k_gemm_tc5) where its tiles fill the SM pairs.
int qgemm_tc4(hd_ctx *ctx, const hd_weight *w, const float *X, float *Y, int T, int exact) {
    const int64_t N = w->rows, K = w->cols;
    const size_t plane = ((size_t)T * K * 2 + 255) & ~(size_t)255;
    const size_t need = exact ? 2 * plane + (size_t)T * sizeof(int) : plane;
    int rc = hd_ensure_hbuf(ctx, &ctx->xbf, &ctx->xbf_bytes, (need + 3) / 4 * 4);
    if (rc) return rc;
    const size_t wplane = ((size_t)N * K * 2 + 255) & ~(size_t)255;
    rc = hd_ensure_hbuf(ctx, &ctx->wbf, &ctx->wbf_bytes, (exact ? 2 : 1) * wplane);
    if (rc) return rc;
    uint8_t *xb = (uint8_t *)ctx->xbf, *wb = (uint8_t *)ctx->wbf;
    int *rowshift = exact ? (int *)(xb + 2 * plane) : nullptr;
    const WView v = wview(w);
    const int nrb = (int)((N + 31) / 32), nw = nrb * ((w->units + 7) / 8);
    const int64_t n8 = (int64_t)T * K / 8;
    const int xv = n8 >= PREP_XV_BIG ? 1 : PREP_XV;
    const int nx = exact ? T : (int)((n8 + 256 * xv - 1) / (256 * xv));
    cudaError_t e = cudaSuccess;
    HD_TYPE_SWITCH(w->type, TT, {
        if (exact)
            e = hd_launch(ctx, k_prep<TT, 1>, dim3((unsigned)(nw + nx)), dim3(256), 0, v, (uint16_t *)wb,
                          (uint16_t *)(wb + wplane), w->f16_shift, nrb, nw, X, T, (uint16_t *)xb,
                          (uint16_t *)(xb + plane), rowshift);
        else
            e = hd_launch(ctx, k_prep<TT, 0>, dim3((unsigned)(nw + nx)), dim3(256), 0, v, (uint16_t *)wb,
                          (uint16_t *)nullptr, 0, nrb, nw, X, T, (uint16_t *)xb, (uint16_t *)nullptr, (int *)nullptr);
    });
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm (operand preparation): %s", cudaGetErrorString(e));
    if (!exact) {
        // The pair GEMM where its 256-row tiles fill the SM pairs (measured on
        // B200, prep + GEMM: 18944 x 3584 Q4_K at T = 512 721 against 616
        // TFLOP/s, 3584 x 3584 at T = 2048 911 against 798, 4864 x 896 Q5_0
        // 682 against 637); with fewer tiles (896 x 4864: 44 tiles for 74
        // pairs) the one-SM kernel, 466 against 459.  HACEDLE_TC5 = 1 / 0
        // forces it on / off.
        const char *v5 = getenv("HACEDLE_TC5");
        // (K in two parts counts double: taken on long K only)
        const int64_t tiles2 = ((N + 255) / 256) * ((T + 191) / 192) * (N % 4 == 0 && K >= 2048 ? 2 : 1);
        const bool pair = v5 && *v5 ? *v5 != '0' : tiles2 >= ctx->sm_count / 2;
        if (pair) return launch_tc5(ctx, wb, xb, N, K, T, Y, (int)((w->units + 1) / 2));
    }

    const int64_t mt = (N + 127) / 128;
    int bt = tc4_pick_bt(mt, T, ctx->sm_count, exact);
    if (const char *env = getenv("HACEDLE_TC_BT")) {
        const int b = atoi(env);
        if (b >= 16 && b <= (exact ? 160 : 256) && b % 16 == 0) bt = b;
    }
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm: cuTensorMapEncodeTiled is not available");
    const CUtensorMapDataType dt = exact ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap tw, twl, tx, txl;
    auto make = [&](CUtensorMap *m, void *ptr, int64_t rows, int box_rows) {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
        cuuint64_t strides[1] = {(cuuint64_t)K * 2};
        cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
        cuuint32_t estr[2] = {1, 1};
        return enc(m, dt, 2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    };
    CUresult cr = make(&tw, wb, N, 128);
    if (cr == CUDA_SUCCESS) cr = make(&twl, exact ? wb + wplane : wb, N, 128);
    if (cr == CUDA_SUCCESS) cr = make(&tx, xb, T, bt);
    if (cr == CUDA_SUCCESS) cr = make(&txl, exact ? xb + plane : xb, T, bt);
    // Output chunks by TMA store when the rows of Y are 16-byte multiples.
    CUtensorMap ty;
    int ytma = 0;
    if (cr == CUDA_SUCCESS && N % 4 == 0 && getenv("HACEDLE_TC4_DIRECT_STORE") == nullptr) {
        cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)T};
        cuuint64_t strides[1] = {(cuuint64_t)N * 4};
        cuuint32_t box[2] = {128, (cuuint32_t)TC4_ECH};
        cuuint32_t estr[2] = {1, 1};
        cr = enc(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, Y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                 CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        ytma = 1;
    } else {
        ty = tx;
    }
    if (cr != CUDA_SUCCESS) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm: cuTensorMapEncodeTiled failed (%d)", (int)cr);

    const size_t smem = (size_t)tc4_stages(bt, exact) * tc4_stage_bytes(bt, exact) + TC4_EPI_BYTES + 1024;
    const int ntm = (int)mt, ntiles = ntm * ((T + bt - 1) / bt);
    const int grid = ntiles < ctx->sm_count ? ntiles : ctx->sm_count;
    const int ksteps = (int)((w->units + 1) / 2);
    if (exact) {
        e = cudaFuncSetAttribute(k_gemm_tc4<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess)
            e = hd_launch(ctx, k_gemm_tc4<1>, dim3(grid), dim3(TC4_THREADS), smem, tw, twl, tx, txl, ty, Y, T, (int)N,
                          bt, ntm, ntiles, ksteps, w->f16_shift, (const int *)rowshift, ytma, ctx->flag);
    } else {
        e = cudaFuncSetAttribute(k_gemm_tc4<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess)
            e = hd_launch(ctx, k_gemm_tc4<0>, dim3(grid), dim3(TC4_THREADS), smem, tw, twl, tx, txl, ty, Y, T, (int)N,
                          bt, ntm, ntiles, ksteps, 0, (const int *)nullptr, ytma, ctx->flag);
    }
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm (tcgen05 two-pass): %s", cudaGetErrorString(e));
    return HD_OK;
}

}  // namespace

// Fewest tokens for the two-pass path: 128 (HACEDLE_TC4_MIN_T overrides the
// threshold; 0 disables the path).
int hd_tc4_min_t() {
    const char *env = getenv("HACEDLE_TC4_MIN_T");
    return env ? atoi(env) : 128;
}

// From hd_tc4_min_t() tokens, and for rows % 128 != 0 at any T, the two-pass
// kernel; below, rows % 128 == 0 uses the streamed v3 kernel (the v1 kernel
// only runs with the two-pass kernel off, HACEDLE_TC4_MIN_T=0).
// exact != 0 (rows % 128 == 0 only): the fp32-accuracy mode -- exact weights
// and x, each split into fp16 hi + lo, three MMAs per product.
int hd_qgemm_tc(hd_ctx *ctx, const hd_weight *w, const float *X, float *Y, int T, int exact) {
    HD_REQUIRE(ctx, w->cols % 8 == 0, HD_E_SHAPE, "hd_qgemm: K must be a multiple of 8");
    const int64_t mt = (w->rows + 127) / 128;
    {
        // The exact-product mode stays on the streamed kernel where that one
        // runs (rows % 128 == 0): its accumulation order reproduces the fp32
        // oracle's greedy tokens on the 0.5B-shaped decoder, the two-pass
        // order (one K chain per tile) flips a near tie after 15 tokens.
        // HACEDLE_TC4_EXACT=1 sends it to the two-pass kernel as well.
        // Rows not a multiple of 128 take the two-pass kernel at any T: the v1
        // kernel it replaces there is 3-4x slower (T = 64 on the 8-rank
        // slices of the 7B-shaped layer: 65-347 against 22-93 us).
        const int min_t = hd_tc4_min_t();
        const bool ex_v4 = w->rows % 128 != 0 || getenv("HACEDLE_TC4_EXACT") != nullptr;
        if (min_t > 0 && (T >= min_t || w->rows % 128 != 0) && (!exact || ex_v4))
            return qgemm_tc4(ctx, w, X, Y, T, exact);
    }
    cudaError_t e = cudaSuccess;
    const bool v3 = w->rows % 128 == 0 && ((uintptr_t)Y & 15) == 0 && (exact || getenv("HACEDLE_TC_V1") == nullptr);
    HD_REQUIRE(ctx, v3 || !exact, HD_E_UNSUPPORTED, "hd_qgemm: the exact tensor-core mode needs rows % 128 == 0");
    if (v3) {
        // activations for the TMA: bf16, or (exact) fp16 hi and lo planes and
        // the per-row shifts
        const size_t plane = ((size_t)T * w->cols * 2 + 255) & ~(size_t)255;
        const size_t need = exact ? 2 * plane + (size_t)T * sizeof(int) : plane;
        int rc = hd_ensure_hbuf(ctx, &ctx->xbf, &ctx->xbf_bytes, (need + 3) / 4 * 4);
        if (rc) return rc;
        uint8_t *xb = (uint8_t *)ctx->xbf;
        int *rowshift = exact ? (int *)(xb + 2 * plane) : nullptr;
        const int64_t n = (int64_t)T * w->cols;
        if (exact)
            e = hd_launch(ctx, k_to_f16_split, dim3((unsigned)T), dim3(256), 0, X, (int)w->cols, (__half *)xb,
                          (__half *)(xb + plane), rowshift);
        else
            e = hd_launch(ctx, k_to_bf16, dim3((unsigned)((n / 4 + 255) / 256 + 1)), dim3(256), 0, X,
                          (__nv_bfloat16 *)xb, n);
        if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm (activation convert): %s", cudaGetErrorString(e));
        // Token tile and K split by a cost model: rounds of items per SM x
        // steps per item x cycles per step (the MMA's 2*BT per product plus
        // ~200 cycles of per-step overhead); ties go to the smaller tile.
        const int ksteps = (int)((w->units + 1) / 2);
        auto ksplit = [&](int cand) {
            return (2 * mt * ((T + cand - 1) / cand) <= ctx->sm_count && w->units >= 8) ? 2 : 1;
        };
        const int top = exact ? 160 : 208;
        int bt = 64;
        double best = 1e30;
        for (int cand : {64, 128, top}) {
            if (cand > 64 && T <= cand / 2) continue;
            const int64_t tiles = mt * ((T + cand - 1) / cand);
            const int ck = ksplit(cand);
            const double rounds = (double)((tiles * ck + ctx->sm_count - 1) / ctx->sm_count);
            const double cost = rounds * ((ksteps + ck - 1) / ck) * ((exact ? 6.0 : 2.0) * cand + 200.0);
            if (cost < best - 1e-9) { best = cost; bt = cand; }
        }
        const char *bt_env = getenv("HACEDLE_TC_BT");
        if (bt_env && (atoi(bt_env) == 64 || atoi(bt_env) == 128 || atoi(bt_env) == top)) bt = atoi(bt_env);
        const int ks = ksplit(bt);
        EncodeTiledFn enc = encode_tiled();
        if (!enc) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm: cuTensorMapEncodeTiled is not available");
        CUtensorMap tm, tm_lo;
        cuuint64_t dims[2] = {(cuuint64_t)w->cols, (cuuint64_t)T};
        cuuint64_t strides[1] = {(cuuint64_t)w->cols * 2};
        cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)bt};
        cuuint32_t estr[2] = {1, 1};
        const CUtensorMapDataType dt = exact ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        CUresult cr = enc(&tm, dt, 2, xb, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr == CUDA_SUCCESS)
            cr = enc(&tm_lo, dt, 2, exact ? xb + plane : xb, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm: cuTensorMapEncodeTiled failed (%d)", (int)cr);
        if (exact) {
            HD_TYPE_SWITCH(w->type, TT, {
                if (bt == 64) e = launch_tc3<TT, 64, 1>(ctx, w, tm, tm_lo, Y, T, ks, rowshift);
                else if (bt == 128) e = launch_tc3<TT, 128, 1>(ctx, w, tm, tm_lo, Y, T, ks, rowshift);
                else e = launch_tc3<TT, 160, 1>(ctx, w, tm, tm_lo, Y, T, ks, rowshift);
            });
        } else {
            HD_TYPE_SWITCH(w->type, TT, {
                if (bt == 64) e = launch_tc3<TT, 64, 0>(ctx, w, tm, tm_lo, Y, T, ks, rowshift);
                else if (bt == 128) e = launch_tc3<TT, 128, 0>(ctx, w, tm, tm_lo, Y, T, ks, rowshift);
                else e = launch_tc3<TT, 208, 0>(ctx, w, tm, tm_lo, Y, T, ks, rowshift);
            });
        }
        if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm (tcgen05 v3): %s", cudaGetErrorString(e));
        return HD_OK;
    }
    int bt = 64;
    if (T > 64 && mt * ((T + 127) / 128) >= ctx->sm_count) bt = 128;
    if (T > 128 && mt * ((T + 255) / 256) >= 2 * ctx->sm_count) bt = 256;
    HD_TYPE_SWITCH(w->type, TT, {
        if (bt == 64) e = launch_tc<TT, 64>(ctx, w, X, Y, T);
        else if (bt == 128) e = launch_tc<TT, 128>(ctx, w, X, Y, T);
        else e = launch_tc<TT, 256>(ctx, w, X, Y, T);
    });
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm (tcgen05): %s", cudaGetErrorString(e));
    return HD_OK;
}

// Reads and clears the device error flag of the bounded waits.
extern "C" int hd_ctx_check_device_errors(hd_ctx *ctx) {
    if (!ctx) return HD_E_ARG;
    int v = 0;
    HD_CUDA_TRY(ctx, cudaMemcpyAsync(&v, ctx->flag, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    HD_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    if (v) {
        HD_CUDA_TRY(ctx, cudaMemsetAsync(ctx->flag, 0, sizeof(int), ctx->stream));
        return hd_fail(ctx, HD_E_TIMEOUT, "a bounded device wait expired (code %d)", v);
    }
    return HD_OK;
}
