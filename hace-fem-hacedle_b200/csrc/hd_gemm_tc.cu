// hd_gemm_tc.cu -- prefill Q-GEMM on the 5th-generation tensor cores.
//
// Y[t][n] = sum_k X[t][k] W[n][k] with W a quantized GGUF weight and X fp32.
// One CTA computes a 128 (weight rows) x BT (tokens) tile with
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
#include <cuda.h>

#include "hd_internal.cuh"

namespace {

constexpr int STAGES = 4;
constexpr int BK = 64;                       // K per stage (one 128-byte swizzle row of bf16)
constexpr int A_BYTES = 128 * BK * 2;        // 16 KB
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
// Bounded wait: true when the phase completed, false (flag set) on expiry.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int *flag) {
    if (mbar_try(bar, parity)) return true;
    long long t0 = clock64();
    while (!mbar_try(bar, parity)) {
        if (clock64() - t0 > SPIN_LIMIT || *(volatile int *)flag) {
            atomicExch(flag, HD_E_TIMEOUT);
            return false;
        }
    }
    return true;
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

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

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


// ------------------------------------------------------------------- v2
// Same MMA/TMEM structure, with every operand streamed asynchronously:
// activations are converted to bf16 once and arrive by TMA (2-D tiled copy,
// SWIZZLE_128B, straight into the layout the MMA reads); the raw quantized
// bytes of each 128-row x 2-unit stage arrive by 1-D bulk copies, STAGES
// ahead of use.  Eight warps dequantize shared -> shared (raw bytes -> bf16
// swizzled rows), one warp issues the copies, one warp owns TMEM and the
// MMAs.  Requires rows % 128 == 0 (every bulk copy is a whole, 16-byte
// aligned span of 128 rows); other shapes use the v1 kernel above.

template <int TYPE>
struct Raw {
    // byte offsets inside a stage's raw region (unit h = 0/1 of the pair)
    static constexpr int Q = 0;                                        // q[h]
    static constexpr int QB = TYPE == HD_TYPE_Q8_0 ? 4096 : 2048;      // bytes per unit of q (128 rows)
    static constexpr int AUX = 2 * QB;                                 // Q5_0 qh[h] 512 B, Q6_K highs[h] 1 KB
    static constexpr int AUXB = TYPE == HD_TYPE_Q5_0 ? 512 : TYPE == HD_TYPE_Q6_K ? 1024 : 0;
    static constexpr int META = AUX + 2 * AUXB;                        // Q8_0/Q5_0 d[h] 256 B; Q4_K/Q6_K 2 KB per sb
    static constexpr int METAB = (TYPE == HD_TYPE_Q8_0 || TYPE == HD_TYPE_Q5_0) ? 256 : 2048;
    static constexpr int METAN = (TYPE == HD_TYPE_Q8_0 || TYPE == HD_TYPE_Q5_0) ? 2 : 1;
    static constexpr int DSB = META + METAN * METAB;                   // Q6_K d 256 B
    static constexpr int END = DSB + (TYPE == HD_TYPE_Q6_K ? 256 : 0);
    static constexpr int BYTES = (END + 1023) & ~1023;
};

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
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

// 32 values of unit u (pair half h) of row r from a stage's raw bytes.
template <int TYPE>
__device__ __forceinline__ void raw_values(const uint8_t *raw, int r, int h, int u, float (&v)[32]) {
    using R = Raw<TYPE>;
    if constexpr (TYPE == HD_TYPE_Q8_0) {
        const uint4 *p = (const uint4 *)(raw + R::Q + h * R::QB + r * 32);
        uint4 a = p[0], b = p[1];
        float d = h2f(*(const uint16_t *)(raw + R::META + h * R::METAB + r * 2));
        uint32_t wd[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            uint32_t x = wd[i] ^ 0x80808080u;
#pragma unroll
            for (int c = 0; c < 4; c++) v[4 * i + c] = (mag(x, c) - 8388736.0f) * d;
        }
    } else if constexpr (TYPE == HD_TYPE_Q5_0) {
        uint4 a = *(const uint4 *)(raw + R::Q + h * R::QB + r * 16);
        uint32_t qh = *(const uint32_t *)(raw + R::AUX + h * R::AUXB + r * 4);
        float d = h2f(*(const uint16_t *)(raw + R::META + h * R::METAB + r * 2));
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
        uint4 a = *(const uint4 *)(raw + R::Q + h * R::QB + r * 16);
        uint4 m = *(const uint4 *)(raw + R::META + r * 16);
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
        uint4 a = *(const uint4 *)(raw + R::Q + h * R::QB + r * 16);
        uint2 hb = *(const uint2 *)(raw + R::AUX + h * R::AUXB + r * 8);
        const int8_t *scp = (const int8_t *)(raw + R::META + r * 16);
        float d = h2f(*(const uint16_t *)(raw + R::DSB + r * 2));
        int s0 = 2 * (u & 7);
        float dl = d * (float)scp[s0], dh = d * (float)scp[s0 + 1];
        uint32_t wd[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int sh = 4 - 2 * i;
            uint32_t hx = sh >= 0 ? (hb.x << sh) : (hb.x >> -sh), hy = sh >= 0 ? (hb.y << sh) : (hb.y >> -sh);
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
struct TC2 {
    static constexpr int STAGES = BT >= 256 ? 3 : 4;
    static constexpr int XB = BT * 128;                       // bf16 activation tile
    static constexpr int STAGE = A_BYTES + XB + Raw<TYPE>::BYTES;
    static constexpr size_t SMEM = (size_t)STAGES * STAGE + 1024;
};

template <int TYPE, int BT>
__global__ void __launch_bounds__(320, 1) k_qgemm_tc2(WView w, const __grid_constant__ CUtensorMap tmx,
                                                     float *__restrict__ Y, int T, int N, int *flag) {
    using C = TC2<TYPE, BT>;
    using R = Raw<TYPE>;
    constexpr int ST = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t load_full[ST], a_full[ST], stage_empty[ST], acc_bar;
    __shared__ uint32_t tmem_base_sh;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * 128, t0 = blockIdx.y * BT;
    const int units = w.units, ksteps = (units + 1) / 2;
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; s++) {
            mbar_init(smem_u32(&load_full[s]), 1);
            mbar_init(smem_u32(&a_full[s]), 256);
            mbar_init(smem_u32(&stage_empty[s]), 1);
        }
        mbar_init(smem_u32(&acc_bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmx) : "memory");
    }
    if (warp == 9) {
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

    if (warp == 8) {
        // ---- copy engine driver
        if (lane == 0) {
            for (int ks = 0; ks < ksteps; ks++) {
                const int s = ks % ST, round = ks / ST;
                if (!mbar_wait(smem_u32(&stage_empty[s]), (round & 1) ^ 1, flag)) break;
                uint8_t *stg = base + s * C::STAGE;
                const uint32_t bar = smem_u32(&load_full[s]);
                const int ua = 2 * ks, ub = 2 * ks + 1;
                const bool has_b = ub < units;
                uint32_t bytes = C::XB + (has_b ? 2 : 1) * (R::QB + R::AUXB);
                if (R::METAN == 2) bytes += (has_b ? 2 : 1) * R::METAB;
                else bytes += R::METAB;
                if (TYPE == HD_TYPE_Q6_K) bytes += 256;
                mbar_expect_tx(bar, bytes);
                tma_2d(smem_u32(stg + A_BYTES), &tmx, ks * BK, t0, bar);
                uint8_t *raw = stg + A_BYTES + C::XB;
                for (int h = 0; h < (has_b ? 2 : 1); h++) {
                    const int u = ua + h;
                    const int64_t ur = (int64_t)u * w.rows + n0;
                    bulk_g2s(smem_u32(raw + R::Q + h * R::QB), w.q + ur * (R::QB / 128), R::QB, bar);
                    if (R::AUXB) bulk_g2s(smem_u32(raw + R::AUX + h * R::AUXB), w.aux + ur * (R::AUXB / 128), R::AUXB, bar);
                    if (R::METAN == 2) bulk_g2s(smem_u32(raw + R::META + h * R::METAB), w.meta + ur * 2, R::METAB, bar);
                }
                if (R::METAN == 1) {
                    const int64_t sr = (int64_t)(ua >> 3) * w.rows + n0;
                    bulk_g2s(smem_u32(raw + R::META), w.meta + sr * 16, R::METAB, bar);
                    if (TYPE == HD_TYPE_Q6_K) bulk_g2s(smem_u32(raw + R::DSB), w.dsb + sr, 256, bar);
                }
            }
        }
        __syncwarp();
    } else if (warp == 9) {
        // ---- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(BT);
            for (int ks = 0; ks < ksteps; ks++) {
                const int s = ks % ST, round = ks / ST;
                if (!mbar_wait(smem_u32(&a_full[s]), round & 1, flag)) break;
                tc_fence_after();
                uint8_t *stg = base + s * C::STAGE;
                const uint32_t a0 = smem_u32(stg), b0 = smem_u32(stg + A_BYTES);
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
                                 smem_u32(&stage_empty[s]))
                             : "memory");
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&acc_bar))
                         : "memory");
        }
        __syncwarp();
    } else {
        // ---- dequantizers: thread (row r, unit half h) of each stage
        const int r = threadIdx.x & 127, h = threadIdx.x >> 7;
        for (int ks = 0; ks < ksteps; ks++) {
            const int s = ks % ST, round = ks / ST;
            if (!mbar_wait(smem_u32(&load_full[s]), round & 1, flag)) break;
            uint8_t *stg = base + s * C::STAGE;
            const int u = 2 * ks + h;
            float v[32];
            if (u < units) {
                raw_values<TYPE>(stg + A_BYTES + C::XB, r, h, u, v);
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] = 0.f;
            }
            store_sw128(stg, r, 4 * h, v);
            fence_async_smem();
            mbar_arrive(smem_u32(&a_full[s]));
        }
    }

    // ---- epilogue: warps 0-7
    if (warp < 8) {
        const bool ok = mbar_wait(smem_u32(&acc_bar), 0, flag);
        tc_fence_after();
        const int q = warp & 3, half = warp >> 2;
        const int64_t n = n0 + 32 * q + lane;
        for (int c0 = half * (BT / 2); c0 < (half + 1) * (BT / 2); c0 += 16) {
            uint32_t rr[16];
            const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0;
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                "[%16];"
                : "=r"(rr[0]), "=r"(rr[1]), "=r"(rr[2]), "=r"(rr[3]), "=r"(rr[4]), "=r"(rr[5]), "=r"(rr[6]),
                  "=r"(rr[7]), "=r"(rr[8]), "=r"(rr[9]), "=r"(rr[10]), "=r"(rr[11]), "=r"(rr[12]), "=r"(rr[13]),
                  "=r"(rr[14]), "=r"(rr[15])
                : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (ok && n < N) {
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int t = t0 + c0 + j;
                    if (t < T) Y[(int64_t)t * N + n] = __uint_as_float(rr[j]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BT));
    }
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

template <int TYPE, int BT>
cudaError_t launch_tc2(hd_ctx *ctx, const hd_weight *w, const CUtensorMap &tm, float *Y, int T) {
    constexpr size_t smem = TC2<TYPE, BT>::SMEM;
    cudaError_t e = cudaFuncSetAttribute(k_qgemm_tc2<TYPE, BT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)(w->rows / 128), (unsigned)((T + BT - 1) / BT));
    return hd_launch(ctx, k_qgemm_tc2<TYPE, BT>, grid, dim3(320), smem, wview(w), tm, Y, T, (int)w->rows, ctx->flag);
}

}  // namespace

// Token tile: 128 (64 for short inputs), or 256 when that still gives two
// tiles per SM.  rows % 128 == 0 uses the streamed v2 kernel.
int hd_qgemm_tc(hd_ctx *ctx, const hd_weight *w, const float *X, float *Y, int T) {
    HD_REQUIRE(ctx, w->cols % 8 == 0, HD_E_SHAPE, "hd_qgemm: K must be a multiple of 8");
    const int64_t mt = (w->rows + 127) / 128;
    cudaError_t e = cudaSuccess;
    if (w->rows % 128 == 0 && getenv("HACEDLE_TC_V1") == nullptr) {
        // bf16 copy of the activations for the TMA
        const size_t need = (size_t)T * w->cols * sizeof(__nv_bfloat16);
        int rc = hd_ensure_hbuf(ctx, &ctx->xbf, &ctx->xbf_bytes, (need + 3) / 4 * 4);
        if (rc) return rc;
        const int64_t n = (int64_t)T * w->cols;
        e = hd_launch(ctx, k_to_bf16, dim3((unsigned)((n / 4 + 255) / 256 + 1)), dim3(256), 0, X,
                      (__nv_bfloat16 *)ctx->xbf, n);
        if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm (bf16 convert): %s", cudaGetErrorString(e));
        int bt = T <= 64 ? 64 : 128;
        if (T > 128 && mt * ((T + 255) / 256) >= 2 * ctx->sm_count) bt = 256;
        CUtensorMap tm;
        cuuint64_t dims[2] = {(cuuint64_t)w->cols, (cuuint64_t)T};
        cuuint64_t strides[1] = {(cuuint64_t)w->cols * 2};
        cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)bt};
        cuuint32_t estr[2] = {1, 1};
        EncodeTiledFn enc = encode_tiled();
        if (!enc) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm: cuTensorMapEncodeTiled is not available");
        CUresult cr = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ctx->xbf, dims, strides, box,
                                             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm: cuTensorMapEncodeTiled failed (%d)", (int)cr);
        HD_TYPE_SWITCH(w->type, TT, {
            if (bt == 64) e = launch_tc2<TT, 64>(ctx, w, tm, Y, T);
            else if (bt == 128) e = launch_tc2<TT, 128>(ctx, w, tm, Y, T);
            else e = launch_tc2<TT, 256>(ctx, w, tm, Y, T);
        });
        if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm (tcgen05 v2): %s", cudaGetErrorString(e));
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
