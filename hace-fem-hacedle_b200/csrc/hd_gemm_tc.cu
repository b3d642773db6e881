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

}  // namespace

// Token tile: the widest of 64/128/256 that still gives every SM a tile.
int hd_qgemm_tc(hd_ctx *ctx, const hd_weight *w, const float *X, float *Y, int T) {
    HD_REQUIRE(ctx, w->cols % 8 == 0, HD_E_SHAPE, "hd_qgemm: K must be a multiple of 8");
    const int64_t mt = (w->rows + 127) / 128;
    int bt = 64;
    if (T > 64 && mt * ((T + 127) / 128) >= ctx->sm_count) bt = 128;
    if (T > 128 && mt * ((T + 255) / 256) >= 2 * ctx->sm_count) bt = 256;
    cudaError_t e = cudaSuccess;
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
