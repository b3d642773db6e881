// hd_gemv_tc.cu -- decode Q-GEMV at batch 5..16 on the 5th-generation tensor
// cores: y[b] = W x[b] (+bias, +residual) for b < B, with the fp32-accumulate
// contract of the CUDA-core kernels (||y - y_ref||_inf <= 1e-5 ||y_ref||_inf).
//
// Exact products.  The A operand holds the weight's quant integers with the
// offset removed (at most 8 significant bits: exact in bf16), the B operand
// the activations split exactly into three bf16 parts x = x1 + x2 + x3 (8 + 8
// + 8 significand bits), so every product the tensor core forms is exact and
// only the fp32 accumulation rounds.  Each scale group of the weight (a
// 32-value unit; Q6_K: a 16-value half unit) has its own accumulator of 48
// TMEM columns; the epilogue thread of a weight row multiplies the group sums
// by the group's fp32 scale and adds them in group order (Q4_K also subtracts
// min * sum(x) over the unit).  The three parts sit side by side along N (48
// B rows: part p, batch row n at row 16p + n), so one MMA per 16 K values
// reads the weight slice once.
//
// Work split.  A CTA owns a tile of 128 weight rows and one of S contiguous
// ranges of its units (K parts); the S CTAs of a tile form a thread-block
// cluster.  Each thread issues its activation loads and then all of its
// weight loads at once, then decodes the weights into SWIZZLE_128B K-major
// bf16 tiles of 64 K values in shared memory in rounds of 4 units, each round
// released to the MMA thread by an mbarrier.
//
// Tensor memory: a ring of 8 group accumulators of 48 columns in two halves
// of 4, one round of 4 units per half (Q6_K: half a round).  The MMA thread
// commits a half when its groups are issued and the epilogue frees it once
// read, so that any number of groups fits.
//
// K reduction.  The 16 per-row sums of a CTA go to the CTA of the cluster
// that owns the row (the 128 rows split into S contiguous ranges) through
// distributed shared memory; after a cluster barrier the owner adds the S
// partial sums in K-part order and stores y.  Fixed orders throughout: the
// results are bitwise reproducible.
//
// Warp 0 allocates TMEM and one lane issues the MMAs (M = 128, N = 48, K =
// 16), a round at a time in straight-line code: for MMAs this short the issue
// rate of a single thread, not the tensor pipe, is the limit.  Warps 1-16
// load and decode (thread dt = t - 32: row dt % 128, unit slot dt / 128), and
// 1-4 are also the epilogue (warp w reads TMEM lanes 32 (w % 4).. = rows).
// Every mbarrier wait is bounded (HD_E_TIMEOUT in the context's flag word),
// every thread reaches both cluster barriers on every path, and TMEM is freed
// after the MMAs have completed.
#include <cstdlib>

#include "hd_internal.cuh"
#include "hd_tc.cuh"
#include "hd_units.cuh"

namespace {

constexpr int TV_DQW = 16;                        // load/decode warps: 128 rows x 4 unit slots
constexpr int TV_THREADS = (TV_DQW + 1) * 32;     // + the TMEM/MMA warp
constexpr int TV_MMA = 0;                         // the TMEM/MMA warp
constexpr int TV_UMAX = 16;                       // units per CTA (registers: 4 rounds)
constexpr int TV_ROUNDS = (TV_UMAX + 3) / 4;
constexpr int TV_SMAX = 16;                       // K parts (cluster size)
constexpr int TV_TCOLS = 512;                     // TMEM columns allocated (ring: 8 x 48)
constexpr int TV_N = 48;                          // MMA N: 3 activation parts x 16 batch rows
constexpr int TV_XI = (64 * TV_UMAX + TV_DQW * 32 - 1) / (TV_DQW * 32);   // activation items per thread
constexpr int TV_SMEM_MIN = 120 * 1024;           // one CTA per SM (the whole TMEM budget is safe)
constexpr int TV_SMEM_CAP = 226 * 1024;           // dynamic shared memory (1 KB left for the static part)

// Byte offsets from the 1024-aligned base: A tiles [ceil(U/2)][128 rows x
// 128 B], B tiles [ceil(U/2)][48 rows x 128 B], scales float2 [U][128], unit
// sums of x [U][16], partial sums [S][16][ceil(128/S)].
struct TvLayout {
    int b, scl, xs, red, total;
};
__host__ __device__ inline TvLayout tv_layout(int umax, int S) {
    TvLayout L;
    const int na = (umax + 1) / 2;
    L.b = na * 16384;
    L.scl = L.b + na * TV_N * 128;
    L.xs = L.scl + umax * 128 * 8;
    L.red = L.xs + umax * 16 * 4;
    L.total = L.red + S * 16 * ((128 + S - 1) / S) * 4;
    return L;
}

struct TvArgs {
    WView w;
    const float *x;         // [B][K]
    float *y;               // [B][ldy]
    const float *bias;      // [N] or null
    const float *residual;  // [B][ldy] or null
    int B, N, ldy, K;
    int S, umax;            // K parts, units of the largest part
    int *flag;
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ uint32_t bf2bits(__nv_bfloat162 h) { return *reinterpret_cast<uint32_t *>(&h); }

// (a, b) = hi + mid + lo exactly, each part packed as bf16 pairs: the
// remainder of a round to 8 significand bits is exact in fp32 and has at
// most 16 significant bits, the second remainder at most 8.
__device__ __forceinline__ void split3(float a, float b, uint32_t &w1, uint32_t &w2, uint32_t &w3) {
    const __nv_bfloat162 h1 = __floats2bfloat162_rn(a, b);
    const float ra = a - __low2float(h1), rb = b - __high2float(h1);
    const __nv_bfloat162 h2 = __floats2bfloat162_rn(ra, rb);
    const __nv_bfloat162 h3 = __floats2bfloat162_rn(ra - __low2float(h2), rb - __high2float(h2));
    w1 = bf2bits(h1);
    w2 = bf2bits(h2);
    w3 = bf2bits(h3);
}

template <int TYPE>
__global__ void __launch_bounds__(TV_THREADS, 1) k_qgemv_tc(TvArgs a) {
    constexpr bool Q6 = TYPE == HD_TYPE_Q6_K;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t a_full[TV_ROUNDS], t_full[2], t_empty[2], fin_bar;
    __shared__ uint32_t tmem_sh;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Parameters used only at the end, read now (their constant-cache misses
    // then overlap the prologue instead of delaying the stores).
    float *const yout = a.y;
    const float *const bias = a.bias, *const resid = a.residual;
    asm volatile("" ::"l"(yout), "l"(bias), "l"(resid));
    const int S = a.S;
    const int c = S > 1 ? (int)cluster_rank() : 0;   // K part
    const int tile = blockIdx.x / S;
    const int units = a.w.units, ub = units / S, ur = units % S;
    const int u0 = c * ub + min(c, ur), U = ub + (c < ur ? 1 : 0);
    const int R = (U + 3) >> 2;                      // decode rounds
    const int64_t row0 = (int64_t)tile * 128;
    const TvLayout L = tv_layout(a.umax, S);
    const int rpc = (128 + S - 1) / S;
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *At = base, *Bt = base + L.b;
    float2 *scl = (float2 *)(base + L.scl);
    float *xs = (float *)(base + L.xs), *red = (float *)(base + L.red);

    if (threadIdx.x == 0) {
        for (int i = 0; i < TV_ROUNDS; i++) mbar_init(smem_u32(&a_full[i]), TV_DQW * 32);
        for (int h = 0; h < 2; h++) {
            mbar_init(smem_u32(&t_full[h]), 1);
            mbar_init(smem_u32(&t_empty[h]), 128);
        }
        mbar_init(smem_u32(&fin_bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == TV_MMA) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_sh)),
                     "r"(TV_TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    // Load/decode thread dt (warps 1-16): row dt % 128, unit slot dt / 128.
    // Epilogue thread (warps 1-4): row re, TMEM lane quarter warp % 4.
    const bool dq = warp != TV_MMA;
    const int dt = (int)threadIdx.x - 32, r = dt & 127, js = dt >> 7;
    const bool epi = warp >= 1 && warp <= 4;
    const int re = 32 * (warp & 3) + lane;
    const int64_t row = row0 + r;
    const int items = 64 * U;   // activation items: (batch row n, unit u, quarter q) = 8 values
    URegs<TYPE> reg[TV_ROUNDS];
    float4 xv[TV_XI][2];

    // Every weight unit of the thread before the dependency wait (the
    // weights are not written by the previous kernel; their loads, pinned in
    // place, run while it finishes), then the activations after it.
#pragma unroll
    for (int i = 0; i < TV_ROUNDS; i++) {
        const int u = 4 * i + js;
        if (dq && u < U && row < a.N) load_unit<TYPE>(a.w, row, u0 + u, reg[i]);
        else zero_unit<TYPE>(reg[i]);
    }
    pdl_trigger();
    pdl_wait();
#pragma unroll
    for (int k = 0; k < TV_XI; k++) {
        const int i = k * TV_DQW * 32 + dt;
        xv[k][0] = xv[k][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (dq && i < items) {
            const int n = i / (4 * U), rem = i - n * 4 * U, u = rem >> 2, q = rem & 3;
            if (n < a.B) {
                const float4 *p = (const float4 *)(a.x + (int64_t)n * a.K + (int64_t)(u0 + u) * 32 + q * 8);
                xv[k][0] = __ldg(p);
                xv[k][1] = __ldg(p + 1);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_sh;
    if (S > 1) cluster_arrive_relaxed();   // waited on before the first remote store

    if (dq) {
        // ---- activations: item (n, u, q), three bf16 parts into B rows n,
        // 16 + n, 32 + n; rows n >= B are zeros.  Q4_K: unit sums of x, the
        // 4 quarters (consecutive lanes) added pairwise.
#pragma unroll
        for (int k = 0; k < TV_XI; k++) {
            const int i = k * TV_DQW * 32 + dt;
            const bool in = i < items;
            const int n = in ? i / (4 * U) : 0, rem = i - n * 4 * U, u = rem >> 2, q = rem & 3;
            const float4 v0 = xv[k][0], v1 = xv[k][1];
            if (in) {
                uint4 w[3];
                split3(v0.x, v0.y, w[0].x, w[1].x, w[2].x);
                split3(v0.z, v0.w, w[0].y, w[1].y, w[2].y);
                split3(v1.x, v1.y, w[0].z, w[1].z, w[2].z);
                split3(v1.z, v1.w, w[0].w, w[1].w, w[2].w);
                uint8_t *t = Bt + (u >> 1) * (TV_N * 128) + ((((u & 1) * 4 + q) ^ (n & 7)) * 16);
#pragma unroll
                for (int p = 0; p < 3; p++) *(uint4 *)(t + (16 * p + n) * 128) = w[p];
            }
            if constexpr (TYPE == HD_TYPE_Q4_K) {
                if (k * TV_DQW * 32 < items) {   // uniform over the warp
                    float ps = ((v0.x + v0.y) + (v0.z + v0.w)) + ((v1.x + v1.y) + (v1.z + v1.w));
                    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
                    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
                    if (in && q == 0) xs[u * 16 + n] = ps;
                }
            }
        }
        // ---- weights: round i decodes unit 4i + js of row r (exact
        // integers) into its A tile, and its scales.
#pragma unroll
        for (int i = 0; i < TV_ROUNDS; i++) {
            const int u = 4 * i + js;
            if (u < U) {
                float v[32];
#pragma unroll
                for (int wd = 0; wd < 8; wd++) {
                    float t4[4];
                    chunk_ints<TYPE>(reg[i], wd, t4);
#pragma unroll
                    for (int k = 0; k < 4; k++) v[4 * wd + k] = t4[k];
                }
                store_sw128(At + (u >> 1) * 16384, r, (u & 1) * 4, v);
                const URowScale s = unit_scale<TYPE>(reg[i], u0 + u);
                scl[u * 128 + r] = make_float2(s.s0, TYPE == HD_TYPE_Q4_K ? s.mn : s.s1);
            }
            fence_async_smem();
            mbar_arrive(smem_u32(&a_full[i]));
        }
        // scales and unit sums visible to the epilogue warps
        asm volatile("bar.sync 1, %0;" ::"n"(TV_DQW * 32) : "memory");
        // Warps 5-16 park on a hardware barrier until the epilogue is done,
        // leaving the issue slots to the MMA and epilogue warps.
        if (!epi) asm volatile("bar.sync 2, %0;" ::"n"(TV_DQW * 32) : "memory");
    } else if (lane == 0) {
        // ---- MMA issuer, a round (4 units) at a time in straight-line code.
        // Round rr's groups go to ring half rr & 1 (4 units; Q6_K: 8
        // half-unit groups, both halves).  Descriptors are advanced from
        // precomputed bases (start address in 16-byte units; no carry out of
        // the 14-bit field below 256 KB).
        constexpr uint32_t idesc = idesc_bf16(TV_N);
        const uint64_t adb = sw128_desc(smem_u32(At)), bdb = sw128_desc(smem_u32(Bt));
        for (int rr = 0; rr < R; rr++) {
            if (!mbar_wait(smem_u32(&a_full[rr]), 0, a.flag)) break;
            tc_fence_after();
            const uint64_t ar = adb + (uint64_t)(rr * 2048), br = bdb + (uint64_t)(rr * 2 * TV_N * 8);
            if constexpr (!Q6) {
                const int h = rr & 1;
                if (rr >= 2) {   // the epilogue has read this half
                    if (!mbar_wait(smem_u32(&t_empty[h]), ((rr >> 1) - 1) & 1, a.flag)) break;
                    tc_fence_after();
                }
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (4 * rr + j < U) {
                        const uint32_t d = tmem + (uint32_t)((4 * h + j) * TV_N);
                        const uint64_t ad = ar + (uint64_t)((j >> 1) * 1024 + (j & 1) * 4);
                        const uint64_t bd = br + (uint64_t)((j >> 1) * TV_N * 8 + (j & 1) * 4);
                        asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 0;" ::"r"(d), "l"(ad),
                                     "l"(bd), "r"(idesc));
                        asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 1;" ::"r"(d),
                                     "l"(ad + 2), "l"(bd + 2), "r"(idesc));
                    }
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_u32(&t_full[h]))
                             : "memory");
            } else {
                bool alive = true;
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    if (rr >= 1) {
                        if (!mbar_wait(smem_u32(&t_empty[h]), (rr - 1) & 1, a.flag)) {
                            alive = false;
                            break;
                        }
                        tc_fence_after();
                    }
#pragma unroll
                    for (int j = 0; j < 4; j++) {   // unit 4rr + 2h + j / 2, half j % 2
                        if (4 * rr + 2 * h + (j >> 1) < U) {
                            const uint32_t d = tmem + (uint32_t)((4 * h + j) * TV_N);
                            const uint64_t ad = ar + (uint64_t)(h * 1024 + (j >> 1) * 4 + (j & 1) * 2);
                            const uint64_t bd = br + (uint64_t)(h * TV_N * 8 + (j >> 1) * 4 + (j & 1) * 2);
                            asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 0;" ::"r"(d),
                                         "l"(ad), "l"(bd), "r"(idesc));
                        }
                    }
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                     smem_u32(&t_full[h]))
                                 : "memory");
                }
                if (!alive) break;
            }
        }
        // Completion of this commit covers every MMA issued above (also
        // after a timeout), before TMEM is freed.
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&fin_bar))
                     : "memory");
        mbar_wait_quiet(smem_u32(&fin_bar), 0);
    }
    __syncwarp();

    // ---- epilogue: weight row re (warps 1-4); a group's 48 columns are the
    // three parts' sums of the 16 batch rows, added (x1 + x2) + x3.  Group k
    // of ring half h holds unit 4rr + k (Q6_K: unit 4rr + 2h + k / 2, half
    // k % 2); half h of round rr is committed once.
    float acc[16];
#pragma unroll
    for (int b = 0; b < 16; b++) acc[b] = 0.f;
    const int64_t rowe = row0 + re;
    if (epi) {
        bool ok = true;
        for (int rr = 0; rr < R; rr++) {
#pragma unroll 1
            for (int h = 0; h < 2; h++) {
                if (!Q6 && h != (rr & 1)) continue;
                bool got = true;   // one lane per warp polls, with a short back-off
                if (lane == 0) got = ok && mbar_wait(smem_u32(&t_full[h]), (Q6 ? rr : rr >> 1) & 1, a.flag, 32);
                ok = __shfl_sync(0xffffffffu, got, 0);
                tc_fence_after();
                for (int k = 0; k < 4; k++) {
                    const int u = Q6 ? 4 * rr + 2 * h + (k >> 1) : 4 * rr + k;
                    if (u >= U) break;
                    uint32_t d0[16], d1[16], d2[16];
                    const uint32_t ta = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)((4 * h + k) * TV_N);
                    tmem_ld16_async(ta, d0);
                    tmem_ld16_async(ta + 16, d1);
                    tmem_ld16_async(ta + 32, d2);
                    tmem_wait_ld();
                    tmem_regs_ready(d0);
                    tmem_regs_ready(d1);
                    tmem_regs_ready(d2);
                    float d[16];
#pragma unroll
                    for (int b = 0; b < 16; b++)
                        d[b] = (__uint_as_float(d0[b]) + __uint_as_float(d1[b])) + __uint_as_float(d2[b]);
                    const float2 s = scl[u * 128 + re];
                    if constexpr (Q6) {
                        const float sc = (k & 1) ? s.y : s.x;
#pragma unroll
                        for (int b = 0; b < 16; b++) acc[b] = fmaf(sc, d[b], acc[b]);
                    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
#pragma unroll
                        for (int b = 0; b < 16; b++) acc[b] = fmaf(s.x, d[b], fmaf(-s.y, xs[u * 16 + b], acc[b]));
                    } else {
#pragma unroll
                        for (int b = 0; b < 16; b++) acc[b] = fmaf(s.x, d[b], acc[b]);
                    }
                }
                tc_fence_before();
                mbar_arrive(smem_u32(&t_empty[h]));
            }
        }
        asm volatile("bar.arrive 2, %0;" ::"n"(TV_DQW * 32) : "memory");
    }

    if (S == 1) {
        if (epi && rowe < a.N) {
#pragma unroll
            for (int b = 0; b < 16; b++) {
                if (b >= a.B) break;
                float o = acc[b];
                if (bias) o = o + bias[rowe];
                if (resid) o = resid[(int64_t)b * a.ldy + rowe] + o;
                yout[(int64_t)b * a.ldy + rowe] = o;
            }
        }
    } else {
        cluster_wait();   // every CTA of the cluster runs: its shared memory may be written
        if (epi) {
            const int own = (re * S) >> 7, lo = (own * 128 + S - 1) / S;
            const uint32_t dst = map_rank(smem_u32(red), (uint32_t)own) + (uint32_t)((c * 16 * rpc + (re - lo)) * 4);
#pragma unroll
            for (int b = 0; b < 16; b++) st_cluster(dst + (uint32_t)(b * rpc * 4), acc[b]);
        }
        cluster_arrive_release();
        cluster_wait();
        const int lo = (c * 128 + S - 1) / S, hi = ((c + 1) * 128 + S - 1) / S, nr = hi - lo;
        for (int i = threadIdx.x; i < nr * a.B; i += TV_THREADS) {
            const int b = i / nr, rl = i - b * nr;
            const int64_t rw = row0 + lo + rl;
            if (rw >= a.N) continue;
            float o = red[b * rpc + rl];
            for (int cc = 1; cc < S; cc++) o += red[(cc * 16 + b) * rpc + rl];
            if (bias) o = o + bias[rw];
            if (resid) o = resid[(int64_t)b * a.ldy + rw] + o;
            yout[(int64_t)b * a.ldy + rw] = o;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == TV_MMA) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TV_TCOLS));
    }
}

int env_int(const char *name, int dflt) {
    const char *v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}

// Clusters of S CTAs that fit on the device at once (0: none), per device,
// type and S, asked once; the first ask on a device also sets the kernel's
// attributes there (function attributes are per device).
constexpr int TV_MAX_DEVICES = 64;
template <int TYPE>
int max_clusters(int device, int S) {
    static int known[TV_MAX_DEVICES][TV_SMAX + 1] = {};   // value + 1; 0 = not asked yet
    if (device < 0 || device >= TV_MAX_DEVICES) return 0;
    if (known[device][S]) return known[device][S] - 1;
    cudaFuncSetAttribute(k_qgemv_tc<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, TV_SMEM_CAP);
    cudaFuncSetAttribute(k_qgemv_tc<TYPE>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S);
    cfg.blockDim = dim3(TV_THREADS);
    cfg.dynamicSmemBytes = TV_SMEM_CAP;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, k_qgemv_tc<TYPE>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    known[device][S] = n + 1;
    return n;
}

template <int TYPE>
int run_tc(hd_ctx *ctx, const hd_weight *w, const float *x, float *y, int B, const float *bias, const float *residual,
           bool *done) {
    const int N = (int)w->rows, units = w->units, ntiles = (N + 127) / 128;
    if (ntiles > ctx->sm_count) return HD_OK;
    // K parts: as many as fill the SMs (at most 16), at least enough that a
    // part's units fit in the registers of the decode threads.
    const int smin = (units + TV_UMAX - 1) / TV_UMAX;
    int S = ctx->sm_count / ntiles;
    S = S > TV_SMAX ? TV_SMAX : S;
    S = S > units ? units : S;
    const int s_env = env_int("HACEDLE_GEMV_TC_S", 0);
    if (s_env >= 1 && s_env <= TV_SMAX && s_env <= units) S = s_env;
    while (S >= smin && S > 1 && max_clusters<TYPE>(ctx->device, S) < 1) S--;
    if (S < smin || S < 1) return HD_OK;
    if (max_clusters<TYPE>(ctx->device, 1) < 1) return HD_OK;   // also sets the attributes on this device
    TvArgs a;
    a.w = wview(w);
    a.x = x;
    a.y = y;
    a.bias = bias;
    a.residual = residual;
    a.B = B;
    a.N = N;
    a.ldy = N;
    a.K = (int)w->cols;
    a.S = S;
    a.umax = (units + S - 1) / S;
    a.flag = ctx->flag;
    const TvLayout L = tv_layout(a.umax, S);
    size_t smem = (size_t)L.total + 1024;
    if (smem < (size_t)TV_SMEM_MIN) smem = TV_SMEM_MIN;
    if (smem > (size_t)TV_SMEM_CAP) return HD_OK;
    cudaError_t e = S > 1 ? hd_launch_cluster(ctx, k_qgemv_tc<TYPE>, dim3(ntiles * S), dim3(TV_THREADS), smem, S, a)
                          : hd_launch(ctx, k_qgemv_tc<TYPE>, dim3(ntiles), dim3(TV_THREADS), smem, a);
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_qgemv (tensor cores): %s", cudaGetErrorString(e));
    *done = true;
    return HD_OK;
}

}  // namespace

// Batch 5..16 by default (HACEDLE_GEMV_TC_MIN_B; HACEDLE_GEMV_TC=0 turns the
// path off): at batch <= 4 the CUDA-core kernel is as fast on B200.
int hd_qgemv_tc(hd_ctx *ctx, const hd_weight *w, const float *x, float *y, int B, const float *bias,
                const float *residual, bool *done) {
    *done = false;
    if (env_int("HACEDLE_GEMV_TC", 1) == 0) return HD_OK;
    if (B < env_int("HACEDLE_GEMV_TC_MIN_B", 5) || B > 16) return HD_OK;
    int rc = HD_OK;
    HD_TYPE_SWITCH(w->type, T, rc = run_tc<T>(ctx, w, x, y, B, bias, residual, done));
    return rc;
}
