// hd_gemv_stream.cu -- decode Q-GEMV at batch 1..16 on the tensor cores,
// streamed: y[b] = W x[b] (+bias, +residual), fp32 accumulation.
//
// Why.  A 38-150 MB weight is a bandwidth problem, and two things kept the
// earlier kernels from it: the walk (warps reading 512-byte pieces at a
// stride of rows x 16 bytes, which DRAM serves far below its streaming rate)
// and, for the 4-bit types, the CUDA-core unpacking (about four instructions
// per weight, the whole issue budget of an SM at 0.7 of HBM).  Here:
//  - a CTA owns 128 consecutive rows (one row block; persistent over blocks
//    when there are more blocks than SMs), and every CTA walks the units of
//    K in the same order, 8 units (one K-quant super-block) per stage, so
//    that at any moment the grid reads the same few units of all rows: one
//    near-contiguous stream through the unit-major layout;
//  - a stage (per unit a 2-4 KB contiguous run of quants, its side bytes
//    and scales, then the super-block headers) arrives by bulk copies that
//    the copy warps issue, taking the steps in turn, into a ring of NS
//    stages, each completing on the stage's mbarrier; the consumer warps
//    release a stage through a second mbarrier, so no CTA-wide barrier paces
//    the walk (the first NS stages go out before griddepcontrol.wait);
//  - the products run on the tensor cores (mma.sync m16n8k16, exact fp16
//    quants against x split into fp16 hi/lo, as hd_gemv_small.cu; batch
//    5..16 in two or four MMA column blocks sharing each unpacked
//    fragment); the unpacking, not the MMAs, sets the consumers' pace
//    (~185 warp instructions per 32-row unit at batch 1);
//  - when the row blocks alone leave SMs idle, the K parts of a block form a
//    thread-block cluster whose partial sums meet in the first CTA through
//    distributed shared memory.
// Consumer warp w takes the 32-row tile w % 4 of the block and units
// 2 (w / 4), 2 (w / 4) + 1 of every stage; the four quarters meet in shared memory at
// the end of a block, in a fixed order (as the K parts), so results are
// bitwise reproducible.
#include <cstdlib>

#include "hd_internal.cuh"
#include "hd_mma.cuh"

namespace {

constexpr int ST_CWARPS = 16;    // consumers: 4 tiles of 32 rows x 4 unit quarters of a stage
constexpr int ST_CTHREADS = 32 * ST_CWARPS;
constexpr int ST_CPW = 4;        // copy warps (one warp's bulk copies are processed one after another)
constexpr int ST_THREADS = ST_CTHREADS + 32 * ST_CPW;
constexpr int ST_UG = 8;          // units per stage
constexpr int ST_RB = 128;        // rows per CTA (4 tiles of 32)
constexpr int ST_SMAX = 8;        // K parts (cluster size), at most
constexpr int ST_NSMAX = 10;      // stages, at most
constexpr int ST_SMEM = 226 * 1024;   // dynamic; the copy warps keep a few static bytes
constexpr int ST_MAX_DEV = 64;

// Per unit of a 128-row block in a stage: quants (rows x 16 bytes; Q8_0 32),
// then Q5_0's fifth bits (4 bytes per row) or Q6_K's high bits (8), then
// Q8_0/Q5_0 fp16 scales (2 bytes per row); after the units, the K-quant
// super-block header (16 bytes per row) and Q6_K's super-block scale (2).
template <int TYPE>
struct St;
template <>
struct St<HD_TYPE_Q8_0> { static constexpr int QB = 4096, SIDE = 0, DB = 256, HDR = 0, DSB = 0, NSC = 1; };
template <>
struct St<HD_TYPE_Q5_0> { static constexpr int QB = 2048, SIDE = 512, DB = 256, HDR = 0, DSB = 0, NSC = 1; };
template <>
struct St<HD_TYPE_Q4_K> { static constexpr int QB = 2048, SIDE = 0, DB = 0, HDR = 2048, DSB = 0, NSC = 2; };
template <>
struct St<HD_TYPE_Q6_K> { static constexpr int QB = 2048, SIDE = 1024, DB = 0, HDR = 2048, DSB = 256, NSC = 2; };

template <int TYPE>
struct StL {
    using P = St<TYPE>;
    static constexpr int USTR = P::QB + P::SIDE + P::DB;
    static constexpr int STAGE = (ST_UG * USTR + P::HDR + P::DSB + 127) / 128 * 128;
};

struct StArgs {
    WView w;
    const float *x;         // [B][K]
    float *y;               // [B][N]
    const float *bias;      // [N] or null
    const float *residual;  // [B][N] or null (may be y)
    int B, N, K, units;
    int S;                  // K parts (cluster size)
    int NS;                 // stages
    int upc;                // units per K part, at most
    int nblk;               // row blocks
    int *flag;              // the context's error word (HD_E_TIMEOUT from a wait)
};

// Shared memory (byte offsets, all multiples of 128):
//   x fragments [upc][8 NB] uint4; x scales [upc][NB] float2;
//   row sums [4 quarters][4 tiles][NB][32] float; K-part sums [S][NB][128]
//   (batch 8 and 16: over the stage ring once it is idle);
//   per-warp scales [16][2 units][NSC][32] float; NS stages.
struct StLayout {
    int img, xs, red, part, scl, bar, stage, total;
};
template <int TYPE>
__host__ __device__ inline StLayout st_layout(int NB, int upc, int S, int NS) {
    StLayout L;
    L.img = 0;
    L.xs = L.img + upc * 8 * NB * 16;
    L.red = L.xs + ((upc * NB * 8 + 127) & ~127);
    L.part = L.red + 4 * 4 * NB * 32 * 4;   // batch <= 4; above, over the stage ring
    const int psum = S > 1 ? S * NB * ST_RB * 4 : 0;
    L.scl = L.part + (NB <= 4 ? (psum + 127) / 128 * 128 : 0);
    L.bar = L.scl + ST_CWARPS * 2 * St<TYPE>::NSC * 32 * 4;
    L.stage = L.bar + 2 * 8 * ST_NSMAX + 96;   // full[NS], empty[NS] (stages stay 128-aligned)
    // Batch 8 and 16: the K-part sums (S > 1: one block per CTA, summed
    // after every CTA of the cluster has consumed its last stage) reuse the
    // stage ring.
    const int ring = NS * StL<TYPE>::STAGE;
    if (NB > 4) L.part = L.stage;
    L.total = L.stage + (NB > 4 && psum > ring ? psum : ring);
    return L;
}

// mbarriers and bulk copies (waits bounded by time: HD_E_TIMEOUT in the
// context's flag word, and every other waiter gives up once it is set)
constexpr long long ST_SPIN = 2000000000;   // clock64 cycles (~1 s)
__device__ __forceinline__ void st_bar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void st_arrive(uint32_t bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void st_expect(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool st_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool st_wait(uint32_t bar, uint32_t parity, int *flag, unsigned sleep_ns = 0) {
    if (st_try(bar, parity)) return true;
    const long long t0 = clock64();
    for (unsigned it = 1;; it++) {
        if (sleep_ns) __nanosleep(sleep_ns);
        if (st_try(bar, parity)) return true;
        if ((it & 63) == 0) {
            if (*(volatile int *)flag) return false;
            if (clock64() - t0 > ST_SPIN) {
                atomicExch(flag, HD_E_TIMEOUT);
                return false;
            }
        }
    }
}
__device__ __forceinline__ void st_wait_quiet(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!st_try(bar, parity))
        if (clock64() - t0 > ST_SPIN) return;
}
// global -> this CTA's shared memory, completing on an mbarrier of this CTA
__device__ __forceinline__ void st_bulk(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// the 512 consumer threads (named barrier 1; the copy warp does not take part)
__device__ __forceinline__ void st_csync() { asm volatile("bar.sync 1, %0;" ::"n"(ST_CTHREADS) : "memory"); }

template <int TYPE, int NB>
__global__ void __launch_bounds__(ST_THREADS, 1) k_qgemv_st(StArgs a) {
    using P = St<TYPE>;
    constexpr int NBLK = NB <= 4 ? 1 : NB / 4;   // MMA n-blocks of 8 columns (hi, lo of 4 batch rows)
    constexpr int USTR = StL<TYPE>::USTR, STAGE = StL<TYPE>::STAGE;
    constexpr int ROWB = P::QB / ST_RB;   // quant bytes per row
    constexpr int SR = P::SIDE / ST_RB;   // side bytes per row
    extern __shared__ __align__(128) unsigned char st_sm[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3, tw = wib & 3, uh = (wib >> 2) & 3;
    const int S = a.S, NS = a.NS;
    const int part = S > 1 ? (int)mm_cluster_rank() : 0;
    const int rows = a.N, units = a.units;
    // K part: whole stages (super-blocks) of units
    const int ngtot = (units + ST_UG - 1) / ST_UG;
    const int g0 = part * ngtot / S, g1 = (part + 1) * ngtot / S;
    const int cu0 = g0 * ST_UG, cu1 = min(units, g1 * ST_UG), nu = cu1 - cu0, ngroups = g1 - g0;
    const StLayout L = st_layout<TYPE>(NB, a.upc, S, NS);
    uint4 *img = (uint4 *)(st_sm + L.img);
    float2 *xs2 = (float2 *)(st_sm + L.xs);
    float *red = (float *)(st_sm + L.red);
    float *scl = (float *)(st_sm + L.scl) + (wib & 15) * (2 * P::NSC * 32);
    unsigned char *stg = st_sm + L.stage;
    const uint32_t stg_s = smem_u32(stg);
    const uint32_t full0 = smem_u32(st_sm + L.bar), empty0 = full0 + 8 * ST_NSMAX;
    const WView w = a.w;
    const int gi_lane = (lane & 7) * 4 + (lane >> 3);

    // Items of this CTA: row blocks blk0, blk0 + bstride, ...; steps = items x groups.
    const int blk0 = blockIdx.x / S, bstride = gridDim.x / S;
    const int nitems = blk0 < a.nblk ? (a.nblk - blk0 + bstride - 1) / bstride : 0;
    const int nsteps = nitems * ngroups;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; i++) {
            st_bar_init(full0 + 8 * i, 1);
            st_bar_init(empty0 + 8 * i, ST_CTHREADS);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // Cluster barrier, first phase: at batch <= 4 every thread arrives here
    // and waits before its first remote store (the partner runs); above, the
    // K-part sums overwrite the first CTA's stage ring, so every thread
    // arrives only after its CTA has consumed its last stage.
    constexpr bool LATE = NB > 4;
    if (S > 1 && !LATE) mm_cluster_arrive_relaxed();

    if (wib >= ST_CWARPS) {
        // ---- copy warps: warp c takes steps c, c + ST_CPW, ... (the copies
        // of one warp are processed one after another, those of different
        // warps overlap): step j into stage j % NS once the consumers have
        // released the stage's previous use; lane c issues copy c of the step
        // (per unit the quants, side bytes and scales of the block's rows,
        // each one contiguous run; then the super-block header and scale).
        // Weights do not depend on the previous kernel: the first NS stages
        // go out before the consumers' dependency wait.
        // At most NS copy warps take part: a warp at step j has issued step
        // j - ncw, after the consumers released step j - ncw - NS, so the
        // release of step j - 2 NS it waits beyond is done and the parity of
        // the phase it waits for cannot alias an older one (with more warps
        // than stages it could).
        constexpr int CPU = 1 + (P::SIDE > 0) + (P::DB > 0);
        const int cw = wib - ST_CWARPS, ncw = NS < ST_CPW ? NS : ST_CPW;
        __shared__ int st_issued[ST_CPW];   // per copy warp: one past its last issued step
        bool ok = true;
        int issued = 0;
        // step j = cw + i ncw as (stage, use of the stage, item, group),
        // advanced by additions (no division per step)
        int sidx = cw, use = 0, it = 0, gr = cw;
        while (gr >= ngroups) { gr -= ngroups; it++; }
        for (int j = cw; j < nsteps && ok && cw < ncw; j += ncw) {
            if (j >= NS) {
                if (lane == 0) ok = st_wait(empty0 + 8 * sidx, (use - 1) & 1, a.flag, 200);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
            }
            const int r0 = (blk0 + it * bstride) * ST_RB, nr = min(ST_RB, rows - r0);
            const int u0 = cu0 + gr * ST_UG, nk = min(ST_UG, cu1 - u0);
            const uint32_t s0 = stg_s + (uint32_t)sidx * STAGE, bar = full0 + 8 * sidx;
            const uint32_t tx = (uint32_t)nr * ((uint32_t)nk * (ROWB + SR + (P::DB > 0 ? 2 : 0)) +
                                                (P::HDR > 0 ? 16 : 0) + (P::DSB > 0 ? 2 : 0));
            if (lane == 0) st_expect(bar, tx);
            __syncwarp();
            const int ncp = nk * CPU + (P::HDR > 0) + (P::DSB > 0);
            if (lane < ncp) {
                if (lane < nk * CPU) {
                    const int k = lane / CPU, c = lane - k * CPU;
                    const uint32_t ur = (uint32_t)(u0 + k) * (uint32_t)rows + (uint32_t)r0;
                    const uint32_t dst = s0 + k * USTR;
                    if (c == 0) st_bulk(dst, w.q + (size_t)ur * ROWB, nr * ROWB, bar);
                    else if (P::SIDE > 0 && c == 1) st_bulk(dst + P::QB, w.aux + (size_t)ur * SR, nr * SR, bar);
                    else st_bulk(dst + P::QB + P::SIDE, w.meta + (size_t)ur * 2, nr * 2, bar);
                } else {
                    const uint32_t sr = (uint32_t)(u0 >> 3) * (uint32_t)rows + (uint32_t)r0;
                    const uint32_t dst = s0 + ST_UG * USTR;
                    if (lane == nk * CPU && P::HDR > 0) st_bulk(dst, w.meta + (size_t)sr * 16, nr * 16, bar);
                    else st_bulk(dst + P::HDR, (const unsigned char *)w.dsb + (size_t)sr * 2, nr * 2, bar);
                }
            }
            issued = j + 1;
            sidx += ncw;
            if (sidx >= NS) { sidx -= NS; use++; }
            gr += ncw;
            while (gr >= ngroups) { gr -= ngroups; it++; }
        }
        // The CTA exits only after its copies have landed (also after an
        // error): each warp waits for those of its steps that are the latest
        // use of their stage (step j + NS not issued; a step is issued iff it
        // lies below its warp's count).
        if (lane == 0) st_issued[cw] = issued;
        asm volatile("bar.sync 2, %0;" ::"n"(32 * ST_CPW) : "memory");
        if (lane == 0)
            for (int j = cw; j < issued; j += ncw)
                if (j + NS >= st_issued[(j + NS) % ncw]) st_wait_quiet(full0 + 8 * (j % NS), (j / NS) & 1);
        __syncwarp();
        if (S > 1) {   // the cluster barrier counts every thread: the consumers' two phases
            if (LATE) mm_cluster_arrive_release();
            mm_cluster_wait();
            mm_cluster_arrive_release();
            mm_cluster_wait();
        }
        return;
    }

    pdl_trigger();
    pdl_wait();

    // x fragments of the part's units (as hd_gemv_small.cu): task (unit l,
    // batch row b, quarter q), 8 lanes per (l, b); loads of up to 8 tasks of
    // a thread issued before the first use.
    {
        constexpr int XR = 8;
        const int ntask = nu * NB * 8;
        for (int base = 0; base < ntask; base += XR * ST_CTHREADS) {
            float4 v[XR];
#pragma unroll
            for (int r = 0; r < XR; r++) {
                const int task = base + r * ST_CTHREADS + threadIdx.x;
                const int q = task & 7, lb = task >> 3, l = lb / NB, b = lb - l * NB;
                v[r] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (task < ntask && b < a.B)
                    v[r] = __ldg((const float4 *)(a.x + (int64_t)b * a.K + (int64_t)(cu0 + l) * 32) + q);
            }
#pragma unroll
            for (int r = 0; r < XR; r++) {
                if (base + r * ST_CTHREADS >= ntask) break;   // warp-uniform
                const int task = base + r * ST_CTHREADS + threadIdx.x;
                const bool live = task < ntask;
                const int q = task & 7, lb = task >> 3, l = lb / NB, b = lb - l * NB;
                const float4 xv4 = v[r];
                float mx = fmaxf(fmaxf(fabsf(xv4.x), fabsf(xv4.y)), fmaxf(fabsf(xv4.z), fabsf(xv4.w)));
                float sm = (xv4.x + xv4.y) + (xv4.z + xv4.w);
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) {
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    sm += __shfl_xor_sync(0xffffffffu, sm, o);
                }
                int s = 0;
                if (mx > 0.f) {
                    const int e = (int)((__float_as_uint(mx) >> 23) & 255) - 127;
                    s = 14 - e;
                    s = s < -100 ? -100 : s > 100 ? 100 : s;
                }
                const float up = __int_as_float((127 + s) << 23);
                const float xv[4] = {xv4.x * up, xv4.y * up, xv4.z * up, xv4.w * up};
                __half hi[4], lo[4];
#pragma unroll
                for (int jj = 0; jj < 4; jj++) {
                    hi[jj] = __float2half_rn(xv[jj]);
                    lo[jj] = __float2half_rn(xv[jj] - __half2float(hi[jj]));
                }
                if (live) {
                    uint2 *img2 = (uint2 *)(img + l * 8 * NB);
                    const int tt = q & 3, half = q >> 2;
                    img2[((2 * b) * 4 + tt) * 2 + half] = make_uint2(pack_h2(hi[0], hi[2]), pack_h2(hi[1], hi[3]));
                    img2[((2 * b + 1) * 4 + tt) * 2 + half] = make_uint2(pack_h2(lo[0], lo[2]), pack_h2(lo[1], lo[3]));
                    if (q == 0) xs2[l * NB + b] = make_float2(__int_as_float((127 - s) << 23), sm);
                }
            }
        }
    }
    st_csync();

    float *pt = (float *)(st_sm + L.part);
    float acc[NBLK][4];   // rows g + 8 i of tile tw, batch row 4 nb + t
#pragma unroll
    for (int nb = 0; nb < NBLK; nb++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[nb][i] = 0.f;
    bool ok = true;
    int sidx = 0, use = 0, it = 0, gr = 0;   // step j as (stage, use of the stage, item, group)
    for (int j = 0; j < nsteps; j++) {
        ok = ok && st_wait(full0 + 8 * sidx, use & 1, a.flag);
        __syncwarp();   // this warp's reads of its scale slots of step j - 1 are done
        const int u0 = cu0 + gr * ST_UG, nk = min(ST_UG, cu1 - u0);
        const unsigned char *st = stg + sidx * STAGE;
        const uint32_t st_s = stg_s + (uint32_t)sidx * STAGE;
        const int row_l = tw * 32 + lane;   // this lane's row in the block (scale decode)

        if (ok) {
            // scales of this warp's units (lane = row), (g, i) slot order.
            // A unit past the K part's end (the last stage of a part) is
            // computed from the stage's stale bytes, which stay in bounds,
            // with x and the scales zeroed: no branch, so that the two
            // units' chains interleave.
#pragma unroll
            for (int k4 = 0; k4 < 2; k4++) {
                const int k = uh * 2 + k4;
                {
                    const int u = u0 + k;
                    const unsigned char *su = st + k * USTR;
                    if constexpr (TYPE == HD_TYPE_Q5_0 || TYPE == HD_TYPE_Q8_0) {
                        scl[k4 * 32 + gi_lane] = h2f(*(const uint16_t *)(su + P::QB + P::SIDE + row_l * 2));
                    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
                        const uint4 hd = *(const uint4 *)(st + ST_UG * USTR + row_l * 16);
                        const float d = h2f((uint16_t)(hd.x & 0xFFFF)), dmin = h2f((uint16_t)(hd.x >> 16));
                        int sc, m;
                        q4k_sm_regs(u & 7, hd.y, hd.z, hd.w, sc, m);
                        scl[(k4 * 2) * 32 + gi_lane] = __fmul_rn(d, (float)sc);
                        scl[(k4 * 2 + 1) * 32 + gi_lane] = __fmul_rn(dmin, (float)m);
                    } else {
                        const int8_t *sc = (const int8_t *)(st + ST_UG * USTR + row_l * 16);
                        const float d = h2f(*(const uint16_t *)(st + ST_UG * USTR + P::HDR + row_l * 2));
                        const int s0 = 2 * (u & 7);
                        scl[(k4 * 2) * 32 + gi_lane] = __fmul_rn(d, (float)sc[s0]);
                        scl[(k4 * 2 + 1) * 32 + gi_lane] = __fmul_rn(d, (float)sc[s0 + 1]);
                    }
                }
            }
            __syncwarp();
#pragma unroll
            for (int k4 = 0; k4 < 2; k4++) {
                const int k = uh * 2 + k4;
                const bool live = k < nk;
                {
                    const int l = live ? u0 + k - cu0 : 0;
                    const uint32_t su_s = st_s + k * USTR;
                    const unsigned char *su = st + k * USTR;
                    uint32_t r[4], r2[4];
                    if constexpr (TYPE == HD_TYPE_Q8_0) {
                        // rows of 32 bytes: the quant halves are 16 bytes apart
                        ldsm4(su_s + tw * 1024 + lane * 32, r);
                        ldsm4(su_s + tw * 1024 + lane * 32 + 16, r2);
                    } else {
                        ldsm4(su_s + tw * 512 + lane * 16, r);
                    }
                    uint32_t ex[4][2];
#pragma unroll
                    for (int i = 0; i < 4; i++) ex[i][0] = ex[i][1] = 0;
                    if constexpr (TYPE == HD_TYPE_Q5_0) {
                        const uint32_t *qh = (const uint32_t *)(su + P::QB) + tw * 32 + g;
#pragma unroll
                        for (int i = 0; i < 4; i++) ex[i][0] = qh[8 * i] >> t;
                    } else if constexpr (TYPE == HD_TYPE_Q6_K) {
                        const uint2 *hb = (const uint2 *)(su + P::QB) + tw * 32 + g;
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const uint2 h = hb[8 * i];
                            ex[i][0] = h.x >> (2 * t);
                            ex[i][1] = h.y >> (2 * t);
                        }
                    }
                    float4 d4 = *(const float4 *)(scl + (k4 * P::NSC) * 32 + g * 4);
                    float4 e4 = make_float4(0.f, 0.f, 0.f, 0.f);
                    if constexpr (P::NSC == 2) e4 = *(const float4 *)(scl + (k4 * 2 + 1) * 32 + g * 4);
                    if (!live) d4 = e4 = make_float4(0.f, 0.f, 0.f, 0.f);
                    const float dv[4] = {d4.x, d4.y, d4.z, d4.w}, ev[4] = {e4.x, e4.y, e4.z, e4.w};
                    // n-block nb holds batch rows 4 nb .. 4 nb + 3 (hi and lo
                    // columns); this lane's accumulator column is batch row 4 nb + t
                    uint4 bf[NBLK];
                    float2 ps[NBLK];
#pragma unroll
                    for (int nb = 0; nb < NBLK; nb++) {
                        bf[nb] = make_uint4(0, 0, 0, 0);
                        if (live && (NB >= 4 || g < 2 * NB)) bf[nb] = img[l * 8 * NB + nb * 32 + lane];
                        ps[nb] = live && 4 * nb + t < NB ? xs2[l * NB + 4 * nb + t] : make_float2(0.f, 0.f);
                    }
                    const float z[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int m = 0; m < 2; m++) {
                        uint32_t A0[4], A1[4];   // rows g + 16 m, g + 8 + 16 m
                        unpack_word<TYPE>(r[2 * m], ex[2 * m][0], ex[2 * m][1], A0);
                        unpack_word<TYPE>(r[2 * m + 1], ex[2 * m + 1][0], ex[2 * m + 1][1], A1);
                        uint32_t B0[4], B1[4];
                        if constexpr (TYPE == HD_TYPE_Q8_0) {
                            unpack_word<TYPE>(r2[2 * m], 0, 0, B0);
                            unpack_word<TYPE>(r2[2 * m + 1], 0, 0, B1);
                        }
#pragma unroll
                        for (int nb = 0; nb < NBLK; nb++) {
                            float e0[4], e1[4];
                            mma16816(e0, A0[0], A1[0], A0[1], A1[1], bf[nb].x, bf[nb].y, z);
                            if constexpr (TYPE == HD_TYPE_Q8_0) {
                                mma16816(e0, B0[0], B1[0], B0[1], B1[1], bf[nb].z, bf[nb].w, e0);
                            } else if constexpr (TYPE == HD_TYPE_Q6_K) {
                                mma16816(e1, A0[2], A1[2], A0[3], A1[3], bf[nb].z, bf[nb].w, z);
                            } else {
                                mma16816(e0, A0[2], A1[2], A0[3], A1[3], bf[nb].z, bf[nb].w, e0);
                            }
#pragma unroll
                            for (int h = 0; h < 2; h++) {
                                const int i = 2 * m + h;
                                float &ac = acc[nb][i];
                                ac = fmaf(dv[i] * ps[nb].x, e0[2 * h] + e0[2 * h + 1], ac);
                                if constexpr (TYPE == HD_TYPE_Q6_K)
                                    ac = fmaf(ev[i] * ps[nb].x, e1[2 * h] + e1[2 * h + 1], ac);
                                if constexpr (TYPE == HD_TYPE_Q4_K) ac = fmaf(-ev[i], ps[nb].y, ac);
                            }
                        }
                    }
                }
            }
        }
        st_arrive(empty0 + 8 * sidx);   // this thread's reads of the stage are done

        if (gr == ngroups - 1) {
            // ---- the block is done: its row sums (unit quarters added in
            // order), across the K parts of the cluster, then stored
            const int r0 = (blk0 + it * bstride) * ST_RB;
#pragma unroll
            for (int nb = 0; nb < NBLK; nb++) {
                if (4 * nb + t < NB) {
#pragma unroll
                    for (int i = 0; i < 4; i++)   // uh: quarter
                        red[((uh * 4 + tw) * NB + 4 * nb + t) * 32 + g + 8 * i] = acc[nb][i];
                }
#pragma unroll
                for (int i = 0; i < 4; i++) acc[nb][i] = 0.f;
            }
            st_csync();
            const int ntask = ST_RB * a.B;
            if (S == 1) {
                if (ok) {
                    for (int task = threadIdx.x; task < ntask; task += ST_CTHREADS) {
                        const int rr = task & (ST_RB - 1), b = task >> 7, row = r0 + rr;
                        if (row < rows) {
                            const int ti = rr >> 5, ri = rr & 31;
                            float o = (red[((0 * 4 + ti) * NB + b) * 32 + ri] + red[((1 * 4 + ti) * NB + b) * 32 + ri]) +
                                      (red[((2 * 4 + ti) * NB + b) * 32 + ri] + red[((3 * 4 + ti) * NB + b) * 32 + ri]);
                            if (a.bias) o = o + a.bias[row];
                            if (a.residual) o = a.residual[(int64_t)b * rows + row] + o;
                            a.y[(int64_t)b * rows + row] = o;
                        }
                    }
                }
                if (it + 1 < nitems) st_csync();   // red is rewritten at the next block's end
            } else {
                // every CTA of the cluster runs (and, at batch > 4, has
                // consumed its last stage: the first CTA's ring takes the sums)
                if (LATE) mm_cluster_arrive_release();
                mm_cluster_wait();
                for (int task = threadIdx.x; task < ntask; task += ST_CTHREADS) {
                    const int rr = task & (ST_RB - 1), b = task >> 7, ti = rr >> 5, ri = rr & 31;
                    const float o = (red[((0 * 4 + ti) * NB + b) * 32 + ri] + red[((1 * 4 + ti) * NB + b) * 32 + ri]) +
                                    (red[((2 * 4 + ti) * NB + b) * 32 + ri] + red[((3 * 4 + ti) * NB + b) * 32 + ri]);
                    mm_st_cluster(mm_mapa(smem_u32(pt + (part * NB + b) * ST_RB + rr), 0), o);
                }
                mm_cluster_arrive_release();
                mm_cluster_wait();
                if (part == 0 && ok && !*(volatile int *)a.flag) {
                    for (int task = threadIdx.x; task < ntask; task += ST_CTHREADS) {
                        const int rr = task & (ST_RB - 1), b = task >> 7, row = r0 + rr;
                        if (row < rows) {
                            float o = pt[b * ST_RB + rr];
                            for (int p = 1; p < S; p++) o += pt[(p * NB + b) * ST_RB + rr];
                            if (a.bias) o = o + a.bias[row];
                            if (a.residual) o = a.residual[(int64_t)b * rows + row] + o;
                            a.y[(int64_t)b * rows + row] = o;
                        }
                    }
                }
            }
        }
        if (++sidx == NS) { sidx = 0; use++; }
        if (++gr == ngroups) { gr = 0; it++; }
    }
}

int st_env(const char *name, int dflt) {
    const char *v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}

struct StPlan {
    int S, NS, upc, nblk, grid;
    size_t smem;
    bool ok;
};

template <int TYPE>
StPlan st_plan(int rows, int units, int NB, int sms, int (*clusters_fit)(int S, size_t smem) = nullptr) {
    StPlan p{};
    p.nblk = (rows + ST_RB - 1) / ST_RB;
    const int ngtot = (units + ST_UG - 1) / ST_UG;
    int S = st_env("HACEDLE_ST_S", 0);
    if (S < 1) {
        // One CTA per SM: the K parts of a block are a cluster, and all the
        // clusters must run at once (a cluster's CTAs share a GPC, so the
        // number that fit depends on S, not only on the SM count).
        S = p.nblk >= sms ? 1 : sms / p.nblk;
        S = S > ST_SMAX ? ST_SMAX : S;
        while (S > 1 && clusters_fit) {
            const int upc = ((ngtot + S - 1) / S) * ST_UG;
            const size_t sm = (size_t)st_layout<TYPE>(NB, upc, S, 3).total;
            if (clusters_fit(S, sm) >= p.nblk) break;
            S--;
        }
    }
    S = S > ST_SMAX ? ST_SMAX : S;
    S = S > ngtot ? ngtot : S;
    if (S < 1) S = 1;
    p.S = S;
    p.upc = ((ngtot + S - 1) / S) * ST_UG;
    int NS = st_env("HACEDLE_ST_NS", ST_NSMAX);
    NS = NS > ST_NSMAX ? ST_NSMAX : NS < 3 ? 3 : NS;
    while (NS > 3 && (size_t)st_layout<TYPE>(NB, p.upc, S, NS).total > (size_t)ST_SMEM) NS--;
    p.NS = NS;
    p.smem = (size_t)st_layout<TYPE>(NB, p.upc, S, NS).total;
    p.ok = p.smem <= (size_t)ST_SMEM;
    // persistent over row blocks when there are more blocks than SMs (S = 1)
    p.grid = S > 1 ? p.nblk * S : (p.nblk < sms ? p.nblk : sms);
    return p;
}

template <int TYPE, int NB>
bool st_attr(int device) {
    static signed char done[ST_MAX_DEV];
    if (device < 0 || device >= ST_MAX_DEV) return false;
    if (done[device]) return done[device] > 0;
    const bool ok = cudaFuncSetAttribute(k_qgemv_st<TYPE, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, ST_SMEM) ==
                    cudaSuccess;
    if (!ok) cudaGetLastError();
    done[device] = ok ? 1 : -1;
    return ok;
}

// Clusters of S CTAs of this kernel (one per SM at the full shared-memory
// size) that the device runs at once.
template <int TYPE, int NB>
int st_clusters_fit(int S, size_t) {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    if (!st_attr<TYPE, NB>(dev)) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S * 64);
    cfg.blockDim = dim3(ST_THREADS);
    cfg.dynamicSmemBytes = ST_SMEM;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)S;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, k_qgemv_st<TYPE, NB>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

template <int TYPE, int NB>
int launch_st(hd_ctx *ctx, StArgs a, const char *name) {
    const StPlan p = st_plan<TYPE>(a.N, a.units, NB, ctx->sm_count, st_clusters_fit<TYPE, NB>);
    if (!p.ok) return hd_fail(ctx, HD_E_SHAPE, "%s: streamed GEMV plan does not fit", name);
    if (!st_attr<TYPE, NB>(ctx->device)) return hd_fail(ctx, HD_E_CUDA, "%s: shared-memory attribute refused", name);
    a.S = p.S;
    a.NS = p.NS;
    a.upc = p.upc;
    a.nblk = p.nblk;
    cudaError_t e = p.S > 1 ? hd_launch_cluster(ctx, k_qgemv_st<TYPE, NB>, dim3(p.grid), dim3(ST_THREADS), p.smem,
                                                p.S, a)
                            : hd_launch(ctx, k_qgemv_st<TYPE, NB>, dim3(p.grid), dim3(ST_THREADS), p.smem, a);
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "%s: %s", name, cudaGetErrorString(e));
    return HD_OK;
}

}  // namespace

// Whether the streamed GEMV takes this weight: rows a multiple of 8 (16-byte
// copies of the side bytes and scales), unit * row offsets in 32 bits, and
// a plan that fits shared memory.
bool hd_qgemv_stream_fits(const hd_weight *w, int B, int sms) {
    if (B < 1 || B > 16 || !hd_type_supported(w->type) || w->rows % 8 != 0) return false;
    if ((int64_t)w->units * w->rows >= ((int64_t)1 << 31) / 32) return false;
    // bulk copies: 16-byte aligned sources
    if (((uintptr_t)w->q | (uintptr_t)w->aux | (uintptr_t)w->meta | (uintptr_t)w->dsb) & 15) return false;
    const int nb = B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : B <= 8 ? 8 : 16;
    bool ok = false;
    HD_TYPE_SWITCH(w->type, TT, ok = st_plan<TT>((int)w->rows, w->units, nb, sms).ok);
    return ok;
}

int hd_qgemv_stream(hd_ctx *ctx, const hd_weight *w, const float *x, float *y, int B, const float *bias,
                    const float *residual, const char *name) {
    HD_REQUIRE(ctx, hd_qgemv_stream_fits(w, B, ctx->sm_count), HD_E_SHAPE, "%s: shape outside the streamed GEMV",
               name);
    StArgs a;
    a.w = wview(w);
    a.x = x;
    a.y = y;
    a.bias = bias;
    a.residual = residual;
    a.B = B;
    a.N = (int)w->rows;
    a.K = (int)w->cols;
    a.units = w->units;
    a.S = a.NS = a.upc = a.nblk = 1;
    a.flag = ctx->flag;
    const int nb = B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : B <= 8 ? 8 : 16;
    int rc = HD_E_TYPE;
    HD_TYPE_SWITCH(w->type, TT, {
        rc = nb == 1    ? launch_st<TT, 1>(ctx, a, name)
             : nb == 2  ? launch_st<TT, 2>(ctx, a, name)
             : nb == 4  ? launch_st<TT, 4>(ctx, a, name)
             : nb == 8  ? launch_st<TT, 8>(ctx, a, name)
                        : launch_st<TT, 16>(ctx, a, name);
    });
    return rc;
}
