// hd_gemv_small.cu -- decode Q-GEMV for matrices of a few MB at batch 1..16
// with the products on the tensor cores: y[b] = W x[b] (+bias, +residual),
// fp32 accumulation.
//
// Why.  A 3 MB weight streams in under half a microsecond; in a chain of
// dependent launches what is left is latency: the dependency wait, one L2
// round trip for x, the arithmetic of the CTA with the most work, the
// reduction and the store.  This kernel keeps every part of that short:
//  - every weight byte of the CTA is requested (cp.async into shared memory,
//    one 512-byte run per 32-row unit) before griddepcontrol.wait, so the
//    weights arrive while the previous kernel finishes;
//  - after the wait the CTA turns its slice of x into fp16 MMA fragments in
//    one pass (8 lanes per unit and batch row, maxima and sums by warp
//    shuffles) and meets once at a barrier;
//  - each warp then runs mma.sync m16n8k16 over a few units: one LOP3 and
//    one exact fp16 subtract or multiply-add per pair of quants, 4 MMAs per
//    unit and 8 batch rows, so the cost per unit hardly grows with the batch;
//  - the warps' per-row sums meet in shared memory at a second barrier, and
//    when the matrix has too few 32-row tiles to fill the SMs, the K parts of
//    a tile form a thread-block cluster whose partial sums go to the first
//    CTA of the cluster through distributed shared memory.
// No workspace, no tickets, no global atomics: the sums are added in fixed
// orders (units in a warp, warps in a CTA, K parts in a cluster), so results
// are bitwise reproducible.
//
// Exactness (as hd_gemv_mma.cu): A holds the quant integers with the type's
// offset removed, exact in fp16; B holds x * 2^s (s per unit and batch row)
// split into fp16 hi and lo columns, so every product is exact and only the
// fp32 accumulation rounds.  The fragment orders are those of hd_gemv_mma.cu.
#include <cstdlib>

#include "hd_internal.cuh"
#include "hd_mma.cuh"

namespace {

constexpr int SM_MAXW = 14;   // warps per CTA, at most (two CTAs of 73 registers a thread per SM)
constexpr int SM_UMAX = 2;    // units per warp, at most (their A fragments stay in registers)
constexpr int SM_SMAX = 8;    // K parts (cluster size), at most
constexpr int SM_MAX_DEV = 64;

struct SmArgs {
    WView w, w1;            // w1: the up weight of a SwiGLU pair (else w)
    const float *x;         // [B][K]
    float *y;               // [B][N]
    const float *bias;      // [N] or null
    const float *residual;  // [B][N] or null (may be y)
    int B, N, K, units;
    int S;                  // K parts: CTAs of a cluster along x
    int W;                  // warps per CTA
    int upc;                // units per K part, at most
    int umax;               // units per warp, at most
    const float *nw;        // [K] RMSNorm weight: y = W rmsnorm(x) (null: W x)
    float eps;
};

// Bytes per unit of a 32-row tile in a warp's stage: quants (Q8_0 two
// 512-byte halves), then Q5_0's fifth bits (4 bytes per row) or Q6_K's high
// bits (8 bytes per row) in (g, i) slot order (row = g + 8 i at slot 4 g + i).
// K-quant super-block headers (16 bytes per row) follow the units.
template <int TYPE>
struct Sm;
template <>
struct Sm<HD_TYPE_Q8_0> { static constexpr int QU = 1024, SIDE = 0, HDR = 0, NSC = 1; };
template <>
struct Sm<HD_TYPE_Q5_0> { static constexpr int QU = 512, SIDE = 128, HDR = 0, NSC = 1; };
template <>
struct Sm<HD_TYPE_Q4_K> { static constexpr int QU = 512, SIDE = 0, HDR = 512, NSC = 2; };
template <>
struct Sm<HD_TYPE_Q6_K> { static constexpr int QU = 512, SIDE = 256, HDR = 512, NSC = 2; };

// Shared-memory layout (byte offsets; every part a multiple of 16 bytes):
//   x fragments  [upc][8 NB] uint4
//   x scales     [upc][NB] float4 {2^-s, sum of the unit's x, sum of x^2, 0}
//   row sums     [W][NB][32] float
//   K-part sums  [S][NB][32] float, then [S][NB] sums of x^2 (S > 1)
//   per warp     copy stage [umax][QU + SIDE] + [nsb][HDR], then the per-row
//                scales [umax][NSC][32] float
struct SmLayout {
    int img, xs, red, part, warp0, stage, hdr, scl, wbytes, total, nsb;
};
template <int TYPE>
__host__ __device__ inline SmLayout sm_layout(int NB, int upc, int W, int S, int umax) {
    using P = Sm<TYPE>;
    SmLayout L;
    L.img = 0;
    L.xs = L.img + upc * 8 * NB * 16;
    L.red = L.xs + upc * NB * 16;
    L.part = L.red + W * 32 * NB * 4;
    L.warp0 = L.part + (S > 1 ? S * 32 * NB * 4 + ((S * NB * 4 + 15) & ~15) : 0);
    L.nsb = P::HDR ? (umax + 7) / 8 + 1 : 0;   // super-blocks a warp's units can touch
    L.stage = 0;
    L.hdr = L.stage + umax * (P::QU + P::SIDE);
    L.scl = L.hdr + L.nsb * P::HDR;
    L.wbytes = L.scl + umax * P::NSC * 32 * 4;
    L.total = L.warp0 + W * L.wbytes;
    return L;
}

__device__ __forceinline__ float sm_silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// PR = 1: a SwiGLU pair.  A 32-row tile then holds 16 rows of the gate
// weight (lanes 0..15, the first MMA M tile) and the same 16 rows of the up
// weight (lanes 16..31, the second), and the epilogue writes silu(g) * u for
// its 16 output rows.
template <int TYPE, int NB, int PR>
__global__ void __launch_bounds__(32 * SM_MAXW, 2) k_qgemv_sm(SmArgs a) {
    using P = Sm<TYPE>;
    constexpr int RT = PR ? 16 : 32;   // output rows per tile
    constexpr int NT8 = NB >= 4 ? NB / 4 : 1;   // MMA column tiles of 8 (hi/lo x 4 batch rows)
    constexpr int USTR = P::QU + P::SIDE;
    extern __shared__ __align__(128) unsigned char sm_sm[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5, W = a.W, S = a.S;
    const int g = lane >> 2, t = lane & 3;
    const int part = S > 1 ? (int)mm_cluster_rank() : 0;
    const int tile = blockIdx.x / S;
    const int rows = a.N, units = a.units;
    const int cu0 = part * units / S, cu1 = (part + 1) * units / S, nu = cu1 - cu0;   // 32-bit: units * S < 2^31
    const int wu0 = cu0 + wib * nu / W, wu1 = cu0 + (wib + 1) * nu / W, nwu = wu1 - wu0;
    const SmLayout L = sm_layout<TYPE>(NB, a.upc, W, S, a.umax);
    uint4 *img = (uint4 *)(sm_sm + L.img);
    float4 *xs4 = (float4 *)(sm_sm + L.xs);
    float *red = (float *)(sm_sm + L.red);
    unsigned char *wsm = sm_sm + L.warp0 + wib * L.wbytes;
    const unsigned char *stg = wsm + L.stage;
    const uint32_t stg_s = smem_u32(stg);
    const int hdr_off = L.hdr - L.stage;   // from the stage
    float *scl = (float *)(wsm + L.scl);
    // 1. This warp's weights: lane = row of the tile (rows past N read the
    // last row; their sums are not stored).
    const WView w = (PR && lane >= 16) ? a.w1 : a.w;
    const int row = min(tile * RT + (PR ? (lane & 15) : lane), rows - 1);
    const int gi = (lane & 7) * 4 + (lane >> 3);
    const int sb0 = wu0 >> 3;
    uint32_t dreg[SM_UMAX];    // Q8_0/Q5_0: the row's fp16 scale per unit; Q6_K: d per super-block
#pragma unroll
    for (int k = 0; k < SM_UMAX; k++) dreg[k] = 0;
#pragma unroll
    for (int k = 0; k < SM_UMAX; k++) {
        if (k < nwu) {
            const uint32_t ur = (uint32_t)(wu0 + k) * (uint32_t)rows + (uint32_t)row;
            const uint32_t s0 = stg_s + k * USTR;
            if constexpr (TYPE == HD_TYPE_Q8_0) {
                cp16(s0 + lane * 16, w.q + (size_t)ur * 32);
                cp16(s0 + 512 + lane * 16, w.q + (size_t)ur * 32 + 16);
            } else {
                cp16(s0 + lane * 16, w.q + (size_t)ur * 16);
            }
            if constexpr (TYPE == HD_TYPE_Q5_0) cp4(s0 + P::QU + gi * 4, w.aux + (size_t)ur * 4);
            if constexpr (TYPE == HD_TYPE_Q6_K) cp8(s0 + P::QU + gi * 8, w.aux + (size_t)ur * 8);
            if constexpr (TYPE == HD_TYPE_Q5_0 || TYPE == HD_TYPE_Q8_0)
                dreg[k] = ld_pin_u16((const unsigned short *)w.meta + ur);
        }
    }
    if constexpr (P::HDR > 0) {
        const int sb1 = nwu > 0 ? (wu1 - 1) >> 3 : sb0 - 1;
#pragma unroll
        for (int j = 0; j < (SM_UMAX + 7) / 8 + 1; j++) {
            const int sb = sb0 + j;
            if (sb <= sb1) {
                const uint32_t sr = (uint32_t)sb * (uint32_t)rows + (uint32_t)row;
                cp16(stg_s + hdr_off + j * P::HDR + lane * 16, w.meta + (size_t)sr * 16);
                if constexpr (TYPE == HD_TYPE_Q6_K) dreg[j] = ld_pin_u16(w.dsb + sr);
            }
        }
    }
    cp_commit();
    if (S > 1) mm_cluster_arrive_relaxed();   // waited on before the first remote store
    pdl_trigger();

    // 2. Before the dependency wait (nothing here is written by the previous
    // kernel): once the warp's copies have landed, the per-row scales of its
    // units (lane = row, (g, i) slot order) and every unit unpacked into the
    // exact fp16 A fragments of its MMAs, stored per lane.
    cp_wait<0>();
    __syncwarp();
#pragma unroll
    for (int k = 0; k < SM_UMAX; k++) {
        if (k < nwu) {
            const int u = wu0 + k;
            if constexpr (TYPE == HD_TYPE_Q5_0 || TYPE == HD_TYPE_Q8_0) {
                scl[k * 32 + gi] = h2f((uint16_t)dreg[k]);
            } else if constexpr (TYPE == HD_TYPE_Q4_K) {
                const uint4 hd = *(const uint4 *)(stg + hdr_off + ((u >> 3) - sb0) * P::HDR + lane * 16);
                const float d = h2f((uint16_t)(hd.x & 0xFFFF)), dmin = h2f((uint16_t)(hd.x >> 16));
                int sc, m;
                q4k_sm_regs(u & 7, hd.y, hd.z, hd.w, sc, m);
                scl[(k * 2) * 32 + gi] = __fmul_rn(d, (float)sc);
                scl[(k * 2 + 1) * 32 + gi] = __fmul_rn(dmin, (float)m);
            } else {
                const int j = (u >> 3) - sb0;
                const int8_t *sc = (const int8_t *)(stg + hdr_off + j * P::HDR + lane * 16);
                uint32_t dj = dreg[0];
#pragma unroll
                for (int jj = 1; jj < (SM_UMAX + 7) / 8 + 1; jj++)
                    if (jj == j) dj = dreg[jj];
                const float d = h2f((uint16_t)dj);
                const int s0 = 2 * (u & 7);
                scl[(k * 2) * 32 + gi] = __fmul_rn(d, (float)sc[s0]);
                scl[(k * 2 + 1) * 32 + gi] = __fmul_rn(d, (float)sc[s0 + 1]);
            }
        }
    }
    uint4 fa[SM_UMAX][2][2];   // [unit][M tile][k-step]: A fragments a0..a3
#pragma unroll
    for (int k = 0; k < SM_UMAX; k++) {
        if (k < nwu) {
            const uint32_t st_s = stg_s + k * USTR;
            const unsigned char *st = stg + k * USTR;
            uint32_t r[4], r2[4];
            ldsm4(st_s + lane * 16, r);
            if constexpr (TYPE == HD_TYPE_Q8_0) ldsm4(st_s + 512 + lane * 16, r2);
            uint32_t ex[4][2];
#pragma unroll
            for (int i = 0; i < 4; i++) ex[i][0] = ex[i][1] = 0;
            if constexpr (TYPE == HD_TYPE_Q5_0) {
                const uint4 qh = *(const uint4 *)(st + P::QU + g * 16);
                ex[0][0] = qh.x >> t;
                ex[1][0] = qh.y >> t;
                ex[2][0] = qh.z >> t;
                ex[3][0] = qh.w >> t;
            } else if constexpr (TYPE == HD_TYPE_Q6_K) {
                const uint4 h01 = *(const uint4 *)(st + P::QU + g * 32);
                const uint4 h23 = *(const uint4 *)(st + P::QU + g * 32 + 16);
                ex[0][0] = h01.x >> (2 * t);
                ex[0][1] = h01.y >> (2 * t);
                ex[1][0] = h01.z >> (2 * t);
                ex[1][1] = h01.w >> (2 * t);
                ex[2][0] = h23.x >> (2 * t);
                ex[2][1] = h23.y >> (2 * t);
                ex[3][0] = h23.z >> (2 * t);
                ex[3][1] = h23.w >> (2 * t);
            }
#pragma unroll
            for (int m = 0; m < 2; m++) {
                uint32_t A0[4], A1[4];   // rows g + 16 m, g + 8 + 16 m
                unpack_word<TYPE>(r[2 * m], ex[2 * m][0], ex[2 * m][1], A0);
                unpack_word<TYPE>(r[2 * m + 1], ex[2 * m + 1][0], ex[2 * m + 1][1], A1);
                fa[k][m][0] = make_uint4(A0[0], A1[0], A0[1], A1[1]);
                if constexpr (TYPE == HD_TYPE_Q8_0) {
                    uint32_t B0[4], B1[4];
                    unpack_word<TYPE>(r2[2 * m], 0, 0, B0);
                    unpack_word<TYPE>(r2[2 * m + 1], 0, 0, B1);
                    fa[k][m][1] = make_uint4(B0[0], B1[0], B0[1], B1[1]);
                } else {
                    fa[k][m][1] = make_uint4(A0[2], A1[2], A0[3], A1[3]);
                }
            }
        } else {
#pragma unroll
            for (int m = 0; m < 2; m++) fa[k][m][0] = fa[k][m][1] = make_uint4(0, 0, 0, 0);
        }
    }
    __syncwarp();   // the scales come from other lanes
    pdl_wait();

    // 3. x fragments of the part's units: task (unit l, batch row b, quarter
    // q) = 8 lanes per (l, b), lane q holds x[4q .. 4q + 3] of the unit.  A
    // thread's loads (up to XR tasks) are all issued before the first use.
    {
        constexpr int XR = NB >= 2 ? 2 : 1;
        const int ntask = nu * NB * 8, nthr = 32 * W;
        for (int base = 0; base < ntask; base += XR * nthr) {   // warp-uniform trip counts
            float4 v[XR], nv[XR];
#pragma unroll
            for (int r = 0; r < XR; r++) {
                const int task = base + r * nthr + threadIdx.x;
                const int q = task & 7, lb = task >> 3, l = lb / NB, b = lb - l * NB;
                v[r] = make_float4(0.f, 0.f, 0.f, 0.f);
                nv[r] = make_float4(1.f, 1.f, 1.f, 1.f);
                if (task < ntask && b < a.B) {
                    v[r] = __ldg((const float4 *)(a.x + (int64_t)b * a.K + (int64_t)(cu0 + l) * 32) + q);
                    if (a.nw) nv[r] = __ldg((const float4 *)(a.nw + (int64_t)(cu0 + l) * 32) + q);
                }
            }
#pragma unroll
            for (int r = 0; r < XR; r++) {
                if (base + r * nthr >= ntask) break;   // warp-uniform
                const int task = base + r * nthr + threadIdx.x;
                const bool live = task < ntask;
                const int q = task & 7, lb = task >> 3, l = lb / NB, b = lb - l * NB;
                // with a norm weight: x * w here, the 1 / rms factor on the sums
                const float4 x0 = v[r];
                const float4 xv4 = make_float4(__fmul_rn(x0.x, nv[r].x), __fmul_rn(x0.y, nv[r].y),
                                               __fmul_rn(x0.z, nv[r].z), __fmul_rn(x0.w, nv[r].w));
                float mx = fmaxf(fmaxf(fabsf(xv4.x), fabsf(xv4.y)), fmaxf(fabsf(xv4.z), fabsf(xv4.w)));
                float sm = (xv4.x + xv4.y) + (xv4.z + xv4.w);
                float sq = fmaf(x0.x, x0.x, x0.y * x0.y) + fmaf(x0.z, x0.z, x0.w * x0.w);
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) {
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    sm += __shfl_xor_sync(0xffffffffu, sm, o);
                    sq += __shfl_xor_sync(0xffffffffu, sq, o);
                }
                // 2^s with the unit's largest |x| in [2^14, 2^15): x * 2^s fits
                // fp16 with room; s within [-100, 100] (a zero unit keeps s = 0)
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
                for (int j = 0; j < 4; j++) {
                    hi[j] = __float2half_rn(xv[j]);
                    lo[j] = __float2half_rn(xv[j] - __half2float(hi[j]));
                }
                if (live) {
                    // uint4 (l, column c, tt = q & 3): pairs (4tt, 4tt+2), (4tt+1,
                    // 4tt+3) of the low half, then the same of the high half
                    uint2 *img2 = (uint2 *)(img + l * 8 * NB);
                    const int tt = q & 3, half = q >> 2;
                    img2[((2 * b) * 4 + tt) * 2 + half] = make_uint2(pack_h2(hi[0], hi[2]), pack_h2(hi[1], hi[3]));
                    img2[((2 * b + 1) * 4 + tt) * 2 + half] = make_uint2(pack_h2(lo[0], lo[2]), pack_h2(lo[1], lo[3]));
                    if (q == 0) xs4[l * NB + b] = make_float4(__int_as_float((127 - s) << 23), sm, sq, 0.f);
                }
            }
        }
    }
    __syncthreads();

    // 4. MMAs over the warp's units (A fragments in registers since before
    // the wait); each unit's sums go into acc in unit order.  acc[i][j]: row
    // g + 8 i of the tile, batch row 4 j + t.
    float acc[4][NT8];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < NT8; j++) acc[i][j] = 0.f;
#pragma unroll
    for (int k = 0; k < SM_UMAX; k++) {
        if (k < nwu) {   // warp-uniform
            const int l = wu0 + k - cu0;
            const float4 d4 = *(const float4 *)(scl + (k * P::NSC) * 32 + g * 4);
            float4 e4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if constexpr (P::NSC == 2) e4 = *(const float4 *)(scl + (k * 2 + 1) * 32 + g * 4);
            const float dv[4] = {d4.x, d4.y, d4.z, d4.w}, ev[4] = {e4.x, e4.y, e4.z, e4.w};
            const float z[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < NT8; j++) {
                uint4 bf = make_uint4(0, 0, 0, 0);
                if (NB >= 4 || g < 2 * NB) bf = img[l * 8 * NB + j * 32 + lane];
                const int b = 4 * j + t;
                const float4 ps = b < NB ? xs4[l * NB + b] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int m = 0; m < 2; m++) {
                    const uint4 &f0 = fa[k][m][0], &f1 = fa[k][m][1];
                    float e0[4], e1[4];
                    mma16816(e0, f0.x, f0.y, f0.z, f0.w, bf.x, bf.y, z);
                    if constexpr (TYPE == HD_TYPE_Q6_K)
                        mma16816(e1, f1.x, f1.y, f1.z, f1.w, bf.z, bf.w, z);
                    else
                        mma16816(e0, f1.x, f1.y, f1.z, f1.w, bf.z, bf.w, e0);
                    // c0/c1: row g + 16 m, columns hi / lo of batch row b; c2/c3: row + 8
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const int i = 2 * m + h;
                        acc[i][j] = fmaf(dv[i] * ps.x, e0[2 * h] + e0[2 * h + 1], acc[i][j]);
                        if constexpr (TYPE == HD_TYPE_Q6_K)
                            acc[i][j] = fmaf(ev[i] * ps.x, e1[2 * h] + e1[2 * h + 1], acc[i][j]);
                        if constexpr (TYPE == HD_TYPE_Q4_K) acc[i][j] = fmaf(-ev[i], ps.y, acc[i][j]);
                    }
                }
            }
        }
    }

    // 5. The warps' row sums, added in warp order.
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < NT8; j++) {
            const int b = 4 * j + t;
            if (b < NB) red[(wib * NB + b) * 32 + g + 8 * i] = acc[i][j];
        }
    __syncthreads();
    // Task (output row rr of the tile, batch row b) = RT b + rr, strided over
    // the CTA's threads.
    const int nthr = 32 * W, ntask = RT * a.B;
    auto warp_sum = [&](int rr, int b) {   // all loads first, then the sum in warp order
        float p[SM_MAXW];
#pragma unroll
        for (int ww = 0; ww < SM_MAXW; ww++) p[ww] = ww < W ? red[(ww * NB + b) * 32 + rr] : 0.f;
        float v = p[0];
#pragma unroll
        for (int ww = 1; ww < SM_MAXW; ww++)
            if (ww < W) v += p[ww];
        return v;
    };
    auto part_ssq = [&](int b) {   // sum of x^2 over the part's units, in unit order
        float v = 0.f;
        for (int l = 0; l < nu; l++) v += xs4[l * NB + b].z;
        return v;
    };
    auto store = [&](int rr, int b, float vg, float vu, float ssq) {
        const int orow = tile * RT + rr;
        if (orow >= rows) return;
        if (a.nw) {
            const float rs = 1.0f / sqrtf(ssq / (float)a.K + a.eps);
            vg = vg * rs;
            vu = vu * rs;
        }
        if (PR) {
            a.y[(int64_t)b * rows + orow] = sm_silu_mul(vg, vu);
        } else {
            float o = vg;
            if (a.bias) o = o + a.bias[orow];
            if (a.residual) o = a.residual[(int64_t)b * rows + orow] + o;
            a.y[(int64_t)b * rows + orow] = o;
        }
    };
    if (S == 1) {
        for (int task = threadIdx.x; task < ntask; task += nthr) {
            const int rr = task % RT, b = task / RT;
            store(rr, b, warp_sum(rr, b), PR ? warp_sum(rr + 16, b) : 0.f, a.nw ? part_ssq(b) : 0.f);
        }
        return;
    }

    // 6. K parts of a cluster: every part's sums (and sums of x^2) into the
    // first CTA, added in part order there.
    float *pt = (float *)(sm_sm + L.part);
    float *pss = pt + S * NB * 32;
    mm_cluster_wait();   // every CTA of the cluster runs: its shared memory may be written
    for (int task = threadIdx.x; task < ntask; task += nthr) {
        const int rr = task % RT, b = task / RT;
        mm_st_cluster(mm_mapa(smem_u32(pt + (part * NB + b) * 32 + rr), 0), warp_sum(rr, b));
        if (PR) mm_st_cluster(mm_mapa(smem_u32(pt + (part * NB + b) * 32 + rr + 16), 0), warp_sum(rr + 16, b));
        if (a.nw && rr == 0) mm_st_cluster(mm_mapa(smem_u32(pss + part * NB + b), 0), part_ssq(b));
    }
    mm_cluster_arrive_release();
    mm_cluster_wait();
    if (part != 0) return;
    for (int task = threadIdx.x; task < ntask; task += nthr) {
        const int rr = task % RT, b = task / RT;
        float pg[SM_SMAX], pu[SM_SMAX], ps[SM_SMAX];
#pragma unroll
        for (int p = 0; p < SM_SMAX; p++) {
            pg[p] = p < S ? pt[(p * NB + b) * 32 + rr] : 0.f;
            pu[p] = (PR && p < S) ? pt[(p * NB + b) * 32 + rr + 16] : 0.f;
            ps[p] = (a.nw && p < S) ? pss[p * NB + b] : 0.f;
        }
        float vg = pg[0], vu = pu[0], ss = ps[0];
#pragma unroll
        for (int p = 1; p < SM_SMAX; p++)
            if (p < S) {
                vg += pg[p];
                vu += pu[p];
                ss += ps[p];
            }
        store(rr, b, vg, vu, ss);
    }
}

int sm_env(const char *name, int dflt) {
    const char *v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}

// Launch plan: K parts S (cluster size) so that tiles x S fills the SMs,
// warps W so that each warp takes about `upw` units.
struct SmPlan {
    int S, W, upc, umax;
    size_t smem;
    bool ok;
};

template <int TYPE>
SmPlan sm_plan(int rows, int units, int NB, int sms, bool pair) {
    SmPlan p{};
    const int tiles = pair ? (rows + 15) / 16 : (rows + 31) / 32;
    const int cap = SM_UMAX * SM_MAXW;   // units one CTA holds
    int S = sm_env("HACEDLE_SM_S", 0);
    if (S < 1) {
        S = (sms + tiles - 1) / tiles;
        const int smin = (units + cap - 1) / cap;
        S = S < smin ? smin : S;
        // Few tiles: the largest cluster.  Measured on B200 (896 x 4864,
        // 28 tiles: 6 parts by the rule above), 8 parts: Q4_K B=1/4 3.33/3.82
        // against 3.37/4.06 us, Q6_K 3.69/4.28 against 3.79/4.41.
        if (S >= 6) S = SM_SMAX;
    }
    S = S > SM_SMAX ? SM_SMAX : S;
    S = S > units ? units : S;
    if (S < 1) S = 1;
    const int upc = (units + S - 1) / S;
    int W = sm_env("HACEDLE_SM_W", 0);
    if (W < 1) W = (upc + SM_UMAX - 1) / SM_UMAX;
    if (W < (upc + SM_UMAX - 1) / SM_UMAX) W = (upc + SM_UMAX - 1) / SM_UMAX;
    W = W > upc ? upc : W;
    if (W < 1) W = 1;
    const int umax = (upc + W - 1) / W;
    p.S = S;
    p.W = W;
    p.upc = upc;
    p.umax = umax;
    p.ok = umax <= SM_UMAX && W <= SM_MAXW;
    p.smem = (size_t)sm_layout<TYPE>(NB, upc, W, S, umax).total;
    if (p.smem > 227 * 1024) p.ok = false;
    return p;
}

template <int TYPE, int NB, int PR>
bool sm_attr(int device) {
    static signed char done[SM_MAX_DEV];
    if (device < 0 || device >= SM_MAX_DEV) return false;
    if (done[device]) return done[device] > 0;
    const bool ok = cudaFuncSetAttribute(k_qgemv_sm<TYPE, NB, PR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024) == cudaSuccess;
    if (!ok) cudaGetLastError();
    done[device] = ok ? 1 : -1;
    return ok;
}

template <int TYPE, int NB, int PR>
int launch_sm(hd_ctx *ctx, SmArgs a, const char *name) {
    const SmPlan p = sm_plan<TYPE>(a.N, a.units, NB, ctx->sm_count, PR != 0);
    if (!p.ok) return hd_fail(ctx, HD_E_SHAPE, "%s: small-matrix GEMV plan does not fit", name);
    if (!sm_attr<TYPE, NB, PR>(ctx->device))
        return hd_fail(ctx, HD_E_CUDA, "%s: shared-memory attribute refused", name);
    a.S = p.S;
    a.W = p.W;
    a.upc = p.upc;
    a.umax = p.umax;
    const int tiles = PR ? (a.N + 15) / 16 : (a.N + 31) / 32;
    cudaError_t e = p.S > 1 ? hd_launch_cluster(ctx, k_qgemv_sm<TYPE, NB, PR>, dim3(tiles * p.S), dim3(32 * p.W),
                                                p.smem, p.S, a)
                            : hd_launch(ctx, k_qgemv_sm<TYPE, NB, PR>, dim3(tiles), dim3(32 * p.W), p.smem, a);
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "%s: %s", name, cudaGetErrorString(e));
    return HD_OK;
}

template <int TYPE, int NB>
int launch_sm_pr(hd_ctx *ctx, const SmArgs &a, bool pair, const char *name) {
    return pair ? launch_sm<TYPE, NB, 1>(ctx, a, name) : launch_sm<TYPE, NB, 0>(ctx, a, name);
}

}  // namespace

// Whether the small-matrix kernel takes this weight (or gate/up pair) at this
// batch: a plan whose warps hold at most 2 units and whose shared memory fits
// one CTA.
bool hd_qgemv_small_fits(const hd_weight *w, int B, int sms, bool pair) {
    if (B < 1 || B > 16 || !hd_type_supported(w->type) || w->rows < 1) return false;
    if ((int64_t)w->units * w->rows >= ((int64_t)1 << 31)) return false;
    const int nb = B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : B <= 8 ? 8 : 16;
    bool ok = false;
    HD_TYPE_SWITCH(w->type, TT, ok = sm_plan<TT>((int)w->rows, w->units, nb, sms, pair).ok);
    return ok;
}

// y = W x (+bias, +residual), or with w_up a SwiGLU pair silu(W x) * (W_up x),
// with norm_w first x -> rmsnorm(x) ((x * w) / rms(x), the 1 / rms factor
// applied to the row sums).
int hd_qgemv_small(hd_ctx *ctx, const hd_weight *w, const hd_weight *w_up, const float *x, float *y, int B,
                   const float *bias, const float *residual, const float *norm_w, float eps, const char *name) {
    const bool pair = w_up != nullptr;
    HD_REQUIRE(ctx, hd_qgemv_small_fits(w, B, ctx->sm_count, pair), HD_E_SHAPE,
               "%s: shape outside the small-matrix GEMV", name);
    if (pair)
        HD_REQUIRE(ctx, w_up->type == w->type && w_up->rows == w->rows && w_up->cols == w->cols && !bias && !residual,
                   HD_E_ARG, "%s: a SwiGLU pair takes two weights of one type and shape, no bias or residual", name);
    SmArgs a;
    a.w = wview(w);
    a.w1 = pair ? wview(w_up) : a.w;
    a.x = x;
    a.y = y;
    a.bias = bias;
    a.residual = residual;
    a.B = B;
    a.N = (int)w->rows;
    a.K = (int)w->cols;
    a.units = w->units;
    a.S = a.W = a.upc = a.umax = 1;
    a.nw = norm_w;
    a.eps = eps;
    const int nb = B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : B <= 8 ? 8 : 16;
    int rc = HD_E_TYPE;
    HD_TYPE_SWITCH(w->type, TT, {
        switch (nb) {
        case 1: rc = launch_sm_pr<TT, 1>(ctx, a, pair, name); break;
        case 2: rc = launch_sm_pr<TT, 2>(ctx, a, pair, name); break;
        case 4: rc = launch_sm_pr<TT, 4>(ctx, a, pair, name); break;
        case 8: rc = launch_sm_pr<TT, 8>(ctx, a, pair, name); break;
        default: rc = launch_sm_pr<TT, 16>(ctx, a, pair, name); break;
        }
    });
    return rc;
}
