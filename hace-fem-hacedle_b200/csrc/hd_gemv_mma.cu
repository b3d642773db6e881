// hd_gemv_mma.cu -- decode Q-GEMV at batch <= 4 with the products on the
// tensor cores: y[b] = W x[b] (+bias, +residual), fp32 accumulation.
//
// Why.  On CUDA cores every weight value costs a byte_perm, a share of the
// masks and shifts that unpack it, and one FFMA per batch row; on the
// large matrices that issue load, not HBM, bounded the streamed kernel
// (hd_gemv_sk.cu: ~150 instructions per 32-row unit, 0.31-0.36 of HBM).
// Here one LOP3 turns two quants into an fp16 pair, one fp16 subtract or
// multiply-add removes the magic offset exactly, and mma.sync m16n8k16 does
// all the multiply-adds of a unit for up to 4 batch rows at once.
//
// Exactness.  A (weights) holds the quant integers with the type's offset
// removed (Q4_K 0..15, Q5_0 -16..15, Q6_K -32..31, Q8_0 -128..127): exact in
// fp16.  B (activations) holds x * 2^s split into fp16 hi + lo parts as two
// columns (s per unit and batch row puts the unit's largest |x| in
// [2^14, 2^15)), so x is kept to ~22 bits; every product is exact and only
// the fp32 accumulation rounds.  The epilogue adds the hi and lo columns,
// undoes 2^s exactly and applies the row's fp32 scale per unit (Q4_K also
// subtracts min * sum(x), Q6_K applies one scale per 16-value half).
//
// Fragments.  A unit of 32 rows is 32 x 16 bytes of nibbles in shared
// memory, so ldmatrix.x4 hands thread (g = lane / 4, t = lane % 4) word t of
// rows g, g+8, g+16 and g+24: values 4t..4t+3 (low nibbles) and 16+4t..
// 16+4t+3 (high nibbles).  The MMA's K order is permuted to match: k-step 0
// holds values 0..15 and k-step 1 values 16..31, and within a k-step thread
// t's pairs (k 2t, 2t+1) and (k 2t+8, 2t+9) are values (4t, 4t+2) and
// (4t+1, 4t+3) -- exactly the nibble pairs one LOP3 with a 0x000F000F-style
// mask picks out.  The activation fragments are written in the same order.
//
// Work split, pipeline and reduction: as hd_gemv_sk.cu (stream-K over quads
// of 4 units of 32-row tiles, no wave quantization; partial tiles meet in
// the workspace in slot order).  Weights, side bytes and super-block
// headers travel to a per-warp shared-memory ring by cp.async, NS - 1 quads
// ahead; the first quads are requested before griddepcontrol.wait.
#include <cstdlib>

#include "hd_internal.cuh"
#include "hd_mma.cuh"

namespace {

constexpr int MM_WPB = 4;  // warps per CTA

struct MmArgs {
    WView w;
    const float *x;         // [B][K]
    float *y;               // [B][N]
    const float *bias;      // [N] or null
    const float *residual;  // [B][N] or null
    int B, N, K, units, tiles;
    int Q;                  // quads: tiles * units / 4
    int W;                  // warps in the grid
    int maxseg;             // workspace slots per tile
    float *ws;              // [tiles][maxseg][NB][32]
    int *tickets;           // [tiles], zero between launches
};

// Bytes of one stage (a quad of 4 units of one 32-row tile) per type.
//   Q4_K: quants 4 x 512, header 32 x 16
//   Q5_0: quants 4 x 512, qh 4 x 128 ([unit][g][i], row = g + 8 i), d 4 x 64
//   Q6_K: quants 4 x 512, high bits 4 x 256 ([unit][g][i] of 8 bytes),
//         sub-block scales 32 x 16, d 32 x 2
//   Q8_0: quants 4 x 1024 (two 512-byte halves per unit), d 4 x 64
template <int TYPE>
struct Mm;
template <>
struct Mm<HD_TYPE_Q4_K> {
    static constexpr int QU = 512, SIDE = 0, HDR = 512, DB = 0, NS = 4, NSC = 2;
};
template <>
struct Mm<HD_TYPE_Q5_0> {
    static constexpr int QU = 512, SIDE = 128, HDR = 0, DB = 256, NS = 4, NSC = 1;
};
template <>
struct Mm<HD_TYPE_Q6_K> {
    static constexpr int QU = 512, SIDE = 256, HDR = 512, DB = 64, NS = 3, NSC = 2;
};
template <>
struct Mm<HD_TYPE_Q8_0> {
    static constexpr int QU = 1024, SIDE = 0, HDR = 0, DB = 256, NS = 3, NSC = 1;
};

template <int TYPE>
struct MmLayout {
    using P = Mm<TYPE>;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_SIDE = 4 * P::QU;
    static constexpr int OFF_HDR = OFF_SIDE + 4 * P::SIDE;
    static constexpr int OFF_D = OFF_HDR + P::HDR;
    static constexpr int STAGE = (OFF_D + P::DB + 127) / 128 * 128;
};

// Per-warp shared memory: x fragments [UMAX][8 NB][4] uint4 (4 KB), per
// (unit, batch) {2^-s, sum x} [UMAX][4] float2, decoded scales
// [NSC][4 units][8][4] floats, then NS stages.
template <int TYPE, int NB>
struct MmWarp {
    static constexpr int UMAX = 32 / NB;
    static constexpr int OFF_IMG = 0;
    static constexpr int OFF_XS = 4096;
    static constexpr int OFF_SC = OFF_XS + UMAX * 4 * 8;
    static constexpr int OFF_ST = OFF_SC + Mm<TYPE>::NSC * 512;
    static constexpr int BYTES = OFF_ST + Mm<TYPE>::NS * MmLayout<TYPE>::STAGE;
};

template <int TYPE, int NB>
__global__ void __launch_bounds__(32 * MM_WPB) k_qgemv_mma(MmArgs a) {
    using P = Mm<TYPE>;
    using L = MmLayout<TYPE>;
    using WL = MmWarp<TYPE, NB>;
    constexpr int NS = P::NS, UMAX = WL::UMAX;
    extern __shared__ __align__(128) unsigned char mm_sm[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    unsigned char *wsm = mm_sm + (size_t)wib * WL::BYTES;
    uint4 *img = (uint4 *)(wsm + WL::OFF_IMG);
    float2 *xs2 = (float2 *)(wsm + WL::OFF_XS);
    float *scl = (float *)(wsm + WL::OFF_SC);
    unsigned char *stg = wsm + WL::OFF_ST;
    const uint32_t stg_s = smem_u32(stg);

    const int gw = blockIdx.x * MM_WPB + wib;
    // The grid is whole CTAs: warps past the W that own the quads have no work
    // (warp-uniform exit; the kernel has no CTA barrier).
    if (gw >= a.W) {
        pdl_trigger();
        return;
    }
    const int Q = a.Q, units = a.units, qpt = units / 4, rows = a.N;
    const int q0 = (int)((int64_t)gw * Q / a.W), q1 = (int)((int64_t)(gw + 1) * Q / a.W);
    const WView w = a.w;

    // Issue position (quads NS - 1 ahead of consumption).
    int itile = q0 / qpt, iu = (q0 - itile * qpt) * 4;
    auto issue = [&](int stage) {
        const uint32_t s0 = stg_s + stage * L::STAGE;
        const int row = min(itile * 32 + lane, rows - 1);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t ur = (uint32_t)(iu + k) * rows + row;
            if constexpr (TYPE == HD_TYPE_Q8_0) {
                cp16(s0 + L::OFF_Q + k * P::QU + lane * 16, w.q + (size_t)ur * 32);
                cp16(s0 + L::OFF_Q + k * P::QU + 512 + lane * 16, w.q + (size_t)ur * 32 + 16);
            } else {
                cp16(s0 + L::OFF_Q + k * P::QU + lane * 16, w.q + (size_t)ur * 16);
            }
            const int gi = ((lane & 7) * 4 + (lane >> 3));  // (g, i) slot of this row
            if constexpr (TYPE == HD_TYPE_Q5_0) cp4(s0 + L::OFF_SIDE + k * P::SIDE + gi * 4, w.aux + (size_t)ur * 4);
            if constexpr (TYPE == HD_TYPE_Q6_K) cp8(s0 + L::OFF_SIDE + k * P::SIDE + gi * 8, w.aux + (size_t)ur * 8);
            if constexpr (TYPE == HD_TYPE_Q5_0 || TYPE == HD_TYPE_Q8_0) {
                if (lane < 16) {  // the unit's 32 fp16 scales, 4 bytes (2 rows) per lane; rows is even
                    const int r2 = min(itile * 32 + 2 * lane, rows - 2);
                    cp4(s0 + L::OFF_D + k * 64 + lane * 4, w.meta + ((size_t)(iu + k) * rows + r2) * 2);
                }
            }
        }
        if constexpr (TYPE == HD_TYPE_Q4_K || TYPE == HD_TYPE_Q6_K) {
            const uint32_t sr = (uint32_t)(iu >> 3) * rows + row;
            cp16(s0 + L::OFF_HDR + lane * 16, w.meta + (size_t)sr * 16);
            if constexpr (TYPE == HD_TYPE_Q6_K) {
                if (lane < 16) {
                    const int r2 = min(itile * 32 + 2 * lane, rows - 2);
                    cp4(s0 + L::OFF_D + lane * 4, w.dsb + (size_t)(iu >> 3) * rows + r2);
                }
            }
        }
        iu += 4;
        if (iu == units) {
            iu = 0;
            itile++;
        }
    };

#pragma unroll
    for (int s = 0; s < NS - 1; s++) {
        if (q0 + s < q1) issue(s);
        cp_commit();
    }
    pdl_trigger();
    pdl_wait();

    int tile = q0 / qpt, u = (q0 - tile * qpt) * 4;             // consumed position
    int seg0 = q0;                                              // segment start (quads)
    int seg1 = (tile + 1) * qpt < q1 ? (tile + 1) * qpt : q1;   // segment end
    int cbeg = q0, cend = q0;                                   // staged x chunk (quads)
    float acc[4] = {0.f, 0.f, 0.f, 0.f};                        // rows g + 8 i, batch t

    auto flush = [&]() {
        const int t0 = tile * qpt, t1 = t0 + qpt;
        float out[4];
        bool write = false;
        if (seg0 == t0 && seg1 == t1) {
#pragma unroll
            for (int i = 0; i < 4; i++) out[i] = acc[i];
            write = true;
        } else {
            const int gf = (int)(((int64_t)(t0 + 1) * a.W - 1) / Q), gl = (int)(((int64_t)t1 * a.W - 1) / Q);
            const int nseg = gl - gf + 1, slot = gw - gf;
            float *base = a.ws + (size_t)tile * a.maxseg * NB * 32;
            if (t < NB) {
#pragma unroll
                for (int i = 0; i < 4; i++) __stcg(base + ((size_t)slot * NB + t) * 32 + g + 8 * i, acc[i]);
            }
            __threadfence();
            __syncwarp();
            int last = 0;
            if (lane == 0) last = atomicAdd(a.tickets + tile, 1) == nseg - 1;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence();
#pragma unroll
                for (int i = 0; i < 4; i++) out[i] = 0.f;
                if (t < NB) {
                    for (int k = 0; k < nseg; k++) {
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            out[i] += k == slot ? acc[i] : __ldcg(base + ((size_t)k * NB + t) * 32 + g + 8 * i);
                    }
                }
                if (lane == 0) a.tickets[tile] = 0;
                write = true;
            }
        }
        if (write && t < a.B) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int row = tile * 32 + g + 8 * i;
                if (row < rows) {
                    float o = out[i];
                    if (a.bias) o = o + a.bias[row];
                    if (a.residual) o = a.residual[(int64_t)t * rows + row] + o;
                    a.y[(int64_t)t * rows + row] = o;
                }
            }
        }
    };

    int stage = 0;
    for (int q = q0; q < q1; q++) {
        if (q == cend) {  // x chunk boundary (warp-uniform)
            if (q == seg1) {
                flush();
                tile++;
                u = 0;
                seg0 = q;
                seg1 = (tile + 1) * qpt < q1 ? (tile + 1) * qpt : q1;
#pragma unroll
                for (int i = 0; i < 4; i++) acc[i] = 0.f;
            }
            const int n = (seg1 - q) * 4 < UMAX ? (seg1 - q) * 4 : UMAX;  // units
            cbeg = q;
            cend = q + n / 4;
            __syncwarp();
            // lane task: unit l = lane / NB of the chunk, batch row b = lane % NB
            const int l = lane / NB, b = lane % NB;
            if (l < n && b < a.B) {
                const float4 *src = (const float4 *)(a.x + (int64_t)b * a.K + (int64_t)(u + l) * 32);
                float v[32];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float4 f = __ldg(src + j);
                    v[4 * j] = f.x;
                    v[4 * j + 1] = f.y;
                    v[4 * j + 2] = f.z;
                    v[4 * j + 3] = f.w;
                }
                float h0 = 0.f, h1 = 0.f, mx = 0.f;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    h0 += (v[4 * j] + v[4 * j + 1]) + (v[4 * j + 2] + v[4 * j + 3]);
                    h1 += (v[16 + 4 * j] + v[16 + 4 * j + 1]) + (v[16 + 4 * j + 2] + v[16 + 4 * j + 3]);
                }
#pragma unroll
                for (int j = 0; j < 32; j++) mx = fmaxf(mx, fabsf(v[j]));
                // 2^s with the largest |x| in [2^14, 2^15): x * 2^s fits fp16
                // with room; s within [-100, 100] (a zero unit keeps s = 0)
                int s = 0;
                if (mx > 0.f) {
                    const int e = (int)((__float_as_uint(mx) >> 23) & 255) - 127;
                    s = 14 - e;
                    s = s < -100 ? -100 : s > 100 ? 100 : s;
                }
                const float up = __int_as_float((127 + s) << 23);
                xs2[l * 4 + b] = make_float2(__int_as_float((127 - s) << 23), h0 + h1);
                uint4 *dst = img + l * 8 * NB;
#pragma unroll
                for (int tt = 0; tt < 4; tt++) {
                    __half hi[8], lo[8];
                    const int idx[8] = {4 * tt, 4 * tt + 2, 4 * tt + 1, 4 * tt + 3,
                                        16 + 4 * tt, 16 + 4 * tt + 2, 16 + 4 * tt + 1, 16 + 4 * tt + 3};
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const float xv = v[idx[j]] * up;
                        hi[j] = __float2half_rn(xv);
                        lo[j] = __float2half_rn(xv - __half2float(hi[j]));
                    }
                    dst[(2 * b) * 4 + tt] = make_uint4(pack_h2(hi[0], hi[1]), pack_h2(hi[2], hi[3]),
                                                       pack_h2(hi[4], hi[5]), pack_h2(hi[6], hi[7]));
                    dst[(2 * b + 1) * 4 + tt] = make_uint4(pack_h2(lo[0], lo[1]), pack_h2(lo[2], lo[3]),
                                                           pack_h2(lo[4], lo[5]), pack_h2(lo[6], lo[7]));
                }
            }
            __syncwarp();
        }
        // the quad's stage has landed; refill the stage consumed last
        cp_wait<NS - 2>();
        __syncwarp();
        {
            const int nxt = stage == 0 ? NS - 1 : stage - 1;
            if (q + NS - 1 < q1) issue(nxt);
            cp_commit();
        }
        const unsigned char *st = stg + stage * L::STAGE;
        const uint32_t st_s = stg_s + stage * L::STAGE;
        // lane = row: decode this row's scales for the quad's 4 units
        {
            const int gi = (lane & 7) * 4 + (lane >> 3);
            if constexpr (TYPE == HD_TYPE_Q5_0 || TYPE == HD_TYPE_Q8_0) {
#pragma unroll
                for (int k = 0; k < 4; k++)
                    scl[k * 32 + gi] = h2f(*(const uint16_t *)(st + L::OFF_D + k * 64 + lane * 2));
            } else if constexpr (TYPE == HD_TYPE_Q4_K) {
                const uint4 hd = *(const uint4 *)(st + L::OFF_HDR + lane * 16);
                const float d = h2f((uint16_t)(hd.x & 0xFFFF)), dmin = h2f((uint16_t)(hd.x >> 16));
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    int sc, m;
                    q4k_sm_regs((u + k) & 7, hd.y, hd.z, hd.w, sc, m);
                    scl[k * 32 + gi] = __fmul_rn(d, (float)sc);
                    scl[128 + k * 32 + gi] = __fmul_rn(dmin, (float)m);
                }
            } else {  // Q6_K: two sub-block scales per unit
                const float d = h2f(*(const uint16_t *)(st + L::OFF_D + lane * 2));
                const int8_t *sc = (const int8_t *)(st + L::OFF_HDR + lane * 16);
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int s0 = 2 * ((u + k) & 7);
                    scl[k * 32 + gi] = __fmul_rn(d, (float)sc[s0]);
                    scl[128 + k * 32 + gi] = __fmul_rn(d, (float)sc[s0 + 1]);
                }
            }
        }
        __syncwarp();
        const int l0 = (q - cbeg) * 4;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int l = l0 + k;
            uint4 bf = make_uint4(0, 0, 0, 0);
            if (g < 2 * NB) bf = img[l * 8 * NB + lane];
            const float2 ps = xs2[l * 4 + t];  // {2^-s, sum x} of batch row t
            const float4 d4 = *(const float4 *)(scl + k * 32 + g * 4);
            float4 e4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if constexpr (P::NSC == 2) e4 = *(const float4 *)(scl + 128 + k * 32 + g * 4);
            uint32_t r[4], r2[4];
            ldsm4(st_s + L::OFF_Q + k * P::QU + lane * 16, r);
            if constexpr (TYPE == HD_TYPE_Q8_0) ldsm4(st_s + L::OFF_Q + k * P::QU + 512 + lane * 16, r2);
            uint32_t ex[4][2];
#pragma unroll
            for (int i = 0; i < 4; i++) ex[i][0] = ex[i][1] = 0;
            if constexpr (TYPE == HD_TYPE_Q5_0) {
                const uint4 qh = *(const uint4 *)(st + L::OFF_SIDE + k * P::SIDE + g * 16);
                ex[0][0] = qh.x >> t;
                ex[1][0] = qh.y >> t;
                ex[2][0] = qh.z >> t;
                ex[3][0] = qh.w >> t;
            } else if constexpr (TYPE == HD_TYPE_Q6_K) {
                const uint4 h01 = *(const uint4 *)(st + L::OFF_SIDE + k * P::SIDE + g * 32);
                const uint4 h23 = *(const uint4 *)(st + L::OFF_SIDE + k * P::SIDE + g * 32 + 16);
                ex[0][0] = h01.x >> (2 * t);
                ex[0][1] = h01.y >> (2 * t);
                ex[1][0] = h01.z >> (2 * t);
                ex[1][1] = h01.w >> (2 * t);
                ex[2][0] = h23.x >> (2 * t);
                ex[2][1] = h23.y >> (2 * t);
                ex[3][0] = h23.z >> (2 * t);
                ex[3][1] = h23.w >> (2 * t);
            }
            const float dv[4] = {d4.x, d4.y, d4.z, d4.w}, ev[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
            for (int m = 0; m < 2; m++) {  // rows 16 m .. 16 m + 15
                uint32_t A0[4], A1[4];      // rows g + 16 m, g + 8 + 16 m
                unpack_word<TYPE>(r[2 * m], ex[2 * m][0], ex[2 * m][1], A0);
                unpack_word<TYPE>(r[2 * m + 1], ex[2 * m + 1][0], ex[2 * m + 1][1], A1);
                const float z[4] = {0.f, 0.f, 0.f, 0.f};
                float d0[4], d1[4];
                if constexpr (TYPE == HD_TYPE_Q8_0) {
                    uint32_t B0[4], B1[4];
                    unpack_word<TYPE>(r2[2 * m], 0, 0, B0);
                    unpack_word<TYPE>(r2[2 * m + 1], 0, 0, B1);
                    mma16816(d0, A0[0], A1[0], A0[1], A1[1], bf.x, bf.y, z);
                    mma16816(d0, B0[0], B1[0], B0[1], B1[1], bf.z, bf.w, d0);
                } else if constexpr (TYPE == HD_TYPE_Q6_K) {
                    mma16816(d0, A0[0], A1[0], A0[1], A1[1], bf.x, bf.y, z);
                    mma16816(d1, A0[2], A1[2], A0[3], A1[3], bf.z, bf.w, z);
                } else {
                    mma16816(d0, A0[0], A1[0], A0[1], A1[1], bf.x, bf.y, z);
                    mma16816(d0, A0[2], A1[2], A0[3], A1[3], bf.z, bf.w, d0);
                }
                // c0/c1: row g + 16 m, columns hi / lo of batch t; c2/c3: row + 8
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int i = 2 * m + h;
                    if constexpr (TYPE == HD_TYPE_Q6_K) {
                        acc[i] = fmaf(dv[i] * ps.x, d0[2 * h] + d0[2 * h + 1], acc[i]);
                        acc[i] = fmaf(ev[i] * ps.x, d1[2 * h] + d1[2 * h + 1], acc[i]);
                    } else {
                        acc[i] = fmaf(dv[i] * ps.x, d0[2 * h] + d0[2 * h + 1], acc[i]);
                        if constexpr (TYPE == HD_TYPE_Q4_K) acc[i] = fmaf(-ev[i], ps.y, acc[i]);
                    }
                }
            }
        }
        u += 4;
        stage = stage == NS - 1 ? 0 : stage + 1;
    }
    cp_wait<0>();
    flush();
}

constexpr int MM_MAX_DEV = 64;

template <int TYPE, int NB>
int mm_occupancy(int device) {
    static int cache[MM_MAX_DEV];
    if (device < 0 || device >= MM_MAX_DEV) return 0;
    int &c = cache[device];
    if (c) return c;
    const size_t smem = (size_t)MM_WPB * MmWarp<TYPE, NB>::BYTES;
    if (cudaFuncSetAttribute(k_qgemv_mma<TYPE, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_qgemv_mma<TYPE, NB>, 32 * MM_WPB, smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    c = n;
    return n;
}

int mm_env(const char *name, int dflt) {
    const char *v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}

template <int TYPE, int NB>
int launch_mm(hd_ctx *ctx, MmArgs a, const char *name) {
    const int lmin = mm_env("HACEDLE_MM_LMIN", 2);  // quads per warp, at least
    const int occ = mm_occupancy<TYPE, NB>(ctx->device);
    if (occ < 1) return hd_fail(ctx, HD_E_CUDA, "%s: tensor-core GEMV does not fit on an SM", name);
    const size_t smem = (size_t)MM_WPB * MmWarp<TYPE, NB>::BYTES;
    int64_t wmax = a.Q / (lmin > 0 ? lmin : 1);
    if (wmax < 1) wmax = 1;
    int64_t ctas = (int64_t)ctx->sm_count * occ;
    if (ctas * MM_WPB > wmax) ctas = (wmax + MM_WPB - 1) / MM_WPB;
    a.W = (int)(ctas * MM_WPB);
    if (a.W > a.Q) a.W = a.Q;  // every warp owns at least one quad
    const int64_t lseg = a.Q / a.W, qpt = a.units / 4;
    a.maxseg = (int)((qpt + lseg - 1) / lseg + 1);
    int rc = hd_ensure_workspace(ctx, (size_t)a.tiles * a.maxseg * NB * 32 * sizeof(float), (size_t)a.tiles);
    if (rc) return rc;
    a.ws = (float *)ctx->ws;
    a.tickets = ctx->tickets;
    cudaError_t e = hd_launch(ctx, k_qgemv_mma<TYPE, NB>, dim3((unsigned)ctas), dim3(32 * MM_WPB), smem, a);
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "%s: %s", name, cudaGetErrorString(e));
    return HD_OK;
}

}  // namespace

// Whether the tensor-core GEMV takes this weight: rows of whole quads,
// unit * row offsets in 32 bits, and (types whose fp16 scales travel two
// rows per 4-byte copy) an even row count.
bool hd_qgemv_mma_fits(const hd_weight *w) {
    if (w->units % 4 != 0 || (int64_t)w->units * w->rows >= ((int64_t)1 << 31)) return false;
    if (w->type != HD_TYPE_Q4_K && w->rows % 2 != 0) return false;
    return hd_type_supported(w->type);
}

int hd_qgemv_mma(hd_ctx *ctx, const hd_weight *w, const float *x, float *y, int B, const float *bias,
                 const float *residual, const char *name) {
    HD_REQUIRE(ctx, hd_qgemv_mma_fits(w), HD_E_SHAPE, "%s: tensor-core GEMV needs cols %% 128 == 0 and even rows",
               name);
    MmArgs a;
    a.w = wview(w);
    a.x = x;
    a.y = y;
    a.bias = bias;
    a.residual = residual;
    a.B = B;
    a.N = (int)w->rows;
    a.K = (int)w->cols;
    a.units = w->units;
    a.tiles = (int)((w->rows + 31) / 32);
    a.Q = a.tiles * (a.units / 4);
    a.W = 1;
    a.maxseg = 1;
    a.ws = nullptr;
    a.tickets = nullptr;
    const int nb = B <= 1 ? 1 : B <= 2 ? 2 : 4;
    int rc = HD_E_TYPE;
    HD_TYPE_SWITCH(w->type, TT, {
        rc = nb == 1 ? launch_mm<TT, 1>(ctx, a, name) : nb == 2 ? launch_mm<TT, 2>(ctx, a, name)
                                                                : launch_mm<TT, 4>(ctx, a, name);
    });
    return rc;
}
