// hd_gemv_sk.cu -- streamed decode Q-GEMV for batch <= 4 on matrices large
// enough to stream at HBM bandwidth: y[b] = W x[b] (+bias, +residual).
//
// Work split ("stream-K").  A row tile is 32 output rows; lane l of a warp
// owns row 32 * tile + l, so one warp-wide 16-byte load reads one unit of 32
// rows as one contiguous 512-byte span of the unit-major layout.  The
// (row tile, unit) pairs are flattened tile-major and cut into quads of 4
// consecutive units of one tile (a row holds a multiple of 4 units); warp g
// of the W warps in the grid takes the contiguous quad range
// [g Q / W, (g + 1) Q / W).  Every warp gets the same number of quads (+-1),
// so there is no wave quantization: a grid sized to the resident warps runs
// as one wave whatever the matrix shape.
//
// Loads.  Each lane keeps the next quad of its row in flight in a 4-slot
// register ring: the slot consumed for unit k of a quad is refilled with unit
// k of the next quad, so the load pipeline runs across quad, chunk and
// row-tile boundaries.  Q4_K's super-block header and Q6_K's super-block
// scale are loaded once per quad (a quad never straddles a super-block).
// The first quad is requested before griddepcontrol.wait, overlapping the
// previous kernel in the stream (weights are never written by it).  Rows
// past N load row N - 1 (valid memory; their sums are never stored).
//
// Activations.  A warp stages the x of up to 32 / NB units of its range in
// its own slice of shared memory; lane l loads unit l's 32 values per batch
// row and forms their two 16-value half sums, which carry the quant offsets
// (unit_fma) and reach the other lanes by shuffles.  No CTA barrier is used
// anywhere: the warps of a CTA are independent.
//
// Reduction.  A warp whose range covers a whole tile writes y directly.  A
// tile split over several warps meets in the workspace: each warp writes its
// segment's partial row sums to its slot (slots in unit order), and the warp
// that takes the last ticket adds the slots in slot order.  Every sum has a
// fixed order (units in order within a segment, segments in order), so the
// results are bitwise reproducible for a given grid.
#include <cstdlib>

#include "hd_internal.cuh"
#include "hd_units.cuh"

namespace {

constexpr int SK_MAX_WPB = 8;  // warps per CTA (upper bound of the launch)
#ifndef SK_MIN_CTAS
#define SK_MIN_CTAS 3          // resident 256-thread CTAs per SM the registers must allow
#endif

struct SkArgs {
    WView w;
    const float *x;         // [B][K]
    float *y;               // [B][N]
    const float *bias;      // [N] or null
    const float *residual;  // [B][N] or null
    int B, N, K, units, tiles;
    int Q;                  // quads: tiles * units / 4
    int W;                  // warps in the grid
    int maxseg;             // workspace slots per tile
    float *ws;              // [tiles][maxseg][NB][32] partial row sums
    int *tickets;           // [tiles], zero between launches
};

// Per-unit registers (Slot) and per-quad registers (Extra) of one lane's row.
template <int TYPE>
struct SkSlot;
template <>
struct SkSlot<HD_TYPE_Q8_0> { uint4 a, b; uint32_t d; };
template <>
struct SkSlot<HD_TYPE_Q5_0> { uint4 a; uint32_t qh, d; };
template <>
struct SkSlot<HD_TYPE_Q4_K> { uint4 a; };
template <>
struct SkSlot<HD_TYPE_Q6_K> { uint4 a; uint2 h; uint32_t sc2; };  // sc2: the unit's two sub-block scales
template <int TYPE>
struct SkExtra { uint32_t unused; };
template <>
struct SkExtra<HD_TYPE_Q4_K> { uint4 m; };   // super-block header: d, dmin, 12 scale bytes
template <>
struct SkExtra<HD_TYPE_Q6_K> { uint32_t d; }; // super-block scale

// 16-byte load of streamed weight bytes: read once, so not kept in L1.
__device__ __forceinline__ uint4 ld_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// The per-unit arrays of unit u of a row; ur = u * rows + row, sr = the
// row's super-block index (u >> 3) * rows + row.
template <int TYPE>
__device__ __forceinline__ void sk_load(const WView &w, uint32_t ur, uint32_t sr, int u, SkSlot<TYPE> &g) {
    if constexpr (TYPE == HD_TYPE_Q8_0) {
        const uint4 *p = (const uint4 *)(w.q + (size_t)ur * 32);
        g.a = ld_stream(p);
        g.b = ld_stream(p + 1);
        g.d = __ldg((const unsigned short *)w.meta + ur);
    } else if constexpr (TYPE == HD_TYPE_Q5_0) {
        g.a = ld_stream(w.q + (size_t)ur * 16);
        g.qh = __ldg((const unsigned int *)w.aux + ur);
        g.d = __ldg((const unsigned short *)w.meta + ur);
    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
        g.a = ld_stream(w.q + (size_t)ur * 16);
    } else {
        g.a = ld_stream(w.q + (size_t)ur * 16);
        g.h = __ldg((const uint2 *)w.aux + ur);
        g.sc2 = __ldg((const unsigned short *)(w.meta + (size_t)sr * 16) + (u & 7));  // scales 2(u&7), 2(u&7)+1
    }
}

// Super-block fields of a row (super-block row index sr).
template <int TYPE>
__device__ __forceinline__ void sk_load_extra(const WView &w, uint32_t sr, SkExtra<TYPE> &e) {
    if constexpr (TYPE == HD_TYPE_Q4_K) e.m = __ldg((const uint4 *)(w.meta + (size_t)sr * 16));
    else if constexpr (TYPE == HD_TYPE_Q6_K) e.d = __ldg(w.dsb + sr);
}

// acc[b] += unit u . x[b] with the arithmetic of unit_fma.  xs: this unit's
// 8 float4 of x for batch row 0 in shared memory, batch row b at float4
// offset b * XSTRIDE; xh: the unit's two half sums per batch row.
template <int TYPE, int NB, int XSTRIDE>
__device__ __forceinline__ void sk_dot(const SkSlot<TYPE> &s, const SkExtra<TYPE> &e, int u, const float4 *xs,
                                       const float (&xh)[NB][2], float (&acc)[NB]) {
    int xoff[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) xoff[b] = b * XSTRIDE;
    URegs<TYPE> g;
    if constexpr (TYPE == HD_TYPE_Q8_0) {
        g.a = s.a;
        g.b = s.b;
        g.d = s.d;
    } else if constexpr (TYPE == HD_TYPE_Q5_0) {
        g.a = s.a;
        g.qh = s.qh;
        g.d = s.d;
    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
        g.a = s.a;
        g.m = e.m;
    } else {
        g.a = s.a;
        g.h = s.h;
        g.d = e.d;
        // unit_fma reads byte (2(u&7)) & 3 of word 2(u&7) >> 2: place the two
        // scales there
        const uint32_t wsc = s.sc2 << (16 * (u & 1));
        g.sc = make_uint4(wsc, wsc, wsc, wsc);
    }
    unit_fma<TYPE, NB>(g, u, xs, xoff, &xh[0][0], 2, acc);
}

template <int TYPE, int NB>
__global__ void __launch_bounds__(32 * SK_MAX_WPB, SK_MIN_CTAS) k_qgemv_sk(SkArgs a) {
    constexpr int UMAX = 32 / NB;     // units of x staged per chunk (a multiple of 4)
    constexpr int XSTRIDE = UMAX * 8;  // float4 between batch rows in a warp's x slice
    extern __shared__ float4 sk_sm[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    float4 *xs = sk_sm + (size_t)wib * NB * XSTRIDE;  // [NB][UMAX][8]
    const int g = blockIdx.x * (blockDim.x >> 5) + wib;
    // The grid is whole CTAs: warps past the W that own the quads have no work
    // (warp-uniform exit; the kernel has no CTA barrier).
    if (g >= a.W) {
        pdl_trigger();
        return;
    }
    const int Q = a.Q, units = a.units, qpt = units / 4, rows = a.N;
    const int q0 = (int)((int64_t)g * Q / a.W), q1 = (int)((int64_t)(g + 1) * Q / a.W);

    // Load position: tile, first unit of the quad, ur = unit * rows + row.
    int ltile = q0 / qpt, lu = (q0 - ltile * qpt) * 4;
    int lrow = min(ltile * 32 + lane, rows - 1);
    uint32_t ur = (uint32_t)lu * rows + lrow;
    SkSlot<TYPE> ring[4];
    SkExtra<TYPE> ec, en;
    if (q0 < q1) {
        const uint32_t sr = (uint32_t)(lu >> 3) * rows + lrow;
#pragma unroll
        for (int k = 0; k < 4; k++) sk_load<TYPE>(a.w, ur + k * rows, sr, lu + k, ring[k]);
        sk_load_extra<TYPE>(a.w, sr, ec);
    }
    pdl_trigger();
    pdl_wait();

    int tile = ltile, u = lu;                                   // consumed position
    int seg0 = q0;                                              // segment start (quads)
    int seg1 = (tile + 1) * qpt < q1 ? (tile + 1) * qpt : q1;   // segment end
    int cbeg = q0, cend = q0;                                   // staged chunk (quads)
    float acc[NB], h0[NB], h1[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) acc[b] = h0[b] = h1[b] = 0.f;

    // The finished segment [seg0, seg1) of `tile`: y directly, or a partial.
    auto flush = [&]() {
        const int row = tile * 32 + lane;
        const int t0 = tile * qpt, t1 = t0 + qpt;
        float out[NB];
        bool write = false;
        if (seg0 == t0 && seg1 == t1) {
#pragma unroll
            for (int b = 0; b < NB; b++) out[b] = acc[b];
            write = true;
        } else {
            // warps owning the first and the last quad of the tile
            const int gf = (int)(((int64_t)(t0 + 1) * a.W - 1) / Q), gl = (int)(((int64_t)t1 * a.W - 1) / Q);
            const int nseg = gl - gf + 1, slot = g - gf;
            float *base = a.ws + (size_t)tile * a.maxseg * NB * 32;
#pragma unroll
            for (int b = 0; b < NB; b++) __stcg(base + ((size_t)slot * NB + b) * 32 + lane, acc[b]);
            __threadfence();
            __syncwarp();
            int last = 0;
            if (lane == 0) last = atomicAdd(a.tickets + tile, 1) == nseg - 1;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence();
#pragma unroll
                for (int b = 0; b < NB; b++) out[b] = 0.f;
                for (int k = 0; k < nseg; k++) {
#pragma unroll
                    for (int b = 0; b < NB; b++)
                        out[b] += k == slot ? acc[b] : __ldcg(base + ((size_t)k * NB + b) * 32 + lane);
                }
                if (lane == 0) a.tickets[tile] = 0;
                write = true;
            }
        }
        if (write && row < rows) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
                if (b < a.B) {
                    float o = out[b];
                    if (a.bias) o = o + a.bias[row];
                    if (a.residual) o = a.residual[(int64_t)b * rows + row] + o;
                    a.y[(int64_t)b * rows + row] = o;
                }
            }
        }
    };

    for (int q = q0; q < q1; q++) {
        if (q == cend) {  // chunk boundary (warp-uniform)
            if (q == seg1) {
                flush();
                tile++;
                u = 0;
                seg0 = q;
                seg1 = (tile + 1) * qpt < q1 ? (tile + 1) * qpt : q1;
#pragma unroll
                for (int b = 0; b < NB; b++) acc[b] = 0.f;
            }
            const int n = (seg1 - q) * 4 < UMAX ? (seg1 - q) * 4 : UMAX;  // units
            cbeg = q;
            cend = q + n / 4;
            __syncwarp();
            if (lane < n) {
                for (int b = 0; b < a.B; b++) {
                    const float4 *src = (const float4 *)(a.x + (int64_t)b * a.K + (int64_t)(u + lane) * 32);
                    float4 *dst = xs + b * XSTRIDE + lane * 8;
                    float hs[2];
#pragma unroll
                    for (int hf = 0; hf < 2; hf++) {  // one 16-value half at a time
                        float4 v[4];
#pragma unroll
                        for (int j = 0; j < 4; j++) v[j] = __ldg(src + 4 * hf + j);
                        float sx = 0.f;
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            sx += (v[j].x + v[j].y) + (v[j].z + v[j].w);
                            dst[4 * hf + j] = v[j];
                        }
                        hs[hf] = sx;
                    }
#pragma unroll
                    for (int bb = 0; bb < NB; bb++)
                        if (bb == b) {
                            h0[bb] = hs[0];
                            h1[bb] = hs[1];
                        }
                }
            }
            __syncwarp();
        }
        // advance the load position to the next quad
        const bool more = q + 1 < q1;
        lu += 4;
        if (lu == units) {
            lu = 0;
            ltile++;
            lrow = min(ltile * 32 + lane, rows - 1);
            ur = (uint32_t)lrow;
        } else {
            ur += 4u * rows;
        }
        const uint32_t srn = (uint32_t)(lu >> 3) * rows + lrow;
        if (more) sk_load_extra<TYPE>(a.w, srn, en);
        const int l0 = (q - cbeg) * 4;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            float xh[NB][2];
#pragma unroll
            for (int b = 0; b < NB; b++) {
                xh[b][0] = __shfl_sync(0xffffffffu, h0[b], l0 + k);
                xh[b][1] = __shfl_sync(0xffffffffu, h1[b], l0 + k);
            }
            sk_dot<TYPE, NB, XSTRIDE>(ring[k], ec, u + k, xs + (l0 + k) * 8, xh, acc);
            if (more) sk_load<TYPE>(a.w, ur + k * rows, srn, lu + k, ring[k]);
        }
        ec = en;
        u += 4;
    }
    flush();
}

// Resident CTAs per SM of one instance (per device: function attributes
// are per device).
constexpr int SK_MAX_DEV = 64;

template <int TYPE, int NB>
int sk_occupancy(int device, int wpb, size_t smem) {
    static int cache[SK_MAX_DEV][SK_MAX_WPB + 1];
    if (device < 0 || device >= SK_MAX_DEV || wpb < 1 || wpb > SK_MAX_WPB) return 0;
    int &c = cache[device][wpb];
    if (c) return c;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(k_qgemv_sk<TYPE, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
        return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_qgemv_sk<TYPE, NB>, 32 * wpb, smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    c = n;
    return n;
}

int env_int(const char *name, int dflt) {
    const char *v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}

template <int TYPE, int NB>
int launch_sk(hd_ctx *ctx, SkArgs a, const char *name) {
    const int wpb = env_int("HACEDLE_SK_WPB", 8);
    const int lmin = env_int("HACEDLE_SK_LMIN", 2);  // quads per warp, at least
    if (wpb < 1 || wpb > SK_MAX_WPB) return hd_fail(ctx, HD_E_ARG, "%s: HACEDLE_SK_WPB outside 1..8", name);
    const size_t smem = (size_t)wpb * 32 * 8 * sizeof(float4);  // NB x UMAX = 32 units of x per warp
    const int occ = sk_occupancy<TYPE, NB>(ctx->device, wpb, smem);
    if (occ < 1) return hd_fail(ctx, HD_E_CUDA, "%s: streamed GEMV does not fit on an SM", name);
    int64_t wmax = a.Q / (lmin > 0 ? lmin : 1);
    if (wmax < 1) wmax = 1;
    int64_t ctas = (int64_t)ctx->sm_count * occ;
    if (ctas * wpb > wmax) ctas = (wmax + wpb - 1) / wpb;
    a.W = (int)(ctas * wpb);
    if (a.W > a.Q) a.W = a.Q;  // every warp owns at least one quad
    // slots per tile: segments of at least floor(Q / W) quads each
    const int64_t lseg = a.Q / a.W, qpt = a.units / 4;
    a.maxseg = (int)((qpt + lseg - 1) / lseg + 1);
    int rc = hd_ensure_workspace(ctx, (size_t)a.tiles * a.maxseg * NB * 32 * sizeof(float), (size_t)a.tiles);
    if (rc) return rc;
    a.ws = (float *)ctx->ws;
    a.tickets = ctx->tickets;
    cudaError_t e = hd_launch(ctx, k_qgemv_sk<TYPE, NB>, dim3((unsigned)ctas), dim3(32 * wpb), smem, a);
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "%s: %s", name, cudaGetErrorString(e));
    return HD_OK;
}

}  // namespace

// Whether the streamed kernel takes this weight: rows of whole quads, and
// unit * row offsets in 32 bits.
bool hd_qgemv_sk_fits(const hd_weight *w) {
    return w->units % 4 == 0 && (int64_t)w->units * w->rows < ((int64_t)1 << 31);
}

// Streamed Q-GEMV, batch 1..4 (y = W x (+bias, +residual)).
int hd_qgemv_sk(hd_ctx *ctx, const hd_weight *w, const float *x, float *y, int B, const float *bias,
                const float *residual, const char *name) {
    HD_REQUIRE(ctx, hd_qgemv_sk_fits(w), HD_E_SHAPE, "%s: streamed GEMV needs cols %% 128 == 0", name);
    SkArgs a;
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
        rc = nb == 1 ? launch_sk<TT, 1>(ctx, a, name) : nb == 2 ? launch_sk<TT, 2>(ctx, a, name)
                                                                : launch_sk<TT, 4>(ctx, a, name);
    });
    return rc;
}
