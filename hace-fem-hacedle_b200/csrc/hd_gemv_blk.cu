// hd_gemv_blk.cu -- decode Q-GEMV for large matrices at batch <= 4 in blocks
// laid over the weight's storage order: y[b] = W x[b] (+bias, +residual).
//
// Why.  In the unit-major layout one unit of consecutive rows is contiguous.
// A CTA here is 8 warps on 8 adjacent 32-row tiles (lane = row) times a
// group of UG consecutive units, so for every unit it reads 8 x 512 bytes =
// 4 KB of contiguous weight, and short-lived CTAs sweep the matrix the way a
// streaming copy does.  Measured on B200 in CUDA-graph chains of launches over
// weight copies larger than L2, read-only walks of 34-68 MB moved 4.3-5.2 TB/s
// in this pattern against 3.4 TB/s for a persistent warp-range walk (each
// warp's consecutive units 512 bytes apart at a stride of rows x 16 bytes).
//
// Loads.  Before griddepcontrol.wait every lane issues cp.async copies of
// its row's UG units (16-byte quant chunks, Q5_0's 4-byte high bits, Q6_K's
// 8-byte high bits, Q4_K's 16-byte super-block header) into shared memory,
// and loads the 2-byte scales into registers: the whole block is in flight
// at once with few registers.  Rows past N load row N - 1 (valid memory;
// their sums are never stored).
//
// Activations.  The group's x (UG units x B rows) and its 16-value half sums
// (which carry the quant offsets, unit_fma) are staged once per CTA.
//
// Reduction.  With one group the CTA writes y.  Otherwise each CTA writes its
// partial row sums to the workspace [group][NB][N] and the CTA that takes a
// row block's last ticket adds the groups in group order -- fixed orders, so
// results are bitwise reproducible.
#include <cstdlib>

#include "hd_internal.cuh"
#include "hd_units.cuh"

namespace {

constexpr int BK_WARPS = 8;  // 32-row tiles per CTA

template <int TYPE>
struct BkUg {
    static constexpr int value = TYPE == HD_TYPE_Q8_0 ? 4 : 8;  // units per group
};

struct BlkArgs {
    WView w;
    const float *x;         // [B][K]
    float *y;               // [B][N]
    const float *bias;      // [N] or null
    const float *residual;  // [B][N] or null
    int B, N, K, units, G;  // G: unit groups (gridDim.y)
    float *ws;              // [G][NB][N] partial row sums
    int *tickets;           // [row blocks], zero between launches
};

// Shared-memory bytes per (unit, row) of the staged copies, and per row of
// the super-block header.
template <int TYPE>
struct BkStage {
    static constexpr int Q = TYPE == HD_TYPE_Q8_0 ? 32 : 16;  // quants
    static constexpr int A = TYPE == HD_TYPE_Q5_0 ? 4 : TYPE == HD_TYPE_Q6_K ? 8 : 0;  // high bits
    static constexpr int H = TYPE == HD_TYPE_Q4_K ? 16 : 0;  // super-block header
};

__device__ __forceinline__ uint32_t bk_smem(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void bk_cp16(uint32_t s, const void *g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(g) : "memory");
}
__device__ __forceinline__ void bk_cp8(uint32_t s, const void *g) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(g) : "memory");
}
__device__ __forceinline__ void bk_cp4(uint32_t s, const void *g) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(g) : "memory");
}

template <int TYPE, int NB>
__global__ void __launch_bounds__(32 * BK_WARPS) k_qgemv_blk(BlkArgs a) {
    constexpr int UG = BkUg<TYPE>::value;
    using ST = BkStage<TYPE>;
    constexpr int ROWS = 32 * BK_WARPS;
    extern __shared__ __align__(16) unsigned char bk_sm[];
    // [UG][ROWS][Q] quants, [UG][ROWS][A] high bits, [ROWS][H] header,
    // x [NB][UG][32] floats, half sums [NB][UG][2]
    unsigned char *sq = bk_sm;
    unsigned char *sa = sq + UG * ROWS * ST::Q;
    unsigned char *sh = sa + UG * ROWS * ST::A;
    float *sx = (float *)(sh + ROWS * ST::H);
    float *sxh = sx + NB * UG * 32;
    const int t = threadIdx.x;
    const int rb = blockIdx.x, grp = blockIdx.y;
    const int row = rb * ROWS + t;  // warp wib, lane: tile rb * 8 + wib
    const int lrow = row < a.N ? row : a.N - 1;
    const int u0 = grp * UG, nu = a.units - u0 < UG ? a.units - u0 : UG;
    const WView w = a.w;

    uint32_t d16[UG];  // Q8_0 / Q5_0 unit scales, Q6_K the units' two sub-block scales
    uint32_t d6 = 0;   // Q6_K super-block scale
#pragma unroll
    for (int k = 0; k < UG; k++) {
        d16[k] = 0;
        if (k < nu) {
            const uint32_t ur = (uint32_t)(u0 + k) * a.N + lrow;
            if constexpr (TYPE == HD_TYPE_Q8_0) {
                bk_cp16(bk_smem(sq + (k * ROWS + t) * 32), w.q + (size_t)ur * 32);
                bk_cp16(bk_smem(sq + (k * ROWS + t) * 32 + 16), w.q + (size_t)ur * 32 + 16);
                d16[k] = __ldg((const unsigned short *)w.meta + ur);
            } else {
                bk_cp16(bk_smem(sq + (k * ROWS + t) * 16), w.q + (size_t)ur * 16);
                if constexpr (TYPE == HD_TYPE_Q5_0) {
                    bk_cp4(bk_smem(sa + (k * ROWS + t) * 4), w.aux + (size_t)ur * 4);
                    d16[k] = __ldg((const unsigned short *)w.meta + ur);
                } else if constexpr (TYPE == HD_TYPE_Q6_K) {
                    bk_cp8(bk_smem(sa + (k * ROWS + t) * 8), w.aux + (size_t)ur * 8);
                    const uint32_t sr = (uint32_t)((u0 + k) >> 3) * a.N + lrow;
                    d16[k] = __ldg((const unsigned short *)(w.meta + (size_t)sr * 16) + ((u0 + k) & 7));
                }
            }
        }
    }
    if constexpr (TYPE == HD_TYPE_Q4_K || TYPE == HD_TYPE_Q6_K) {  // a group lies in one super-block
        const uint32_t sr = (uint32_t)(u0 >> 3) * a.N + lrow;
        if constexpr (TYPE == HD_TYPE_Q4_K) bk_cp16(bk_smem(sh + t * 16), w.meta + (size_t)sr * 16);
        if constexpr (TYPE == HD_TYPE_Q6_K) d6 = __ldg(w.dsb + sr);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    pdl_trigger();
    pdl_wait();

    // x of the group and its half sums (fixed order), for every batch row
    for (int i = t; i < a.B * nu * 8; i += ROWS) {
        const int b = i / (nu * 8), r = i - b * nu * 8, k = r >> 3, j = r & 7;
        ((float4 *)sx)[(b * UG + k) * 8 + j] = __ldg((const float4 *)(a.x + (int64_t)b * a.K + (int64_t)(u0 + k) * 32) + j);
    }
    __syncthreads();
    for (int i = t; i < a.B * nu * 2; i += ROWS) {
        const int b = i / (nu * 2), r = i - b * nu * 2, k = r >> 1, hf = r & 1;
        const float4 *p = (const float4 *)sx + (b * UG + k) * 8 + 4 * hf;
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) s += (p[j].x + p[j].y) + (p[j].z + p[j].w);
        sxh[(b * UG + k) * 2 + hf] = s;
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();

    int xoff[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) xoff[b] = b < a.B ? b * UG * 8 : 0;
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) acc[b] = 0.f;
#pragma unroll
    for (int k = 0; k < UG; k++) {
        if (k < nu) {
            URegs<TYPE> g;
            if constexpr (TYPE == HD_TYPE_Q8_0) {
                g.a = *(const uint4 *)(sq + (k * ROWS + t) * 32);
                g.b = *(const uint4 *)(sq + (k * ROWS + t) * 32 + 16);
                g.d = d16[k];
            } else if constexpr (TYPE == HD_TYPE_Q5_0) {
                g.a = *(const uint4 *)(sq + (k * ROWS + t) * 16);
                g.qh = *(const uint32_t *)(sa + (k * ROWS + t) * 4);
                g.d = d16[k];
            } else if constexpr (TYPE == HD_TYPE_Q4_K) {
                g.a = *(const uint4 *)(sq + (k * ROWS + t) * 16);
                g.m = *(const uint4 *)(sh + t * 16);
            } else {
                g.a = *(const uint4 *)(sq + (k * ROWS + t) * 16);
                g.h = *(const uint2 *)(sa + (k * ROWS + t) * 8);
                g.d = d6;
                // unit_fma reads byte (2(u&7)) & 3 of word 2(u&7) >> 2
                const uint32_t wsc = d16[k] << (16 * ((u0 + k) & 1));
                g.sc = make_uint4(wsc, wsc, wsc, wsc);
            }
            unit_fma<TYPE, NB>(g, u0 + k, (const float4 *)sx + k * 8, xoff, sxh + k * 2, UG * 2, acc);
        }
    }

    if (a.G == 1) {
        if (row < a.N) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
                if (b < a.B) {
                    float o = acc[b];
                    if (a.bias) o = o + a.bias[row];
                    if (a.residual) o = a.residual[(int64_t)b * a.N + row] + o;
                    a.y[(int64_t)b * a.N + row] = o;
                }
            }
        }
        return;
    }
    // partial row sums, then the row block's last CTA adds the groups in order
    if (row < a.N) {
#pragma unroll
        for (int b = 0; b < NB; b++)
            if (b < a.B) __stcg(a.ws + ((size_t)grp * NB + b) * a.N + row, acc[b]);
    }
    // One fence after the barrier: the barrier makes the CTA's partial stores
    // visible to thread 0, and its gpu-scope fence (cumulative) orders them
    // before the ticket.
    __syncthreads();
    __shared__ int last;
    if (t == 0) {
        __threadfence();
        last = atomicAdd(a.tickets + rb, 1) == a.G - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (row < a.N) {
#pragma unroll
        for (int b = 0; b < NB; b++) {
            if (b < a.B) {
                float s = 0.f;
                for (int gg = 0; gg < a.G; gg++) s += gg == grp ? acc[b] : __ldcg(a.ws + ((size_t)gg * NB + b) * a.N + row);
                if (a.bias) s = s + a.bias[row];
                if (a.residual) s = a.residual[(int64_t)b * a.N + row] + s;
                a.y[(int64_t)b * a.N + row] = s;
            }
        }
    }
    if (t == 0) a.tickets[rb] = 0;
}

template <int TYPE, int NB>
size_t blk_smem() {
    using ST = BkStage<TYPE>;
    constexpr int UG = BkUg<TYPE>::value, ROWS = 32 * BK_WARPS;
    return (size_t)UG * ROWS * (ST::Q + ST::A) + (size_t)ROWS * ST::H + (size_t)NB * UG * 32 * 4 + NB * UG * 2 * 4;
}

template <int TYPE, int NB>
int launch_blk(hd_ctx *ctx, BlkArgs a, const char *name) {
    const size_t smem = blk_smem<TYPE, NB>();
    static bool attr[64] = {};
    if (ctx->device >= 0 && ctx->device < 64 && !attr[ctx->device]) {
        cudaError_t e = cudaFuncSetAttribute(k_qgemv_blk<TYPE, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "%s: %s", name, cudaGetErrorString(e));
        attr[ctx->device] = true;
    }
    const int rbs = (a.N + 32 * BK_WARPS - 1) / (32 * BK_WARPS);
    if (a.G > 1) {
        int rc = hd_ensure_workspace(ctx, (size_t)a.G * NB * a.N * sizeof(float), (size_t)rbs);
        if (rc) return rc;
        a.ws = (float *)ctx->ws;
        a.tickets = ctx->tickets;
    }
    cudaError_t e = hd_launch(ctx, k_qgemv_blk<TYPE, NB>, dim3((unsigned)rbs, (unsigned)a.G), dim3(32 * BK_WARPS),
                              smem, a);
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "%s: %s", name, cudaGetErrorString(e));
    return HD_OK;
}

}  // namespace

// Whether the block kernel takes this weight: a group of 8 units lies in one
// super-block (K-quants have 8 units per super-block, so always), unit * row
// offsets fit 32 bits, and at most 65535 unit groups.
bool hd_qgemv_blk_fits(const hd_weight *w) {
    const int ug = w->type == HD_TYPE_Q8_0 ? 4 : 8;
    return (int64_t)w->units * w->rows < ((int64_t)1 << 31) && (w->units + ug - 1) / ug <= 65535 &&
           hd_type_supported(w->type);
}

int hd_qgemv_blk(hd_ctx *ctx, const hd_weight *w, const float *x, float *y, int B, const float *bias,
                 const float *residual, const char *name) {
    HD_REQUIRE(ctx, hd_qgemv_blk_fits(w), HD_E_SHAPE, "%s: the block GEMV does not take this weight", name);
    BlkArgs a;
    a.w = wview(w);
    a.x = x;
    a.y = y;
    a.bias = bias;
    a.residual = residual;
    a.B = B;
    a.N = (int)w->rows;
    a.K = (int)w->cols;
    a.units = w->units;
    const int ug = w->type == HD_TYPE_Q8_0 ? 4 : 8;
    a.G = (w->units + ug - 1) / ug;
    a.ws = nullptr;
    a.tickets = nullptr;
    const int nb = B <= 1 ? 1 : B <= 2 ? 2 : 4;
    int rc = HD_E_TYPE;
    HD_TYPE_SWITCH(w->type, TT, {
        rc = nb == 1 ? launch_blk<TT, 1>(ctx, a, name) : nb == 2 ? launch_blk<TT, 2>(ctx, a, name)
                                                                : launch_blk<TT, 4>(ctx, a, name);
    });
    return rc;
}
