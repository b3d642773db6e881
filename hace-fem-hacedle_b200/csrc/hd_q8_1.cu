// hd_q8_1.cu -- the integer activation path: x quantized to 8-bit blocks of
// 32 (llama.cpp's Q8_1 idea, this library's block layout) and Q-GEMV on
// int8 dot products (dp4a) instead of fp32 FMAs.
//
// Block of 32 activations (48 bytes, 16-aligned):
//   int8 q[32]; float d; int16 s0, s1; 4 bytes zero
// with d = max|x| / 127, q = round-to-nearest-even(x * (1/d)) (all zero for
// an all-zero block), s0 / s1 = sum of q over values 0-15 / 16-31.
// Every weight type decodes a 32-value unit to small integers q_j (int8 in
// 4-byte words) with per-half scale a_h and offset b_h, w_j = a_h q_j - b_h:
//   Q8_0: q int8,  a = d,          b = 0
//   Q5_0: q 0..31, a = d,          b = 16 d
//   Q4_K: q 0..15, a = d sc,       b = dmin m
//   Q6_K: q 0..63, a_h = d sc_h,   b_h = 32 a_h   (halves = the 16-value sub-blocks)
// so that sum_j w_j x_j ~= d_x (a_0 dot_0 - b_0 s0 + a_1 dot_1 - b_1 s1), the
// dot_h being int32 dp4a sums over a half.  The reference has no such path
// (it is the next step after its i8 ops, ops/q_ops.rs:11-13 and
// ops/fused.rs:52-57); its accuracy contract is the bf16 one (2e-2 relative to
// the fp32 product), from the 1/254 rounding of the activations.
#include "hd_internal.cuh"

namespace {

struct __align__(16) XBlk {
    int8_t q[32];
    float d;
    int16_t s0, s1;
    int32_t pad;
};
static_assert(sizeof(XBlk) == 48, "Q8_1 block layout");

// One warp per 32-value block: lane j quantizes value j.
__global__ void k_quant_q8_1(const float *__restrict__ x, int64_t nblocks, XBlk *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int64_t blk = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (blk >= nblocks) return;
    const float v = x[blk * 32 + lane];
    float m = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float d = __fdiv_rn(m, 127.f);
    const float id = d > 0.f ? __fdiv_rn(1.f, d) : 0.f;
    const int q = __float2int_rn(__fmul_rn(v, id));
    int s = q;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);  // sums within each 16-lane half
    XBlk *b = out + blk;
    b->q[lane] = (int8_t)q;
    if (lane == 0) {
        b->d = d;
        b->s0 = (int16_t)s;
        b->pad = 0;
    }
    if (lane == 16) b->s1 = (int16_t)s;
}

// Unit u of row r as 8 words of int8 quants (values 0-15 in q[0..3], 16-31 in
// q[4..7]) and the per-half scale / offset.
template <int TYPE>
__device__ __forceinline__ void unit_int8(const WView &w, int64_t r, int u, uint32_t (&q)[8], float &a0, float &b0,
                                          float &a1, float &b1) {
    const int64_t ur = (int64_t)u * w.rows + r;
    if constexpr (TYPE == HD_TYPE_Q8_0) {
        const uint4 *p = (const uint4 *)(w.q + ur * 32);
        const uint4 x = __ldg(p), y = __ldg(p + 1);
        q[0] = x.x; q[1] = x.y; q[2] = x.z; q[3] = x.w;
        q[4] = y.x; q[5] = y.y; q[6] = y.z; q[7] = y.w;
        a0 = a1 = h2f(__ldg((const unsigned short *)w.meta + ur));
        b0 = b1 = 0.f;
    } else if constexpr (TYPE == HD_TYPE_Q5_0) {
        const uint4 x = __ldg((const uint4 *)(w.q + ur * 16));
        const uint32_t qh = __ldg((const unsigned int *)w.aux + ur);
        const uint32_t wd[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            q[i] = (wd[i] & 0x0F0F0F0Fu) | ((qh >> i) & 0x10101010u);
            q[4 + i] = ((wd[i] >> 4) & 0x0F0F0F0Fu) | ((qh << (4 - i)) & 0x10101010u);
        }
        a0 = a1 = h2f(__ldg((const unsigned short *)w.meta + ur));
        b0 = b1 = __fmul_rn(16.f, a0);
    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
        const uint4 x = __ldg((const uint4 *)(w.q + ur * 16));
        const uint4 m = __ldg((const uint4 *)(w.meta + ((int64_t)(u >> 3) * w.rows + r) * 16));
        int sc, mn;
        q4k_sm_regs(u & 7, m.y, m.z, m.w, sc, mn);
        const uint32_t wd[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            q[i] = wd[i] & 0x0F0F0F0Fu;
            q[4 + i] = (wd[i] >> 4) & 0x0F0F0F0Fu;
        }
        a0 = a1 = __fmul_rn(h2f((uint16_t)(m.x & 0xFFFF)), (float)sc);
        b0 = b1 = __fmul_rn(h2f((uint16_t)(m.x >> 16)), (float)mn);
    } else {
        const int64_t sr = (int64_t)(u >> 3) * w.rows + r;
        const uint4 x = __ldg((const uint4 *)(w.q + ur * 16));
        const uint2 h = __ldg((const uint2 *)w.aux + ur);
        const int8_t *scp = (const int8_t *)(w.meta + sr * 16);
        const float d = h2f(__ldg(w.dsb + sr));
        const int s0 = 2 * (u & 7);
        const uint32_t wd[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int sh = 4 - 2 * i;
            const uint32_t hx = sh >= 0 ? (h.x << sh) : (h.x >> -sh), hy = sh >= 0 ? (h.y << sh) : (h.y >> -sh);
            q[i] = (wd[i] & 0x0F0F0F0Fu) | (hx & 0x30303030u);
            q[4 + i] = ((wd[i] >> 4) & 0x0F0F0F0Fu) | (hy & 0x30303030u);
        }
        a0 = __fmul_rn(d, (float)__ldg(scp + s0));
        a1 = __fmul_rn(d, (float)__ldg(scp + s0 + 1));
        b0 = __fmul_rn(32.f, a0);
        b1 = __fmul_rn(32.f, a1);
    }
}

// grid (row blocks of 32, K chunks), QW warps per CTA (lane = weight row,
// warp = unit slot); warp w of chunk c takes the chunk's units w, w + QW, ...
// (one unit per warp when QW covers the chunk, so that every unit's loads are
// in flight at once); the QW warp sums meet in shared memory in warp order;
// with several chunks the last CTA of a row block (ticket) adds the chunk
// partials in chunk order, so results are reproducible.
template <int TYPE, int NB, int QW>
__global__ void __launch_bounds__(QW * 32) k_qgemv_q8_1(WView w, const XBlk *__restrict__ xq, float *__restrict__ y,
                                                        int B, int64_t N, int upc, float *ws, int *tickets) {
    extern __shared__ float red_raw[];
    float(*red)[NB][32] = reinterpret_cast<float(*)[NB][32]>(red_raw);  // [QW][NB][32]
    __shared__ int last;
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t r = (int64_t)blockIdx.x * 32 + lane;
    const int u0 = blockIdx.y * upc, u1 = min(w.units, u0 + upc);
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) acc[b] = 0.f;
    if (r < N) {
        for (int u = u0 + warp; u < u1; u += QW) {
            uint32_t q[8];
            float a0, b0, a1, b1;
            unit_int8<TYPE>(w, r, u, q, a0, b0, a1, b1);
#pragma unroll
            for (int b = 0; b < NB; b++) {
                if (b < B) {
                    const XBlk *xb = xq + (int64_t)b * w.units + u;
                    const uint4 x0 = __ldg((const uint4 *)xb), x1 = __ldg((const uint4 *)xb + 1);
                    const uint4 x2 = __ldg((const uint4 *)xb + 2);
                    int d0 = 0, d1 = 0;
                    d0 = __dp4a((int)q[0], (int)x0.x, d0);
                    d0 = __dp4a((int)q[1], (int)x0.y, d0);
                    d0 = __dp4a((int)q[2], (int)x0.z, d0);
                    d0 = __dp4a((int)q[3], (int)x0.w, d0);
                    d1 = __dp4a((int)q[4], (int)x1.x, d1);
                    d1 = __dp4a((int)q[5], (int)x1.y, d1);
                    d1 = __dp4a((int)q[6], (int)x1.z, d1);
                    d1 = __dp4a((int)q[7], (int)x1.w, d1);
                    const float dx = __uint_as_float(x2.x);
                    const int s0 = (int)(int16_t)(x2.y & 0xFFFF), s1 = (int)(int16_t)(x2.y >> 16);
                    const float h0 = __fsub_rn(__fmul_rn(a0, (float)d0), __fmul_rn(b0, (float)s0));
                    const float h1 = __fsub_rn(__fmul_rn(a1, (float)d1), __fmul_rn(b1, (float)s1));
                    acc[b] = __fadd_rn(acc[b], __fmul_rn(dx, __fadd_rn(h0, h1)));
                }
            }
        }
    }
#pragma unroll
    for (int b = 0; b < NB; b++) red[warp][b][lane] = acc[b];
    __syncthreads();
    // warp w finishes batch rows w, w + 8 (NB <= 16)
    for (int b = warp; b < B; b += QW) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < QW; j++) s = __fadd_rn(s, red[j][b][lane]);
        red[0][b][lane] = s;
    }
    __syncthreads();
    if (gridDim.y == 1) {
        if (warp == 0 && r < N)
            for (int b = 0; b < B; b++) y[(int64_t)b * N + r] = red[0][b][lane];
        return;
    }
    float *part = ws + ((int64_t)blockIdx.x * gridDim.y + blockIdx.y) * NB * 32;
    if (warp == 0)
        for (int b = 0; b < B; b++) __stcg(part + b * 32 + lane, red[0][b][lane]);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = (atomicAdd(tickets + blockIdx.x, 1) == (int)gridDim.y - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    const float *p0 = ws + (int64_t)blockIdx.x * gridDim.y * NB * 32;
    for (int b = warp; b < B; b += QW) {
        float s = 0.f;
        for (int c = 0; c < (int)gridDim.y; c++) s = __fadd_rn(s, __ldcg(p0 + (int64_t)c * NB * 32 + b * 32 + lane));
        if (r < N) y[(int64_t)b * N + r] = s;
    }
    if (threadIdx.x == 0) tickets[blockIdx.x] = 0;
}

template <int TYPE, int NB, int QW>
cudaError_t launch_q8w(hd_ctx *ctx, const hd_weight *w, const XBlk *xq, float *y, int B, int kc, int upc) {
    const int64_t rb = (w->rows + 31) / 32;
    const size_t smem = (size_t)QW * NB * 32 * sizeof(float);
    if (smem > 48 * 1024) {
        const cudaError_t e =
            cudaFuncSetAttribute(k_qgemv_q8_1<TYPE, NB, QW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return hd_launch(ctx, k_qgemv_q8_1<TYPE, NB, QW>, dim3((unsigned)rb, (unsigned)kc), dim3(QW * 32), smem, wview(w),
                     xq, y, B, w->rows, upc, (float *)ctx->ws, ctx->tickets);
}

template <int TYPE, int NB>
cudaError_t launch_q8(hd_ctx *ctx, const hd_weight *w, const XBlk *xq, float *y, int B, int kc, int upc) {
    return upc > 8 ? launch_q8w<TYPE, NB, 32>(ctx, w, xq, y, B, kc, upc) : launch_q8w<TYPE, NB, 8>(ctx, w, xq, y, B, kc, upc);
}

}  // namespace

extern "C" int hd_quantize_q8_1(hd_ctx *ctx, const float *x, int B, int64_t K, void *blocks_dev) {
    if (!ctx || !x || !blocks_dev) return hd_fail(ctx, HD_E_ARG, "hd_quantize_q8_1: null argument");
    HD_REQUIRE(ctx, B >= 0 && K > 0 && K % 32 == 0, HD_E_SHAPE, "hd_quantize_q8_1: K %lld must be a multiple of 32",
               (long long)K);
    HD_REQUIRE(ctx, ((uintptr_t)blocks_dev & 15) == 0, HD_E_ARG, "hd_quantize_q8_1: blocks must be 16-byte aligned");
    const int64_t nb = (int64_t)B * (K / 32);
    if (nb == 0) return HD_OK;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_quant_q8_1, dim3((unsigned)((nb * 32 + 255) / 256)), dim3(256), 0, x, nb,
                               (XBlk *)blocks_dev));
    return HD_OK;
}

extern "C" int hd_qgemv_q8_1(hd_ctx *ctx, const hd_weight *w, const void *blocks_dev, float *y, int B) {
    if (!ctx || !w || !blocks_dev || !y) return hd_fail(ctx, HD_E_ARG, "hd_qgemv_q8_1: null argument");
    HD_REQUIRE(ctx, B >= 1 && B <= 16, HD_E_ARG, "hd_qgemv_q8_1: batch %d outside 1..16", B);
    HD_REQUIRE(ctx, ((uintptr_t)blocks_dev & 15) == 0, HD_E_ARG, "hd_qgemv_q8_1: blocks must be 16-byte aligned");
    // K chunks so that about one CTA per SM is busy, at least 8 units each;
    // a chunk of more than 8 units runs 32 warps (one unit each up to 32)
    const int64_t rb = (w->rows + 31) / 32;
    int kc = (int)((ctx->sm_count + rb - 1) / rb);
    const int maxkc = (w->units + 7) / 8;
    kc = kc < 1 ? 1 : kc > maxkc ? maxkc : kc;
    const int upc = (w->units + kc - 1) / kc;
    kc = (w->units + upc - 1) / upc;
    if (kc > 1) {
        const int rc = hd_ensure_workspace(ctx, (size_t)rb * kc * 16 * 32 * sizeof(float), (size_t)rb);
        if (rc) return rc;
    }
    const XBlk *xq = (const XBlk *)blocks_dev;
    cudaError_t e = cudaSuccess;
    HD_TYPE_SWITCH(w->type, TT, {
        if (B == 1) e = launch_q8<TT, 1>(ctx, w, xq, y, B, kc, upc);
        else if (B <= 4) e = launch_q8<TT, 4>(ctx, w, xq, y, B, kc, upc);
        else if (B <= 8) e = launch_q8<TT, 8>(ctx, w, xq, y, B, kc, upc);
        else e = launch_q8<TT, 16>(ctx, w, xq, y, B, kc, upc);
    });
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_qgemv_q8_1: %s", cudaGetErrorString(e));
    return HD_OK;
}
