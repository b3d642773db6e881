// hd_elementwise.cu -- RMSNorm, RoPE, softmax, SwiGLU, add and argmax.
// These are small HBM-bound kernels around the projections; each reads its
// inputs once and writes once.
#include <cfloat>

#include "hd_internal.cuh"

int hd_ensure_hbuf(hd_ctx *ctx, float **buf, size_t *have, size_t need);

namespace {

template <int NT>
__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float s = 0.f;
    if (w == 0) {
        s = l < NT / 32 ? red[l] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (l == 0) red[32] = s;
    }
    __syncthreads();
    return red[32];
}

template <int NT>
__device__ __forceinline__ float block_max(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        float s = l < NT / 32 ? red[l] : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, o));
        if (l == 0) red[32] = s;
    }
    __syncthreads();
    return red[32];
}

// One CTA per row.  mode 0: y = (x*w)*r (NativeBackend::rmsnorm order);
// mode 1: y = (x*r)*w (rmsnorm_f32 order).  r = 1/sqrt(ss/dim + eps).
template <int NT>
__global__ void __launch_bounds__(NT) k_rmsnorm(const float *__restrict__ x, const float *__restrict__ w,
                                                float *residual, float *__restrict__ y, int dim, float eps,
                                                int mode) {
    __shared__ float red[33];
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x;
    const float *xr = x + row * dim;
    float *rr = residual ? residual + row * dim : nullptr;
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += NT) {
        float v = xr[i];
        if (rr) {
            v = rr[i] + v;
            rr[i] = v;
        }
        ss = fmaf(v, v, ss);
    }
    ss = block_sum<NT>(ss, red);
    const float r = 1.0f / sqrtf(ss / (float)dim + eps);
    for (int i = threadIdx.x; i < dim; i += NT) {
        float v = rr ? rr[i] : xr[i];
        y[row * dim + i] = mode == 0 ? __fmul_rn(__fmul_rn(v, w[i]), r) : __fmul_rn(__fmul_rn(v, r), w[i]);
    }
}

// NEOX RoPE in place: one thread per (token, head, i < hd/2).
__global__ void k_rope_neox(float *x, const int32_t *__restrict__ pos, const float *__restrict__ freq, int tokens,
                            int heads, int hd) {
    pdl_wait();
    pdl_trigger();
    const int half = hd >> 1;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)tokens * heads * half) return;
    int i = (int)(idx % half);
    int64_t th = idx / half;
    int t = (int)(th / heads);
    float *v = x + th * hd;
    float angle = __fdiv_rn((float)pos[t], freq[i]);
    float c = cosf(angle), s = sinf(angle);
    float x0 = v[i], x1 = v[i + half];
    v[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    v[i + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

__global__ void k_rope_interleaved(const float *__restrict__ x, const float *__restrict__ cs,
                                   const float *__restrict__ sn, float *__restrict__ out, int64_t pairs) {
    pdl_wait();
    pdl_trigger();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= pairs) return;
    int64_t i0 = 2 * i, i1 = i0 + 1;
    float x0 = x[i0], x1 = x[i1], c = cs[i0], s = sn[i0];
    out[i0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    out[i1] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
}

template <int NT>
__global__ void __launch_bounds__(NT) k_softmax(float *x, int n) {
    __shared__ float red[33];
    pdl_wait();
    pdl_trigger();
    float *r = x + (int64_t)blockIdx.x * n;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += NT) m = fmaxf(m, r[i]);
    m = block_max<NT>(m, red);
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += NT) s += expf(r[i] - m);
    s = block_sum<NT>(s, red);
    for (int i = threadIdx.x; i < n; i += NT) r[i] = expf(r[i] - m) / s;
}

__global__ void k_swiglu(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ y,
                         int64_t n) {
    pdl_wait();
    pdl_trigger();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float gv = g[i];
    float s = gv / (1.0f + expf(-gv));
    y[i] = __fmul_rn(s, u[i]);
}

__global__ void k_add(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ y, int64_t n) {
    pdl_wait();
    pdl_trigger();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = a[i] + b[i];
}

// (value, index) ordering of ArgMaxSampler: larger value wins, the lower
// index wins a tie, NaN never wins.
__device__ __forceinline__ bool am_better(float v, int64_t i, float bv, int64_t bi) {
    return v > bv || (v == bv && i < bi);
}

// Two-stage argmax: CTA (c, row) reduces chunk c of the row into a partial;
// the last CTA of the row (atomic ticket) reduces the partials.  A NaN at
// index 0 makes the sequential scan return 0 -- kept as a special case.
template <int NT>
__global__ void __launch_bounds__(NT) k_argmax(const float *__restrict__ x, int64_t n, int64_t chunk,
                                               float *pv, int64_t *pi, int *tickets, int32_t *out) {
    __shared__ float sv[NT];
    __shared__ int64_t si[NT];
    __shared__ int last;
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.y;
    const int c = blockIdx.x, nc = gridDim.x;
    const float *r = x + row * n;
    float bv = -INFINITY;
    int64_t bi = INT64_MAX;
    int64_t lo = (int64_t)c * chunk, hi = min(n, lo + chunk);
    for (int64_t i = lo + threadIdx.x; i < hi; i += NT) {
        float v = r[i];
        if (am_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int s = NT / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s && am_better(sv[threadIdx.x + s], si[threadIdx.x + s], sv[threadIdx.x], si[threadIdx.x])) {
            sv[threadIdx.x] = sv[threadIdx.x + s];
            si[threadIdx.x] = si[threadIdx.x + s];
        }
        __syncthreads();
    }
    if (nc == 1) {
        if (threadIdx.x == 0) {
            float x0 = r[0];
            out[row] = (n == 0 || x0 != x0 || si[0] == INT64_MAX) ? 0 : (int32_t)si[0];
        }
        return;
    }
    if (threadIdx.x == 0) {
        __stcg(pv + row * nc + c, sv[0]);
        __stcg((long long *)pi + row * nc + c, (long long)si[0]);
        __threadfence();
        last = (atomicAdd(tickets + row, 1) == nc - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    bv = -INFINITY;
    bi = INT64_MAX;
    for (int i = threadIdx.x; i < nc; i += NT) {
        float v = __ldcg(pv + row * nc + i);
        int64_t ii = (int64_t)__ldcg((const long long *)pi + row * nc + i);
        if (am_better(v, ii, bv, bi)) { bv = v; bi = ii; }
    }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int s = NT / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s && am_better(sv[threadIdx.x + s], si[threadIdx.x + s], sv[threadIdx.x], si[threadIdx.x])) {
            sv[threadIdx.x] = sv[threadIdx.x + s];
            si[threadIdx.x] = si[threadIdx.x + s];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        float x0 = r[0];
        out[row] = (x0 != x0 || si[0] == INT64_MAX) ? 0 : (int32_t)si[0];
        tickets[row] = 0;
    }
}

// dst[b][g*n + j] = src[g][b][j]: CTA (column block, b, g), no index
// division; float4 accesses when n % 4 == 0 and both buffers are 16-byte
// aligned (VEC = 4), else one float per thread.
template <int VEC>
__global__ void k_gather_columns(const float *__restrict__ src, float *__restrict__ dst, int G, int B, int64_t n) {
    pdl_wait();
    pdl_trigger();
    const int64_t j = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * VEC;
    if (j >= n) return;
    const int b = blockIdx.y, g = blockIdx.z;
    const float *s = src + ((int64_t)g * B + b) * n + j;
    float *d = dst + ((int64_t)b * G + g) * n + j;
    if constexpr (VEC == 4) *(float4 *)d = __ldg((const float4 *)s);
    else *d = __ldg(s);
}

inline unsigned blocks_for(int64_t n, int nt) { return (unsigned)((n + nt - 1) / nt); }

}  // namespace

extern "C" int hd_rmsnorm(hd_ctx *ctx, const float *x, const float *w, float *residual, float *y, int64_t rows,
                          int dim, float eps) {
    if (!ctx || !x || !w || !y) return hd_fail(ctx, HD_E_ARG, "hd_rmsnorm: null argument");
    HD_REQUIRE(ctx, rows >= 0 && dim > 0, HD_E_SHAPE, "hd_rmsnorm: bad shape");
    if (rows == 0) return HD_OK;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_rmsnorm<256>, dim3((unsigned)rows), dim3(256), 0, x, w, residual, y, dim, eps, 0));
    return HD_OK;
}

extern "C" int hd_rmsnorm_graph(hd_ctx *ctx, const float *x, const float *w, float *y, int64_t rows, int dim,
                                float eps) {
    if (!ctx || !x || !w || !y) return hd_fail(ctx, HD_E_ARG, "hd_rmsnorm_graph: null argument");
    HD_REQUIRE(ctx, rows >= 0 && dim > 0, HD_E_SHAPE, "hd_rmsnorm_graph: bad shape");
    if (rows == 0) return HD_OK;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_rmsnorm<256>, dim3((unsigned)rows), dim3(256), 0, x, w, (float *)nullptr, y,
                               dim, eps, 1));
    return HD_OK;
}

extern "C" int hd_rope_neox(hd_ctx *ctx, float *x, const int32_t *pos, int tokens, int heads, int head_dim,
                            float theta) {
    if (!ctx || !x || !pos) return hd_fail(ctx, HD_E_ARG, "hd_rope_neox: null argument");
    HD_REQUIRE(ctx, tokens >= 0 && heads > 0 && head_dim > 0 && head_dim % 2 == 0 && head_dim <= 1024, HD_E_SHAPE,
               "hd_rope_neox: bad shape");
    if (tokens == 0) return HD_OK;
    int rc = hd_ensure_rope(ctx, head_dim, theta);
    if (rc) return rc;
    int64_t n = (int64_t)tokens * heads * (head_dim / 2);
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_rope_neox, dim3(blocks_for(n, 256)), dim3(256), 0, x, pos,
                               (const float *)ctx->rope_freq, tokens, heads, head_dim));
    return HD_OK;
}

extern "C" int hd_rope_interleaved(hd_ctx *ctx, const float *x, const float *cs, const float *sn, float *out,
                                   int64_t rows, int last_dim) {
    if (!ctx || !x || !cs || !sn || !out) return hd_fail(ctx, HD_E_ARG, "hd_rope_interleaved: null argument");
    HD_REQUIRE(ctx, rows >= 0 && last_dim > 0 && last_dim % 2 == 0, HD_E_SHAPE,
               "hd_rope_interleaved: last dim must be even (RopeError::ShapeMismatch)");
    int64_t pairs = rows * (last_dim / 2);
    if (pairs == 0) return HD_OK;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_rope_interleaved, dim3(blocks_for(pairs, 256)), dim3(256), 0, x, cs, sn, out,
                               pairs));
    return HD_OK;
}

extern "C" int hd_softmax_rows(hd_ctx *ctx, float *x, int64_t rows, int n) {
    if (!ctx || !x) return hd_fail(ctx, HD_E_ARG, "hd_softmax_rows: null argument");
    if (rows <= 0 || n <= 0) return HD_OK;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_softmax<256>, dim3((unsigned)rows), dim3(256), 0, x, n));
    return HD_OK;
}

extern "C" int hd_swiglu(hd_ctx *ctx, const float *g, const float *u, float *y, int64_t n) {
    if (!ctx || !g || !u || !y) return hd_fail(ctx, HD_E_ARG, "hd_swiglu: null argument");
    if (n <= 0) return HD_OK;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_swiglu, dim3(blocks_for(n, 256)), dim3(256), 0, g, u, y, n));
    return HD_OK;
}

extern "C" int hd_add(hd_ctx *ctx, const float *a, const float *b, float *y, int64_t n) {
    if (!ctx || !a || !b || !y) return hd_fail(ctx, HD_E_ARG, "hd_add: null argument");
    if (n <= 0) return HD_OK;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_add, dim3(blocks_for(n, 256)), dim3(256), 0, a, b, y, n));
    return HD_OK;
}

extern "C" int hd_argmax_rows(hd_ctx *ctx, const float *x, int64_t rows, int64_t n, int32_t *idx) {
    if (!ctx || !idx || (n > 0 && !x)) return hd_fail(ctx, HD_E_ARG, "hd_argmax_rows: null argument");
    if (rows <= 0) return HD_OK;
    HD_REQUIRE(ctx, rows <= 65535, HD_E_SHAPE, "hd_argmax_rows: at most 65535 rows");
    if (n <= 0) {
        HD_CUDA_TRY(ctx, cudaMemsetAsync(idx, 0, rows * sizeof(int32_t), ctx->stream));
        return HD_OK;
    }
    int64_t chunk = 8192;
    int64_t nc = (n + chunk - 1) / chunk;
    if (nc > 256) {
        nc = 256;
        chunk = (n + nc - 1) / nc;
    }
    if (nc > 1) {
        int rc = hd_ensure_workspace(ctx, (size_t)rows * nc * (sizeof(float) + sizeof(int64_t)) + 64, (size_t)rows);
        if (rc) return rc;
    }
    float *pv = (float *)ctx->ws;
    int64_t *pi = (int64_t *)(pv + ((rows * nc + 1) & ~(int64_t)1));
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_argmax<256>, dim3((unsigned)nc, (unsigned)rows), dim3(256), 0, x, n, chunk, pv,
                               pi, ctx->tickets, idx));
    return HD_OK;
}

extern "C" int hd_gather_columns(hd_ctx *ctx, const float *src, float *dst, int G, int B, int64_t n) {
    if (!ctx || !src || !dst) return hd_fail(ctx, HD_E_ARG, "hd_gather_columns: null argument");
    HD_REQUIRE(ctx, G > 0 && B > 0 && n > 0, HD_E_SHAPE, "hd_gather_columns: bad shape");
    HD_REQUIRE(ctx, B <= 65535 && G <= 65535, HD_E_SHAPE, "hd_gather_columns: B and G at most 65535");
    const bool v4 = n % 4 == 0 && ((uintptr_t)src & 15) == 0 && ((uintptr_t)dst & 15) == 0;
    if (v4)
        HD_CUDA_TRY(ctx, hd_launch(ctx, k_gather_columns<4>, dim3(blocks_for(n / 4, 256), (unsigned)B, (unsigned)G),
                                   dim3(256), 0, src, dst, G, B, n));
    else
        HD_CUDA_TRY(ctx, hd_launch(ctx, k_gather_columns<1>, dim3(blocks_for(n, 256), (unsigned)B, (unsigned)G),
                                   dim3(256), 0, src, dst, G, B, n));
    return HD_OK;
}
