// hd_gemm_f32.cu -- fp32 CUDA-core GEMMs: the exact-weight prefill Q-GEMM
// (HD_PREC_FP32: each weight is dequantized bit-exactly, then multiplied in
// fp32) and the dense f32 matmul of the graph executor.
#include <cstdlib>

#include "hd_internal.cuh"

int hd_qgemm_tc(hd_ctx *ctx, const hd_weight *w, const float *X, float *Y, int T, int exact);
int hd_tc4_min_t();
int hd_qgemm_rows_f32(hd_ctx *ctx, const hd_weight *w, const float *X, float *Y, int T);
int hd_ensure_hbuf(hd_ctx *ctx, float **buf, size_t *have, size_t need);

namespace {

constexpr int BN = 128, BT = 64;

// Y[t][n] = sum_k X[t][k] W[n][k]; CTA tile 128 weight rows x 64 tokens,
// 256 threads with 8 rows x 4 tokens each; K advances one 32-value unit per
// step.  Threads 0..127 dequantize one row's unit each into shared memory,
// threads 128..255 stage the activations.
template <int TYPE>
__global__ void __launch_bounds__(256) k_qgemm_f32(WView w, const float *__restrict__ X, float *__restrict__ Y, int T,
                                                  int N) {
    __shared__ __align__(16) float Ws[32][BN];
    __shared__ __align__(16) float Xs[32][BT];
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int n0 = blockIdx.x * BN, t0 = blockIdx.y * BT;
    const int K = w.units * 32;
    float acc[4][8];
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
        for (int i = 0; i < 8; i++) acc[j][i] = 0.f;
    for (int u = 0; u < w.units; u++) {
        if (tid < BN) {
            float v[32];
            int64_t n = n0 + tid;
            if (n < N) decode_unit_exact<TYPE>(w, n, u, v);
            else {
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] = 0.f;
            }
#pragma unroll
            for (int j = 0; j < 32; j++) Ws[j][tid] = v[j];
        } else {
            for (int q = tid - BN; q < BT * 8; q += 256 - BN) {
                int t = q >> 3, c4 = q & 7;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (t0 + t < T) v = __ldg((const float4 *)(X + (int64_t)(t0 + t) * K + u * 32) + c4);
                Xs[4 * c4 + 0][t] = v.x;
                Xs[4 * c4 + 1][t] = v.y;
                Xs[4 * c4 + 2][t] = v.z;
                Xs[4 * c4 + 3][t] = v.w;
            }
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < 32; k++) {
            float4 w0 = *(const float4 *)&Ws[k][tx * 8], w1 = *(const float4 *)&Ws[k][tx * 8 + 4];
            float4 xv = *(const float4 *)&Xs[k][ty * 4];
            float wr[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            float xr[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int i = 0; i < 8; i++) acc[j][i] = fmaf(xr[j], wr[i], acc[j][i]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
        int t = t0 + ty * 4 + j;
        if (t >= T) continue;
        float *yr = Y + (int64_t)t * N + n0 + tx * 8;
        if (n0 + tx * 8 + 8 <= N && (N & 3) == 0) {
            ((float4 *)yr)[0] = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
            ((float4 *)yr)[1] = make_float4(acc[j][4], acc[j][5], acc[j][6], acc[j][7]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++)
                if (n0 + tx * 8 + i < N) yr[i] = acc[j][i];
        }
    }
}

// Dense out[m][n] = sum_k a[m][k] b[k][n]; 64x64 tile, 4x4 per thread.
__global__ void __launch_bounds__(256) k_matmul_f32(const float *__restrict__ a, const float *__restrict__ b,
                                                   float *__restrict__ out, int64_t m, int64_t n, int64_t k) {
    __shared__ float As[16][64 + 1];
    __shared__ float Bs[16][64];
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = (int64_t)blockIdx.y * 64, n0 = (int64_t)blockIdx.x * 64;
    float acc[4][4] = {};
    for (int64_t k0 = 0; k0 < k; k0 += 16) {
        for (int i = tid; i < 64 * 16; i += 256) {
            int r = i / 16, c = i % 16;
            int64_t gm = m0 + r, gk = k0 + c;
            As[c][r] = (gm < m && gk < k) ? a[gm * k + gk] : 0.f;
            int rb = i / 64, cb = i % 64;
            int64_t gk2 = k0 + rb, gn = n0 + cb;
            Bs[rb][cb] = (gk2 < k && gn < n) ? b[gk2 * n + gn] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; kk++) {
            float ar[4], br[4];
#pragma unroll
            for (int i = 0; i < 4; i++) ar[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; j++) br[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int64_t gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
            if (gm < m && gn < n) out[gm * n + gn] = acc[i][j];
        }
}

}  // namespace

int hd_qgemm_f32(hd_ctx *ctx, const hd_weight *w, const float *X, float *Y, int T) {
    dim3 grid((unsigned)((w->rows + BN - 1) / BN), (unsigned)((T + BT - 1) / BT));
    WView v = wview(w);
    cudaError_t e = cudaSuccess;
    HD_TYPE_SWITCH(w->type, TT, e = hd_launch(ctx, k_qgemm_f32<TT>, grid, dim3(256), 0, v, X, Y, T, (int)w->rows));
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_qgemm: %s", cudaGetErrorString(e));
    return HD_OK;
}

extern "C" int hd_qgemm(hd_ctx *ctx, const hd_weight *w, const float *X, float *Y, int T, int precision) {
    if (!ctx || !w || !X || !Y) return hd_fail(ctx, HD_E_ARG, "hd_qgemm: null argument");
    HD_REQUIRE(ctx, T >= 0, HD_E_ARG, "hd_qgemm: T < 0");
    HD_REQUIRE(ctx, ((uintptr_t)X & 15) == 0 && ((uintptr_t)Y & 15) == 0, HD_E_ARG,
               "hd_qgemm: X and Y must be 16-byte aligned");
    if (T == 0) return HD_OK;
    if (precision == HD_PREC_FP32) {
        // More than 16 rows and a weight the exact-product tensor-core mode
        // takes (rows % 128 == 0 for the streamed kernel, any rows for the
        // two-pass kernel): exact weights and x as fp16 hi + lo, 3 MMAs per
        // product, fp32 accumulation.  Otherwise: up to 1024 rows, groups of
        // 16 rows on the batch Q-GEMV kernel; beyond, the 128 x 64 tiled
        // kernel.  HACEDLE_FP32_CUDA_CORES=1 keeps fp32 products on the CUDA
        // cores.
        const int min_t = hd_tc4_min_t();
        if (T > 16 && (w->rows % 128 == 0 || (min_t > 0 && T >= min_t)) &&
            getenv("HACEDLE_FP32_CUDA_CORES") == nullptr)
            return hd_qgemm_tc(ctx, w, X, Y, T, 1);
        const char *lim = getenv("HACEDLE_ROWS_GEMV_MAX");
        const int maxrows = lim ? atoi(lim) : 1024;
        if (T <= maxrows) return hd_qgemm_rows_f32(ctx, w, X, Y, T);
        return hd_qgemm_f32(ctx, w, X, Y, T);
    }
    if (precision == HD_PREC_BF16_TC) return hd_qgemm_tc(ctx, w, X, Y, T, 0);
    return hd_fail(ctx, HD_E_ARG, "hd_qgemm: unknown precision %d", precision);
}

extern "C" int hd_qgemm_host(hd_ctx *ctx, const hd_weight *w, const float *X_host, float *Y_host, int T,
                             int precision) {
    if (!ctx || !w || !X_host || !Y_host) return hd_fail(ctx, HD_E_ARG, "hd_qgemm_host: null argument");
    size_t xb = (size_t)T * w->cols * sizeof(float), yb = (size_t)T * w->rows * sizeof(float);
    int rc = hd_ensure_hbuf(ctx, &ctx->hbuf_x, &ctx->hbuf_x_bytes, xb);
    if (!rc) rc = hd_ensure_hbuf(ctx, &ctx->hbuf_y, &ctx->hbuf_y_bytes, yb);
    if (rc) return rc;
    HD_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->hbuf_x, X_host, xb, cudaMemcpyHostToDevice, ctx->stream));
    rc = hd_qgemm(ctx, w, ctx->hbuf_x, ctx->hbuf_y, T, precision);
    if (rc) return rc;
    HD_CUDA_TRY(ctx, cudaMemcpyAsync(Y_host, ctx->hbuf_y, yb, cudaMemcpyDeviceToHost, ctx->stream));
    return hd_ctx_check_device_errors(ctx);
}

namespace {

// dst [C][R] = src [R][C] transposed, 32 x 32 tiles through shared memory
// (one padding column, so the column reads do not share banks).
__global__ void __launch_bounds__(256) k_transpose(const float *__restrict__ src, float *__restrict__ dst, int64_t R,
                                                   int64_t C) {
    __shared__ float tile[32][33];
    pdl_wait();
    pdl_trigger();
    const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int i = ty; i < 32; i += 8) {
        const int64_t r = r0 + i, c = c0 + tx;
        if (r < R && c < C) tile[i][tx] = src[r * C + c];
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int64_t c = c0 + i, r = r0 + tx;
        if (r < R && c < C) dst[c * R + r] = tile[tx][i];
    }
}

int transpose(hd_ctx *ctx, const float *src, float *dst, int64_t R, int64_t C) {
    if (R == 0 || C == 0) return HD_OK;
    HD_REQUIRE(ctx, (R + 31) / 32 < 65536, HD_E_SHAPE, "transpose: %lld rows", (long long)R);
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_transpose, dim3((unsigned)((C + 31) / 32), (unsigned)((R + 31) / 32)), dim3(256),
                               0, src, dst, R, C));
    return HD_OK;
}

}  // namespace

// Y [N][T] = W X for X [K][T] (the [k, n] operand layout of
// ComputeBackend::matmul_q4k/q6k): X is copied to token-major [T][K] on the
// device, hd_qgemm runs, and its [T][N] result is copied to [N][T].
extern "C" int hd_qgemm_kt(hd_ctx *ctx, const hd_weight *w, const float *X_kt, float *Y_nt, int T, int precision) {
    if (!ctx || !w || !X_kt || !Y_nt) return hd_fail(ctx, HD_E_ARG, "hd_qgemm_kt: null argument");
    HD_REQUIRE(ctx, T >= 0, HD_E_ARG, "hd_qgemm_kt: T < 0");
    if (T == 0) return HD_OK;
    const size_t xb = (size_t)T * w->cols * sizeof(float), yb = (size_t)T * w->rows * sizeof(float);
    int rc = hd_ensure_hbuf(ctx, &ctx->kt_x, &ctx->kt_x_bytes, xb);
    if (!rc) rc = hd_ensure_hbuf(ctx, &ctx->kt_y, &ctx->kt_y_bytes, yb);
    if (!rc) rc = transpose(ctx, X_kt, ctx->kt_x, w->cols, T);
    if (!rc) rc = hd_qgemm(ctx, w, ctx->kt_x, ctx->kt_y, T, precision);
    if (!rc) rc = transpose(ctx, ctx->kt_y, Y_nt, T, w->rows);
    return rc;
}

extern "C" int hd_qgemm_kt_host(hd_ctx *ctx, const hd_weight *w, const float *X_kt_host, float *Y_nt_host, int T,
                                int precision) {
    if (!ctx || !w || !X_kt_host || !Y_nt_host) return hd_fail(ctx, HD_E_ARG, "hd_qgemm_kt_host: null argument");
    HD_REQUIRE(ctx, T >= 0, HD_E_ARG, "hd_qgemm_kt_host: T < 0");
    if (T == 0) return HD_OK;
    const size_t xb = (size_t)T * w->cols * sizeof(float), yb = (size_t)T * w->rows * sizeof(float);
    int rc = hd_ensure_hbuf(ctx, &ctx->hbuf_x, &ctx->hbuf_x_bytes, xb);
    if (!rc) rc = hd_ensure_hbuf(ctx, &ctx->hbuf_y, &ctx->hbuf_y_bytes, yb);
    if (rc) return rc;
    HD_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->hbuf_x, X_kt_host, xb, cudaMemcpyHostToDevice, ctx->stream));
    rc = hd_qgemm_kt(ctx, w, ctx->hbuf_x, ctx->hbuf_y, T, precision);
    if (rc) return rc;
    HD_CUDA_TRY(ctx, cudaMemcpyAsync(Y_nt_host, ctx->hbuf_y, yb, cudaMemcpyDeviceToHost, ctx->stream));
    HD_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return hd_ctx_check_device_errors(ctx);
}

extern "C" int hd_matmul_f32(hd_ctx *ctx, const float *a, const float *b, float *out, int64_t m, int64_t n,
                             int64_t k) {
    if (!ctx || !a || !b || !out) return hd_fail(ctx, HD_E_ARG, "hd_matmul_f32: null argument");
    HD_REQUIRE(ctx, m >= 0 && n >= 0 && k >= 0 && m < (1ll << 31) * 64, HD_E_SHAPE, "hd_matmul_f32: bad shape");
    if (m == 0 || n == 0) return HD_OK;
    dim3 grid((unsigned)((n + 63) / 64), (unsigned)((m + 63) / 64));
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_matmul_f32, grid, dim3(256), 0, a, b, out, m, n, k));
    return HD_OK;
}
