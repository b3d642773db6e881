// hd_weight.cu -- device weight handles: upload with re-layout, its inverse,
// bit-exact dequantization (QuantTensorView::dequantize) and embedding rows.
#include <cmath>
#include <cstring>

#include "hd_internal.cuh"

namespace {

__device__ __forceinline__ uint16_t ld16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// One thread per (row, unit): GGUF block bytes -> the unit-major arrays.
template <int TYPE>
__global__ void k_relayout(const uint8_t *__restrict__ src, WView w, uint8_t *q, uint8_t *aux, uint8_t *meta,
                           uint16_t *dsb) {
    pdl_wait();
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t total = w.rows * (int64_t)w.units;
    if (idx >= total) return;
    int64_t r = idx / w.units;
    int u = (int)(idx % w.units);
    int64_t ur = (int64_t)u * w.rows + r;
    if (TYPE == HD_TYPE_Q8_0) {
        const uint8_t *b = src + (r * w.units + u) * 34;
        for (int j = 0; j < 32; j++) q[ur * 32 + j] = b[2 + j];
        ((uint16_t *)meta)[ur] = ld16(b);
    } else if (TYPE == HD_TYPE_Q5_0) {
        const uint8_t *b = src + (r * w.units + u) * 22;
        uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
        for (int j = 0; j < 16; j++) q[ur * 16 + j] = b[6 + j];
        uint32_t qr = 0;
        for (int wd = 0; wd < 4; wd++)
            for (int c = 0; c < 4; c++) {
                qr |= ((qh >> (4 * wd + c)) & 1u) << (8 * c + 4 + wd);        // value 4wd+c
                qr |= ((qh >> (16 + 4 * wd + c)) & 1u) << (8 * c + wd);       // value 16+4wd+c
            }
        ((uint32_t *)aux)[ur] = qr;
        ((uint16_t *)meta)[ur] = ld16(b);
    } else if (TYPE == HD_TYPE_Q4_K) {
        int nsb = w.units / 8, sb = u >> 3, s = u & 7;
        const uint8_t *b = src + (r * nsb + sb) * 144;
        int c = s >> 1, hf = s & 1;
        for (int j = 0; j < 16; j++) {
            int lo = (b[16 + 32 * c + j] >> (4 * hf)) & 15;
            int hi = (b[16 + 32 * c + j + 16] >> (4 * hf)) & 15;
            q[ur * 16 + j] = (uint8_t)(lo | (hi << 4));
        }
        if (s == 0)
            for (int i = 0; i < 16; i++) meta[((int64_t)sb * w.rows + r) * 16 + i] = b[i];
    } else {  // Q6_K
        int nsb = w.units / 8, sb = u >> 3, s = u & 7;
        const uint8_t *b = src + (r * nsb + sb) * 210;
        int h = s >> 2, k = s & 3;
        uint32_t h0 = 0, h1 = 0;
        for (int j = 0; j < 16; j++) {
            int lo0 = (b[64 * h + 32 * (k & 1) + j] >> (k < 2 ? 0 : 4)) & 15;
            int lo1 = (b[64 * h + 32 * (k & 1) + j + 16] >> (k < 2 ? 0 : 4)) & 15;
            q[ur * 16 + j] = (uint8_t)(lo0 | (lo1 << 4));
            uint32_t hb0 = (b[128 + 32 * h + j] >> (2 * k)) & 3u;
            uint32_t hb1 = (b[128 + 32 * h + j + 16] >> (2 * k)) & 3u;
            int wd = j >> 2, cc = j & 3;
            h0 |= hb0 << (8 * cc + 2 * wd);
            h1 |= hb1 << (8 * cc + 2 * wd);
        }
        ((uint2 *)aux)[ur] = make_uint2(h0, h1);
        if (s == 0) {
            for (int i = 0; i < 16; i++) meta[((int64_t)sb * w.rows + r) * 16 + i] = b[192 + i];
            dsb[(int64_t)sb * w.rows + r] = ld16(b + 208);
        }
    }
}

// Inverse of k_relayout.  Q8_0/Q5_0: one thread per (row, unit); Q4_K/Q6_K:
// one thread per (row, super-block), since two units share GGUF bytes.
// Upper bound of |w| over one unit of one row (exact decoded values never
// exceed it), max-reduced as float bits (non-negative floats order as ints).
template <int TYPE>
__global__ void k_wbound(WView w, unsigned int *out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    float b = 0.f;
    if (i < w.rows * (int64_t)w.units) {
        const int u = (int)(i / w.rows);
        const int64_t r = i % w.rows, ur = (int64_t)u * w.rows + r;
        if constexpr (TYPE == HD_TYPE_Q8_0 || TYPE == HD_TYPE_Q5_0) {
            b = fabsf(h2f(((const uint16_t *)w.meta)[ur])) * (TYPE == HD_TYPE_Q8_0 ? 128.f : 16.f);
        } else if constexpr (TYPE == HD_TYPE_Q4_K) {
            const uint8_t *m = w.meta + ((int64_t)(u >> 3) * w.rows + r) * 16;
            int sc, mn;
            q4k_sm(u & 7, m + 4, sc, mn);
            b = fabsf(h2f(*(const uint16_t *)m)) * (float)sc * 15.f + fabsf(h2f(*(const uint16_t *)(m + 2))) * (float)mn;
        } else {
            const int64_t sr = (int64_t)(u >> 3) * w.rows + r;
            const int8_t *sc = (const int8_t *)(w.meta + sr * 16) + 2 * (u & 7);
            const float d = fabsf(h2f(w.dsb[sr]));
            b = d * 32.f * fmaxf(fabsf((float)sc[0]), fabsf((float)sc[1]));
        }
    }
    if (!(b == b)) b = INFINITY;
    for (int o = 16; o > 0; o >>= 1) b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, o));
    if ((threadIdx.x & 31) == 0 && b > 0.f) atomicMax(out, __float_as_uint(b));
}

template <int TYPE>
__global__ void k_unlayout(WView w, uint8_t *__restrict__ dst) {
    pdl_wait();
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool kq = (TYPE == HD_TYPE_Q4_K || TYPE == HD_TYPE_Q6_K);
    int per_row = kq ? w.units / 8 : w.units;
    if (idx >= w.rows * (int64_t)per_row) return;
    int64_t r = idx / per_row;
    int i = (int)(idx % per_row);
    if (TYPE == HD_TYPE_Q8_0) {
        int64_t ur = (int64_t)i * w.rows + r;
        uint8_t *b = dst + (r * w.units + i) * 34;
        uint16_t d = ((const uint16_t *)w.meta)[ur];
        b[0] = d & 255;
        b[1] = d >> 8;
        for (int j = 0; j < 32; j++) b[2 + j] = w.q[ur * 32 + j];
    } else if (TYPE == HD_TYPE_Q5_0) {
        int64_t ur = (int64_t)i * w.rows + r;
        uint8_t *b = dst + (r * w.units + i) * 22;
        uint16_t d = ((const uint16_t *)w.meta)[ur];
        uint32_t qr = ((const uint32_t *)w.aux)[ur], qh = 0;
        for (int wd = 0; wd < 4; wd++)
            for (int c = 0; c < 4; c++) {
                qh |= ((qr >> (8 * c + 4 + wd)) & 1u) << (4 * wd + c);
                qh |= ((qr >> (8 * c + wd)) & 1u) << (16 + 4 * wd + c);
            }
        b[0] = d & 255;
        b[1] = d >> 8;
        for (int k = 0; k < 4; k++) b[2 + k] = (qh >> (8 * k)) & 255;
        for (int j = 0; j < 16; j++) b[6 + j] = w.q[ur * 16 + j];
    } else if (TYPE == HD_TYPE_Q4_K) {
        uint8_t *b = dst + (r * per_row + i) * 144;
        for (int k = 0; k < 16; k++) b[k] = w.meta[((int64_t)i * w.rows + r) * 16 + k];
        for (int s = 0; s < 8; s++) {
            const uint8_t *q = w.q + ((int64_t)(8 * i + s) * w.rows + r) * 16;
            int c = s >> 1, hf = s & 1;
            for (int j = 0; j < 16; j++) {
                uint8_t v0 = q[j] & 15, v1 = q[j] >> 4;
                uint8_t *p0 = b + 16 + 32 * c + j, *p1 = p0 + 16;
                *p0 = hf ? (uint8_t)((*p0 & 0x0F) | (v0 << 4)) : (uint8_t)((*p0 & 0xF0) | v0);
                *p1 = hf ? (uint8_t)((*p1 & 0x0F) | (v1 << 4)) : (uint8_t)((*p1 & 0xF0) | v1);
            }
        }
    } else {  // Q6_K
        uint8_t *b = dst + (r * per_row + i) * 210;
        for (int k = 0; k < 192; k++) b[k] = 0;
        for (int s = 0; s < 8; s++) {
            int64_t ur = (int64_t)(8 * i + s) * w.rows + r;
            const uint8_t *q = w.q + ur * 16;
            uint2 hb = ((const uint2 *)w.aux)[ur];
            int h = s >> 2, k = s & 3;
            for (int j = 0; j < 16; j++) {
                int wd = j >> 2, cc = j & 3;
                uint8_t lo0 = q[j] & 15, lo1 = q[j] >> 4;
                uint8_t hb0 = (hb.x >> (8 * cc + 2 * wd)) & 3, hb1 = (hb.y >> (8 * cc + 2 * wd)) & 3;
                b[64 * h + 32 * (k & 1) + j] |= (uint8_t)(lo0 << (k < 2 ? 0 : 4));
                b[64 * h + 32 * (k & 1) + j + 16] |= (uint8_t)(lo1 << (k < 2 ? 0 : 4));
                b[128 + 32 * h + j] |= (uint8_t)(hb0 << (2 * k));
                b[128 + 32 * h + j + 16] |= (uint8_t)(hb1 << (2 * k));
            }
        }
        for (int k = 0; k < 16; k++) b[192 + k] = w.meta[((int64_t)i * w.rows + r) * 16 + k];
        uint16_t d = w.dsb[(int64_t)i * w.rows + r];
        b[208] = d & 255;
        b[209] = d >> 8;
    }
}

// Full f32 tensor, one thread per (row, unit); consecutive threads walk a row.
template <int TYPE>
__global__ void k_dequant(WView w, float *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= w.rows * (int64_t)w.units) return;
    int64_t r = idx / w.units;
    int u = (int)(idx % w.units);
    float v[32];
    decode_unit_exact<TYPE>(w, r, u, v);
    float4 *o = (float4 *)(out + r * (int64_t)w.units * 32 + (int64_t)u * 32);
#pragma unroll
    for (int j = 0; j < 8; j++) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

// Embedding rows: out[i][:] = dequantized row ids[i], zeros when out of range.
template <int TYPE>
__global__ void k_embed(WView w, const int32_t *__restrict__ ids, int n, float *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)n * w.units) return;
    int i = (int)(idx / w.units);
    int u = (int)(idx % w.units);
    int32_t r = ids[i];
    float v[32];
    if (r >= 0 && r < w.rows) {
        decode_unit_exact<TYPE>(w, r, u, v);
    } else {
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = 0.f;
    }
    float4 *o = (float4 *)(out + (int64_t)i * w.units * 32 + (int64_t)u * 32);
#pragma unroll
    for (int j = 0; j < 8; j++) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

int upload_common(hd_ctx *ctx, const uint8_t *src, bool src_on_device, size_t nbytes, int type, int64_t rows,
                  int64_t cols, hd_weight **out) {
    if (!ctx || !src || !out) return hd_fail(ctx, HD_E_ARG, "hd_weight_upload: null argument");
    *out = nullptr;
    HD_REQUIRE(ctx, hd_type_supported(type), HD_E_TYPE, "hd_weight_upload: ggml type %d not carried", type);
    int be = hd_block_elems(type), bb = hd_block_bytes(type);
    HD_REQUIRE(ctx, rows > 0 && cols > 0 && cols % be == 0, HD_E_SHAPE,
               "hd_weight_upload: shape [%lld, %lld] is not rows of whole %d-value blocks", (long long)rows,
               (long long)cols, be);
    HD_REQUIRE(ctx, cols / 32 <= (1 << 30) && rows <= ((int64_t)1 << 40), HD_E_SHAPE, "hd_weight_upload: too large");
    size_t expect = (size_t)rows * (size_t)(cols / be) * (size_t)bb;
    HD_REQUIRE(ctx, nbytes == expect, HD_E_SHAPE, "hd_weight_upload: %zu bytes given, shape needs %zu", nbytes,
               expect);
    hd_weight *w = new hd_weight();
    w->type = type;
    w->rows = rows;
    w->cols = cols;
    w->gguf_bytes = nbytes;
    w->units = (int)(cols / 32);
    w->nsb = (int)(cols / 256);
    size_t U = (size_t)w->units, R = (size_t)rows, SB = (size_t)w->nsb;
    size_t qb = type == HD_TYPE_Q8_0 ? U * R * 32 : U * R * 16;
    size_t ab = type == HD_TYPE_Q5_0 ? U * R * 4 : type == HD_TYPE_Q6_K ? U * R * 8 : 0;
    size_t mb = (type == HD_TYPE_Q8_0 || type == HD_TYPE_Q5_0) ? U * R * 2 : SB * R * 16;
    size_t db = type == HD_TYPE_Q6_K ? SB * R * 2 : 0;
    size_t off_q = 0, off_a = align256(qb), off_m = off_a + align256(ab), off_d = off_m + align256(mb);
    w->alloc_bytes = off_d + align256(db) + 256;
    if (cudaMalloc(&w->base, w->alloc_bytes) != cudaSuccess) {
        size_t want = w->alloc_bytes;
        delete w;
        cudaGetLastError();
        return hd_fail(ctx, HD_E_OOM, "hd_weight_upload: cudaMalloc(%zu) failed", want);
    }
    w->q = w->base + off_q;
    w->aux = ab ? w->base + off_a : nullptr;
    w->meta = w->base + off_m;
    w->dsb = db ? (uint16_t *)(w->base + off_d) : nullptr;

    uint8_t *tmp = nullptr;
    const uint8_t *dsrc = src;
    if (!src_on_device) {
        if (cudaMalloc(&tmp, nbytes) != cudaSuccess) {
            cudaFree(w->base);
            delete w;
            cudaGetLastError();
            return hd_fail(ctx, HD_E_OOM, "hd_weight_upload: staging %zu bytes", nbytes);
        }
        cudaError_t e = cudaMemcpyAsync(tmp, src, nbytes, cudaMemcpyHostToDevice, ctx->stream);
        if (e != cudaSuccess) {
            cudaFree(tmp);
            cudaFree(w->base);
            delete w;
            return hd_fail(ctx, HD_E_CUDA, "hd_weight_upload: copy: %s", cudaGetErrorString(e));
        }
        dsrc = tmp;
    }
    WView v = wview(w);
    int64_t n = rows * (int64_t)w->units;
    dim3 grid((unsigned)((n + 255) / 256));
    cudaError_t e = cudaSuccess;
    HD_TYPE_SWITCH(type, T, e = hd_launch(ctx, k_relayout<T>, grid, dim3(256), 0, dsrc, v, w->q, w->aux, w->meta,
                                          w->dsb));
    // scale bound for the exact-product GEMM (f16_shift)
    unsigned int *bound = nullptr, hb = 0;
    if (e == cudaSuccess && cudaMalloc(&bound, sizeof(unsigned int)) != cudaSuccess) e = cudaErrorMemoryAllocation;
    if (e == cudaSuccess) e = cudaMemsetAsync(bound, 0, sizeof(unsigned int), ctx->stream);
    if (e == cudaSuccess)
        HD_TYPE_SWITCH(type, T, e = hd_launch(ctx, k_wbound<T>, grid, dim3(256), 0, v, bound));
    if (e == cudaSuccess) e = cudaMemcpyAsync(&hb, bound, sizeof(hb), cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (bound) cudaFree(bound);
    if (tmp) cudaFree(tmp);
    if (e != cudaSuccess) {
        cudaFree(w->base);
        delete w;
        return hd_fail(ctx, HD_E_CUDA, "hd_weight_upload: relayout: %s", cudaGetErrorString(e));
    }
    {
        float bmax;
        memcpy(&bmax, &hb, sizeof(bmax));
        int sh = 0;
        if (bmax > 0.f && bmax < INFINITY) {
            int ex;
            frexpf(32768.f / bmax, &ex);  // 2^(ex-1) <= 32768 / bmax < 2^ex
            sh = ex - 1;
        }
        w->f16_shift = sh < -60 ? -60 : sh > 60 ? 60 : sh;
    }
    *out = w;
    return HD_OK;
}

}  // namespace

extern "C" int hd_weight_upload(hd_ctx *ctx, const uint8_t *gguf_host, size_t nbytes, int ggml_type, int64_t rows,
                                int64_t cols, hd_weight **out) {
    if (ctx) cudaSetDevice(ctx->device);
    return upload_common(ctx, gguf_host, false, nbytes, ggml_type, rows, cols, out);
}

extern "C" int hd_weight_upload_device(hd_ctx *ctx, const uint8_t *gguf_dev, size_t nbytes, int ggml_type,
                                       int64_t rows, int64_t cols, hd_weight **out) {
    if (ctx) cudaSetDevice(ctx->device);
    return upload_common(ctx, gguf_dev, true, nbytes, ggml_type, rows, cols, out);
}

extern "C" int hd_weight_free(hd_ctx *ctx, hd_weight *w) {
    if (!w) return HD_E_ARG;
    if (ctx) cudaStreamSynchronize(ctx->stream);
    cudaFree(w->base);
    delete w;
    return HD_OK;
}

extern "C" int hd_weight_info(const hd_weight *w, int *type, int64_t *rows, int64_t *cols, size_t *gguf_bytes) {
    if (!w) return HD_E_ARG;
    if (type) *type = w->type;
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (gguf_bytes) *gguf_bytes = w->gguf_bytes;
    return HD_OK;
}

extern "C" int hd_weight_download(hd_ctx *ctx, const hd_weight *w, uint8_t *gguf_host, size_t nbytes) {
    if (!ctx || !w || !gguf_host) return hd_fail(ctx, HD_E_ARG, "hd_weight_download: null argument");
    HD_REQUIRE(ctx, nbytes == w->gguf_bytes, HD_E_SHAPE, "hd_weight_download: need %zu bytes", w->gguf_bytes);
    uint8_t *tmp = nullptr;
    HD_CUDA_TRY(ctx, cudaMalloc(&tmp, nbytes));
    bool kq = w->type == HD_TYPE_Q4_K || w->type == HD_TYPE_Q6_K;
    int64_t n = w->rows * (int64_t)(kq ? w->units / 8 : w->units);
    dim3 grid((unsigned)((n + 127) / 128));
    WView v = wview(w);
    cudaError_t e = cudaSuccess;
    HD_TYPE_SWITCH(w->type, T, e = hd_launch(ctx, k_unlayout<T>, grid, dim3(128), 0, v, tmp));
    if (e == cudaSuccess) e = cudaMemcpyAsync(gguf_host, tmp, nbytes, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_weight_download: %s", cudaGetErrorString(e));
    return HD_OK;
}

extern "C" int hd_dequantize(hd_ctx *ctx, const hd_weight *w, float *out_dev, size_t n) {
    if (!ctx || !w || !out_dev) return hd_fail(ctx, HD_E_ARG, "hd_dequantize: null argument");
    HD_REQUIRE(ctx, n == (size_t)w->rows * (size_t)w->cols, HD_E_SHAPE, "hd_dequantize: out holds %zu, need %lld",
               n, (long long)(w->rows * w->cols));
    HD_REQUIRE(ctx, ((uintptr_t)out_dev & 15) == 0, HD_E_ARG, "hd_dequantize: out must be 16-byte aligned");
    int64_t total = w->rows * (int64_t)w->units;
    dim3 grid((unsigned)((total + 255) / 256));
    WView v = wview(w);
    cudaError_t e = cudaSuccess;
    HD_TYPE_SWITCH(w->type, T, e = hd_launch(ctx, k_dequant<T>, grid, dim3(256), 0, v, out_dev));
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_dequantize: %s", cudaGetErrorString(e));
    return HD_OK;
}

extern "C" int hd_embed(hd_ctx *ctx, const hd_weight *table, const int32_t *ids_dev, int n, float *out_dev) {
    if (!ctx || !table || (n > 0 && (!ids_dev || !out_dev))) return hd_fail(ctx, HD_E_ARG, "hd_embed: null argument");
    HD_REQUIRE(ctx, n >= 0, HD_E_ARG, "hd_embed: n < 0");
    if (n == 0) return HD_OK;
    HD_REQUIRE(ctx, ((uintptr_t)out_dev & 15) == 0, HD_E_ARG, "hd_embed: out must be 16-byte aligned");
    int64_t total = (int64_t)n * table->units;
    dim3 grid((unsigned)((total + 255) / 256));
    WView v = wview(table);
    cudaError_t e = cudaSuccess;
    HD_TYPE_SWITCH(table->type, T, e = hd_launch(ctx, k_embed<T>, grid, dim3(256), 0, v, ids_dev, n, out_dev));
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "hd_embed: %s", cudaGetErrorString(e));
    return HD_OK;
}
