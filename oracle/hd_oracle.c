/*
 * hd_oracle.c -- CPU oracle for the quantized-weight hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: tests/, the smoke
 * entry point and bench.py's cpu_baseline / reference arm call it.  It is
 * never linked into libhacedle_cuda.so and no product code path reaches it.
 *
 * It restates, in plain C, the arithmetic of the reference crate
 * (cosda-dev/hace-fem-hacedle, Rust, single-threaded) for this path:
 *
 *   dequant   src/quant_view/q4k_tensor_view.rs:180-222 (Q5_0), :278-309 (Q8_0)
 *             with IEEE binary16 scale decoding (the reference's f16_to_f32 at
 *             :123-136 uses the biased f32 exponent and is 2^127 too large; the
 *             reference's own golden blocks, produced by gguf-py 0.19.0, use IEEE).
 *             Q4_K / Q6_K follow the ggml block layout that the reference's
 *             golden generators exercise (scripts/t3_q6k_extract.py:36-47,
 *             tests/golden/manifest.yaml:1-7), with the association
 *             (d*sc)*q - dmin*m and (d*sc)*q; the reference's own Q4_K/Q6_K
 *             readers (:142-178, :224-276) read a different, wrong layout.
 *   GEMV      core/tensor_ops/matmul.rs:4-21 (sequential k = 0..K-1 in f32)
 *   GEMM      core/ops/matmul.rs:16-51
 *   RMSNorm   src/quant_view/dequant_dispatcher.rs:85-93 / src/ops/rmsnorm.rs:8-13
 *             and core/ops/rmsnorm.rs:16-82 (graph-executor variant)
 *   RoPE      src/ops/rope.rs:5-31 (per-head NEOX split-half, theta 1e6) and
 *             core/ops/rope.rs:16-64 (interleaved pairs from cos/sin tables)
 *   softmax   dequant_dispatcher.rs:117-128
 *   SiLU      src/ops/silu.rs:5-13
 *   argmax    runtime/sampler/argmax.rs:8-24 (first max wins, strict >)
 *   embedding core/tensor_ops/embedding.rs:4-17 (out-of-range id -> zeros)
 *   int8 dot  ops/batch.rs:3-29, ops/simd.rs:20-31 (scalar path, wrapping i32)
 *   fused     ops/fused.rs:52-57
 *   add       core/ops/add.rs:16-43
 *   block     core/ops/block.rs:51-238, with the corrections documented in
 *             hdo_decoder_generate() below.
 *
 * Build: gcc -O2 -ffp-contract=off -fno-fast-math -fopenmp (oracle/Makefile).
 * No FMA contraction, so every product and sum rounds exactly as the scalar
 * Rust code does.
 */
#include <stdint.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ggml type ids (gguf 0.19.0 GGMLQuantizationType). The reference's QuantType
 * discriminants (q4k_tensor_view.rs:9-19) are not ggml ids; the C ABI uses these. */
enum { HDO_F32 = 0, HDO_F16 = 1, HDO_Q5_0 = 6, HDO_Q8_0 = 8, HDO_Q4_K = 12,
       HDO_Q6_K = 14, HDO_BF16 = 30 };

int hdo_type_block(int type, int *block_elems, int *block_bytes) {
    switch (type) {
    case HDO_Q8_0: *block_elems = 32;  *block_bytes = 34;  return 0;
    case HDO_Q5_0: *block_elems = 32;  *block_bytes = 22;  return 0;
    case HDO_Q4_K: *block_elems = 256; *block_bytes = 144; return 0;
    case HDO_Q6_K: *block_elems = 256; *block_bytes = 210; return 0;
    case HDO_F16:  *block_elems = 1;   *block_bytes = 2;   return 0;
    case HDO_BF16: *block_elems = 1;   *block_bytes = 2;   return 0;
    case HDO_F32:  *block_elems = 1;   *block_bytes = 4;   return 0;
    default: return -1;
    }
}

static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE-754 binary16 -> binary32, exact for every input (subnormals, inf, NaN). */
float hdo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0) {
        /* zero or subnormal: m * 2^-24, exact in f32 */
        float v = (float)m * 5.9604644775390625e-8f;
        return sign ? -v : v;
    }
    if (e == 31) return bits_f32(sign | 0x7F800000u | (m << 13));
    return bits_f32(sign | ((e - 15u + 127u) << 23) | (m << 13));
}

float hdo_bf16_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline uint32_t rd32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* Q8_0: 34-byte block = f16 d | int8 qs[32]; y = (f32)qs[j] * d.
 * Loop structure of dequant_q8_0_exact (q4k_tensor_view.rs:278-309). */
static void dq_q8_0(const uint8_t *data, size_t nbytes, float *out, size_t n) {
    size_t blocks = nbytes / 34, elems = n < blocks * 32 ? n : blocks * 32;
    for (size_t b = 0; b < blocks; b++) {
        const uint8_t *blk = data + b * 34;
        float d = hdo_f16_to_f32(rd16(blk));
        for (int j = 0; j < 32; j++) {
            size_t idx = b * 32 + j;
            if (idx >= elems) return;
            out[idx] = (float)(int8_t)blk[2 + j] * d;
        }
    }
}

/* Q5_0: 22-byte block = f16 d | u32 qh | qs[16]; element j takes the low
 * (j < 16) or high (j >= 16) nibble of qs[j % 16] plus bit j of qh as bit 4;
 * y = ((f32)q - 16) * d.  dequant_q5_0_exact (q4k_tensor_view.rs:180-222). */
static void dq_q5_0(const uint8_t *data, size_t nbytes, float *out, size_t n) {
    size_t blocks = nbytes / 22, elems = n < blocks * 32 ? n : blocks * 32;
    for (size_t b = 0; b < blocks; b++) {
        const uint8_t *blk = data + b * 22;
        float d = hdo_f16_to_f32(rd16(blk));
        uint32_t qh = rd32(blk + 2);
        for (int j = 0; j < 32; j++) {
            size_t idx = b * 32 + j;
            if (idx >= elems) return;
            uint32_t bit = (qh >> j) & 1u;
            uint32_t ql = j < 16 ? (blk[6 + j] & 0x0Fu) : (blk[6 + j - 16] >> 4);
            uint32_t q = ql | (bit << 4);
            out[idx] = ((float)q - 16.0f) * d;
        }
    }
}

/* Q4_K 6-bit scale/min unpacking from the 12 packed bytes (llama.cpp's
 * get_scale_min_k4 layout, as BASELINE's generator describes). */
static inline void q4k_scale_min(int j, const uint8_t *s, uint8_t *sc, uint8_t *mn) {
    if (j < 4) {
        *sc = s[j] & 63u;
        *mn = s[j + 4] & 63u;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0x0Fu) | ((s[j - 4] >> 6) << 4));
        *mn = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* Q4_K: 144-byte super-block of 256 = f16 d | f16 dmin | scales[12] | qs[128].
 * Chunk c (64 values) uses sub-blocks 2c and 2c+1; its 32 bytes qs[32c..]
 * hold values 64c+l in the low nibble and 64c+32+l in the high nibble.
 * y = (d*sc)*q - (dmin*m), evaluated left to right as gguf-py does. */
static void dq_q4_k(const uint8_t *data, size_t nbytes, float *out, size_t n) {
    size_t blocks = nbytes / 144, elems = n < blocks * 256 ? n : blocks * 256;
    for (size_t b = 0; b < blocks; b++) {
        const uint8_t *blk = data + b * 144;
        float d = hdo_f16_to_f32(rd16(blk)), dmin = hdo_f16_to_f32(rd16(blk + 2));
        const uint8_t *sc = blk + 4, *qs = blk + 16;
        for (int c = 0; c < 4; c++) {
            uint8_t s1, m1, s2, m2;
            q4k_scale_min(2 * c, sc, &s1, &m1);
            q4k_scale_min(2 * c + 1, sc, &s2, &m2);
            float d1 = d * (float)s1, o1 = dmin * (float)m1;
            float d2 = d * (float)s2, o2 = dmin * (float)m2;
            for (int l = 0; l < 32; l++) {
                size_t i0 = b * 256 + 64 * c + l, i1 = i0 + 32;
                uint8_t byte = qs[32 * c + l];
                if (i0 < elems) out[i0] = d1 * (float)(byte & 0x0Fu) - o1;
                if (i1 < elems) out[i1] = d2 * (float)(byte >> 4) - o2;
            }
        }
    }
}

/* Q6_K: 210-byte super-block = ql[128] | qh[64] | int8 scales[16] | f16 d.
 * Half h (128 values): value 128h+32k+l (k = 0..3, l = 0..31) takes the low
 * (k < 2) or high nibble of ql[64h + 32(k&1) + l] and 2 bits (2k..2k+1) of
 * qh[32h + l]; q6 = that - 32; scale index = value / 16; y = (d*sc)*q6. */
static void dq_q6_k(const uint8_t *data, size_t nbytes, float *out, size_t n) {
    size_t blocks = nbytes / 210, elems = n < blocks * 256 ? n : blocks * 256;
    for (size_t b = 0; b < blocks; b++) {
        const uint8_t *blk = data + b * 210;
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t *sc = (const int8_t *)(blk + 192);
        float d = hdo_f16_to_f32(rd16(blk + 208));
        for (int h = 0; h < 2; h++) {
            for (int k = 0; k < 4; k++) {
                for (int l = 0; l < 32; l++) {
                    int e = 128 * h + 32 * k + l;
                    size_t idx = b * 256 + e;
                    if (idx >= elems) continue;
                    uint8_t lb = ql[64 * h + 32 * (k & 1) + l];
                    uint32_t lo = (k < 2) ? (lb & 0x0Fu) : (lb >> 4);
                    uint32_t hi = (qh[32 * h + l] >> (2 * k)) & 3u;
                    int q = (int)(lo | (hi << 4)) - 32;
                    float ds = d * (float)sc[e / 16];
                    out[idx] = ds * (float)q;
                }
            }
        }
    }
}

/* QuantTensorView::dequantize (q4k_tensor_view.rs:63-114). Returns 0, or -1
 * for a type this path does not carry. */
int hdo_dequantize(int type, const uint8_t *data, size_t nbytes, float *out, size_t n) {
    switch (type) {
    case HDO_Q8_0: dq_q8_0(data, nbytes, out, n); return 0;
    case HDO_Q5_0: dq_q5_0(data, nbytes, out, n); return 0;
    case HDO_Q4_K: dq_q4_k(data, nbytes, out, n); return 0;
    case HDO_Q6_K: dq_q6_k(data, nbytes, out, n); return 0;
    case HDO_F16: {
        size_t c = n < nbytes / 2 ? n : nbytes / 2;
        for (size_t i = 0; i < c; i++) out[i] = hdo_f16_to_f32(rd16(data + 2 * i));
        return 0;
    }
    case HDO_BF16: {
        size_t c = n < nbytes / 2 ? n : nbytes / 2;
        for (size_t i = 0; i < c; i++) out[i] = hdo_bf16_to_f32(rd16(data + 2 * i));
        return 0;
    }
    case HDO_F32: {
        size_t c = n < nbytes / 4 ? n : nbytes / 4;
        memcpy(out, data, c * 4);
        return 0;
    }
    default: return -1;
    }
}

static inline void set_threads(int threads) {
#ifdef _OPENMP
    omp_set_num_threads(threads > 0 ? threads : 1);
#else
    (void)threads;
#endif
}

/* matmul_vec_matrix (core/tensor_ops/matmul.rs:4-21): y[i] = sum_{j<K} x[j]*W[i*K+j],
 * summed sequentially from 0.  Rows are independent, so the row-parallel form
 * below gives the same bits for any thread count; eight rows run interleaved
 * only to keep the scalar adder busy (each row's order is unchanged). */
void hdo_matmul_vec_matrix(const float *x, const float *W, int64_t N, int64_t K, float *y) {
    for (int64_t i = 0; i < N; i++) {
        const float *w = W + i * K;
        float s = 0.0f;
        for (int64_t j = 0; j < K; j++) s += x[j] * w[j];
        y[i] = s;
    }
}

static void gemv_rows(const float *x, const float *W, int64_t r0, int64_t r1, int64_t K, float *y) {
    int64_t i = r0;
    for (; i + 8 <= r1; i += 8) {
        float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const float *w = W + i * K;
        for (int64_t j = 0; j < K; j++) {
            float xj = x[j];
            for (int r = 0; r < 8; r++) s[r] += xj * w[r * K + j];
        }
        for (int r = 0; r < 8; r++) y[i + r] = s[r];
    }
    for (; i < r1; i++) {
        const float *w = W + i * K;
        float s = 0.0f;
        for (int64_t j = 0; j < K; j++) s += x[j] * w[j];
        y[i] = s;
    }
}

/* Y[b] = W * X[b] for b < B on an f32 weight, row-parallel over `threads`. */
void hdo_gemv_f32(const float *W, int64_t N, int64_t K, const float *X, int B, float *Y, int threads) {
    set_threads(threads);
    for (int b = 0; b < B; b++) {
        const float *x = X + (int64_t)b * K;
        float *y = Y + (int64_t)b * N;
#pragma omp parallel
        {
#ifdef _OPENMP
            int t = omp_get_thread_num(), nt = omp_get_num_threads();
#else
            int t = 0, nt = 1;
#endif
            int64_t per = ((N + nt - 1) / nt + 7) / 8 * 8;
            int64_t r0 = (int64_t)t * per, r1 = r0 + per < N ? r0 + per : N;
            if (r0 < r1) gemv_rows(x, W, r0, r1, K, y);
        }
    }
}

/* The reference's quantized matmul path as it runs today: dequantize the whole
 * weight tensor (QuantTensorView::dequantize, cloned per call at block.rs:75-93),
 * then the sequential GEMV loops (block.rs:104-128).  Returns 0 or -1. */
int hdo_qgemv(int type, const uint8_t *Wq, size_t nbytes, int64_t N, int64_t K,
              const float *X, int B, float *Y, int threads) {
    float *W = (float *)malloc((size_t)N * (size_t)K * sizeof(float));
    if (!W) return -1;
    int rc = hdo_dequantize(type, Wq, nbytes, W, (size_t)N * (size_t)K);
    if (rc == 0) hdo_gemv_f32(W, N, K, X, B, Y, threads);
    free(W);
    return rc;
}

/* NativeBackend::rmsnorm (dequant_dispatcher.rs:85-93) per row:
 * ss = sum x^2 (sequential), r = 1/sqrt(ss/n + eps), y = (x*w)*r. */
void hdo_rmsnorm(const float *x, const float *w, float *y, int64_t rows, int64_t dim, float eps) {
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * dim;
        float ss = 0.0f;
        for (int64_t i = 0; i < dim; i++) ss += xr[i] * xr[i];
        float rms = 1.0f / sqrtf(ss / (float)dim + eps);
        for (int64_t i = 0; i < dim; i++) y[r * dim + i] = xr[i] * w[i] * rms;
    }
}

/* rmsnorm_f32 (core/ops/rmsnorm.rs:16-61), the graph-executor operator:
 * mean_sq = (sum v^2)/dim, inv = 1/sqrtf(mean_sq+eps), out = v*inv*w.
 * sqrtf is the default-feature Newton iteration (:63-82). */
static float newton_sqrtf(float x) {
    if (x <= 0.0f) return 0.0f;
    float y = x;
    for (int i = 0; i < 6; i++) y = 0.5f * (y + x / y);
    return y;
}
void hdo_rmsnorm_graph(const float *x, const float *w, float *y, int64_t rows, int64_t dim,
                       float eps, int newton) {
    for (int64_t r = 0; r < rows; r++) {
        float ms = 0.0f;
        for (int64_t i = 0; i < dim; i++) { float v = x[r * dim + i]; ms += v * v; }
        ms /= (float)dim;
        float inv = 1.0f / (newton ? newton_sqrtf(ms + eps) : sqrtf(ms + eps));
        for (int64_t i = 0; i < dim; i++) y[r * dim + i] = x[r * dim + i] * inv * w[i];
    }
}

/* RoPE inverse-frequency denominators of src/ops/rope.rs:14: theta^(2i/d) in f32. */
void hdo_rope_freqs(int head_dim, float theta, float *freq) {
    for (int i = 0; i < head_dim / 2; i++)
        freq[i] = powf(theta, 2.0f * (float)i / (float)head_dim);
}

/* apply_rope_pairwise (src/ops/rope.rs:5-31) on every head of every token:
 * angle = pos / theta^(2i/d); (x0, x1) -> (x0 c - x1 s, x0 s + x1 c) with x1 = x[i + d/2]. */
void hdo_rope_neox(float *x, int64_t tokens, int heads, int head_dim, const int32_t *pos, float theta) {
    float freq[512];
    hdo_rope_freqs(head_dim, theta, freq);
    int half = head_dim / 2;
    for (int64_t t = 0; t < tokens; t++) {
        for (int h = 0; h < heads; h++) {
            float *v = x + (t * heads + h) * head_dim;
            for (int i = 0; i < half; i++) {
                float angle = (float)pos[t] / freq[i];
                float c = cosf(angle), s = sinf(angle);
                float x0 = v[i], x1 = v[i + half];
                v[i] = x0 * c - x1 * s;
                v[i + half] = x0 * s + x1 * c;
            }
        }
    }
}

/* rope_f32 (core/ops/rope.rs:16-64): interleaved pairs (2i, 2i+1) of each row,
 * rotated by cos/sin tables of the same shape as x (index 2i is read). */
void hdo_rope_interleaved(const float *x, const float *cosv, const float *sinv, float *out,
                          int64_t rows, int64_t last_dim) {
    for (int64_t r = 0; r < rows; r++) {
        int64_t base = r * last_dim;
        for (int64_t i = 0; i < last_dim / 2; i++) {
            int64_t i0 = base + 2 * i, i1 = i0 + 1;
            float x0 = x[i0], x1 = x[i1], c = cosv[i0], s = sinv[i0];
            out[i0] = x0 * c - x1 * s;
            out[i1] = x1 * c + x0 * s;
        }
    }
}

/* NativeBackend::softmax (dequant_dispatcher.rs:117-128), in place. */
void hdo_softmax(float *x, int64_t n) {
    if (n <= 0) return;
    float m = -INFINITY;
    for (int64_t i = 0; i < n; i++) m = fmaxf(m, x[i]);
    float s = 0.0f;
    for (int64_t i = 0; i < n; i++) s += expf(x[i] - m);
    for (int64_t i = 0; i < n; i++) x[i] = expf(x[i] - m) / s;
}

/* silu (src/ops/silu.rs:5-13): v / (1 + exp(-v)). */
void hdo_silu(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = x[i] / (1.0f + expf(-x[i]));
}

/* SwiGLU as Qwen2 defines it: silu(gate) * up.  (core/ops/block.rs:221 computes
 * gate*up/(1+exp(-|up|)), which is not SwiGLU; the oracle does not reproduce it.) */
void hdo_swiglu(const float *g, const float *u, float *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        float s = g[i] / (1.0f + expf(-g[i]));
        y[i] = s * u[i];
    }
}

/* add_f32 (core/ops/add.rs:16-43). */
void hdo_add_f32(const float *a, const float *b, float *out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = a[i] + b[i];
}

/* matmul_f32 (core/ops/matmul.rs:16-51): out[m,n] = sum_k a[m,k] b[k,n], k sequential. */
void hdo_matmul_f32(const float *a, const float *b, float *out, int64_t m, int64_t n, int64_t k) {
    for (int64_t i = 0; i < m; i++)
        for (int64_t j = 0; j < n; j++) {
            float acc = 0.0f;
            for (int64_t l = 0; l < k; l++) acc += a[i * k + l] * b[l * n + j];
            out[i * n + j] = acc;
        }
}

/* ArgMaxSampler::sample (runtime/sampler/argmax.rs:8-24): first index of the
 * maximum, strict >; 0 for an empty slice. */
uint32_t hdo_argmax(const float *x, int64_t n) {
    if (n <= 0) return 0;
    int64_t bi = 0;
    float bv = x[0];
    for (int64_t i = 0; i < n; i++)
        if (x[i] > bv) { bv = x[i]; bi = i; }
    return (uint32_t)bi;
}

/* embedding_lookup (core/tensor_ops/embedding.rs:4-17): row copy, zeros when
 * the id or the row end is out of range. */
void hdo_embedding_lookup(uint32_t token, const float *table, int64_t table_len, int64_t vocab,
                          int64_t hidden, float *out) {
    int64_t start = (int64_t)token * hidden;
    if ((int64_t)token >= vocab || start + hidden > table_len) {
        memset(out, 0, (size_t)hidden * sizeof(float));
        return;
    }
    memcpy(out, table + start, (size_t)hidden * sizeof(float));
}

/* GQA decode attention for one token (the corrected form of block.rs:138-173):
 * head h reads kv head h / (n_heads / n_kv); score_i = (sum_d q.k_i) / sqrt(hd);
 * p = softmax(score) (dequant_dispatcher.rs:117-128); out_d = sum_i p_i v_i[d].
 * Cache layout [pos][n_kv][hd] (KvCache, block.rs:241-282). */
void hdo_attention_decode(const float *q, const float *kc, const float *vc, int64_t len,
                          int n_heads, int n_kv, int hd, float *out, float *scratch) {
    int rep = n_heads / n_kv;
    float scale = sqrtf((float)hd);
    for (int h = 0; h < n_heads; h++) {
        int kvh = h / rep;
        const float *qh = q + (int64_t)h * hd;
        for (int64_t i = 0; i < len; i++) {
            const float *k = kc + (i * n_kv + kvh) * hd;
            float s = 0.0f;
            for (int d = 0; d < hd; d++) s += qh[d] * k[d];
            scratch[i] = s / scale;
        }
        hdo_softmax(scratch, len);
        for (int d = 0; d < hd; d++) {
            float s = 0.0f;
            for (int64_t i = 0; i < len; i++) s += scratch[i] * vc[(i * n_kv + kvh) * hd + d];
            out[(int64_t)h * hd + d] = s;
        }
    }
}

/* dot_batch (ops/batch.rs:3-29) on the default-feature scalar path: 32-wide
 * chunks (ops/simd.rs:20-31) then the tail, all in wrapping i32. */
int32_t hdo_dot_i8(const int8_t *a, const int8_t *b, int64_t n) {
    uint32_t acc = 0;
    for (int64_t i = 0; i < n; i++) acc += (uint32_t)((int32_t)a[i] * (int32_t)b[i]);
    return (int32_t)acc;
}

/* fused_qdot_qadd_qacc_i8 (ops/fused.rs:52-57): out = dot + bias + carry
 * (wrapping), carry = out. */
int32_t hdo_fused_qdot_qadd_qacc_i8(const int8_t *a, const int8_t *b, int64_t n, int32_t bias,
                                    int32_t *carry) {
    uint32_t out = (uint32_t)hdo_dot_i8(a, b, n) + (uint32_t)bias + (uint32_t)*carry;
    *carry = (int32_t)out;
    return (int32_t)out;
}

/* ------------------------------------------------------------------------- */
/* Qwen2-shaped decoder (BrainBlock::forward, core/ops/block.rs:51-238, made   */
/* correct).  Deviations from the reference block, each deliberate:           */
/*   - RoPE on every head of q and k (the reference rotates head 0 only,      */
/*     dequant_dispatcher.rs:95-115 called at block.rs:131-132);              */
/*   - GQA kv head = h / (n_heads/n_kv) with full head_dim dot products       */
/*     (block.rs:145,168,286 read one scalar per token with h % n_kv);        */
/*   - o_proj applied (dequantized but unused at block.rs:154-173);           */
/*   - SwiGLU = silu(gate)*up (block.rs:221 differs);                         */
/*   - q/k/v biases added after the projection (Qwen2);                       */
/*   - quant types per matrix come from the caller (block.rs hard-codes them).*/
/* Weights here are already-dequantized f32 (dequantize is deterministic, so  */
/* dequantizing once gives the same numbers as the per-call dequant).         */
/* ------------------------------------------------------------------------- */
typedef struct {
    int hidden, n_layers, n_heads, n_kv, head_dim, ffn, vocab, max_ctx;
    float eps, theta;
} hdo_model_cfg;

typedef struct {
    const float *attn_norm, *ffn_norm;
    const float *wq, *bq, *wk, *bk, *wv, *bv, *wo, *wg, *wu, *wd;
} hdo_layer_w;

static void gemv1(const float *W, int64_t N, int64_t K, const float *x, float *y) {
#pragma omp parallel
    {
#ifdef _OPENMP
        int t = omp_get_thread_num(), nt = omp_get_num_threads();
#else
        int t = 0, nt = 1;
#endif
        int64_t per = ((N + nt - 1) / nt + 7) / 8 * 8;
        int64_t r0 = (int64_t)t * per, r1 = r0 + per < N ? r0 + per : N;
        if (r0 < r1) gemv_rows(x, W, r0, r1, K, y);
    }
}

/* One decode step at position `pos` for token `tok`; writes logits when
 * `logits` is not NULL.  kcache/vcache: [layer][max_ctx][n_kv][hd]. */
static void decoder_step(const hdo_model_cfg *c, const hdo_layer_w *L, const float *out_norm,
                         const float *embed, int32_t tok, int pos, float *kcache, float *vcache,
                         float *logits, float *ws) {
    int H = c->hidden, hd = c->head_dim, nq = c->n_heads * hd, nkv = c->n_kv * hd, F = c->ffn;
    float *h = ws, *xn = h + H, *q = xn + H, *k = q + nq, *v = k + nkv, *att = v + nkv,
          *o = att + nq, *g = o + H, *u = g + F, *a = u + F, *dn = a + F, *sc = dn + H;
    hdo_embedding_lookup((uint32_t)tok, embed, (int64_t)c->vocab * H, c->vocab, H, h);
    int32_t p = pos;
    for (int l = 0; l < c->n_layers; l++) {
        const hdo_layer_w *w = &L[l];
        hdo_rmsnorm(h, w->attn_norm, xn, 1, H, c->eps);
        gemv1(w->wq, nq, H, xn, q);
        gemv1(w->wk, nkv, H, xn, k);
        gemv1(w->wv, nkv, H, xn, v);
        for (int i = 0; i < nq; i++) q[i] = q[i] + w->bq[i];
        for (int i = 0; i < nkv; i++) { k[i] = k[i] + w->bk[i]; v[i] = v[i] + w->bv[i]; }
        hdo_rope_neox(q, 1, c->n_heads, hd, &p, c->theta);
        hdo_rope_neox(k, 1, c->n_kv, hd, &p, c->theta);
        size_t lay = (size_t)l * c->max_ctx * nkv;
        memcpy(kcache + lay + (size_t)pos * nkv, k, nkv * sizeof(float));
        memcpy(vcache + lay + (size_t)pos * nkv, v, nkv * sizeof(float));
        hdo_attention_decode(q, kcache + lay, vcache + lay, pos + 1, c->n_heads, c->n_kv, hd, att, sc);
        gemv1(w->wo, H, nq, att, o);
        for (int i = 0; i < H; i++) h[i] = h[i] + o[i];
        hdo_rmsnorm(h, w->ffn_norm, xn, 1, H, c->eps);
        gemv1(w->wg, F, H, xn, g);
        gemv1(w->wu, F, H, xn, u);
        hdo_swiglu(g, u, a, F);
        gemv1(w->wd, H, F, a, dn);
        for (int i = 0; i < H; i++) h[i] = h[i] + dn[i];
    }
    if (logits) {
        hdo_rmsnorm(h, out_norm, xn, 1, H, c->eps);
        gemv1(embed, c->vocab, H, xn, logits);
    }
}

/* Prefill `n_prompt` ids token by token, then greedy-decode `n_gen` ids
 * (ArgMaxSampler).  The LM head is the tied f32 embedding.  out_tokens gets
 * n_gen ids; if last_logits is not NULL it receives the logits that chose the
 * final id.  Returns 0, or -1 on a bad size or allocation failure. */
int hdo_decoder_generate_all(const hdo_model_cfg *c, const hdo_layer_w *L, const float *out_norm,
                             const float *embed, const int32_t *prompt, int n_prompt, int n_gen,
                             int32_t *out_tokens, float *all_logits, int threads);

int hdo_decoder_generate(const hdo_model_cfg *c, const hdo_layer_w *L, const float *out_norm,
                         const float *embed, const int32_t *prompt, int n_prompt, int n_gen,
                         int32_t *out_tokens, float *last_logits, int threads) {
    float *all = NULL;
    if (last_logits && n_gen > 0) {
        all = (float *)malloc((size_t)n_gen * c->vocab * sizeof(float));
        if (!all) return -1;
    }
    int rc = hdo_decoder_generate_all(c, L, out_norm, embed, prompt, n_prompt, n_gen, out_tokens, all, threads);
    if (rc == 0 && all) memcpy(last_logits, all + (size_t)(n_gen - 1) * c->vocab, (size_t)c->vocab * sizeof(float));
    free(all);
    return rc;
}

/* The same, keeping the logits that chose every generated id: all_logits
 * [n_gen][vocab] (row g chose out_tokens[g]), or NULL. */
int hdo_decoder_generate_all(const hdo_model_cfg *c, const hdo_layer_w *L, const float *out_norm,
                             const float *embed, const int32_t *prompt, int n_prompt, int n_gen,
                             int32_t *out_tokens, float *all_logits, int threads) {
    if (n_prompt < 1 || n_prompt + n_gen > c->max_ctx || c->head_dim > 1024) return -1;
    set_threads(threads);
    size_t kv = (size_t)c->n_layers * c->max_ctx * c->n_kv * c->head_dim;
    float *kc = (float *)calloc(kv, sizeof(float)), *vc = (float *)calloc(kv, sizeof(float));
    size_t wsn = (size_t)4 * c->hidden + 2 * (size_t)c->n_heads * c->head_dim +
                 2 * (size_t)c->n_kv * c->head_dim + 3 * (size_t)c->ffn + (size_t)c->max_ctx + 64;
    float *ws = (float *)malloc(wsn * sizeof(float));
    float *logits = (float *)malloc((size_t)c->vocab * sizeof(float));
    if (!kc || !vc || !ws || !logits) { free(kc); free(vc); free(ws); free(logits); return -1; }
    for (int t = 0; t < n_prompt; t++)
        decoder_step(c, L, out_norm, embed, prompt[t], t, kc, vc, t == n_prompt - 1 ? logits : NULL, ws);
    for (int g = 0; g < n_gen; g++) {
        int32_t next = (int32_t)hdo_argmax(logits, c->vocab);
        out_tokens[g] = next;
        if (all_logits) memcpy(all_logits + (size_t)g * c->vocab, logits, (size_t)c->vocab * sizeof(float));
        if (g + 1 < n_gen)
            decoder_step(c, L, out_norm, embed, next, n_prompt + g, kc, vc, logits, ws);
    }
    free(kc); free(vc); free(ws); free(logits);
    return 0;
}

/* ---------------------------------------------------------------- Q8_1 path
 * The integer activation path of libhacedle_cuda (no reference counterpart;
 * it follows on the i8 ops of ops/q_ops.rs:11-13).  Blocks of 32 activations:
 * d = max|x| / 127, q = rint(x * (1/d)) (round half to even; 0 for a zero
 * block), s0 / s1 = sum of q over values 0-15 / 16-31. */
void hdo_quantize_q8_1(const float *x, int64_t nblocks, int8_t *q, float *d, int32_t *s) {
    for (int64_t b = 0; b < nblocks; b++) {
        const float *v = x + b * 32;
        float m = 0.f;
        for (int j = 0; j < 32; j++) m = fabsf(v[j]) > m ? fabsf(v[j]) : m;
        float db = m / 127.f, id = db > 0.f ? 1.f / db : 0.f;
        int s0 = 0, s1 = 0;
        for (int j = 0; j < 32; j++) {
            int qq = (int)nearbyintf(v[j] * id);
            q[b * 32 + j] = (int8_t)qq;
            if (j < 16) s0 += qq; else s1 += qq;
        }
        d[b] = db;
        s[2 * b] = s0;
        s[2 * b + 1] = s1;
    }
}

/* Unit u (32 values) of a row of GGUF blocks as small integers q[32] with
 * per-half scale a and offset o (w = a q - o), the decomposition the device
 * kernel uses: Q8_0 (q, d, 0); Q5_0 (q5, d, 16 d); Q4_K (q4, d sc, dmin m);
 * Q6_K (q6 unsigned, d sc_h, 32 d sc_h). */
static int unit_ints(int type, const uint8_t *row, int u, int q[32], float a[2], float o[2]) {
    if (type == 8) {
        const uint8_t *blk = row + (size_t)u * 34;
        float d = hdo_f16_to_f32(rd16(blk));
        for (int j = 0; j < 32; j++) q[j] = (int8_t)blk[2 + j];
        a[0] = a[1] = d;
        o[0] = o[1] = 0.f;
    } else if (type == 6) {
        const uint8_t *blk = row + (size_t)u * 22;
        float d = hdo_f16_to_f32(rd16(blk));
        uint32_t qh = rd32(blk + 2);
        for (int j = 0; j < 32; j++) {
            uint32_t ql = j < 16 ? (blk[6 + j] & 0x0Fu) : (blk[6 + j - 16] >> 4);
            q[j] = (int)(ql | (((qh >> j) & 1u) << 4));
        }
        a[0] = a[1] = d;
        o[0] = o[1] = 16.f * d;
    } else if (type == 12) {
        const uint8_t *blk = row + (size_t)(u / 8) * 144;
        const int uu = u % 8, c = uu / 2, hi = uu % 2;
        float d = hdo_f16_to_f32(rd16(blk)), dmin = hdo_f16_to_f32(rd16(blk + 2));
        uint8_t sc, mn;
        q4k_scale_min(uu, blk + 4, &sc, &mn);
        for (int l = 0; l < 32; l++) {
            uint8_t byte = blk[16 + 32 * c + l];
            q[l] = hi ? (byte >> 4) : (byte & 0x0F);
        }
        a[0] = a[1] = d * (float)sc;
        o[0] = o[1] = dmin * (float)mn;
    } else if (type == 14) {
        const uint8_t *blk = row + (size_t)(u / 8) * 210;
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t *sc = (const int8_t *)(blk + 192);
        float d = hdo_f16_to_f32(rd16(blk + 208));
        const int uu = u % 8;
        for (int l = 0; l < 32; l++) {
            int e = 32 * uu + l, h = e / 128, k = (e % 128) / 32, ll = e % 32;
            uint8_t lb = ql[64 * h + 32 * (k & 1) + ll];
            uint32_t lo = (k < 2) ? (lb & 0x0Fu) : (lb >> 4);
            uint32_t hb = (qh[32 * h + ll] >> (2 * k)) & 3u;
            q[l] = (int)(lo | (hb << 4));
        }
        a[0] = d * (float)sc[2 * uu];
        a[1] = d * (float)sc[2 * uu + 1];
        o[0] = 32.f * a[0];
        o[1] = 32.f * a[1];
    } else {
        return -1;
    }
    return 0;
}

/* y[b][r] = sum over units (in order) of dx (a0 dot0 - o0 s0 + a1 dot1 - o1 s1). */
int hdo_qgemv_q8_1(int type, const uint8_t *W, int64_t N, int64_t K, const int8_t *xq, const float *xd,
                   const int32_t *xs, int B, float *y) {
    int be, bb;
    if (hdo_type_block(type, &be, &bb) != 0) return -1;
    const int64_t units = K / 32, row_bytes = K / be * bb;
    int q[32];
    float a[2], o[2];
    for (int64_t r = 0; r < N; r++) {
        const uint8_t *row = W + r * row_bytes;
        for (int b = 0; b < B; b++) {
            float acc = 0.f;
            for (int64_t u = 0; u < units; u++) {
                if (unit_ints(type, row, (int)u, q, a, o) != 0) return -1;
                const int8_t *x = xq + ((int64_t)b * units + u) * 32;
                int d0 = 0, d1 = 0;
                for (int j = 0; j < 16; j++) d0 += q[j] * x[j];
                for (int j = 16; j < 32; j++) d1 += q[j] * x[j];
                const int32_t *s = xs + 2 * ((int64_t)b * units + u);
                float h0 = a[0] * (float)d0 - o[0] * (float)s[0];
                float h1 = a[1] * (float)d1 - o[1] * (float)s[1];
                acc = acc + xd[(int64_t)b * units + u] * (h0 + h1);
            }
            y[(int64_t)b * N + r] = acc;
        }
    }
    return 0;
}
