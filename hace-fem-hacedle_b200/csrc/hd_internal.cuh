// hd_internal.cuh -- shared internals of libhacedle_cuda.so (sm_100a).
//
// Device weight layout.  hd_weight_upload re-lays a GGUF tensor [rows x cols]
// out as structure-of-arrays over 32-value "units" (cols/32 units per row),
// unit-major with rows contiguous, so that a warp whose lanes own consecutive
// rows reads one unit of 32 rows as one contiguous 512-byte (or 1 KB) span:
//
//   Q8_0  q    [units][rows][32] int8          meta f16 d [units][rows]
//   Q5_0  q    [units][rows][16] nibbles       aux  u32 qh' [units][rows]
//                                               meta f16 d [units][rows]
//   Q4_K  q    [units][rows][16] nibbles       meta 16 B (d, dmin, scales[12])
//                                                    [superblocks][rows]
//   Q6_K  q    [units][rows][16] low nibbles   aux  8 B high bits [units][rows]
//                                               meta int8 scales[16] [sb][rows]
//                                               dsb  f16 d [sb][rows]
//
// Nibble byte j (0..15) of a unit holds value j in its low and value j+16 in
// its high nibble (Q5_0's own GGUF order; Q4_K and Q6_K are re-ordered to it).
// The 5th bit of Q5_0 and the two high bits of Q6_K are re-ordered so that
// one shift and one mask place them at bits 4-5 of the byte that holds the
// value (see unit_q5_0 / unit_q6_k).  The byte count is exactly the GGUF byte
// count: the re-layout is a permutation and hd_weight_download inverts it.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>

#include "../../include/hacedle_cuda.h"

#define HD_LIB_VERSION "hacedle_cuda 0.1 (sm_100a)"

struct hd_ctx {
    int device = 0;
    int sm_count = 148;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    bool pdl = true;                 // programmatic dependent launch between kernels
    std::string err;
    void *ws = nullptr;              // split-K partial sums (device)
    size_t ws_bytes = 0;
    int *tickets = nullptr;          // split-K arrival counters (device, kept zero)
    size_t n_tickets = 0;
    uint64_t launches = 0;
    float *rope_freq = nullptr;      // theta^(2i/d) table (device)
    int rope_hd = 0;
    float rope_theta = 0.f;
    float *hbuf_x = nullptr, *hbuf_y = nullptr;   // staging for *_host entry points
    size_t hbuf_x_bytes = 0, hbuf_y_bytes = 0;
    int *flag = nullptr;             // device error flag for bounded waits
    float *scratch = nullptr;        // gate/up outputs when a SwiGLU pair runs unfused
    size_t scratch_bytes = 0;
    float *xbf = nullptr;            // bf16 copy of GEMM activations (TMA source)
    size_t xbf_bytes = 0;
    float *wbf = nullptr;            // dequantized weight rows of the two-pass GEMM (TMA source)
    size_t wbf_bytes = 0;
    float *samp = nullptr;           // logits processor: sorted rows, segment offsets, sort scratch
    size_t samp_bytes = 0;
    float *kt_x = nullptr, *kt_y = nullptr;   // token-major copies for the [K][T] Q-GEMM entry points
    size_t kt_x_bytes = 0, kt_y_bytes = 0;
    unsigned long long *amax_keys = nullptr;  // fused LM-head argmax: 16 keys + a CTA counter, kept zero
};

struct hd_weight {
    int type = 0;
    int64_t rows = 0, cols = 0;
    size_t gguf_bytes = 0;
    int units = 0;                   // cols / 32
    int nsb = 0;                     // cols / 256 (K-quants)
    uint8_t *base = nullptr;         // one allocation holding every array
    size_t alloc_bytes = 0;
    uint8_t *q = nullptr, *aux = nullptr, *meta = nullptr;
    uint16_t *dsb = nullptr;
    // 2^f16_shift * |w| <= 2^15 for every dequantized value w (bound from the
    // block scales at upload): the exact-product tensor-core GEMM splits
    // scaled weights into fp16 halves without overflow
    int f16_shift = 0;
};

// Plain view passed by value to kernels.
struct WView {
    const uint8_t *q, *aux, *meta;
    const uint16_t *dsb;
    int64_t rows;
    int units;
};

static inline WView wview(const hd_weight *w) {
    return WView{w->q, w->aux, w->meta, w->dsb, w->rows, w->units};
}

// ------------------------------------------------------------------ errors
int hd_fail(hd_ctx *ctx, int code, const char *fmt, ...);
#define HD_CUDA_TRY(ctx, expr)                                                         \
    do {                                                                               \
        cudaError_t e_ = (expr);                                                       \
        if (e_ != cudaSuccess)                                                         \
            return hd_fail((ctx), HD_E_CUDA, "%s: %s (%s:%d)", #expr,                  \
                           cudaGetErrorString(e_), __FILE__, __LINE__);                \
    } while (0)
#define HD_REQUIRE(ctx, cond, code, ...)                                               \
    do {                                                                               \
        if (!(cond)) return hd_fail((ctx), (code), __VA_ARGS__);                       \
    } while (0)

int hd_ensure_workspace(hd_ctx *ctx, size_t bytes, size_t tickets);
int hd_ensure_amax_keys(hd_ctx *ctx);
// LM head (+ RMSNorm when norm_w != null) with the greedy argmax fused at
// batch <= 4: logits [B][rows], idx [B].
int hd_lm_head_argmax_run(hd_ctx *ctx, const hd_weight *w, const float *x, const float *norm_w, float eps,
                          float *logits, int32_t *idx, int B);
int hd_ensure_rope(hd_ctx *ctx, int head_dim, float theta);
int hd_check_launch(hd_ctx *ctx, const char *what);
bool hd_type_supported(int t);
int hd_ensure_hbuf(hd_ctx *ctx, float **buf, size_t *have, size_t need);
int hd_qgemm_f32(hd_ctx *ctx, const hd_weight *w, const float *X, float *Y, int T);
// Attention over `rows` query rows (see k_attention in hd_attention.cu).
// early_kv: cache rows below each row's length are final before the
// previous kernel starts (loads may be issued before the dependency wait).
int hd_attention_run(hd_ctx *ctx, const float *q, int64_t qld, const float *kc, const float *vc, const int32_t *lens,
                     int rows, int pos0, int seqT, int n_heads, int n_kv, int hd, int max_ctx, int maxlen, float *out,
                     const char *name, const int32_t *slots = nullptr, const float *rope_freq = nullptr,
                     const int32_t *rope_pos = nullptr, bool early_kv = false);
// Q-GEMV (B <= 16) of rmsnorm(x) with the norm in each CTA's prologue;
// w_up != null: SwiGLU pair.
// The decoder's GEMVs: y = W x, W rmsnorm(x) (norm_w) or the SwiGLU pair
// (w_up), on the kernels its greedy tokens are pinned to (hd_gemv.cu).
int hd_qgemv_pinned(hd_ctx *ctx, const hd_weight *w, const hd_weight *w_up, const float *x, const float *norm_w,
                    float eps, float *y, int B, const float *bias, const float *residual);
int hd_qgemv_norm(hd_ctx *ctx, const hd_weight *w, const hd_weight *w_up, const float *x, const float *norm_w,
                  float eps, float *y, int B, const float *bias, const float *residual);
// Streamed Q-GEMV at batch 1..4 (hd_gemv_sk.cu): y = W x (+bias, +residual);
// the weight must satisfy hd_qgemv_sk_fits (cols % 128 == 0).
bool hd_qgemv_sk_fits(const hd_weight *w);
// Q-GEMV of a few-MB weight at batch 1..16 on the tensor cores, K parts of a
// 32-row tile in a thread-block cluster (hd_gemv_small.cu).
bool hd_qgemv_small_fits(const hd_weight *w, int B, int sms, bool pair = false);
int hd_qgemv_small(hd_ctx *ctx, const hd_weight *w, const hd_weight *w_up, const float *x, float *y, int B,
                   const float *bias, const float *residual, const float *norm_w, float eps, const char *name);
// Streamed Q-GEMV at batch 1..16 on the tensor cores (hd_gemv_stream.cu):
// 128-row blocks walking K in lockstep through a ring of bulk-copied stages.
bool hd_qgemv_stream_fits(const hd_weight *w, int B, int sms);
int hd_qgemv_stream(hd_ctx *ctx, const hd_weight *w, const float *x, float *y, int B, const float *bias,
                    const float *residual, const char *name);
// Q-GEMV at batch 1..4 in 256-row x unit-group blocks (hd_gemv_blk.cu).
bool hd_qgemv_blk_fits(const hd_weight *w);
int hd_qgemv_blk(hd_ctx *ctx, const hd_weight *w, const float *x, float *y, int B, const float *bias,
                 const float *residual, const char *name);
// Q-GEMV at batch 1..4 with the products on the tensor cores (hd_gemv_mma.cu);
// the weight must satisfy hd_qgemv_mma_fits.
bool hd_qgemv_mma_fits(const hd_weight *w);
int hd_qgemv_mma(hd_ctx *ctx, const hd_weight *w, const float *x, float *y, int B, const float *bias,
                 const float *residual, const char *name);
int hd_qgemv_sk(hd_ctx *ctx, const hd_weight *w, const float *x, float *y, int B, const float *bias,
                const float *residual, const char *name);
// Q-GEMV at batch 5..16 on the tensor cores (hd_gemv_tc.cu).  *done = false
// (and HD_OK) when the batch or shape is outside what the kernel takes; the
// caller then runs the CUDA-core kernels.
int hd_qgemv_tc(hd_ctx *ctx, const hd_weight *w, const float *x, float *y, int B, const float *bias,
                const float *residual, bool *done);
// Fused q|k|v rows (row stride ld): RoPE on q and k heads in place, rotated k
// and v appended to cache sequence r / T at position pos[r].
int hd_rope_kv_append(hd_ctx *ctx, float *qkv, int64_t ld, const int32_t *pos, int rows, int T, int n_heads, int n_kv,
                      int hd, float *kc, float *vc, int max_ctx);

// Launch with programmatic stream serialization, so the next kernel's
// pre-dependency prologue (weight prefetch) overlaps this one's tail.
template <typename... KArgs, typename... Args>
static inline cudaError_t hd_launch(hd_ctx *ctx, void (*kern)(KArgs...), dim3 grid, dim3 block,
                                    size_t smem, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = ctx->pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ctx->launches++;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// The same with thread-block clusters of `cluster` CTAs along x (grid.x a
// multiple of it).
template <typename... KArgs, typename... Args>
static inline cudaError_t hd_launch_cluster(hd_ctx *ctx, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                            int cluster, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = ctx->pdl ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    ctx->launches++;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ------------------------------------------------------- device utilities
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Read-only loads that stay where they are written.  __ldg loads are marked
// invariant, so the compiler may move them past griddepcontrol.wait to their
// first use; weight loads meant to overlap the previous kernel use these.
__device__ __forceinline__ uint32_t ld_pin_u16(const void *p) {
    unsigned short v;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ld_pin_u32(const void *p) {
    uint32_t v;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ld_pin_v2(const void *p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ld_pin_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ float h2f(uint16_t h) {
    return __half2float(__ushort_as_half(h));   // exact, subnormals kept
}

// Float value 2^23 + byte c of v (exact): byte_perm builds 0x4B0000bb.
__device__ __forceinline__ float mag(uint32_t v, int c) {
    return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u + (uint32_t)c));
}

// Q4_K 6-bit scale/min of sub-block j from the 12 packed bytes
// (llama.cpp get_scale_min_k4 layout).
__device__ __forceinline__ void q4k_sm(int j, const uint8_t *s, int &sc, int &m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// Same, with the 12 scale bytes held in three words (bytes 4..15 of the
// super-block header: s[0..3] in y, s[4..7] in z, s[8..11] in w).
__device__ __forceinline__ void q4k_sm_regs(int j, uint32_t y, uint32_t z, uint32_t w, int &sc, int &m) {
    int sh = 8 * (j & 3);
    uint32_t by = (y >> sh) & 255u, bz = (z >> sh) & 255u, bw = (w >> sh) & 255u;
    if (j < 4) {
        sc = (int)(by & 63u);
        m = (int)(bz & 63u);
    } else {
        sc = (int)((bw & 15u) | ((by >> 6) << 4));
        m = (int)((bw >> 4) | ((bz >> 6) << 4));
    }
}

// Exact dequantization of unit u of row r into out[32], in the oracle's
// operation order (no FMA contraction: explicit _rn intrinsics).
template <int TYPE>
__device__ __forceinline__ void decode_unit_exact(const WView &w, int64_t r, int u, float *out) {
    const int64_t ur = (int64_t)u * w.rows + r;
    if (TYPE == HD_TYPE_Q8_0) {
        const int8_t *q = (const int8_t *)(w.q + ur * 32);
        float d = h2f(((const uint16_t *)w.meta)[ur]);
#pragma unroll
        for (int j = 0; j < 32; j++) out[j] = __fmul_rn((float)q[j], d);
    } else if (TYPE == HD_TYPE_Q5_0) {
        const uint8_t *q = w.q + ur * 16;
        uint32_t qh = ((const uint32_t *)w.aux)[ur];
        float d = h2f(((const uint16_t *)w.meta)[ur]);
#pragma unroll
        for (int j = 0; j < 16; j++) {
            int wd = j >> 2, c = j & 3;
            int lo = (q[j] & 15) | (((qh >> (8 * c + 4 + wd)) & 1) << 4);
            int hi = (q[j] >> 4) | (((qh >> (8 * c + wd)) & 1) << 4);
            out[j] = __fmul_rn(__fsub_rn((float)lo, 16.0f), d);
            out[j + 16] = __fmul_rn(__fsub_rn((float)hi, 16.0f), d);
        }
    } else if (TYPE == HD_TYPE_Q4_K) {
        const uint8_t *q = w.q + ur * 16;
        const uint8_t *mt = w.meta + ((int64_t)(u >> 3) * w.rows + r) * 16;
        float d = h2f(mt[0] | (mt[1] << 8)), dmin = h2f(mt[2] | (mt[3] << 8));
        int sc, m;
        q4k_sm(u & 7, mt + 4, sc, m);
        float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
#pragma unroll
        for (int j = 0; j < 16; j++) {
            out[j] = __fsub_rn(__fmul_rn(d1, (float)(q[j] & 15)), m1);
            out[j + 16] = __fsub_rn(__fmul_rn(d1, (float)(q[j] >> 4)), m1);
        }
    } else {  // Q6_K
        const uint8_t *q = w.q + ur * 16;
        uint2 hb = ((const uint2 *)w.aux)[ur];
        const int8_t *sc = (const int8_t *)(w.meta + ((int64_t)(u >> 3) * w.rows + r) * 16);
        float d = h2f(w.dsb[(int64_t)(u >> 3) * w.rows + r]);
        int s0 = 2 * (u & 7);
        float dlo = __fmul_rn(d, (float)sc[s0]), dhi = __fmul_rn(d, (float)sc[s0 + 1]);
#pragma unroll
        for (int j = 0; j < 16; j++) {
            int wd = j >> 2, c = j & 3;
            int hlo = (hb.x >> (8 * c + 2 * wd)) & 3, hhi = (hb.y >> (8 * c + 2 * wd)) & 3;
            int qlo = ((q[j] & 15) | (hlo << 4)) - 32, qhi = ((q[j] >> 4) | (hhi << 4)) - 32;
            out[j] = __fmul_rn(dlo, (float)qlo);
            out[j + 16] = __fmul_rn(dhi, (float)qhi);
        }
    }
}

__host__ __device__ static inline int hd_block_elems(int t) {
    return (t == HD_TYPE_Q4_K || t == HD_TYPE_Q6_K) ? 256 : (t == HD_TYPE_Q8_0 || t == HD_TYPE_Q5_0) ? 32 : 1;
}
__host__ __device__ static inline int hd_block_bytes(int t) {
    return t == HD_TYPE_Q8_0 ? 34 : t == HD_TYPE_Q5_0 ? 22 : t == HD_TYPE_Q4_K ? 144 : t == HD_TYPE_Q6_K ? 210 : 0;
}

// Selects the kernel instance for a runtime type id.
#define HD_TYPE_SWITCH(t, T, ...)                                   \
    switch (t) {                                                    \
    case HD_TYPE_Q8_0: { constexpr int T = HD_TYPE_Q8_0; __VA_ARGS__; break; } \
    case HD_TYPE_Q5_0: { constexpr int T = HD_TYPE_Q5_0; __VA_ARGS__; break; } \
    case HD_TYPE_Q4_K: { constexpr int T = HD_TYPE_Q4_K; __VA_ARGS__; break; } \
    case HD_TYPE_Q6_K: { constexpr int T = HD_TYPE_Q6_K; __VA_ARGS__; break; } \
    default: break;                                                 \
    }
