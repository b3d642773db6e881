// hd_attention.cu -- device KV cache append and GQA attention.
//
// Cache layout [seq][max_ctx][n_kv][head_dim] f32, the KvCache layout of
// core/ops/block.rs:241-282 with a leading sequence index.
//
// One CTA per (query row, kv head) serves the n_heads/n_kv query heads that
// share that kv head, so every K/V row is read once for all of them.  Scores
// go to shared memory, softmax is the exact two-pass form of
// NativeBackend::softmax (max, sum of exp, exp/sum), then each thread sums
// p_i * v_i[d] over positions for its (head, d) outputs.
#include "hd_internal.cuh"

namespace {

__global__ void k_kv_append(const float *__restrict__ k, const float *__restrict__ v, float *kc, float *vc,
                            const int32_t *__restrict__ pos0, int seqs, int tokens, int width, int max_ctx) {
    pdl_wait();
    pdl_trigger();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t total = (int64_t)seqs * tokens * width;
    if (i >= total) return;
    int e = (int)(i % width);
    int64_t st = i / width;
    int t = (int)(st % tokens), s = (int)(st / tokens);
    int p = pos0[s] + t;
    if (p < 0 || p >= max_ctx) return;  // KvCache::append ignores pos >= max_seq_len
    int64_t dst = ((int64_t)s * max_ctx + p) * width + e;
    kc[dst] = k[i];
    vc[dst] = v[i];
}

// rows: query rows; row r reads cache sequence cseq(r) with length len(r):
//   decode  (lens != null): cseq = r, len = lens[r]
//   prefill (lens == null): rows are seqT consecutive tokens per sequence,
//                           cseq = r / seqT, len = pos0 + r % seqT + 1
template <int HD>
__global__ void __launch_bounds__(128) k_attention(const float *__restrict__ q, const float *__restrict__ kc,
                                                   const float *__restrict__ vc, const int32_t *__restrict__ lens,
                                                   int pos0, int seqT, int n_heads, int n_kv, int max_ctx,
                                                   float scale, float *__restrict__ out) {
    extern __shared__ float sm[];
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x, kvh = blockIdx.y;
    const int rep = n_heads / n_kv, h0 = kvh * rep;
    const int cseq = lens ? r : r / seqT;
    int L = lens ? lens[r] : pos0 + r % seqT + 1;
    L = L < 0 ? 0 : L > max_ctx ? max_ctx : L;
    float *qs = sm;               // [rep][HD]
    float *sc = sm + rep * HD;    // [rep][L]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *qr = q + ((int64_t)r * n_heads + h0) * HD;
    for (int i = tid; i < rep * HD; i += 128) qs[i] = qr[i];
    __syncthreads();
    const int64_t cbase = (int64_t)cseq * max_ctx;
    constexpr int PL = HD / 32;  // dims per lane
    for (int p = warp; p < L; p += 4) {
        const float *kp = kc + ((cbase + p) * n_kv + kvh) * HD;
        float kv[PL];
#pragma unroll
        for (int j = 0; j < PL; j++) kv[j] = kp[lane + 32 * j];
        for (int h = 0; h < rep; h++) {
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < PL; j++) s = fmaf(qs[h * HD + lane + 32 * j], kv[j], s);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) sc[h * L + p] = __fdiv_rn(s, scale);
        }
    }
    __syncthreads();
    for (int h = warp; h < rep; h += 4) {
        float *row = sc + h * L;
        float m = -INFINITY;
        for (int p = lane; p < L; p += 32) m = fmaxf(m, row[p]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float s = 0.f;
        for (int p = lane; p < L; p += 32) s += expf(row[p] - m);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        for (int p = lane; p < L; p += 32) row[p] = expf(row[p] - m) / s;
    }
    __syncthreads();
    for (int i = tid; i < rep * HD; i += 128) {
        const int h = i / HD, d = i % HD;
        const float *pr = sc + h * L;
        const float *vp = vc + (cbase * n_kv + kvh) * HD + d;
        float s0 = 0.f, s1 = 0.f;
        int p = 0;
        for (; p + 1 < L; p += 2) {
            s0 = fmaf(pr[p], vp[(int64_t)p * n_kv * HD], s0);
            s1 = fmaf(pr[p + 1], vp[(int64_t)(p + 1) * n_kv * HD], s1);
        }
        if (p < L) s0 = fmaf(pr[p], vp[(int64_t)p * n_kv * HD], s0);
        out[((int64_t)r * n_heads + h0 + h) * HD + d] = s0 + s1;
    }
}

template <int HD>
cudaError_t launch_attn(hd_ctx *ctx, int rows, int n_heads, int n_kv, int maxlen, const float *q, const float *kc,
                        const float *vc, const int32_t *lens, int pos0, int seqT, int max_ctx, float *out) {
    int rep = n_heads / n_kv;
    size_t smem = (size_t)rep * (HD + maxlen) * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_attention<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    float scale = sqrtf((float)HD);
    return hd_launch(ctx, k_attention<HD>, dim3(rows, n_kv), dim3(128), smem, q, kc, vc, lens, pos0, seqT, n_heads,
                     n_kv, max_ctx, scale, out);
}

}  // namespace

int hd_attention_run(hd_ctx *ctx, const float *q, const float *kc, const float *vc, const int32_t *lens, int rows,
                     int pos0, int seqT, int n_heads, int n_kv, int hd, int max_ctx, int maxlen, float *out,
                     const char *name) {
    if (!ctx || !q || !kc || !vc || !out) return hd_fail(ctx, HD_E_ARG, "%s: null argument", name);
    HD_REQUIRE(ctx, n_heads > 0 && n_kv > 0 && n_heads % n_kv == 0, HD_E_SHAPE,
               "%s: n_heads %d is not a multiple of n_kv %d", name, n_heads, n_kv);
    HD_REQUIRE(ctx, max_ctx > 0 && maxlen <= max_ctx, HD_E_SHAPE, "%s: length beyond max_ctx", name);
    size_t smem = (size_t)(n_heads / n_kv) * (hd + maxlen) * sizeof(float);
    HD_REQUIRE(ctx, smem <= 200 * 1024, HD_E_UNSUPPORTED, "%s: %d positions x %d heads exceed shared memory", name,
               maxlen, n_heads / n_kv);
    if (rows == 0) return HD_OK;
    cudaError_t e;
    if (hd == 64) e = launch_attn<64>(ctx, rows, n_heads, n_kv, maxlen, q, kc, vc, lens, pos0, seqT, max_ctx, out);
    else if (hd == 128) e = launch_attn<128>(ctx, rows, n_heads, n_kv, maxlen, q, kc, vc, lens, pos0, seqT, max_ctx, out);
    else if (hd == 32) e = launch_attn<32>(ctx, rows, n_heads, n_kv, maxlen, q, kc, vc, lens, pos0, seqT, max_ctx, out);
    else return hd_fail(ctx, HD_E_UNSUPPORTED, "%s: head_dim %d (32, 64 or 128 supported)", name, hd);
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "%s: %s", name, cudaGetErrorString(e));
    return HD_OK;
}

extern "C" int hd_kv_append(hd_ctx *ctx, const float *k, const float *v, float *kc, float *vc, const int32_t *pos0,
                            int seqs, int tokens, int n_kv, int head_dim, int max_ctx) {
    if (!ctx || !k || !v || !kc || !vc || !pos0) return hd_fail(ctx, HD_E_ARG, "hd_kv_append: null argument");
    HD_REQUIRE(ctx, seqs >= 0 && tokens >= 0 && n_kv > 0 && head_dim > 0 && max_ctx > 0, HD_E_SHAPE,
               "hd_kv_append: bad shape");
    int64_t total = (int64_t)seqs * tokens * n_kv * head_dim;
    if (total == 0) return HD_OK;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_kv_append, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, k, v, kc, vc,
                               pos0, seqs, tokens, n_kv * head_dim, max_ctx));
    return HD_OK;
}

extern "C" int hd_attention_decode(hd_ctx *ctx, const float *q, const float *kc, const float *vc,
                                   const int32_t *len, int seqs, int n_heads, int n_kv, int head_dim, int max_ctx,
                                   float *out) {
    if (!len) return hd_fail(ctx, HD_E_ARG, "hd_attention_decode: null lengths");
    return hd_attention_run(ctx, q, kc, vc, len, seqs, 0, 1, n_heads, n_kv, head_dim, max_ctx, max_ctx, out,
                            "hd_attention_decode");
}

extern "C" int hd_attention_prefill(hd_ctx *ctx, const float *q, const float *kc, const float *vc, int T, int pos0,
                                    int n_heads, int n_kv, int head_dim, int max_ctx, float *out) {
    if (T < 0 || pos0 < 0) return hd_fail(ctx, HD_E_ARG, "hd_attention_prefill: negative size");
    return hd_attention_run(ctx, q, kc, vc, nullptr, T, pos0, T > 0 ? T : 1, n_heads, n_kv, head_dim, max_ctx,
                            pos0 + T, out, "hd_attention_prefill");
}
