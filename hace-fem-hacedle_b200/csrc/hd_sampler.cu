// hd_sampler.cu -- the logits processor and a categorical sampler on the device.
//
// hd_logits_process is LogitsProcessor::process (src/x/provider/candle/
// lmhead.rs:42-111) on every row, with the reference's arithmetic:
//   temperature  l /= max(t, 0.001)                               (:55-60)
//   top-p        walk the logits in descending order adding
//                min(exp(l), 1) in f32 until the sum reaches top_p; that
//                logit is the threshold (0.0 if the sum never reaches it);
//                logits below it become -inf                      (:63-84)
//   top-k        threshold = the (top_k+1)-th largest logit after top-p when
//                0 < top_k < n, else -inf; logits below it become -inf (:87-101)
// (exp of the raw logit, not of a softmax probability, and the k+1-th value as
// the top-k threshold, are the reference's definitions and are kept.)
// Rows are sorted descending once (cub segmented radix sort), one thread per
// row walks its sorted row for the top-p sum in the reference's sequential
// order (usually one step: any logit >= 0 adds 1), and top-k reads the same
// sorted row: after top-p masking the first entries of the descending order
// are unchanged.  A final pass masks each row at max(top-p, top-k) threshold.
//
// hd_sample_rows draws one index per row from softmax(logits) (masked -inf
// entries have probability 0).  Row r uses one Philox4x32-10 block (Salmon
// et al., "Parallel random numbers: as easy as 1, 2, 3", SC'11) with counter
// (offset + r, 0, 0) and key = seed: u = (word0 >> 8) * 2^-24.  A CTA of 256
// threads splits the row into 256 contiguous chunks; thread t sums
// exp(l - max) over its chunk in index order, thread 0 forms the exclusive
// prefix of the chunk sums in thread order, target = u * total, and the
// thread whose chunk holds the target walks it in index order.  The
// arithmetic is fixed by (n, the 256 chunks), so a draw is reproducible.
#include <cub/device/device_segmented_radix_sort.cuh>

#include "hd_internal.cuh"

namespace {

constexpr int SNT = 256;

__device__ __forceinline__ void philox_round(uint32_t (&c)[4], const uint32_t (&k)[2]) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0], p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k[0], n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k[1];
    c[1] = (uint32_t)p1;
    c[3] = (uint32_t)p0;
    c[0] = n0;
    c[2] = n2;
}

__device__ uint32_t philox_word0(uint64_t ctr, uint64_t seed) {
    uint32_t c[4] = {(uint32_t)ctr, (uint32_t)(ctr >> 32), 0u, 0u};
    uint32_t k[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
#pragma unroll
    for (int r = 0; r < 10; r++) {
        philox_round(c, k);
        k[0] += 0x9E3779B9u;
        k[1] += 0xBB67AE85u;
    }
    return c[0];
}

__global__ void k_temperature(float *x, int64_t total, float t) {
    pdl_wait();
    pdl_trigger();
    const float d = fmaxf(t, 0.001f);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = __fdiv_rn(x[i], d);
}

__global__ void k_seg_offsets(int *off, int rows, int n) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r <= rows) off[r] = r * n;
}

// One thread per row: the top-p threshold (sequential f32 walk of the sorted
// row, as the reference sums) and the top-k threshold; thr[r] = the larger.
__global__ void k_thresholds(const float *__restrict__ sorted, int rows, int64_t n, float top_p, int64_t top_k,
                             float *__restrict__ thr) {
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const float *s = sorted + (int64_t)r * n;
    float cum = 0.f, tp = 0.f;
    for (int64_t i = 0; i < n; i++) {
        const float p = s[i];
        cum = __fadd_rn(cum, fminf(expf(p), 1.f));
        if (cum >= top_p) {
            tp = p;
            break;
        }
    }
    float tk = -INFINITY;
    if (top_k > 0 && top_k < n) {
        const float v = s[top_k];
        tk = v >= tp ? v : -INFINITY;  // entries below the top-p threshold are -inf by then
    }
    thr[r] = fmaxf(tp, tk);
}

__global__ void k_mask(float *x, int64_t n, int64_t total, const float *__restrict__ thr) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
        if (x[i] < thr[i / n]) x[i] = -INFINITY;
}

__global__ void __launch_bounds__(SNT) k_sample(const float *__restrict__ logits, int64_t n, uint64_t seed,
                                                uint64_t offset, int32_t *__restrict__ out) {
    __shared__ float red[SNT], pre[SNT + 1];
    __shared__ float target_sh;
    pdl_wait();
    pdl_trigger();
    const int t = threadIdx.x;
    const float *x = logits + (int64_t)blockIdx.x * n;
    float m = -INFINITY;
    for (int64_t i = t; i < n; i += SNT) m = fmaxf(m, x[i]);
    red[t] = m;
    __syncthreads();
    for (int w = SNT / 2; w > 0; w >>= 1) {
        if (t < w) red[t] = fmaxf(red[t], red[t + w]);
        __syncthreads();
    }
    m = red[0];
    __syncthreads();
    const int64_t C = (n + SNT - 1) / SNT, i0 = (int64_t)t * C, i1 = min(n, i0 + C);
    float s = 0.f;
    if (m > -INFINITY)
        for (int64_t i = i0; i < i1; i++) s = __fadd_rn(s, expf(__fsub_rn(x[i], m)));
    red[t] = s;
    __syncthreads();
    if (t == 0) {
        float acc = 0.f;
        for (int j = 0; j < SNT; j++) {
            pre[j] = acc;
            acc = __fadd_rn(acc, red[j]);
        }
        pre[SNT] = acc;
        const float u = (float)(philox_word0(offset + blockIdx.x, seed) >> 8) * (1.0f / 16777216.0f);
        target_sh = __fmul_rn(u, acc);
        out[blockIdx.x] = -1;  // no finite logit: -1
    }
    __syncthreads();
    const float total = pre[SNT], target = target_sh;
    if (!(total > 0.f)) return;
    // the chunk holding the target; a target rounded up to the total goes to
    // the last chunk with mass
    bool mine = pre[t] <= target && target < pre[t + 1];
    if (target >= total) {
        int last = SNT - 1;
        while (last > 0 && !(red[last] > 0.f)) last--;
        mine = t == last;
    }
    if (!mine) return;
    float acc = pre[t];
    int64_t pick = -1;
    for (int64_t i = i0; i < i1; i++) {
        const float e = expf(__fsub_rn(x[i], m));
        if (e > 0.f) pick = i;
        acc = __fadd_rn(acc, e);
        if (acc > target && e > 0.f) break;
    }
    out[blockIdx.x] = (int32_t)pick;
}

}  // namespace

extern "C" int hd_logits_process(hd_ctx *ctx, float *logits, int64_t rows, int64_t n, float temperature, float top_p,
                                 int64_t top_k) {
    if (!ctx || !logits) return hd_fail(ctx, HD_E_ARG, "hd_logits_process: null argument");
    HD_REQUIRE(ctx, rows >= 0 && n > 0 && rows * n < ((int64_t)1 << 31), HD_E_SHAPE,
               "hd_logits_process: rows x n must be below 2^31 (rows %lld, n %lld)", (long long)rows, (long long)n);
    if (rows == 0) return HD_OK;
    const int64_t total = rows * n;
    const unsigned g = (unsigned)((total + 255) / 256 < 4 * (int64_t)ctx->sm_count ? (total + 255) / 256
                                                                                    : 4 * (int64_t)ctx->sm_count);
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_temperature, dim3(g), dim3(256), 0, logits, total, temperature));
    // scratch: sorted rows | thresholds | segment offsets | sort workspace
    size_t sort_bytes = 0;
    cub::DeviceSegmentedRadixSort::SortKeysDescending(nullptr, sort_bytes, (const float *)nullptr, (float *)nullptr,
                                                      (int)total, (int)rows, (const int *)nullptr,
                                                      (const int *)nullptr, 0, 32, ctx->stream);
    const size_t a_sorted = ((size_t)total * 4 + 255) & ~(size_t)255, a_thr = ((size_t)rows * 4 + 255) & ~(size_t)255;
    const size_t a_off = ((size_t)(rows + 1) * 4 + 255) & ~(size_t)255;
    int rc = hd_ensure_hbuf(ctx, &ctx->samp, &ctx->samp_bytes, a_sorted + a_thr + a_off + sort_bytes);
    if (rc) return rc;
    uint8_t *base = (uint8_t *)ctx->samp;
    float *sorted = (float *)base, *thr = (float *)(base + a_sorted);
    int *off = (int *)(base + a_sorted + a_thr);
    void *tmp = base + a_sorted + a_thr + a_off;
    k_seg_offsets<<<(unsigned)((rows + 1 + 255) / 256), 256, 0, ctx->stream>>>(off, (int)rows, (int)n);
    ctx->launches++;
    HD_CUDA_TRY(ctx, cub::DeviceSegmentedRadixSort::SortKeysDescending(tmp, sort_bytes, (const float *)logits, sorted,
                                                                       (int)total, (int)rows, off, off + 1, 0, 32,
                                                                       ctx->stream));
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_thresholds, dim3((unsigned)((rows + 31) / 32)), dim3(32), 0,
                               (const float *)sorted, (int)rows, n, top_p, top_k, thr));
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_mask, dim3(g), dim3(256), 0, logits, n, total, (const float *)thr));
    return HD_OK;
}

extern "C" int hd_sample_rows(hd_ctx *ctx, const float *logits, int64_t rows, int64_t n, uint64_t seed,
                              uint64_t offset, int32_t *idx) {
    if (!ctx || !logits || !idx) return hd_fail(ctx, HD_E_ARG, "hd_sample_rows: null argument");
    HD_REQUIRE(ctx, rows >= 0 && rows <= 2147483647 && n > 0 && n < ((int64_t)1 << 31), HD_E_SHAPE,
               "hd_sample_rows: bad shape (rows %lld, n %lld)", (long long)rows, (long long)n);
    if (rows == 0) return HD_OK;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_sample, dim3((unsigned)rows), dim3(SNT), 0, logits, n, seed, offset, idx));
    return HD_OK;
}
