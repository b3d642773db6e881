// hd_decoder.cu -- Qwen2-shaped decoder run natively on the device.
//
// This is BrainBlock::forward (core/ops/block.rs:51-238) for every layer, made
// correct (RoPE on all heads, GQA kv head h/(nh/nkv), o_proj applied,
// silu(gate)*up, q/k/v biases), followed by the final RMSNorm, the tied LM
// head and ArgMaxSampler (runtime/sampler/argmax.rs:8-24).
//
// Prefill runs all seqs x n_prompt tokens at once: projections through the
// Q-GEMM (fp32 exact-weight or bf16 tcgen05), causal attention per sequence,
// KV cache filled in place.  Decode captures one step -- embed, 24 layers,
// norm, LM head, argmax, state update -- as a CUDA graph and replays it once
// per generated token; positions, lengths, the current tokens and the output
// history live in device memory, so every replay is the same graph.  With at
// most 16 sequences per step the projections are Q-GEMVs with fused bias,
// residual and SwiGLU epilogues; above that they are Q-GEMMs.
//
// KV cache: [layer][seq][max_ctx][n_kv][head_dim] f32.
#include <cstdlib>
#include <cstring>
#include <vector>

#include "hd_internal.cuh"

struct hd_decoder {
    hd_ctx *ctx = nullptr;
    hd_decoder_config c{};
    struct Layer {
        const hd_weight *wq, *wk, *wv, *wo, *wg, *wu, *wd;
        float *bq, *bk, *bv, *attn_norm, *ffn_norm;
        // q, k and v stacked by rows into one weight (owned) and one bias,
        // when their types and widths agree: one projection per layer
        hd_weight *wqkv = nullptr;
        float *bqkv = nullptr;
    };
    std::vector<Layer> L;
    float *out_norm = nullptr;
    const hd_weight *embed = nullptr;
    float *kc = nullptr, *vc = nullptr;
    // decode state, sized for max_seqs
    float *h = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *a = nullptr,
          *g = nullptr, *tmp = nullptr, *logits = nullptr, *qkv = nullptr;
    int32_t *tok = nullptr, *pos = nullptr, *lens = nullptr, *amax = nullptr, *step = nullptr, *hist = nullptr;
    size_t hist_cap = 0;
    std::vector<void *> allocs;
};

namespace {

__global__ void k_bias_add(float *y, const float *__restrict__ b, int64_t rows, int n) {
    pdl_wait();
    pdl_trigger();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < rows * n) y[i] += b[i % n];
}

// Copies row (s*T + T-1) of src [S*T][n] to dst [S][n].
__global__ void k_gather_last(const float *__restrict__ src, float *__restrict__ dst, int S, int T, int n) {
    pdl_wait();
    pdl_trigger();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)S * n) return;
    int s = (int)(i / n), j = (int)(i % n);
    dst[i] = src[((int64_t)s * T + T - 1) * n + j];
}

// After prefill: first generated token, positions and lengths.  With
// teacher forcing (forced [S][n_gen]) the next input is the forced id.
__global__ void k_start(const int32_t *amax, int32_t *tok, int32_t *pos, int32_t *lens, int32_t *step,
                        int32_t *hist, int S, int n_prompt, int n_gen, const int32_t *forced) {
    pdl_wait();
    pdl_trigger();
    int s = threadIdx.x + blockIdx.x * blockDim.x;
    if (s < S) {
        tok[s] = forced ? forced[(int64_t)s * n_gen] : amax[s];
        hist[(int64_t)s * n_gen] = amax[s];
        pos[s] = n_prompt;
        lens[s] = n_prompt + 1;
    }
    if (s == 0) *step = 0;
}

// End of a decode step: the argmax is recorded and becomes the next input
// (with teacher forcing, the forced id of this step does).
__global__ void k_step_end(const int32_t *amax, int32_t *tok, int32_t *pos, int32_t *lens, int32_t *step,
                           int32_t *hist, int S, int n_gen, const int32_t *forced) {
    pdl_wait();
    pdl_trigger();
    __shared__ int st;
    if (threadIdx.x == 0) st = *step + 1;
    __syncthreads();
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
        tok[s] = forced && st < n_gen ? forced[(int64_t)s * n_gen + st] : amax[s];
        if (st < n_gen) hist[(int64_t)s * n_gen + st] = amax[s];
        pos[s] += 1;
        lens[s] += 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) *step = st;
}

template <typename T>
int dalloc(hd_decoder *d, T **p, size_t n) {
    void *q = nullptr;
    if (cudaMalloc(&q, n * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return hd_fail(d->ctx, HD_E_OOM, "decoder: cudaMalloc(%zu) failed", n * sizeof(T));
    }
    d->allocs.push_back(q);
    *p = (T *)q;
    return HD_OK;
}

int upload_vec(hd_decoder *d, float **dst, const float *src, size_t n) {
    int rc = dalloc(d, dst, n);
    if (rc) return rc;
    HD_CUDA_TRY(d->ctx, cudaMemcpy(*dst, src, n * sizeof(float), cudaMemcpyHostToDevice));
    return HD_OK;
}

// y = W x (+bias) for `rows` activation rows; GEMV up to 16 rows, GEMM above.
// With `residual` (which may alias y for GEMV): y = residual + W x.
int linear(hd_decoder *d, const hd_weight *w, const float *x, float *y, int rows, const float *bias, float *residual,
           int prec) {
    hd_ctx *ctx = d->ctx;
    if (rows <= 16) return hd_qgemv_pinned(ctx, w, nullptr, x, nullptr, 0.f, y, rows, bias, residual);
    float *out = residual ? d->tmp : y;
    int rc = hd_qgemm(ctx, w, x, out, rows, prec);
    if (rc) return rc;
    int64_t n = (int64_t)rows * w->rows;
    if (bias) {
        HD_CUDA_TRY(ctx, hd_launch(ctx, k_bias_add, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, out,
                                   (const float *)bias, (int64_t)rows, (int)w->rows));
    }
    if (residual) return hd_add(ctx, residual, out, y, n);
    return HD_OK;
}

int ffn_gate_up(hd_decoder *d, const hd_decoder::Layer &l, const float *x, float *a, int rows, int prec) {
    if (rows <= 16) return hd_qgemv_pinned(d->ctx, l.wg, l.wu, x, nullptr, 0.f, a, rows, nullptr, nullptr);
    int rc = hd_qgemm(d->ctx, l.wg, x, d->g, rows, prec);
    if (!rc) rc = hd_qgemm(d->ctx, l.wu, x, d->tmp, rows, prec);
    if (!rc) rc = hd_swiglu(d->ctx, d->g, d->tmp, a, (int64_t)rows * d->c.ffn);
    return rc;
}

// One decoder layer over `rows` activation rows held in d->h.  Attention:
// decode (lens != null, one row per sequence) or prefill (rows = S*T).
int layer_forward(hd_decoder *d, int li, int rows, const int32_t *pos, const int32_t *lens, int S, int T, int prec,
                  const int32_t *pos0_zero) {
    hd_ctx *ctx = d->ctx;
    const hd_decoder_config &c = d->c;
    const hd_decoder::Layer &l = d->L[li];
    const int hd = c.head_dim, nkv = c.n_kv * hd;
    const size_t lay = (size_t)li * c.max_seqs * c.max_ctx * nkv;
    // up to 16 rows the RMSNorm runs inside the projection that consumes it
    const bool gemv = rows <= 16 && l.wqkv;
    int rc = gemv ? HD_OK : hd_rmsnorm(ctx, d->h, l.attn_norm, nullptr, d->xn, rows, c.hidden, c.eps);
    if (l.wqkv) {
        // one q|k|v projection, RoPE + cache append in one kernel, attention
        // reading q from the fused rows
        const int64_t ld = l.wqkv->rows;
        if (!rc)
            rc = gemv ? hd_qgemv_pinned(ctx, l.wqkv, nullptr, d->h, l.attn_norm, c.eps, d->qkv, rows, l.bqkv, nullptr)
                      : linear(d, l.wqkv, d->xn, d->qkv, rows, l.bqkv, nullptr, prec);
        // decode: RoPE and the cache append run inside the attention kernel
        if (!rc && !lens)
            rc = hd_rope_kv_append(ctx, d->qkv, ld, pos, rows, T, c.n_heads, c.n_kv, hd, d->kc + lay, d->vc + lay,
                                   c.max_ctx);
        if (rc) return rc;
        if (lens)
            rc = hd_attention_run(ctx, d->qkv, ld, d->kc + lay, d->vc + lay, lens, S, 0, 1, c.n_heads, c.n_kv, hd,
                                  c.max_ctx, c.max_ctx, d->att, "decoder attention", nullptr, ctx->rope_freq, pos,
                                  true);  // cache rows below pos were written a step or more earlier
        else
            rc = hd_attention_run(ctx, d->qkv, ld, d->kc + lay, d->vc + lay, nullptr, rows, 0, T, c.n_heads, c.n_kv,
                                  hd, c.max_ctx, T, d->att, "decoder prefill attention");
    } else {
        if (!rc) rc = linear(d, l.wq, d->xn, d->q, rows, l.bq, nullptr, prec);
        if (!rc) rc = linear(d, l.wk, d->xn, d->k, rows, l.bk, nullptr, prec);
        if (!rc) rc = linear(d, l.wv, d->xn, d->v, rows, l.bv, nullptr, prec);
        if (!rc) rc = hd_rope_neox(ctx, d->q, pos, rows, c.n_heads, hd, c.theta);
        if (!rc) rc = hd_rope_neox(ctx, d->k, pos, rows, c.n_kv, hd, c.theta);
        if (rc) return rc;
        if (lens) {
            rc = hd_kv_append(ctx, d->k, d->v, d->kc + lay, d->vc + lay, pos, S, 1, c.n_kv, hd, c.max_ctx);
            if (!rc) rc = hd_attention_run(ctx, d->q, 0, d->kc + lay, d->vc + lay, lens, S, 0, 1, c.n_heads, c.n_kv,
                                           hd, c.max_ctx, c.max_ctx, d->att, "decoder attention");
        } else {
            rc = hd_kv_append(ctx, d->k, d->v, d->kc + lay, d->vc + lay, pos0_zero, S, T, c.n_kv, hd, c.max_ctx);
            if (!rc) rc = hd_attention_run(ctx, d->q, 0, d->kc + lay, d->vc + lay, nullptr, rows, 0, T, c.n_heads,
                                           c.n_kv, hd, c.max_ctx, T, d->att, "decoder prefill attention");
        }
    }
    if (!rc) rc = linear(d, l.wo, d->att, d->h, rows, nullptr, d->h, prec);
    if (gemv) {
        if (!rc) rc = hd_qgemv_pinned(ctx, l.wg, l.wu, d->h, l.ffn_norm, c.eps, d->a, rows, nullptr, nullptr);
    } else {
        if (!rc) rc = hd_rmsnorm(ctx, d->h, l.ffn_norm, nullptr, d->xn, rows, c.hidden, c.eps);
        if (!rc) rc = ffn_gate_up(d, l, d->xn, d->a, rows, prec);
    }
    if (!rc) rc = linear(d, l.wd, d->a, d->h, rows, nullptr, d->h, prec);
    return rc;
}

// Final norm, LM head and argmax for S rows of `hid`.
int head(hd_decoder *d, const float *hid, int S, int prec) {
    hd_ctx *ctx = d->ctx;
    int rc;
    if (S <= 16 && getenv("HACEDLE_DECODER_UNFUSED") == nullptr) {
        // final norm, LM head and (up to 4 rows) the greedy argmax in one launch
        return hd_lm_head_argmax_run(ctx, d->embed, hid, d->out_norm, d->c.eps, d->logits, d->amax, S);
    }
    rc = hd_rmsnorm(ctx, hid, d->out_norm, nullptr, d->xn, S, d->c.hidden, d->c.eps);
    if (!rc) rc = linear(d, d->embed, d->xn, d->logits, S, nullptr, nullptr, prec);
    if (!rc) rc = hd_argmax_rows(ctx, d->logits, S, d->c.vocab, d->amax);
    return rc;
}

int decode_step(hd_decoder *d, int S, int n_gen, int prec, const int32_t *forced) {
    hd_ctx *ctx = d->ctx;
    int rc = hd_embed(ctx, d->embed, d->tok, S, d->h);
    for (int li = 0; !rc && li < d->c.n_layers; li++) rc = layer_forward(d, li, S, d->pos, d->lens, S, 1, prec, nullptr);
    if (!rc) rc = head(d, d->h, S, prec);
    if (rc) return rc;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_step_end, dim3(1), dim3(256), 0, (const int32_t *)d->amax, d->tok, d->pos,
                               d->lens, d->step, d->hist, S, n_gen, forced));
    return HD_OK;
}

void free_all(hd_decoder *d) {
    for (hd_decoder::Layer &l : d->L)
        if (l.wqkv) {
            hd_weight_free(d->ctx, l.wqkv);
            l.wqkv = nullptr;
        }
    for (void *p : d->allocs) cudaFree(p);
    d->allocs.clear();
}

// Stacks q, k and v by rows: the GGUF bytes of a weight are its rows in
// order, so the stacked weight is the three byte strings one after another.
int build_qkv(hd_decoder *d, hd_decoder::Layer &D, const hd_layer_weights &l) {
    hd_ctx *ctx = d->ctx;
    const hd_weight *ws[3] = {l.wq, l.wk, l.wv};
    for (const hd_weight *w : ws)
        if (w->type != l.wq->type || w->cols != l.wq->cols) return HD_OK;  // keep separate projections
    size_t total = 0;
    for (const hd_weight *w : ws) total += w->gguf_bytes;
    std::vector<uint8_t> bytes(total);
    size_t off = 0;
    for (const hd_weight *w : ws) {
        int rc = hd_weight_download(ctx, w, bytes.data() + off, w->gguf_bytes);
        if (rc) return rc;
        off += w->gguf_bytes;
    }
    const int64_t rows = l.wq->rows + l.wk->rows + l.wv->rows;
    int rc = hd_weight_upload(ctx, bytes.data(), total, l.wq->type, rows, l.wq->cols, &D.wqkv);
    if (rc) return rc;
    std::vector<float> b((size_t)rows);
    memcpy(b.data(), l.bq, sizeof(float) * l.wq->rows);
    memcpy(b.data() + l.wq->rows, l.bk, sizeof(float) * l.wk->rows);
    memcpy(b.data() + l.wq->rows + l.wk->rows, l.bv, sizeof(float) * l.wv->rows);
    return upload_vec(d, &D.bqkv, b.data(), (size_t)rows);
}

}  // namespace

extern "C" int hd_decoder_create(hd_ctx *ctx, const hd_decoder_config *cfg, const hd_layer_weights *layers,
                                 const float *out_norm_host, const hd_weight *embed, hd_decoder **out) {
    if (!ctx || !cfg || !layers || !out_norm_host || !embed || !out)
        return hd_fail(ctx, HD_E_ARG, "hd_decoder_create: null argument");
    *out = nullptr;
    const hd_decoder_config &c = *cfg;
    HD_REQUIRE(ctx, c.hidden > 0 && c.n_layers > 0 && c.n_heads > 0 && c.n_kv > 0 && c.n_heads % c.n_kv == 0 &&
                        c.n_heads * c.head_dim > 0 && c.ffn > 0 && c.vocab > 0 && c.max_ctx > 0 && c.max_seqs > 0 &&
                        c.max_seqs <= 4096,
               HD_E_SHAPE, "hd_decoder_create: bad config");
    HD_REQUIRE(ctx, embed->rows == c.vocab && embed->cols == c.hidden, HD_E_SHAPE,
               "hd_decoder_create: embedding is [%lld, %lld], config wants [%d, %d]", (long long)embed->rows,
               (long long)embed->cols, c.vocab, c.hidden);
    const int nq = c.n_heads * c.head_dim, nkv = c.n_kv * c.head_dim;
    for (int i = 0; i < c.n_layers; i++) {
        const hd_layer_weights &l = layers[i];
        bool ok = l.wq && l.wk && l.wv && l.wo && l.wg && l.wu && l.wd && l.bq && l.bk && l.bv && l.attn_norm &&
                  l.ffn_norm;
        HD_REQUIRE(ctx, ok, HD_E_ARG, "hd_decoder_create: layer %d has a null weight", i);
        ok = l.wq->rows == nq && l.wq->cols == c.hidden && l.wk->rows == nkv && l.wk->cols == c.hidden &&
             l.wv->rows == nkv && l.wv->cols == c.hidden && l.wo->rows == c.hidden && l.wo->cols == nq &&
             l.wg->rows == c.ffn && l.wg->cols == c.hidden && l.wu->rows == c.ffn && l.wu->cols == c.hidden &&
             l.wd->rows == c.hidden && l.wd->cols == c.ffn;
        HD_REQUIRE(ctx, ok, HD_E_SHAPE, "hd_decoder_create: layer %d weight shapes do not match the config", i);
    }
    cudaSetDevice(ctx->device);
    hd_decoder *d = new hd_decoder();
    d->ctx = ctx;
    d->c = c;
    d->embed = embed;
    int rc = HD_OK;
    d->L.resize(c.n_layers);
    for (int i = 0; i < c.n_layers && !rc; i++) {
        const hd_layer_weights &l = layers[i];
        hd_decoder::Layer &D = d->L[i];
        D.wq = l.wq; D.wk = l.wk; D.wv = l.wv; D.wo = l.wo; D.wg = l.wg; D.wu = l.wu; D.wd = l.wd;
        rc = upload_vec(d, &D.bq, l.bq, nq);
        if (!rc) rc = upload_vec(d, &D.bk, l.bk, nkv);
        if (!rc) rc = upload_vec(d, &D.bv, l.bv, nkv);
        if (!rc) rc = upload_vec(d, &D.attn_norm, l.attn_norm, c.hidden);
        if (!rc) rc = upload_vec(d, &D.ffn_norm, l.ffn_norm, c.hidden);
        if (!rc && getenv("HACEDLE_DECODER_UNFUSED") == nullptr) rc = build_qkv(d, D, l);
    }
    if (!rc) rc = upload_vec(d, &d->out_norm, out_norm_host, c.hidden);
    size_t kvn = (size_t)c.n_layers * c.max_seqs * c.max_ctx * nkv;
    if (!rc) rc = dalloc(d, &d->kc, kvn);
    if (!rc) rc = dalloc(d, &d->vc, kvn);
    if (!rc) rc = hd_ensure_rope(ctx, c.head_dim, c.theta);
    if (rc) {
        free_all(d);
        delete d;
        return rc;
    }
    *out = d;
    return HD_OK;
}

extern "C" int hd_decoder_free(hd_decoder *d) {
    if (!d) return HD_E_ARG;
    cudaStreamSynchronize(d->ctx->stream);
    free_all(d);
    delete d;
    return HD_OK;
}

extern "C" int hd_decoder_generate(hd_decoder *d, const int32_t *prompts, int S, int n_prompt, int n_gen, int prec,
                                   int32_t *out, float *decode_ms, float *prefill_ms) {
    return hd_decoder_generate_ex(d, prompts, S, n_prompt, n_gen, prec, nullptr, out, nullptr, decode_ms, prefill_ms);
}

extern "C" int hd_decoder_generate_ex(hd_decoder *d, const int32_t *prompts, int S, int n_prompt, int n_gen,
                                      int prec, const int32_t *forced_host, int32_t *out, float *logits_host,
                                      float *decode_ms, float *prefill_ms) {
    if (!d || !prompts || !out) return d ? hd_fail(d->ctx, HD_E_ARG, "hd_decoder_generate: null argument") : HD_E_ARG;
    hd_ctx *ctx = d->ctx;
    const hd_decoder_config &c = d->c;
    HD_REQUIRE(ctx, S >= 1 && S <= c.max_seqs, HD_E_ARG, "hd_decoder_generate: %d sequences (max %d)", S, c.max_seqs);
    HD_REQUIRE(ctx, n_prompt >= 1 && n_gen >= 1 && n_prompt + n_gen <= c.max_ctx, HD_E_ARG,
               "hd_decoder_generate: prompt %d + generate %d exceeds max_ctx %d", n_prompt, n_gen, c.max_ctx);
    HD_REQUIRE(ctx, prec == HD_PREC_FP32 || prec == HD_PREC_BF16_TC, HD_E_ARG, "hd_decoder_generate: precision");
    cudaSetDevice(ctx->device);
    const int nq = c.n_heads * c.head_dim, nkv = c.n_kv * c.head_dim;
    const int R = S * n_prompt;  // prefill rows
    const int Rm = R > S ? R : S;

    // Activations sized for the prefill (the decode step reuses them).
    std::vector<void *> mark(d->allocs);
    auto release = [&]() {
        for (size_t i = mark.size(); i < d->allocs.size(); i++) cudaFree(d->allocs[i]);
        d->allocs.resize(mark.size());
    };
    int rc = dalloc(d, &d->h, (size_t)Rm * c.hidden);
    if (!rc) rc = dalloc(d, &d->xn, (size_t)Rm * c.hidden);
    if (!rc) rc = dalloc(d, &d->q, (size_t)Rm * nq);
    if (!rc) rc = dalloc(d, &d->qkv, (size_t)Rm * (nq + 2 * nkv));
    if (!rc) rc = dalloc(d, &d->k, (size_t)Rm * nkv);
    if (!rc) rc = dalloc(d, &d->v, (size_t)Rm * nkv);
    if (!rc) rc = dalloc(d, &d->att, (size_t)Rm * nq);
    if (!rc) rc = dalloc(d, &d->a, (size_t)Rm * c.ffn);
    if (!rc) rc = dalloc(d, &d->g, (size_t)Rm * c.ffn);
    size_t tmpn = (size_t)Rm * (c.ffn > c.hidden ? c.ffn : c.hidden);
    if (!rc) rc = dalloc(d, &d->tmp, tmpn);
    if (!rc) rc = dalloc(d, &d->logits, (size_t)S * c.vocab);
    int32_t *ids = nullptr, *ppos = nullptr, *zero = nullptr, *forced = nullptr;
    if (!rc && forced_host) rc = dalloc(d, &forced, (size_t)S * n_gen);
    if (!rc) rc = dalloc(d, &ids, (size_t)R);
    if (!rc) rc = dalloc(d, &ppos, (size_t)R);
    if (!rc) rc = dalloc(d, &zero, (size_t)S);
    if (!rc) rc = dalloc(d, &d->tok, (size_t)S);
    if (!rc) rc = dalloc(d, &d->pos, (size_t)S);
    if (!rc) rc = dalloc(d, &d->lens, (size_t)S);
    if (!rc) rc = dalloc(d, &d->amax, (size_t)S);
    if (!rc) rc = dalloc(d, &d->step, 1);
    if (!rc) rc = dalloc(d, &d->hist, (size_t)S * n_gen);
    if (rc) {
        release();
        return rc;
    }
    std::vector<int32_t> hp(R);
    for (int i = 0; i < R; i++) hp[i] = i % n_prompt;
    // Work runs on the context's own non-blocking stream, ordered after the
    // caller's stream: stream capture is not allowed on the legacy default
    // stream, which a caller may have selected.
    cudaStream_t user = ctx->stream, st = ctx->own_stream;
    cudaEvent_t e0, e1, e2;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventCreate(&e2);
    cudaEventRecord(e0, user);
    cudaStreamWaitEvent(st, e0, 0);
    ctx->stream = st;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    float t_pre = 0.f, t_dec = 0.f;
    do {
        if ((rc = hd_ctx_reserve_workspace(ctx, (size_t)64 << 20))) break;
        // the context's RoPE table may have been rebuilt for another head
        // size since create (hd_rope_neox); the kernels below read it
        if ((rc = hd_ensure_rope(ctx, c.head_dim, c.theta))) break;
        if ((rc = hd_ensure_hbuf(ctx, &ctx->scratch, &ctx->scratch_bytes, (size_t)2 * 16 * c.ffn * sizeof(float))))
            break;
        if (cudaMemcpyAsync(ids, prompts, (size_t)R * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(ppos, hp.data(), (size_t)R * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemsetAsync(zero, 0, (size_t)S * 4, st) != cudaSuccess ||
            (forced && cudaMemcpyAsync(forced, forced_host, (size_t)S * n_gen * 4, cudaMemcpyHostToDevice, st) !=
                           cudaSuccess)) {
            rc = hd_fail(ctx, HD_E_CUDA, "hd_decoder_generate: staging copies failed");
            break;
        }
        cudaEventRecord(e0, st);
        // ---- prefill
        rc = hd_embed(ctx, d->embed, ids, R, d->h);
        for (int li = 0; !rc && li < c.n_layers; li++) rc = layer_forward(d, li, R, ppos, nullptr, S, n_prompt, prec, zero);
        if (rc) break;
        if (cudaSuccess != hd_launch(ctx, k_gather_last, dim3((unsigned)(((int64_t)S * c.hidden + 255) / 256)),
                                     dim3(256), 0, (const float *)d->h, d->tmp, S, n_prompt, c.hidden)) {
            rc = hd_fail(ctx, HD_E_CUDA, "hd_decoder_generate: gather");
            break;
        }
        if ((rc = head(d, d->tmp, S, HD_PREC_FP32))) break;
        if (cudaSuccess != hd_launch(ctx, k_start, dim3((unsigned)((S + 255) / 256)), dim3(256), 0,
                                     (const int32_t *)d->amax, d->tok, d->pos, d->lens, d->step, d->hist, S, n_prompt,
                                     n_gen, (const int32_t *)forced)) {
            rc = hd_fail(ctx, HD_E_CUDA, "hd_decoder_generate: start");
            break;
        }
        cudaEventRecord(e1, st);
        const size_t step_logits = (size_t)S * c.vocab;
        if (logits_host && cudaMemcpyAsync(logits_host, d->logits, step_logits * 4, cudaMemcpyDeviceToHost, st) !=
                               cudaSuccess) {
            rc = hd_fail(ctx, HD_E_CUDA, "hd_decoder_generate: logits copy");
            break;
        }
        if (cudaStreamSynchronize(st) != cudaSuccess) {
            rc = hd_fail(ctx, HD_E_CUDA, "hd_decoder_generate: prefill: %s", cudaGetErrorString(cudaGetLastError()));
            break;
        }
        if ((rc = hd_ctx_check_device_errors(ctx))) break;
        cudaEventElapsedTime(&t_pre, e0, e1);
        // ---- decode: capture one step, replay n_gen - 1 times
        if (n_gen > 1) {
            if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
                rc = hd_fail(ctx, HD_E_CUDA, "hd_decoder_generate: begin capture");
                break;
            }
            rc = decode_step(d, S, n_gen, HD_PREC_FP32, forced);
            cudaError_t ce = cudaStreamEndCapture(st, &graph);
            cudaGetLastError();
            if (rc) break;
            if (ce != cudaSuccess || cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) {
                rc = hd_fail(ctx, HD_E_CUDA, "hd_decoder_generate: graph: %s", cudaGetErrorString(ce));
                break;
            }
            cudaEventRecord(e1, st);
            for (int i = 0; i < n_gen - 1; i++) {
                if (cudaGraphLaunch(exec, st) != cudaSuccess) {
                    rc = hd_fail(ctx, HD_E_CUDA, "hd_decoder_generate: graph launch");
                    break;
                }
                if (logits_host && cudaMemcpyAsync(logits_host + (size_t)(i + 1) * step_logits, d->logits,
                                                   step_logits * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) {
                    rc = hd_fail(ctx, HD_E_CUDA, "hd_decoder_generate: logits copy");
                    break;
                }
            }
            if (rc) break;
            cudaEventRecord(e2, st);
        }
        if (cudaMemcpyAsync(out, d->hist, (size_t)S * n_gen * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess) {
            rc = hd_fail(ctx, HD_E_CUDA, "hd_decoder_generate: decode: %s", cudaGetErrorString(cudaGetLastError()));
            break;
        }
        if (n_gen > 1) cudaEventElapsedTime(&t_dec, e1, e2);
    } while (0);
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    cudaStreamSynchronize(st);
    ctx->stream = user;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaEventDestroy(e2);
    release();
    if (decode_ms) *decode_ms = t_dec;
    if (prefill_ms) *prefill_ms = t_pre;
    return rc;
}
