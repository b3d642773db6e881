// hd_attention.cu -- device KV cache append and GQA attention.
//
// Cache layout [seq][max_ctx][n_kv][head_dim] f32, the KvCache layout of
// core/ops/block.rs:241-282 with a leading sequence index.
//
// A CTA serves the rep = n_heads/n_kv query heads that share one kv head, so
// each K/V row is read once for all of them, over a range of 64-position
// chunks: K and V chunks are staged in shared memory, scores are full
// head_dim dot products, and the softmax runs online across chunks (running
// max, rescaled sum and output).  For decode, where there are few query rows,
// a row's positions are split over P CTAs; each writes its (max, sum, output)
// partial to the workspace and the last to arrive (atomic ticket) combines
// them in chunk order, so the result is deterministic.  The result equals
// NativeBackend::softmax followed by sum_i p_i v_i up to rounding order.
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

// Fused q/k/v rows [rows][ld] = q heads | k heads | v heads: NEOX RoPE on the
// q and k heads in place (the arithmetic of k_rope_neox), and the rotated k
// and v of row r appended to cache sequence r / T at position pos[r].
__global__ void k_rope_kv_append(float *qkv, int64_t ld, const int32_t *__restrict__ pos,
                                 const float *__restrict__ freq, int rows, int T, int n_heads, int n_kv, int hd,
                                 float *kc, float *vc, int max_ctx) {
    pdl_wait();
    pdl_trigger();
    const int half = hd >> 1, nr = n_heads + n_kv;
    const int64_t nrot = (int64_t)rows * nr * half, nv = (int64_t)rows * n_kv * hd;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx < nrot) {
        const int i = (int)(idx % half);
        const int64_t rh = idx / half;
        const int head = (int)(rh % nr), r = (int)(rh / nr);
        float *v = qkv + (int64_t)r * ld + (int64_t)head * hd;
        const int p = pos[r];
        const float angle = __fdiv_rn((float)p, freq[i]);
        const float c = cosf(angle), sn = sinf(angle);
        const float x0 = v[i], x1 = v[i + half];
        const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
        const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
        v[i] = y0;
        v[i + half] = y1;
        if (head >= n_heads && p >= 0 && p < max_ctx) {  // KvCache::append ignores pos >= max_seq_len
            float *dst = kc + (((int64_t)(r / T) * max_ctx + p) * n_kv + (head - n_heads)) * hd;
            dst[i] = y0;
            dst[i + half] = y1;
        }
    } else if (idx < nrot + nv) {
        const int64_t j = idx - nrot;
        const int e = (int)(j % ((int64_t)n_kv * hd)), r = (int)(j / ((int64_t)n_kv * hd));
        const int p = pos[r];
        if (p >= 0 && p < max_ctx)
            vc[((int64_t)(r / T) * max_ctx + p) * n_kv * hd + e] = qkv[(int64_t)r * ld + (int64_t)nr * hd + e];
    }
}

// rows: query rows; row r reads cache sequence cseq(r) with length len(r):
//   decode  (lens != null): cseq = slots ? slots[r] : r, len = lens[r]
//   prefill (lens == null): rows are seqT consecutive tokens per sequence,
//                           cseq = r / seqT, len = pos0 + r % seqT + 1
constexpr int CH = 64;     // positions per chunk
constexpr int ANT = 512;   // threads per CTA: one score and one output chain each (rep x 64 <= 512 for rep <= 8)
constexpr int MAXREP = 16;

// EARLY (the decoder's decode steps): the K and V rows of the CTA's first
// chunk are loaded before griddepcontrol.wait, overlapping the previous
// kernel.  Only callers whose cache rows below the new position were written
// at least one kernel before the previous one may set it (the decoder: a step
// earlier), and lens / slots likewise; the new position's row is replaced
// from shared memory as usual.
template <int HD, bool EARLY>
__global__ void __launch_bounds__(ANT, (EARLY || HD == 128) ? 1 : 2) k_attention(const float *__restrict__ q, int64_t qld, const float *__restrict__ kc,
                                                   const float *__restrict__ vc, const int32_t *__restrict__ lens,
                                                   int pos0, int seqT, int n_heads, int n_kv, int max_ctx,
                                                   float scale, int P, int cpc, float *ws, int *tickets,
                                                   const int32_t *__restrict__ slots, const float *__restrict__ rfreq,
                                                   const int32_t *__restrict__ rpos, float *kcw, float *vcw,
                                                   float *__restrict__ out) {
    extern __shared__ float sm[];
    constexpr int KP = HD + 1;                      // padded K row
    // Register blocking (the same arithmetic per output): a thread takes JB
    // positions of a head's scores (sharing each q load) and DV consecutive
    // dimensions of a head's output (one p load and one vector of V per
    // step); rep <= 16 and HD <= 128 keep both within one pass of 512 threads.
    constexpr int JB = 2, JS = CH / JB, DV = HD >= 128 ? 4 : 2, DQ = HD / DV;
    static_assert(MAXREP * DQ <= ANT && MAXREP * JS <= ANT, "one pass");
    // A chunk's K and V rows: CH * HD / 4 float4 each, NLD per thread per
    // batch.  All loads of a batch are issued before any is stored, so the
    // chunk costs one memory latency per batch rather than one per float4.
    constexpr int NF4 = CH * (HD / 4) / ANT, NB = HD > 64 ? 4 : 8, NLD = NF4 < NB ? NF4 : NB;
    float4 pk[EARLY ? NLD : 1], pv[EARLY ? NLD : 1];
    bool pre = false;
    if constexpr (EARLY) {
        const int re = blockIdx.x, pe = blockIdx.z;
        const int cs = lens ? (slots ? slots[re] : re) : re / seqT;
        int Le = lens ? lens[re] : pos0 + re % seqT + 1;
        Le = Le < 0 ? 0 : Le > max_ctx ? max_ctx : Le;
        const int ce = pe * cpc, j0 = ce * CH;
        if (ce < (Le + CH - 1) / CH) {
            const int nj = min(CH, Le - j0);
#pragma unroll
            for (int u = 0; u < NLD; u++) {
                const int i = threadIdx.x + u * ANT, j = i / (HD / 4), d4 = i % (HD / 4);
                if (j < nj) {
                    const int64_t g = (((int64_t)cs * max_ctx + j0 + j) * n_kv + blockIdx.y) * HD + 4 * d4;
                    pk[u] = __ldg((const float4 *)(kc + g));
                    pv[u] = __ldg((const float4 *)(vc + g));
                }
            }
            pre = true;
        }
    }
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x, kvh = blockIdx.y, p = blockIdx.z;
    const int rep = n_heads / n_kv, h0 = kvh * rep;
    const int cseq = lens ? (slots ? slots[r] : r) : r / seqT;
    int L = lens ? lens[r] : pos0 + r % seqT + 1;
    L = L < 0 ? 0 : L > max_ctx ? max_ctx : L;
    const int nchunks = (L + CH - 1) / CH;
    const int Pr = nchunks == 0 ? 1 : (nchunks + cpc - 1) / cpc;
    if (p >= Pr) return;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float *qs = sm;                                        // [rep][KP]
    float *Ks = qs + rep * KP;                             // [CH][KP]
    float *Vs = sm + ((rep * KP + CH * KP + 3) & ~3);      // [CH][HD], 16-byte aligned for float4 stores
    float *S = Vs + CH * HD;                               // [rep][CH]
    float *mrun = S + rep * CH, *lrun = mrun + MAXREP, *alpha = lrun + MAXREP;
    float *knew = alpha + MAXREP, *vnew = knew + HD;       // fused decode: the new position's k and v
    const float *qr = q + (int64_t)r * qld + (int64_t)h0 * HD;
    // Fused decode (rfreq != null): q of the fused q|k|v row is rotated here
    // (NEOX RoPE with the arithmetic of k_rope_kv_append), and the CTA whose
    // chunk holds the new position rotates this kv head's k, appends k and v
    // to the cache, and uses them from shared memory for that position.
    const bool fused = rfreq != nullptr;
    const int pn = fused ? rpos[r] : -1;
    const bool owner = fused && pn >= 0 && pn < L && (pn / CH) / cpc == p;
    if (fused) {
        constexpr int half = HD / 2;
        for (int i = tid; i < rep * half; i += ANT) {
            const int h = i / half, d = i % half;
            const float angle = __fdiv_rn((float)pn, rfreq[d]);
            const float c = cosf(angle), sn = sinf(angle);
            const float x0 = qr[h * HD + d], x1 = qr[h * HD + d + half];
            qs[h * KP + d] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
            qs[h * KP + d + half] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
        }
        if (owner) {
            const float *kr = q + (int64_t)r * qld + (int64_t)(n_heads + kvh) * HD;
            const float *vr = q + (int64_t)r * qld + (int64_t)(n_heads + n_kv + kvh) * HD;
            const int64_t dst = (((int64_t)cseq * max_ctx + pn) * n_kv + kvh) * HD;
            for (int d = tid; d < half; d += ANT) {
                const float angle = __fdiv_rn((float)pn, rfreq[d]);
                const float c = cosf(angle), sn = sinf(angle);
                const float x0 = kr[d], x1 = kr[d + half];
                const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
                const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
                knew[d] = y0;
                knew[d + half] = y1;
                kcw[dst + d] = y0;
                kcw[dst + d + half] = y1;
            }
            for (int d = tid; d < HD; d += ANT) {
                vnew[d] = vr[d];
                vcw[dst + d] = vr[d];
            }
        }
    } else {
        for (int i = tid; i < rep * HD; i += ANT) qs[(i / HD) * KP + i % HD] = qr[i];
    }
    if (tid < rep) {
        mrun[tid] = -INFINITY;
        lrun[tid] = 0.f;
    }
    const int npairs = rep * HD;
    const bool oth = tid < rep * DQ;   // this thread's outputs: head tid / DQ, dimensions 4 (tid % DQ) ..
    const int ph_h = oth ? tid / DQ : 0, pd0 = DV * (tid % DQ);
    float o[DV];
#pragma unroll
    for (int c = 0; c < DV; c++) o[c] = 0.f;
    const int64_t cbase = (int64_t)cseq * max_ctx;
    const int c1 = min(nchunks, (p + 1) * cpc);
    static_assert(NF4 == NLD, "one load batch per chunk");
    // Software pipeline over the CTA's chunks: chunk c + 1's K and V rows are
    // loaded into registers while chunk c is computed, so a CTA that walks
    // several chunks pays one memory latency, not one per chunk.  Only the
    // timing of the loads changes, not any arithmetic.
    float4 kr[NLD], vr[NLD];
    auto load_chunk = [&](int c) {
        const int j0 = c * CH, nj = min(CH, L - j0);
#pragma unroll
        for (int u = 0; u < NLD; u++) {
            const int i = tid + u * ANT, j = i / (HD / 4), d4 = i % (HD / 4);
            if (j < nj) {
                const int64_t g = ((cbase + j0 + j) * n_kv + kvh) * HD + 4 * d4;
                kr[u] = __ldg((const float4 *)(kc + g));
                vr[u] = __ldg((const float4 *)(vc + g));
            }
        }
    };
    if (p * cpc < c1) {
        if (EARLY && pre) {   // loaded before the dependency wait
#pragma unroll
            for (int u = 0; u < NLD; u++) {
                kr[u] = pk[EARLY ? u : 0];
                vr[u] = pv[EARLY ? u : 0];
            }
        } else {
            load_chunk(p * cpc);
        }
    }
    for (int c = p * cpc; c < c1; c++) {
        const int j0 = c * CH, nj = min(CH, L - j0);
        __syncthreads();
#pragma unroll
        for (int u = 0; u < NLD; u++) {
            const int i = tid + u * ANT, j = i / (HD / 4), d4 = i % (HD / 4);
            if (j < nj) {
                float *kd = Ks + j * KP + 4 * d4;
                kd[0] = kr[u].x; kd[1] = kr[u].y; kd[2] = kr[u].z; kd[3] = kr[u].w;
                *(float4 *)(Vs + j * HD + 4 * d4) = vr[u];
            }
        }
        if (c + 1 < c1) load_chunk(c + 1);   // in flight during this chunk's compute
        __syncthreads();
        if (owner && c == pn / CH) {  // the new position, from shared memory (not re-read from the cache)
            const int j = pn - j0;
            for (int d = tid; d < HD; d += ANT) {
                Ks[j * KP + d] = knew[d];
                Vs[j * HD + d] = vnew[d];
            }
            __syncthreads();
        }
        if (tid < rep * JS) {   // positions j0, j0 + JS, ... of head h (rows past nj: computed, not stored)
            const int h = tid / JS, j0 = tid % JS;
            const float *qh = qs + h * KP, *kj = Ks + j0 * KP;
            float sc[JB];
#pragma unroll
            for (int r = 0; r < JB; r++) sc[r] = 0.f;
#pragma unroll 8
            for (int d = 0; d < HD; d++) {
                const float qd = qh[d];
#pragma unroll
                for (int r = 0; r < JB; r++) sc[r] = fmaf(qd, kj[r * JS * KP + d], sc[r]);
            }
#pragma unroll
            for (int r = 0; r < JB; r++)
                if (j0 + r * JS < nj) S[h * CH + j0 + r * JS] = __fdiv_rn(sc[r], scale);
        }
        __syncthreads();
        for (int h = warp; h < rep; h += ANT / 32) {
            float *row = S + h * CH;
            float mc = -INFINITY;
            for (int j = lane; j < nj; j += 32) mc = fmaxf(mc, row[j]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, off));
            const float mold = mrun[h], mnew = fmaxf(mold, mc);
            float sum = 0.f;
            for (int j = lane; j < nj; j += 32) {
                const float e = expf(row[j] - mnew);
                row[j] = e;
                sum += e;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            __syncwarp();
            if (lane == 0) {
                const float a = mold == -INFINITY ? 0.f : expf(mold - mnew);
                alpha[h] = a;
                lrun[h] = lrun[h] * a + sum;
                mrun[h] = mnew;
            }
        }
        __syncthreads();
        if (oth) {
            const float *ph = S + ph_h * CH, *vd = Vs + pd0;
            const float al = alpha[ph_h];
            float ac[DV];
#pragma unroll
            for (int c = 0; c < DV; c++) ac[c] = o[c] * al;
            for (int j = 0; j < nj; j++) {
                const float pj = ph[j];
                if constexpr (DV == 4) {
                    const float4 v = *(const float4 *)(vd + j * HD);
                    ac[0] = fmaf(pj, v.x, ac[0]);
                    ac[1] = fmaf(pj, v.y, ac[1]);
                    ac[2] = fmaf(pj, v.z, ac[2]);
                    ac[3] = fmaf(pj, v.w, ac[3]);
                } else {
                    const float2 v = *(const float2 *)(vd + j * HD);
                    ac[0] = fmaf(pj, v.x, ac[0]);
                    ac[1] = fmaf(pj, v.y, ac[1]);
                }
            }
#pragma unroll
            for (int c = 0; c < DV; c++) o[c] = ac[c];
        }
    }
    __syncthreads();
    if (Pr == 1) {
        if (oth) {
#pragma unroll
            for (int c = 0; c < DV; c++)
                out[((int64_t)r * n_heads + h0 + ph_h) * HD + pd0 + c] = L > 0 ? o[c] / lrun[ph_h] : 0.f;
        }
        return;
    }
    // Split row: publish (max, sum, output) and let the last CTA combine.
    const int W = HD + 2;
    float *part = ws + (((int64_t)r * n_kv + kvh) * P) * rep * W;
    if (oth) {
#pragma unroll
        for (int c = 0; c < DV; c++) __stcg(part + (int64_t)p * rep * W + ph_h * W + pd0 + c, o[c]);
    }
    if (tid < rep) {
        __stcg(part + (int64_t)p * rep * W + tid * W + HD, mrun[tid]);
        __stcg(part + (int64_t)p * rep * W + tid * W + HD + 1, lrun[tid]);
    }
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (tid == 0) last = (atomicAdd(tickets + r * n_kv + kvh, 1) == Pr - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int i = tid; i < npairs; i += ANT) {
        const int h = i / HD, d = i % HD;
        float M = -INFINITY;
#pragma unroll 8
        for (int pp = 0; pp < Pr; pp++) M = fmaxf(M, __ldcg(part + (int64_t)pp * rep * W + h * W + HD));
        float O = 0.f, Ls = 0.f;
#pragma unroll 8
        for (int pp = 0; pp < Pr; pp++) {
            const float *pt = part + (int64_t)pp * rep * W + h * W;
            const float e = expf(__ldcg(pt + HD) - M);
            O = fmaf(__ldcg(pt + d), e, O);
            Ls = fmaf(__ldcg(pt + HD + 1), e, Ls);
        }
        out[((int64_t)r * n_heads + h0 + h) * HD + d] = O / Ls;
    }
    if (tid == 0) tickets[r * n_kv + kvh] = 0;
}

template <int HD>
size_t attn_smem(int rep) {
    return (size_t)(((rep * (HD + 1) + CH * (HD + 1) + 3) & ~3) + CH * HD + rep * CH + 3 * MAXREP + 2 * HD) *
           sizeof(float);
}

template <int HD, bool EARLY>
cudaError_t launch_attn_t(hd_ctx *ctx, int rows, int n_heads, int n_kv, int P, int cpc, const float *q, int64_t qld,
                          const float *kc, const float *vc, const int32_t *lens, int pos0, int seqT, int max_ctx,
                          const int32_t *slots, const float *rfreq, const int32_t *rpos, float *out) {
    const int rep = n_heads / n_kv;
    const size_t smem = attn_smem<HD>(rep);
    if (smem > 48 * 1024) {
        cudaError_t e =
            cudaFuncSetAttribute(k_attention<HD, EARLY>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    const float scale = sqrtf((float)HD);
    return hd_launch(ctx, k_attention<HD, EARLY>, dim3(rows, n_kv, P), dim3(ANT), smem, q, qld, kc, vc, lens, pos0,
                     seqT, n_heads, n_kv, max_ctx, scale, P, cpc, (float *)ctx->ws, ctx->tickets, slots, rfreq, rpos,
                     (float *)kc, (float *)vc, out);
}

template <int HD>
cudaError_t launch_attn(hd_ctx *ctx, int rows, int n_heads, int n_kv, int P, int cpc, const float *q, int64_t qld,
                        const float *kc, const float *vc, const int32_t *lens, int pos0, int seqT, int max_ctx,
                        const int32_t *slots, const float *rfreq, const int32_t *rpos, float *out, bool early) {
    return early ? launch_attn_t<HD, true>(ctx, rows, n_heads, n_kv, P, cpc, q, qld, kc, vc, lens, pos0, seqT, max_ctx,
                                           slots, rfreq, rpos, out)
                 : launch_attn_t<HD, false>(ctx, rows, n_heads, n_kv, P, cpc, q, qld, kc, vc, lens, pos0, seqT,
                                            max_ctx, slots, rfreq, rpos, out);
}

}  // namespace

int hd_attention_run(hd_ctx *ctx, const float *q, int64_t qld, const float *kc, const float *vc, const int32_t *lens,
                     int rows, int pos0, int seqT, int n_heads, int n_kv, int hd, int max_ctx, int maxlen, float *out,
                     const char *name, const int32_t *slots, const float *rope_freq, const int32_t *rope_pos,
                     bool early_kv) {
    if (!ctx || !q || !kc || !vc || !out) return hd_fail(ctx, HD_E_ARG, "%s: null argument", name);
    HD_REQUIRE(ctx, n_heads > 0 && n_kv > 0 && n_heads % n_kv == 0 && n_heads / n_kv <= MAXREP, HD_E_SHAPE,
               "%s: n_heads %d must be a multiple of n_kv %d, at most %d per kv head", name, n_heads, n_kv, MAXREP);
    HD_REQUIRE(ctx, max_ctx > 0 && maxlen <= max_ctx, HD_E_SHAPE, "%s: length beyond max_ctx", name);
    HD_REQUIRE(ctx, hd == 32 || hd == 64 || hd == 128, HD_E_UNSUPPORTED, "%s: head_dim %d (32, 64 or 128)", name, hd);
    if (rows == 0) return HD_OK;
    // Decode: split positions so that about two CTAs per SM are busy.
    const int maxchunks = (maxlen + CH - 1) / CH > 0 ? (maxlen + CH - 1) / CH : 1;
    int P = 1;
    if (lens) {
        const int64_t ctas = (int64_t)rows * n_kv;
        const int64_t want = (2 * (int64_t)ctx->sm_count + ctas - 1) / ctas;
        P = (int)(want < maxchunks ? want : maxchunks);
        if (P < 1) P = 1;
    }
    const int cpc = (maxchunks + P - 1) / P;
    P = (maxchunks + cpc - 1) / cpc;
    HD_REQUIRE(ctx, P <= 65535, HD_E_SHAPE, "%s: too many position splits", name);
    if (P > 1) {
        const size_t need = (size_t)rows * n_kv * P * (n_heads / n_kv) * (hd + 2) * sizeof(float);
        int rc = hd_ensure_workspace(ctx, need, (size_t)rows * n_kv);
        if (rc) return rc;
    }
    // The early K/V loads pay off when the CTAs fit in about one wave (a few
    // sequences); with many sequences their registers cost more than the
    // overlap gives (256 sequences: 6.6 -> 6.8 ms per step).
    early_kv = early_kv && (int64_t)rows * n_kv * P <= 2 * (int64_t)ctx->sm_count;
    cudaError_t e;
    if (qld == 0) qld = (int64_t)n_heads * hd;
    if (hd == 64) e = launch_attn<64>(ctx, rows, n_heads, n_kv, P, cpc, q, qld, kc, vc, lens, pos0, seqT, max_ctx, slots, rope_freq, rope_pos, out, early_kv);
    else if (hd == 128)
        e = launch_attn<128>(ctx, rows, n_heads, n_kv, P, cpc, q, qld, kc, vc, lens, pos0, seqT, max_ctx, slots, rope_freq, rope_pos, out, early_kv);
    else e = launch_attn<32>(ctx, rows, n_heads, n_kv, P, cpc, q, qld, kc, vc, lens, pos0, seqT, max_ctx, slots, rope_freq, rope_pos, out, early_kv);
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "%s: %s", name, cudaGetErrorString(e));
    return HD_OK;
}

int hd_rope_kv_append(hd_ctx *ctx, float *qkv, int64_t ld, const int32_t *pos, int rows, int T, int n_heads, int n_kv,
                      int hd, float *kc, float *vc, int max_ctx) {
    const int64_t n = (int64_t)rows * ((int64_t)(n_heads + n_kv) * (hd / 2) + (int64_t)n_kv * hd);
    if (n == 0) return HD_OK;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_rope_kv_append, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, qkv, ld, pos,
                               (const float *)ctx->rope_freq, rows, T, n_heads, n_kv, hd, kc, vc, max_ctx));
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
    return hd_attention_run(ctx, q, 0, kc, vc, len, seqs, 0, 1, n_heads, n_kv, head_dim, max_ctx, max_ctx, out,
                            "hd_attention_decode");
}

extern "C" int hd_attention_prefill(hd_ctx *ctx, const float *q, const float *kc, const float *vc, int T, int pos0,
                                    int n_heads, int n_kv, int head_dim, int max_ctx, float *out) {
    if (T < 0 || pos0 < 0) return hd_fail(ctx, HD_E_ARG, "hd_attention_prefill: negative size");
    return hd_attention_run(ctx, q, 0, kc, vc, nullptr, T, pos0, T > 0 ? T : 1, n_heads, n_kv, head_dim, max_ctx,
                            pos0 + T, out, "hd_attention_prefill");
}
