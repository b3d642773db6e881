// hd_gemv.cu -- decode Q-GEMV: y[b] = W x[b] (+bias, +residual, or SwiGLU of
// a gate/up pair) for b < B <= 16, fp32 accumulation, weights unpacked in
// registers straight from the unit-major layout.
//
// Work split.  A CTA owns RC consecutive output rows over the whole of K (or
// over one of S slices of K when K is very long for few rows).  Its NT = RC*G
// threads form G groups: thread t owns row t % RC and the units
// t / RC, t / RC + G, ...; lanes on consecutive rows read one unit of
// consecutive rows as one contiguous span of the unit-major layout.  RC is
// about rows / SMs, so there is roughly one CTA per SM and every CTA streams
// its whole slice of W with all of its loads in flight at once.
//
// Reduction.  Per-row partial sums meet in shared memory and are added in a
// fixed order (group 0, 1, ..., G-1), so results are bitwise reproducible.
// With S > 1 the CTAs of a row tile publish partials to the workspace and the
// last to arrive (atomic ticket) adds them in split order and resets the
// ticket.
//
// x.  Activations are read from global memory through L1 after the
// dependency wait; lanes that share a unit read the same addresses (a
// broadcast).  Q4_K's per-unit sums of x, needed for its min term, are
// computed once per CTA into shared memory.
//
// Overlap.  The first chunk of each thread's weight loads is issued before
// griddepcontrol.wait: under programmatic dependent launch those loads run
// while the previous kernel in the stream is still finishing.  Nothing the
// previous kernel writes is read or written before the wait.
//
// Unpacking.  Bytes become floats exactly via byte_perm into 0x4B0000bb
// (= 2^23 + byte) and one subtraction of 2^23 + offset; Q5_0's fifth bit and
// Q6_K's two high bits are merged into the bytes by one shift and one mask
// thanks to the re-ordering done at upload (hd_internal.cuh).
#include "hd_internal.cuh"

namespace {

constexpr int UC = 4;  // units per thread per register chunk

struct GemvArgs {
    WView w0, w1;          // w1: the up weight of a SwiGLU pair
    const float *x;        // [B][K]
    float *y;              // [B][ldy]
    const float *bias;     // [N] or null
    const float *residual; // [B][ldy] or null
    float *ws;             // split-K partials [S][NB][Neff]
    int *tickets;          // [tiles]
    int B, N, ldy, K;
    int RC, G;             // rows per CTA, unit groups per CTA
    int U, S;              // units per split, splits
    int pair;              // 1: SwiGLU of (w0, w1)
};
template <int TYPE>
struct URegs;
template <>
struct URegs<HD_TYPE_Q8_0> { uint4 a, b; uint32_t d; };
template <>
struct URegs<HD_TYPE_Q5_0> { uint4 a; uint32_t qh, d; };
template <>
struct URegs<HD_TYPE_Q4_K> { uint4 a, m; };
template <>
struct URegs<HD_TYPE_Q6_K> { uint4 a, sc; uint2 h; uint32_t d; };

template <int TYPE>
__device__ __forceinline__ void load_unit(const WView &w, int64_t r, int u, URegs<TYPE> &g) {
    const int64_t ur = (int64_t)u * w.rows + r;
    if constexpr (TYPE == HD_TYPE_Q8_0) {
        const uint4 *p = (const uint4 *)(w.q + ur * 32);
        g.a = __ldg(p);
        g.b = __ldg(p + 1);
        g.d = __ldg((const unsigned short *)w.meta + ur);
    } else if constexpr (TYPE == HD_TYPE_Q5_0) {
        g.a = __ldg((const uint4 *)(w.q + ur * 16));
        g.qh = __ldg((const unsigned int *)w.aux + ur);
        g.d = __ldg((const unsigned short *)w.meta + ur);
    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
        g.a = __ldg((const uint4 *)(w.q + ur * 16));
        g.m = __ldg((const uint4 *)(w.meta + ((int64_t)(u >> 3) * w.rows + r) * 16));
    } else {
        const int64_t sr = (int64_t)(u >> 3) * w.rows + r;
        g.a = __ldg((const uint4 *)(w.q + ur * 16));
        g.h = __ldg((const uint2 *)w.aux + ur);
        g.sc = __ldg((const uint4 *)(w.meta + sr * 16));
        g.d = __ldg(w.dsb + sr);
    }
}

template <int TYPE>
__device__ __forceinline__ void zero_unit(URegs<TYPE> &g) {
    if constexpr (TYPE == HD_TYPE_Q8_0) {
        g.a = g.b = make_uint4(0, 0, 0, 0);
        g.d = 0;
    } else if constexpr (TYPE == HD_TYPE_Q5_0) {
        g.a = make_uint4(0, 0, 0, 0);
        g.qh = 0;
        g.d = 0;
    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
        g.a = g.m = make_uint4(0, 0, 0, 0);
    } else {
        g.a = g.sc = make_uint4(0, 0, 0, 0);
        g.h = make_uint2(0, 0);
        g.d = 0;
    }
}

__device__ __forceinline__ uint32_t w4(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ uint32_t shl_or_shr(uint32_t v, int s) { return s >= 0 ? (v << s) : (v >> -s); }

__device__ __forceinline__ float dot4(float a0, float a1, float a2, float a3, const float4 &x, float s) {
    s = fmaf(a0, x.x, s);
    s = fmaf(a1, x.y, s);
    s = fmaf(a2, x.z, s);
    return fmaf(a3, x.w, s);
}

// acc[b] += unit(u) . x[b][unit]; xs points at this unit's 32 floats of batch
// row 0, batch rows `xstride4` float4s apart.
template <int TYPE, int NB>
__device__ __forceinline__ void unit_fma(const URegs<TYPE> &g, int u, const float4 *xs, int xstride4,
                                         const float *xsum, int xsum_stride, float (&acc)[NB]) {
    if constexpr (TYPE == HD_TYPE_Q8_0) {
        float s[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) s[b] = 0.f;
#pragma unroll
        for (int wd = 0; wd < 8; wd++) {
            uint32_t v = (wd < 4 ? w4(g.a, wd) : w4(g.b, wd - 4)) ^ 0x80808080u;
            const float o = 8388736.0f;  // 2^23 + 128
            float f0 = mag(v, 0) - o, f1 = mag(v, 1) - o, f2 = mag(v, 2) - o, f3 = mag(v, 3) - o;
#pragma unroll
            for (int b = 0; b < NB; b++) s[b] = dot4(f0, f1, f2, f3, xs[b * xstride4 + wd], s[b]);
        }
        float d = h2f((uint16_t)g.d);
#pragma unroll
        for (int b = 0; b < NB; b++) acc[b] = fmaf(d, s[b], acc[b]);
    } else if constexpr (TYPE == HD_TYPE_Q5_0) {
        float s[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) s[b] = 0.f;
#pragma unroll
        for (int wd = 0; wd < 4; wd++) {
            uint32_t v = w4(g.a, wd);
            uint32_t lo = (v & 0x0F0F0F0Fu) | ((g.qh >> wd) & 0x10101010u);
            uint32_t hi = ((v >> 4) & 0x0F0F0F0Fu) | ((g.qh << (4 - wd)) & 0x10101010u);
            const float o = 8388624.0f;  // 2^23 + 16
            float l0 = mag(lo, 0) - o, l1 = mag(lo, 1) - o, l2 = mag(lo, 2) - o, l3 = mag(lo, 3) - o;
            float h0 = mag(hi, 0) - o, h1 = mag(hi, 1) - o, h2 = mag(hi, 2) - o, h3 = mag(hi, 3) - o;
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float t = dot4(l0, l1, l2, l3, xs[b * xstride4 + wd], s[b]);
                s[b] = dot4(h0, h1, h2, h3, xs[b * xstride4 + 4 + wd], t);
            }
        }
        float d = h2f((uint16_t)g.d);
#pragma unroll
        for (int b = 0; b < NB; b++) acc[b] = fmaf(d, s[b], acc[b]);
    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
        float s[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) s[b] = 0.f;
#pragma unroll
        for (int wd = 0; wd < 4; wd++) {
            uint32_t v = w4(g.a, wd);
            uint32_t lo = v & 0x0F0F0F0Fu, hi = (v >> 4) & 0x0F0F0F0Fu;
            const float o = 8388608.0f;  // 2^23
            float l0 = mag(lo, 0) - o, l1 = mag(lo, 1) - o, l2 = mag(lo, 2) - o, l3 = mag(lo, 3) - o;
            float h0 = mag(hi, 0) - o, h1 = mag(hi, 1) - o, h2 = mag(hi, 2) - o, h3 = mag(hi, 3) - o;
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float t = dot4(l0, l1, l2, l3, xs[b * xstride4 + wd], s[b]);
                s[b] = dot4(h0, h1, h2, h3, xs[b * xstride4 + 4 + wd], t);
            }
        }
        int sc, m;
        q4k_sm_regs(u & 7, g.m.y, g.m.z, g.m.w, sc, m);
        float d = h2f((uint16_t)(g.m.x & 0xFFFF)), dmin = h2f((uint16_t)(g.m.x >> 16));
        float d1 = d * (float)sc, m1 = dmin * (float)m;
#pragma unroll
        for (int b = 0; b < NB; b++) acc[b] = fmaf(d1, s[b], fmaf(-m1, xsum[b * xsum_stride], acc[b]));
    } else {  // Q6_K
        float sl[NB], sh[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) sl[b] = sh[b] = 0.f;
#pragma unroll
        for (int wd = 0; wd < 4; wd++) {
            uint32_t v = w4(g.a, wd);
            uint32_t lo = (v & 0x0F0F0F0Fu) | (shl_or_shr(g.h.x, 4 - 2 * wd) & 0x30303030u);
            uint32_t hi = ((v >> 4) & 0x0F0F0F0Fu) | (shl_or_shr(g.h.y, 4 - 2 * wd) & 0x30303030u);
            const float o = 8388640.0f;  // 2^23 + 32
            float l0 = mag(lo, 0) - o, l1 = mag(lo, 1) - o, l2 = mag(lo, 2) - o, l3 = mag(lo, 3) - o;
            float h0 = mag(hi, 0) - o, h1 = mag(hi, 1) - o, h2 = mag(hi, 2) - o, h3 = mag(hi, 3) - o;
#pragma unroll
            for (int b = 0; b < NB; b++) {
                sl[b] = dot4(l0, l1, l2, l3, xs[b * xstride4 + wd], sl[b]);
                sh[b] = dot4(h0, h1, h2, h3, xs[b * xstride4 + 4 + wd], sh[b]);
            }
        }
        int s0 = 2 * (u & 7);
        uint32_t scw = w4(g.sc, s0 >> 2);
        int8_t c0 = (int8_t)((scw >> (8 * (s0 & 3))) & 255), c1 = (int8_t)((scw >> (8 * ((s0 & 3) + 1))) & 255);
        float d = h2f((uint16_t)g.d);
        float dl = d * (float)c0, dh = d * (float)c1;
#pragma unroll
        for (int b = 0; b < NB; b++) acc[b] = fmaf(dl, sl[b], fmaf(dh, sh[b], acc[b]));
    }
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

template <int TYPE, int NB, int P>
__global__ void __launch_bounds__(256) k_qgemv(GemvArgs a) {
    extern __shared__ float sm[];
    const int t = threadIdx.x, NT = blockDim.x;
    const int RC = a.RC, G = a.G;
    const int tile = blockIdx.x, split = blockIdx.y;
    const int r = t % RC, g = t / RC;
    const int64_t row = (int64_t)tile * RC + r;
    const bool ok = row < a.N && g < G;
    const int u0 = split * a.U;
    const int u1 = min(a.w0.units, u0 + a.U);
    const WView wa = a.w0, wb = a.w1;

    URegs<TYPE> cur[UC][P + 1];
#pragma unroll
    for (int c = 0; c < UC; c++) {
        const int u = u0 + g + c * G;
#pragma unroll
        for (int p = 0; p <= P; p++) {
            if (ok && u < u1) load_unit<TYPE>(p ? wb : wa, row, u, cur[c][p]);
            else zero_unit<TYPE>(cur[c][p]);
        }
    }
    pdl_trigger();
    pdl_wait();

    // Q4_K: sum of x over every unit of this CTA's K range, per batch row.
    float *xsum = sm;                         // [NB][U]
    float *red = sm + (TYPE == HD_TYPE_Q4_K ? NB * a.U : 0);  // [NT][P+1][NB]
    if constexpr (TYPE == HD_TYPE_Q4_K) {
        const int nu = u1 - u0;
        for (int i = t; i < NB * nu; i += NT) {
            const int b = i / nu, ul = i % nu;
            float s = 0.f;
            if (b < a.B) {
                const float4 *p = (const float4 *)(a.x + (int64_t)b * a.K + (int64_t)(u0 + ul) * 32);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    float4 v = p[j];
                    s += (v.x + v.y) + (v.z + v.w);
                }
            }
            xsum[b * a.U + ul] = s;
        }
        __syncthreads();
    }

    float acc[P + 1][NB];
#pragma unroll
    for (int p = 0; p <= P; p++)
#pragma unroll
        for (int b = 0; b < NB; b++) acc[p][b] = 0.f;

    const int xs4 = a.K / 4;  // float4 per batch row of x
    for (int base = u0 + g; base < u1; base += UC * G) {
        if (base != u0 + g) {
#pragma unroll
            for (int c = 0; c < UC; c++) {
                const int u = base + c * G;
#pragma unroll
                for (int p = 0; p <= P; p++) {
                    if (ok && u < u1) load_unit<TYPE>(p ? wb : wa, row, u, cur[c][p]);
                    else zero_unit<TYPE>(cur[c][p]);
                }
            }
        }
#pragma unroll
        for (int c = 0; c < UC; c++) {
            const int u = base + c * G;
            if (ok && u < u1) {
                const float4 *xp = (const float4 *)(a.x + (int64_t)u * 32);
#pragma unroll
                for (int p = 0; p <= P; p++)
                    unit_fma<TYPE, NB>(cur[c][p], u, xp, xs4, xsum + (u - u0), a.U, acc[p]);
            }
        }
    }

    // Per-row sums over the G groups, in group order.
#pragma unroll
    for (int p = 0; p <= P; p++)
#pragma unroll
        for (int b = 0; b < NB; b++) red[(t * (P + 1) + p) * NB + b] = acc[p][b];
    __syncthreads();

    const int64_t neff = P ? 2 * (int64_t)a.N : (int64_t)a.N;
    auto epilogue = [&](int64_t rw, int b, float v, float vu) {
        if (P) {
            a.y[(int64_t)b * a.ldy + rw] = silu_mul(v, vu);
        } else {
            if (a.bias) v = v + a.bias[rw];
            if (a.residual) v = a.residual[(int64_t)b * a.ldy + rw] + v;
            a.y[(int64_t)b * a.ldy + rw] = v;
        }
    };
    const int nout = RC * a.B;
    if (a.S == 1) {
        for (int j = t; j < nout; j += NT) {
            const int rr = j % RC, b = j / RC;
            const int64_t rw = (int64_t)tile * RC + rr;
            if (rw >= a.N) continue;
            float v[P + 1];
#pragma unroll
            for (int p = 0; p <= P; p++) {
                float s = 0.f;
                for (int gg = 0; gg < G; gg++) s += red[((gg * RC + rr) * (P + 1) + p) * NB + b];
                v[p] = s;
            }
            epilogue(rw, b, v[0], v[P]);
        }
        return;
    }

    // Split-K: publish this CTA's row sums, the last CTA of the tile reduces.
    for (int j = t; j < nout; j += NT) {
        const int rr = j % RC, b = j / RC;
        const int64_t rw = (int64_t)tile * RC + rr;
        if (rw >= a.N) continue;
#pragma unroll
        for (int p = 0; p <= P; p++) {
            float s = 0.f;
            for (int gg = 0; gg < G; gg++) s += red[((gg * RC + rr) * (P + 1) + p) * NB + b];
            __stcg(a.ws + ((int64_t)split * NB + b) * neff + (p ? a.N + rw : rw), s);
        }
    }
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (t == 0) last = (atomicAdd(a.tickets + tile, 1) == a.S - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int j = t; j < nout; j += NT) {
        const int rr = j % RC, b = j / RC;
        const int64_t rw = (int64_t)tile * RC + rr;
        if (rw >= a.N) continue;
        float v[P + 1];
#pragma unroll
        for (int p = 0; p <= P; p++) {
            float s = 0.f;
            for (int sp = 0; sp < a.S; sp++) s += __ldcg(a.ws + ((int64_t)sp * NB + b) * neff + (p ? a.N + rw : rw));
            v[p] = s;
        }
        epilogue(rw, b, v[0], v[P]);
    }
    if (t == 0) a.tickets[tile] = 0;
}

struct Plan {
    int nb, RC, G, nt, U, S, tiles;
    size_t smem;
};

int pad_batch(int B) { return B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : B <= 8 ? 8 : 16; }

// RC ~ rows / SMs (one CTA per SM), G groups of RC threads (NT <= 256, no more
// groups than units).  Split K only when the row tiles alone leave most SMs
// idle and every split still gives each group a unit or more.
Plan plan_gemv(int N, int units, int B, bool pair, int sms) {
    Plan p;
    p.nb = pad_batch(B);
    int RC = (N + sms - 1) / sms;
    RC = RC < 1 ? 1 : RC > 32 ? 32 : RC;
    int G = 256 / RC;
    if (G > units) G = units;
    p.RC = RC;
    p.G = G;
    p.nt = RC * G;
    p.tiles = (N + RC - 1) / RC;
    int S = 1;
    if (p.tiles * 2 < sms && units >= 2 * G) {
        S = (sms + p.tiles - 1) / p.tiles;
        if (S > units / G) S = units / G;
        if (S < 1) S = 1;
    }
    p.U = (units + S - 1) / S;
    p.S = (units + p.U - 1) / p.U;
    const int P1 = pair ? 2 : 1;
    p.smem = (size_t)p.nt * P1 * p.nb * sizeof(float) + (size_t)p.nb * p.U * sizeof(float);
    return p;
}

template <int TYPE, int NB, int P>
cudaError_t launch_inst(hd_ctx *ctx, const Plan &p, const GemvArgs &a) {
    if (p.smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_qgemv<TYPE, NB, P>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)p.smem);
        if (e != cudaSuccess) return e;
    }
    return hd_launch(ctx, k_qgemv<TYPE, NB, P>, dim3(p.tiles, p.S), dim3(p.nt), p.smem, a);
}

template <int TYPE>
cudaError_t launch_type(hd_ctx *ctx, const Plan &p, const GemvArgs &a) {
    const bool pr = a.pair != 0;
    switch (p.nb) {
    case 1: return pr ? launch_inst<TYPE, 1, 1>(ctx, p, a) : launch_inst<TYPE, 1, 0>(ctx, p, a);
    case 2: return pr ? launch_inst<TYPE, 2, 1>(ctx, p, a) : launch_inst<TYPE, 2, 0>(ctx, p, a);
    case 4: return pr ? launch_inst<TYPE, 4, 1>(ctx, p, a) : launch_inst<TYPE, 4, 0>(ctx, p, a);
    case 8: return launch_inst<TYPE, 8, 0>(ctx, p, a);
    default: return launch_inst<TYPE, 16, 0>(ctx, p, a);
    }
}

}  // namespace
int hd_ensure_hbuf(hd_ctx *ctx, float **buf, size_t *have, size_t need);
namespace {

int run_gemv(hd_ctx *ctx, const hd_weight *w, const hd_weight *w_up, const float *x, float *y, int B,
             const float *bias, const float *residual, const char *name) {
    if (!ctx || !w || !x || !y) return hd_fail(ctx, HD_E_ARG, "%s: null argument", name);
    HD_REQUIRE(ctx, B >= 1 && B <= 16, HD_E_ARG, "%s: batch %d outside 1..16", name, B);
    HD_REQUIRE(ctx, ((uintptr_t)x & 15) == 0, HD_E_ARG, "%s: x must be 16-byte aligned", name);
    if (w_up)
        HD_REQUIRE(ctx, w_up->type == w->type && w_up->rows == w->rows && w_up->cols == w->cols, HD_E_SHAPE,
                   "%s: gate and up weights differ in type or shape", name);
    if (w_up && pad_batch(B) >= 8) {
        // Two plain GEMVs into scratch, then the elementwise SwiGLU (the fused
        // pair would hold 2 x 16 accumulators per thread at this batch).
        size_t one = (size_t)B * w->rows;
        int rc = hd_ensure_hbuf(ctx, &ctx->scratch, &ctx->scratch_bytes, 2 * one * sizeof(float));
        if (!rc) rc = run_gemv(ctx, w, nullptr, x, ctx->scratch, B, nullptr, nullptr, name);
        if (!rc) rc = run_gemv(ctx, w_up, nullptr, x, ctx->scratch + one, B, nullptr, nullptr, name);
        if (!rc) rc = hd_swiglu(ctx, ctx->scratch, ctx->scratch + one, y, (int64_t)one);
        return rc;
    }
    Plan p = plan_gemv((int)w->rows, w->units, B, w_up != nullptr, ctx->sm_count);
    if (p.S > 1) {
        size_t neff = (size_t)w->rows * (w_up ? 2 : 1);
        int rc = hd_ensure_workspace(ctx, (size_t)p.S * p.nb * neff * sizeof(float), (size_t)p.tiles);
        if (rc) return rc;
    }
    GemvArgs a;
    a.w0 = wview(w);
    a.w1 = w_up ? wview(w_up) : a.w0;
    a.x = x;
    a.y = y;
    a.bias = bias;
    a.residual = residual;
    a.ws = (float *)ctx->ws;
    a.tickets = ctx->tickets;
    a.B = B;
    a.N = (int)w->rows;
    a.ldy = (int)w->rows;
    a.K = (int)w->cols;
    a.RC = p.RC;
    a.G = p.G;
    a.U = p.U;
    a.S = p.S;
    a.pair = w_up ? 1 : 0;
    cudaError_t e = cudaSuccess;
    HD_TYPE_SWITCH(w->type, T, e = launch_type<T>(ctx, p, a));
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "%s: %s", name, cudaGetErrorString(e));
    return HD_OK;
}

}  // namespace

extern "C" int hd_qgemv(hd_ctx *ctx, const hd_weight *w, const float *x_dev, float *y_dev, int B,
                        const float *bias_dev, const float *residual_dev) {
    return run_gemv(ctx, w, nullptr, x_dev, y_dev, B, bias_dev, residual_dev, "hd_qgemv");
}

extern "C" int hd_qgemv_swiglu(hd_ctx *ctx, const hd_weight *w_gate, const hd_weight *w_up, const float *x_dev,
                               float *y_dev, int B) {
    if (!w_up) return hd_fail(ctx, HD_E_ARG, "hd_qgemv_swiglu: null up weight");
    return run_gemv(ctx, w_gate, w_up, x_dev, y_dev, B, nullptr, nullptr, "hd_qgemv_swiglu");
}

int hd_ensure_hbuf(hd_ctx *ctx, float **buf, size_t *have, size_t need) {
    if (need <= *have) return HD_OK;
    HD_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    cudaFree(*buf);
    *buf = nullptr;
    *have = 0;
    HD_CUDA_TRY(ctx, cudaMalloc(buf, need));
    *have = need;
    return HD_OK;
}

extern "C" int hd_qgemv_host(hd_ctx *ctx, const hd_weight *w, const float *x_host, float *y_host, int B) {
    if (!ctx || !w || !x_host || !y_host) return hd_fail(ctx, HD_E_ARG, "hd_qgemv_host: null argument");
    HD_REQUIRE(ctx, B >= 1 && B <= 16, HD_E_ARG, "hd_qgemv_host: batch %d outside 1..16", B);
    size_t xb = (size_t)B * w->cols * sizeof(float), yb = (size_t)B * w->rows * sizeof(float);
    int rc = hd_ensure_hbuf(ctx, &ctx->hbuf_x, &ctx->hbuf_x_bytes, xb);
    if (!rc) rc = hd_ensure_hbuf(ctx, &ctx->hbuf_y, &ctx->hbuf_y_bytes, yb);
    if (rc) return rc;
    HD_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->hbuf_x, x_host, xb, cudaMemcpyHostToDevice, ctx->stream));
    rc = hd_qgemv(ctx, w, ctx->hbuf_x, ctx->hbuf_y, B, nullptr, nullptr);
    if (rc) return rc;
    HD_CUDA_TRY(ctx, cudaMemcpyAsync(y_host, ctx->hbuf_y, yb, cudaMemcpyDeviceToHost, ctx->stream));
    HD_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return HD_OK;
}
