// hd_gemv.cu -- decode Q-GEMV: y[b] = W x[b] (+bias, +residual, or SwiGLU of
// a gate/up pair) for b < B <= 16, fp32 accumulation, weights unpacked in
// registers straight from the unit-major layout.
//
// Work split.  A CTA owns RC consecutive output rows over the whole of K.
// Its NT = RC*G threads form G groups: thread t owns row t % RC and the units
// t / RC, t / RC + G, ...; lanes on consecutive rows read one unit of
// consecutive rows as one contiguous span of the unit-major layout.  RC is
// about rows / SMs but small enough that each thread holds about one unit, so
// an SM runs ~28 warps (up to 1024 threads per CTA at batch <= 2) and all of
// its weight loads are in flight at once.
//
// Reduction.  Per-row partial sums meet in shared memory and are added in a
// fixed order (groups of 16, then the group sums), so results are bitwise
// reproducible.
//
// x.  Activations are read from global memory through L1 after the
// dependency wait; lanes that share a unit read the same addresses (a
// broadcast).  Sums of x over each half unit, which carry the quant offsets
// (see unit_fma), are computed once per CTA into shared memory.
//
// Overlap.  The first chunk of each thread's weight loads is issued before
// griddepcontrol.wait: under programmatic dependent launch those loads run
// while the previous kernel in the stream is still finishing.  Nothing the
// previous kernel writes is read or written before the wait.
//
// Unpacking.  One byte_perm turns a quant byte into the float 2 + q/64
// exactly; Q5_0's fifth bit and Q6_K's two high bits are merged into the bytes
// by one shift and one mask thanks to the re-ordering done at upload
// (hd_internal.cuh).
#include <cstdlib>

#include "hd_internal.cuh"
#include "hd_units.cuh"

namespace {


struct GemvArgs {
    WView w0, w1;          // w1: the up weight of a SwiGLU pair
    const float *x;        // [B][K]
    float *y;              // [B][ldy]
    const float *bias;     // [N] or null
    const float *residual; // [B][ldy] or null
    int B, N, ldy, K;
    int RC, G;             // rows per CTA, unit groups per CTA
    int pair;              // 1: SwiGLU of (w0, w1)
    const float *nw;       // [K] RMSNorm weight: x is normalized first (null: x as is)
    float eps;
    int32_t *amax;         // [B] greedy id of each output row (null: none)
    unsigned long long *keys;  // [16] argmax keys + [1] CTA counter (zero between launches)
};

// Argmax key of (value v, index i): larger keys win, so the float's order
// goes to the high word (sign-magnitude flipped to unsigned order; -0 counts
// as +0 and NaN as the lowest key, so NaN never wins) and the complement of
// the index to the low word (a tie goes to the lower index) -- the order of
// ArgMaxSampler::sample's strict > scan (runtime/sampler/argmax.rs:8-24).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t i) {
    if (v != v) return 0ull;
    uint32_t b = v == 0.f ? 0u : __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (0xFFFFFFFFu - i);
}

// RMSNorm scales of B rows of x [B][K] (1 / sqrt(mean(x^2) + eps)) into
// rs[b], by the whole CTA in a fixed order: per-thread strided sums, warp
// shuffles, warp partials added in warp order.  nred: NWARPS_MAX x NB floats.
// The CTA is whole warps (the launchers round block sizes up to 32).
template <int NB>
__device__ __forceinline__ void norm_scales(const float *__restrict__ x, int K, int B, float eps, float *nred,
                                            float *rs) {
    float ss[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) ss[b] = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
#pragma unroll
        for (int b = 0; b < NB; b++)
            if (b < B) {
                const float v = x[(int64_t)b * K + k];
                ss[b] = fmaf(v, v, ss[b]);
            }
    }
#pragma unroll
    for (int b = 0; b < NB; b++)
        for (int o = 16; o > 0; o >>= 1) ss[b] += __shfl_xor_sync(0xffffffffu, ss[b], o);
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0)
#pragma unroll
        for (int b = 0; b < NB; b++) nred[warp * NB + b] = ss[b];
    __syncthreads();
    if ((int)threadIdx.x < B) {
        float t = 0.f;
        for (int w = 0; w < nw; w++) t += nred[w * NB + threadIdx.x];
        rs[threadIdx.x] = 1.0f / sqrtf(t / (float)K + eps);
    }
    __syncthreads();
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// Threads per CTA and units per register chunk for a padded batch NB; a
// SwiGLU pair (P = 1) holds two weights' registers, so half the threads.
template <int NB, int P>
struct GemvShape {
    static constexpr int MAXT = (NB <= 2 ? 1024 : NB <= 4 ? 512 : 256) >> P;
    static constexpr int UCT = NB <= 2 ? 2 : 4;
};

template <int TYPE, int NB, int P>
__global__ void __launch_bounds__(GemvShape<NB, P>::MAXT) k_qgemv(GemvArgs a) {
    constexpr int UCT = GemvShape<NB, P>::UCT;
    extern __shared__ float sm[];
    const int t = threadIdx.x, NT = blockDim.x;
    const int RC = a.RC, G = a.G;
    const int tile = blockIdx.x;
    const int r = t % RC, g = t / RC;
    const int64_t row = (int64_t)tile * RC + r;
    const bool ok = row < a.N && g < G;
    const int u0 = 0, u1 = a.w0.units, nu = u1 - u0;
    const WView wa = a.w0, wb = a.w1;

    URegs<TYPE> cur[UCT][P + 1];
#pragma unroll
    for (int c = 0; c < UCT; c++) {
        const int u = u0 + g + c * G;
#pragma unroll
        for (int p = 0; p <= P; p++) {
            if (ok && u < u1) load_unit<TYPE>(p ? wb : wa, row, u, cur[c][p]);
            else zero_unit<TYPE>(cur[c][p]);
        }
    }
    pdl_trigger();
    pdl_wait();
    __shared__ unsigned long long skey[16];  // argmax: the CTA's best key per batch row
    __shared__ int slast;
    if (P == 0 && a.amax && t < 16) skey[t] = 0ull;

    // Sums of x over each 16-value half unit, per batch row: [NB][nu][2].
    float *xh = sm;
    float *red = sm + (TYPE == HD_TYPE_Q8_0 ? 0 : NB * nu * 2);   // [NT][P+1][NB]
    float *red2 = red + NT * (P + 1) * NB;                            // [RC*NB*(P+1)][nch]
    // With a norm weight: x normalized into shared memory [B][K] first.
    const float *xsrc = a.x;
    if (a.nw) {
        __shared__ float nred[32 * NB], rs[NB];
        const int nch0 = (G + 15) / 16;
        float *xsm = red2 + RC * NB * (P + 1) * (nch0 > 1 ? nch0 : 0);
        xsm = (float *)(((uintptr_t)xsm + 15) & ~(uintptr_t)15);  // float4 reads
        norm_scales<NB>(a.x, a.K, a.B, a.eps, nred, rs);
        for (int i = t; i < a.B * a.K; i += NT) {
            const int b = i / a.K, k = i - b * a.K;
            xsm[i] = __fmul_rn(__fmul_rn(a.x[i], a.nw[k]), rs[b]);
        }
        __syncthreads();
        xsrc = xsm;
    }
    if constexpr (TYPE != HD_TYPE_Q8_0) {
        for (int i = t; i < NB * nu * 2; i += NT) {
            const int b = i / (nu * 2), ul = (i >> 1) % nu, hf = i & 1;
            float sx = 0.f;
            if (b < a.B) {
                const float4 *p4 = (const float4 *)(xsrc + (int64_t)b * a.K + (int64_t)(u0 + ul) * 32 + hf * 16);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float4 v = p4[j];
                    sx += (v.x + v.y) + (v.z + v.w);
                }
            }
            xh[i] = sx;
        }
        __syncthreads();
    }

    float acc[P + 1][NB];
#pragma unroll
    for (int p = 0; p <= P; p++)
#pragma unroll
        for (int b = 0; b < NB; b++) acc[p][b] = 0.f;

    int xoff[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) xoff[b] = b < a.B ? b * (a.K / 4) : 0;
    for (int base = u0 + g; base < u1; base += UCT * G) {
        if (base != u0 + g) {
#pragma unroll
            for (int c = 0; c < UCT; c++) {
                const int u = base + c * G;
#pragma unroll
                for (int p = 0; p <= P; p++) {
                    if (ok && u < u1) load_unit<TYPE>(p ? wb : wa, row, u, cur[c][p]);
                    else zero_unit<TYPE>(cur[c][p]);
                }
            }
        }
#pragma unroll
        for (int c = 0; c < UCT; c++) {
            const int u = base + c * G;
            if (ok && u < u1) {
                const float4 *xp = (const float4 *)(xsrc + (int64_t)u * 32);
#pragma unroll
                for (int p = 0; p <= P; p++)
                    unit_fma<TYPE, NB>(cur[c][p], u, xp, xoff, xh + (u - u0) * 2, nu * 2, acc[p]);
            }
        }
    }

    // Per-row sums over the G groups in a fixed order: groups of 16 first
    // (when G > 16), then the group sums.
#pragma unroll
    for (int p = 0; p <= P; p++)
#pragma unroll
        for (int b = 0; b < NB; b++) red[(t * (P + 1) + p) * NB + b] = acc[p][b];
    __syncthreads();
    const int nout = RC * a.B * (P + 1);
    const int nch = (G + 15) / 16;
    if (nch > 1) {
        for (int i = t; i < nout * nch; i += NT) {
            const int o = i / nch, c = i % nch;
            const int rr = o % RC, bp = o / RC, b = bp % a.B, p = bp / a.B;
            float s = 0.f;
            for (int gg = c * 16; gg < min(G, c * 16 + 16); gg++) s += red[((gg * RC + rr) * (P + 1) + p) * NB + b];
            red2[o * nch + c] = s;
        }
        __syncthreads();
    }
    for (int i = t; i < RC * a.B; i += NT) {
        const int rr = i % RC, b = i / RC;
        const int64_t rw = (int64_t)tile * RC + rr;
        if (rw >= a.N) continue;
        float v[P + 1];
#pragma unroll
        for (int p = 0; p <= P; p++) {
            float s = 0.f;
            if (nch > 1) {
                const int o = (p * a.B + b) * RC + rr;
                for (int c = 0; c < nch; c++) s += red2[o * nch + c];
            } else {
                for (int gg = 0; gg < G; gg++) s += red[((gg * RC + rr) * (P + 1) + p) * NB + b];
            }
            v[p] = s;
        }
        if (P) {
            a.y[(int64_t)b * a.ldy + rw] = silu_mul(v[0], v[P]);
        } else {
            float o = v[0];
            if (a.bias) o = o + a.bias[rw];
            if (a.residual) o = a.residual[(int64_t)b * a.ldy + rw] + o;
            a.y[(int64_t)b * a.ldy + rw] = o;
            if (!P && a.amax) atomicMax(&skey[b], argmax_key(o, (uint32_t)rw));
        }
    }
    if (P == 0 && a.amax) {
        // the CTA's best key per batch row into the global keys; the last CTA
        // turns them into ids (0 when a row's first value is NaN, as the
        // sequential scan gives) and clears them for the next launch
        __syncthreads();
        if (t < a.B) atomicMax(a.keys + t, skey[t]);
        __threadfence();
        __syncthreads();
        if (t == 0) slast = atomicAdd(a.keys + 16, 1ull) == (unsigned long long)gridDim.x - 1;
        __syncthreads();
        if (slast) {
            __threadfence();
            if (t < a.B) {
                const unsigned long long k = atomicExch(a.keys + t, 0ull);
                const float y0 = __ldcg(a.y + (int64_t)t * a.ldy);
                a.amax[t] = (y0 != y0 || k == 0ull) ? 0 : (int32_t)(0xFFFFFFFFu - (uint32_t)k);
            }
            if (t == 0) a.keys[16] = 0ull;
        }
    }
}

// ------------------------------------------------ batch 5..16 (padded 8, 16)
// Register-blocked: the x loads, not the FMAs, bound the kernel above at
// batch >= 8 (one float4 load per 4 FMAs).  Here lane l of warp w owns rows
// 4l..4l+3 of a 128-row tile and one unit of K at a time, so each float4 of x
// (the same address across the warp: one broadcast) feeds 16 FMAs.  Weights
// are decoded chunk by chunk (4 values of 4 rows) into their exact fp32
// values.  The (tile, unit) pairs are dealt out in tile-major order, 8 per
// CTA (one per warp), so every SM gets the same work; warps of one tile meet
// in shared memory, and a tile spread over several CTAs meets in the
// workspace, where the last CTA to arrive adds the segments in CTA order --
// fixed orders throughout, so results are bitwise reproducible.

template <int TYPE, int NB, int PT>
__global__ void __launch_bounds__(32 * NB, 1)
    k_qgemv_rb(GemvArgs a, int ntiles, int S, float *ws, int *tickets) {
    constexpr bool per_tile = PT != 0;
    constexpr int NT = 32 * NB;  // 8 unit slots x NB / 8 batch groups of 8
    // x of each slot's unit [8][NB][32] during the main loop, then the
    // per-slot partial sums [8][NB][128 rows]
    extern __shared__ float sm[];
    __shared__ int last;
    // warp = (batch group bg, unit slot): rows of the tile x unit x 8 batch rows
    const int warp = (threadIdx.x >> 5) & 7, bg = threadIdx.x >> 8, lane = threadIdx.x & 31;
    // blockIdx.y: group of 16 rows of x (more than 16 rows: a batch of GEMVs)
    const int grp = blockIdx.y, B = a.B - 16 * grp < 16 ? a.B - 16 * grp : 16;
    const float *X = a.x + (int64_t)grp * 16 * a.K;
    float *Yo = a.y + (int64_t)grp * 16 * a.ldy;
    const float *Rs = a.residual ? a.residual + (int64_t)grp * 16 * a.ldy : nullptr;
    int *tk = tickets + grp * ntiles;
    const int64_t cta = (int64_t)grp * gridDim.x + blockIdx.x;
    __shared__ float nred[32 * NB], rs[NB];
    const int units = a.w0.units;
    const int nwu = ntiles * units, g0 = blockIdx.x * 8;
    // Flattened: warp w takes pair g0 + w (one unit).  Per tile (tall
    // matrices, at least one tile per SM): CTA = tile, warp w the units
    // w, w + 8, ...
    const int gw = g0 + warp;
    const bool wok = per_tile || gw < nwu;
    const int tile = per_tile ? (int)blockIdx.x : wok ? gw / units : 0;
    const int ufirst = per_tile ? warp : wok ? gw - tile * units : units;
    const int ustep = per_tile ? 8 : units;
    const int64_t row0 = (int64_t)tile * 128 + 4 * lane;

    URegs<TYPE> cur[4];
#pragma unroll
    for (int rr = 0; rr < 4; rr++) {
        if (ufirst < units && row0 + rr < a.N) load_unit<TYPE>(a.w0, row0 + rr, ufirst, cur[rr]);
        else zero_unit<TYPE>(cur[rr]);
    }
    pdl_trigger();
    pdl_wait();

    float acc[4][8];
#pragma unroll
    for (int rr = 0; rr < 4; rr++)
#pragma unroll
        for (int b = 0; b < 8; b++) acc[rr][b] = 0.f;
    const int bbase = 8 * bg, nbw = B - bbase < 8 ? B - bbase : 8;  // this warp's batch rows
    if (a.nw) norm_scales<NB>(X, a.K, B, a.eps, nred, rs);
    // flattened: one pass (straight-line code); per tile: the warp's units
    for (int u = ufirst; u < units; u = per_tile ? u + ustep : units) {
        if (per_tile && u != ufirst) {
#pragma unroll
            for (int rr = 0; rr < 4; rr++) {
                if (row0 + rr < a.N) load_unit<TYPE>(a.w0, row0 + rr, u, cur[rr]);
                else zero_unit<TYPE>(cur[rr]);
            }
        }
        float4 *xs = (float4 *)sm + (warp * NB + bbase) * 8;
        __syncwarp();
        for (int i = lane; i < nbw * 8; i += 32) {
            float4 v = __ldg((const float4 *)(X + (int64_t)(bbase + (i >> 3)) * a.K + (int64_t)u * 32) + (i & 7));
            if (a.nw) {  // RMSNorm on the fly: (x * w) * r
                const float4 wn = __ldg((const float4 *)(a.nw + (int64_t)u * 32) + (i & 7));
                const float r = rs[bbase + (i >> 3)];
                v = make_float4(__fmul_rn(__fmul_rn(v.x, wn.x), r), __fmul_rn(__fmul_rn(v.y, wn.y), r),
                                __fmul_rn(__fmul_rn(v.z, wn.z), r), __fmul_rn(__fmul_rn(v.w, wn.w), r));
            }
            xs[i] = v;
        }
        __syncwarp();
        URowScale scl[4];
#pragma unroll
        for (int rr = 0; rr < 4; rr++) scl[rr] = unit_scale<TYPE>(cur[rr], u);
#pragma unroll
        for (int wd = 0; wd < 8; wd++) {
            float v[4][4];
#pragma unroll
            for (int rr = 0; rr < 4; rr++) chunk_vals<TYPE>(cur[rr], scl[rr], wd, v[rr]);
            // 4 batch rows at a time, component-major: 16 independent FMAs
            // between two that share an accumulator
#pragma unroll
            for (int b0 = 0; b0 < 8; b0 += 4) {
                if (b0 < nbw) {
                    float xv[4][4];
#pragma unroll
                    for (int bb = 0; bb < 4; bb++) {
                        const float4 t4 = b0 + bb < nbw ? xs[(b0 + bb) * 8 + wd] : make_float4(0.f, 0.f, 0.f, 0.f);
                        xv[bb][0] = t4.x;
                        xv[bb][1] = t4.y;
                        xv[bb][2] = t4.z;
                        xv[bb][3] = t4.w;
                    }
#pragma unroll
                    for (int k = 0; k < 4; k++)
#pragma unroll
                        for (int rr = 0; rr < 4; rr++)
#pragma unroll
                            for (int bb = 0; bb < 4; bb++)
                                acc[rr][b0 + bb] = fmaf(v[rr][k], xv[bb][k], acc[rr][b0 + bb]);
                }
            }
        }
    }
    __syncthreads();  // x no longer needed: the buffer takes the partial sums
#pragma unroll
    for (int rr = 0; rr < 4; rr++)
#pragma unroll
        for (int b = 0; b < 8; b++) sm[(warp * NB + bbase + b) * 128 + 4 * lane + rr] = acc[rr][b];
    __syncthreads();

    // One segment per tile this CTA touches: its warps w0..w1-1 add up in
    // order; a tile spread over several CTAs meets in the workspace, where the
    // last CTA to arrive adds the segments in CTA order.  Workspace slot of a
    // CTA's segment: its CTA index x S + the segment's rank in the CTA (only
    // the first CTA of a tile can hold it as a later segment).
    const int g1 = g0 + 8 < nwu ? g0 + 8 : nwu;
    const int t_first = per_tile ? tile : g0 / units, t_last = per_tile ? tile : (g1 - 1) / units;
    for (int t = t_first; t <= t_last; t++) {
        const int w0 = per_tile ? 0 : (t * units > g0 ? t * units : g0) - g0;
        const int w1 = per_tile ? 8 : ((t + 1) * units < g1 ? (t + 1) * units : g1) - g0;
        const int cf = t * units / 8, cl = ((t + 1) * units - 1) / 8;
        const int nseg = per_tile ? 1 : cl - cf + 1, slot = t - t_first;
        for (int o = threadIdx.x; o < 128 * NB; o += NT) {
            const int b = o >> 7, rl = o & 127;
            const int64_t row = (int64_t)t * 128 + rl;
            if (b >= B || row >= a.N) continue;
            float s = 0.f;
            for (int w = w0; w < w1; w++) s += sm[(w * NB + b) * 128 + rl];
            if (nseg == 1) {
                if (a.bias) s = s + a.bias[row];
                if (Rs) s = Rs[(int64_t)b * a.ldy + row] + s;
                Yo[(int64_t)b * a.ldy + row] = s;
            } else {
                __stcg(ws + ((cta * S + slot) * NB + b) * 128 + rl, s);
            }
        }
        if (nseg == 1) continue;
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) last = (atomicAdd(tk + t, 1) == nseg - 1);
        __syncthreads();
        if (last) {
            __threadfence();
            const int sf = t - cf * 8 / units;  // slot of the tile in its first CTA
            // 4 rows per thread-step (16-byte loads), the partials of a step
            // requested together, then added in CTA order
            for (int o4 = threadIdx.x; o4 < 32 * NB; o4 += NT) {
                const int b = o4 >> 5, r4 = (o4 & 31) * 4;
                if (b >= B) continue;
                const int64_t cbase = (int64_t)grp * gridDim.x;
                const float4 *p = (const float4 *)(ws + (((cbase + cf) * S + sf) * NB + b) * 128 + r4);
                float4 sum = __ldcg(p);
                for (int c0 = cf + 1; c0 <= cl; c0 += 8) {
                    float4 part[8];
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        if (c0 + j <= cl) part[j] = __ldcg((const float4 *)(ws + (((cbase + c0 + j) * S) * NB + b) * 128 + r4));
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        if (c0 + j <= cl) {
                            sum.x += part[j].x;
                            sum.y += part[j].y;
                            sum.z += part[j].z;
                            sum.w += part[j].w;
                        }
                }
                const float sv[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int64_t row = (int64_t)t * 128 + r4 + k;
                    if (row >= a.N) break;
                    float s = sv[k];
                    if (a.bias) s = s + a.bias[row];
                    if (Rs) s = Rs[(int64_t)b * a.ldy + row] + s;
                    Yo[(int64_t)b * a.ldy + row] = s;
                }
            }
            if (threadIdx.x == 0) tk[t] = 0;
        }
        __syncthreads();
    }
}

struct Plan {
    int nb, RC, G, nt, tiles;
    size_t smem;
};

int pad_batch(int B) { return B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : B <= 8 ? 8 : 16; }
int max_threads(int nb, bool pair) { return (nb <= 2 ? 1024 : nb <= 4 ? 512 : 256) >> (pair ? 1 : 0); }

// Launch shape, from a sweep of rows-per-CTA x threads-per-CTA on B200 in a
// PDL chain of back-to-back GEMVs:
//  - about 2 units per thread (4 at batch >= 8 or for very tall matrices);
//  - CTAs small enough in registers (<= 512 threads at batch <= 2, 256 at
//    3..4, 128 above) that the next kernel's CTA fits beside them, so its weight
//    prefetch overlaps this one -- unless the row tiles leave SMs idle anyway;
//  - 8..32 rows per CTA (whole 32-byte sectors, x broadcast across lanes),
//    at most about rows / SMs rounded up to a power of two.
// HACEDLE_GEMV_NT / HACEDLE_GEMV_RC override the thread cap and the rows per
// CTA (tuning knobs).
static int env_int(const char *name, int dflt) {
    const char *v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}
static int pow2ceil(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

Plan plan_gemv(int N, int units, int B, bool pair, int sms) {
    Plan p;
    p.nb = pad_batch(B);
    const int MT = max_threads(p.nb, pair);
    const bool tall = N >= 64 * sms;
    const int upt = (p.nb >= 8 || tall) ? 4 : 2;
    int G = pow2ceil((units + upt - 1) / upt);
    if (G > units) G = units;
    const int ntcap = p.nb <= 2 ? 512 : p.nb <= 4 ? 256 : 128;
    int rc_hi = pow2ceil((N + sms - 1) / sms);
    rc_hi = rc_hi < 8 ? 8 : rc_hi > 32 ? 32 : rc_hi;
    int RC = ntcap / G;
    RC = RC < 8 ? 8 : RC > rc_hi ? rc_hi : RC;
    const int nt_env = env_int("HACEDLE_GEMV_NT", 0), rc_env = env_int("HACEDLE_GEMV_RC", 0);
    if (rc_env >= 1 && rc_env <= 32) RC = rc_env;
    int cap = MT;
    if (nt_env >= 32 && nt_env < cap) cap = nt_env;
    if (RC > cap) RC = cap;
    if (nt_env >= 32) G = cap / RC < units ? cap / RC : units;
    if (RC * G > cap) G = cap / RC;
    if (G < 1) G = 1;
    if (RC > N) RC = N;
    p.RC = RC;
    p.G = G;
    p.nt = (RC * G + 31) / 32 * 32;  // whole warps (threads past RC*G own no unit group)
    p.tiles = (N + RC - 1) / RC;
    const int P1 = pair ? 2 : 1, nch = (G + 15) / 16;
    p.smem = ((size_t)p.nb * units * 2 + (size_t)p.nt * P1 * p.nb + (size_t)RC * p.nb * P1 * (nch > 1 ? nch : 0)) *
             sizeof(float);
    return p;
}

template <int TYPE, int NB, int P>
cudaError_t launch_inst(hd_ctx *ctx, const Plan &p, const GemvArgs &a) {
    if (p.smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_qgemv<TYPE, NB, P>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)p.smem);
        if (e != cudaSuccess) return e;
    }
    return hd_launch(ctx, k_qgemv<TYPE, NB, P>, dim3(p.tiles), dim3(p.nt), p.smem, a);
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

template <int TYPE, int NB, int PT>
cudaError_t launch_rb(hd_ctx *ctx, const GemvArgs &a, int ntiles, int ctas, int S, int groups) {
    const size_t smem = (size_t)8 * NB * 128 * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(k_qgemv_rb<TYPE, NB, PT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    return hd_launch(ctx, k_qgemv_rb<TYPE, NB, PT>, dim3(ctas, groups), dim3(32 * NB), smem, a, ntiles, S, ctx->ws,
                     ctx->tickets);
}

// Batch 5..16: the (128-row tile, unit) pairs in tile-major order, 8 per CTA
// (one per warp), so that the CTAs fill the SMs evenly; with at least one
// tile per SM, one CTA per tile instead (no partial sums to combine).
int run_gemv_rb(hd_ctx *ctx, const GemvArgs &a, int type, const char *name) {
    const int nb = a.B <= 8 ? 8 : 16, groups = (a.B + 15) / 16;
    const int ntiles = (a.N + 127) / 128, units = a.w0.units;
    const int per_tile = ntiles >= ctx->sm_count ? 1 : 0;
    const int64_t nwu = (int64_t)ntiles * units;
    const int ctas = per_tile ? ntiles : (int)((nwu + 7) / 8);
    const int S = (8 + units - 1) / units + 1;  // tiles one CTA can touch
    if (!per_tile) {
        int rc = hd_ensure_workspace(ctx, (size_t)ctas * groups * S * nb * 128 * sizeof(float),
                                     (size_t)ntiles * groups);
        if (rc) return rc;
    }
    cudaError_t e = cudaSuccess;
    HD_TYPE_SWITCH(type, T, {
        if (per_tile)
            e = nb == 8 ? launch_rb<T, 8, 1>(ctx, a, ntiles, ctas, S, groups)
                        : launch_rb<T, 16, 1>(ctx, a, ntiles, ctas, S, groups);
        else
            e = nb == 8 ? launch_rb<T, 8, 0>(ctx, a, ntiles, ctas, S, groups)
                        : launch_rb<T, 16, 0>(ctx, a, ntiles, ctas, S, groups);
    });
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "%s: %s", name, cudaGetErrorString(e));
    return HD_OK;
}

// Plain GEMVs at batch <= 4 on weights below HACEDLE_GEMV_SMALL_KB kilobytes
// (default 16 MB) that no large-matrix kernel took go to the small-matrix
// tensor-core kernel (hd_gemv_small.cu).  Measured on B200 in CUDA-graph
// chains over weight copies larger than L2, microseconds per launch, against
// the CTA kernel below: 0.5B-shaped Q5_0 4864 x 896 B=1 2.6 (3.3), B=4 3.2
// (5.8); Q6_K / Q4_K 896 x 4864 B=4 4.4 / 4.1 (7.3 / 7.3); Q5_0 1152 x 896
// B=1 2.2 (4.2); Q4_K 3584 x 3584 B=4 9.4 (21; 10.5 on the large-matrix
// tensor-core kernel).  Q8_0 weights of under 2 MB at batch 2..4 stay on the
// CTA kernel (896 x 896 B=4 3.5 against 4.3), and batch 5..16 on the tcgen05
// kernel (its x conversion per CTA costs more there).  HACEDLE_GEMV_SMALL = 0
// turns it off, = 1 sends every plain GEMV that fits to it (any batch).
bool small_gemv(const hd_weight *w, int B, int sms, bool pair = false) {
    const char *v = getenv("HACEDLE_GEMV_SMALL");
    const int e = v && *v ? atoi(v) : -1;
    if (e == 0) return false;
    if (e != 1) {
        const size_t lim = (size_t)env_int("HACEDLE_GEMV_SMALL_KB", 16384) * 1024;
        if (B > 4 || w->gguf_bytes >= lim) return false;
        if (w->type == HD_TYPE_Q8_0 && B >= 2 && w->gguf_bytes < ((size_t)2 << 20)) return false;
    }
    return hd_qgemv_small_fits(w, B, sms, pair);
}

// Plain GEMVs (no norm, no SwiGLU pair) at batch <= 4 on large weights take
// one of four kernels laid out for streaming (measured on B200 in CUDA-graph
// chains over weight copies larger than L2, fractions of the HBM copy peak):
//  - batch 1, weights of HACEDLE_GEMV_BIG_KB kilobytes and more (default
//    16 MB): the block kernel (hd_gemv_blk.cu; 7B-shaped Q5_0/Q4_K/Q6_K
//    0.48/0.38/0.47, Q8_0 LM head 0.69; the streamed kernel below
//    0.40/0.35/0.35/0.65);
//  - batch 2..4 on weights of HACEDLE_GEMV_MID_KB and more (default 4 MB),
//    and batch 1 from there up to HACEDLE_GEMV_BIG_KB: the streamed
//    tensor-core kernel (hd_gemv_stream.cu), whose time barely grows with
//    the batch (batch 4 Q5_0/Q4_K/Q6_K/Q8_0 0.38/0.33/0.32/0.68 against
//    0.23/0.20/0.24/0.36 on the others, batch 2 0.40/0.34/0.33/0.66 against
//    0.33/0.27/0.32/0.55; Q4_K 3584 x 3584 6.6-6.7 us at batch 1..4 against
//    7.7-9.1 on the small-matrix kernel);
//  - otherwise at batch 2..4, weights of HACEDLE_GEMV_MID_KB and more that
//    the small-matrix kernel does not take: the mma.sync kernel
//    (hd_gemv_mma.cu).
// HACEDLE_GEMV_ST / HACEDLE_GEMV_BLK / HACEDLE_GEMV_MMA / HACEDLE_GEMV_SK = 1
// send every batch <= 4 GEMV that fits to that kernel (in this order of
// precedence), = 0 turn it off.  Returns 4 (streamed tensor cores), 3
// (block), 2 (mma.sync), 1 (streamed CUDA cores) or 0 (the CTA kernel below).
int big_gemv_kernel(const hd_weight *w, int B, int sms) {
    auto env = [](const char *name) { const char *v = getenv(name); return v && *v ? atoi(v) : -1; };
    const int eb = env("HACEDLE_GEMV_BLK"), em = env("HACEDLE_GEMV_MMA"), es = env("HACEDLE_GEMV_SK");
    if (env("HACEDLE_GEMV_ST") == 1 && hd_qgemv_stream_fits(w, B, sms)) return 4;
    if (eb == 1 && hd_qgemv_blk_fits(w)) return 3;
    if (em == 1 && hd_qgemv_mma_fits(w)) return 2;
    if (es == 1 && hd_qgemv_sk_fits(w)) return 1;
    const size_t big = (size_t)env_int("HACEDLE_GEMV_BIG_KB", 16384) * 1024;
    const size_t mid = (size_t)env_int("HACEDLE_GEMV_MID_KB", 4096) * 1024;
    const bool blk_ok = eb != 0 && hd_qgemv_blk_fits(w), mma_ok = em != 0 && hd_qgemv_mma_fits(w);
    if (env("HACEDLE_GEMV_ST") != 0 && hd_qgemv_stream_fits(w, B, sms) && w->gguf_bytes >= mid &&
        (B >= 2 || w->gguf_bytes < big))
        return 4;
    if (B == 1) return w->gguf_bytes >= big && blk_ok ? 3 : 0;
    if ((B == 2 || w->type == HD_TYPE_Q8_0) && w->gguf_bytes >= big && blk_ok) return 3;
    if (w->gguf_bytes >= mid && mma_ok && !small_gemv(w, B, sms)) return 2;
    if (w->gguf_bytes >= big && blk_ok) return 3;
    return 0;
}

// Batch 5..16 on the streamed tensor-core kernel (weights of
// HACEDLE_GEMV_MID_KB and more whose x fragments fit its shared memory)
// instead of the tcgen05 or register-blocked kernels.  Measured on B200 in
// CUDA-graph chains, us per launch: batch 8 Q5_0 / Q4_K 18944 x 3584 24.7 /
// 21.7 against 49.3 / 51.4, Q8_0 151936 x 896 41.3 against 126.3 (batch 16
// 59.0 against 220.8), Q4_K 3584 x 3584 8.7 against 20.0 (batch 16 12.6
// against 30.4); on the 3 MB decode-sweep weights the tcgen05 kernel stays
// (batch 16 7.0-8.5 against 7.9-11.7).  Where the x fragments of the whole
// batch do not fit (long K), the batch goes in chunks of 8 or 4 rows, each
// launch re-reading the weight: batch 16 Q5_0 18944 x 3584 as 2 x 8, Q6_K
// 3584 x 18944 as 4 x 4 (~2 x 25 and ~4 x 27 us against 83 and 152).
// Returns the chunk size (0: not this kernel).  HACEDLE_GEMV_ST = 1 forces
// it, = 0 turns it off.
int stream_gemv_b16(const hd_weight *w, int B, int sms) {
    const char *v = getenv("HACEDLE_GEMV_ST");
    const int e = v && *v ? atoi(v) : -1;
    if (e == 0) return 0;
    if (e != 1 && w->gguf_bytes < (size_t)env_int("HACEDLE_GEMV_MID_KB", 4096) * 1024) return 0;
    if (hd_qgemv_stream_fits(w, B, sms)) return B;
    if (B > 8 && hd_qgemv_stream_fits(w, 8, sms)) return 8;
    return hd_qgemv_stream_fits(w, 4, sms) ? 4 : 0;
}

// pinned: the decoder's GEMVs -- the CTA kernel at batch <= 4 and the
// tcgen05 kernel at 5..16, the kernels its greedy tokens are pinned to (the
// small-matrix and large-matrix kernels sum in other orders; at a step whose
// top-2 logits are nearly tied that can change a greedy id).
int run_gemv(hd_ctx *ctx, const hd_weight *w, const hd_weight *w_up, const float *x, float *y, int B,
             const float *bias, const float *residual, const char *name, const float *nw = nullptr,
             float eps = 0.f, int32_t *amax = nullptr, bool pinned = false) {
    if (amax && (w_up || B > 4)) {  // the fused argmax rides on the CTA kernel at batch <= 4
        int rc = run_gemv(ctx, w, w_up, x, y, B, bias, residual, name, nw, eps, nullptr, pinned);
        return rc ? rc : hd_argmax_rows(ctx, y, B, w->rows, amax);
    }
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
        if (!rc) rc = run_gemv(ctx, w, nullptr, x, ctx->scratch, B, nullptr, nullptr, name, nw, eps, nullptr, pinned);
        if (!rc)
            rc = run_gemv(ctx, w_up, nullptr, x, ctx->scratch + one, B, nullptr, nullptr, name, nw, eps, nullptr, pinned);
        if (!rc) rc = hd_swiglu(ctx, ctx->scratch, ctx->scratch + one, y, (int64_t)one);
        return rc;
    }
    if (!w_up && !nw && !amax && !pinned) {
        const int k = B <= 4 ? big_gemv_kernel(w, B, ctx->sm_count) : 0;
        if (k == 4) return hd_qgemv_stream(ctx, w, x, y, B, bias, residual, name);
        if (k == 3) return hd_qgemv_blk(ctx, w, x, y, B, bias, residual, name);
        if (k == 2) return hd_qgemv_mma(ctx, w, x, y, B, bias, residual, name);
        if (k == 1) return hd_qgemv_sk(ctx, w, x, y, B, bias, residual, name);
        if (small_gemv(w, B, ctx->sm_count))
            return hd_qgemv_small(ctx, w, nullptr, x, y, B, bias, residual, nullptr, 0.f, name);
    }
    // the fused RMSNorm and the SwiGLU pair (the decoder's projections) on the
    // small-matrix kernel too, where it takes them
    if ((w_up || nw) && !amax && !pinned && small_gemv(w, B, ctx->sm_count, w_up != nullptr))
        return hd_qgemv_small(ctx, w, w_up, x, y, B, bias, residual, nw, eps, name);
    if (!w_up && !nw && !amax && !pinned && B > 4) {
        // in batch chunks of the largest size whose x fragments fit
        const int cb = stream_gemv_b16(w, B, ctx->sm_count);
        for (int b0 = 0; cb && b0 < B; b0 += cb) {
            const int nb = B - b0 < cb ? B - b0 : cb;
            const int64_t xo = (int64_t)b0 * w->cols, yo = (int64_t)b0 * w->rows;
            const int rc = hd_qgemv_stream(ctx, w, x + xo, y + yo, nb, bias, residual ? residual + yo : nullptr, name);
            if (rc || b0 + nb == B) return rc;
        }
    }
    if (!w_up && !nw && !amax) {  // batch 5..16 on the tensor cores, where the shape fits
        bool done = false;
        const int rc = hd_qgemv_tc(ctx, w, x, y, B, bias, residual, &done);
        if (rc || done) return rc;
    }
    GemvArgs a;
    a.w0 = wview(w);
    a.w1 = w_up ? wview(w_up) : a.w0;
    a.x = x;
    a.y = y;
    a.bias = bias;
    a.residual = residual;
    a.B = B;
    a.N = (int)w->rows;
    a.ldy = (int)w->rows;
    a.K = (int)w->cols;
    a.pair = w_up ? 1 : 0;
    a.nw = nw;
    a.eps = eps;
    a.amax = amax;
    a.keys = nullptr;
    if (amax) {
        int rc = hd_ensure_amax_keys(ctx);
        if (rc) return rc;
        a.keys = ctx->amax_keys;
    }
    if (!w_up && pad_batch(B) >= 8 && getenv("HACEDLE_GEMV_RB") == nullptr) return run_gemv_rb(ctx, a, w->type, name);
    Plan p = plan_gemv((int)w->rows, w->units, B, w_up != nullptr, ctx->sm_count);
    if (nw) p.smem += (size_t)B * w->cols * sizeof(float) + 16;  // the normalized x, 16-byte aligned
    a.RC = p.RC;
    a.G = p.G;
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

// fp32 Q-GEMM over T rows of x as groups of 16 rows of the batch kernel
// (exact dequantized weights, fp32 accumulation; the decoder's fp32 steps).
int hd_qgemm_rows_f32(hd_ctx *ctx, const hd_weight *w, const float *X, float *Y, int T) {
    GemvArgs a;
    a.w0 = a.w1 = wview(w);
    a.x = X;
    a.y = Y;
    a.bias = nullptr;
    a.residual = nullptr;
    a.B = T;
    a.N = (int)w->rows;
    a.ldy = (int)w->rows;
    a.K = (int)w->cols;
    a.RC = a.G = 0;
    a.pair = 0;
    a.nw = nullptr;
    a.eps = 0.f;
    a.amax = nullptr;
    a.keys = nullptr;
    return run_gemv_rb(ctx, a, w->type, "hd_qgemm");
}

// y = W rmsnorm(x) (+bias, +residual) or SwiGLU(W_gate x', W_up x') for
// B <= 16 rows: the RMSNorm ((x * w) * r, as hd_rmsnorm) is computed by each
// CTA in its prologue instead of a separate kernel (the decoder's steps).
int hd_qgemv_norm(hd_ctx *ctx, const hd_weight *w, const hd_weight *w_up, const float *x, const float *norm_w,
                  float eps, float *y, int B, const float *bias, const float *residual) {
    if (!norm_w) return hd_fail(ctx, HD_E_ARG, "hd_qgemv_rmsnorm: null norm weight");
    if (w_up && (bias || residual))
        return hd_fail(ctx, HD_E_ARG, "hd_qgemv_rmsnorm: the SwiGLU pair takes no bias or residual");
    return run_gemv(ctx, w, w_up, x, y, B, bias, residual, "hd_qgemv_rmsnorm", norm_w, eps);
}

// The decoder's GEMVs (see run_gemv: pinned).
int hd_qgemv_pinned(hd_ctx *ctx, const hd_weight *w, const hd_weight *w_up, const float *x, const float *norm_w,
                    float eps, float *y, int B, const float *bias, const float *residual) {
    return run_gemv(ctx, w, w_up, x, y, B, bias, residual, "decoder GEMV", norm_w, eps, nullptr, true);
}

// LM head and greedy sampling in one launch at batch <= 4 (larger batches:
// the GEMV, then hd_argmax_rows).
int hd_lm_head_argmax_run(hd_ctx *ctx, const hd_weight *w, const float *x, const float *norm_w, float eps,
                          float *logits, int32_t *idx, int B) {
    if (!ctx || !w || !x || !logits || !idx) return hd_fail(ctx, HD_E_ARG, "hd_lm_head_argmax: null argument");
    return run_gemv(ctx, w, nullptr, x, logits, B, nullptr, nullptr, "hd_lm_head_argmax", norm_w, eps, idx);
}

extern "C" int hd_lm_head_argmax(hd_ctx *ctx, const hd_weight *w, const float *x_dev, const float *norm_w_dev,
                                 float eps, float *logits_dev, int32_t *idx_dev, int B) {
    return hd_lm_head_argmax_run(ctx, w, x_dev, norm_w_dev, eps, logits_dev, idx_dev, B);
}

extern "C" int hd_qgemv_rmsnorm(hd_ctx *ctx, const hd_weight *w, const hd_weight *w_up, const float *x_dev,
                                const float *norm_w_dev, float eps, float *y_dev, int B, const float *bias_dev,
                                const float *residual_dev) {
    return hd_qgemv_norm(ctx, w, w_up, x_dev, norm_w_dev, eps, y_dev, B, bias_dev, residual_dev);
}
