// hd_units.cuh -- registers of one 32-value unit of a weight row in the
// unit-major device layout: loads, per-unit scales and exact values (the
// decode Q-GEMV kernels).
#pragma once
#include "hd_internal.cuh"

namespace {

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

// The loads are pinned (ld_pin_*): issued before griddepcontrol.wait, they
// overlap the previous kernel instead of being moved to their first use.
template <int TYPE>
__device__ __forceinline__ void load_unit(const WView &w, int64_t r, int u, URegs<TYPE> &g) {
    const int64_t ur = (int64_t)u * w.rows + r;
    if constexpr (TYPE == HD_TYPE_Q8_0) {
        const uint4 *p = (const uint4 *)(w.q + ur * 32);
        g.a = ld_pin_v4(p);
        g.b = ld_pin_v4(p + 1);
        g.d = ld_pin_u16((const unsigned short *)w.meta + ur);
    } else if constexpr (TYPE == HD_TYPE_Q5_0) {
        g.a = ld_pin_v4(w.q + ur * 16);
        g.qh = ld_pin_u32((const unsigned int *)w.aux + ur);
        g.d = ld_pin_u16((const unsigned short *)w.meta + ur);
    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
        g.a = ld_pin_v4(w.q + ur * 16);
        g.m = ld_pin_v4(w.meta + ((int64_t)(u >> 3) * w.rows + r) * 16);
    } else {
        const int64_t sr = (int64_t)(u >> 3) * w.rows + r;
        g.a = ld_pin_v4(w.q + ur * 16);
        g.h = ld_pin_v2((const uint2 *)w.aux + ur);
        g.sc = ld_pin_v4(w.meta + sr * 16);
        g.d = ld_pin_u16(w.dsb + sr);
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

// Scales of one unit of one row: values 0-15 use s0, 16-31 use s1; Q4_K
// subtracts mn.  Decoded once per unit, applied per value.
struct URowScale {
    float s0, s1, mn;
};
template <int TYPE>
__device__ __forceinline__ URowScale unit_scale(const URegs<TYPE> &g, int u) {
    URowScale r;
    r.mn = 0.f;
    if constexpr (TYPE == HD_TYPE_Q8_0 || TYPE == HD_TYPE_Q5_0) {
        r.s0 = r.s1 = h2f((uint16_t)g.d);
    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
        int sc, m;
        q4k_sm_regs(u & 7, g.m.y, g.m.z, g.m.w, sc, m);
        r.s0 = r.s1 = __fmul_rn(h2f((uint16_t)(g.m.x & 0xFFFF)), (float)sc);
        r.mn = __fmul_rn(h2f((uint16_t)(g.m.x >> 16)), (float)m);
    } else {
        const int s0 = 2 * (u & 7);
        const uint32_t scw = w4(g.sc, s0 >> 2);
        const float d = h2f((uint16_t)g.d);
        r.s0 = __fmul_rn(d, (float)(int8_t)((scw >> (8 * (s0 & 3))) & 255));
        r.s1 = __fmul_rn(d, (float)(int8_t)((scw >> (8 * ((s0 & 3) + 1))) & 255));
    }
    return r;
}

// Quant values 4wd..4wd+3 of a unit as exact small integers, offset removed
// (Q8_0 -128..127, Q5_0 -16..15, Q4_K 0..15, Q6_K -32..31): a byte c of the
// re-ordered quant bits goes to 2^23 + byte by one byte_perm (mag), and the
// subtraction of 2^23 + offset is exact.
template <int TYPE>
__device__ __forceinline__ void chunk_ints(const URegs<TYPE> &g, int wd, float (&v)[4]) {
    if constexpr (TYPE == HD_TYPE_Q8_0) {
        const uint32_t x = (wd < 4 ? w4(g.a, wd) : w4(g.b, wd - 4)) ^ 0x80808080u;
#pragma unroll
        for (int c = 0; c < 4; c++) v[c] = mag(x, c) - 8388736.0f;
    } else if constexpr (TYPE == HD_TYPE_Q5_0) {
        const uint32_t q = w4(g.a, wd & 3);
        const uint32_t b = wd < 4 ? ((q & 0x0F0F0F0Fu) | ((g.qh >> wd) & 0x10101010u))
                                  : (((q >> 4) & 0x0F0F0F0Fu) | ((g.qh << (8 - wd)) & 0x10101010u));
#pragma unroll
        for (int c = 0; c < 4; c++) v[c] = mag(b, c) - 8388624.0f;
    } else if constexpr (TYPE == HD_TYPE_Q4_K) {
        const uint32_t q = w4(g.a, wd & 3);
        const uint32_t b = wd < 4 ? (q & 0x0F0F0F0Fu) : ((q >> 4) & 0x0F0F0F0Fu);
#pragma unroll
        for (int c = 0; c < 4; c++) v[c] = mag(b, c) - 8388608.0f;
    } else {
        const int i = wd & 3;
        const uint32_t hsel = wd < 4 ? g.h.x : g.h.y;
        const uint32_t b = ((w4(g.a, i) >> (wd < 4 ? 0 : 4)) & 0x0F0F0F0Fu) | (shl_or_shr(hsel, 4 - 2 * i) & 0x30303030u);
#pragma unroll
        for (int c = 0; c < 4; c++) v[c] = mag(b, c) - 8388640.0f;
    }
}

// Values 4wd..4wd+3 of a unit, exact (the dequantized weights): the integer
// times its scale, Q4_K minus its min.
template <int TYPE>
__device__ __forceinline__ void chunk_vals(const URegs<TYPE> &g, const URowScale &sc, int wd, float (&v)[4]) {
    const float s = wd < 4 ? sc.s0 : sc.s1;
    chunk_ints<TYPE>(g, wd, v);
#pragma unroll
    for (int c = 0; c < 4; c++) {
        v[c] = __fmul_rn(v[c], s);
        if constexpr (TYPE == HD_TYPE_Q4_K) v[c] = __fsub_rn(v[c], sc.mn);
    }
}

__device__ __forceinline__ float dot4(float a0, float a1, float a2, float a3, const float4 &x, float s) {
    s = fmaf(a0, x.x, s);
    s = fmaf(a1, x.y, s);
    s = fmaf(a2, x.z, s);
    return fmaf(a3, x.w, s);
}

// acc[b] += unit(u) . x[b][unit]; xs points at this unit's 32 floats of batch
// row 0, batch row b at float4 offset xoff[b].
// The float 2 + byte/64, exact for byte < 128: byte c of v goes to bits
// 16..23 under the exponent byte 0x40 (one byte_perm, no subtraction).  The
// constant 2 is removed per unit with the sum of x (see unit_fma).
__device__ __forceinline__ float f2q(uint32_t v, int c) {
    return __uint_as_float(__byte_perm(v, 0x40000000u, 0x7044u | ((uint32_t)c << 8)));
}

// acc[b] += unit(u) . x[b][unit].  xs points at this unit's 32 floats of batch
// row 0 (float4), batch row b at float4 offset xoff[b] (padded rows read row
// 0, so nothing past the B rows of x is touched); xh holds the sums of
// x over the unit's two 16-value halves, batch rows `xh_stride` apart.
//
// Q5_0, Q4_K and Q6_K form S = sum_j f_j x_j with f_j = 2 + q_j/64, so
// sum_j q_j x_j = 64 S - 128 X (X = sum_j x_j) and each type's offset folds
// into the X term:  Q5_0  d (64 S - 144 X);  Q4_K  64 d1 S - (128 d1 + m1) X;
// Q6_K  dl (64 S_lo - 160 X_lo) + dh (64 S_hi - 160 X_hi).  Q8_0 (signed
// bytes) uses 2^23 + byte and one subtraction per value.
template <int TYPE, int NB>
__device__ __forceinline__ void unit_fma(const URegs<TYPE> &g, int u, const float4 *xs, const int (&xoff)[NB],
                                         const float *xh, int xh_stride, float (&acc)[NB]) {
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
            for (int b = 0; b < NB; b++) s[b] = dot4(f0, f1, f2, f3, xs[xoff[b] + wd], s[b]);
        }
        float d = h2f((uint16_t)g.d);
#pragma unroll
        for (int b = 0; b < NB; b++) acc[b] = fmaf(d, s[b], acc[b]);
    } else if constexpr (TYPE == HD_TYPE_Q6_K) {
        float sl[NB], sh[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) sl[b] = sh[b] = 0.f;
#pragma unroll
        for (int wd = 0; wd < 4; wd++) {
            uint32_t v = w4(g.a, wd);
            uint32_t lo = (v & 0x0F0F0F0Fu) | (shl_or_shr(g.h.x, 4 - 2 * wd) & 0x30303030u);
            uint32_t hi = ((v >> 4) & 0x0F0F0F0Fu) | (shl_or_shr(g.h.y, 4 - 2 * wd) & 0x30303030u);
            float l0 = f2q(lo, 0), l1 = f2q(lo, 1), l2 = f2q(lo, 2), l3 = f2q(lo, 3);
            float h0 = f2q(hi, 0), h1 = f2q(hi, 1), h2 = f2q(hi, 2), h3 = f2q(hi, 3);
#pragma unroll
            for (int b = 0; b < NB; b++) {
                sl[b] = dot4(l0, l1, l2, l3, xs[xoff[b] + wd], sl[b]);
                sh[b] = dot4(h0, h1, h2, h3, xs[xoff[b] + 4 + wd], sh[b]);
            }
        }
        int s0 = 2 * (u & 7);
        uint32_t scw = w4(g.sc, s0 >> 2);
        int8_t c0 = (int8_t)((scw >> (8 * (s0 & 3))) & 255), c1 = (int8_t)((scw >> (8 * ((s0 & 3) + 1))) & 255);
        float d = h2f((uint16_t)g.d);
        float dl = d * (float)c0, dh = d * (float)c1;
#pragma unroll
        for (int b = 0; b < NB; b++) {
            const float xl = xh[b * xh_stride], xr = xh[b * xh_stride + 1];
            acc[b] = fmaf(dl, fmaf(64.f, sl[b], -160.f * xl), acc[b]);
            acc[b] = fmaf(dh, fmaf(64.f, sh[b], -160.f * xr), acc[b]);
        }
    } else {  // Q5_0, Q4_K: one scale per unit
        float s[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) s[b] = 0.f;
#pragma unroll
        for (int wd = 0; wd < 4; wd++) {
            uint32_t v = w4(g.a, wd), lo, hi;
            if constexpr (TYPE == HD_TYPE_Q5_0) {
                lo = (v & 0x0F0F0F0Fu) | ((g.qh >> wd) & 0x10101010u);
                hi = ((v >> 4) & 0x0F0F0F0Fu) | ((g.qh << (4 - wd)) & 0x10101010u);
            } else {
                lo = v & 0x0F0F0F0Fu;
                hi = (v >> 4) & 0x0F0F0F0Fu;
            }
            float l0 = f2q(lo, 0), l1 = f2q(lo, 1), l2 = f2q(lo, 2), l3 = f2q(lo, 3);
            float h0 = f2q(hi, 0), h1 = f2q(hi, 1), h2 = f2q(hi, 2), h3 = f2q(hi, 3);
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float t = dot4(l0, l1, l2, l3, xs[xoff[b] + wd], s[b]);
                s[b] = dot4(h0, h1, h2, h3, xs[xoff[b] + 4 + wd], t);
            }
        }
        if constexpr (TYPE == HD_TYPE_Q5_0) {
            float d = h2f((uint16_t)g.d);
#pragma unroll
            for (int b = 0; b < NB; b++) {
                const float X = xh[b * xh_stride] + xh[b * xh_stride + 1];
                acc[b] = fmaf(d, fmaf(64.f, s[b], -144.f * X), acc[b]);
            }
        } else {
            int sc, m;
            q4k_sm_regs(u & 7, g.m.y, g.m.z, g.m.w, sc, m);
            float d = h2f((uint16_t)(g.m.x & 0xFFFF)), dmin = h2f((uint16_t)(g.m.x >> 16));
            float d1 = d * (float)sc, m1 = dmin * (float)m;
#pragma unroll
            for (int b = 0; b < NB; b++) {
                const float X = xh[b * xh_stride] + xh[b * xh_stride + 1];
                acc[b] = fmaf(64.f * d1, s[b], fmaf(-(128.f * d1 + m1), X, acc[b]));
            }
        }
    }
}

}  // namespace
