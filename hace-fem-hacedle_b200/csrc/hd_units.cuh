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

}  // namespace
