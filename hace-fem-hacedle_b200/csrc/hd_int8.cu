// hd_int8.cu -- the integer q-ops of ops/q_ops.rs and ops/fused.rs.
// Wrapping i32 arithmetic is addition modulo 2^32, which is associative, so a
// parallel reduction gives exactly the bits of the sequential scalar path.
#include "hd_internal.cuh"

namespace {

template <int NT>
__global__ void __launch_bounds__(NT) k_dot_i8(const int8_t *__restrict__ a, const int8_t *__restrict__ b, int64_t n,
                                               const int32_t *bias, int32_t *carry, int32_t *__restrict__ out) {
    __shared__ uint32_t red[NT / 32];
    pdl_wait();
    pdl_trigger();
    const int64_t base = (int64_t)blockIdx.x * n;
    uint32_t acc = 0;
    int64_t i = threadIdx.x;
    if (((base & 3) == 0) && ((uintptr_t)a & 3) == 0 && ((uintptr_t)b & 3) == 0) {
        const int *a4 = (const int *)(a + base), *b4 = (const int *)(b + base);
        int64_t n4 = n >> 2;
        int s = 0;
        for (int64_t j = threadIdx.x; j < n4; j += NT) s = __dp4a(a4[j], b4[j], s);
        acc = (uint32_t)s;
        i = n4 * 4 + threadIdx.x;
    }
    for (; i < n; i += NT) acc += (uint32_t)((int32_t)a[base + i] * (int32_t)b[base + i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t s = 0;
        for (int w = 0; w < NT / 32; w++) s += red[w];
        if (carry) {
            s = s + (uint32_t)bias[blockIdx.x] + (uint32_t)carry[blockIdx.x];
            carry[blockIdx.x] = (int32_t)s;
        }
        out[blockIdx.x] = (int32_t)s;
    }
}

}  // namespace

extern "C" int hd_dot_i8(hd_ctx *ctx, const int8_t *a, const int8_t *b, int64_t n, int count, int32_t *out) {
    if (!ctx || !out || (n > 0 && (!a || !b))) return hd_fail(ctx, HD_E_ARG, "hd_dot_i8: null argument");
    HD_REQUIRE(ctx, n >= 0 && count >= 0, HD_E_ARG, "hd_dot_i8: negative size");
    if (count == 0) return HD_OK;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_dot_i8<256>, dim3(count), dim3(256), 0, a, b, n, (const int32_t *)nullptr,
                               (int32_t *)nullptr, out));
    return HD_OK;
}

extern "C" int hd_fused_qdot_qadd_qacc_i8(hd_ctx *ctx, const int8_t *a, const int8_t *b, int64_t n, int count,
                                          const int32_t *bias, int32_t *carry, int32_t *out) {
    if (!ctx || !out || !bias || !carry || (n > 0 && (!a || !b)))
        return hd_fail(ctx, HD_E_ARG, "hd_fused_qdot_qadd_qacc_i8: null argument");
    HD_REQUIRE(ctx, n >= 0 && count >= 0, HD_E_ARG, "hd_fused_qdot_qadd_qacc_i8: negative size");
    if (count == 0) return HD_OK;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_dot_i8<256>, dim3(count), dim3(256), 0, a, b, n, bias, carry, out));
    return HD_OK;
}
