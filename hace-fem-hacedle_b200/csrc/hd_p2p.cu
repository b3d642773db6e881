// hd_p2p.cu -- the exchange step of row-sharded layers over NVLink, without a
// collective library on the data path.
//
// Rank r of G holds its output slice Y_r [B][n] (rows r*n.. of the weight).
// Every rank keeps a full output buffer F [B][G*n] in memory that the other
// ranks map through CUDA IPC.  hd_push_columns writes Y_r straight into every
// rank's F at columns r*n.. (peer stores over NVLink, in the final layout, so
// there is no separate all-gather or re-layout), then raises its flag in each
// peer's flag array and waits until every peer's flag for this epoch is up in
// its own.  A call ends once all G slices are in this rank's F.
//
// hd_push_columns_multi does the same for up to HD_PUSH_MAX outputs (the
// projections of a layer) in one launch with one completion handshake, so the
// round trip of the flags is paid once per layer instead of once per output.
//
// Ordering: after a CTA barrier, one thread of each CTA fences at system scope
// and takes a ticket; the last CTA fences again and publishes the epoch with a
// release store, and the
// waiting thread reads the peers' epochs with acquire loads, so every peer's
// slice is visible to the kernels that follow on this rank.  The wait is
// bounded (about one second of clock64 time): on expiry the context's device
// flag records HD_E_TIMEOUT and the kernel returns.
#include <cstring>
#include <type_traits>

#include "hd_internal.cuh"

namespace {

constexpr long long P2P_SPIN_LIMIT = 2000000000LL;   // clock64 cycles (~1 s)

__device__ __forceinline__ void st_release_sys(int32_t *p, int32_t v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t *p) {
    int32_t v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// The end of a push: the CTA's stores, then one system-scope fence before its
// ticket; the last CTA publishes the epoch to every peer and waits (bounded)
// until every peer's epoch has reached this one.
__device__ __forceinline__ void push_complete(int32_t *const *__restrict__ flags, int world, int rank, int32_t epoch,
                                              int *tickets, int *err) {
    // The CTA's stores, then one system-scope fence before its ticket.
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = (atomicAdd(tickets, 1) == (int)gridDim.x - 1);
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    *tickets = 0;   // kept zero for the next user
    __threadfence_system();
    for (int r = 0; r < world; r++)
        if (r != rank) st_release_sys(flags[r] + rank, epoch);
    const int32_t *mine = flags[rank];
    const long long t0 = clock64();
    for (int r = 0; r < world; r++) {
        if (r == rank) continue;
        // Epochs only grow: a peer already in a later exchange counts as done.
        while (ld_acquire_sys(mine + r) - epoch < 0) {
            if (clock64() - t0 > P2P_SPIN_LIMIT) {
                atomicExch(err, HD_E_TIMEOUT);
                return;
            }
            __nanosleep(64);
        }
    }
}

// Grid-stride over the [B][n / VEC] vectors of y (VEC = 4: float4 copies,
// n % 4 == 0 and aligned), 4 loads in flight per thread before the stores to
// the `world` outputs; at most 4 CTAs per SM, so that few CTAs take a ticket.
template <int VEC>
__global__ void __launch_bounds__(256) k_push_columns(const float *__restrict__ y, float *const *__restrict__ full,
                                                      int32_t *const *__restrict__ flags, int world, int rank,
                                                      int B, int64_t n, int32_t epoch, int *tickets, int *err) {
    using V = typename std::conditional<VEC == 4, float4, float>::type;
    pdl_wait();
    pdl_trigger();
    // 32-bit index arithmetic: B * n < 2^31 (checked by the host).
    const uint32_t nv = (uint32_t)(n / VEC), total = (uint32_t)B * nv;
    const int64_t ldf = (int64_t)world * n;
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t e0 = blockIdx.x * blockDim.x + threadIdx.x; e0 < total; e0 += 4 * stride) {
        V v[4];
        int64_t dst[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint32_t e = e0 + u * stride;
            dst[u] = -1;
            if (e < total && e >= e0) {   // (e >= e0: no wrap-around)
                const uint32_t b = e / nv, j = (e - b * nv) * VEC;
                v[u] = __ldg((const V *)(y + (int64_t)b * n + j));
                dst[u] = (int64_t)b * ldf + (int64_t)rank * n + j;
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (dst[u] >= 0)
                for (int r = 0; r < world; r++) *(V *)(full[r] + dst[u]) = v[u];
    }
    push_complete(flags, world, rank, epoch, tickets, err);
}

// Up to HD_PUSH_MAX outputs in one launch: output i is y[i] [B][n[i]] into
// full[i][r] [B][world * n[i]]; the same grid-stride walk per output, then
// one handshake.
struct PushItems {
    const float *y[HD_PUSH_MAX];
    float *const *full[HD_PUSH_MAX];
    int64_t n[HD_PUSH_MAX];
    int count;
};

template <int VEC>
__global__ void __launch_bounds__(256) k_push_columns_multi(PushItems it, int32_t *const *__restrict__ flags,
                                                            int world, int rank, int B, int32_t epoch, int *tickets,
                                                            int *err) {
    using V = typename std::conditional<VEC == 4, float4, float>::type;
    pdl_wait();
    pdl_trigger();
    const uint32_t stride = gridDim.x * blockDim.x;
    for (int i = 0; i < it.count; i++) {
        const int64_t n = it.n[i], ldf = (int64_t)world * n;
        const float *__restrict__ y = it.y[i];
        float *const *__restrict__ full = it.full[i];
        const uint32_t nv = (uint32_t)(n / VEC), total = (uint32_t)B * nv;
        for (uint32_t e0 = blockIdx.x * blockDim.x + threadIdx.x; e0 < total; e0 += 4 * stride) {
            V v[4];
            int64_t dst[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint32_t e = e0 + u * stride;
                dst[u] = -1;
                if (e < total && e >= e0) {
                    const uint32_t b = e / nv, j = (e - b * nv) * VEC;
                    v[u] = __ldg((const V *)(y + (int64_t)b * n + j));
                    dst[u] = (int64_t)b * ldf + (int64_t)rank * n + j;
                }
            }
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (dst[u] >= 0)
                    for (int r = 0; r < world; r++) *(V *)(full[r] + dst[u]) = v[u];
        }
    }
    push_complete(flags, world, rank, epoch, tickets, err);
}

}  // namespace

extern "C" int hd_xbuf_alloc(hd_ctx *ctx, size_t bytes, void **dev_ptr) {
    if (!ctx || !dev_ptr || bytes == 0) return hd_fail(ctx, HD_E_ARG, "hd_xbuf_alloc: bad argument");
    *dev_ptr = nullptr;
    if (cudaMalloc(dev_ptr, bytes) != cudaSuccess) {
        cudaGetLastError();
        return hd_fail(ctx, HD_E_OOM, "hd_xbuf_alloc: %zu bytes", bytes);
    }
    HD_CUDA_TRY(ctx, cudaMemset(*dev_ptr, 0, bytes));
    return HD_OK;
}

extern "C" int hd_xbuf_free(hd_ctx *ctx, void *dev_ptr) {
    if (!ctx) return HD_E_ARG;
    if (dev_ptr) HD_CUDA_TRY(ctx, cudaFree(dev_ptr));
    return HD_OK;
}

extern "C" int hd_ipc_handle(hd_ctx *ctx, void *dev_ptr, void *handle_out) {
    if (!ctx || !dev_ptr || !handle_out) return hd_fail(ctx, HD_E_ARG, "hd_ipc_handle: null argument");
    cudaIpcMemHandle_t h;
    HD_CUDA_TRY(ctx, cudaIpcGetMemHandle(&h, dev_ptr));
    static_assert(sizeof(h) == HD_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle_out, &h, sizeof(h));
    return HD_OK;
}

extern "C" int hd_ipc_open(hd_ctx *ctx, const void *handle, void **peer_ptr) {
    if (!ctx || !handle || !peer_ptr) return hd_fail(ctx, HD_E_ARG, "hd_ipc_open: null argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *peer_ptr = nullptr;
    HD_CUDA_TRY(ctx, cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return HD_OK;
}

extern "C" int hd_ipc_close(hd_ctx *ctx, void *peer_ptr) {
    if (!ctx) return HD_E_ARG;
    if (peer_ptr) HD_CUDA_TRY(ctx, cudaIpcCloseMemHandle(peer_ptr));
    return HD_OK;
}

extern "C" int hd_push_columns(hd_ctx *ctx, const float *y_dev, float *const *full_ptrs_dev,
                               int32_t *const *flag_ptrs_dev, int world, int rank, int B, int64_t n,
                               int32_t epoch) {
    if (!ctx || !y_dev || !full_ptrs_dev || !flag_ptrs_dev)
        return hd_fail(ctx, HD_E_ARG, "hd_push_columns: null argument");
    HD_REQUIRE(ctx, world >= 1 && rank >= 0 && rank < world && B >= 1 && B <= 65535 && n >= 1, HD_E_SHAPE,
               "hd_push_columns: bad shape (world %d, rank %d, B %d, n %lld)", world, rank, B, (long long)n);
    HD_REQUIRE(ctx, epoch > 0, HD_E_ARG, "hd_push_columns: epoch must be positive");
    HD_REQUIRE(ctx, (int64_t)B * n < ((int64_t)1 << 31) - 4 * 4 * 256 * 4 * 148, HD_E_SHAPE,
               "hd_push_columns: slice of %lld values is too large", (long long)B * n);
    int rc = hd_ensure_workspace(ctx, 0, 1);
    if (rc) return rc;
    const bool v4 = n % 4 == 0 && ((uintptr_t)y_dev & 15) == 0;
    const int64_t total = (int64_t)B * (v4 ? n / 4 : n);
    int64_t ctas = (total + 255) / 256;
    if (ctas > 4 * (int64_t)ctx->sm_count) ctas = 4 * (int64_t)ctx->sm_count;
    const dim3 grid((unsigned)ctas);
    if (v4)
        HD_CUDA_TRY(ctx, hd_launch(ctx, k_push_columns<4>, grid, dim3(256), 0, y_dev, full_ptrs_dev, flag_ptrs_dev,
                                   world, rank, B, n, epoch, ctx->tickets, ctx->flag));
    else
        HD_CUDA_TRY(ctx, hd_launch(ctx, k_push_columns<1>, grid, dim3(256), 0, y_dev, full_ptrs_dev, flag_ptrs_dev,
                                   world, rank, B, n, epoch, ctx->tickets, ctx->flag));
    return HD_OK;
}

extern "C" int hd_push_columns_multi(hd_ctx *ctx, int count, const float *const *y_devs, float *const *const *full_ptrs_devs,
                                     const int64_t *ns, int32_t *const *flag_ptrs_dev, int world, int rank, int B,
                                     int32_t epoch) {
    if (!ctx || !y_devs || !full_ptrs_devs || !ns || !flag_ptrs_dev)
        return hd_fail(ctx, HD_E_ARG, "hd_push_columns_multi: null argument");
    HD_REQUIRE(ctx, count >= 1 && count <= HD_PUSH_MAX, HD_E_ARG, "hd_push_columns_multi: %d outputs (1..%d)", count,
               HD_PUSH_MAX);
    HD_REQUIRE(ctx, world >= 1 && rank >= 0 && rank < world && B >= 1 && B <= 65535, HD_E_SHAPE,
               "hd_push_columns_multi: bad shape (world %d, rank %d, B %d)", world, rank, B);
    HD_REQUIRE(ctx, epoch > 0, HD_E_ARG, "hd_push_columns_multi: epoch must be positive");
    PushItems it{};
    it.count = count;
    bool v4 = true;
    int64_t most = 0;
    for (int i = 0; i < count; i++) {
        if (!y_devs[i] || !full_ptrs_devs[i]) return hd_fail(ctx, HD_E_ARG, "hd_push_columns_multi: null output %d", i);
        HD_REQUIRE(ctx, ns[i] >= 1 && (int64_t)B * ns[i] < ((int64_t)1 << 31) - 4 * 4 * 256 * 4 * 148, HD_E_SHAPE,
                   "hd_push_columns_multi: output %d slice of %lld values", i, (long long)B * ns[i]);
        it.y[i] = y_devs[i];
        it.full[i] = full_ptrs_devs[i];
        it.n[i] = ns[i];
        v4 = v4 && ns[i] % 4 == 0 && ((uintptr_t)y_devs[i] & 15) == 0;
        most = most > B * ns[i] ? most : B * ns[i];
    }
    int rc = hd_ensure_workspace(ctx, 0, 1);
    if (rc) return rc;
    int64_t ctas = ((v4 ? most / 4 : most) + 255) / 256;
    if (ctas > 4 * (int64_t)ctx->sm_count) ctas = 4 * (int64_t)ctx->sm_count;
    if (ctas < 1) ctas = 1;
    if (v4)
        HD_CUDA_TRY(ctx, hd_launch(ctx, k_push_columns_multi<4>, dim3((unsigned)ctas), dim3(256), 0, it, flag_ptrs_dev,
                                   world, rank, B, epoch, ctx->tickets, ctx->flag));
    else
        HD_CUDA_TRY(ctx, hd_launch(ctx, k_push_columns_multi<1>, dim3((unsigned)ctas), dim3(256), 0, it, flag_ptrs_dev,
                                   world, rank, B, epoch, ctx->tickets, ctx->flag));
    return HD_OK;
}
