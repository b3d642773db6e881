// hd_noalloc.cu -- hd_argmax_rows_noalloc: greedy argmax over rows of logits
// that allocates no device memory at all.
//
// Who needs it: a caller that hands out every byte of device memory from its
// own pool or arena (a serving runtime that carved up HBM at start-up, an
// embedding that must not let a library cudaMalloc behind its back), or one
// on a latency-critical path where cudaMalloc's implicit synchronization is
// not acceptable.  Such a caller cannot create an hd_ctx (whose workspace is
// allocated on demand), so this entry point takes no context: inputs,
// outputs and a stream only.
//
// Scratch.  The two-stage reduction needs partial (value, index) pairs and a
// per-row arrival counter.  They live in g_argmax_scratch below, a
// file-scope __device__ array of HD_ARGMAX_NOALLOC_SCRATCH_BYTES (208 KiB)
// that every GPU which loads this library holds until the process exits.
// Limits: at most HD_ARGMAX_NOALLOC_MAX_ROWS rows, n < 2^31 (the indices
// are int32), and rows x chunks <= 16384 partials (chunks are widened to
// fit).
//
// Set-up.  In host code the array's name is only a stand-in for the device
// address, so the first call on each device (with that device current) asks
// the runtime for the real address with cudaGetSymbolAddress and keeps it,
// with the id of the context it belongs to; a call that finds a different
// context (the device was reset) looks the address up again.  Make the
// first call on a device, and the first after a reset, before any stream
// capture.
//
// Sharing.  Every call uses the same array and leaves its contents behind;
// the counters that must start at zero are cleared on the caller's stream
// before each launch.  Two calls whose work overlaps on the GPU (different
// streams without ordering between them) race on the array.
#include <cuda.h>
#include <stdint.h>

#include <mutex>

#include "hd_internal.cuh"

namespace {

constexpr int kMaxPartials = 16384;
constexpr int kMaxRows = HD_ARGMAX_NOALLOC_MAX_ROWS;
constexpr size_t kValOff = 0;
constexpr size_t kIdxOff = kValOff + sizeof(float) * kMaxPartials;       //  64 KiB
constexpr size_t kTicketOff = kIdxOff + sizeof(long long) * kMaxPartials; // 192 KiB
static_assert(kTicketOff + sizeof(int) * kMaxRows == HD_ARGMAX_NOALLOC_SCRATCH_BYTES, "scratch layout");

static __device__ __align__(256) unsigned char g_argmax_scratch[HD_ARGMAX_NOALLOC_SCRATCH_BYTES];

__device__ __forceinline__ bool better(float v, long long i, float bv, long long bi) {
    return v > bv || (v == bv && i < bi);
}

// CTA (c, row) reduces chunk c of the row; the last CTA of the row to arrive
// reduces the row's partials.  Same result as ArgMaxSampler::sample (first
// maximum, strict >; a NaN at index 0 gives 0).
template <int NT>
__global__ void __launch_bounds__(NT) k_argmax_noalloc(const float *__restrict__ x, long long n, long long chunk,
                                                       unsigned char *scratch, int32_t *out) {
    __shared__ float sv[NT];
    __shared__ long long si[NT];
    __shared__ int last;
    float *pv = (float *)(scratch + kValOff);
    long long *pi = (long long *)(scratch + kIdxOff);
    int *tickets = (int *)(scratch + kTicketOff);
    const long long row = blockIdx.y;
    const int c = blockIdx.x, nc = gridDim.x;
    const float *r = x + row * n;
    float bv = -INFINITY;
    long long bi = LLONG_MAX;
    const long long lo = (long long)c * chunk, hi = min(n, lo + chunk);
    for (long long i = lo + threadIdx.x; i < hi; i += NT) {
        float v = r[i];
        if (better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int s = NT / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s && better(sv[threadIdx.x + s], si[threadIdx.x + s], sv[threadIdx.x], si[threadIdx.x])) {
            sv[threadIdx.x] = sv[threadIdx.x + s];
            si[threadIdx.x] = si[threadIdx.x + s];
        }
        __syncthreads();
    }
    if (nc == 1) {
        if (threadIdx.x == 0) {
            float x0 = r[0];
            out[row] = (x0 != x0 || si[0] == LLONG_MAX) ? 0 : (int32_t)si[0];
        }
        return;
    }
    if (threadIdx.x == 0) {
        __stcg(pv + row * nc + c, sv[0]);
        __stcg(pi + row * nc + c, si[0]);
        __threadfence();
        last = (atomicAdd(tickets + row, 1) == nc - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    bv = -INFINITY;
    bi = LLONG_MAX;
    for (int i = threadIdx.x; i < nc; i += NT) {
        float v = __ldcg(pv + row * nc + i);
        long long ii = __ldcg(pi + row * nc + i);
        if (better(v, ii, bv, bi)) { bv = v; bi = ii; }
    }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int s = NT / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s && better(sv[threadIdx.x + s], si[threadIdx.x + s], sv[threadIdx.x], si[threadIdx.x])) {
            sv[threadIdx.x] = sv[threadIdx.x + s];
            si[threadIdx.x] = si[threadIdx.x + s];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        float x0 = r[0];
        out[row] = (x0 != x0 || si[0] == LLONG_MAX) ? 0 : (int32_t)si[0];
        tickets[row] = 0;
    }
}

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char *g_addr[kMaxDevices] = {};
unsigned long long g_ctx_id[kMaxDevices] = {};  // context the address belongs to

// Unique id of the current CUDA context (cuCtxGetId through the runtime's
// driver entry points, so the library needs no link against libcuda); 0 if
// it cannot be read.
unsigned long long current_context_id() {
    typedef CUresult (*GetCurrent)(CUcontext *);
    typedef CUresult (*GetId)(CUcontext, unsigned long long *);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static bool looked = false;
    if (!looked) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = (GetCurrent)p;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = (GetId)p;
        cudaGetLastError();
        looked = true;
    }
    CUcontext c = nullptr;
    unsigned long long id = 0;
    if (get_current && get_id && get_current(&c) == CUDA_SUCCESS && c && get_id(c, &id) == CUDA_SUCCESS) return id;
    return 0;
}

// Device address of g_argmax_scratch on the current device: looked up once
// per device, and again when the device's context is a new one (after
// cudaDeviceReset the module is loaded again and the array moves).
int scratch_address(unsigned char **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return HD_E_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) return HD_E_UNSUPPORTED;
    std::lock_guard<std::mutex> lk(g_mu);
    const unsigned long long id = current_context_id();
    if (!g_addr[dev] || (id && id != g_ctx_id[dev])) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_argmax_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            return HD_E_CUDA;
        }
        g_addr[dev] = (unsigned char *)p;
        g_ctx_id[dev] = id;
    }
    *out = g_addr[dev];
    return HD_OK;
}

}  // namespace

extern "C" int hd_argmax_rows_noalloc(const float *x_dev, int64_t rows, int64_t n, int32_t *idx_dev, void *stream) {
    if (!idx_dev || (rows > 0 && n > 0 && !x_dev)) return HD_E_ARG;
    if (rows < 0 || n < 0) return HD_E_ARG;
    if (rows > kMaxRows) return HD_E_SHAPE;
    if (n > INT32_MAX) return HD_E_SHAPE;  // the indices are int32
    if (rows == 0) return HD_OK;
    cudaStream_t st = (cudaStream_t)stream;
    if (n == 0) return cudaMemsetAsync(idx_dev, 0, (size_t)rows * sizeof(int32_t), st) == cudaSuccess ? HD_OK
                                                                                                     : HD_E_CUDA;
    unsigned char *scratch = nullptr;
    int rc = scratch_address(&scratch);
    if (rc) return rc;
    long long chunk = 8192, nc = (n + chunk - 1) / chunk;
    long long nc_max = kMaxPartials / rows;
    if (nc_max > 256) nc_max = 256;
    if (nc > nc_max) {
        nc = nc_max;
        chunk = (n + nc - 1) / nc;
    }
    if (nc > 1 && cudaMemsetAsync(scratch + kTicketOff, 0, (size_t)rows * sizeof(int), st) != cudaSuccess)
        return HD_E_CUDA;
    k_argmax_noalloc<256><<<dim3((unsigned)nc, (unsigned)rows), 256, 0, st>>>(x_dev, n, chunk, scratch, idx_dev);
    return cudaGetLastError() == cudaSuccess ? HD_OK : HD_E_CUDA;
}
