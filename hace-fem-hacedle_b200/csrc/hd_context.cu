// hd_context.cu -- context lifetime, errors, workspace and launch accounting.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <vector>

#include "hd_internal.cuh"

int hd_fail(hd_ctx *ctx, int code, const char *fmt, ...) {
    if (ctx) {
        char buf[1024];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        ctx->err = buf;
    }
    return code;
}

int hd_check_launch(hd_ctx *ctx, const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return hd_fail(ctx, HD_E_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
    return HD_OK;
}

bool hd_type_supported(int t) {
    return t == HD_TYPE_Q8_0 || t == HD_TYPE_Q5_0 || t == HD_TYPE_Q4_K || t == HD_TYPE_Q6_K;
}

extern "C" const char *hd_version(void) { return HD_LIB_VERSION; }

extern "C" int hd_ctx_create(int device, hd_ctx **out) {
    if (!out) return HD_E_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return HD_E_CUDA;
    if (cudaSetDevice(device) != cudaSuccess) return HD_E_CUDA;
    hd_ctx *c = new hd_ctx();
    c->device = device;
    cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device);
    if (cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        return HD_E_CUDA;
    }
    c->stream = c->own_stream;
    // HACEDLE_PDL=0 turns programmatic dependent launch off (plain stream order).
    const char *pdl = getenv("HACEDLE_PDL");
    c->pdl = !(pdl && pdl[0] == '0');
    if (cudaMalloc(&c->flag, 64) != cudaSuccess || cudaMemset(c->flag, 0, 64) != cudaSuccess) {
        cudaStreamDestroy(c->own_stream);
        delete c;
        return HD_E_OOM;
    }
    *out = c;
    return HD_OK;
}

extern "C" int hd_ctx_destroy(hd_ctx *ctx) {
    if (!ctx) return HD_E_ARG;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->ws);
    cudaFree(ctx->tickets);
    cudaFree(ctx->rope_freq);
    cudaFree(ctx->hbuf_x);
    cudaFree(ctx->hbuf_y);
    cudaFree(ctx->flag);
    cudaFree(ctx->scratch);
    cudaFree(ctx->xbf);
    cudaFree(ctx->wbf);
    cudaFree(ctx->samp);
    cudaFree(ctx->kt_x);
    cudaFree(ctx->kt_y);
    cudaFree(ctx->amax_keys);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return HD_OK;
}

extern "C" int hd_ctx_set_stream(hd_ctx *ctx, void *stream) {
    if (!ctx) return HD_E_ARG;
    ctx->stream = stream ? (cudaStream_t)stream : ctx->own_stream;
    return HD_OK;
}

extern "C" int hd_ctx_synchronize(hd_ctx *ctx) {
    if (!ctx) return HD_E_ARG;
    HD_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return HD_OK;
}

extern "C" const char *hd_last_error(const hd_ctx *ctx) { return ctx ? ctx->err.c_str() : "null context"; }

extern "C" uint64_t hd_ctx_launch_count(const hd_ctx *ctx) { return ctx ? ctx->launches : 0; }

// Grows the split-K workspace and the ticket array.  Tickets start at zero and
// every split-K launch leaves them at zero.  Growing synchronizes the stream
// (a launch in flight may still use the old buffers), so callers that capture
// graphs reserve first.
int hd_ensure_workspace(hd_ctx *ctx, size_t bytes, size_t tickets) {
    if (bytes > ctx->ws_bytes) {
        size_t nb = bytes < ((size_t)8 << 20) ? ((size_t)8 << 20) : bytes;
        HD_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        cudaFree(ctx->ws);
        ctx->ws = nullptr;
        ctx->ws_bytes = 0;
        if (cudaMalloc(&ctx->ws, nb) != cudaSuccess) return hd_fail(ctx, HD_E_OOM, "workspace %zu bytes", nb);
        ctx->ws_bytes = nb;
    }
    if (tickets > ctx->n_tickets) {
        size_t nt = tickets < 65536 ? 65536 : tickets;
        HD_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        cudaFree(ctx->tickets);
        ctx->tickets = nullptr;
        ctx->n_tickets = 0;
        if (cudaMalloc(&ctx->tickets, nt * sizeof(int)) != cudaSuccess)
            return hd_fail(ctx, HD_E_OOM, "tickets %zu", nt);
        HD_CUDA_TRY(ctx, cudaMemsetAsync(ctx->tickets, 0, nt * sizeof(int), ctx->stream));
        HD_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        ctx->n_tickets = nt;
    }
    return HD_OK;
}

int hd_ensure_amax_keys(hd_ctx *ctx) {
    if (ctx->amax_keys) return HD_OK;
    void *p = nullptr;
    if (cudaMalloc(&p, 17 * sizeof(unsigned long long)) != cudaSuccess) {
        cudaGetLastError();
        return hd_fail(ctx, HD_E_OOM, "argmax keys");
    }
    HD_CUDA_TRY(ctx, cudaMemsetAsync(p, 0, 17 * sizeof(unsigned long long), ctx->stream));
    HD_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    ctx->amax_keys = (unsigned long long *)p;
    return HD_OK;
}

extern "C" int hd_ctx_reserve_workspace(hd_ctx *ctx, size_t bytes) {
    if (!ctx) return HD_E_ARG;
    return hd_ensure_workspace(ctx, bytes, 65536);
}

// theta^(2i/d) for i < d/2, computed on the host in f32 with powf -- the
// expression of src/ops/rope.rs:14 -- so device angles pos/freq[i] round
// exactly as the CPU path's do.
int hd_ensure_rope(hd_ctx *ctx, int head_dim, float theta) {
    if (ctx->rope_freq && ctx->rope_hd == head_dim && ctx->rope_theta == theta) return HD_OK;
    std::vector<float> f(head_dim / 2);
    for (int i = 0; i < head_dim / 2; i++) f[i] = powf(theta, 2.0f * (float)i / (float)head_dim);
    HD_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    cudaFree(ctx->rope_freq);
    ctx->rope_freq = nullptr;
    HD_CUDA_TRY(ctx, cudaMalloc(&ctx->rope_freq, f.size() * sizeof(float)));
    HD_CUDA_TRY(ctx, cudaMemcpy(ctx->rope_freq, f.data(), f.size() * sizeof(float), cudaMemcpyHostToDevice));
    ctx->rope_hd = head_dim;
    ctx->rope_theta = theta;
    return HD_OK;
}
