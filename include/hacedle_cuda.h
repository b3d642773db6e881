/*
 * hacedle_cuda.h -- C ABI of libhacedle_cuda.so, the B200 (sm_100a) kernels for
 * the quantized-weight hot path of the hacedle crate: GGUF block dequantization
 * (Q8_0, Q5_0, Q4_K, Q6_K) fused into GEMV / GEMM, plus the RMSNorm, RoPE,
 * GQA attention, SwiGLU and argmax kernels of a Qwen2-shaped decoder.
 *
 * Conventions
 *  - Every function returns an hd_status (0 = HD_OK).  hd_last_error() gives
 *    the message of the last failure on that context.  No C++ exception
 *    crosses this boundary.
 *  - Pointers named *_dev are device memory; *_host are host memory.  Sizes are
 *    element counts unless named *bytes.
 *  - A weight [rows x cols] is `rows` output rows of `cols` inputs, row-major
 *    with cols contiguous, exactly as a GGUF tensor stores it
 *    (QuantTensorView{data, shape=[rows, cols]}, src/quant_view/q4k_tensor_view.rs:46-61).
 *  - Work is enqueued on the context's stream (hd_ctx_set_stream; default: a
 *    stream the context creates).  Functions taking only device pointers are
 *    asynchronous; *_host functions synchronize before returning.
 *  - One context per host thread; a context is not safe for concurrent use.
 *  - Type ids are ggml's (gguf 0.19.0 GGMLQuantizationType).  The reference's
 *    QuantType discriminants (q4k_tensor_view.rs:9-19) are not ggml ids; a Rust
 *    binding maps enum variants, not their integer values (HD_TYPE_*).
 */
#ifndef HACEDLE_CUDA_H
#define HACEDLE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    HD_OK = 0,
    HD_E_ARG = 1,          /* null pointer or bad argument value          */
    HD_E_SHAPE = 2,        /* MatMulError::ShapeMismatch and kin           */
    HD_E_TYPE = 3,         /* quant type not carried by this library       */
    HD_E_CUDA = 4,         /* a CUDA runtime call failed                   */
    HD_E_TIMEOUT = 5,      /* a bounded device-side wait ran out           */
    HD_E_NCCL = 6,         /* a collective failed                          */
    HD_E_OOM = 7,          /* device allocation failed                     */
    HD_E_UNSUPPORTED = 8   /* valid request this build does not implement */
} hd_status;

enum {
    HD_TYPE_F32 = 0, HD_TYPE_F16 = 1, HD_TYPE_Q5_0 = 6, HD_TYPE_Q8_0 = 8,
    HD_TYPE_Q4_K = 12, HD_TYPE_Q6_K = 14
};

/* GEMM arithmetic: fp32 CUDA-core accumulate (1e-5 relative contract) or
 * bf16 operands on the tcgen05 tensor cores with fp32 accumulation in TMEM
 * (2e-2 relative contract). */
enum { HD_PREC_FP32 = 0, HD_PREC_BF16_TC = 1 };

typedef struct hd_ctx hd_ctx;
typedef struct hd_weight hd_weight;
typedef struct hd_decoder hd_decoder;

/* ---------------------------------------------------------------- context */
/* New context on CUDA device `device`. */
int hd_ctx_create(int device, hd_ctx **out);
int hd_ctx_destroy(hd_ctx *ctx);
/* Enqueue subsequent work on `stream` (a cudaStream_t); NULL restores the
 * context's own (non-blocking) stream.  Pass cudaStreamLegacy for the legacy
 * default stream. */
int hd_ctx_set_stream(hd_ctx *ctx, void *stream);
int hd_ctx_synchronize(hd_ctx *ctx);
/* Make sure the context's split-K workspace holds at least `bytes`, so that
 * later calls allocate nothing (needed before stream capture). */
int hd_ctx_reserve_workspace(hd_ctx *ctx, size_t bytes);
/* Message of the last failure on this context ("" if none). */
const char *hd_last_error(const hd_ctx *ctx);
/* Synchronizes the stream, then reads and clears the device error word that
 * bounded device-side waits set when they expire: HD_E_TIMEOUT if one did. */
int hd_ctx_check_device_errors(hd_ctx *ctx);
/* Number of kernels this context has launched (for launch accounting). */
uint64_t hd_ctx_launch_count(const hd_ctx *ctx);
const char *hd_version(void);

/* ---------------------------------------------------------------- weights */
/* Replaces QuantTensorView::new + its per-call clone (q4k_tensor_view.rs:46-56,
 * core/ops/block.rs:75-89): copies `nbytes` of GGUF blocks once to the device
 * and re-lays them out for the kernels (a lossless permutation of the same
 * bytes).  `cols` must be a multiple of the type's block (32 or 256) and
 * nbytes must equal QuantTensorView::size_bytes (:58-62). */
int hd_weight_upload(hd_ctx *ctx, const uint8_t *gguf_host, size_t nbytes, int ggml_type,
                     int64_t rows, int64_t cols, hd_weight **out);
/* Same, from GGUF bytes already in device memory. */
int hd_weight_upload_device(hd_ctx *ctx, const uint8_t *gguf_dev, size_t nbytes, int ggml_type,
                            int64_t rows, int64_t cols, hd_weight **out);
int hd_weight_free(hd_ctx *ctx, hd_weight *w);
int hd_weight_info(const hd_weight *w, int *ggml_type, int64_t *rows, int64_t *cols,
                   size_t *gguf_bytes);
/* Writes the weight back in GGUF block layout (round trip of the upload). */
int hd_weight_download(hd_ctx *ctx, const hd_weight *w, uint8_t *gguf_host, size_t nbytes);

/* -------------------------------------------------------------- dequant */
/* QuantTensorView::dequantize (q4k_tensor_view.rs:63-114): the full f32
 * tensor, bit-exact with IEEE f16 scales.  out_dev holds rows*cols floats. */
int hd_dequantize(hd_ctx *ctx, const hd_weight *w, float *out_dev, size_t n);

/* ----------------------------------------------------------------- GEMV */
/* Decode Q-GEMV, y[b][i] = sum_k W[i][k] x[b][k] (+ bias[i]) (+ residual[b][i])
 * for b < B <= 16.  Replaces matmul_vec_matrix (core/tensor_ops/matmul.rs:4-21),
 * the projection loops of BrainBlock::forward (core/ops/block.rs:104-128,
 * 210-231) and LMHead::forward (src/x/provider/candle/lmhead.rs:22-38).
 * x_dev [B][cols], y_dev [B][rows]; bias_dev [rows] or NULL; residual_dev
 * [B][rows] or NULL (may alias y_dev).  fp32 accumulate. */
int hd_qgemv(hd_ctx *ctx, const hd_weight *w, const float *x_dev, float *y_dev, int B,
             const float *bias_dev, const float *residual_dev);
/* Gate/up pair with the SwiGLU epilogue: y[b][i] = silu(G x)_i * (U x)_i
 * (src/ops/silu.rs:5-13 applied as Qwen2's silu(gate)*up). */
int hd_qgemv_swiglu(hd_ctx *ctx, const hd_weight *w_gate, const hd_weight *w_up,
                    const float *x_dev, float *y_dev, int B);
/* RMSNorm fused into the projection that consumes it: y = W rmsnorm(x)
 * (+bias, +residual), or with w_up != NULL the SwiGLU pair of rmsnorm(x).
 * Replaces the pair rms_norm (core/tensor_ops/rms_norm.rs:4-13, the block's
 * attn/ffn norms at core/ops/block.rs:96-103, 203-209) + matmul_vec_matrix;
 * the norm is (x * norm_w) * r with r = 1/sqrt(mean(x^2) + eps), as
 * hd_rmsnorm.  norm_w_dev [cols]; B <= 16; other arguments as hd_qgemv. */
int hd_qgemv_rmsnorm(hd_ctx *ctx, const hd_weight *w, const hd_weight *w_up, const float *x_dev,
                     const float *norm_w_dev, float eps, float *y_dev, int B, const float *bias_dev,
                     const float *residual_dev);
/* The reference operator with host slices in and out (matmul_vec_matrix's
 * &[f32] -> Vec<f32> contract): copies x in, runs hd_qgemv, copies y out. */
int hd_qgemv_host(hd_ctx *ctx, const hd_weight *w, const float *x_host, float *y_host, int B);

/* ----------------------------------------------------------------- GEMM */
/* Prefill Q-GEMM, Y[t][i] = sum_k W[i][k] X[t][k] for t < T.  Replaces
 * ComputeBackend::matmul_q4k/q6k (src/quant_view/dequant_dispatcher.rs:10-48,
 * routed by DequantDispatcher::dispatch_matmul :148-154) and matmul_f32 of a
 * quantized operand.  precision: HD_PREC_FP32 or HD_PREC_BF16_TC. */
int hd_qgemm(hd_ctx *ctx, const hd_weight *w, const float *X_dev, float *Y_dev, int T,
             int precision);
int hd_qgemm_host(hd_ctx *ctx, const hd_weight *w, const float *X_host, float *Y_host, int T,
                  int precision);
/* The same product in the operand layout of ComputeBackend::matmul_q4k /
 * matmul_q6k (src/quant_view/dequant_dispatcher.rs:10-48): a = the quantized
 * weight [N][K], b = X_kt [K][T] (b[l][j] at X_kt[l*T + j]), output Y_nt
 * [N][T] (out[i][j] at Y_nt[i*T + j]).  The operands are rearranged on the
 * device around hd_qgemm; a caller holding b quantized dequantizes it first
 * (hd_dequantize of a [K][T] weight gives exactly this layout).  _host: host
 * buffers, copies in and out and a synchronization inside the call. */
int hd_qgemm_kt(hd_ctx *ctx, const hd_weight *w, const float *X_kt_dev, float *Y_nt_dev, int T, int precision);
int hd_qgemm_kt_host(hd_ctx *ctx, const hd_weight *w, const float *X_kt_host, float *Y_nt_host, int T,
                     int precision);
/* Dense f32 GEMM, out[m][n] = sum_k a[m][k] b[k][n] (core/ops/matmul.rs:16-51,
 * ComputeBackend::matmul_f32 dequant_dispatcher.rs:72-83). */
int hd_matmul_f32(hd_ctx *ctx, const float *a_dev, const float *b_dev, float *out_dev, int64_t m,
                  int64_t n, int64_t k);

/* ------------------------------------------------ elementwise / reduction */
/* RMSNorm per row (dequant_dispatcher.rs:85-93, core/tensor_ops/rms_norm.rs:4-13):
 * y = x * w * (1/sqrt(mean(x^2) + eps)).  If residual_dev is not NULL it is
 * added to x first and the sum is written back to residual_dev (fused
 * residual add).  x_dev/y_dev [rows][dim]. */
int hd_rmsnorm(hd_ctx *ctx, const float *x_dev, const float *w_dev, float *residual_dev,
               float *y_dev, int64_t rows, int dim, float eps);
/* rmsnorm_f32 of the graph executor (core/ops/rmsnorm.rs:16-61): v*inv*w. */
int hd_rmsnorm_graph(hd_ctx *ctx, const float *x_dev, const float *w_dev, float *y_dev,
                     int64_t rows, int dim, float eps);
/* Per-head NEOX RoPE in place (apply_rope_pairwise, src/ops/rope.rs:5-31):
 * x_dev [tokens][heads][head_dim]; pos_dev [tokens]. */
int hd_rope_neox(hd_ctx *ctx, float *x_dev, const int32_t *pos_dev, int tokens, int heads,
                 int head_dim, float theta);
/* Interleaved-pair RoPE from cos/sin tables (rope_f32, core/ops/rope.rs:16-64). */
int hd_rope_interleaved(hd_ctx *ctx, const float *x_dev, const float *cos_dev,
                        const float *sin_dev, float *out_dev, int64_t rows, int last_dim);
/* Row softmax in place (NativeBackend::softmax, dequant_dispatcher.rs:117-128). */
int hd_softmax_rows(hd_ctx *ctx, float *x_dev, int64_t rows, int n);
/* out = silu(g) * u (n elements). */
int hd_swiglu(hd_ctx *ctx, const float *g_dev, const float *u_dev, float *out_dev, int64_t n);
/* out = a + b (add_f32, core/ops/add.rs:16-43). */
int hd_add(hd_ctx *ctx, const float *a_dev, const float *b_dev, float *out_dev, int64_t n);
/* First index of each row's maximum, strict > (ArgMaxSampler::sample,
 * runtime/sampler/argmax.rs:8-24); 0 for n == 0. */
int hd_argmax_rows(hd_ctx *ctx, const float *x_dev, int64_t rows, int64_t n, int32_t *idx_dev);
/* LMHead::forward followed by ArgMaxSampler::sample (src/x/provider/candle/
 * lmhead.rs:22-38, runtime/sampler/argmax.rs:8-24): logits_dev [B][rows] =
 * W x (x normalized first, (x * w) * r as hd_rmsnorm, when norm_w_dev is not
 * NULL) and idx_dev [B] = the first index of each row's maximum (0 when the
 * row's first logit is NaN).  B 1..16; up to 4 rows the argmax is folded into
 * the GEMV's epilogue (no second pass over the logits). */
int hd_lm_head_argmax(hd_ctx *ctx, const hd_weight *w, const float *x_dev, const float *norm_w_dev, float eps,
                      float *logits_dev, int32_t *idx_dev, int B);
/* Argmax of each row with no device allocation and no context.  It has no
 * counterpart in the reference.  It is for callers that cannot let a library
 * call cudaMalloc: runtimes that own all device memory through their own pool
 * or arena, and latency-critical paths that cannot afford cudaMalloc's
 * implicit synchronization.  Same result as hd_argmax_rows (first maximum
 * wins, strict >; 0 for n == 0 or a NaN at index 0), enqueued on `stream` (a
 * cudaStream_t; NULL = the legacy default stream) for the current device.
 * Its scratch is one static device array of HD_ARGMAX_NOALLOC_SCRATCH_BYTES
 * that each GPU loading the library keeps until exit.  rows above
 * HD_ARGMAX_NOALLOC_MAX_ROWS, and n of 2^31 or more (the indices are int32),
 * are rejected with HD_E_SHAPE; a device index of 64 or more gives
 * HD_E_UNSUPPORTED.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress), and so does the first call after the
 * device was reset (cudaDeviceReset); make those calls before any stream
 * capture.  All calls share the array: calls that overlap on the GPU race. */
#define HD_ARGMAX_NOALLOC_MAX_ROWS 4096
#define HD_ARGMAX_NOALLOC_SCRATCH_BYTES 212992
int hd_argmax_rows_noalloc(const float *x_dev, int64_t rows, int64_t n, int32_t *idx_dev, void *stream);
/* Embedding rows dequantized from a quantized table (embedding_lookup,
 * core/tensor_ops/embedding.rs:4-17): ids outside [0, rows) give zeros.
 * out_dev [n][cols]. */
int hd_embed(hd_ctx *ctx, const hd_weight *table, const int32_t *ids_dev, int n, float *out_dev);

/* Reassembles row-sharded outputs after an all-gather: src_dev [G][B][n]
 * (rank g's [B][n] slice of output rows g*n..g*n+n-1) -> dst_dev [B][G*n].
 * The reference has no multi-GPU path; this is the exchange step of the
 * row-sharded 7B-shaped layer. */
int hd_gather_columns(hd_ctx *ctx, const float *src_dev, float *dst_dev, int G, int B, int64_t n);

/* Exchange of row-sharded outputs over NVLink, our own kernel in place of
 * an all-gather plus hd_gather_columns.  The reference has no multi-GPU
 * path; this is the exchange step of the row-sharded 7B-shaped layer.
 *
 * Each rank allocates one exchange buffer (hd_xbuf_alloc: cudaMalloc'd,
 * zeroed) that holds its flag array (int32 [G]) and its full output buffers,
 * passes hd_ipc_handle's 64 bytes to the other ranks (any host channel), and
 * maps theirs with hd_ipc_open (hd_ipc_close undoes it).
 *
 * hd_push_columns: rank `rank` of `world` writes y_dev [B][n] (its output rows
 * rank*n..) into every rank's full buffer [B][world*n] at columns rank*n..,
 * then raises its flag (= epoch) in every peer's flag array, and waits until
 * every peer's flag has reached epoch in its own.  full_ptrs_dev and
 * flag_ptrs_dev are DEVICE arrays of `world` pointers, indexed by rank
 * (this rank's own buffers, the peers' IPC mappings); full buffers 16-byte
 * aligned.  Every rank makes the same sequence of calls with the same,
 * growing epochs (> 0).  The wait is bounded (about 1 s): on expiry the
 * context's device error flag holds HD_E_TIMEOUT (hd_ctx_check_device_errors).
 * Reuse: give each output two full buffers and alternate them between
 * consecutive exchanges of that output (hacedle_cuda.shard.PeerExchange does).
 * Then no peer overwrites what a rank still reads: a peer writes exchange
 * u + 2 of an output into the buffer that holds exchange u only after its own
 * exchange u + 1 has seen this rank's flag, which this rank raises only after
 * every kernel it enqueued before that exchange has completed (the kernel
 * waits for its stream predecessors before it stores).  So the result of an
 * exchange stays valid for every kernel a rank enqueues before its next
 * exchange of the same output. */
#define HD_IPC_HANDLE_BYTES 64
int hd_xbuf_alloc(hd_ctx *ctx, size_t bytes, void **dev_ptr);
int hd_xbuf_free(hd_ctx *ctx, void *dev_ptr);
int hd_ipc_handle(hd_ctx *ctx, void *dev_ptr, void *handle_out);
int hd_ipc_open(hd_ctx *ctx, const void *handle, void **peer_ptr);
int hd_ipc_close(hd_ctx *ctx, void *peer_ptr);
int hd_push_columns(hd_ctx *ctx, const float *y_dev, float *const *full_ptrs_dev, int32_t *const *flag_ptrs_dev,
                    int world, int rank, int B, int64_t n, int32_t epoch);
/* hd_push_columns_multi: the same for `count` (1..HD_PUSH_MAX) outputs of one
 * layer in one launch with one completion handshake: output i is y_devs[i]
 * [B][ns[i]] into the full buffers of DEVICE pointer array full_ptrs_devs[i]
 * ([B][world*ns[i]] each).  y_devs, full_ptrs_devs and ns are HOST arrays of
 * `count` entries.  One epoch covers all the outputs; the reuse rule above
 * applies per output. */
#define HD_PUSH_MAX 16
int hd_push_columns_multi(hd_ctx *ctx, int count, const float *const *y_devs, float *const *const *full_ptrs_devs,
                          const int64_t *ns, int32_t *const *flag_ptrs_dev, int world, int rank, int B,
                          int32_t epoch);

/* ------------------------------------------------------- KV and attention */
/* Device KV cache (KvCache::append, core/ops/block.rs:268-282, KvArena
 * runtime/kv_cache.rs:8-34): caches are [seq][max_ctx][n_kv][head_dim] f32;
 * k/v_dev [seq][tokens][n_kv][head_dim] written at positions pos0[s] + t. */
int hd_kv_append(hd_ctx *ctx, const float *k_dev, const float *v_dev, float *kcache_dev,
                 float *vcache_dev, const int32_t *pos0_dev, int seqs, int tokens, int n_kv,
                 int head_dim, int max_ctx);
/* GQA decode attention, one query token per sequence (block.rs:138-173 with
 * kv head = h / (n_heads/n_kv)): q_dev [seq][n_heads][hd], attends to cache
 * positions [0, len[s]); out_dev [seq][n_heads][hd]. */
int hd_attention_decode(hd_ctx *ctx, const float *q_dev, const float *kcache_dev,
                        const float *vcache_dev, const int32_t *len_dev, int seqs, int n_heads,
                        int n_kv, int head_dim, int max_ctx, float *out_dev);
/* Causal prefill attention for one sequence: q_dev [T][n_heads][hd] at
 * positions pos0..pos0+T-1 attends to cache positions [0, pos0+t]. */
int hd_attention_prefill(hd_ctx *ctx, const float *q_dev, const float *kcache_dev,
                         const float *vcache_dev, int T, int pos0, int n_heads, int n_kv,
                         int head_dim, int max_ctx, float *out_dev);

/* ------------------------------------------------------------ integer ops */
/* exec_q_dot / dot_batch (ops/q_ops.rs:11-13, ops/batch.rs:3-29): wrapping
 * i32 dot of two i8 vectors, for `count` independent pairs of length n
 * (a_dev, b_dev [count][n]); out_dev [count]. */
int hd_dot_i8(hd_ctx *ctx, const int8_t *a_dev, const int8_t *b_dev, int64_t n, int count,
              int32_t *out_dev);
/* fused_qdot_qadd_qacc_i8 (ops/fused.rs:52-57) for `count` independent
 * streams: out = dot + bias + carry (wrapping), carry = out. */
int hd_fused_qdot_qadd_qacc_i8(hd_ctx *ctx, const int8_t *a_dev, const int8_t *b_dev, int64_t n,
                               int count, const int32_t *bias_dev, int32_t *carry_dev,
                               int32_t *out_dev);

/* ---------------------------------------------------------------- decoder */
/* Qwen2-shaped decoder run natively on the device: BrainBlock::forward
 * (core/ops/block.rs:51-238, corrected: RoPE on all heads, GQA h/(nh/nkv),
 * o_proj applied, silu(gate)*up, q/k/v biases) for every layer, then the
 * final RMSNorm, the tied LM head and greedy argmax (runtime/sampler/argmax.rs). */
typedef struct {
    int hidden, n_layers, n_heads, n_kv, head_dim, ffn, vocab;
    int max_ctx;    /* positions per sequence in the KV cache */
    int max_seqs;   /* sequences decoded together (1..256)     */
    float eps, theta;
} hd_decoder_config;

typedef struct {
    const hd_weight *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    /* host f32 vectors, copied at create time */
    const float *bq, *bk, *bv, *attn_norm, *ffn_norm;
} hd_layer_weights;

int hd_decoder_create(hd_ctx *ctx, const hd_decoder_config *cfg, const hd_layer_weights *layers,
                      const float *out_norm_host, const hd_weight *embed, hd_decoder **out);
int hd_decoder_free(hd_decoder *dec);
/* Prefill `n_prompt` ids of each of `seqs` sequences (prompts_host
 * [seqs][n_prompt]) and greedy-decode n_gen ids each (out_host [seqs][n_gen]).
 * prefill_precision: HD_PREC_FP32 or HD_PREC_BF16_TC.  Decode steps replay a
 * captured CUDA graph.  If step_ms_out is not NULL it receives the device time
 * of the decode loop in milliseconds. */
int hd_decoder_generate(hd_decoder *dec, const int32_t *prompts_host, int seqs, int n_prompt,
                        int n_gen, int prefill_precision, int32_t *out_host, float *decode_ms_out,
                        float *prefill_ms_out);
/* hd_decoder_generate with two additions (either may be NULL):
 * forced_host [seqs][n_gen]: teacher forcing -- the input of decode step g
 * (g >= 1) is forced_host[s][g - 1] instead of the previous greedy id; out_host
 * still receives the greedy id of every step (the argmax of its logits).
 * logits_host [n_gen][seqs][vocab]: the logits of every step (row g chose
 * out_host[s][g]): LMHead::forward's output (src/x/provider/candle/lmhead.rs:22-38)
 * for each generated position.  Copying the logits out adds a device-to-host
 * copy per step to the decode time. */
int hd_decoder_generate_ex(hd_decoder *dec, const int32_t *prompts_host, int seqs, int n_prompt,
                           int n_gen, int prefill_precision, const int32_t *forced_host, int32_t *out_host,
                           float *logits_host, float *decode_ms_out, float *prefill_ms_out);

/* ------------------------------------------------------ Q8_1 integer path */
/* Activations as 8-bit blocks of 32 (48 bytes each, 16-byte aligned):
 * int8 q[32]; float d; int16 s0, s1; 4 bytes zero -- d = max|x| / 127,
 * q = round-half-even(x * (1/d)), s0 / s1 = sum of q over values 0-15 / 16-31.
 * blocks_dev holds B * K / 32 blocks, row b's blocks contiguous. */
int hd_quantize_q8_1(hd_ctx *ctx, const float *x_dev, int B, int64_t K, void *blocks_dev);
/* y[b][n] = sum over 32-value units of d_x (a_0 dot_0 - o_0 s0 + a_1 dot_1 - o_1 s1),
 * dot_h the int32 dot of the weight's small-integer quants with q over half h
 * (dp4a), w = a_h q - o_h per half (Q8_0: d, 0; Q5_0: d, 16d; Q4_K: d sc,
 * dmin m; Q6_K: d sc_h, 32 d sc_h).  B 1..16.  Accuracy: the 2e-2 relative
 * contract of the bf16 path (activations rounded to 1/254 of a block's range).
 * The next step after the reference's i8 ops (ops/q_ops.rs:11-13). */
int hd_qgemv_q8_1(hd_ctx *ctx, const hd_weight *w, const void *blocks_dev, float *y_dev, int B);

/* ---------------------------------------------------------------- sampler */
/* LogitsProcessor::process (src/x/provider/candle/lmhead.rs:42-111) in place on
 * rows x n logits, with the reference's definitions: l /= max(temperature,
 * 0.001); top-p threshold = the logit at which the descending-order f32 sum of
 * min(exp(l), 1) first reaches top_p (0.0 if it never does); top-k threshold =
 * the (top_k+1)-th largest logit after top-p (none when top_k is 0 or >= n);
 * logits below either threshold become -inf.  rows * n < 2^31. */
int hd_logits_process(hd_ctx *ctx, float *logits_dev, int64_t rows, int64_t n, float temperature,
                      float top_p, int64_t top_k);
/* One index per row drawn from softmax(logits) (-inf entries never drawn;
 * -1 for a row with no finite logit).  Row r uses the Philox4x32-10 block at
 * counter offset + r under key `seed`, so draws are reproducible. */
int hd_sample_rows(hd_ctx *ctx, const float *logits_dev, int64_t rows, int64_t n, uint64_t seed,
                   uint64_t offset, int32_t *idx_dev);

/* -------------------------------------------------------- KV-cache arena */
/* The device KV-cache manager (runtime/kv_cache.rs: KvArena :8-34, SessionKv
 * :37-56, SoulKv / SoulMemoryRegistry :58-118, KvCacheManager :121-127).
 * The arena is `slots` KV slots in HBM, K and V each
 * [layers][slots][max_ctx][n_kv][head_dim] f32 (hd_kv_layer gives one
 * layer's [slots][max_ctx][n_kv][head_dim] block).  Sessions (by id, under a
 * soul id) and snapshots each hold one slot.  KvError: SessionNotFound /
 * SoulNotFound -> HD_E_ARG, ContextFull -> HD_E_SHAPE, AllocationFailed ->
 * HD_E_OOM (message names the case).  An arena is used from its context's
 * thread, like the context. */
typedef struct hd_kv_arena hd_kv_arena;
typedef struct {            /* KvSnapshot (kv_cache.rs:83-88)                   */
    uint64_t snapshot_id;
    int32_t token_position; /* positions copied                                 */
    int32_t slot;           /* the slot holding the copy                        */
    uint64_t kv_offset;     /* byte offset of that slot within a layer's block  */
    uint64_t timestamp;     /* logical clock of the arena (one tick per snapshot) */
} hd_kv_snapshot_t;

int hd_kv_arena_create(hd_ctx *ctx, int layers, int n_kv, int head_dim, int max_ctx, int slots,
                       hd_kv_arena **out);
int hd_kv_arena_free(hd_kv_arena *arena);
int hd_kv_layer(hd_kv_arena *arena, int layer, float **k_dev, float **v_dev);
/* KvCacheManager::allocate / SoulKv::get_or_create_session: the session's
 * slot (an existing session keeps its slot and position). */
int hd_kv_allocate(hd_kv_arena *arena, const char *session_id, const char *soul_id, int *slot);
int hd_kv_release(hd_kv_arena *arena, const char *session_id);
int hd_kv_session(hd_kv_arena *arena, const char *session_id, int *slot, int *position);
/* KvCacheManager::append: the session's position advances by `count`
 * (ContextFull beyond max_ctx, position unchanged). */
int hd_kv_advance(hd_kv_arena *arena, const char *session_id, int count);
int hd_kv_soul_sessions(hd_kv_arena *arena, const char *soul_id, int *count);
/* KvCacheManager::snapshot / restore: copy the session's cached positions
 * (every layer, K and V) into a free slot / back into `session_id` (created
 * under the snapshot's soul if new: a branch), whose position becomes the
 * snapshot's.  Snapshots stay valid until hd_kv_snapshot_free. */
int hd_kv_snapshot(hd_kv_arena *arena, const char *session_id, hd_kv_snapshot_t *out);
int hd_kv_restore(hd_kv_arena *arena, const hd_kv_snapshot_t *snap, const char *session_id);
int hd_kv_snapshot_free(hd_kv_arena *arena, const hd_kv_snapshot_t *snap);
/* Slot-indexed device ops on one layer's block: row r's k/v appended to slot
 * slots[r] at pos[r]; decode attention of row r over slot slots[r]'s first
 * len[r] positions (otherwise as hd_attention_decode). */
int hd_kv_append_slots(hd_ctx *ctx, const float *k_dev, const float *v_dev, float *kc_dev, float *vc_dev,
                       const int32_t *slots_dev, const int32_t *pos_dev, int rows, int n_kv, int head_dim,
                       int max_ctx);
int hd_attention_decode_slots(hd_ctx *ctx, const float *q_dev, const float *kc_dev, const float *vc_dev,
                              const int32_t *slots_dev, const int32_t *len_dev, int rows, int n_heads, int n_kv,
                              int head_dim, int max_ctx, float *out_dev);

/* ------------------------------------------------------------ GGUF reader */
/* Replaces GgufLoader::load_std, GgufTensorIndex::parse and tensor_bytes
 * (src/x/loader/gguf/loader.rs:64-141, tensor_index.rs:24-170, header.rs:54-84)
 * with a reader of the published GGUF v2/v3 layout (gguf 0.19.0 GGUFWriter):
 * u32 value types (STRING = 8, ARRAY = 9, UINT64 = 10 ...), tensor infos as
 * {name, n_dims, dims, ggml_type, offset}, data aligned to general.alignment,
 * tensor sizes from the ggml block tables.  Host only (no context, no GPU),
 * except hd_gguf_upload.  A malformed or truncated file fails with HD_E_ARG
 * (HD_E_UNSUPPORTED for other versions or array element types); the message
 * of the last failed hd_gguf_* call on this thread is hd_gguf_error(). */
typedef struct hd_gguf hd_gguf;
typedef struct {
    const char *name;       /* owned by the handle                            */
    int32_t ggml_type;
    int32_t n_dims;         /* 1..4                                           */
    int64_t dims[4];        /* ggml order: dims[0] is the contiguous axis (a
                               [rows x cols] weight has dims {cols, rows}); 1 past n_dims */
    uint64_t offset;        /* absolute file offset of the tensor's data      */
    uint64_t nbytes;        /* 0 when the type's block size is not known here */
    const uint8_t *data;    /* host pointer into the handle's bytes           */
} hd_gguf_tensor_info;

/* Maps the file read-only (the handle keeps the mapping until hd_gguf_close). */
int hd_gguf_open(const char *path, hd_gguf **out);
/* Parses a copy of `nbytes` bytes already in host memory. */
int hd_gguf_open_memory(const uint8_t *bytes, size_t nbytes, hd_gguf **out);
int hd_gguf_close(hd_gguf *g);
const char *hd_gguf_error(void);
int hd_gguf_counts(const hd_gguf *g, uint32_t *version, int64_t *n_tensors, int64_t *n_kv,
                   uint64_t *alignment);
/* Tensor i in file order; GgufLoader::get_tensor (loader.rs:112-114) by name. */
int hd_gguf_tensor(const hd_gguf *g, int64_t i, hd_gguf_tensor_info *out);
int hd_gguf_find_tensor(const hd_gguf *g, const char *name, int64_t *index);
/* Metadata entry i: key, value type (GGUFValueType), and for arrays the
 * element type and length (-1 and 0 otherwise). */
int hd_gguf_kv(const hd_gguf *g, int64_t i, const char **key, int32_t *type, int32_t *arr_type,
               uint64_t *arr_len);
int hd_gguf_find_key(const hd_gguf *g, const char *key, int64_t *index);
/* Scalar integers and bools as int64; floats (and integers) as double. */
int hd_gguf_kv_int(const hd_gguf *g, int64_t i, int64_t *out);
int hd_gguf_kv_float(const hd_gguf *g, int64_t i, double *out);
/* A string value (j = 0) or element j of a string array: pointer and length
 * (not NUL-terminated). */
int hd_gguf_kv_string(const hd_gguf *g, int64_t i, uint64_t j, const char **s, uint64_t *len);
/* A numeric array: pointer to its little-endian elements and their count (a
 * numeric scalar reads as an array of one, e.g. a u64 above INT64_MAX). */
int hd_gguf_kv_array(const hd_gguf *g, int64_t i, const void **data, uint64_t *n);
/* hd_weight_upload of the named 2-D Q8_0 / Q5_0 / Q4_K / Q6_K tensor
 * (rows = dims[1], cols = dims[0]). */
int hd_gguf_upload(hd_ctx *ctx, const hd_gguf *g, const char *name, hd_weight **out);

#ifdef __cplusplus
}
#endif
#endif /* HACEDLE_CUDA_H */
