"""Python binding of libhacedle_cuda.so (ctypes over the C ABI in include/hacedle_cuda.h).

Device buffers are torch tensors; their data pointers cross the C ABI as
plain addresses.  There is no CPU fallback: every call goes to the CUDA
library, and loading fails loudly when the library is missing.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import synth  # noqa: F401

_PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(_PKG, "..", ".."))
LIB_PATH = os.path.join(ROOT, "lib", "libhacedle_cuda.so")

HD_OK, HD_E_ARG, HD_E_SHAPE, HD_E_TYPE, HD_E_CUDA, HD_E_TIMEOUT, HD_E_NCCL, HD_E_OOM, HD_E_UNSUPPORTED = range(9)
TYPE_Q5_0, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K = 6, 8, 12, 14
PREC_FP32, PREC_BF16_TC = 0, 1
CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy

# Every symbol include/hacedle_cuda.h declares.
EXPORTS = [
    "hd_ctx_create", "hd_ctx_destroy", "hd_ctx_set_stream", "hd_ctx_synchronize", "hd_ctx_reserve_workspace",
    "hd_last_error", "hd_ctx_launch_count", "hd_version", "hd_ctx_check_device_errors",
    "hd_weight_upload", "hd_weight_upload_device", "hd_weight_free", "hd_weight_info", "hd_weight_download",
    "hd_dequantize", "hd_qgemv", "hd_qgemv_swiglu", "hd_qgemv_rmsnorm", "hd_qgemv_host", "hd_qgemm", "hd_qgemm_host",
    "hd_qgemm_kt", "hd_qgemm_kt_host", "hd_matmul_f32",
    "hd_rmsnorm", "hd_rmsnorm_graph", "hd_rope_neox", "hd_rope_interleaved", "hd_softmax_rows", "hd_swiglu",
    "hd_add", "hd_argmax_rows", "hd_argmax_rows_noalloc", "hd_lm_head_argmax", "hd_embed", "hd_kv_append", "hd_attention_decode", "hd_attention_prefill",
    "hd_dot_i8", "hd_fused_qdot_qadd_qacc_i8", "hd_gather_columns", "hd_decoder_create", "hd_decoder_free", "hd_decoder_generate",
    "hd_decoder_generate_ex", "hd_gguf_open", "hd_gguf_open_memory", "hd_gguf_close", "hd_gguf_error", "hd_gguf_counts", "hd_gguf_tensor",
    "hd_gguf_find_tensor", "hd_gguf_kv", "hd_gguf_find_key", "hd_gguf_kv_int", "hd_gguf_kv_float", "hd_gguf_kv_string",
    "hd_gguf_kv_array", "hd_gguf_upload", "hd_logits_process", "hd_sample_rows",
    "hd_xbuf_alloc", "hd_xbuf_free", "hd_ipc_handle", "hd_ipc_open", "hd_ipc_close", "hd_push_columns", "hd_push_columns_multi",
    "hd_kv_arena_create", "hd_kv_arena_free", "hd_kv_layer", "hd_kv_allocate", "hd_kv_release", "hd_kv_session",
    "hd_kv_advance", "hd_kv_soul_sessions", "hd_kv_snapshot", "hd_kv_restore", "hd_kv_snapshot_free",
    "hd_kv_append_slots", "hd_attention_decode_slots", "hd_quantize_q8_1", "hd_qgemv_q8_1",
]


class HdError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"hacedle_cuda error {code}: {msg}")
        self.code = code


_lib = None
V, I, I64, SZ, F = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_float


def lib() -> C.CDLL:
    """Load the in-tree library (built by `make -C hace-fem-hacedle_b200`)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"libhacedle_cuda.so is missing at {LIB_PATH}; run __graft_entry__.build()")
    L = C.CDLL(LIB_PATH)
    sig = {
        "hd_ctx_create": [I, C.POINTER(V)], "hd_ctx_destroy": [V], "hd_ctx_set_stream": [V, V],
        "hd_ctx_synchronize": [V], "hd_ctx_reserve_workspace": [V, SZ], "hd_last_error": [V],
        "hd_ctx_launch_count": [V], "hd_version": [], "hd_ctx_check_device_errors": [V],
        "hd_weight_upload": [V, V, SZ, I, I64, I64, C.POINTER(V)],
        "hd_weight_upload_device": [V, V, SZ, I, I64, I64, C.POINTER(V)],
        "hd_weight_free": [V, V],
        "hd_weight_info": [V, C.POINTER(I), C.POINTER(I64), C.POINTER(I64), C.POINTER(SZ)],
        "hd_weight_download": [V, V, V, SZ], "hd_dequantize": [V, V, V, SZ],
        "hd_qgemv": [V, V, V, V, I, V, V], "hd_qgemv_swiglu": [V, V, V, V, V, I], "hd_qgemv_host": [V, V, V, V, I],
        "hd_qgemv_rmsnorm": [V, V, V, V, V, F, V, I, V, V],
        "hd_qgemm": [V, V, V, V, I, I], "hd_qgemm_host": [V, V, V, V, I, I],
        "hd_qgemm_kt": [V, V, V, V, I, I], "hd_qgemm_kt_host": [V, V, V, V, I, I], "hd_matmul_f32": [V, V, V, V, I64, I64, I64],
        "hd_rmsnorm": [V, V, V, V, V, I64, I, F], "hd_rmsnorm_graph": [V, V, V, V, I64, I, F],
        "hd_rope_neox": [V, V, V, I, I, I, F], "hd_rope_interleaved": [V, V, V, V, V, I64, I],
        "hd_softmax_rows": [V, V, I64, I], "hd_swiglu": [V, V, V, V, I64], "hd_add": [V, V, V, V, I64],
        "hd_argmax_rows": [V, V, I64, I64, V], "hd_embed": [V, V, V, I, V],
        "hd_argmax_rows_noalloc": [V, I64, I64, V, V],
        "hd_lm_head_argmax": [V, V, V, V, F, V, V, I],
        "hd_gather_columns": [V, V, V, I, I, I64],
        "hd_xbuf_alloc": [V, SZ, C.POINTER(V)], "hd_xbuf_free": [V, V], "hd_ipc_handle": [V, V, V],
        "hd_ipc_open": [V, V, C.POINTER(V)], "hd_ipc_close": [V, V],
        "hd_push_columns": [V, V, V, V, I, I, I, I64, I],
        "hd_push_columns_multi": [V, I, V, V, V, V, I, I, I, I],
        "hd_kv_append": [V, V, V, V, V, V, I, I, I, I, I],
        "hd_attention_decode": [V, V, V, V, V, I, I, I, I, I, V],
        "hd_attention_prefill": [V, V, V, V, I, I, I, I, I, I, V],
        "hd_dot_i8": [V, V, V, I64, I, V], "hd_fused_qdot_qadd_qacc_i8": [V, V, V, I64, I, V, V, V],
        "hd_decoder_create": [V, V, V, V, V, C.POINTER(V)], "hd_decoder_free": [V],
        "hd_decoder_generate": [V, V, I, I, I, I, V, V, V],
        "hd_decoder_generate_ex": [V, V, I, I, I, I, V, V, V, V, V],
        "hd_gguf_open": [C.c_char_p, C.POINTER(V)], "hd_gguf_open_memory": [V, SZ, C.POINTER(V)], "hd_gguf_close": [V],
        "hd_gguf_error": [], "hd_gguf_counts": [V, V, V, V, V], "hd_gguf_tensor": [V, I64, V],
        "hd_gguf_find_tensor": [V, C.c_char_p, V], "hd_gguf_kv": [V, I64, V, V, V, V],
        "hd_gguf_find_key": [V, C.c_char_p, V], "hd_gguf_kv_int": [V, I64, V], "hd_gguf_kv_float": [V, I64, V],
        "hd_gguf_kv_string": [V, I64, C.c_uint64, V, V], "hd_gguf_kv_array": [V, I64, V, V],
        "hd_gguf_upload": [V, V, C.c_char_p, C.POINTER(V)],
        "hd_logits_process": [V, V, I64, I64, F, F, I64], "hd_sample_rows": [V, V, I64, I64, C.c_uint64, C.c_uint64, V],
        "hd_kv_arena_create": [V, I, I, I, I, I, C.POINTER(V)], "hd_kv_arena_free": [V], "hd_kv_layer": [V, I, V, V],
        "hd_kv_allocate": [V, C.c_char_p, C.c_char_p, V], "hd_kv_release": [V, C.c_char_p],
        "hd_kv_session": [V, C.c_char_p, V, V], "hd_kv_advance": [V, C.c_char_p, I],
        "hd_kv_soul_sessions": [V, C.c_char_p, V], "hd_kv_snapshot": [V, C.c_char_p, V],
        "hd_kv_restore": [V, V, C.c_char_p], "hd_kv_snapshot_free": [V, V],
        "hd_kv_append_slots": [V, V, V, V, V, V, V, I, I, I, I],
        "hd_attention_decode_slots": [V, V, V, V, V, V, I, I, I, I, I, V],
        "hd_quantize_q8_1": [V, V, I, I64, V], "hd_qgemv_q8_1": [V, V, V, V, I],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = I
    L.hd_last_error.restype = C.c_char_p
    L.hd_gguf_error.restype = C.c_char_p
    L.hd_version.restype = C.c_char_p
    L.hd_ctx_launch_count.restype = C.c_uint64
    _lib = L
    return L


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t.ctypes.data
    return t.data_ptr()


class Weight:
    """Device weight handle (hd_weight): GGUF bytes uploaded once."""

    def __init__(self, ctx: "Context", ggml_type: int, raw: np.ndarray, rows: int, cols: int):
        raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
        self.ctx, self.type, self.rows, self.cols, self.nbytes = ctx, ggml_type, rows, cols, raw.size
        h = V()
        ctx._check(lib().hd_weight_upload(ctx.h, raw.ctypes.data, raw.size, ggml_type, rows, cols, C.byref(h)))
        self.h = h

    @classmethod
    def from_handle(cls, ctx: "Context", h, ggml_type: int, rows: int, cols: int, nbytes: int) -> "Weight":
        """Wrap a handle the library made (hd_gguf_upload)."""
        w = cls.__new__(cls)
        w.ctx, w.type, w.rows, w.cols, w.nbytes, w.h = ctx, ggml_type, rows, cols, nbytes, h
        return w

    def download(self) -> np.ndarray:
        out = np.zeros(self.nbytes, np.uint8)
        self.ctx._check(lib().hd_weight_download(self.ctx.h, self.h, out.ctypes.data, out.size))
        return out

    def free(self):
        # after the context is closed its device memory is gone with it
        if self.h and getattr(self.ctx, "h", None):
            lib().hd_weight_free(self.ctx.h, self.h)
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Context:
    """One hd_ctx on `device`; work goes on torch's current stream."""

    def __init__(self, device: int = 0, use_torch_stream: bool = True):
        import torch

        h = V()
        rc = lib().hd_ctx_create(device, C.byref(h))
        if rc != HD_OK:
            raise HdError(rc, f"hd_ctx_create({device}) failed")
        self.h = h
        self.device = device
        if use_torch_stream:
            self.set_stream(torch.cuda.current_stream(device).cuda_stream)

    def set_stream(self, stream: int | None):
        """Enqueue on `stream` (a cudaStream_t as int).  Handle 0, torch's
        default stream, is the legacy default stream: it is passed as
        cudaStreamLegacy (1), because NULL selects the context's own stream."""
        self._check(lib().hd_ctx_set_stream(self.h, stream if stream else CUDA_STREAM_LEGACY))

    def _check(self, rc: int):
        if rc != HD_OK:
            raise HdError(rc, lib().hd_last_error(self.h).decode())

    def last_error(self) -> str:
        return lib().hd_last_error(self.h).decode()

    @property
    def launches(self) -> int:
        return int(lib().hd_ctx_launch_count(self.h))

    def synchronize(self):
        self._check(lib().hd_ctx_synchronize(self.h))

    def check_device_errors(self):
        self._check(lib().hd_ctx_check_device_errors(self.h))

    def reserve_workspace(self, nbytes: int):
        self._check(lib().hd_ctx_reserve_workspace(self.h, nbytes))

    def weight(self, ggml_type: int, raw, rows: int, cols: int) -> Weight:
        return Weight(self, ggml_type, raw, rows, cols)

    # ---- kernels (device tensors) ----
    def quantize_q8_1(self, x, blocks):
        """x [B, K] f32 -> blocks (uint8 device tensor of B*K/32*48 bytes)."""
        B, K = x.shape
        self._check(lib().hd_quantize_q8_1(self.h, _ptr(x), B, K, _ptr(blocks)))

    def qgemv_q8_1(self, w: Weight, blocks, y, B: int):
        self._check(lib().hd_qgemv_q8_1(self.h, w.h, _ptr(blocks), _ptr(y), B))

    def logits_process(self, logits, temperature: float, top_p: float, top_k: int):
        """LogitsProcessor::process in place on a [rows, n] device tensor."""
        rows, n = (1, logits.numel()) if logits.dim() == 1 else logits.shape
        self._check(lib().hd_logits_process(self.h, _ptr(logits), rows, n, temperature, top_p, top_k))

    def sample(self, logits, idx, seed: int, offset: int = 0):
        """One index per row of [rows, n] logits into int32 idx[rows]."""
        rows, n = (1, logits.numel()) if logits.dim() == 1 else logits.shape
        self._check(lib().hd_sample_rows(self.h, _ptr(logits), rows, n, seed, offset, _ptr(idx)))

    def dequantize(self, w: Weight, out):
        self._check(lib().hd_dequantize(self.h, w.h, _ptr(out), out.numel()))

    def qgemv(self, w: Weight, x, y, bias=None, residual=None):
        B = x.shape[0] if x.dim() == 2 else 1
        self._check(lib().hd_qgemv(self.h, w.h, _ptr(x), _ptr(y), B, _ptr(bias), _ptr(residual)))

    def qgemv_swiglu(self, wg: Weight, wu: Weight, x, y):
        B = x.shape[0] if x.dim() == 2 else 1
        self._check(lib().hd_qgemv_swiglu(self.h, wg.h, wu.h, _ptr(x), _ptr(y), B))

    def qgemv_norm(self, w: Weight, x, norm_w, y, eps: float = 1e-6, w_up: Weight | None = None, bias=None,
                   residual=None):
        B = x.shape[0] if x.dim() == 2 else 1
        self._check(lib().hd_qgemv_rmsnorm(self.h, w.h, w_up.h if w_up else None, _ptr(x), _ptr(norm_w), eps,
                                           _ptr(y), B, _ptr(bias), _ptr(residual)))

    def qgemv_host(self, w: Weight, x: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        """Host x [B][cols] -> host y [B][rows]; `out` (float32, C-contiguous,
        e.g. a pinned buffer) receives y when given."""
        x = np.ascontiguousarray(x, np.float32).reshape(-1, w.cols)
        if out is None:
            out = np.zeros((x.shape[0], w.rows), np.float32)
        elif out.dtype != np.float32 or not out.flags.c_contiguous or out.size != x.shape[0] * w.rows:
            raise ValueError("out must be a C-contiguous float32 array of B x rows")
        self._check(lib().hd_qgemv_host(self.h, w.h, x.ctypes.data, out.ctypes.data, x.shape[0]))
        return out

    def qgemm(self, w: Weight, X, Y, precision: int = PREC_FP32):
        self._check(lib().hd_qgemm(self.h, w.h, _ptr(X), _ptr(Y), X.shape[0], precision))

    def qgemm_host(self, w: Weight, X: np.ndarray, precision: int = PREC_FP32) -> np.ndarray:
        X = np.ascontiguousarray(X, np.float32).reshape(-1, w.cols)
        Y = np.zeros((X.shape[0], w.rows), np.float32)
        self._check(lib().hd_qgemm_host(self.h, w.h, X.ctypes.data, Y.ctypes.data, X.shape[0], precision))
        return Y

    def qgemm_kt(self, w: Weight, X_kt, Y_nt, precision: int = PREC_FP32):
        """Y_nt [N][T] = W X_kt for X_kt [K][T] (ComputeBackend::matmul_q4k's layout)."""
        self._check(lib().hd_qgemm_kt(self.h, w.h, _ptr(X_kt), _ptr(Y_nt), X_kt.shape[1], precision))

    def qgemm_kt_host(self, w: Weight, X_kt: np.ndarray, precision: int = PREC_FP32) -> np.ndarray:
        X_kt = np.ascontiguousarray(X_kt, np.float32).reshape(w.cols, -1)
        Y = np.zeros((w.rows, X_kt.shape[1]), np.float32)
        self._check(lib().hd_qgemm_kt_host(self.h, w.h, X_kt.ctypes.data, Y.ctypes.data, X_kt.shape[1], precision))
        return Y

    def matmul_f32(self, a, b, out):
        self._check(lib().hd_matmul_f32(self.h, _ptr(a), _ptr(b), _ptr(out), a.shape[0], b.shape[1], a.shape[1]))

    def rmsnorm(self, x, w, y, eps: float = 1e-6, residual=None):
        dim = w.numel()
        self._check(lib().hd_rmsnorm(self.h, _ptr(x), _ptr(w), _ptr(residual), _ptr(y), x.numel() // dim, dim, eps))

    def rmsnorm_graph(self, x, w, y, eps: float = 1e-5):
        dim = w.numel()
        self._check(lib().hd_rmsnorm_graph(self.h, _ptr(x), _ptr(w), _ptr(y), x.numel() // dim, dim, eps))

    def rope_neox(self, x, pos, heads: int, head_dim: int, theta: float = 1e6):
        self._check(lib().hd_rope_neox(self.h, _ptr(x), _ptr(pos), pos.numel(), heads, head_dim, theta))

    def rope_interleaved(self, x, cos, sin, out):
        last = x.shape[-1]
        self._check(lib().hd_rope_interleaved(self.h, _ptr(x), _ptr(cos), _ptr(sin), _ptr(out), x.numel() // last,
                                              last))

    def softmax_rows(self, x):
        n = x.shape[-1]
        self._check(lib().hd_softmax_rows(self.h, _ptr(x), x.numel() // n, n))

    def swiglu(self, g, u, y):
        self._check(lib().hd_swiglu(self.h, _ptr(g), _ptr(u), _ptr(y), g.numel()))

    def add(self, a, b, y):
        self._check(lib().hd_add(self.h, _ptr(a), _ptr(b), _ptr(y), a.numel()))

    def lm_head_argmax(self, w: Weight, x, logits, idx, norm_w=None, eps: float = 1e-6):
        """logits = W rmsnorm(x) (W x without norm_w), idx = greedy id per row."""
        B = x.shape[0] if x.dim() == 2 else 1
        self._check(lib().hd_lm_head_argmax(self.h, w.h, _ptr(x), _ptr(norm_w), eps, _ptr(logits), _ptr(idx), B))

    def argmax_rows(self, x, idx):
        n = x.shape[-1]
        rows = x.numel() // n if n else idx.numel()
        self._check(lib().hd_argmax_rows(self.h, _ptr(x), rows, n, _ptr(idx)))

    def gather_columns(self, src, dst, G: int, B: int, n: int):
        self._check(lib().hd_gather_columns(self.h, _ptr(src), _ptr(dst), G, B, n))

    def embed(self, table: Weight, ids, out):
        self._check(lib().hd_embed(self.h, table.h, _ptr(ids), ids.numel(), _ptr(out)))

    def kv_append(self, k, v, kc, vc, pos0, seqs, tokens, n_kv, head_dim, max_ctx):
        self._check(lib().hd_kv_append(self.h, _ptr(k), _ptr(v), _ptr(kc), _ptr(vc), _ptr(pos0), seqs, tokens, n_kv,
                                       head_dim, max_ctx))

    def attention_decode(self, q, kc, vc, lens, n_heads, n_kv, head_dim, max_ctx, out):
        self._check(lib().hd_attention_decode(self.h, _ptr(q), _ptr(kc), _ptr(vc), _ptr(lens), lens.numel(), n_heads,
                                              n_kv, head_dim, max_ctx, _ptr(out)))

    def attention_prefill(self, q, kc, vc, T, pos0, n_heads, n_kv, head_dim, max_ctx, out):
        self._check(lib().hd_attention_prefill(self.h, _ptr(q), _ptr(kc), _ptr(vc), T, pos0, n_heads, n_kv, head_dim,
                                               max_ctx, _ptr(out)))

    def dot_i8(self, a, b, out):
        n = a.shape[-1]
        self._check(lib().hd_dot_i8(self.h, _ptr(a), _ptr(b), n, a.numel() // n if n else out.numel(), _ptr(out)))

    def fused_qdot_qadd_qacc_i8(self, a, b, bias, carry, out):
        n = a.shape[-1]
        self._check(lib().hd_fused_qdot_qadd_qacc_i8(self.h, _ptr(a), _ptr(b), n, out.numel(), _ptr(bias),
                                                     _ptr(carry), _ptr(out)))

    def close(self):
        if getattr(self, "h", None):
            lib().hd_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _DecCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "n_layers", "n_heads", "n_kv", "head_dim", "ffn", "vocab", "max_ctx",
                                        "max_seqs")] + [("eps", C.c_float), ("theta", C.c_float)]


class _LayerW(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd", "bq", "bk", "bv", "attn_norm",
                                           "ffn_norm")]


class KvSnapshot(C.Structure):
    """hd_kv_snapshot_t (KvSnapshot)."""
    _fields_ = [("snapshot_id", C.c_uint64), ("token_position", C.c_int32), ("slot", C.c_int32),
                ("kv_offset", C.c_uint64), ("timestamp", C.c_uint64)]


class KvArena:
    """hd_kv_arena: the device KV-cache manager (KvCacheManager over a pool of
    `slots` KV slots, K and V [layers][slots][max_ctx][n_kv][head_dim] f32)."""

    def __init__(self, ctx: "Context", layers: int, n_kv: int, head_dim: int, max_ctx: int, slots: int):
        self.ctx, self.layers, self.n_kv, self.head_dim, self.max_ctx, self.slots = \
            ctx, layers, n_kv, head_dim, max_ctx, slots
        h = V()
        ctx._check(lib().hd_kv_arena_create(ctx.h, layers, n_kv, head_dim, max_ctx, slots, C.byref(h)))
        self.h = h

    def layer(self, li: int):
        """(k, v) device addresses of layer li's [slots][max_ctx][n_kv][head_dim] blocks."""
        k, v = V(), V()
        self.ctx._check(lib().hd_kv_layer(self.h, li, C.byref(k), C.byref(v)))
        return k.value, v.value

    def allocate(self, session: str, soul: str) -> int:
        s = C.c_int()
        self.ctx._check(lib().hd_kv_allocate(self.h, session.encode(), soul.encode(), C.byref(s)))
        return s.value

    def release(self, session: str):
        self.ctx._check(lib().hd_kv_release(self.h, session.encode()))

    def session(self, session: str):
        """(slot, position)."""
        s, p = C.c_int(), C.c_int()
        self.ctx._check(lib().hd_kv_session(self.h, session.encode(), C.byref(s), C.byref(p)))
        return s.value, p.value

    def advance(self, session: str, count: int):
        self.ctx._check(lib().hd_kv_advance(self.h, session.encode(), count))

    def soul_sessions(self, soul: str) -> int:
        n = C.c_int()
        self.ctx._check(lib().hd_kv_soul_sessions(self.h, soul.encode(), C.byref(n)))
        return n.value

    def snapshot(self, session: str) -> KvSnapshot:
        s = KvSnapshot()
        self.ctx._check(lib().hd_kv_snapshot(self.h, session.encode(), C.byref(s)))
        return s

    def restore(self, snap: KvSnapshot, session: str):
        self.ctx._check(lib().hd_kv_restore(self.h, C.byref(snap), session.encode()))

    def snapshot_free(self, snap: KvSnapshot):
        self.ctx._check(lib().hd_kv_snapshot_free(self.h, C.byref(snap)))

    def append(self, li: int, k, v, slots, pos):
        """Rows of k, v [rows, n_kv * head_dim] into layer li at (slots[r], pos[r])."""
        kc, vc = self.layer(li)
        self.ctx._check(lib().hd_kv_append_slots(self.ctx.h, _ptr(k), _ptr(v), kc, vc, _ptr(slots), _ptr(pos),
                                                 k.shape[0], self.n_kv, self.head_dim, self.max_ctx))

    def attention(self, li: int, q, slots, lens, n_heads: int, out):
        kc, vc = self.layer(li)
        self.ctx._check(lib().hd_attention_decode_slots(self.ctx.h, _ptr(q), kc, vc, _ptr(slots), _ptr(lens),
                                                        q.shape[0], n_heads, self.n_kv, self.head_dim, self.max_ctx,
                                                        _ptr(out)))

    def free(self):
        if getattr(self, "h", None) and getattr(self.ctx, "h", None):
            lib().hd_kv_arena_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Decoder:
    """hd_decoder: the Qwen2-shaped decoder on the device.

    `model` is synth.gen_decoder()'s dict: cfg, layers (each weight a tuple
    (ggml_type, raw bytes, rows, cols) plus f32 bias / norm vectors), out_norm,
    embed.  Weights are uploaded once."""

    def __init__(self, ctx: Context, model: dict, max_ctx: int, max_seqs: int = 1):
        cfg = model["cfg"]
        self.ctx, self.cfg = ctx, cfg
        self.weights, self._keep = [], []
        arr = (_LayerW * cfg["n_layers"])()
        for i, L in enumerate(model["layers"]):
            for name in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
                t, raw, n, k = L[name]
                w = ctx.weight(t, raw, n, k)
                self.weights.append(w)
                setattr(arr[i], name, w.h)
            for name in ("bq", "bk", "bv", "attn_norm", "ffn_norm"):
                a = np.ascontiguousarray(L[name], np.float32)
                self._keep.append(a)
                setattr(arr[i], name, a.ctypes.data)
        t, raw, n, k = model["embed"]
        self.embed = ctx.weight(t, raw, n, k)
        on = np.ascontiguousarray(model["out_norm"], np.float32)
        c = _DecCfg(cfg["hidden"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv"], cfg["head_dim"], cfg["ffn"],
                    cfg["vocab"], max_ctx, max_seqs, cfg["eps"], cfg["theta"])
        h = V()
        ctx._check(lib().hd_decoder_create(ctx.h, C.byref(c), arr, on.ctypes.data, self.embed.h, C.byref(h)))
        self.h = h
        self._keep.clear()

    def generate(self, prompts: np.ndarray, n_gen: int, precision: int = PREC_FP32):
        """prompts [seqs, n_prompt] int32 -> (tokens [seqs, n_gen], decode_ms, prefill_ms)."""
        p = np.ascontiguousarray(prompts, np.int32)
        if p.ndim == 1:
            p = p[None]
        out = np.zeros((p.shape[0], n_gen), np.int32)
        dm, pm = C.c_float(), C.c_float()
        self.ctx._check(lib().hd_decoder_generate(self.h, p.ctypes.data, p.shape[0], p.shape[1], n_gen, precision,
                                                  out.ctypes.data, C.byref(dm), C.byref(pm)))
        return out, dm.value, pm.value

    def generate_forced(self, prompts: np.ndarray, forced: np.ndarray | None, n_gen: int,
                        precision: int = PREC_FP32):
        """Teacher-forced decode (hd_decoder_generate_ex): the input of step g
        >= 1 is forced[s, g - 1] (forced None: the greedy ids, as generate).
        Returns (greedy ids [seqs, n_gen], logits [n_gen, seqs, vocab],
        decode_ms, prefill_ms)."""
        p = np.ascontiguousarray(prompts, np.int32)
        if p.ndim == 1:
            p = p[None]
        f = None if forced is None else np.ascontiguousarray(forced, np.int32).reshape(p.shape[0], n_gen)
        out = np.zeros((p.shape[0], n_gen), np.int32)
        logits = np.zeros((n_gen, p.shape[0], self.cfg["vocab"]), np.float32)
        dm, pm = C.c_float(), C.c_float()
        self.ctx._check(lib().hd_decoder_generate_ex(self.h, p.ctypes.data, p.shape[0], p.shape[1], n_gen, precision,
                                                     None if f is None else f.ctypes.data, out.ctypes.data,
                                                     logits.ctypes.data, C.byref(dm), C.byref(pm)))
        return out, logits, dm.value, pm.value

    def free(self):
        if getattr(self, "h", None) and getattr(self.ctx, "h", None):
            lib().hd_decoder_free(self.h)
        self.h = None
        for w in self.weights:
            w.free()
        self.weights = []
        if getattr(self, "embed", None):
            self.embed.free()
            self.embed = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
