"""ctypes front end of the CPU oracle (oracle/hd_oracle.c).

TEST INFRASTRUCTURE ONLY: tests/, the smoke entry point and bench.py's
cpu_baseline / reference arm import this module as the checker.  The product
library (libhacedle_cuda.so) never imports, links or calls it.

Every function restates the reference's arithmetic; the C file names the
reference file:line each one follows.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")

GGML_F32, GGML_F16, GGML_Q5_0, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K, GGML_BF16 = 0, 1, 6, 8, 12, 14, 30
BLOCK = {GGML_Q8_0: (32, 34), GGML_Q5_0: (32, 22), GGML_Q4_K: (256, 144), GGML_Q6_K: (256, 210),
         GGML_F16: (1, 2), GGML_BF16: (1, 2), GGML_F32: (1, 4)}

_f32p = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_i8p = C.POINTER(C.c_int8)
_i32p = C.POINTER(C.c_int32)


def build() -> str:
    """Compile the oracle with its Makefile (gcc, no FMA contraction)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        L.hdo_f16_to_f32.restype = C.c_float
        L.hdo_f16_to_f32.argtypes = [C.c_uint16]
        L.hdo_dequantize.restype = C.c_int
        L.hdo_dequantize.argtypes = [C.c_int, _u8p, C.c_size_t, _f32p, C.c_size_t]
        L.hdo_gemv_f32.argtypes = [_f32p, C.c_int64, C.c_int64, _f32p, C.c_int, _f32p, C.c_int]
        L.hdo_qgemv.restype = C.c_int
        L.hdo_qgemv.argtypes = [C.c_int, _u8p, C.c_size_t, C.c_int64, C.c_int64, _f32p, C.c_int, _f32p, C.c_int]
        L.hdo_matmul_vec_matrix.argtypes = [_f32p, _f32p, C.c_int64, C.c_int64, _f32p]
        L.hdo_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int64, C.c_int64, C.c_float]
        L.hdo_rmsnorm_graph.argtypes = [_f32p, _f32p, _f32p, C.c_int64, C.c_int64, C.c_float, C.c_int]
        L.hdo_rope_freqs.argtypes = [C.c_int, C.c_float, _f32p]
        L.hdo_rope_neox.argtypes = [_f32p, C.c_int64, C.c_int, C.c_int, _i32p, C.c_float]
        L.hdo_rope_interleaved.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int64, C.c_int64]
        L.hdo_softmax.argtypes = [_f32p, C.c_int64]
        L.hdo_silu.argtypes = [_f32p, _f32p, C.c_int64]
        L.hdo_swiglu.argtypes = [_f32p, _f32p, _f32p, C.c_int64]
        L.hdo_add_f32.argtypes = [_f32p, _f32p, _f32p, C.c_int64]
        L.hdo_matmul_f32.argtypes = [_f32p, _f32p, _f32p, C.c_int64, C.c_int64, C.c_int64]
        L.hdo_argmax.restype = C.c_uint32
        L.hdo_argmax.argtypes = [_f32p, C.c_int64]
        L.hdo_embedding_lookup.argtypes = [C.c_uint32, _f32p, C.c_int64, C.c_int64, C.c_int64, _f32p]
        L.hdo_attention_decode.argtypes = [_f32p, _f32p, _f32p, C.c_int64, C.c_int, C.c_int, C.c_int,
                                           _f32p, _f32p]
        L.hdo_dot_i8.restype = C.c_int32
        L.hdo_dot_i8.argtypes = [_i8p, _i8p, C.c_int64]
        L.hdo_fused_qdot_qadd_qacc_i8.restype = C.c_int32
        L.hdo_fused_qdot_qadd_qacc_i8.argtypes = [_i8p, _i8p, C.c_int64, C.c_int32, _i32p]
        L.hdo_quantize_q8_1.argtypes = [_f32p, C.c_int64, _i8p, _f32p, _i32p]
        L.hdo_qgemv_q8_1.restype = C.c_int
        L.hdo_qgemv_q8_1.argtypes = [C.c_int, _u8p, C.c_int64, C.c_int64, _i8p, _f32p, _i32p, C.c_int, _f32p]
        for fn in (L.hdo_decoder_generate, L.hdo_decoder_generate_all):
            fn.restype = C.c_int
            fn.argtypes = [C.c_void_p, C.c_void_p, _f32p, _f32p, _i32p, C.c_int, C.c_int, _i32p, _f32p, C.c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def f16_to_f32(h: int) -> float:
    return lib().hdo_f16_to_f32(h)


def dequantize(ggml_type: int, raw, n: int) -> np.ndarray:
    """QuantTensorView::dequantize (q4k_tensor_view.rs:63-114) with IEEE f16 scales."""
    raw = np.ascontiguousarray(np.frombuffer(bytes(raw), np.uint8) if isinstance(raw, (bytes, bytearray))
                               else raw, dtype=np.uint8).reshape(-1)
    out = np.zeros(n, np.float32)
    rc = lib().hdo_dequantize(ggml_type, _p(raw, _u8p), raw.size, _p(out, _f32p), n)
    if rc != 0:
        raise ValueError(f"oracle: unsupported ggml type {ggml_type}")
    return out


def gemv_f32(W: np.ndarray, X: np.ndarray, threads: int = 1) -> np.ndarray:
    """Y[b] = W @ X[b] with each row summed sequentially (core/tensor_ops/matmul.rs:4-21)."""
    W = _f32(W)
    X = _f32(X).reshape(-1, W.shape[1])
    Y = np.zeros((X.shape[0], W.shape[0]), np.float32)
    lib().hdo_gemv_f32(_p(W, _f32p), W.shape[0], W.shape[1], _p(X, _f32p), X.shape[0], _p(Y, _f32p), threads)
    return Y


def qgemv(ggml_type: int, raw: np.ndarray, N: int, K: int, X: np.ndarray, threads: int = 1) -> np.ndarray:
    """The reference's path: whole-tensor dequantize, then sequential GEMV per batch row."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    X = _f32(X).reshape(-1, K)
    Y = np.zeros((X.shape[0], N), np.float32)
    rc = lib().hdo_qgemv(ggml_type, _p(raw, _u8p), raw.size, N, K, _p(X, _f32p), X.shape[0], _p(Y, _f32p),
                         threads)
    if rc != 0:
        raise ValueError("oracle: qgemv failed")
    return Y


def matmul_vec_matrix(x, W, out_dim: int, in_dim: int) -> np.ndarray:
    x, W = _f32(x), _f32(W)
    y = np.zeros(out_dim, np.float32)
    lib().hdo_matmul_vec_matrix(_p(x, _f32p), _p(W, _f32p), out_dim, in_dim, _p(y, _f32p))
    return y


def rmsnorm(x, w, eps: float = 1e-6) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    y = np.zeros_like(x)
    dim = w.size
    lib().hdo_rmsnorm(_p(x, _f32p), _p(w, _f32p), _p(y, _f32p), x.size // dim, dim, eps)
    return y


def rmsnorm_graph(x, w, eps: float = 1e-5, newton: bool = False) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    y = np.zeros_like(x)
    dim = w.size
    lib().hdo_rmsnorm_graph(_p(x, _f32p), _p(w, _f32p), _p(y, _f32p), x.size // dim, dim, eps, int(newton))
    return y


def rope_freqs(head_dim: int, theta: float = 1e6) -> np.ndarray:
    f = np.zeros(head_dim // 2, np.float32)
    lib().hdo_rope_freqs(head_dim, theta, _p(f, _f32p))
    return f


def rope_neox(x, pos, head_dim: int, theta: float = 1e6) -> np.ndarray:
    """x [tokens, heads*head_dim]; pos [tokens]; returns a rotated copy."""
    x = _f32(x).copy()
    pos = np.ascontiguousarray(pos, dtype=np.int32).reshape(-1)
    T = pos.size
    heads = x.size // (T * head_dim)
    lib().hdo_rope_neox(_p(x, _f32p), T, heads, head_dim, _p(pos, _i32p), theta)
    return x


def rope_interleaved(x, cos, sin) -> np.ndarray:
    x, cos, sin = _f32(x), _f32(cos), _f32(sin)
    out = np.zeros_like(x)
    last = x.shape[-1]
    lib().hdo_rope_interleaved(_p(x, _f32p), _p(cos, _f32p), _p(sin, _f32p), _p(out, _f32p), x.size // last, last)
    return out


def softmax(x) -> np.ndarray:
    x = _f32(x).copy()
    lib().hdo_softmax(_p(x, _f32p), x.size)
    return x


def silu(x) -> np.ndarray:
    x = _f32(x)
    y = np.zeros_like(x)
    lib().hdo_silu(_p(x, _f32p), _p(y, _f32p), x.size)
    return y


def swiglu(g, u) -> np.ndarray:
    g, u = _f32(g), _f32(u)
    y = np.zeros_like(g)
    lib().hdo_swiglu(_p(g, _f32p), _p(u, _f32p), _p(y, _f32p), g.size)
    return y


def add_f32(a, b) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    y = np.zeros_like(a)
    lib().hdo_add_f32(_p(a, _f32p), _p(b, _f32p), _p(y, _f32p), a.size)
    return y


def matmul_f32(a, b) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    n = b.shape[1]
    out = np.zeros((m, n), np.float32)
    lib().hdo_matmul_f32(_p(a, _f32p), _p(b, _f32p), _p(out, _f32p), m, n, k)
    return out


def argmax(x) -> int:
    x = _f32(x)
    return int(lib().hdo_argmax(_p(x, _f32p), x.size))


def embedding_lookup(token: int, table, vocab: int, hidden: int) -> np.ndarray:
    table = _f32(table)
    out = np.zeros(hidden, np.float32)
    lib().hdo_embedding_lookup(token, _p(table, _f32p), table.size, vocab, hidden, _p(out, _f32p))
    return out


def attention_decode(q, kcache, vcache, n_heads: int, n_kv: int, head_dim: int) -> np.ndarray:
    """q [n_heads*hd]; caches [len, n_kv, hd]."""
    q, kc, vc = _f32(q), _f32(kcache), _f32(vcache)
    L = kc.size // (n_kv * head_dim)
    out = np.zeros(n_heads * head_dim, np.float32)
    scratch = np.zeros(max(L, 1), np.float32)
    lib().hdo_attention_decode(_p(q, _f32p), _p(kc, _f32p), _p(vc, _f32p), L, n_heads, n_kv, head_dim,
                               _p(out, _f32p), _p(scratch, _f32p))
    return out


def dot_i8(a, b) -> int:
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    return int(lib().hdo_dot_i8(_p(a, _i8p), _p(b, _i8p), min(a.size, b.size)))


def fused_qdot_qadd_qacc_i8(a, b, bias: int, carry: int):
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    c = C.c_int32(carry)
    out = lib().hdo_fused_qdot_qadd_qacc_i8(_p(a, _i8p), _p(b, _i8p), min(a.size, b.size), bias, C.byref(c))
    return int(out), int(c.value)


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "n_layers", "n_heads", "n_kv", "head_dim", "ffn", "vocab",
                                        "max_ctx")] + [("eps", C.c_float), ("theta", C.c_float)]


class _Layer(C.Structure):
    _fields_ = [(n, _f32p) for n in ("attn_norm", "ffn_norm", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "wg",
                                      "wu", "wd")]


def decoder_generate(cfg: dict, layers: list, out_norm, embed, prompt, n_gen: int, threads: int = 8,
                     return_logits: bool = False, all_logits: bool = False):
    """Prefill `prompt` token by token, then greedy-decode `n_gen` ids.

    cfg: hidden, n_layers, n_heads, n_kv, head_dim, ffn, vocab, eps, theta.
    layers: list of dicts of f32 arrays (attn_norm, ffn_norm, wq, bq, wk, bk, wv, bv, wo, wg, wu, wd),
    already dequantized.  embed: f32 [vocab, hidden] (tied LM head).
    return_logits: also the logits that chose the last id; all_logits: also
    the logits of every step, [n_gen, vocab] (row g chose id g)."""
    prompt = np.ascontiguousarray(prompt, dtype=np.int32)
    c = _Cfg(cfg["hidden"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv"], cfg["head_dim"], cfg["ffn"],
             cfg["vocab"], prompt.size + n_gen, cfg["eps"], cfg["theta"])
    keep = []
    arr = (_Layer * len(layers))()
    for i, Lw in enumerate(layers):
        for name in _Layer._fields_:
            a = _f32(Lw[name[0]])
            keep.append(a)
            setattr(arr[i], name[0], _p(a, _f32p))
    on, em = _f32(out_norm), _f32(embed)
    out = np.zeros(n_gen, np.int32)
    if all_logits:
        logits = np.zeros((n_gen, cfg["vocab"]), np.float32)
        fn = lib().hdo_decoder_generate_all
    else:
        logits = np.zeros(cfg["vocab"], np.float32) if return_logits else None
        fn = lib().hdo_decoder_generate
    rc = fn(C.addressof(c), C.addressof(arr), _p(on, _f32p), _p(em, _f32p), _p(prompt, _i32p), prompt.size, n_gen,
            _p(out, _i32p), _p(logits, _f32p) if logits is not None else None, threads)
    if rc != 0:
        raise RuntimeError("oracle: decoder_generate failed")
    return (out, logits) if (return_logits or all_logits) else out


def dequant_model(model: dict):
    """A synth.gen_decoder() model with every quantized weight dequantized
    (f32 [rows, cols]); returns (layers, out_norm, embed) for decoder_generate."""
    layers = []
    for L in model["layers"]:
        d = {k: L[k] for k in ("bq", "bk", "bv", "attn_norm", "ffn_norm")}
        for k in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
            t, raw, n, kk = L[k]
            d[k] = dequantize(t, raw, n * kk).reshape(n, kk)
        layers.append(d)
    t, raw, n, kk = model["embed"]
    return layers, model["out_norm"], dequantize(t, raw, n * kk).reshape(n, kk)


# ---------------------------------------------------------------- sampler
def logits_process(logits, temperature: float, top_p: float, top_k: int) -> np.ndarray:
    """LogitsProcessor::process (src/x/provider/candle/lmhead.rs:42-111) on each
    row of [rows, n] f32 logits, in the reference's order and arithmetic:
    apply_temperature (:55-60) l / max(t, 0.001); apply_top_p (:63-84) the
    descending-order sequential f32 sum of min(exp(l), 1) (f32 exp: numpy's,
    the reference's is the platform libm's) until it reaches top_p, whose logit
    is the threshold (0.0 if never reached); apply_top_k (:87-101) the
    (top_k+1)-th largest logit after top-p; logits below a threshold -> -inf."""
    x = np.array(logits, dtype=np.float32, copy=True)
    rows = x.reshape(1, -1) if x.ndim == 1 else x
    t = np.float32(max(np.float32(temperature), np.float32(0.001)))
    rows /= t
    for r in rows:
        s = np.sort(r)[::-1]
        with np.errstate(over="ignore"):                # exp overflows to inf, then min(., 1) = 1
            c = np.minimum(np.exp(s), np.float32(1.0)).astype(np.float32)
        cum = np.cumsum(c, dtype=np.float32)          # sequential f32 adds
        hit = np.nonzero(cum >= np.float32(top_p))[0]
        tp = s[hit[0]] if hit.size else np.float32(0.0)
        r[r < tp] = -np.inf
        if 0 < top_k < r.size:
            tk = np.sort(r)[::-1][top_k]
            r[r < tk] = -np.inf
    return x


_PHILOX_M = (0xD2511F53, 0xCD9E8D57)
_PHILOX_W = (0x9E3779B9, 0xBB67AE85)


def philox4x32_10(ctr, key) -> tuple:
    """Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11; the Random123 round:
    (hi(M1 c2) ^ c1 ^ k0, lo(M1 c2), hi(M0 c0) ^ c3 ^ k1, lo(M0 c0)), key
    bumped by the Weyl constants after each of 10 rounds)."""
    c = [int(v) & 0xFFFFFFFF for v in ctr]
    k = [int(v) & 0xFFFFFFFF for v in key]
    for _ in range(10):
        p0, p1 = _PHILOX_M[0] * c[0], _PHILOX_M[1] * c[2]
        c = [((p1 >> 32) ^ c[1] ^ k[0]) & 0xFFFFFFFF, p1 & 0xFFFFFFFF,
             ((p0 >> 32) ^ c[3] ^ k[1]) & 0xFFFFFFFF, p0 & 0xFFFFFFFF]
        k = [(k[0] + _PHILOX_W[0]) & 0xFFFFFFFF, (k[1] + _PHILOX_W[1]) & 0xFFFFFFFF]
    return tuple(c)


def sample_uniform(seed: int, ctr: int) -> np.float32:
    w = philox4x32_10((ctr & 0xFFFFFFFF, ctr >> 32, 0, 0), (seed & 0xFFFFFFFF, seed >> 32))[0]
    return np.float32(w >> 8) * np.float32(1.0 / 16777216.0)


def sample_rows(logits, seed: int, offset: int = 0, nt: int = 256):
    """The draw of hd_sample_rows in the same f32 operation order: chunk sums
    of exp(l - max) over nt contiguous chunks, their sequential exclusive
    prefix, target = u * total, the walk of the chunk that holds it.  Returns
    (indices, margins): margin = distance of the target to the nearest edge
    of the drawn entry's interval, relative to the total (where the platform
    exp's last-bit differences could move a draw)."""
    x = np.asarray(logits, np.float32)
    x = x.reshape(1, -1) if x.ndim == 1 else x
    n = x.shape[1]
    C_ = -(-n // nt)
    idx, margin = [], []
    for r, row in enumerate(x):
        m = row.max()
        if not np.isfinite(m):
            idx.append(-1)
            margin.append(np.inf)
            continue
        e = np.exp((row - m).astype(np.float32)).astype(np.float32)
        sums = np.zeros(nt, np.float32)
        for t in range(nt):
            ch = e[t * C_:min(n, (t + 1) * C_)]
            sums[t] = np.cumsum(ch, dtype=np.float32)[-1] if ch.size else np.float32(0)
        pre = np.concatenate([[np.float32(0)], np.cumsum(sums, dtype=np.float32)]).astype(np.float32)
        total = pre[-1]
        target = np.float32(sample_uniform(seed, offset + r) * total)
        if target >= total:
            t = max(j for j in range(nt) if sums[j] > 0)
        else:
            t = next(j for j in range(nt) if pre[j] <= target < pre[j + 1])
        ch = e[t * C_:min(n, (t + 1) * C_)]
        acc = np.cumsum(np.concatenate([[pre[t]], ch]).astype(np.float32), dtype=np.float32)[1:]
        pick, lo = -1, pre[t]
        for i in range(ch.size):
            if ch[i] > 0:
                pick = t * C_ + i
            if acc[i] > target and ch[i] > 0:
                break
            lo = acc[i]
        hi = acc[pick - t * C_] if pick >= 0 else lo
        idx.append(pick)
        margin.append(float(min(target - lo, hi - target)) / float(total))
    return np.array(idx, np.int32), np.array(margin)


# ---------------------------------------------------------------- Q8_1 path
def quantize_q8_1(X):
    """X [B, K] f32 -> (q int8 [B, K], d f32 [B, K/32], s int32 [B, K/32, 2])."""
    X = np.ascontiguousarray(X, np.float32)
    B, K = X.shape
    nb = B * (K // 32)
    q = np.zeros(B * K, np.int8)
    d = np.zeros(nb, np.float32)
    s = np.zeros(2 * nb, np.int32)
    lib().hdo_quantize_q8_1(_p(X, _f32p), nb, _p(q, _i8p), _p(d, _f32p), _p(s, _i32p))
    return q.reshape(B, K), d.reshape(B, K // 32), s.reshape(B, K // 32, 2)


def qgemv_q8_1(ggml_type: int, raw, N: int, K: int, q, d, s) -> np.ndarray:
    """Y [B, N] of the integer path over GGUF blocks and quantized activations."""
    raw = np.ascontiguousarray(raw, np.uint8)
    q, d, s = (np.ascontiguousarray(a) for a in (q, d, s))
    B = q.shape[0]
    y = np.zeros((B, N), np.float32)
    rc = lib().hdo_qgemv_q8_1(ggml_type, _p(raw, _u8p), N, K, _p(q, _i8p), _p(d, _f32p), _p(s, _i32p), B,
                              _p(y, _f32p))
    assert rc == 0
    return y
