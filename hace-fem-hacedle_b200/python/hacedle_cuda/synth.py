"""Seeded synthetic GGUF weights and activations for the benchmark workloads.

All inputs are synthetic (no model files exist on these machines).  Each
generator draws from numpy's PCG64 with the value distributions of the five
workloads (scales drawn in f32 then rounded to f16) and packs the draws into
the byte layout of ggml blocks, row-major with K contiguous: a weight
[N rows, K cols] is N rows of K/block_elems blocks.

Block layouts (bytes):
  Q8_0  34  = f16 d | int8 qs[32]
  Q5_0  22  = f16 d | u32 qh | qs[16]   (low nibbles = values 0..15, high = 16..31)
  Q4_K  144 = f16 d | f16 dmin | scales[12] (6-bit sc/m, get_scale_min_k4) | qs[128]
  Q6_K  210 = ql[128] | qh[64] | int8 scales[16] | f16 d
"""
from __future__ import annotations

import numpy as np

GGML_Q5_0, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K = 6, 8, 12, 14
BLOCK = {GGML_Q8_0: (32, 34), GGML_Q5_0: (32, 22), GGML_Q4_K: (256, 144), GGML_Q6_K: (256, 210)}
TYPE_NAME = {GGML_Q8_0: "Q8_0", GGML_Q5_0: "Q5_0", GGML_Q4_K: "Q4_K", GGML_Q6_K: "Q6_K"}
NAME_TYPE = {v: k for k, v in TYPE_NAME.items()}


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def _f16_bits(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float32).astype(np.float16).view(np.uint16)


def nbytes(ggml_type: int, N: int, K: int) -> int:
    be, bb = BLOCK[ggml_type]
    assert K % be == 0
    return N * (K // be) * bb


# --------------------------------------------------------------- packers
def pack_q8_0(d_bits: np.ndarray, q: np.ndarray) -> np.ndarray:
    nb = d_bits.size
    out = np.zeros((nb, 34), np.uint8)
    out[:, 0:2] = d_bits.astype(np.uint16).reshape(nb, 1).view(np.uint8)
    out[:, 2:34] = q.astype(np.int8).reshape(nb, 32).view(np.uint8)
    return out


def pack_q5_0(d_bits: np.ndarray, q: np.ndarray) -> np.ndarray:
    nb = d_bits.size
    q = q.astype(np.uint32).reshape(nb, 32)
    out = np.zeros((nb, 22), np.uint8)
    out[:, 0:2] = d_bits.astype(np.uint16).reshape(nb, 1).view(np.uint8)
    qh = ((q >> 4) & 1) << np.arange(32, dtype=np.uint32)
    out[:, 2:6] = qh.sum(axis=1, dtype=np.uint64).astype(np.uint32).reshape(nb, 1).view(np.uint8)
    out[:, 6:22] = ((q[:, :16] & 15) | ((q[:, 16:] & 15) << 4)).astype(np.uint8)
    return out


def pack_q4_k(d_bits, dmin_bits, sc, m, q) -> np.ndarray:
    nb = d_bits.size
    sc = sc.astype(np.uint8).reshape(nb, 8)
    m = m.astype(np.uint8).reshape(nb, 8)
    q = q.astype(np.uint8).reshape(nb, 4, 2, 32)
    out = np.zeros((nb, 144), np.uint8)
    out[:, 0:2] = d_bits.astype(np.uint16).reshape(nb, 1).view(np.uint8)
    out[:, 2:4] = dmin_bits.astype(np.uint16).reshape(nb, 1).view(np.uint8)
    s = np.zeros((nb, 12), np.uint8)
    s[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    s[:, 4:8] = (m[:, 0:4] & 63) | ((m[:, 4:8] >> 4) << 6)
    s[:, 8:12] = (sc[:, 4:8] & 15) | ((m[:, 4:8] & 15) << 4)
    out[:, 4:16] = s
    out[:, 16:144] = (q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(nb, 128)
    return out


def pack_q6_k(d_bits, sc, q) -> np.ndarray:
    nb = d_bits.size
    q = q.astype(np.uint8).reshape(nb, 2, 4, 32)  # [half, quarter, l]
    lo, hi = q & 15, q >> 4
    out = np.zeros((nb, 210), np.uint8)
    ql = np.zeros((nb, 2, 2, 32), np.uint8)       # [half, k&1, l]
    ql[:, :, 0, :] = lo[:, :, 0, :] | (lo[:, :, 2, :] << 4)
    ql[:, :, 1, :] = lo[:, :, 1, :] | (lo[:, :, 3, :] << 4)
    qh = hi[:, :, 0, :] | (hi[:, :, 1, :] << 2) | (hi[:, :, 2, :] << 4) | (hi[:, :, 3, :] << 6)
    out[:, 0:128] = ql.reshape(nb, 128)
    out[:, 128:192] = qh.reshape(nb, 64)
    out[:, 192:208] = sc.astype(np.int8).reshape(nb, 16).view(np.uint8)
    out[:, 208:210] = d_bits.astype(np.uint16).reshape(nb, 1).view(np.uint8)
    return out


# ------------------------------------------------------------ generators
def gen_weight(ggml_type: int, N: int, K: int, seed: int) -> np.ndarray:
    """Packed weight bytes, shape [N, K/block_elems*block_bytes] uint8."""
    be, bb = BLOCK[ggml_type]
    if K % be:
        raise ValueError(f"K={K} is not a multiple of the {TYPE_NAME[ggml_type]} block ({be})")
    nb = N * (K // be)
    g = rng(seed)
    if ggml_type == GGML_Q8_0:
        d = _f16_bits(g.uniform(0.002, 0.02, nb))
        q = g.integers(-127, 128, (nb, 32), dtype=np.int16)
        out = pack_q8_0(d, q)
    elif ggml_type == GGML_Q5_0:
        d = _f16_bits(g.uniform(0.002, 0.02, nb))
        q = g.integers(0, 32, (nb, 32), dtype=np.uint8)
        out = pack_q5_0(d, q)
    elif ggml_type == GGML_Q4_K:
        d = _f16_bits(g.uniform(1e-4, 1e-3, nb))
        dmin = _f16_bits(g.uniform(1e-4, 1e-3, nb))
        sc = g.integers(0, 64, (nb, 8), dtype=np.uint8)
        m = g.integers(0, 64, (nb, 8), dtype=np.uint8)
        q = g.integers(0, 16, (nb, 256), dtype=np.uint8)
        out = pack_q4_k(d, dmin, sc, m, q)
    elif ggml_type == GGML_Q6_K:
        d = _f16_bits(g.uniform(1e-4, 1e-3, nb))
        sc = g.integers(-64, 65, (nb, 16), dtype=np.int16)
        q = g.integers(0, 64, (nb, 256), dtype=np.uint8)
        out = pack_q6_k(d, sc, q)
    else:
        raise ValueError(f"unsupported type {ggml_type}")
    return out.reshape(N, (K // be) * bb)


def gen_activations(B: int, K: int, seed: int) -> np.ndarray:
    return rng(seed).standard_normal((B, K), dtype=np.float32)


# ------------------------------------------------ 0.5B-shaped decoder weights
QWEN05B = dict(hidden=896, n_layers=24, n_heads=14, n_kv=2, head_dim=64, ffn=4864, vocab=151936,
               eps=1e-6, theta=1e6)
QWEN7B_LAYER = dict(hidden=3584, n_heads=28, n_kv=4, head_dim=128, ffn=18944)


def down_type(layer: int) -> int:
    """ffn_down is Q4_K, with Q6_K in every third layer (layer % 3 == 2)."""
    return GGML_Q6_K if layer % 3 == 2 else GGML_Q4_K


def gen_decoder(cfg: dict, seed: int = 4) -> dict:
    """Random weights for the Qwen2-shaped decoder.  attn_q/k/v/o and ffn_gate/up
    (K = hidden) are Q5_0, ffn_down Q4_K (Q6_K when layer % 3 == 2), the tied
    embedding Q8_0; q/k/v biases ~ N(0, 0.02); norm weights ~ 1 + N(0, 0.02)."""
    H, hd = cfg["hidden"], cfg["head_dim"]
    nq, nkv, F = cfg["n_heads"] * hd, cfg["n_kv"] * hd, cfg["ffn"]
    g = rng(seed)
    sub = lambda: int(g.integers(0, 2**31 - 1))  # noqa: E731
    layers = []
    for li in range(cfg["n_layers"]):
        L = {
            "wq": (GGML_Q5_0, gen_weight(GGML_Q5_0, nq, H, sub()), nq, H),
            "wk": (GGML_Q5_0, gen_weight(GGML_Q5_0, nkv, H, sub()), nkv, H),
            "wv": (GGML_Q5_0, gen_weight(GGML_Q5_0, nkv, H, sub()), nkv, H),
            "wo": (GGML_Q5_0, gen_weight(GGML_Q5_0, H, nq, sub()), H, nq),
            "wg": (GGML_Q5_0, gen_weight(GGML_Q5_0, F, H, sub()), F, H),
            "wu": (GGML_Q5_0, gen_weight(GGML_Q5_0, F, H, sub()), F, H),
        }
        dt = down_type(li)
        L["wd"] = (dt, gen_weight(dt, H, F, sub()), H, F)
        L["bq"] = (g.standard_normal(nq, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        L["bk"] = (g.standard_normal(nkv, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        L["bv"] = (g.standard_normal(nkv, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        L["attn_norm"] = (1 + g.standard_normal(H, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        L["ffn_norm"] = (1 + g.standard_normal(H, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        layers.append(L)
    out_norm = (1 + g.standard_normal(H, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    embed = (GGML_Q8_0, gen_weight(GGML_Q8_0, cfg["vocab"], H, sub()), cfg["vocab"], H)
    return {"cfg": dict(cfg), "layers": layers, "out_norm": out_norm, "embed": embed}


def gen_prompt(n: int, vocab: int, seed: int = 4) -> np.ndarray:
    return rng(seed + 1000).integers(0, vocab, n, dtype=np.int64).astype(np.int32)
