"""The oracle, pinned against the reference's own golden vectors (CPU only).

Mirrors the reference's dequant parity tests (tests/t1_q8_0_bit_exact.rs,
tests/q5_0_bit_exact.rs, tests/q4k_parity.rs, tests/dequant_layout_test.rs,
tests/rope_parity.rs) but with the IEEE f16 decode that the gguf-py goldens use.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from hacedle_cuda import synth as S

NAMES = {O.GGML_Q8_0: "q8_0", O.GGML_Q5_0: "q5_0", O.GGML_Q4_K: "q4_k", O.GGML_Q6_K: "q6_k"}


def _rd(golden_dir, name, dt):
    return np.fromfile(os.path.join(golden_dir, name), dt)


def test_layout_constants():
    # tests/dequant_layout_test.rs:4-38 -- bytes per block 34/22/144/210.
    assert O.BLOCK[O.GGML_Q8_0] == (32, 34)
    assert O.BLOCK[O.GGML_Q5_0] == (32, 22)
    assert O.BLOCK[O.GGML_Q4_K] == (256, 144)
    assert O.BLOCK[O.GGML_Q6_K] == (256, 210)
    for t, (be, bb) in O.BLOCK.items():
        if t in NAMES:
            assert S.BLOCK[t] == (be, bb)
            assert S.nbytes(t, 896, 4864 if be == 256 else 896) == 896 * (4864 if be == 256 else 896) // be * bb


@pytest.mark.parametrize("t", list(NAMES))
def test_reference_golden_block_bit_exact(golden_dir, t):
    nm = NAMES[t]
    raw = _rd(golden_dir, f"ref_{nm}_block.raw", np.uint8)
    exp = _rd(golden_dir, f"ref_{nm}_block.f32", np.float32)
    y = O.dequantize(t, raw, exp.size)
    assert np.array_equal(y.view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("t", list(NAMES))
@pytest.mark.parametrize("kind", ["rand", "edge"])
def test_gguf_py_vectors_bit_exact(golden_dir, t, kind):
    nm = NAMES[t]
    raw = _rd(golden_dir, f"gguf_{nm}_{kind}.raw", np.uint8)
    exp = _rd(golden_dir, f"gguf_{nm}_{kind}.f32", np.float32)
    y = O.dequantize(t, raw, exp.size)
    same = (y.view(np.uint32) == exp.view(np.uint32)) | (np.isnan(y) & np.isnan(exp))
    assert same.all()


def test_generator_matches_gguf_fixture(golden_dir):
    # The committed random blocks are the workload generators' own output.
    for t, nm in NAMES.items():
        raw = _rd(golden_dir, f"gguf_{nm}_rand.raw", np.uint8)
        assert np.array_equal(raw, S.gen_weight(t, 4, 512, 100 + t).reshape(-1))


def test_f16_decode_known_values():
    # The reference's f16_to_f32 (q4k_tensor_view.rs:123-136) is 2^127 too large;
    # IEEE binary16 is what every golden uses.
    assert O.f16_to_f32(0x3C00) == 1.0
    assert O.f16_to_f32(0xC000) == -2.0
    assert O.f16_to_f32(0x7BFF) == 65504.0
    assert O.f16_to_f32(0x0001) == 2.0 ** -24
    assert O.f16_to_f32(0x0400) == 2.0 ** -14
    assert np.isinf(O.f16_to_f32(0x7C00))


@pytest.mark.parametrize("pos", [0, 1, 128, 1024])
def test_rope_golden(golden_dir, pos):
    # parity_test/rope/pos*.bin were computed in numpy float64 and rounded; the
    # reference (src/ops/rope.rs) and the oracle compute the angle in f32.
    x = _rd(golden_dir, "rope_in.f32", np.float32)
    exp = _rd(golden_dir, f"rope_pos{pos}.f32", np.float32)
    y = O.rope_neox(x[None], np.array([pos]), 64)[0]
    tol = 1e-6 if pos <= 1 else 1e-5
    assert np.abs(y - exp).max() <= tol


def test_gqa_head_mapping(golden_dir):
    # parity_test/gqa: query head h reads kv head h // 7 (14 heads, 2 kv heads).
    k = _rd(golden_dir, "gqa_k_raw.f32", np.float32).reshape(2, 64)
    ke = _rd(golden_dir, "gqa_k_expanded.f32", np.float32).reshape(14, 64)
    for h in range(14):
        assert np.array_equal(ke[h], k[h // 7])
    # The oracle's attention uses the same map: a query equal to kv head 1's key
    # direction on head 7 attends to kv head 1's values.
    kc = np.zeros((1, 2, 64), np.float32)
    vc = np.zeros((1, 2, 64), np.float32)
    vc[0, 0, :] = 1.0
    vc[0, 1, :] = 2.0
    out = O.attention_decode(np.ones(14 * 64, np.float32), kc, vc, 14, 2, 64).reshape(14, 64)
    assert np.all(out[:7] == 1.0) and np.all(out[7:] == 2.0)


def test_oproj_gemv_golden(golden_dir):
    # golden/block0_operators/10_o_proj.bin = W_o . 09_attention_output.bin (numpy).
    w = _rd(golden_dir, "oproj_w16.f32", np.float32).reshape(16, 896)
    x = _rd(golden_dir, "oproj_x.f32", np.float32)
    y = _rd(golden_dir, "oproj_y16.f32", np.float32)
    yo = O.gemv_f32(w, x[None])[0]
    assert np.abs(yo - y).max() <= 1e-6
    assert np.array_equal(O.matmul_vec_matrix(x, w, 16, 896), yo)


def test_gemv_thread_count_invariant():
    # Row-parallel oracle: bits do not depend on the thread count.
    W = S.gen_weight(S.GGML_Q5_0, 64, 256, 3)
    X = S.gen_activations(3, 256, 4)
    y1 = O.qgemv(S.GGML_Q5_0, W, 64, 256, X, threads=1)
    y4 = O.qgemv(S.GGML_Q5_0, W, 64, 256, X, threads=4)
    assert np.array_equal(y1, y4)
    Wf = O.dequantize(S.GGML_Q5_0, W, 64 * 256).reshape(64, 256)
    for b in range(3):
        assert np.array_equal(y1[b], O.matmul_vec_matrix(X[b], Wf, 64, 256))


def test_rmsnorm_golden_vector():
    # core/tensor_ops/rms_norm.rs:16-23 golden: [1,2,3,4], w=1, eps=1e-5.
    y = O.rmsnorm(np.array([1, 2, 3, 4], np.float32), np.ones(4, np.float32), 1e-5)
    r = 1.0 / np.sqrt(np.float32(30.0 / 4.0 + 1e-5))
    assert np.allclose(y, np.array([1, 2, 3, 4]) * r, rtol=1e-6)


def test_softmax_silu_argmax_semantics():
    s = O.softmax(np.array([1.0, 2.0, 3.0], np.float32))
    assert abs(s.sum() - 1.0) < 1e-6 and s[2] > s[1] > s[0]
    x = np.array([-1.0, 0.0, 2.0], np.float32)
    assert np.allclose(O.silu(x), x / (1 + np.exp(-x)), rtol=1e-6)
    # first max wins; empty -> 0; NaN at index 0 -> 0
    assert O.argmax(np.array([1, 5, 5, 2], np.float32)) == 1
    assert O.argmax(np.array([], np.float32)) == 0
    assert O.argmax(np.array([np.nan, 5, 7], np.float32)) == 0
    assert O.argmax(np.array([-np.inf, -np.inf], np.float32)) == 0


def test_int8_ops_wrapping():
    a = np.full(300000, 127, np.int8)
    b = np.full(300000, 127, np.int8)
    exp = np.int64(127 * 127 * 300000)
    exp = int(((exp + 2**31) % 2**32) - 2**31)
    assert O.dot_i8(a, b) == exp
    out, carry = O.fused_qdot_qadd_qacc_i8(a[:64], b[:64], 5, 7)
    assert out == 127 * 127 * 64 + 12 and carry == out


def test_embedding_out_of_range():
    t = np.arange(12, dtype=np.float32)
    assert np.array_equal(O.embedding_lookup(1, t, 3, 4), [4, 5, 6, 7])
    assert np.array_equal(O.embedding_lookup(3, t, 3, 4), [0, 0, 0, 0])


def test_rope_interleaved_and_graph_rmsnorm():
    x = np.arange(8, dtype=np.float32).reshape(2, 4)
    c = np.cos(np.arange(8, dtype=np.float32)).reshape(2, 4)
    s = np.sin(np.arange(8, dtype=np.float32)).reshape(2, 4)
    o = O.rope_interleaved(x, c, s)
    assert np.allclose(o[0, 0], x[0, 0] * c[0, 0] - x[0, 1] * s[0, 0])
    assert np.allclose(o[0, 1], x[0, 1] * c[0, 0] + x[0, 0] * s[0, 0])
    y = O.rmsnorm_graph(x, np.ones(4, np.float32), 1e-5, newton=True)
    y2 = O.rmsnorm_graph(x, np.ones(4, np.float32), 1e-5, newton=False)
    assert np.allclose(y, y2, rtol=1e-6)


def test_tiny_decoder_is_deterministic():
    cfg = dict(hidden=64, n_layers=3, n_heads=4, n_kv=2, head_dim=16, ffn=256, vocab=97, eps=1e-6, theta=1e6)
    m = S.gen_decoder(cfg, seed=11)
    layers = []
    for L in m["layers"]:
        d = {k: L[k] for k in ("bq", "bk", "bv", "attn_norm", "ffn_norm")}
        for k in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
            t, raw, n, kk = L[k]
            d[k] = O.dequantize(t, raw, n * kk).reshape(n, kk)
        layers.append(d)
    t, raw, n, kk = m["embed"]
    emb = O.dequantize(t, raw, n * kk).reshape(n, kk)
    prompt = S.gen_prompt(8, cfg["vocab"])
    a = O.decoder_generate(cfg, layers, m["out_norm"], emb, prompt, 6, threads=1)
    b = O.decoder_generate(cfg, layers, m["out_norm"], emb, prompt, 6, threads=4)
    assert np.array_equal(a, b)
    assert a.min() >= 0 and a.max() < cfg["vocab"]
