"""Writes the GGUF fixtures of the reader tests with gguf-py's GGUFWriter
(the writer of the reference's golden tooling, gguf 0.19.0):

- qwen2_tiny.gguf: a tiny Qwen2-shaped decoder (synth.gen_decoder(TINY,
  seed=21): Q5_0 attention and gate/up, Q4_K / Q6_K down, tied Q8_0
  token_embd, f32 biases and norms) under llama.cpp's qwen2 tensor names and
  metadata, plus one metadata entry of every value type;
- align64.gguf: two tiny tensors with general.alignment = 64.

Run from the repository root: python tests/golden/make_gguf_fixtures.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [ROOT, os.path.join(ROOT, "hace-fem-hacedle_b200", "python")]

import gguf  # noqa: E402

from hacedle_cuda import synth as S  # noqa: E402

TINY = dict(hidden=64, n_layers=3, n_heads=2, n_kv=1, head_dim=32, ffn=256, vocab=256, eps=1e-6, theta=1e6)
OUT = os.path.dirname(os.path.abspath(__file__))
QT = {S.GGML_Q5_0: gguf.GGMLQuantizationType.Q5_0, S.GGML_Q8_0: gguf.GGMLQuantizationType.Q8_0,
      S.GGML_Q4_K: gguf.GGMLQuantizationType.Q4_K, S.GGML_Q6_K: gguf.GGMLQuantizationType.Q6_K}


def _quant(w, name, mat):
    t, raw, rows, cols = mat
    w.add_tensor(name, np.asarray(raw, np.uint8).reshape(rows, -1), raw_dtype=QT[t])


def qwen2_tiny(path):
    m = S.gen_decoder(TINY, seed=21)
    c = m["cfg"]
    w = gguf.GGUFWriter(path, "qwen2")
    w.add_context_length(64)
    w.add_embedding_length(c["hidden"])
    w.add_block_count(c["n_layers"])
    w.add_feed_forward_length(c["ffn"])
    w.add_head_count(c["n_heads"])
    w.add_head_count_kv(c["n_kv"])
    w.add_rope_freq_base(c["theta"])
    w.add_layer_norm_rms_eps(c["eps"])
    # one entry of every value type, for the reader's metadata tests
    w.add_uint8("test.u8", 200)
    w.add_int8("test.i8", -100)
    w.add_uint16("test.u16", 60000)
    w.add_int16("test.i16", -30000)
    w.add_uint32("test.u32", 4000000000)
    w.add_int32("test.i32", -2000000000)
    w.add_float32("test.f32", 0.15625)
    w.add_bool("test.bool", True)
    w.add_uint64("test.u64", 2 ** 63 + 5)
    w.add_int64("test.i64", -(2 ** 62))
    w.add_float64("test.f64", 2.718281828459045)
    w.add_string("test.str", "héllo gguf")
    w.add_array("test.arr_i32", [1, -2, 3, -4])
    w.add_array("test.arr_f32", [0.5, -1.25])
    w.add_array("tokenizer.ggml.tokens", [f"tok{i}" for i in range(12)] + ["", "é"])
    _quant(w, "token_embd.weight", m["embed"])
    for i, L in enumerate(m["layers"]):
        b = f"blk.{i}."
        w.add_tensor(b + "attn_norm.weight", L["attn_norm"])
        for k, nm in (("wq", "attn_q"), ("wk", "attn_k"), ("wv", "attn_v")):
            _quant(w, b + nm + ".weight", L[k])
        w.add_tensor(b + "attn_q.bias", L["bq"])
        w.add_tensor(b + "attn_k.bias", L["bk"])
        w.add_tensor(b + "attn_v.bias", L["bv"])
        _quant(w, b + "attn_output.weight", L["wo"])
        w.add_tensor(b + "ffn_norm.weight", L["ffn_norm"])
        _quant(w, b + "ffn_gate.weight", L["wg"])
        _quant(w, b + "ffn_up.weight", L["wu"])
        _quant(w, b + "ffn_down.weight", L["wd"])
    w.add_tensor("output_norm.weight", m["out_norm"])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def align64(path):
    w = gguf.GGUFWriter(path, "test")
    w.add_custom_alignment(64)
    w.add_tensor("a", np.arange(3, dtype=np.float32))
    t, raw, rows, cols = (S.GGML_Q8_0, S.gen_weight(S.GGML_Q8_0, 2, 64, 9), 2, 64)
    _quant(w, "b", (t, raw, rows, cols))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


if __name__ == "__main__":
    qwen2_tiny(os.path.join(OUT, "qwen2_tiny.gguf"))
    align64(os.path.join(OUT, "align64.gguf"))
    for f in ("qwen2_tiny.gguf", "align64.gguf"):
        print(f, os.path.getsize(os.path.join(OUT, f)))
