"""Regenerates the committed golden fixtures in this folder.

Usage: python make_golden.py REFERENCE_CHECKOUT -- the path of a checkout of
the reference repository -- with the gguf package installed (gguf-py 0.19.0,
the version the reference's own goldens cite in tests/golden/manifest.yaml:6).
Nothing at test time reads the reference checkout; the tests read only the
files written here.

Fixtures:
  ref_<type>_block.raw / .f32   one real GGUF block and its gguf-py dequant,
                                copied from the reference's parity fixtures:
      parity_test/q8_0/blk0_attn_v_q8_0_first_block.{raw,bin}
      parity_test/q5_0/blk0_attn_q_q5_0_first_block.{raw,bin}
      parity_test/q6_k/blk0_ffn_down_q6_k_first_block.{raw,bin}
      tests/golden/q4k_block_000.bin, q4k_block_000_f32_gguf.bin
  gguf_<type>_rand.raw / .f32   seeded synthetic blocks (the workload
                                generators) dequantized by gguf-py
  gguf_<type>_edge.raw / .f32   blocks whose f16 scales are 0, -0, subnormal,
                                the largest normal and negative, with extreme q
  rope_pos<p>.f32, rope_in.f32  parity_test/rope/pos*.bin (NEOX RoPE of one
                                64-wide head, theta 1e6, numpy float64 math)
  gqa_k_raw.f32, gqa_k_expanded.f32   parity_test/gqa/*: kv head = h / 7
  oproj_w16.f32, oproj_x.f32, oproj_y16.f32   rows 0..15 of the block-0 o_proj
                                weight (golden/qwen2505b/block0/blk_0_attn_output_weight.bin),
                                its input (golden/block0_operators/09_attention_output.bin)
                                and output rows (10_o_proj.bin): y = W x
  minimal.hgraph, chain_rms_rope_mm.hgraph   tests/fixtures/*.hgraph
  manifest.json                 sizes and sha256 of everything above
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = ""  # the reference checkout, from the command line
sys.path[:0] = [os.path.join(HERE, "..", "..", "hace-fem-hacedle_b200", "python")]

from hacedle_cuda import synth as S  # noqa: E402


def main() -> None:
    import gguf
    from gguf.quants import dequantize as gdq

    gt = {S.GGML_Q8_0: gguf.GGMLQuantizationType.Q8_0, S.GGML_Q5_0: gguf.GGMLQuantizationType.Q5_0,
          S.GGML_Q4_K: gguf.GGMLQuantizationType.Q4_K, S.GGML_Q6_K: gguf.GGMLQuantizationType.Q6_K}
    names = {S.GGML_Q8_0: "q8_0", S.GGML_Q5_0: "q5_0", S.GGML_Q4_K: "q4_k", S.GGML_Q6_K: "q6_k"}
    copies = {
        "ref_q8_0_block.raw": "parity_test/q8_0/blk0_attn_v_q8_0_first_block.raw",
        "ref_q8_0_block.f32": "parity_test/q8_0/blk0_attn_v_q8_0_first_block.bin",
        "ref_q5_0_block.raw": "parity_test/q5_0/blk0_attn_q_q5_0_first_block.raw",
        "ref_q5_0_block.f32": "parity_test/q5_0/blk0_attn_q_q5_0_first_block.bin",
        "ref_q6_k_block.raw": "parity_test/q6_k/blk0_ffn_down_q6_k_first_block.raw",
        "ref_q6_k_block.f32": "parity_test/q6_k/blk0_ffn_down_q6_k_first_block.bin",
        "ref_q4_k_block.raw": "tests/golden/q4k_block_000.bin",
        "ref_q4_k_block.f32": "tests/golden/q4k_block_000_f32_gguf.bin",
        "gqa_k_raw.f32": "parity_test/gqa/k_raw.bin",
        "gqa_k_expanded.f32": "parity_test/gqa/k_expanded.bin",
        "minimal.hgraph": "tests/fixtures/minimal.hgraph",
        "chain_rms_rope_mm.hgraph": "tests/fixtures/chain_rms_rope_mm.hgraph",
    }
    for p in (0, 1, 128, 1024):
        copies[f"rope_pos{p}.f32"] = f"parity_test/rope/pos{p}.bin"
    for dst, src in copies.items():
        shutil.copyfile(os.path.join(REF, src), os.path.join(HERE, dst))
    x = ((np.arange(64, dtype=np.float32) - 32) / 64).astype(np.float32)
    x.tofile(os.path.join(HERE, "rope_in.f32"))

    w = np.fromfile(os.path.join(REF, "golden/qwen2505b/block0/blk_0_attn_output_weight.bin"), np.float32)
    w.reshape(896, 896)[:16].tofile(os.path.join(HERE, "oproj_w16.f32"))
    shutil.copyfile(os.path.join(REF, "golden/block0_operators/09_attention_output.bin"),
                    os.path.join(HERE, "oproj_x.f32"))
    y = np.fromfile(os.path.join(REF, "golden/block0_operators/10_o_proj.bin"), np.float32)
    y[:16].tofile(os.path.join(HERE, "oproj_y16.f32"))

    for t, nm in names.items():
        be, bb = S.BLOCK[t]
        raw = S.gen_weight(t, 4, 2 * 256, 100 + t)
        raw.tofile(os.path.join(HERE, f"gguf_{nm}_rand.raw"))
        gdq(raw, gt[t]).astype(np.float32).reshape(-1).tofile(os.path.join(HERE, f"gguf_{nm}_rand.f32"))
        edge = _edge_blocks(t)
        edge.tofile(os.path.join(HERE, f"gguf_{nm}_edge.raw"))
        gdq(edge, gt[t]).astype(np.float32).reshape(-1).tofile(os.path.join(HERE, f"gguf_{nm}_edge.f32"))

    manifest = {}
    for fn in sorted(os.listdir(HERE)):
        if fn.endswith((".py", ".json")):
            continue
        data = open(os.path.join(HERE, fn), "rb").read()
        manifest[fn] = {"bytes": len(data), "sha256": hashlib.sha256(data).hexdigest()}
    manifest["_sources"] = {k: v for k, v in copies.items()}
    manifest["_gguf"] = "gguf-py 0.19.0 (gguf.quants.dequantize)"
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)


_SCALES = np.array([0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0xFBFF, 0x3C00], np.uint16)


def _edge_blocks(t: int) -> np.ndarray:
    """One block per edge scale (0, -0, smallest subnormal, largest subnormal,
    smallest normal, largest normal, its negative, 1.0) with extreme quants."""
    n = _SCALES.size
    g = S.rng(77 + t)
    if t == S.GGML_Q8_0:
        q = g.integers(-128, 128, (n, 32))
        q[:, 0], q[:, 1] = -128, 127
        return S.pack_q8_0(_SCALES, q)
    if t == S.GGML_Q5_0:
        q = g.integers(0, 32, (n, 32))
        q[:, 0], q[:, 31] = 0, 31
        return S.pack_q5_0(_SCALES, q)
    if t == S.GGML_Q4_K:
        sc = g.integers(0, 64, (n, 8))
        m = g.integers(0, 64, (n, 8))
        sc[:, 7], m[:, 7] = 63, 63
        q = g.integers(0, 16, (n, 256))
        q[:, 0], q[:, 255] = 0, 15
        return S.pack_q4_k(_SCALES, _SCALES[::-1].copy(), sc, m, q)
    sc = g.integers(-128, 128, (n, 16))
    sc[:, 0], sc[:, 15] = -128, 127
    q = g.integers(0, 64, (n, 256))
    q[:, 0], q[:, 255] = 0, 63
    return S.pack_q6_k(_SCALES, sc, q)


if __name__ == "__main__":
    if len(sys.argv) != 2 or not os.path.isdir(sys.argv[1]):
        sys.exit("usage: python make_golden.py REFERENCE_CHECKOUT")
    REF = sys.argv[1]
    main()
