"""GGUF file -> device: hd_gguf_upload of every quantized matrix of the tiny
Qwen2 fixture dequantizes bit-exactly to the oracle, and the decoder built
from the file (hacedle_cuda.gguf.qwen2_model) reproduces the oracle's greedy
tokens for the same file."""
import os

import numpy as np
import pytest

from hacedle_cuda import gguf as G
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TINY_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "qwen2_tiny.gguf")


def test_upload_from_gguf_dequantizes_exactly(ctx):
    import torch
    g = G.GGUF(TINY_PATH)
    n = 0
    for t in g.tensors:
        if t["type"] not in (6, 8, 12, 14):
            continue
        w = g.upload(ctx, t["name"])
        rows, cols = int(t["dims"][1]), int(t["dims"][0])
        out = torch.empty(rows * cols, device="cuda")
        ctx.dequantize(w, out)
        ref = O.dequantize(t["type"], g.tensor_bytes(t["name"]), rows * cols)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32)), t["name"]
        w.free()
        n += 1
    assert n == 1 + 3 * 7


@pytest.mark.parametrize("seqs,n_prompt,n_gen", [(1, 9, 8), (3, 6, 5)])
def test_decoder_from_gguf_matches_oracle(ctx, seqs, n_prompt, n_gen):
    import hacedle_cuda as hc
    from hacedle_cuda import synth as S
    model = G.qwen2_model(G.GGUF(TINY_PATH))
    cfg = model["cfg"]
    prompts = np.stack([S.gen_prompt(n_prompt, cfg["vocab"], seed=40 + s) for s in range(seqs)])
    dec = hc.Decoder(ctx, model, max_ctx=n_prompt + n_gen, max_seqs=max(seqs, 2))
    toks, _, _ = dec.generate(prompts, n_gen)
    dec.free()
    layers, on, emb = O.dequant_model(model)
    ref = np.stack([O.decoder_generate(cfg, layers, on, emb, p, n_gen, threads=8) for p in prompts])
    assert np.array_equal(toks, ref), (toks, ref)
