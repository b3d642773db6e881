"""The device decoder (hd_decoder_*) against the oracle's greedy tokens.

The fp32 path (exact dequantized weights, fp32 accumulation everywhere) must
reproduce the oracle's greedy tokens exactly.  The bf16 tensor-core prefill
is reported by its agreement with them.
"""
import json
import os

import numpy as np
import pytest

import hacedle_cuda as hc
from hacedle_cuda import synth as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SMALL = dict(hidden=128, n_layers=3, n_heads=4, n_kv=2, head_dim=32, ffn=256, vocab=1000, eps=1e-6, theta=1e6)


def _oracle_tokens(model, prompts, n_gen):
    layers, on, emb = O.dequant_model(model)
    return np.stack([O.decoder_generate(model["cfg"], layers, on, emb, p, n_gen, threads=8) for p in prompts])


@pytest.mark.parametrize("seqs,n_prompt,n_gen", [(1, 12, 10), (3, 7, 9), (8, 6, 5), (20, 5, 4)])
def test_small_decoder_matches_oracle(ctx, seqs, n_prompt, n_gen):
    model = S.gen_decoder(SMALL, seed=21)
    prompts = np.stack([S.gen_prompt(n_prompt, SMALL["vocab"], seed=30 + s) for s in range(seqs)])
    dec = hc.Decoder(ctx, model, max_ctx=n_prompt + n_gen, max_seqs=max(seqs, 4))
    toks, dms, pms = dec.generate(prompts, n_gen)
    ref = _oracle_tokens(model, prompts, n_gen)
    assert np.array_equal(toks, ref), (toks, ref)
    # a second call on the same decoder starts from a clean state
    toks2, _, _ = dec.generate(prompts, n_gen)
    assert np.array_equal(toks2, ref)
    dec.free()


def test_decoder_rejects_bad_requests(ctx):
    model = S.gen_decoder(SMALL, seed=22)
    dec = hc.Decoder(ctx, model, max_ctx=16, max_seqs=2)
    with pytest.raises(hc.HdError):
        dec.generate(np.zeros((3, 4), np.int32), 4)      # more sequences than max_seqs
    with pytest.raises(hc.HdError):
        dec.generate(np.zeros((1, 12), np.int32), 8)     # beyond max_ctx
    dec.free()


def test_q05b_greedy_tokens_match_oracle_golden(ctx, golden_dir):
    """Qwen2.5-0.5B-shaped decoder, prefill 512 ids, greedy 128 (batch 1)."""
    gold = json.load(open(os.path.join(golden_dir, "decoder_q05b_tokens.json")))
    model = S.gen_decoder(S.QWEN05B, seed=4)
    prompt = S.gen_prompt(gold["n_prompt"], S.QWEN05B["vocab"], seed=4)
    dec = hc.Decoder(ctx, model, max_ctx=gold["n_prompt"] + gold["n_gen"], max_seqs=1)
    toks, dms, pms = dec.generate(prompt[None], gold["n_gen"])
    assert toks[0].tolist() == gold["tokens"]
    tb, _, _ = dec.generate(prompt[None], gold["n_gen"], precision=hc.PREC_BF16_TC)
    agree = int(np.sum(tb[0] == np.array(gold["tokens"])))
    print(f"decode {dms:.2f} ms for {gold['n_gen'] - 1} steps, prefill {pms:.2f} ms; bf16 prefill agrees on "
          f"{agree}/{gold['n_gen']} tokens")
    dec.free()
