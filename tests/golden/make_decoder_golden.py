"""Greedy tokens of the 0.5B-shaped decoder from the CPU oracle.

Workload: Qwen2.5-0.5B shape (hidden 896, 24 layers, 14/2 heads, head_dim 64,
FFN 4864, vocab 151936, tied Q8_0 embedding), random weights from
synth.gen_decoder(seed=4), prefill of 512 ids from synth.gen_prompt(512), then
128 greedy tokens.  Writes beside this script:

- decoder_q05b_tokens.json: the 128 greedy ids;
- decoder_q05b_teacher.npz: per step g, a sample of the logits that chose id
  g (`idx`/`val` [128, 64]: the step's 16 largest logits, then 48 fixed
  indices drawn once with seed 7), the step's max |logit| (`absmax`), its
  greedy id (`top1`), the lead of the largest logit over the second
  (`margin`), and the step's conditioning (`sens`): how far the oracle's own
  sampled logits move, relative to absmax, when layer 0's attention-norm
  weights are nudged up by one ulp.  Most steps move by ~1e-6; a few (where
  attention is nearly one-hot between two positions) by ~1e-3.  A
  teacher-forced device run feeds the greedy ids back and compares its
  logits with these, with a per-step bound that grows with `sens`.

Takes a few minutes on 8 cores (the oracle runs token by token, as the
reference's BrainBlock::forward does).
"""
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.join(HERE, "..", "..")
sys.path[:0] = [ROOT, os.path.join(ROOT, "hace-fem-hacedle_b200", "python")]

from hacedle_cuda import synth as S  # noqa: E402
from oracle import oracle as O  # noqa: E402


def main(n_prompt=512, n_gen=128, threads=os.cpu_count()):
    t0 = time.time()
    model = S.gen_decoder(S.QWEN05B, seed=4)
    prompt = S.gen_prompt(n_prompt, S.QWEN05B["vocab"], seed=4)
    layers, out_norm, embed = O.dequant_model(model)
    toks, logits = O.decoder_generate(S.QWEN05B, layers, out_norm, embed, prompt, n_gen, threads=threads,
                                      all_logits=True)
    fixed = np.sort(np.random.default_rng(7).choice(S.QWEN05B["vocab"], 48, replace=False)).astype(np.int32)
    idx = np.zeros((n_gen, 64), np.int32)
    for g in range(n_gen):
        top = np.argsort(-logits[g], kind="stable")[:16].astype(np.int32)
        idx[g] = np.concatenate([top, fixed])
    val = np.take_along_axis(logits, idx, axis=1).astype(np.float32)
    srt = -np.sort(-logits, axis=1)[:, :2]
    absmax = np.abs(logits).max(axis=1).astype(np.float32)
    # conditioning: the same run with one norm vector one ulp larger
    layers[0]["attn_norm"] = np.nextafter(np.asarray(layers[0]["attn_norm"], np.float32), np.float32(np.inf))
    _, nudged = O.decoder_generate(S.QWEN05B, layers, out_norm, embed, prompt, n_gen, threads=threads,
                                   all_logits=True)
    sens = (np.abs(np.take_along_axis(nudged, idx, axis=1) - val).max(axis=1) / absmax).astype(np.float32)
    np.savez(os.path.join(HERE, "decoder_q05b_teacher.npz"), idx=idx, val=val, absmax=absmax,
             top1=np.asarray(toks, np.int32), margin=(srt[:, 0] - srt[:, 1]).astype(np.float32), sens=sens)
    res = {"config": "Qwen2.5-0.5B shape, synth.gen_decoder(seed=4), prompt synth.gen_prompt(512, seed=4)",
           "n_prompt": n_prompt, "n_gen": n_gen, "tokens": [int(t) for t in toks],
           "oracle_seconds": round(time.time() - t0, 1)}
    with open(os.path.join(HERE, "decoder_q05b_tokens.json"), "w") as f:
        json.dump(res, f, indent=1)
    print(res["tokens"][:16], res["oracle_seconds"])


if __name__ == "__main__":
    main()
