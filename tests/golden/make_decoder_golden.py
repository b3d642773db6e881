"""Greedy tokens of the 0.5B-shaped decoder from the CPU oracle.

Workload: Qwen2.5-0.5B shape (hidden 896, 24 layers, 14/2 heads, head_dim 64,
FFN 4864, vocab 151936, tied Q8_0 embedding), random weights from
synth.gen_decoder(seed=4), prefill of 512 ids from synth.gen_prompt(512), then
128 greedy tokens.  Writes decoder_q05b_tokens.json beside this script.  Takes
a few minutes on 8 cores (the oracle runs token by token, as the reference's
BrainBlock::forward does).
"""
import json
import os
import sys
import time

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
    toks = O.decoder_generate(S.QWEN05B, layers, out_norm, embed, prompt, n_gen, threads=threads)
    res = {"config": "Qwen2.5-0.5B shape, synth.gen_decoder(seed=4), prompt synth.gen_prompt(512, seed=4)",
           "n_prompt": n_prompt, "n_gen": n_gen, "tokens": [int(t) for t in toks],
           "oracle_seconds": round(time.time() - t0, 1)}
    with open(os.path.join(HERE, "decoder_q05b_tokens.json"), "w") as f:
        json.dump(res, f, indent=1)
    print(res["tokens"][:16], res["oracle_seconds"])


if __name__ == "__main__":
    main()
