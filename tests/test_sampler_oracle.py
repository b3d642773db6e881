"""The sampler's oracle on the CPU: Philox4x32-10 against the published
Random123 known-answer vectors, and logits_process against a literal
per-element restatement of LogitsProcessor (src/x/provider/candle/
lmhead.rs:42-111), quirks included (exp of raw logits, threshold 0.0 when the
top-p sum never reaches top_p, the (top_k+1)-th value as top-k threshold)."""
import math

import numpy as np
import pytest

from oracle import oracle as O


def test_philox_known_answers():
    assert O.philox4x32_10((0, 0, 0, 0), (0, 0)) == (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)
    assert O.philox4x32_10((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2) == (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)
    assert O.philox4x32_10((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0)) == \
        (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)


def _literal(logits, temperature, top_p, top_k):
    """The reference's three loops, element by element, in f32."""
    f = np.float32
    v = [f(x) for x in logits]
    t = max(f(temperature), f(0.001))
    v = [f(x / t) for x in v]
    srt = sorted(v, reverse=True)
    cum, thr = f(0.0), f(0.0)
    for p in srt:
        with np.errstate(over="ignore"):
            cum = f(cum + min(f(np.exp(f(p))), f(1.0)))
        if cum >= f(top_p):
            thr = p
            break
    v = [x if x >= thr else f(-math.inf) for x in v]
    srt = sorted(v, reverse=True)
    thk = srt[top_k] if 0 < top_k < len(srt) else f(-math.inf)
    return np.array([x if x >= thk else f(-math.inf) for x in v], np.float32)


@pytest.mark.parametrize("scale,t,top_p,top_k", [(3.0, 0.7, 0.9, 0), (3.0, 1.0, 0.9, 5), (0.5, 1.3, 0.95, 40),
                                                 (-1.0, 1.0, 0.5, 0), (1.0, 0.0, 0.9, 3), (1.0, 1.0, 2.0, 0),
                                                 (1.0, 1.0, 0.0, 0), (2.0, 1.0, 1.0, 199)])
def test_logits_process_matches_literal_loops(scale, t, top_p, top_k):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(200) * scale).astype(np.float32)
    if scale < 0:                         # log-probability-like row: a long top-p walk
        x = (x - 8.0).astype(np.float32)
    got = O.logits_process(x, t, top_p, top_k)
    want = _literal(x, t, top_p, top_k)
    assert np.array_equal(got, want)


def test_sample_oracle_degenerate_rows():
    x = np.full((2, 300), -np.inf, np.float32)
    x[0, 123] = 5.0
    idx, _ = O.sample_rows(x, seed=7)
    assert idx.tolist() == [123, -1]
