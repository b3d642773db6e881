"""hd_lm_head_argmax: LMHead::forward and ArgMaxSampler::sample in one call
(src/x/provider/candle/lmhead.rs:22-38, runtime/sampler/argmax.rs:8-24).
Up to 4 rows the argmax is folded into the GEMV's epilogue.  The logits must
be bitwise those of hd_qgemv_rmsnorm (the same kernel), and the ids those of
the oracle's argmax: first maximum wins (strict >), 0 when a row's first
logit is NaN."""
import numpy as np
import pytest

import hacedle_cuda as hc
from hacedle_cuda import synth as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _weight_with_tie(V, K, seed):
    """Q8_0 [V, K] whose rows 300 and 500 are the same bytes with a scale 64x
    the largest, so that they tie for the maximum of every row of logits."""
    raw = S.gen_weight(S.GGML_Q8_0, V, K, seed).reshape(V, -1).copy()
    blocks = raw[300].reshape(-1, 34)
    d = np.frombuffer(blocks[:, :2].tobytes(), np.float16).astype(np.float32) * np.float32(64)
    blocks[:, :2] = np.frombuffer(d.astype(np.float16).tobytes(), np.uint8).reshape(-1, 2)
    raw[300] = blocks.reshape(-1)
    raw[500] = raw[300]
    return raw.reshape(-1)


@pytest.mark.parametrize("B", [1, 2, 3, 4, 7])
@pytest.mark.parametrize("norm", [True, False])
def test_lm_head_argmax_matches_gemv_and_oracle(ctx, monkeypatch, B, norm):
    import torch
    # the plain reference GEMV on the CTA kernel (the one the fused argmax rides
    # on), not the block, tensor-core, streamed or stream-K kernels large
    # weights take
    monkeypatch.setenv("HACEDLE_GEMV_ST", "0")
    monkeypatch.setenv("HACEDLE_GEMV_BLK", "0")
    monkeypatch.setenv("HACEDLE_GEMV_MMA", "0")
    monkeypatch.setenv("HACEDLE_GEMV_SK", "0")
    V, K = 20000, 896
    raw = S.gen_weight(S.GGML_Q8_0, V, K, 5 + B)
    w = ctx.weight(S.GGML_Q8_0, raw, V, K)
    X = S.gen_activations(B, K, 6 + B)
    nw = (1 + 0.02 * S.rng(7).standard_normal(K)).astype(np.float32)
    x, nwd = torch.from_numpy(X).cuda(), torch.from_numpy(nw).cuda()
    logits = torch.empty(B, V, device="cuda")
    idx = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    ctx.lm_head_argmax(w, x, logits, idx, norm_w=nwd if norm else None)
    ref_logits = torch.empty(B, V, device="cuda")
    if norm:
        ctx.qgemv_norm(w, x, nwd, ref_logits)
    else:
        ctx.qgemv(w, x, ref_logits)
    ctx.check_device_errors()
    lg = logits.cpu().numpy()
    assert np.array_equal(lg.view(np.uint32), ref_logits.cpu().numpy().view(np.uint32))
    assert [int(v) for v in idx.cpu()] == [O.argmax(lg[b]) for b in range(B)]
    # again: the keys and the counter were left clear
    ctx.lm_head_argmax(w, x, logits, idx, norm_w=nwd if norm else None)
    assert [int(v) for v in idx.cpu()] == [O.argmax(lg[b]) for b in range(B)]
    w.free()


def test_lm_head_argmax_tie_and_nan(ctx):
    import torch
    V, K, B = 4096, 256, 3
    raw = _weight_with_tie(V, K, 9)
    w = ctx.weight(S.GGML_Q8_0, raw, V, K)
    X = np.abs(S.gen_activations(B, K, 10))
    X[:, :] = np.where(S.rng(11).random((B, K)) < 0.5, X, X)   # positive x: rows 300/500 lead clearly
    logits = torch.empty(B, V, device="cuda")
    idx = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    ctx.lm_head_argmax(w, torch.from_numpy(X).cuda(), logits, idx)
    lg = logits.cpu().numpy()
    assert np.array_equal(lg[:, 300], lg[:, 500])
    got = [int(v) for v in idx.cpu()]
    assert got == [O.argmax(lg[b]) for b in range(B)]
    assert all(g == 300 for g in got if lg[0, 300] == lg[0].max())
    w.free()
    # row 0 of the weight with NaN scales: every logit row starts with NaN -> id 0
    raw2 = S.gen_weight(S.GGML_Q8_0, V, K, 12).reshape(V, -1).copy()
    raw2[0].reshape(-1, 34)[:, :2] = np.frombuffer(np.array([np.nan], np.float16).tobytes(), np.uint8)
    w2 = ctx.weight(S.GGML_Q8_0, raw2.reshape(-1), V, K)
    ctx.lm_head_argmax(w2, torch.from_numpy(X).cuda(), logits, idx)
    lg2 = logits.cpu().numpy()
    assert np.isnan(lg2[:, 0]).all()
    assert [int(v) for v in idx.cpu()] == [0] * B == [O.argmax(lg2[b]) for b in range(B)]
    w2.free()
