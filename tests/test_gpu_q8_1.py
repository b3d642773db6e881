"""The Q8_1 integer path: activation blocks bit-exact with the oracle's
quantization, the dp4a Q-GEMV within 1e-5 of the oracle's integer path on the
same blocks (only the summation order differs) and within the 2e-2 contract
of the fp32 product, bitwise-stable reruns."""
import numpy as np
import pytest

from hacedle_cuda import synth as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _blocks(ctx, X):
    import torch
    B, K = X.shape
    blk = torch.empty(B * K // 32 * 48, dtype=torch.uint8, device="cuda")
    ctx.quantize_q8_1(torch.from_numpy(X).cuda(), blk)
    return blk


def test_quantize_matches_oracle(ctx):
    rng = np.random.default_rng(2)
    X = (rng.standard_normal((5, 640)) * rng.uniform(0.01, 100, (5, 1))).astype(np.float32)
    X[1, 32:64] = 0.0                                   # an all-zero block
    X[2, 0:32] = np.linspace(-3, 3, 32, dtype=np.float32)
    blk = _blocks(ctx, X).cpu().numpy().reshape(5, 20, 48)
    q, d, s = O.quantize_q8_1(X)
    assert np.array_equal(blk[:, :, :32].view(np.int8).reshape(5, 640), q)
    assert np.array_equal(blk[:, :, 32:36].copy().view(np.float32)[..., 0], d)
    assert np.array_equal(blk[:, :, 36:40].copy().view(np.int16).astype(np.int32), s)


@pytest.mark.parametrize("t,N,K", [(S.GGML_Q5_0, 4864, 896), (S.GGML_Q6_K, 896, 4864), (S.GGML_Q4_K, 896, 4864),
                                   (S.GGML_Q8_0, 896, 896), (S.GGML_Q5_0, 100, 96), (S.GGML_Q6_K, 33, 256)])
@pytest.mark.parametrize("B", [1, 3, 4, 9, 16])
def test_qgemv_q8_1_matches_oracle(ctx, t, N, K, B):
    import torch
    raw = S.gen_weight(t, N, K, 170 + t)
    X = S.gen_activations(B, K, 171 + B)
    w = ctx.weight(t, raw, N, K)
    blk = _blocks(ctx, X)
    Y = torch.full((B, N), float("nan"), device="cuda")
    ctx.qgemv_q8_1(w, blk, Y, B)
    ctx.check_device_errors()
    got = Y.cpu().numpy()
    q, d, s = O.quantize_q8_1(X)
    ref = O.qgemv_q8_1(t, raw, N, K, q, d, s)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()
    full = X @ O.dequantize(t, raw, N * K).reshape(N, K).T
    assert np.abs(got - full).max() <= 2e-2 * np.abs(full).max()
    Y2 = torch.empty_like(Y)
    ctx.qgemv_q8_1(w, blk, Y2, B)
    torch.cuda.synchronize()
    assert torch.equal(Y, Y2)
