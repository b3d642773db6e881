"""The Qwen2.5-7B-shaped layer's projections at their own shapes, against the
oracle (the row-sharded GEMV order of core/tensor_ops/matmul.rs:4-21).

Matrices: q/o [3584 x 3584], k/v [512 x 3584], gate/up [18944 x 3584] in
Q4_K, down [3584 x 18944] in Q6_K (BASELINE generators), whole and as the
row slices one of 8 ranks holds (448, 64, 2368 and 448 rows -- not multiples
of 128).  Batch 1 and 4 run the decode Q-GEMV (fp32 contract, 1e-5); 64 and
512 tokens run the tcgen05 Q-GEMM with bf16 operands (2e-2, the bf16
tensor-core contract).  Norm-wise: ||y - y_ref||_inf <= tol ||y_ref||_inf.
"""
import numpy as np
import pytest

from hacedle_cuda import shard
from hacedle_cuda import synth as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu
H, F, NQ, NKV = 3584, 18944, 28 * 128, 4 * 128
MATS = {"q": (S.GGML_Q4_K, NQ, H), "k": (S.GGML_Q4_K, NKV, H), "gate": (S.GGML_Q4_K, F, H),
        "down": (S.GGML_Q6_K, H, F)}


def _rel_err(y, ref):
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def _weights(name, ranks):
    t, N, K = MATS[name]
    raw = S.gen_weight(t, N, K, seed=50 + list(MATS).index(name))
    if ranks == 1:
        return t, N, K, raw
    # rank 3 of `ranks`: a middle slice
    sl = shard.row_slice(raw, t, N, K, 3, ranks)
    return t, N // ranks, K, sl


@pytest.mark.parametrize("name", list(MATS))
@pytest.mark.parametrize("ranks", [1, 8])
@pytest.mark.parametrize("B", [1, 4])
def test_layer7b_gemv(ctx, name, ranks, B):
    import torch
    t, N, K, raw = _weights(name, ranks)
    X = S.gen_activations(B, K, 60)
    w = ctx.weight(t, raw, N, K)
    y = torch.full((B, N), float("nan"), device="cuda")
    ctx.qgemv(w, torch.from_numpy(X).cuda(), y)
    ctx.check_device_errors()
    ref = O.qgemv(t, raw, N, K, X, threads=8)
    assert _rel_err(y.cpu().numpy(), ref) <= 1e-5
    w.free()


@pytest.mark.parametrize("name", list(MATS))
@pytest.mark.parametrize("ranks", [1, 8])
@pytest.mark.parametrize("T", [64, 512])
def test_layer7b_gemm_bf16(ctx, name, ranks, T):
    import torch
    import hacedle_cuda as hc
    t, N, K, raw = _weights(name, ranks)
    X = S.gen_activations(T, K, 61)
    w = ctx.weight(t, raw, N, K)
    Y = torch.full((T, N), float("nan"), device="cuda")
    ctx.qgemm(w, torch.from_numpy(X).cuda(), Y, precision=hc.PREC_BF16_TC)
    ctx.check_device_errors()
    Wf = O.dequantize(t, raw, N * K).reshape(N, K)
    ref = X @ Wf.T
    got = Y.cpu().numpy()
    assert np.isfinite(got).all()
    assert _rel_err(got, ref) <= 2e-2
    w.free()
