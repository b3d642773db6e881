"""tcgen05 prefill Q-GEMM (bf16 operands, fp32 accumulate in TMEM) against the
oracle: ||Y - Y_ref||_inf <= 2e-2 * ||Y_ref||_inf (the bf16 tensor-core
contract), no bounded device wait expired, and bitwise-stable reruns."""
import numpy as np
import pytest

import hacedle_cuda as hc
from oracle import oracle as O
from hacedle_cuda import synth as S

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.mark.parametrize("t,N,K", [(S.GGML_Q5_0, 4864, 896), (S.GGML_Q4_K, 896, 4864), (S.GGML_Q6_K, 896, 4864),
                                   (S.GGML_Q8_0, 896, 896)])
@pytest.mark.parametrize("T", [128, 512])
def test_qgemm_tc_config_shapes(ctx, t, N, K, T):
    import torch
    raw = S.gen_weight(t, N, K, 60 + t)
    X = S.gen_activations(T, K, 61)
    w = ctx.weight(t, raw, N, K)
    Y = torch.empty(T, N, device="cuda")
    ctx.qgemm(w, torch.from_numpy(X).cuda(), Y, precision=1)
    ctx.check_device_errors()
    got = Y.cpu().numpy()
    Wf = O.dequantize(t, raw, N * K).reshape(N, K)
    ref = X @ Wf.T
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err <= TOL, err
    Y2 = torch.empty(T, N, device="cuda")
    ctx.qgemm(w, torch.from_numpy(X).cuda(), Y2, precision=1)
    torch.cuda.synchronize()
    assert torch.equal(Y, Y2)


@pytest.mark.parametrize("t,N,K,T", [(S.GGML_Q5_0, 100, 96, 1), (S.GGML_Q5_0, 200, 160, 70), (S.GGML_Q4_K, 130, 512, 33),
                                     (S.GGML_Q6_K, 257, 256, 257), (S.GGML_Q8_0, 64, 64, 300)])
def test_qgemm_tc_ragged(ctx, t, N, K, T):
    import torch
    raw = S.gen_weight(t, N, K, 70 + N)
    X = S.gen_activations(T, K, 71)
    w = ctx.weight(t, raw, N, K)
    Y = torch.full((T, N), float("nan"), device="cuda")
    ctx.qgemm(w, torch.from_numpy(X).cuda(), Y, precision=1)
    ctx.check_device_errors()
    ref = X @ O.dequantize(t, raw, N * K).reshape(N, K).T
    got = Y.cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() / np.abs(ref).max() <= TOL


def test_qgemm_tc_prefill_2048(ctx):
    import torch
    t, N, K, T = S.GGML_Q5_0, 4864, 896, 2048
    raw = S.gen_weight(t, N, K, 5)
    X = S.gen_activations(T, K, 6)
    w = ctx.weight(t, raw, N, K)
    Y = torch.empty(T, N, device="cuda")
    ctx.qgemm(w, torch.from_numpy(X).cuda(), Y, precision=1)
    ctx.check_device_errors()
    ref = X @ O.dequantize(t, raw, N * K).reshape(N, K).T   # the oracle's weights, fp32 products
    got = Y.cpu().numpy()
    assert np.abs(got - ref).max() / np.abs(ref).max() <= TOL
    Yf = torch.empty(T, N, device="cuda")
    ctx.qgemm(w, torch.from_numpy(X).cuda(), Yf, precision=0)   # exact-weight fp32 path
    torch.cuda.synchronize()
    assert np.abs(Yf.cpu().numpy() - ref).max() / np.abs(ref).max() <= 1e-5


@pytest.mark.parametrize("t,N,K,T", [(S.GGML_Q5_0, 256, 96, 70), (S.GGML_Q4_K, 384, 512, 257),
                                     (S.GGML_Q6_K, 128, 768, 33), (S.GGML_Q8_0, 256, 160, 300),
                                     (S.GGML_Q5_0, 128, 896, 64)])
@pytest.mark.parametrize("bt", ["", "64", "128", "208"])
@pytest.mark.parametrize("path", ["streamed", "two_pass"])
def test_qgemm_tc_streamed_ragged_tiles(ctx, monkeypatch, t, N, K, T, bt, path):
    """Streamed kernel (rows % 128 == 0): odd unit counts (a half-empty last K
    step), token tails, the two-way K split of small grids, every token tile;
    the same cases through the two-pass kernel (dequantize, then TMA GEMM)."""
    import torch
    if bt:
        monkeypatch.setenv("HACEDLE_TC_BT", bt)
    monkeypatch.setenv("HACEDLE_TC4_MIN_T", "0" if path == "streamed" else "1")
    raw = S.gen_weight(t, N, K, 80 + N)
    X = S.gen_activations(T, K, 81)
    w = ctx.weight(t, raw, N, K)
    Y = torch.full((T, N), float("nan"), device="cuda")
    ctx.qgemm(w, torch.from_numpy(X).cuda(), Y, precision=1)
    ctx.check_device_errors()
    ref = X @ O.dequantize(t, raw, N * K).reshape(N, K).T
    got = Y.cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() / np.abs(ref).max() <= TOL
    Y2 = torch.full((T, N), float("nan"), device="cuda")
    ctx.qgemm(w, torch.from_numpy(X).cuda(), Y2, precision=1)
    torch.cuda.synchronize()
    assert torch.equal(Y, Y2)


def test_qgemm_rejects_unaligned_output(ctx):
    """hd_qgemm wants 16-byte aligned X and Y (the TMA and vector-store paths
    need it) and says so, without writing anything."""
    import torch
    t, N, K, T = S.GGML_Q5_0, 256, 256, 40
    w = ctx.weight(t, S.gen_weight(t, N, K, 90), N, K)
    X = torch.from_numpy(S.gen_activations(T, K, 91)).cuda()
    big = torch.full((T * N + 1,), float("nan"), device="cuda")
    with pytest.raises(hc.HdError) as ei:
        ctx.qgemm(w, X, big[1:].view(T, N), precision=1)
    assert ei.value.code == hc.HD_E_ARG
    assert torch.isnan(big).all()


@pytest.mark.parametrize("t,N,K,T", [(S.GGML_Q5_0, 4864, 896, 256), (S.GGML_Q4_K, 896, 4864, 37),
                                     (S.GGML_Q6_K, 300, 768, 100), (S.GGML_Q8_0, 151936 // 8, 896, 20)])
def test_qgemm_fp32_row_groups(ctx, t, N, K, T):
    """fp32 Q-GEMM of up to 1024 rows runs as 16-row groups of the batch
    Q-GEMV kernel: the oracle's product within 1e-5, bitwise-stable reruns."""
    import torch
    raw = S.gen_weight(t, N, K, 110 + T)
    X = S.gen_activations(T, K, 111)
    w = ctx.weight(t, raw, N, K)
    Y = torch.empty(T, N, device="cuda")
    Xd = torch.from_numpy(X).cuda()
    ctx.qgemm(w, Xd, Y, precision=0)
    ctx.check_device_errors()
    ref = O.qgemv(t, raw, N, K, X, threads=8)
    got = Y.cpu().numpy()
    assert np.abs(got - ref).max() / np.abs(ref).max() <= 1e-5
    Y2 = torch.empty(T, N, device="cuda")
    ctx.qgemm(w, Xd, Y2, precision=0)
    torch.cuda.synchronize()
    assert torch.equal(Y, Y2)


@pytest.mark.parametrize("t,N,K", [(S.GGML_Q5_0, 256, 896), (S.GGML_Q4_K, 128, 1024), (S.GGML_Q6_K, 384, 512),
                                   (S.GGML_Q8_0, 128, 256)])
@pytest.mark.parametrize("path", ["streamed", "two_pass"])
def test_qgemm_fp32_tensor_core_row_scaling(ctx, monkeypatch, t, N, K, path):
    """fp32 precision on the tensor cores splits x and the weights into fp16
    halves after power-of-two scaling per activation row: rows whose
    magnitudes differ by 10 orders each keep 1e-5 of their own maximum."""
    import torch
    monkeypatch.setenv("HACEDLE_TC4_MIN_T", "0" if path == "streamed" else "1")
    if path == "two_pass":
        monkeypatch.setenv("HACEDLE_TC4_EXACT", "1")
    T = 48
    raw = S.gen_weight(t, N, K, 130 + t)
    X = S.gen_activations(T, K, 131)
    X *= np.float32(10.0) ** np.linspace(-6, 4, T, dtype=np.float32)[:, None]
    w = ctx.weight(t, raw, N, K)
    Y = torch.empty(T, N, device="cuda")
    ctx.qgemm(w, torch.from_numpy(X).cuda(), Y, precision=0)
    ctx.check_device_errors()
    ref = O.qgemv(t, raw, N, K, X, threads=8)
    got = Y.cpu().numpy()
    err = np.abs(got - ref).max(axis=1) / np.abs(ref).max(axis=1)
    assert err.max() <= 1e-5, err.max()


@pytest.mark.parametrize("t,N,K,T", [(S.GGML_Q5_0, 100, 96, 1), (S.GGML_Q5_0, 200, 160, 70),
                                     (S.GGML_Q4_K, 130, 512, 33), (S.GGML_Q6_K, 257, 256, 257),
                                     (S.GGML_Q8_0, 64, 64, 300), (S.GGML_Q4_K, 1000, 768, 129)])
@pytest.mark.parametrize("bt", ["", "16", "112", "256"])
def test_qgemm_two_pass_any_rows(ctx, monkeypatch, t, N, K, T, bt):
    """Two-pass kernel on row counts that are not multiples of 128 (rows past
    N arrive as TMA zero fill and are not stored), odd unit counts, token tails
    and token tiles from 16 to 256; NaN-filled outputs must be fully written."""
    import torch
    monkeypatch.setenv("HACEDLE_TC4_MIN_T", "1")
    if bt:
        monkeypatch.setenv("HACEDLE_TC_BT", bt)
    raw = S.gen_weight(t, N, K, 140 + N)
    X = S.gen_activations(T, K, 141)
    w = ctx.weight(t, raw, N, K)
    Y = torch.full((T, N), float("nan"), device="cuda")
    ctx.qgemm(w, torch.from_numpy(X).cuda(), Y, precision=1)
    ctx.check_device_errors()
    ref = X @ O.dequantize(t, raw, N * K).reshape(N, K).T
    got = Y.cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() / np.abs(ref).max() <= TOL


@pytest.mark.parametrize("t,N,K,T", [(S.GGML_Q5_0, 200, 160, 70), (S.GGML_Q6_K, 257, 256, 257),
                                     (S.GGML_Q4_K, 1000, 768, 129), (S.GGML_Q8_0, 4864, 896, 300)])
def test_qgemm_fp32_two_pass_any_rows(ctx, monkeypatch, t, N, K, T):
    """Exact-product mode of the two-pass kernel, any row count: the oracle's
    fp32 product within 1e-5 of its maximum, bitwise-stable reruns."""
    import torch
    monkeypatch.setenv("HACEDLE_TC4_MIN_T", "1")
    monkeypatch.setenv("HACEDLE_TC4_EXACT", "1")
    raw = S.gen_weight(t, N, K, 150 + N)
    X = S.gen_activations(T, K, 151)
    w = ctx.weight(t, raw, N, K)
    Xd = torch.from_numpy(X).cuda()
    Y = torch.full((T, N), float("nan"), device="cuda")
    ctx.qgemm(w, Xd, Y, precision=0)
    ctx.check_device_errors()
    ref = O.qgemv(t, raw, N, K, X, threads=8)
    got = Y.cpu().numpy()
    assert np.abs(got - ref).max() / np.abs(ref).max() <= 1e-5
    Y2 = torch.empty(T, N, device="cuda")
    ctx.qgemm(w, Xd, Y2, precision=0)
    torch.cuda.synchronize()
    assert torch.equal(Y, Y2)


@pytest.mark.parametrize("t,N,K,T", [(S.GGML_Q5_0, 100, 96, 1), (S.GGML_Q5_0, 257, 160, 70), (S.GGML_Q4_K, 896, 512, 33),
                                     (S.GGML_Q6_K, 1000, 256, 300), (S.GGML_Q8_0, 4864, 896, 129),
                                     (S.GGML_Q4_K, 1152, 1024, 2048)])
@pytest.mark.parametrize("bt", ["", "64", "160", "256"])
def test_qgemm_pair_gemm(ctx, monkeypatch, t, N, K, T, bt):
    """The bf16 two-pass GEMM on SM pairs (k_gemm_tc5: tcgen05.mma.cta_group::2,
    M = 256 over two CTAs of a cluster, each CTA loading half of the token
    tile): any row count (a peer whose 128 rows lie past N stores nothing),
    token tails, token tiles 64..256; NaN-filled outputs fully written; equal
    to the one-SM kernel's result within the bf16 contract, reruns bitwise
    equal."""
    import torch
    monkeypatch.setenv("HACEDLE_TC4_MIN_T", "1")
    monkeypatch.setenv("HACEDLE_TC5", "1")
    if bt:
        monkeypatch.setenv("HACEDLE_TC_BT", bt)
    raw = S.gen_weight(t, N, K, 160 + N)
    X = S.gen_activations(T, K, 161)
    w = ctx.weight(t, raw, N, K)
    Xd = torch.from_numpy(X).cuda()
    outs = []
    for _ in range(2):
        Y = torch.full((T, N), float("nan"), device="cuda")
        ctx.qgemm(w, Xd, Y, precision=1)
        ctx.check_device_errors()
        outs.append(Y.cpu().numpy())
    monkeypatch.setenv("HACEDLE_TC5", "0")
    Y1 = torch.full((T, N), float("nan"), device="cuda")
    ctx.qgemm(w, Xd, Y1, precision=1)
    ctx.check_device_errors()
    ref = X @ O.dequantize(t, raw, N * K).reshape(N, K).T
    got = outs[0]
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() / np.abs(ref).max() <= TOL
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    one_sm = Y1.cpu().numpy()
    assert np.abs(got - one_sm).max() <= 1e-6 * np.abs(ref).max()
    w.free()


@pytest.mark.parametrize("t,N,K,T", [(S.GGML_Q5_0, 260, 160, 70), (S.GGML_Q4_K, 896, 4864, 2048),
                                     (S.GGML_Q6_K, 1000, 768, 300), (S.GGML_Q8_0, 4864, 896, 129),
                                     (S.GGML_Q4_K, 896, 512, 33)])
@pytest.mark.parametrize("bt", ["", "64", "256"])
@pytest.mark.parametrize("forced", [True, False])
def test_qgemm_pair_gemm_two_k_parts(ctx, monkeypatch, t, N, K, T, bt, forced):
    """The pair GEMM with K in two parts (HACEDLE_TC5_KS=2, or the cost
    model's choice where the tiles leave SM pairs idle, as on the 896 x 4864
    Q4_K weight at T = 2048): Y zeroed, each part's sums added by TMA; any row
    count, token tails, an odd number of K-step pairs; equal to the oracle
    within the bf16 contract and reruns bitwise equal (two addends onto zero
    sum the same in either order)."""
    import torch
    monkeypatch.setenv("HACEDLE_TC4_MIN_T", "1")
    if forced:
        monkeypatch.setenv("HACEDLE_TC5", "1")
        monkeypatch.setenv("HACEDLE_TC5_KS", "2")
    if bt:
        monkeypatch.setenv("HACEDLE_TC_BT", bt)
    raw = S.gen_weight(t, N, K, 170 + N)
    X = S.gen_activations(T, K, 171)
    w = ctx.weight(t, raw, N, K)
    Xd = torch.from_numpy(X).cuda()
    outs = []
    for _ in range(2):
        Y = torch.full((T, N), float("nan"), device="cuda")
        ctx.qgemm(w, Xd, Y, precision=1)
        ctx.check_device_errors()
        outs.append(Y.cpu().numpy())
    ref = X @ O.dequantize(t, raw, N * K).reshape(N, K).T
    assert np.isfinite(outs[0]).all()
    assert np.abs(outs[0] - ref).max() / np.abs(ref).max() <= TOL
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    w.free()
