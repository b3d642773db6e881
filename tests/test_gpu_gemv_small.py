"""The small-matrix decode Q-GEMV (k_qgemv_sm, hd_gemv_small.cu: mma.sync
over 32-row tiles, K parts of a tile in a thread-block cluster) against the
oracle, forced onto every shape with HACEDLE_GEMV_SMALL=1 and the
large-matrix kernels off.  It is the default for plain GEMVs at batch 1..4 on
weights under 16 MB (the decode sweep's 0.5B-shaped matrices at batch 1 and
4); the forced runs also cover batch 5..16.

Cases: every quant type; ragged row tiles; one to eight K parts
(HACEDLE_SM_S) and one to fourteen warps per CTA (HACEDLE_SM_W); batch 1..16
(padded to 1, 2, 4, 8, 16); bias and in-place residual; reruns bitwise equal;
units of x spanning many binades.  Bar: the fp32 contract
||y - y_ref||_inf <= 1e-5 ||y_ref||_inf."""
import numpy as np
import pytest

from hacedle_cuda import synth as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TYPES = [S.GGML_Q8_0, S.GGML_Q5_0, S.GGML_Q4_K, S.GGML_Q6_K]
REL_TOL = 1e-5


def _rel_err(y, ref):
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def _small(monkeypatch, s="", w=""):
    monkeypatch.setenv("HACEDLE_GEMV_ST", "0")
    monkeypatch.setenv("HACEDLE_GEMV_BLK", "0")
    monkeypatch.setenv("HACEDLE_GEMV_MMA", "0")
    monkeypatch.setenv("HACEDLE_GEMV_SK", "0")
    monkeypatch.setenv("HACEDLE_GEMV_SMALL", "1")
    monkeypatch.setenv("HACEDLE_SM_S", s)
    monkeypatch.setenv("HACEDLE_SM_W", w)


def _run(ctx, t, N, K, B, seed, X=None, bias=False, residual=False, reps=1):
    import torch
    raw = S.gen_weight(t, N, K, seed)
    if X is None:
        X = S.gen_activations(B, K, seed + 1)
    w = ctx.weight(t, raw, N, K)
    x = torch.from_numpy(X).cuda()
    ref = O.qgemv(t, raw, N, K, X, threads=8)
    bt = None
    if bias:
        bh = S.rng(seed + 2).standard_normal(N, dtype=np.float32) * np.float32(0.02)
        bt = torch.from_numpy(bh).cuda()
        ref = ref + bh[None, :]
    rh = None
    if residual:
        rh = S.rng(seed + 3).standard_normal((B, N), dtype=np.float32)
        ref = rh + ref
    outs = []
    for _ in range(reps):
        if residual:
            y = torch.from_numpy(rh.copy()).cuda()
            ctx.qgemv(w, x, y, bias=bt, residual=y)
        else:
            y = torch.full((B, N), float("nan"), dtype=torch.float32, device="cuda")
            ctx.qgemv(w, x, y, bias=bt)
        ctx.check_device_errors()
        outs.append(y.cpu().numpy())
    w.free()
    return outs, ref


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("N,K,B", [(7, 256, 1), (34, 512, 2), (100, 768, 3), (896, 1024, 4), (4866, 1280, 1),
                                   (896, 4864, 4), (257, 2304, 5), (4865, 1280, 9), (4864, 896 + 128, 16),
                                   (896, 4864, 16), (1, 256, 7), (33, 8192, 12)])
def test_small_gemv_matches_oracle(ctx, monkeypatch, t, N, K, B):
    _small(monkeypatch)
    outs, ref = _run(ctx, t, N, K, B, 700 + N + K + B + t)
    assert np.isfinite(outs[0]).all()
    assert _rel_err(outs[0], ref) <= REL_TOL


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("s,w", [("1", "1"), ("1", "14"), ("2", "3"), ("3", ""), ("5", "2"), ("8", "1"), ("8", "7")])
@pytest.mark.parametrize("B", [1, 4, 16])
def test_small_gemv_cluster_and_warp_splits(ctx, monkeypatch, t, s, w, B):
    """K-part counts 1..8 and warp counts (one or two units per warp) on a
    ragged tile count, with bias and in-place residual, three runs bitwise
    equal."""
    _small(monkeypatch, s, w)
    outs, ref = _run(ctx, t, 200, 2048, B, 60 + B + t, bias=True, residual=(B != 4), reps=3)
    assert _rel_err(outs[0], ref) <= REL_TOL
    for o in outs[1:]:
        assert np.array_equal(outs[0].view(np.uint32), o.view(np.uint32))


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("B", [3, 16])
def test_small_gemv_extreme_activations(ctx, monkeypatch, t, B):
    """Units whose x spans many binades (the per-unit power-of-two scale and
    the fp16 hi/lo split), an all-zero unit, and huge and tiny magnitudes."""
    _small(monkeypatch)
    N, K = 256, 1024
    X = S.gen_activations(B, K, 78)
    X[0, :32] *= np.float32(1e-30)
    X[1, 32:64] = 0.0
    X[1, 64:96] *= np.float32(1e25)
    X[2, ::7] *= np.float32(1e6)
    outs, ref = _run(ctx, t, N, K, B, 77, X=X)
    for b in range(B):  # row by row: the rows' magnitudes differ by decades
        assert _rel_err(outs[0][b], ref[b]) <= REL_TOL, b


def test_small_gemv_is_the_default_for_the_sweep_shapes(ctx):
    """Without overrides the 0.5B-shaped sweep matrices take the small-matrix
    kernel at batch 1 and 4 and meet the contract."""
    for (t, N, K) in [(S.GGML_Q5_0, 4864, 896), (S.GGML_Q6_K, 896, 4864), (S.GGML_Q4_K, 896, 4864)]:
        for B in (1, 2, 4):
            outs, ref = _run(ctx, t, N, K, B, 31 + B)
            assert _rel_err(outs[0], ref) <= REL_TOL, (t, B)


def _norm_ref(t, raw, N, K, X, nw, eps=1e-6):
    xn = O.rmsnorm(X, nw, eps).reshape(X.shape[0], K)
    return O.qgemv(t, raw, N, K, xn, threads=8)


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("N,K,B", [(1152, 1024, 1), (896, 4864, 2), (257, 2304, 4), (100, 768, 3), (33, 8192, 9)])
@pytest.mark.parametrize("s", ["", "1", "4"])
def test_small_gemv_fused_rmsnorm(ctx, monkeypatch, t, N, K, B, s):
    """W rmsnorm(x) (+bias, +residual) with the norm in the kernel: x * w
    into the fragments, the sums of x^2 reduced with the row sums (across the
    K parts of a cluster too), 1 / rms applied to the row sums."""
    import torch
    _small(monkeypatch, s)
    raw = S.gen_weight(t, N, K, 300 + B)
    X = S.gen_activations(B, K, 301)
    nw = (1.0 + 0.02 * S.rng(302).standard_normal(K)).astype(np.float32)
    bh = (0.02 * S.rng(303).standard_normal(N)).astype(np.float32)
    rh = S.rng(304).standard_normal((B, N), dtype=np.float32)
    ref = rh + (_norm_ref(t, raw, N, K, X, nw) + bh[None, :])
    w = ctx.weight(t, raw, N, K)
    y = torch.from_numpy(rh.copy()).cuda()
    ctx.qgemv_norm(w, torch.from_numpy(X).cuda(), torch.from_numpy(nw).cuda(), y, bias=torch.from_numpy(bh).cuda(),
                   residual=y)
    ctx.check_device_errors()
    assert _rel_err(y.cpu().numpy(), ref) <= REL_TOL
    w.free()


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("N,K,B", [(4864, 1024, 1), (4864, 1024, 4), (200, 2048, 2), (17, 512, 3), (896, 4864, 12)])
@pytest.mark.parametrize("norm", [False, True])
@pytest.mark.parametrize("s", ["", "3"])
def test_small_gemv_swiglu_pair(ctx, monkeypatch, t, N, K, B, norm, s):
    """silu(W_gate x) * (W_up x), optionally of rmsnorm(x): a 32-row tile
    holds 16 gate rows and the same 16 up rows; reruns bitwise equal."""
    import torch
    _small(monkeypatch, s)
    rg, ru = S.gen_weight(t, N, K, 410 + B), S.gen_weight(t, N, K, 411 + B)
    X = S.gen_activations(B, K, 412)
    nw = (1.0 + 0.02 * S.rng(413).standard_normal(K)).astype(np.float32)
    xin = O.rmsnorm(X, nw, 1e-6).reshape(B, K) if norm else X
    ref = O.swiglu(O.qgemv(t, rg, N, K, xin, threads=8), O.qgemv(t, ru, N, K, xin, threads=8)).reshape(B, N)
    wg, wu = ctx.weight(t, rg, N, K), ctx.weight(t, ru, N, K)
    x = torch.from_numpy(X).cuda()
    outs = []
    for _ in range(2):
        y = torch.full((B, N), float("nan"), device="cuda")
        if norm:
            ctx.qgemv_norm(wg, x, torch.from_numpy(nw).cuda(), y, w_up=wu)
        else:
            ctx.qgemv_swiglu(wg, wu, x, y)
        ctx.check_device_errors()
        outs.append(y.cpu().numpy())
    assert np.isfinite(outs[0]).all()
    assert _rel_err(outs[0], ref) <= 2 * REL_TOL
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    wg.free()
    wu.free()


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("N,K,B", [(128, 256, 1), (2048, 1024, 4), (1000, 768, 3), (4096, 2048, 2), (19000, 512, 1),
                                   (896, 4864, 4), (3584, 9472, 1), (4864, 1024, 16), (896, 4864, 9), (2048, 1024, 8),
                                   (1000, 768, 13)])
@pytest.mark.parametrize("s", ["", "1", "3"])
def test_streamed_tc_gemv_matches_oracle(ctx, monkeypatch, t, N, K, B, s):
    """The streamed tensor-core GEMV (k_qgemv_st, hd_gemv_stream.cu:
    128-row blocks walking K in lockstep through a ring of bulk-copied
    stages, persistent over blocks when they outnumber the SMs, K parts in a
    cluster otherwise; batch 5..16 in two or four MMA column blocks), forced
    with HACEDLE_GEMV_ST=1 onto small and ragged shapes, with bias and
    in-place residual; reruns bitwise equal."""
    monkeypatch.setenv("HACEDLE_GEMV_ST", "1")
    monkeypatch.setenv("HACEDLE_ST_S", s)
    outs, ref = _run(ctx, t, N, K, B, 900 + N + K + B + t, bias=True, residual=(B % 2 == 1), reps=2)
    assert np.isfinite(outs[0]).all()
    assert _rel_err(outs[0], ref) <= REL_TOL
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


@pytest.mark.parametrize("t,N,K,B", [(S.GGML_Q5_0, 18944, 3584, 16), (S.GGML_Q6_K, 1024, 18944, 11),
                                     (S.GGML_Q4_K, 3584, 3584, 16)])
def test_streamed_tc_gemv_batch_chunks(ctx, t, N, K, B):
    """Default routing at batch 5..16 on weights of 4 MB and more: the
    streamed kernel, in chunks of 8 or 4 batch rows where the whole batch's
    x fragments do not fit its shared memory (long K), with bias and
    in-place residual; reruns bitwise equal."""
    outs, ref = _run(ctx, t, N, K, B, 950 + B + t, bias=True, residual=True, reps=2)
    assert np.isfinite(outs[0]).all()
    assert _rel_err(outs[0], ref) <= REL_TOL
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
