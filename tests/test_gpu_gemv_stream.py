"""Decode Q-GEMV kernels of batch 1..4 for large matrices against the oracle:
the block kernel (k_qgemv_blk, the default for weights of 16 MB and more),
the tensor-core kernel (k_qgemv_mma) and the streamed CUDA-core kernel
(k_qgemv_sk), each forced onto every shape it fits.

The stream-K kernel gives every warp an equal contiguous range of the
flattened (32-row tile, unit) space; tiles split over several warps meet in
the workspace and the warp holding the last ticket adds the segments in
order.  HACEDLE_GEMV_SK=1 sends every plain batch <= 4 GEMV to it (by default
only weights of 16 MB and more go there); HACEDLE_SK_LMIN / HACEDLE_SK_WPB
change the grid so that tiles split into many short segments.  Bar: the fp32
contract ||y - y_ref||_inf <= 1e-5 ||y_ref||_inf, and bitwise-equal reruns.
"""
import numpy as np
import pytest

from hacedle_cuda import synth as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TYPES = [S.GGML_Q8_0, S.GGML_Q5_0, S.GGML_Q4_K, S.GGML_Q6_K]
REL_TOL = 1e-5


def _rel_err(y, ref):
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def _case(ctx, t, N, K, B, seed, bias=False, residual=False, reps=1):
    import torch
    raw = S.gen_weight(t, N, K, seed)
    X = S.gen_activations(B, K, seed + 1)
    w = ctx.weight(t, raw, N, K)
    x = torch.from_numpy(X).cuda()
    ref = O.qgemv(t, raw, N, K, X, threads=8)
    b = None
    if bias:
        bh = S.rng(seed + 2).standard_normal(N, dtype=np.float32) * np.float32(0.02)
        b = torch.from_numpy(bh).cuda()
        ref = ref + bh[None, :]
    rh = None
    if residual:
        rh = S.rng(seed + 3).standard_normal((B, N), dtype=np.float32)
        ref = rh + ref
    outs = []
    for _ in range(reps):
        if residual:
            y = torch.from_numpy(rh.copy()).cuda()  # in place: y = residual + W x
            ctx.qgemv(w, x, y, bias=b, residual=y)
        else:
            y = torch.full((B, N), float("nan"), dtype=torch.float32, device="cuda")
            ctx.qgemv(w, x, y, bias=b)
        ctx.check_device_errors()
        outs.append(y.cpu().numpy())
    w.free()
    return outs, ref


def _kernel(monkeypatch, kernel, lmin=""):
    """Route every batch <= 4 GEMV that fits to the block kernel (k_qgemv_blk),
    the tensor-core kernel (k_qgemv_mma) or the streamed CUDA-core kernel
    (k_qgemv_sk)."""
    monkeypatch.setenv("HACEDLE_GEMV_BLK", "1" if kernel == "blk" else "0")
    monkeypatch.setenv("HACEDLE_GEMV_MMA", "1" if kernel == "mma" else "0")
    monkeypatch.setenv("HACEDLE_GEMV_SK", "1")
    if lmin:
        monkeypatch.setenv("HACEDLE_MM_LMIN" if kernel == "mma" else "HACEDLE_SK_LMIN", lmin)


@pytest.mark.parametrize("kernel", ["blk", "mma", "sk"])
@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("N,K,B", [(7, 256, 1), (34, 512, 2), (100, 768, 3), (896, 1024, 4), (4866, 1280, 1),
                                   (896, 4864, 4), (257, 2304, 2), (4096, 8192, 1), (4865, 1280, 3)])
@pytest.mark.parametrize("lmin", ["", "1", "3"])
def test_streamed_gemv_matches_oracle(ctx, monkeypatch, kernel, t, N, K, B, lmin):
    _kernel(monkeypatch, kernel, lmin)
    outs, ref = _case(ctx, t, N, K, B, 500 + N + K + B + t)
    assert np.isfinite(outs[0]).all()
    assert _rel_err(outs[0], ref) <= REL_TOL


@pytest.mark.parametrize("kernel", ["blk", "mma", "sk"])
@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("wpb", ["1", "3", "8"])
def test_streamed_gemv_epilogues_and_reruns(ctx, monkeypatch, kernel, t, wpb):
    """bias, in-place residual, every batch 1..4, and three runs bitwise equal
    (tickets return to zero after every launch)."""
    _kernel(monkeypatch, kernel, "5")
    monkeypatch.setenv("HACEDLE_SK_WPB", wpb)
    for B in (1, 2, 3, 4):
        outs, ref = _case(ctx, t, 1000, 1024, B, 40 + B, bias=True, residual=(B % 2 == 0), reps=3)
        assert _rel_err(outs[0], ref) <= REL_TOL
        for o in outs[1:]:
            assert np.array_equal(outs[0].view(np.uint32), o.view(np.uint32))


@pytest.mark.parametrize("t,N,K", [(S.GGML_Q5_0, 18944, 3584), (S.GGML_Q4_K, 18944, 3584),
                                   (S.GGML_Q6_K, 3584, 18944), (S.GGML_Q8_0, 151936, 896)])
@pytest.mark.parametrize("B", [1, 4])
def test_streamed_gemv_large_shapes(ctx, t, N, K, B):
    """The large-matrix shapes (16 MB and more: the tensor-core kernel by
    default): 7B-shaped gate/up and down, and the tied LM head."""
    outs, ref = _case(ctx, t, N, K, B, 900 + t + B)
    assert _rel_err(outs[0], ref) <= REL_TOL


@pytest.mark.parametrize("t", TYPES)
def test_mma_gemv_extreme_activations(ctx, monkeypatch, t):
    """Units whose x spans many binades (the per-unit power-of-two scale and
    the fp16 hi/lo split), an all-zero unit, and huge and tiny magnitudes."""
    import torch
    _kernel(monkeypatch, "mma")
    N, K, B = 256, 1024, 3
    raw = S.gen_weight(t, N, K, 77)
    X = S.gen_activations(B, K, 78)
    X[0, :32] *= np.float32(1e-30)                    # a tiny unit
    X[1, 32:64] = 0.0                                 # a zero unit
    X[1, 64:96] *= np.float32(1e25)                   # a huge unit
    X[2, ::7] *= np.float32(1e6)                      # mixed magnitudes inside units
    w = ctx.weight(t, raw, N, K)
    y = torch.empty(B, N, device="cuda")
    ctx.qgemv(w, torch.from_numpy(X).cuda(), y)
    ctx.check_device_errors()
    ref = O.qgemv(t, raw, N, K, X, threads=8)
    for b in range(B):  # row by row: the rows' magnitudes differ by decades
        assert _rel_err(y.cpu().numpy()[b], ref[b]) <= REL_TOL, b
    w.free()
