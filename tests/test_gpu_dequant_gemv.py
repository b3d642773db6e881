"""CUDA dequant and decode Q-GEMV against the oracle (B200).

Dequantized weights must be bit-exact.  GEMV outputs must be within 1e-5
relative of the oracle's sequential-sum GEMV, norm-wise:
||y - y_ref||_inf <= 1e-5 * ||y_ref||_inf (the fp32-accumulate contract).
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from hacedle_cuda import synth as S

pytestmark = pytest.mark.gpu
TYPES = [S.GGML_Q8_0, S.GGML_Q5_0, S.GGML_Q4_K, S.GGML_Q6_K]
NAMES = {S.GGML_Q8_0: "q8_0", S.GGML_Q5_0: "q5_0", S.GGML_Q4_K: "q4_k", S.GGML_Q6_K: "q6_k"}
REL_TOL = 1e-5


def _torch():
    import torch
    return torch


def _dequant_gpu(ctx, w, rows, cols):
    torch = _torch()
    out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    ctx.dequantize(w, out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _rel_err(y, ref):
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("t", TYPES)
def test_golden_blocks_bit_exact(ctx, golden_dir, t):
    nm = NAMES[t]
    for kind in ("ref_{}_block", "gguf_{}_rand", "gguf_{}_edge"):
        base = kind.format(nm)
        if kind.startswith("ref"):
            raw = np.fromfile(os.path.join(golden_dir, base + ".raw"), np.uint8)
            exp = np.fromfile(os.path.join(golden_dir, base + ".f32"), np.float32)
        else:
            raw = np.fromfile(os.path.join(golden_dir, base + ".raw"), np.uint8)
            exp = np.fromfile(os.path.join(golden_dir, base + ".f32"), np.float32)
        be, bb = S.BLOCK[t]
        nblk = raw.size // bb
        cols = be if kind.startswith("ref") or kind.endswith("edge") else 512
        rows = nblk * be // cols
        w = ctx.weight(t, raw, rows, cols)
        y = _dequant_gpu(ctx, w, rows, cols)
        same = (y.view(np.uint32) == exp.view(np.uint32)) | (np.isnan(y) & np.isnan(exp))
        assert same.all(), base
        assert np.array_equal(w.download(), raw), base


@pytest.mark.parametrize("t,N,K", [(S.GGML_Q8_0, 896, 896), (S.GGML_Q5_0, 4864, 896), (S.GGML_Q6_K, 896, 4864),
                                   (S.GGML_Q4_K, 896, 4864), (S.GGML_Q5_0, 37, 96), (S.GGML_Q4_K, 3, 512)])
def test_dequant_full_tensor_bit_exact_and_round_trip(ctx, t, N, K):
    raw = S.gen_weight(t, N, K, 1234 + t)
    w = ctx.weight(t, raw, N, K)
    y = _dequant_gpu(ctx, w, N, K)
    ref = O.dequantize(t, raw, N * K)
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(w.download(), raw.reshape(-1))


def test_dequant_random_bytes_bit_exact(ctx):
    # Any byte pattern is a block (subnormal, inf and NaN scales included).
    g = np.random.default_rng(5)
    for t in TYPES:
        be, bb = S.BLOCK[t]
        raw = g.integers(0, 256, (16, (512 // be) * bb), dtype=np.uint8)
        w = ctx.weight(t, raw, 16, 512)
        y = _dequant_gpu(ctx, w, 16, 512)
        ref = O.dequantize(t, raw, 16 * 512)
        same = (y.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(y) & np.isnan(ref))
        assert same.all()
        assert np.array_equal(w.download(), raw.reshape(-1))


def test_upload_rejects_bad_shapes(ctx):
    import hacedle_cuda as hc
    raw = S.gen_weight(S.GGML_Q8_0, 4, 64, 1)
    with pytest.raises(hc.HdError) as e:
        ctx.weight(S.GGML_Q8_0, raw, 4, 48)
    assert e.value.code == hc.HD_E_SHAPE
    with pytest.raises(hc.HdError) as e:
        ctx.weight(S.GGML_Q8_0, raw[:, :-1], 4, 64)
    assert e.value.code == hc.HD_E_SHAPE
    with pytest.raises(hc.HdError) as e:
        ctx.weight(2, raw, 4, 64)  # Q4_0: not on this path
    assert e.value.code == hc.HD_E_TYPE


def _gemv_case(ctx, t, N, K, B, seed, bias=False, residual=False):
    torch = _torch()
    raw = S.gen_weight(t, N, K, seed)
    X = S.gen_activations(B, K, seed + 1)
    w = ctx.weight(t, raw, N, K)
    x = torch.from_numpy(X).cuda()
    y = torch.empty(B, N, dtype=torch.float32, device="cuda")
    ref = O.qgemv(t, raw, N, K, X, threads=8)
    b = r = None
    if bias:
        bh = S.rng(seed + 2).standard_normal(N, dtype=np.float32) * np.float32(0.02)
        b = torch.from_numpy(bh).cuda()
        ref = ref + bh[None, :]
    if residual:
        rh = S.rng(seed + 3).standard_normal((B, N), dtype=np.float32)
        r = torch.from_numpy(rh).cuda()
        y = r  # in place: y = residual + W x
        ref = rh + ref
    ctx.qgemv(w, x, y, bias=b, residual=r)
    torch.cuda.synchronize()
    return y.cpu().numpy(), ref


@pytest.mark.parametrize("t,N,K", [(S.GGML_Q8_0, 896, 896), (S.GGML_Q5_0, 4864, 896), (S.GGML_Q6_K, 896, 4864),
                                   (S.GGML_Q4_K, 896, 4864)])
@pytest.mark.parametrize("B", [1, 4, 16])
def test_gemv_config_shapes(ctx, t, N, K, B):
    y, ref = _gemv_case(ctx, t, N, K, B, 10 + t)
    assert _rel_err(y, ref) <= REL_TOL


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("N,K,B", [(1, 256, 1), (100, 512, 3), (129, 256, 2), (300, 768, 5), (257, 2304, 7),
                                   (64, 256, 16), (1000, 256, 9)])
def test_gemv_ragged_shapes(ctx, t, N, K, B):
    y, ref = _gemv_case(ctx, t, N, K, B, 77 + N + K + B)
    assert _rel_err(y, ref) <= REL_TOL


@pytest.mark.parametrize("t", [S.GGML_Q5_0, S.GGML_Q6_K])
def test_gemv_bias_and_residual_epilogues(ctx, t):
    K = 896 if t == S.GGML_Q5_0 else 4864
    y, ref = _gemv_case(ctx, t, 1152, K, 1, 5, bias=True)
    assert _rel_err(y, ref) <= REL_TOL
    y, ref = _gemv_case(ctx, t, 896, K, 4, 6, residual=True)
    assert _rel_err(y, ref) <= REL_TOL


@pytest.mark.parametrize("B", [1, 2, 4, 8, 16])
def test_gemv_swiglu_pair(ctx, B):
    torch = _torch()
    N, K = 4864, 896
    rg, ru = S.gen_weight(S.GGML_Q5_0, N, K, 21), S.gen_weight(S.GGML_Q5_0, N, K, 22)
    X = S.gen_activations(B, K, 23)
    wg, wu = ctx.weight(S.GGML_Q5_0, rg, N, K), ctx.weight(S.GGML_Q5_0, ru, N, K)
    x = torch.from_numpy(X).cuda()
    y = torch.empty(B, N, dtype=torch.float32, device="cuda")
    ctx.qgemv_swiglu(wg, wu, x, y)
    torch.cuda.synchronize()
    g = O.qgemv(S.GGML_Q5_0, rg, N, K, X, threads=8)
    u = O.qgemv(S.GGML_Q5_0, ru, N, K, X, threads=8)
    ref = O.swiglu(g, u).reshape(B, N)
    assert _rel_err(y.cpu().numpy(), ref) <= 2 * REL_TOL


def test_gemv_deterministic_and_host_entry(ctx):
    torch = _torch()
    t, N, K = S.GGML_Q4_K, 896, 4864
    raw = S.gen_weight(t, N, K, 99)
    X = S.gen_activations(4, K, 98)
    w = ctx.weight(t, raw, N, K)
    x = torch.from_numpy(X).cuda()
    ys = []
    for _ in range(3):
        y = torch.empty(4, N, dtype=torch.float32, device="cuda")
        ctx.qgemv(w, x, y)
        ys.append(y.cpu().numpy())
    assert all(np.array_equal(ys[0].view(np.uint32), a.view(np.uint32)) for a in ys[1:])
    yh = ctx.qgemv_host(w, X)
    assert np.array_equal(yh.view(np.uint32), ys[0].view(np.uint32))


def test_gemv_lm_head_q8_0(ctx):
    # The tied LM head shape: 151936 x 896 Q8_0 (144.6 MB), batch 1.
    y, ref = _gemv_case(ctx, S.GGML_Q8_0, 151936, 896, 1, 314)
    assert _rel_err(y, ref) <= REL_TOL


@pytest.mark.parametrize("t,N,K,B,bias,residual", [(S.GGML_Q5_0, 1152, 896, 8, True, False),
                                                    (S.GGML_Q4_K, 896, 4864, 12, False, True),
                                                    (S.GGML_Q6_K, 4864, 4864, 16, True, True),
                                                    (S.GGML_Q8_0, 384, 2048, 6, False, False),
                                                    (S.GGML_Q5_0, 19000, 512, 16, False, True),
                                                    (S.GGML_Q4_K, 18944, 256, 9, True, False)])
@pytest.mark.parametrize("tensor_cores", [True, False])
def test_gemv_batched_register_blocked(ctx, monkeypatch, t, N, K, B, bias, residual, tensor_cores):
    """Batch 5..16: epilogues and bitwise-stable reruns, through the tensor-core
    kernel where the shape fits it and, with it switched off, through the
    register-blocked CUDA-core kernel (the K split over CTAs, the
    one-CTA-per-tile mode of tall matrices with >= 148 tiles of 128 rows)."""
    torch = _torch()
    monkeypatch.setenv("HACEDLE_GEMV_ST", "0")   # the streamed kernel has its own tests
    if not tensor_cores:
        monkeypatch.setenv("HACEDLE_GEMV_TC", "0")
    y, ref = _gemv_case(ctx, t, N, K, B, 200 + B, bias=bias, residual=residual)
    assert _rel_err(y, ref) <= REL_TOL
    raw = S.gen_weight(t, N, K, 300 + B)
    w = ctx.weight(t, raw, N, K)
    x = torch.from_numpy(S.gen_activations(B, K, 301)).cuda()
    y1 = torch.empty(B, N, device="cuda")
    y2 = torch.empty(B, N, device="cuda")
    ctx.qgemv(w, x, y1)
    ctx.qgemv(w, x, y2)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


# Tensor-core batch kernel: K parts S (1 = no cluster, 16 = the largest
# cluster), units per part up to 16 (the accumulator ring reused for Q6_K's
# half-unit groups and past 8 units), ragged row tiles, batch 5 and 16.
@pytest.mark.parametrize("t,N,K,B,parts", [(S.GGML_Q5_0, 4864, 512, 16, "1"), (S.GGML_Q8_0, 300, 2048, 5, "4"),
                                           (S.GGML_Q6_K, 896, 4864, 16, "16"), (S.GGML_Q4_K, 384, 4096, 12, "8"),
                                           (S.GGML_Q6_K, 257, 2048, 7, "4"), (S.GGML_Q8_0, 4864, 896, 9, ""),
                                           (S.GGML_Q5_0, 896, 4864, 13, ""), (S.GGML_Q8_0, 1000, 512, 16, "3")])
def test_gemv_tensor_core_k_parts(ctx, monkeypatch, t, N, K, B, parts):
    """Batch 5..16 on the tensor cores (exact integer weights times an exact
    three-way bf16 split of x, fp32 scales per group) against the oracle, with
    bias and residual epilogues, and bitwise-equal reruns."""
    torch = _torch()
    monkeypatch.setenv("HACEDLE_GEMV_ST", "0")   # the streamed kernel has its own tests
    if parts:
        monkeypatch.setenv("HACEDLE_GEMV_TC_S", parts)
    y, ref = _gemv_case(ctx, t, N, K, B, 500 + B, bias=True, residual=(B % 2 == 1))
    assert _rel_err(y, ref) <= REL_TOL
    w = ctx.weight(t, S.gen_weight(t, N, K, 600 + B), N, K)
    x = torch.from_numpy(S.gen_activations(B, K, 601)).cuda()
    y1 = torch.empty(B, N, device="cuda")
    y2 = torch.empty(B, N, device="cuda")
    ctx.qgemv(w, x, y1)
    ctx.qgemv(w, x, y2)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    ctx.check_device_errors()


@pytest.mark.parametrize("t,N,K,B", [(S.GGML_Q5_0, 1152, 896, 1), (S.GGML_Q5_0, 896, 896, 3), (S.GGML_Q8_0, 896, 896, 4),
                                     (S.GGML_Q6_K, 512, 768, 9), (S.GGML_Q4_K, 384, 512, 16)])
def test_gemv_fused_rmsnorm(ctx, t, N, K, B):
    """hd_qgemv_rmsnorm (the norm in each CTA's prologue) against the oracle's
    RMSNorm followed by its GEMV, with bias and in-place residual."""
    torch = _torch()
    raw = S.gen_weight(t, N, K, 400 + B)
    X = S.gen_activations(B, K, 401)
    nw = (1.0 + 0.02 * S.rng(402).standard_normal(K)).astype(np.float32)
    bh = (0.02 * S.rng(403).standard_normal(N)).astype(np.float32)
    rh = S.rng(404).standard_normal((B, N), dtype=np.float32)
    xn = O.rmsnorm(X, nw, 1e-6).reshape(B, K)
    ref = rh + (O.qgemv(t, raw, N, K, xn, threads=8) + bh[None, :])
    w = ctx.weight(t, raw, N, K)
    y = torch.from_numpy(rh.copy()).cuda()
    ctx.qgemv_norm(w, torch.from_numpy(X).cuda(), torch.from_numpy(nw).cuda(), y, bias=torch.from_numpy(bh).cuda(),
                   residual=y)
    torch.cuda.synchronize()
    assert _rel_err(y.cpu().numpy(), ref) <= REL_TOL


@pytest.mark.parametrize("B", [1, 4, 12])
def test_gemv_fused_rmsnorm_swiglu_pair(ctx, B):
    torch = _torch()
    N, K = 4864, 896
    rg, ru = S.gen_weight(S.GGML_Q5_0, N, K, 410), S.gen_weight(S.GGML_Q5_0, N, K, 411)
    X = S.gen_activations(B, K, 412)
    nw = (1.0 + 0.02 * S.rng(413).standard_normal(K)).astype(np.float32)
    xn = O.rmsnorm(X, nw, 1e-6).reshape(B, K)
    ref = O.swiglu(O.qgemv(S.GGML_Q5_0, rg, N, K, xn, threads=8), O.qgemv(S.GGML_Q5_0, ru, N, K, xn, threads=8))
    wg, wu = ctx.weight(S.GGML_Q5_0, rg, N, K), ctx.weight(S.GGML_Q5_0, ru, N, K)
    y = torch.empty(B, N, device="cuda")
    ctx.qgemv_norm(wg, torch.from_numpy(X).cuda(), torch.from_numpy(nw).cuda(), y, w_up=wu)
    torch.cuda.synchronize()
    assert _rel_err(y.cpu().numpy(), ref.reshape(B, N)) <= 2 * REL_TOL
