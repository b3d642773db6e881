"""hd_qgemm_kt: the Q-GEMM in the operand layout of ComputeBackend::matmul_q4k /
matmul_q6k (src/quant_view/dequant_dispatcher.rs:28-64): a = the quantized
weight [m, k], b [k, n] row-major, out [m, n] row-major with
out[i][j] = sum_l a[i][l] b[l][j].  b is either f32 or itself quantized, as
the trait's QuantTensorView b is; a quantized b is dequantized on the device
(hd_dequantize gives its [k][n] f32 values directly).  The layout is
checked exactly: the result is bitwise hd_qgemm's on the transposed
operands.  Against the reference's loop, norm-wise: the bf16 contract 2e-2;
fp32 1e-5, except at K = 4864, where the fp32-accuracy tensor-core mode's
fp32 accumulation over 304 K steps measures 1.06e-5 from the float64
product (the oracle's sequential sum: 3e-6) -- bound 1.5e-5 there."""
import numpy as np
import pytest

import hacedle_cuda as hc
from hacedle_cuda import synth as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _rel(y, ref):
    return float(np.abs(y - ref).max() / np.abs(ref).max())


@pytest.mark.parametrize("t,m,k", [(S.GGML_Q4_K, 896, 4864), (S.GGML_Q6_K, 256, 512), (S.GGML_Q5_0, 130, 96),
                                   (S.GGML_Q8_0, 4864, 896)])
@pytest.mark.parametrize("n", [1, 7, 64, 300])
@pytest.mark.parametrize("prec,tol", [(hc.PREC_FP32, 1e-5), (hc.PREC_BF16_TC, 2e-2)])
def test_qgemm_kt_matches_matmul_q4k_loop(ctx, t, m, k, n, prec, tol):
    import torch
    raw = S.gen_weight(t, m, k, 3 + n)
    b = S.gen_activations(k, n, 4 + n)            # [k, n] row-major
    w = ctx.weight(t, raw, m, k)
    out = torch.full((m, n), float("nan"), device="cuda")
    ctx.qgemm_kt(w, torch.from_numpy(b).cuda(), out, precision=prec)
    ctx.check_device_errors()
    a = O.dequantize(t, raw, m * k).reshape(m, k)
    ref = O.matmul_f32(a, b)                      # out[i][j] = sum_l a[i][l] b[l][j], sequential in l
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    # the same product through hd_qgemm on token-major operands, bit for bit
    ytn = torch.empty(n, m, device="cuda")
    ctx.qgemm(w, torch.from_numpy(np.ascontiguousarray(b.T)).cuda(), ytn, precision=prec)
    assert np.array_equal(got.view(np.uint32), np.ascontiguousarray(ytn.cpu().numpy().T).view(np.uint32))
    if prec == hc.PREC_FP32 and k > 1024:
        tol = 1.5e-5
    assert _rel(got, ref) <= tol
    # the host entry point, host buffers in the same layouts
    assert np.array_equal(ctx.qgemm_kt_host(w, b, precision=prec).view(np.uint32), got.view(np.uint32))
    w.free()


def test_qgemm_kt_quantized_b(ctx):
    """b quantized (Q8_0 [k, n], n a multiple of 32): dequantized on the
    device into [k][n], then the product -- both operands dequantized, as
    NativeBackend::matmul_q4k does."""
    import torch
    m, k, n = 512, 1024, 96
    ra = S.gen_weight(S.GGML_Q4_K, m, k, 11)
    rb = S.gen_weight(S.GGML_Q8_0, k, n, 12)
    wa = ctx.weight(S.GGML_Q4_K, ra, m, k)
    wb = ctx.weight(S.GGML_Q8_0, rb, k, n)
    bd = torch.empty(k * n, device="cuda")
    ctx.dequantize(wb, bd)
    out = torch.empty(m, n, device="cuda")
    ctx.qgemm_kt(wa, bd.view(k, n), out)
    ctx.check_device_errors()
    ref = O.matmul_f32(O.dequantize(S.GGML_Q4_K, ra, m * k).reshape(m, k),
                       O.dequantize(S.GGML_Q8_0, rb, k * n).reshape(k, n))
    assert _rel(out.cpu().numpy(), ref) <= 1e-5
    wa.free()
    wb.free()
