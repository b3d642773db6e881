"""CUDA RMSNorm, RoPE, softmax, SwiGLU, argmax, embedding, KV cache, GQA
attention, integer q-ops and the fp32 GEMMs against the oracle (B200).

Tolerances follow the reference's drift budget (golden/drift_budget.yaml):
rmsnorm / rope / silu 1e-6 absolute at unit scale; attention 1e-5; integer
ops bit-exact.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from hacedle_cuda import synth as S

pytestmark = pytest.mark.gpu


def T():
    import torch
    return torch


def cuda(a):
    return T().from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    T().cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("rows,dim", [(1, 896), (7, 3584), (3, 5), (2, 4864)])
def test_rmsnorm(ctx, rows, dim):
    g = S.rng(dim)
    x = g.standard_normal((rows, dim), dtype=np.float32) * np.float32(3)
    w = (1 + g.standard_normal(dim, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    y = T().empty(rows, dim, device="cuda")
    ctx.rmsnorm(cuda(x), cuda(w), y, 1e-6)
    ref = O.rmsnorm(x, w, 1e-6)
    assert np.abs(host(y) - ref).max() <= 2e-6 * np.abs(ref).max()
    # fused residual add: residual += x, y = rmsnorm(residual)
    r = g.standard_normal((rows, dim), dtype=np.float32)
    rd = cuda(r)
    ctx.rmsnorm(cuda(x), cuda(w), y, 1e-6, residual=rd)
    s = (r + x).astype(np.float32)
    assert np.array_equal(host(rd), s)
    ref = O.rmsnorm(s, w, 1e-6)
    assert np.abs(host(y) - ref).max() <= 2e-6 * np.abs(ref).max()
    # graph-executor variant (eps 1e-5, v*inv*w order)
    ctx.rmsnorm_graph(cuda(x), cuda(w), y, 1e-5)
    ref = O.rmsnorm_graph(x, w, 1e-5)
    assert np.abs(host(y) - ref).max() <= 2e-6 * np.abs(ref).max()


def test_rope_neox_golden_and_oracle(ctx, golden_dir):
    x = np.fromfile(os.path.join(golden_dir, "rope_in.f32"), np.float32)
    for pos in (0, 1, 128, 1024):
        xd = cuda(x[None].copy())
        ctx.rope_neox(xd, cuda(np.array([pos], np.int32)), 1, 64)
        exp = np.fromfile(os.path.join(golden_dir, f"rope_pos{pos}.f32"), np.float32)
        y = host(xd)[0]
        assert np.abs(y - O.rope_neox(x[None], np.array([pos]), 64)[0]).max() <= 1e-6
        assert np.abs(y - exp).max() <= 1e-5
    # 14 heads x 64 over 512 positions, and head_dim 128 (7B shape)
    for heads, hd, Tn in ((14, 64, 512), (28, 128, 7)):
        g = S.rng(heads)
        q = g.standard_normal((Tn, heads * hd), dtype=np.float32)
        pos = np.arange(Tn, dtype=np.int32) * 3
        qd = cuda(q)
        ctx.rope_neox(qd, cuda(pos), heads, hd)
        ref = O.rope_neox(q, pos, hd)
        assert np.abs(host(qd) - ref).max() <= 2e-5


def test_rope_interleaved(ctx):
    g = S.rng(3)
    x = g.standard_normal((5, 64), dtype=np.float32)
    ang = g.uniform(0, 6.3, (5, 64)).astype(np.float32)
    c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    out = T().empty(5, 64, device="cuda")
    ctx.rope_interleaved(cuda(x), cuda(c), cuda(s), out)
    assert np.array_equal(host(out), O.rope_interleaved(x, c, s))


def test_softmax_swiglu_add(ctx):
    g = S.rng(4)
    x = g.standard_normal((14, 640), dtype=np.float32) * np.float32(4)
    xd = cuda(x)
    ctx.softmax_rows(xd)
    ref = np.stack([O.softmax(r) for r in x])
    assert np.abs(host(xd) - ref).max() <= 1e-6
    a, b = g.standard_normal(4864, dtype=np.float32) * 5, g.standard_normal(4864, dtype=np.float32)
    y = T().empty(4864, device="cuda")
    ctx.swiglu(cuda(a), cuda(b), y)
    assert np.abs(host(y) - O.swiglu(a, b)).max() <= 1e-6 * np.abs(O.swiglu(a, b)).max() + 1e-7
    ctx.add(cuda(a), cuda(b), y)
    assert np.array_equal(host(y), O.add_f32(a, b))


@pytest.mark.parametrize("n", [1, 7, 8192, 8193, 151936, 2_000_000])
def test_argmax_first_max_wins(ctx, n):
    g = S.rng(n)
    x = g.standard_normal((3, n), dtype=np.float32)
    if n > 10:
        x[0, [5, n - 1]] = 100.0      # tie: the lower index wins
        x[1, 0] = np.nan              # NaN at 0: the scan never moves
        x[2, n // 2] = np.inf
    idx = T().empty(3, dtype=T().int32, device="cuda")
    ctx.argmax_rows(cuda(x), idx)
    got = host(idx)
    assert [int(v) for v in got] == [O.argmax(r) for r in x]


def test_embed_rows_and_out_of_range(ctx):
    t = S.GGML_Q8_0
    raw = S.gen_weight(t, 1000, 896, 8)
    w = ctx.weight(t, raw, 1000, 896)
    ids = np.array([0, 999, 17, 1000, -1, 512], np.int32)
    out = T().empty(ids.size, 896, device="cuda")
    ctx.embed(w, cuda(ids), out)
    full = O.dequantize(t, raw, 1000 * 896)
    for i, tok in enumerate(ids):
        exp = O.embedding_lookup(int(tok) & 0xFFFFFFFF, full, 1000, 896)
        assert np.array_equal(host(out)[i], exp)


def _attn_ref(q, kc, vc, L, nh, nkv, hd):
    return O.attention_decode(q, kc[:L], vc[:L], nh, nkv, hd)


@pytest.mark.parametrize("nh,nkv,hd,max_ctx", [(14, 2, 64, 640), (28, 4, 128, 300), (8, 8, 32, 64)])
def test_kv_append_and_decode_attention(ctx, nh, nkv, hd, max_ctx):
    g = S.rng(nh + hd)
    seqs = 3
    lens = np.array([1, max_ctx // 2, max_ctx], np.int32)
    kc = T().zeros(seqs, max_ctx, nkv, hd, device="cuda")
    vc = T().zeros(seqs, max_ctx, nkv, hd, device="cuda")
    K = g.standard_normal((seqs, max_ctx, nkv, hd), dtype=np.float32)
    Vv = g.standard_normal((seqs, max_ctx, nkv, hd), dtype=np.float32)
    ctx.kv_append(cuda(K), cuda(Vv), kc, vc, cuda(np.zeros(seqs, np.int32)), seqs, max_ctx, nkv, hd, max_ctx)
    assert np.array_equal(host(kc), K) and np.array_equal(host(vc), Vv)
    q = g.standard_normal((seqs, nh * hd), dtype=np.float32) * np.float32(2)
    out = T().empty(seqs, nh * hd, device="cuda")
    ctx.attention_decode(cuda(q), kc, vc, cuda(lens), nh, nkv, hd, max_ctx, out)
    got = host(out)
    for s in range(seqs):
        ref = _attn_ref(q[s], K[s], Vv[s], lens[s], nh, nkv, hd)
        assert np.abs(got[s] - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_kv_append_single_token_positions(ctx):
    kc = T().zeros(2, 16, 2, 64, device="cuda")
    vc = T().zeros(2, 16, 2, 64, device="cuda")
    k = T().ones(2, 1, 2, 64, device="cuda")
    pos = cuda(np.array([3, 15], np.int32))
    ctx.kv_append(k, k * 2, kc, vc, pos, 2, 1, 2, 64, 16)
    h = host(kc)
    assert h[0, 3].min() == 1 and h[1, 15].min() == 1 and h.sum() == 2 * 128
    assert host(vc).sum() == 4 * 128


def test_prefill_attention_causal(ctx):
    nh, nkv, hd, Tn, max_ctx = 14, 2, 64, 96, 128
    g = S.rng(9)
    K = g.standard_normal((1, max_ctx, nkv, hd), dtype=np.float32)
    Vv = g.standard_normal((1, max_ctx, nkv, hd), dtype=np.float32)
    q = g.standard_normal((Tn, nh * hd), dtype=np.float32)
    out = T().empty(Tn, nh * hd, device="cuda")
    pos0 = 5
    ctx.attention_prefill(cuda(q), cuda(K), cuda(Vv), Tn, pos0, nh, nkv, hd, max_ctx, out)
    got = host(out)
    for t in (0, 1, 50, Tn - 1):
        ref = _attn_ref(q[t], K[0], Vv[0], pos0 + t + 1, nh, nkv, hd)
        assert np.abs(got[t] - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_int8_dot_and_fused(ctx):
    g = S.rng(12)
    for n in (0, 1, 31, 32, 33, 4096, 300001):
        a = g.integers(-128, 128, (4, n), dtype=np.int8)
        b = g.integers(-128, 128, (4, n), dtype=np.int8)
        out = T().empty(4, dtype=T().int32, device="cuda")
        ctx.dot_i8(cuda(a), cuda(b), out)
        assert [int(v) for v in host(out)] == [O.dot_i8(a[i], b[i]) for i in range(4)]
    a = np.full((2, 300000), 127, np.int8)
    bias = np.array([5, -7], np.int32)
    carry = cuda(np.array([7, 2**31 - 1], np.int32))
    out = T().empty(2, dtype=T().int32, device="cuda")
    for _ in range(2):
        ctx.fused_qdot_qadd_qacc_i8(cuda(a), cuda(a), cuda(bias), carry, out)
    c0 = [7, 2**31 - 1]
    for _ in range(2):
        r = [O.fused_qdot_qadd_qacc_i8(a[i], a[i], int(bias[i]), c0[i]) for i in range(2)]
        c0 = [x[1] for x in r]
    assert [int(v) for v in host(out)] == [x[0] for x in r]
    assert [int(v) for v in host(carry)] == c0


def test_matmul_f32_dense(ctx):
    g = S.rng(13)
    a = g.standard_normal((70, 130), dtype=np.float32)
    b = g.standard_normal((130, 33), dtype=np.float32)
    out = T().empty(70, 33, device="cuda")
    ctx.matmul_f32(cuda(a), cuda(b), out)
    ref = O.matmul_f32(a, b)
    assert np.abs(host(out) - ref).max() <= 1e-5 * np.abs(ref).max()


@pytest.mark.parametrize("t,N,K", [(S.GGML_Q5_0, 4864, 896), (S.GGML_Q4_K, 896, 4864), (S.GGML_Q6_K, 200, 512),
                                   (S.GGML_Q8_0, 130, 96)])
@pytest.mark.parametrize("Tn", [1, 77, 128])
def test_qgemm_fp32_exact_weights(ctx, t, N, K, Tn):
    raw = S.gen_weight(t, N, K, 40 + t)
    X = S.gen_activations(Tn, K, 41)
    w = ctx.weight(t, raw, N, K)
    Y = T().empty(Tn, N, device="cuda")
    ctx.qgemm(w, cuda(X), Y, precision=0)
    ref = O.qgemv(t, raw, N, K, X, threads=8)
    got = host(Y)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()
    assert np.array_equal(ctx.qgemm_host(w, X, precision=0).view(np.uint32), got.view(np.uint32))


@pytest.mark.parametrize("G,B,n", [(1, 1, 4), (2, 5, 1792), (8, 3, 64), (3, 7, 33), (2, 512, 9472)])
def test_gather_columns(ctx, G, B, n):
    """[G][B][n] rank blocks -> [B][G*n] rows (the row-sharded layer's
    reassembly after the all-gather): float4 path when n % 4 == 0, scalar
    otherwise; bit-exact copy."""
    from hacedle_cuda import shard
    src = np.random.default_rng(G * 1000 + B + n).standard_normal((G, B, n), dtype=np.float32)
    dst = T().empty(B, G * n, device="cuda")
    ctx.gather_columns(cuda(src), dst, G, B, n)
    T().cuda.synchronize()
    assert np.array_equal(host(dst), shard.gather_columns_reference(src, G, B, n))
