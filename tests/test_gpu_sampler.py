"""Device logits processor and sampler against the oracle.

hd_logits_process must equal oracle.logits_process bit for bit (masks and the
temperature-divided values), over vocab-sized rows and the reference's edge
cases.  hd_sample_rows must draw the oracle's index wherever the target is
more than 1e-5 of the row mass from an interval edge (closer, the f32 exp of
the device and of numpy may round the partial sums differently), reproduce its
draws for the same seed and counter, and follow softmax(logits) in
distribution."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,n", [(4, 151936), (3, 1000), (1, 7)])
@pytest.mark.parametrize("scale,t,top_p,top_k", [(3.0, 0.7, 0.9, 0), (3.0, 1.0, 0.9, 50), (0.5, 1.3, 0.95, 40),
                                                 (-1.0, 1.0, 0.9, 0), (1.0, 0.0, 0.9, 3), (1.0, 1.0, 2.0, 0),
                                                 (2.0, 1.0, 1.0, 6)])
def test_logits_process_matches_oracle(ctx, rows, n, scale, t, top_p, top_k):
    import torch
    rng = np.random.default_rng(rows * 7 + n)
    x = (rng.standard_normal((rows, n)) * abs(scale)).astype(np.float32)
    if scale < 0:
        x = (x - np.float32(np.log(n)) - 1.0).astype(np.float32)   # log-probability-like: long top-p walks
    d = torch.from_numpy(x).cuda()
    ctx.logits_process(d, t, top_p, top_k)
    got = d.cpu().numpy()
    want = O.logits_process(x, t, top_p, top_k)
    assert np.array_equal(np.isinf(got), np.isinf(want))
    assert np.array_equal(got[np.isfinite(want)], want[np.isfinite(want)])


def test_sample_matches_oracle_and_reproduces(ctx):
    import torch
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((64, 5000)) * 2.0).astype(np.float32)
    x[5, :] = -np.inf
    x[6, :] = -np.inf
    x[6, 4321] = 1.0
    d = torch.from_numpy(x).cuda()
    idx = torch.empty(64, dtype=torch.int32, device="cuda")
    ctx.sample(d, idx, seed=1234, offset=77)
    got = idx.cpu().numpy()
    want, margin = O.sample_rows(x, seed=1234, offset=77)
    sure = margin > 1e-5
    assert sure.sum() >= 60
    assert np.array_equal(got[sure], want[sure])
    assert got[5] == -1 and got[6] == 4321
    idx2 = torch.empty_like(idx)
    ctx.sample(d, idx2, seed=1234, offset=77)
    assert torch.equal(idx, idx2)
    ctx.sample(d, idx2, seed=1234, offset=78)
    assert not torch.equal(idx, idx2)


def test_sample_follows_softmax(ctx):
    import torch
    logits = np.array([2.0, 1.0, 0.5, 0.0, -1.0, -np.inf, 1.5, -3.0], np.float32)
    R = 20000
    d = torch.from_numpy(np.tile(logits, (R, 1))).cuda()
    idx = torch.empty(R, dtype=torch.int32, device="cuda")
    ctx.sample(d, idx, seed=99)
    counts = np.bincount(idx.cpu().numpy(), minlength=8)
    p = np.exp(logits - logits.max())
    p /= p.sum()
    assert counts[5] == 0
    sigma = np.sqrt(R * p * (1 - p))
    assert np.all(np.abs(counts - R * p) <= 5 * sigma + 1), (counts, R * p)


def test_process_then_sample_top_k_one_is_argmax(ctx):
    import torch
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((8, 3000)) * 3).astype(np.float32)
    d = torch.from_numpy(x).cuda()
    ctx.logits_process(d, 1.0, 2.0, 1)       # top_k = 1 keeps the two largest (the reference's k+1)
    idx = torch.empty(8, dtype=torch.int32, device="cuda")
    ctx.sample(d, idx, seed=3)
    top2 = np.argsort(-x, axis=1)[:, :2]
    assert all(int(i) in set(t) for i, t in zip(idx.cpu().numpy(), top2))
