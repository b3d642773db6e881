"""The device KV-cache manager (hd_kv_*): KvCacheManager bookkeeping with
the reference's KvError cases, slot-indexed appends, snapshot / restore
(branching) as device copies of every layer, and decode attention over
sessions in scattered slots against the oracle."""
import numpy as np
import pytest

import hacedle_cuda as hc
from oracle import oracle as O

pytestmark = pytest.mark.gpu

L, NKV, HD, CTX = 3, 2, 64, 48


def test_sessions_souls_and_errors(ctx):
    a = hc.KvArena(ctx, L, NKV, HD, CTX, slots=3)
    s0 = a.allocate("s0", "alice")
    s1 = a.allocate("s1", "alice")
    s2 = a.allocate("s2", "bob")
    assert len({s0, s1, s2}) == 3
    assert a.allocate("s0", "alice") == s0                  # get_or_create keeps the session
    assert a.soul_sessions("alice") == 2 and a.soul_sessions("bob") == 1
    with pytest.raises(hc.HdError) as e:
        a.allocate("s3", "bob")
    assert e.value.code == hc.HD_E_OOM and "AllocationFailed" in str(e.value)
    a.advance("s0", 40)
    with pytest.raises(hc.HdError) as e:
        a.advance("s0", 9)
    assert e.value.code == hc.HD_E_SHAPE and "ContextFull" in str(e.value)
    assert a.session("s0") == (s0, 40)
    with pytest.raises(hc.HdError) as e:
        a.session("nobody")
    assert e.value.code == hc.HD_E_ARG and "SessionNotFound" in str(e.value)
    a.release("s2")
    with pytest.raises(hc.HdError) as e:
        a.soul_sessions("bob")
    assert "SoulNotFound" in str(e.value)
    assert a.allocate("s3", "carol") == s2                   # the freed slot is reused
    a.free()


def _fill(a, torch, rng, session, tokens):
    slot, pos = a.session(session)
    ks, vs = [], []
    for li in range(L):
        k = torch.from_numpy(rng.standard_normal((tokens, NKV * HD)).astype(np.float32)).cuda()
        v = torch.from_numpy(rng.standard_normal((tokens, NKV * HD)).astype(np.float32)).cuda()
        sl = torch.full((tokens,), slot, dtype=torch.int32, device="cuda")
        ps = torch.arange(pos, pos + tokens, dtype=torch.int32, device="cuda")
        a.append(li, k, v, sl, ps)
        ks.append(k.cpu().numpy())
        vs.append(v.cpu().numpy())
    a.advance(session, tokens)
    return ks, vs


def test_snapshot_restore_branch_and_attention(ctx):
    import torch
    rng = np.random.default_rng(8)
    a = hc.KvArena(ctx, L, NKV, HD, CTX, slots=6)
    a.allocate("x", "soul")
    a.allocate("pad", "soul")
    a.allocate("y", "soul")
    k1, v1 = _fill(a, torch, rng, "x", 20)
    snap = a.snapshot("x")
    assert snap.token_position == 20
    k2, v2 = _fill(a, torch, rng, "x", 10)          # x continues past the snapshot
    a.restore(snap, "branch")                       # a new session from the snapshot
    assert a.session("branch")[1] == 20
    ky, vy = _fill(a, torch, rng, "y", 33)
    # decode attention of one query row per session, scattered slots
    sessions = ["x", "branch", "y"]
    slots = torch.tensor([a.session(s)[0] for s in sessions], dtype=torch.int32, device="cuda")
    lens = torch.tensor([a.session(s)[1] for s in sessions], dtype=torch.int32, device="cuda")
    nh = 6
    q = torch.from_numpy(rng.standard_normal((3, nh * HD)).astype(np.float32)).cuda()
    out = torch.empty(3, nh * HD, device="cuda")
    for li in range(L):
        a.attention(li, q, slots, lens, nh, out)
        got = out.cpu().numpy()
        keys = [np.concatenate([k1[li], k2[li]]), k1[li], ky[li]]
        vals = [np.concatenate([v1[li], v2[li]]), v1[li], vy[li]]
        for r in range(3):
            ref = O.attention_decode(q[r].cpu().numpy(), keys[r].reshape(-1, NKV, HD), vals[r].reshape(-1, NKV, HD),
                                     nh, NKV, HD)
            assert np.allclose(got[r], ref.reshape(-1), rtol=1e-5, atol=1e-6), (li, r)
    a.snapshot_free(snap)
    with pytest.raises(hc.HdError):
        a.restore(snap, "again")
    a.free()
