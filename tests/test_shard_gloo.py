"""Row-sharded projection over 2 CPU ranks (gloo): each rank slices its rows
out of the GGUF bytes, computes its part with the oracle, the ranks all-gather,
and the reassembled output equals the unsharded product bit for bit (rows are
independent sums, so sharding does not change any row's arithmetic)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys

    sys.path[:0] = [ROOT, os.path.join(ROOT, "hace-fem-hacedle_b200", "python")]
    import datetime

    import torch
    import torch.distributed as dist

    from hacedle_cuda import shard, synth as S
    from oracle import oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        res = {}
        for t, N, K in ((S.GGML_Q4_K, 64, 512), (S.GGML_Q6_K, 32, 768), (S.GGML_Q5_0, 96, 256)):
            raw = S.gen_weight(t, N, K, seed=5 + t)
            X = S.gen_activations(3, K, seed=6)
            part = shard.row_slice(raw, t, N, K, rank, world)
            n = N // world
            y = torch.from_numpy(O.qgemv(t, part, n, K, X))           # [B][n]
            out = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(out, y)
            full = shard.gather_columns_reference(torch.stack(out).numpy(), world, 3, n)
            res[t] = bool(np.array_equal(full, O.qgemv(t, raw, N, K, X)))
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_row_sharded_projection_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, res in got:
        assert all(res.values()), (rank, res)


def test_row_range_rejects_uneven_split():
    from hacedle_cuda import shard

    assert shard.row_range(3584, 3, 8) == (1344, 1792)
    with pytest.raises(ValueError):
        shard.row_range(100, 0, 8)


def test_exchange_layout():
    """PeerExchange buffer layout: the int32 flag array [world] first, then two
    full outputs [B][N] per projection (consecutive pushes alternate), each
    region 256-byte aligned, nothing overlapping, identical on every rank (it
    is a function of the shapes)."""
    from hacedle_cuda import shard
    shapes = [(512, 3584), (512, 512), (1, 33), (64, 18944)]
    for world in (1, 2, 8, 65):
        offs, total = shard.exchange_layout(world, shapes)
        flat = [o for pair in offs for o in pair]
        sizes = [4 * B * N for (B, N) in shapes for _ in range(2)]
        assert flat[0] >= 4 * world and all(o % 256 == 0 for o in flat)
        ends = [o + sz for o, sz in zip(flat, sizes)]
        assert all(e <= o2 for e, o2 in zip(ends, flat[1:]))
        assert total >= ends[-1] and total % 256 == 0
