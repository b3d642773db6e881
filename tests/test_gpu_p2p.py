"""NVLink exchange of row-sharded outputs (hd_push_columns through
hacedle_cuda.shard.PeerExchange) on 2 GPUs, one process per GPU: every rank
ends with every rank's slice, bit-exact, in the final [B][G*n] layout, for
the float4 and the one-float paths and for repeated exchanges (growing
epochs).  Skipped on machines with fewer than two GPUs."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import sys
    sys.path[:0] = [ROOT, os.path.join(ROOT, "hace-fem-hacedle_b200", "python")]
    try:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        import hacedle_cuda as hc
        from hacedle_cuda import shard

        def ago(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        ctx = hc.Context(rank)
        cases = [(5, 100), (3, 33), (16, 1792)]
        ex = shard.PeerExchange(ctx, world, rank, [(B, n * world) for B, n in cases], ago)
        ok = True
        for rep in range(2):
            for i, (B, n) in enumerate(cases):
                ys = [np.random.default_rng(1000 * rep + 10 * i + r).standard_normal((B, n), dtype=np.float32)
                      for r in range(world)]
                y = torch.from_numpy(ys[rank]).cuda()
                ex.push(i, y, B, n)
                got = ex.full(i, B).cpu().numpy()
                want = np.concatenate(ys, axis=1)
                ok = ok and np.array_equal(got, want)
        ctx.check_device_errors()
        dist.barrier()
        ex.close()
        ctx.close()
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # reported to the parent
        q.put((rank, False, f"{type(e).__name__}: {e}"))


def test_push_columns_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, port = 2, _free_port()
    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    procs = [mctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, ok, msg = q.get(timeout=240)
            res[r] = (ok, msg)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert all(res[r][0] for r in range(world)), res
