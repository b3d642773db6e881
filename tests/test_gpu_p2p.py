"""NVLink exchange of row-sharded outputs (hd_push_columns through
hacedle_cuda.shard.PeerExchange) on 2 GPUs, one process per GPU: every rank
ends with every rank's slice, bit-exact, in the final [B][G*n] layout, for
the float4 and the one-float paths and for repeated exchanges (growing
epochs); many exchanges with a device consumer between them and no host
synchronization; several outputs in one launch with one handshake
(hd_push_columns_multi, PeerExchange.push_all), mixed with single pushes;
and the bounded wait expiring when a rank skips an exchange
(the context reports HD_E_TIMEOUT and stays usable).  Skipped on machines
with fewer than two GPUs.  Host messages go over gloo; no NCCL, no NVLS."""
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


def _rank_pipelined(rank, world, port, q):
    """Many exchanges back to back with no host synchronization: push, a
    device kernel that copies the exchanged output out (the consumer), the
    next push of the same output.  Rank 1 stalls on the device before each of
    its copies, so rank 0 runs ahead: a peer that overwrote an output still
    being read would corrupt rank 1's copies."""
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
        cases = [(4, 1024), (1, 448)]
        ex = shard.PeerExchange(ctx, world, rank, [(B, n * world) for B, n in cases], ago)
        E = 24
        ys = {(e, i): [np.random.default_rng(100 * e + 10 * i + r).standard_normal((B, n), dtype=np.float32)
                       for r in range(world)] for e in range(E) for i, (B, n) in enumerate(cases)}
        dev = {k: torch.from_numpy(v[rank]).cuda() for k, v in ys.items()}
        outs = {k: torch.empty(cases[k[1]][0], cases[k[1]][1] * world, device="cuda") for k in ys}
        torch.cuda.synchronize()
        dist.barrier()
        for e in range(E):
            for i, (B, n) in enumerate(cases):
                ex.push(i, dev[(e, i)], B, n)
                if rank == 1:
                    torch.cuda._sleep(200000)   # a slow consumer (~0.1 ms)
                outs[(e, i)].copy_(ex.full(i, B))
        torch.cuda.synchronize()
        ctx.check_device_errors()
        ok = all(np.array_equal(outs[k].cpu().numpy(), np.concatenate(v, axis=1)) for k, v in ys.items())
        dist.barrier()
        ex.close()
        ctx.close()
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # reported to the parent
        q.put((rank, False, f"{type(e).__name__}: {e}"))


def _rank_multi(rank, world, port, q):
    """push_all: the outputs of a layer (shapes of both vector widths) in one
    launch, back to back with a slow consumer on rank 1, alternating with
    single pushes of the same outputs."""
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
        for cases in ([(4, 1792), (4, 256), (4, 9472)], [(3, 33), (3, 100), (3, 5)]):   # float4 / one-float paths
            B = cases[0][0]
            ex = shard.PeerExchange(ctx, world, rank, [(B, n * world) for _, n in cases], ago)
            E = 8
            ys = {(e, i): [np.random.default_rng(1000 * e + 10 * i + r).standard_normal((B, n), dtype=np.float32)
                           for r in range(world)] for e in range(E) for i, (_, n) in enumerate(cases)}
            dev = {k: torch.from_numpy(v[rank]).cuda() for k, v in ys.items()}
            outs = {k: torch.empty(B, cases[k[1]][1] * world, device="cuda") for k in ys}
            torch.cuda.synchronize()
            dist.barrier()
            for e in range(E):
                if e % 3 == 2:   # every third exchange output by output
                    for i, (_, n) in enumerate(cases):
                        ex.push(i, dev[(e, i)], B, n)
                else:
                    ex.push_all([(i, dev[(e, i)], n) for i, (_, n) in enumerate(cases)], B)
                if rank == 1:
                    torch.cuda._sleep(200000)   # a slow consumer
                for i in range(len(cases)):
                    outs[(e, i)].copy_(ex.full(i, B))
            torch.cuda.synchronize()
            ctx.check_device_errors()
            ok = all(np.array_equal(outs[k].cpu().numpy(), np.concatenate(v, axis=1)) for k, v in ys.items())
            dist.barrier()
            ex.close()
            if not ok:
                break
        ctx.close()
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # reported to the parent
        q.put((rank, False, f"{type(e).__name__}: {e}"))


def _rank_timeout(rank, world, port, q):
    """Rank 1 skips an exchange: rank 0's bounded wait for its flag runs out
    (about 1 s) and the context reports HD_E_TIMEOUT; the GPU stays usable."""
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
        B, n = 2, 256
        ex = shard.PeerExchange(ctx, world, rank, [(B, n * world)], ago)
        y = torch.ones(B, n, device="cuda")
        ex.push(0, y, B, n)           # both ranks
        torch.cuda.synchronize()
        ctx.check_device_errors()
        dist.barrier()
        ok = True
        if rank == 0:
            ex.push(0, y, B, n)       # rank 1 never pushes this one
            torch.cuda.synchronize()
            try:
                ctx.check_device_errors()
                ok = False
            except hc.HdError as err:
                ok = err.code == hc.HD_E_TIMEOUT
            z = torch.arange(8, device="cuda", dtype=torch.float32).sum()   # the context still works
            ok = ok and float(z) == 28.0
        dist.barrier()
        ex.close()
        ctx.close()
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # reported to the parent
        q.put((rank, False, f"{type(e).__name__}: {e}"))


def _run(target):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    world, port = 2, _free_port()
    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    procs = [mctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
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


def test_push_columns_pipelined_two_gpus():
    _run(_rank_pipelined)


def test_push_columns_multi_two_gpus():
    _run(_rank_multi)


def test_push_columns_bounded_wait_times_out_two_gpus():
    _run(_rank_timeout)


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
