"""Output-row sharding of a projection across ranks (the 7B-shaped layer).

Rank g of G owns rows [g*N/G, (g+1)*N/G) of every weight: a contiguous byte
range of the GGUF tensor, since GGUF stores whole rows of blocks.  Each rank
computes Y_g = X W_g^T as [B][N/G].  Two exchanges build Y [B][N] on every
rank: an all-gather over ranks ([G][B][N/G]) followed by hd_gather_columns,
or PeerExchange, which writes each rank's slice straight into every rank's
Y over NVLink (hd_push_columns, IPC-mapped buffers).
"""
from __future__ import annotations

import numpy as np

from .synth import BLOCK


def row_range(N: int, rank: int, world: int) -> tuple[int, int]:
    if N % world:
        raise ValueError(f"{N} rows do not split evenly over {world} ranks")
    n = N // world
    return rank * n, (rank + 1) * n


def row_slice(raw: np.ndarray, ggml_type: int, N: int, K: int, rank: int, world: int) -> np.ndarray:
    """GGUF bytes of this rank's rows (raw is [N, row_bytes] or flat)."""
    be, bb = BLOCK[ggml_type]
    row_bytes = (K // be) * bb
    r0, r1 = row_range(N, rank, world)
    return np.ascontiguousarray(np.asarray(raw, np.uint8).reshape(N, row_bytes)[r0:r1])


def gather_columns_reference(gathered: np.ndarray, world: int, B: int, n_shard: int) -> np.ndarray:
    """[G][B][n] -> [B][G*n] (what hd_gather_columns computes on the device)."""
    return np.ascontiguousarray(gathered.reshape(world, B, n_shard).transpose(1, 0, 2).reshape(B, world * n_shard))


def exchange_layout(world: int, shapes: list[tuple[int, int]]) -> tuple[list[tuple[int, int]], int]:
    """Byte offsets of the two full output buffers [B][N] of every entry of
    `shapes` in an exchange buffer that starts with the int32 flag array
    [world]; every region is 256-byte aligned.  Returns ([(offset of buffer 0,
    offset of buffer 1)] per entry, total bytes)."""
    def up(x):
        return (x + 255) // 256 * 256
    off = up(4 * world)
    offs = []
    for B, N in shapes:
        pair = []
        for _ in range(2):
            pair.append(off)
            off += up(4 * B * N)
        offs.append(tuple(pair))
    return offs, off


class _DeviceView:
    """A float32 [rows][cols] array at a raw device address, for torch.as_tensor."""

    def __init__(self, ptr: int, rows: int, cols: int):
        self.__cuda_array_interface__ = {"shape": (rows, cols), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """NVLink exchange of row-sharded outputs without a collective library.

    Every rank allocates one buffer (flags + two full outputs [B_max][N] per
    entry of `shapes`), shares its IPC handle through `all_gather_object`
    (e.g. torch.distributed.all_gather_object on any backend) and maps the
    others'.  push(i, y, B, n) writes this rank's slice y [B][n] into every
    rank's output i at columns rank*n.. and, on the device, completes once
    all ranks' slices are in this rank's output i (full(i, B) views the
    latest).  Every rank must make the same sequence of push calls.

    Consecutive pushes of output i alternate between its two buffers, so a
    push's result stays valid for every kernel this rank enqueues before its
    next push of output i: the peers write the push after that into the same
    buffer only once this rank's next push has raised its flag, which happens
    after everything enqueued before it has completed."""

    def __init__(self, ctx, world: int, rank: int, shapes: list[tuple[int, int]], all_gather_object):
        import ctypes as C

        import torch

        from . import lib

        self.ctx, self.world, self.rank, self.shapes = ctx, world, rank, list(shapes)
        self.offs, nbytes = exchange_layout(world, self.shapes)
        L = lib()
        p = C.c_void_p()
        ctx._check(L.hd_xbuf_alloc(ctx.h, nbytes, C.byref(p)))
        self.base = p.value
        self.peers = []
        h = (C.c_char * 64)()
        ctx._check(L.hd_ipc_handle(ctx.h, C.c_void_p(self.base), C.addressof(h)))
        handles = all_gather_object(bytes(h))
        bases = []
        for r in range(world):
            if r == rank:
                bases.append(self.base)
                continue
            q = C.c_void_p()
            hb = (C.c_char * 64).from_buffer_copy(handles[r])
            ctx._check(L.hd_ipc_open(ctx.h, C.addressof(hb), C.byref(q)))
            self.peers.append(q.value)
            bases.append(q.value)
        self.flag_ptrs = torch.tensor(bases, dtype=torch.int64, device="cuda")
        # full_ptrs[i][k]: every rank's buffer k of output i, indexed by rank
        self.full_ptrs = [[torch.tensor([b + o for b in bases], dtype=torch.int64, device="cuda") for o in pair]
                          for pair in self.offs]
        self.epoch = 0
        self.uses = [0] * len(self.shapes)   # pushes of each output so far

    def full(self, i: int, B: int):
        """This rank's output i [B][N] as written by the latest push(i)."""
        import torch
        Bmax, N = self.shapes[i]
        if B > Bmax:
            raise ValueError(f"batch {B} beyond the exchange buffer's {Bmax}")
        k = (self.uses[i] + 1) % 2   # buffer of the latest push (push u uses buffer (u - 1) % 2)
        return torch.as_tensor(_DeviceView(self.base + self.offs[i][k], B, N), device="cuda")

    def push(self, i: int, y, B: int, n: int):
        from . import lib
        Bmax, N = self.shapes[i]
        if B > Bmax or n * self.world != N:
            raise ValueError(f"slice [{B}][{n}] does not fit output {i} [{Bmax}][{N}] over {self.world} ranks")
        self.epoch += 1
        k = self.uses[i] % 2
        self.uses[i] += 1
        self.ctx._check(lib().hd_push_columns(self.ctx.h, y.data_ptr(), self.full_ptrs[i][k].data_ptr(),
                                              self.flag_ptrs.data_ptr(), self.world, self.rank, B, n, self.epoch))

    def push_all(self, items, B: int):
        """One exchange of several outputs: items = [(i, y, n), ...], each as
        push(i, y, B, n), in one launch with one completion handshake
        (hd_push_columns_multi).  Every rank makes the same calls."""
        import ctypes as C

        from . import lib
        if not 1 <= len(items) <= 16:
            raise ValueError("push_all takes 1..16 outputs")
        ys, fulls, ns = [], [], []
        for i, y, n in items:
            Bmax, N = self.shapes[i]
            if B > Bmax or n * self.world != N:
                raise ValueError(f"slice [{B}][{n}] does not fit output {i} [{Bmax}][{N}] over {self.world} ranks")
        self.epoch += 1
        for i, y, n in items:
            k = self.uses[i] % 2
            self.uses[i] += 1
            ys.append(y.data_ptr())
            fulls.append(self.full_ptrs[i][k].data_ptr())
            ns.append(n)
        cnt = len(items)
        self.ctx._check(lib().hd_push_columns_multi(self.ctx.h, cnt, (C.c_void_p * cnt)(*ys),
                                                    (C.c_void_p * cnt)(*fulls), (C.c_int64 * cnt)(*ns),
                                                    self.flag_ptrs.data_ptr(), self.world, self.rank, B, self.epoch))

    def close(self):
        import torch

        from . import lib
        torch.cuda.synchronize()
        for q in self.peers:
            lib().hd_ipc_close(self.ctx.h, q)
        self.peers = []
        if self.base:
            lib().hd_xbuf_free(self.ctx.h, self.base)
            self.base = 0
