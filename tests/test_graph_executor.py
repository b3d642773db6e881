"""The HGRF graph executor (hacedle_cuda.graph): the reference's graph fixtures
parsed as GraphView::parse does (runtime/graph_format.rs:66-136), loaded as
GraphLoader::load does (runtime/graph_loader.rs:33-85), every error case of
both, and -- on the GPU -- the loaded ops run through hd_matmul_f32 / hd_add /
hd_rmsnorm_graph (eps 1e-5) / hd_rope_interleaved against the oracle's
composition of the same reference ops."""
import os
import struct

import numpy as np
import pytest

from hacedle_cuda import graph as G
from hacedle_cuda import synth as S
from oracle import oracle as O


def _read(golden_dir, name):
    with open(os.path.join(golden_dir, name), "rb") as f:
        return f.read()


def _graph(nodes, edges, const=b"", magic=G.MAGIC, version=G.VERSION, const_offset=None):
    body = b"".join(G.NODE.pack(*n) for n in nodes) + b"".join(G.EDGE.pack(e) for e in edges)
    off = G.HEADER.size + len(body) if const_offset is None else const_offset
    return G.HEADER.pack(magic, version, len(nodes), len(edges), off) + body + const


def test_fixtures_parse_and_load(golden_dir):
    g = G.parse(_read(golden_dir, "minimal.hgraph"))
    ops = G.load(g)
    assert [(o.kind, o.inputs, o.output) for o in ops] == [(G.OP_MATMUL, (0, 1), 2)]
    g = G.parse(_read(golden_dir, "chain_rms_rope_mm.hgraph"))
    ops = G.load(g)
    assert [(o.kind, o.inputs, o.output) for o in ops] == [(G.OP_RMSNORM, (0, 1), 5), (G.OP_ROPE, (5, 2, 3), 6),
                                                           (G.OP_MATMUL, (6, 4), 7)]
    assert g.const_pool == b""


def test_round_trip_and_const_pool():
    data = _graph([(G.OP_ADD, 0, 2, 2, 7)], [0, 1], const=b"\x01\x02\x03")
    g = G.parse(data)
    assert g.const_pool == b"\x01\x02\x03" and g.nodes[0].authority_offset == 7


@pytest.mark.parametrize("data,kind", [
    (b"HGRF\x01\x00", "OutOfBounds"),                                          # shorter than the header
    (_graph([], [], magic=0x12345678), "InvalidMagic"),
    (_graph([], [], version=2), "UnsupportedVersion"),
    (_graph([(1, 0, 2, 2, 0)], [0, 1])[:-4], "OutOfBounds"),                  # edges cut off
    (_graph([(1, 0, 2, 2, 0)], [0, 1], const_offset=40), "InvalidLayout"),   # const pool inside the edges
    (_graph([(1, 0, 2, 2, 0)], [0, 1], const_offset=10 ** 6), "OutOfBounds"),
])
def test_parse_errors(data, kind):
    with pytest.raises(G.GraphError) as e:
        G.parse(data)
    assert e.value.kind == kind


@pytest.mark.parametrize("nodes,edges,kind", [
    ([(G.OP_MATMUL, 1, 2, 2, 0)], [0, 1], "InvalidInputs"),      # inputs past the edge list
    ([(G.OP_RMSNORM, 0, 1, 2, 0)], [0, 1], "InvalidInputs"),     # RmsNorm needs x and weight
    ([(G.OP_ROPE, 0, 2, 3, 0)], [0, 1, 2], "InvalidInputs"),     # Rope needs x, cos and sin
    ([(9, 0, 2, 2, 0)], [0, 1], "UnsupportedOp"),
])
def test_load_errors(nodes, edges, kind):
    with pytest.raises(G.LoadError) as e:
        G.load(G.parse(_graph(nodes, edges)))
    assert e.value.kind == kind


@pytest.mark.gpu
def test_fixture_graphs_on_device(ctx, golden_dir):
    import torch

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()

    rng = S.rng(31)
    # minimal.hgraph: t2 = t0 [37, 96] x t1 [96, 50]
    a = rng.standard_normal((37, 96), dtype=np.float32)
    b = rng.standard_normal((96, 50), dtype=np.float32)
    t = {0: dev(a), 1: dev(b), 2: torch.full((37, 50), float("nan"), device="cuda")}
    assert G.run(ctx, G.load(G.parse(_read(golden_dir, "minimal.hgraph"))), t) == []
    ref = O.matmul_f32(a, b)
    assert np.abs(t[2].cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max()

    # chain_rms_rope_mm.hgraph: t5 = rmsnorm(t0, t1), t6 = rope(t5, t2, t3), t7 = t6 x t4
    T_, D, N = 12, 64, 40
    x = rng.standard_normal((T_, D), dtype=np.float32)
    w = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    ang = rng.uniform(-3, 3, (T_, D)).astype(np.float32)
    c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    wm = rng.standard_normal((D, N), dtype=np.float32)
    t = {0: dev(x), 1: dev(w), 2: dev(c), 3: dev(s), 4: dev(wm), 5: torch.empty(T_, D, device="cuda"),
         6: torch.empty(T_, D, device="cuda"), 7: torch.full((T_, N), float("nan"), device="cuda")}
    assert G.run(ctx, G.load(G.parse(_read(golden_dir, "chain_rms_rope_mm.hgraph"))), t) == []
    r5 = O.rmsnorm_graph(x, w, 1e-5)
    r6 = O.rope_interleaved(r5, c, s)
    r7 = O.matmul_f32(r6, wm)
    assert np.abs(t[5].cpu().numpy() - r5).max() <= 1e-6 * np.abs(r5).max()
    assert np.abs(t[6].cpu().numpy() - r6).max() <= 1e-6 * np.abs(r6).max()
    assert np.abs(t[7].cpu().numpy() - r7).max() <= 1e-5 * np.abs(r7).max()


@pytest.mark.gpu
def test_mismatched_op_is_skipped_like_the_reference(ctx):
    """GraphExecutor::run ignores an op's ShapeMismatch: its output stays as it
    was and the later ops still run."""
    import torch
    ops = G.load(G.parse(_graph([(G.OP_ADD, 0, 2, 2, 0), (G.OP_ADD, 2, 2, 3, 0)], [0, 1, 0, 0])))
    t = {0: torch.ones(4, 8, device="cuda"), 1: torch.ones(4, 9, device="cuda"),
         2: torch.full((4, 8), 7.0, device="cuda"), 3: torch.zeros(4, 8, device="cuda")}
    skipped = G.run(ctx, ops, t)
    assert skipped == [(0, "Add: ShapeMismatch")]
    assert bool((t[2] == 7.0).all()) and bool((t[3] == 2.0).all())
