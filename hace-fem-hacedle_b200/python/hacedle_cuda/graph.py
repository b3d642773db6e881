"""HGRF operator graphs on the device: the reference's graph executor
(runtime/graph_format.rs, runtime/graph_loader.rs, runtime/executor.rs) with
its ops running through the C ABI instead of the scalar CPU kernels.

File format (graph_format.rs:16-45, little-endian, #[repr(C)] layouts):
  GraphHeader  24 bytes: magic u32 "HGRF", version u16 (1), 2 pad bytes,
               node_count u32, edge_count u32, const_offset u64;
  GraphNode    20 bytes each: op_code u16, 2 pad, input_start u32,
               input_len u16, 2 pad, output u32, authority_offset u32;
  GraphEdge    4 bytes each: tensor_id u32;
  then the constant pool from const_offset to the end of the file.

parse() validates as GraphView::parse does (graph_format.rs:66-136) and
load() builds the op list as GraphLoader::load does (graph_loader.rs:33-85):
MatMul (a, b), Add (a, b), RmsNorm (x, weight; eps 1e-5), Rope (x, cos,
sin); the errors are the reference's GraphError / LoadError cases.  run()
executes the ops in order over a tensor table -- TensorCtx's tensors, here
device tensors keyed by id -- as GraphExecutor::run (executor.rs:39-45):
  MatMul  -> hd_matmul_f32      (core/ops/matmul.rs:16-51)
  Add     -> hd_add             (core/ops/add.rs:16-43)
  RmsNorm -> hd_rmsnorm_graph   (core/ops/rmsnorm.rs:16-61)
  Rope    -> hd_rope_interleaved (core/ops/rope.rs:16-64)
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

MAGIC = struct.unpack("<I", b"HGRF")[0]
VERSION = 1
OP_MATMUL, OP_ADD, OP_RMSNORM, OP_ROPE = 1, 2, 3, 4
HEADER = struct.Struct("<IH2xIIQ")   # 24 bytes
NODE = struct.Struct("<H2xIH2xII")   # 20 bytes
EDGE = struct.Struct("<I")
RMSNORM_EPS = 1e-5                   # graph_loader.rs: RmsNormOp { eps: 1e-5 }


class GraphError(ValueError):
    """GraphView::parse failures: InvalidMagic, UnsupportedVersion,
    OutOfBounds, InvalidLayout (Misaligned cannot happen on a byte copy)."""

    def __init__(self, kind: str):
        super().__init__(kind)
        self.kind = kind


class LoadError(ValueError):
    """GraphLoader::load failures: InvalidInputs, UnsupportedOp."""

    def __init__(self, kind: str):
        super().__init__(kind)
        self.kind = kind


@dataclass(frozen=True)
class Node:
    op_code: int
    input_start: int
    input_len: int
    output: int
    authority_offset: int


@dataclass(frozen=True)
class GraphView:
    version: int
    nodes: tuple
    edges: tuple
    const_pool: bytes


def parse(data: bytes) -> GraphView:
    data = bytes(data)
    if len(data) < HEADER.size:
        raise GraphError("OutOfBounds")
    magic, version, n_nodes, n_edges, const_off = HEADER.unpack_from(data, 0)
    if magic != MAGIC:
        raise GraphError("InvalidMagic")
    if version != VERSION:
        raise GraphError("UnsupportedVersion")
    node_end = HEADER.size + NODE.size * n_nodes
    edge_end = node_end + EDGE.size * n_edges
    if edge_end > len(data):
        raise GraphError("OutOfBounds")
    if const_off < edge_end:
        raise GraphError("InvalidLayout")
    if const_off > len(data):
        raise GraphError("OutOfBounds")
    nodes = tuple(Node(*NODE.unpack_from(data, HEADER.size + i * NODE.size)) for i in range(n_nodes))
    edges = tuple(EDGE.unpack_from(data, node_end + i * EDGE.size)[0] for i in range(n_edges))
    return GraphView(version, nodes, edges, data[const_off:])


@dataclass(frozen=True)
class Op:
    kind: int
    inputs: tuple
    output: int
    authority_offset: int


_ARITY = {OP_MATMUL: 2, OP_ADD: 2, OP_RMSNORM: 2, OP_ROPE: 3}


def load(graph: GraphView) -> list[Op]:
    ops = []
    for n in graph.nodes:
        end = n.input_start + n.input_len
        if end > len(graph.edges):
            raise LoadError("InvalidInputs")
        inputs = graph.edges[n.input_start:end]
        if n.op_code not in _ARITY:
            raise LoadError("UnsupportedOp")
        if len(inputs) < _ARITY[n.op_code]:
            raise LoadError("InvalidInputs")
        ops.append(Op(n.op_code, tuple(inputs[:_ARITY[n.op_code]]), n.output, n.authority_offset))
    return ops


def _check(op: Op, ins: list, out) -> str | None:
    """The reference op's ShapeMismatch conditions, or None."""
    if op.kind == OP_MATMUL:   # core/ops/matmul.rs:21-33
        a, b = ins
        if a.dim() != 2 or b.dim() != 2 or out.dim() != 2:
            return "MatMul: ShapeMismatch"
        if a.shape[1] != b.shape[0] or tuple(out.shape) != (a.shape[0], b.shape[1]):
            return "MatMul: ShapeMismatch"
    elif op.kind == OP_ADD:
        a, b = ins
        if a.shape != b.shape or a.shape != out.shape:
            return "Add: ShapeMismatch"
    elif op.kind == OP_RMSNORM:
        x, w = ins
        if x.shape != out.shape or w.dim() != 1 or x.dim() == 0 or x.shape[-1] != w.shape[0]:
            return "RmsNorm: ShapeMismatch"
    else:                      # core/ops/rope.rs:27-43
        x, c, s = ins
        if x.shape != out.shape or c.shape != s.shape or x.shape != c.shape or (x.dim() and x.shape[-1] % 2):
            return "Rope: ShapeMismatch"
    return None


def run(ctx, ops: list[Op], tensors: dict) -> list[tuple[int, str]]:
    """Executes `ops` in order; tensors maps tensor ids to float32 device
    tensors (outputs pre-allocated with their shapes, as TensorCtx's views
    are).  Like GraphExecutor::run, whose ops discard their Result, an op
    whose shapes do not fit leaves its output untouched and the run goes on;
    the skipped ops are returned as (index, reason).  A tensor id missing
    from the table raises KeyError."""
    skipped = []
    for i, op in enumerate(ops):
        ins = [tensors[t] for t in op.inputs]
        out = tensors[op.output]
        why = _check(op, ins, out)
        if why:
            skipped.append((i, why))
            continue
        if op.kind == OP_MATMUL:
            ctx.matmul_f32(ins[0], ins[1], out)
        elif op.kind == OP_ADD:
            ctx.add(ins[0], ins[1], out)
        elif op.kind == OP_RMSNORM:
            ctx.rmsnorm_graph(ins[0], ins[1], out, RMSNORM_EPS)
        else:
            ctx.rope_interleaved(ins[0], ins[1], ins[2], out)
    return skipped
