"""Graph builders with the reference API (python/tinytensor/graph.py), producing the
node table the C ABI compiles (tt_graph in include/tt_cuda.h).

Shape rules and the exceptions they raise follow the reference builders
(src/graph/graph.cpp:51-200): NumPy broadcasting for binary ops, the batched matmul
rule, transpose axis normalisation, and reductions with optional keepdims.
Additional builders for ops the reference lacks: exp, neg, tanh, reduce_max.
"""

import builtins
import ctypes
from collections.abc import Sequence

import numpy as np

from . import _lib
from ._lib import BroadcastError, DimensionError, IRError, ShapeError, TypeError

float32 = "float32"
float64 = "float64"
_DTYPE_CODE = {float32: 0, float64: 1}

__all__ = [
    "Graph", "Node", "float32", "float64", "add", "sub", "mul", "div", "relu", "sigmoid",
    "matmul", "sum", "mean", "max", "transpose", "exp", "neg", "tanh",
]


def broadcast_shapes(a, b):
    """Tensor::broadcast_shapes (src/core/tensor.cpp:189-215)."""
    r = builtins.max(len(a), len(b))
    out = []
    for i in range(r):
        da = a[i - (r - len(a))] if i >= r - len(a) else 1
        db = b[i - (r - len(b))] if i >= r - len(b) else 1
        if da != db and da != 1 and db != 1:
            raise BroadcastError(f"Shapes {list(a)} and {list(b)} are not broadcastable")
        out.append(db if da == 1 else da)
    return out


class Node:
    """A graph node (the Python face of tinytensor::Node)."""

    __slots__ = ("_graph", "index", "op", "shape", "dtype", "inputs", "id", "name", "dim0", "dim1",
                 "axes", "keepdims", "data", "expr")

    def __init__(self, graph, op, shape, dtype, inputs=(), name=""):
        self._graph = graph
        self.index = len(graph._nodes)
        self.op = op
        self.shape = [int(d) for d in shape]
        self.dtype = dtype
        self.inputs = list(inputs)
        self.id = graph._next_id
        self.name = name
        self.dim0 = self.dim1 = 0
        self.axes = []
        self.keepdims = False
        self.data = None
        self.expr = None

    def __add__(self, other):
        return self._graph.add(self, other)

    def __radd__(self, other):
        return self._graph.add(other, self)

    def __sub__(self, other):
        return self._graph.sub(self, other)

    def __rsub__(self, other):
        return self._graph.sub(other, self)

    def __mul__(self, other):
        return self._graph.mul(self, other)

    def __rmul__(self, other):
        return self._graph.mul(other, self)

    def __truediv__(self, other):
        return self._graph.div(self, other)

    def __rtruediv__(self, other):
        return self._graph.div(other, self)

    def __matmul__(self, other):
        return self._graph.matmul(self, other)

    def __neg__(self):
        return self._graph.neg(self)

    def __hash__(self):
        return id(self)

    def __eq__(self, other):
        return self is other

    def __repr__(self):
        return f"Node(id={self.id}, name='{self.name}', shape={self.shape}, dtype={self.dtype})"


class Graph:
    """Computation graph with the reference builder API."""

    def __init__(self):
        self._nodes = []
        self._inputs = []
        self._outputs = []
        self._next_id = 0
        self._version = 0

    # -- construction ------------------------------------------------------------------
    def _add(self, node):
        self._nodes.append(node)
        self._next_id = node.id + 1
        self._version += 1
        return node

    def _ensure(self, x):
        if isinstance(x, Node):
            if x._graph is not self:
                raise IRError("Node belongs to a different graph")
            return x
        return self.constant(x)

    def input(self, shape: Sequence[int], dtype=float32, name: str = "") -> Node:
        if dtype not in _DTYPE_CODE:
            raise TypeError(f"Unsupported dtype {dtype}")
        if any(int(d) < 0 for d in shape):
            raise IRError("Input shape has a negative dimension")
        if not name:
            name = f"input_{len(self._inputs)}"  # Graph::create_input (graph.cpp:22-33)
        n = self._add(Node(self, _lib.OP_INPUT, shape, dtype, name=name))
        self._inputs.append(n)
        return n

    def constant(self, value, name: str = "") -> Node:
        arr = np.array(value, dtype=np.float32, order="C")  # keeps 0-d scalars 0-d
        n = Node(self, _lib.OP_CONSTANT, arr.shape, float32, name=name or f"const_{self._next_id}")
        n.data = arr
        return self._add(n)

    def _binary(self, op, a, b):
        a, b = self._ensure(a), self._ensure(b)
        if a.dtype != b.dtype:
            raise TypeError(f"DType mismatch in {_OPNAME[op]}")
        return self._add(Node(self, op, broadcast_shapes(a.shape, b.shape), a.dtype, [a, b]))

    def _unary(self, op, a):
        a = self._ensure(a)
        return self._add(Node(self, op, a.shape, a.dtype, [a]))

    def add(self, a, b) -> Node:
        return self._binary(_lib.OP_ADD, a, b)

    def sub(self, a, b) -> Node:
        return self._binary(_lib.OP_SUB, a, b)

    def mul(self, a, b) -> Node:
        return self._binary(_lib.OP_MUL, a, b)

    def div(self, a, b) -> Node:
        return self._binary(_lib.OP_DIV, a, b)

    def relu(self, a) -> Node:
        return self._unary(_lib.OP_RELU, a)

    def sigmoid(self, a) -> Node:
        return self._unary(_lib.OP_SIGMOID, a)

    def exp(self, a) -> Node:
        return self._unary(_lib.OP_EXP, a)

    def neg(self, a) -> Node:
        return self._unary(_lib.OP_NEG, a)

    def tanh(self, a) -> Node:
        return self._unary(_lib.OP_TANH, a)

    def matmul(self, a, b) -> Node:
        """Graph::matmul shape rule (graph.cpp:89-127)."""
        a, b = self._ensure(a), self._ensure(b)
        if a.dtype != b.dtype:
            raise TypeError("DType mismatch in matmul")
        if len(a.shape) < 2 or len(b.shape) < 2:
            raise DimensionError("Unsupported ranks for matmul")
        ka, kb = a.shape[-1], b.shape[-2]
        if ka != kb:
            raise ShapeError(f"Matmul inner dimensions mismatch: {ka} vs {kb}")
        batch = []
        if len(a.shape) > 2 or len(b.shape) > 2:
            batch = broadcast_shapes(a.shape[:-2], b.shape[:-2])
        return self._add(Node(self, _lib.OP_MATMUL, batch + [a.shape[-2], b.shape[-1]], a.dtype, [a, b]))

    def transpose(self, a, dim0: int, dim1: int) -> Node:
        a = self._ensure(a)
        r = len(a.shape)
        d0 = dim0 + r if dim0 < 0 else dim0
        d1 = dim1 + r if dim1 < 0 else dim1
        if not (0 <= d0 < r and 0 <= d1 < r):
            raise DimensionError(f"Invalid transpose axes for rank {r}")
        shape = list(a.shape)
        shape[d0], shape[d1] = shape[d1], shape[d0]
        n = Node(self, _lib.OP_TRANSPOSE, shape, a.dtype, [a])
        n.dim0, n.dim1 = d0, d1
        return self._add(n)

    def _reduce(self, op, a, axes, keepdims):
        a = self._ensure(a)
        r = len(a.shape)
        axes = [] if axes is None else [int(x) for x in axes]
        if not axes:
            norm = set(range(r))
        else:
            norm = set()
            for ax in axes:
                x = ax + r if ax < 0 else ax
                if not 0 <= x < r:
                    raise DimensionError(f"Axis out of range in {_OPNAME[op]}")
                norm.add(x)
        shape = []
        for i in range(r):
            if i in norm:
                if keepdims:
                    shape.append(1)
            else:
                shape.append(a.shape[i])
        n = Node(self, op, shape, a.dtype, [a])
        n.axes = axes
        n.keepdims = bool(keepdims)
        return self._add(n)

    def reduce_sum(self, a, axes=None, keepdims: bool = False) -> Node:
        return self._reduce(_lib.OP_REDUCE_SUM, a, axes, keepdims)

    def reduce_mean(self, a, axes=None, keepdims: bool = False) -> Node:
        return self._reduce(_lib.OP_REDUCE_MEAN, a, axes, keepdims)

    def reduce_max(self, a, axes=None, keepdims: bool = False) -> Node:
        return self._reduce(_lib.OP_REDUCE_MAX, a, axes, keepdims)

    def mark_output(self, node: Node) -> None:
        if node is None:
            raise IRError("Cannot mark null node as output")
        if node not in self._outputs:
            self._outputs.append(node)
            self._version += 1

    @property
    def inputs(self):
        return list(self._inputs)

    @property
    def outputs(self):
        return list(self._outputs)

    @property
    def nodes(self):
        return list(self._nodes)

    # -- C ABI image ---------------------------------------------------------------------
    def _to_c(self, outputs=None):
        """Returns (TTGraph, keepalive) describing this graph for the C ABI."""
        nodes = (_lib.TTNode * builtins.max(1, len(self._nodes)))()
        keep = []
        for i, n in enumerate(self._nodes):
            c = nodes[i]
            c.op = n.op
            c.dtype = _DTYPE_CODE[n.dtype]
            c.num_inputs = len(n.inputs)
            for k, q in enumerate(n.inputs):
                c.inputs[k] = q.index
            if len(n.shape) > _lib.TT_MAX_RANK:
                raise DimensionError(f"rank {len(n.shape)} exceeds {_lib.TT_MAX_RANK}")
            c.rank = len(n.shape)
            for k, d in enumerate(n.shape):
                c.shape[k] = d
            c.id = n.id
            c.dim0, c.dim1 = n.dim0, n.dim1
            c.num_axes = len(n.axes)
            for k, ax in enumerate(n.axes):
                c.axes[k] = ax
            c.keepdims = int(n.keepdims)
            if n.data is not None:
                keep.append(n.data)
                c.data = n.data.ctypes.data
            if n.name:
                b = n.name.encode()
                keep.append(b)
                c.name = b
            if n.expr:
                b = n.expr.encode()
                keep.append(b)
                c.expr = b
        outs = self._outputs if outputs is None else outputs
        ins = (ctypes.c_int32 * builtins.max(1, len(self._inputs)))(*[n.index for n in self._inputs])
        outa = (ctypes.c_int32 * builtins.max(1, len(outs)))(*[n.index for n in outs])
        keep += [nodes, ins, outa]
        g = _lib.TTGraph(len(self._nodes), nodes, len(self._inputs), ins, len(outs), outa)
        return g, keep

    def to_ir(self) -> str:
        """Canonical IR text (IRPrinter::to_string format)."""
        g, keep = self._to_c()
        return _lib.cstr(_lib.lib.tt_graph_ir, ctypes.byref(g))


_OPNAME = {
    _lib.OP_ADD: "add", _lib.OP_SUB: "sub", _lib.OP_MUL: "mul", _lib.OP_DIV: "div",
    _lib.OP_REDUCE_SUM: "reduce_sum", _lib.OP_REDUCE_MEAN: "reduce_mean", _lib.OP_REDUCE_MAX: "reduce_max",
}


def _graph_of(a, b=None):
    if isinstance(a, Node):
        return a._graph
    if isinstance(b, Node):
        return b._graph
    raise TypeError("At least one operand must be a Node")


def add(a, b):
    return _graph_of(a, b).add(a, b)


def sub(a, b):
    return _graph_of(a, b).sub(a, b)


def mul(a, b):
    return _graph_of(a, b).mul(a, b)


def div(a, b):
    return _graph_of(a, b).div(a, b)


def matmul(a, b):
    return _graph_of(a, b).matmul(a, b)


def _unary_node(a):
    if not isinstance(a, Node):
        raise TypeError("Operand must be a Node")
    return a._graph


def relu(a):
    return _unary_node(a).relu(a)


def sigmoid(a):
    return _unary_node(a).sigmoid(a)


def exp(a):
    return _unary_node(a).exp(a)


def neg(a):
    return _unary_node(a).neg(a)


def tanh(a):
    return _unary_node(a).tanh(a)


def sum(a, axes=None, keepdims=False):  # noqa: A001 - reference name
    return _unary_node(a).reduce_sum(a, axes, keepdims)


def mean(a, axes=None, keepdims=False):
    return _unary_node(a).reduce_mean(a, axes, keepdims)


def max(a, axes=None, keepdims=False):  # noqa: A001 - mirrors sum/mean
    return _unary_node(a).reduce_max(a, axes, keepdims)


def transpose(a, dim0, dim1):
    return _unary_node(a).transpose(a, dim0, dim1)
