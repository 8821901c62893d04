"""The input contract: dtypes, shapes, scalar expressions, the tensor DAG, graphs
and host values.

This module restates the data model of CUDACaml's `lib/ir` so that the graphs
this backend runs are the same graphs the reference builds:

* ``Dtype``        -- lib/ir/dtype.ml:9-14 (F32/F64/I32/I64/Bool, sizes 4/8/4/8/1)
* ``Shape``        -- lib/ir/shape.ml (a tuple of extents; scalar = ())
* ``Expr``         -- lib/ir/expr.ml:13-43 (Const/Arg/Index/Binop/Unop/Cmp/
                      Logic/Not/Select/Cast)
* ``Tensor``       -- lib/ir/tensor.ml:11-44 (the 11 node kinds)
* ``Graph``        -- lib/ir/graph.ml (stable post-order topo sort, fan-out
                      counted in uses, params discovered from outputs)
* ``Value``        -- lib/ir/value.ml (contiguous host storage; numpy here)

Node identity is the uid and nothing else, exactly as in the reference: every
table is keyed by ``uid`` and no dict iteration order reaches an output.
"""
from __future__ import annotations

import enum
import itertools
import struct
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

# ---------------------------------------------------------------------------
# Uids (lib/ir/uid.ml): one global counter shared by tensors and expressions.
# ---------------------------------------------------------------------------
_uid_counter = itertools.count(1)


def fresh_uid() -> int:
    return next(_uid_counter)


# ---------------------------------------------------------------------------
# Dtypes (lib/ir/dtype.ml:9-45)
# ---------------------------------------------------------------------------
class Dtype(enum.Enum):
    F32 = "f32"
    F64 = "f64"
    I32 = "i32"
    I64 = "i64"
    BOOL = "bool"

    @property
    def size_in_bytes(self) -> int:
        return {"f32": 4, "f64": 8, "i32": 4, "i64": 8, "bool": 1}[self.value]

    @property
    def is_float(self) -> bool:
        return self in (Dtype.F32, Dtype.F64)

    @property
    def is_int(self) -> bool:
        return self in (Dtype.I32, Dtype.I64)

    @property
    def np(self):
        if self is Dtype.BOOL:
            raise ValueError("Bool tensors are not storable")
        return {"f32": np.float32, "f64": np.float64, "i32": np.int32, "i64": np.int64}[self.value]

    def __repr__(self) -> str:  # pragma: no cover - cosmetic
        return f"Dtype.{self.name}"


F32, F64, I32, I64, BOOL = Dtype.F32, Dtype.F64, Dtype.I32, Dtype.I64, Dtype.BOOL


# ---------------------------------------------------------------------------
# Shapes (lib/ir/shape.ml)
# ---------------------------------------------------------------------------
def shape_of(dims: Sequence[int]) -> tuple:
    dims = tuple(int(d) for d in dims)
    if any(d < 0 for d in dims):
        raise ValueError(f"Shape.of_dims: negative extent in {dims}")
    return dims


SCALAR: tuple = ()


def numel(shape: Sequence[int]) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


def shape_to_string(shape: Sequence[int]) -> str:
    return "[" + ",".join(str(d) for d in shape) + "]"


def row_length(shape: Sequence[int]) -> int:
    """Extent of the last axis; rank 0 is one row of one element
    (lib/backend_interp/cudacaml_backend_interp.ml:269-270)."""
    return shape[-1] if len(shape) else 1


# ---------------------------------------------------------------------------
# Scalar expressions (lib/ir/expr.ml)
# ---------------------------------------------------------------------------
BINOPS = ("add", "sub", "mul", "div", "min", "max", "bit_and", "bit_or", "bit_xor", "shl", "shr")
UNOPS = ("neg", "sqrt", "exp", "log", "abs", "sin", "cos", "erf", "erfinv")
CMPS = ("eq", "ne", "lt", "le", "gt", "ge")
LOGICS = ("and", "or")


class Expr:
    """One node of an element function. ``kind`` is one of const / arg /
    index / binop / unop / cmp / logic / not / select / cast."""

    __slots__ = ("uid", "dtype", "kind", "op", "args", "value")

    def __init__(self, dtype: Dtype, kind: str, op=None, args: tuple = (), value=None):
        self.uid = fresh_uid()
        self.dtype = dtype
        self.kind = kind
        self.op = op
        self.args = tuple(args)
        self.value = value

    def __repr__(self) -> str:  # pragma: no cover - debugging aid
        if self.kind == "const":
            return f"{self.value!r}:{self.dtype.value}"
        if self.kind == "arg":
            return f"arg{self.value}:{self.dtype.value}"
        if self.kind == "index":
            return "index"
        inner = " ".join(repr(a) for a in self.args)
        return f"({self.op or self.kind} {inner})"


@dataclass
class Fn1:
    """First-order element function of one argument (lib/ir/expr.ml:48)."""

    arg1: Expr
    body1: Expr


@dataclass
class Fn2:
    """First-order element function of two arguments (lib/ir/expr.ml:50)."""

    arg_a: Expr
    arg_b: Expr
    body2: Expr


def make_fn1(dtype: Dtype, f) -> Fn1:
    """The HOAS -> first-order bridge (lib/ir/expr.ml:54-57): the closure runs
    once on a fresh placeholder and only the resulting tree is kept."""
    a = Expr(dtype, "arg", value=0)
    return Fn1(a, f(a))


def make_fn2(da: Dtype, db: Dtype, f) -> Fn2:
    a = Expr(da, "arg", value=0)
    b = Expr(db, "arg", value=1)
    return Fn2(a, b, f(a, b))


# ---------------------------------------------------------------------------
# Tensors (lib/ir/tensor.ml)
# ---------------------------------------------------------------------------
TENSOR_KINDS = (
    "param", "iota", "map", "map2", "reduce", "scan", "gather",
    "scatter_add", "matmul", "reshape", "broadcast",
)


class Tensor:
    """A whole-tensor operation. ``deps`` are the direct data dependencies in
    argument order (lib/ir/tensor.ml:50-62)."""

    __slots__ = ("uid", "dtype", "shape", "kind", "name", "fn", "init", "deps")

    def __init__(self, dtype: Dtype, shape, kind: str, deps=(), name=None, fn=None, init=None):
        assert kind in TENSOR_KINDS, kind
        self.uid = fresh_uid()
        self.dtype = dtype
        self.shape = tuple(shape)
        self.kind = kind
        self.deps = tuple(deps)
        self.name = name
        self.fn = fn
        self.init = init

    @property
    def numel(self) -> int:
        return numel(self.shape)

    def __repr__(self) -> str:  # pragma: no cover
        return f"<Tensor n{self.uid} {self.kind} {self.dtype.value} {shape_to_string(self.shape)}>"


# ---------------------------------------------------------------------------
# Graphs (lib/ir/graph.ml)
# ---------------------------------------------------------------------------
class Graph:
    """Named params in, named tensors out. Built from outputs only; params are
    discovered by back-tracing (lib/ir/graph.ml:97-103)."""

    def __init__(self, name: str, outputs):
        outputs = list(outputs)
        if not outputs:
            raise ValueError("Graph.create: a graph needs at least one output")
        seen = set()
        for n, _ in outputs:
            if n in seen:
                raise ValueError(f"Graph.create: duplicate output name {n!r}")
            seen.add(n)
        self.name = name
        self.outputs = [(n, t) for n, t in outputs]
        self.order = self._topo_sort()
        self.fan_out_tbl = {}
        for t in self.order:
            for d in t.deps:
                self.fan_out_tbl[d.uid] = self.fan_out_tbl.get(d.uid, 0) + 1
        params = []
        by_name = {}
        for t in self.order:
            if t.kind == "param":
                u = by_name.get(t.name)
                if u is not None and u != t.uid:
                    raise ValueError(f"Graph.create: two Param nodes named {t.name}")
                if u is None:
                    by_name[t.name] = t.uid
                params.append((t.name, t))
        self.params = params

    def _topo_sort(self):
        # Depth-first post-order, outputs in list order, deps in argument
        # order (lib/ir/graph.ml:51-63). Iterative to survive deep graphs.
        visited = set()
        acc = []
        for _, root in self.outputs:
            if root.uid in visited:
                continue
            stack = [(root, 0)]
            visited.add(root.uid)
            while stack:
                node, i = stack[-1]
                if i < len(node.deps):
                    stack[-1] = (node, i + 1)
                    d = node.deps[i]
                    if d.uid not in visited:
                        visited.add(d.uid)
                        stack.append((d, 0))
                else:
                    stack.pop()
                    acc.append(node)
        return acc

    def topological_order(self):
        return list(self.order)

    def fan_out(self, t: Tensor) -> int:
        return self.fan_out_tbl.get(t.uid, 0)

    def output(self, name: str) -> Tensor:
        for n, t in self.outputs:
            if n == name:
                return t
        raise KeyError(name)

    def param(self, name: str) -> Tensor:
        for n, t in self.params:
            if n == name:
                return t
        raise KeyError(name)

    def to_dot(self) -> str:
        """Graphviz text in the reference's format (graph.ml:115-150): one
        node per tensor labelled ``n<uid> <Kind> <shape> <dtype>``, one edge
        per dependency, names escaped."""
        lines = [f'digraph "{_dot_escape(self.name)}" {{']
        for t in self.order:
            label = f"n{t.uid} {_dot_kind(t)} {shape_to_string(t.shape)} {t.dtype.value}"
            lines.append(f'  n{t.uid} [label="{_dot_escape(label)}"];')
        for t in self.order:
            for d in t.deps:
                lines.append(f"  n{d.uid} -> n{t.uid};")
        lines.append("}")
        return "\n".join(lines) + "\n"


_DOT_KIND = {"iota": "Iota", "map": "Map", "map2": "Map2", "reduce": "Reduce", "scan": "Scan",
             "gather": "Gather", "scatter_add": "Scatter_add", "matmul": "Matmul", "reshape": "Reshape",
             "broadcast": "Broadcast"}


def _dot_kind(t: Tensor) -> str:
    return f"Param {t.name}" if t.kind == "param" else _DOT_KIND[t.kind]


def _dot_escape(s: str) -> str:
    return s.replace("\\", "\\\\").replace('"', '\\"').replace("\n", "\\n")


# ---------------------------------------------------------------------------
# Host values (lib/ir/value.ml): always contiguous, C order, owned storage.
# ---------------------------------------------------------------------------
class Value:
    """A host tensor: a dtype, a shape and a flat contiguous numpy array."""

    __slots__ = ("dtype", "shape", "data")

    def __init__(self, dtype: Dtype, shape, data: np.ndarray):
        shape = tuple(shape)
        if dtype is BOOL:
            raise ValueError("Value.create: Bool tensors are not storable")
        if data.dtype != np.dtype(dtype.np) or data.ndim != 1 or data.size != numel(shape):
            raise ValueError(
                f"Value: storage {data.dtype}[{data.size}] does not hold {dtype.value}{shape_to_string(shape)}")
        if not data.flags["C_CONTIGUOUS"]:
            raise ValueError("Value: storage must be contiguous")
        self.dtype = dtype
        self.shape = shape
        self.data = data

    @staticmethod
    def create(dtype: Dtype, shape) -> "Value":
        """Zero-filled, like the reference's [Value.create]."""
        if dtype is BOOL:
            raise ValueError("Value.create: Bool tensors are not storable")
        return Value(dtype, shape, np.zeros(numel(shape), dtype=dtype.np))

    @staticmethod
    def of_list(dtype: Dtype, shape, items) -> "Value":
        items = list(items)
        if len(items) != numel(shape):
            raise ValueError(
                f"Value.of_list: shape {shape_to_string(shape)} holds {numel(shape)} elements, got {len(items)}")
        return Value(dtype, shape, np.asarray(items, dtype=dtype.np).reshape(-1).copy())

    @staticmethod
    def of_array(dtype: Dtype, shape, arr) -> "Value":
        """Adopt (without copying when possible) a numpy array of the right kind."""
        a = np.ascontiguousarray(np.asarray(arr).reshape(-1))
        if a.dtype != np.dtype(dtype.np):
            raise ValueError(f"Value.of_array: array kind {a.dtype} does not match {dtype.value}")
        return Value(dtype, shape, a)

    @property
    def numel(self) -> int:
        return numel(self.shape)

    @property
    def byte_size(self) -> int:
        return self.numel * self.dtype.size_in_bytes

    def _index(self, i: int, what: str) -> int:
        # flat row-major index in [0, numel): no negative (from-the-end) indexing
        if not 0 <= i < self.data.size:
            raise IndexError(f"Value.{what}: index {i} out of bounds for {self.data.size} elements")
        return i

    def get(self, i: int):
        return self.data[self._index(i, "get")].item()

    def set(self, i: int, v) -> None:
        self.data[self._index(i, "set")] = v

    def to_list(self):
        return self.data.tolist()

    def array(self) -> np.ndarray:
        return self.data.reshape(self.shape) if self.shape else self.data.reshape(())

    def __repr__(self) -> str:  # pragma: no cover
        return f"Value({self.dtype.value}{shape_to_string(self.shape)})"


def f64_bits(x: float) -> int:
    return struct.unpack("<Q", struct.pack("<d", float(x)))[0]


def f32_round(x: float) -> float:
    """round_f32 of lib/backend_interp/cudacaml_backend_interp.ml:36."""
    return struct.unpack("<f", struct.pack("<f", x))[0]
