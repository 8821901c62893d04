"""The user-facing surface, restating CUDACaml's ``Dsl`` (lib/ir/dsl.mli,
lib/ir/dsl.ml). Every function only builds IR nodes; nothing here runs.

Names shadow Python builtins (``map``, ``min``, ``max``, ``abs``) exactly as
the OCaml ``Dsl`` shadows ``Stdlib``; import the module qualified
(``from cudacaml_b200 import dsl as D``).
"""
from __future__ import annotations

import builtins

from .ir import (BOOL, F32, F64, I32, I64, Dtype, Expr, Tensor, make_fn1, make_fn2, numel,
                 shape_of, shape_to_string, SCALAR)

_map = builtins.map


# ---------------------------------------------------------------------------
# Tensors (lib/ir/dsl.ml:1-196)
# ---------------------------------------------------------------------------
def param(name: str, dtype: Dtype, shape) -> Tensor:
    return Tensor(dtype, shape_of(shape), "param", name=name)


def iota(shape) -> Tensor:
    return Tensor(I32, shape_of(shape), "iota")


def map(f, src: Tensor) -> Tensor:  # noqa: A001 - mirrors Dsl.map
    fn = make_fn1(src.dtype, f)
    return Tensor(fn.body1.dtype, src.shape, "map", deps=(src,), fn=fn)


def map2(f, a: Tensor, b: Tensor) -> Tensor:
    # No broadcasting: both operands must have the same shape (dsl.ml:8-13).
    if a.shape != b.shape:
        raise ValueError(f"Dsl.map2: shape mismatch: {shape_to_string(a.shape)} vs {shape_to_string(b.shape)}")
    fn = make_fn2(a.dtype, b.dtype, f)
    return Tensor(fn.body2.dtype, a.shape, "map2", deps=(a, b), fn=fn)


def gather(idx: Tensor, src: Tensor) -> Tensor:
    return Tensor(src.dtype, idx.shape, "gather", deps=(idx, src))


def scatter_add(idx: Tensor, src: Tensor, shape) -> Tensor:
    """out = zeros shape; out[idx[i]] += src[i] (dsl.ml:28-41)."""
    shape = shape_of(shape)
    if idx.shape != src.shape:
        raise ValueError(
            f"Dsl.scatter_add: idx shape {shape_to_string(idx.shape)} does not match src shape {shape_to_string(src.shape)}")
    if src.dtype not in (F32, F64, I32):
        raise ValueError(f"Dsl.scatter_add: dtype {src.dtype.value} cannot be accumulated")
    return Tensor(src.dtype, shape, "scatter_add", deps=(idx, src))


def reshape(shape, src: Tensor) -> Tensor:
    shape = shape_of(shape)
    if numel(shape) != numel(src.shape):
        raise ValueError(
            f"Dsl.reshape: numel mismatch: {shape_to_string(shape)} ({numel(shape)}) vs "
            f"{shape_to_string(src.shape)} ({numel(src.shape)})")
    return Tensor(src.dtype, shape, "reshape", deps=(src,))


def _flatten(src: Tensor) -> Tensor:
    return reshape((numel(src.shape),), src)


def reduce(f, init: Expr, src: Tensor) -> Tensor:
    """Whole-tensor reduction to a scalar; rank >= 2 is flattened first
    (dsl.ml:67-74)."""
    fn = make_fn2(src.dtype, src.dtype, f)
    if len(src.shape) == 1:
        return Tensor(src.dtype, SCALAR, "reduce", deps=(src,), fn=fn, init=init)
    flat = _flatten(src)
    return Tensor(src.dtype, SCALAR, "reduce", deps=(flat,), fn=fn, init=init)


def scan(f, init: Expr, src: Tensor) -> Tensor:
    fn = make_fn2(src.dtype, src.dtype, f)
    if len(src.shape) == 1:
        return Tensor(src.dtype, src.shape, "scan", deps=(src,), fn=fn, init=init)
    flat = _flatten(src)
    scanned = Tensor(src.dtype, flat.shape, "scan", deps=(flat,), fn=fn, init=init)
    return reshape(src.shape, scanned)


def reduce_rows(f, init: Expr, src: Tensor) -> Tensor:
    if len(src.shape) < 2:
        raise ValueError(f"Dsl.reduce_rows: rank >= 2 required, got {shape_to_string(src.shape)}")
    fn = make_fn2(src.dtype, src.dtype, f)
    return Tensor(src.dtype, src.shape[:-1], "reduce", deps=(src,), fn=fn, init=init)


def scan_rows(f, init: Expr, src: Tensor) -> Tensor:
    if len(src.shape) < 2:
        raise ValueError(f"Dsl.scan_rows: rank >= 2 required, got {shape_to_string(src.shape)}")
    fn = make_fn2(src.dtype, src.dtype, f)
    return Tensor(src.dtype, src.shape, "scan", deps=(src,), fn=fn, init=init)


def broadcast(shape, src: Tensor) -> Tensor:
    shape = shape_of(shape)
    if numel(src.shape) != 1:
        raise ValueError(
            f"Dsl.broadcast: source must have exactly one element: {shape_to_string(src.shape)} ({numel(src.shape)})")
    return Tensor(src.dtype, shape, "broadcast", deps=(src,))


def full(dtype: Dtype, shape, v) -> Tensor:
    """A map over iota whose body ignores its argument (dsl.ml:150-153)."""
    return map(lambda _: const(dtype, v), iota(shape))


def scalar(name: str, dtype: Dtype) -> Tensor:
    return param(name, dtype, SCALAR)


def transpose(x: Tensor) -> Tensor:
    """A gather over a computed iota index: out[k] = x[(k mod m) * n + k / m]
    for x : [m; n] (dsl.ml:167-182)."""
    if len(x.shape) != 2:
        raise ValueError(f"Dsl.transpose: rank 2 required, got {shape_to_string(x.shape)}")
    m, n = x.shape
    mi = const(I32, m)
    ni = const(I32, n)

    def body(k):
        q = div(k, mi)
        return add(mul(sub(k, mul(q, mi)), ni), q)

    idx = map(body, iota((n, m)))
    return gather(idx, x)


def matmul(a: Tensor, b: Tensor) -> Tensor:
    if len(a.shape) == 2 and len(b.shape) == 2 and a.shape[1] == b.shape[0]:
        return Tensor(a.dtype, (a.shape[0], b.shape[1]), "matmul", deps=(a, b))
    raise ValueError(
        f"Dsl.matmul: need [m; k] x [k; n], got {shape_to_string(a.shape)} x {shape_to_string(b.shape)}")


# ---------------------------------------------------------------------------
# Scalars, inside element functions (dsl.ml:199-260)
# ---------------------------------------------------------------------------
def const(dtype: Dtype, v) -> Expr:
    if dtype.is_float:
        v = float(v)
    elif dtype is I32:
        v = int(v)
        v = (v + 2**31) % 2**32 - 2**31  # Int32 literals wrap like Int32.of_string
    elif dtype is I64:
        v = int(v)
        v = (v + 2**63) % 2**64 - 2**63
    else:
        v = bool(v)
    return Expr(dtype, "const", value=v)


def index() -> Expr:
    return Expr(I32, "index")


def _binop(op, a: Expr, b: Expr) -> Expr:
    return Expr(a.dtype, "binop", op=op, args=(a, b))


def _unop(op, a: Expr) -> Expr:
    return Expr(a.dtype, "unop", op=op, args=(a,))


def _cmp(op, a: Expr, b: Expr) -> Expr:
    return Expr(BOOL, "cmp", op=op, args=(a, b))


def add(a, b): return _binop("add", a, b)
def sub(a, b): return _binop("sub", a, b)
def mul(a, b): return _binop("mul", a, b)
def div(a, b): return _binop("div", a, b)
def min(a, b): return _binop("min", a, b)  # noqa: A001
def max(a, b): return _binop("max", a, b)  # noqa: A001
def bit_and(a, b): return _binop("bit_and", a, b)
def bit_or(a, b): return _binop("bit_or", a, b)
def bit_xor(a, b): return _binop("bit_xor", a, b)
def shl(a, b): return _binop("shl", a, b)
def shr(a, b): return _binop("shr", a, b)
def neg(a): return _unop("neg", a)
def sqrt(a): return _unop("sqrt", a)
def exp(a): return _unop("exp", a)
def log(a): return _unop("log", a)
def abs(a): return _unop("abs", a)  # noqa: A001
def sin(a): return _unop("sin", a)
def cos(a): return _unop("cos", a)
def erf(a): return _unop("erf", a)
def erfinv(a): return _unop("erfinv", a)
def lt(a, b): return _cmp("lt", a, b)
def le(a, b): return _cmp("le", a, b)
def eq(a, b): return _cmp("eq", a, b)
def ne(a, b): return _cmp("ne", a, b)
def gt(a, b): return _cmp("gt", a, b)
def ge(a, b): return _cmp("ge", a, b)
def and_(a, b): return Expr(BOOL, "logic", op="and", args=(a, b))
def or_(a, b): return Expr(BOOL, "logic", op="or", args=(a, b))
def not_(a): return Expr(BOOL, "not", args=(a,))
def select(c, a, b): return Expr(a.dtype, "select", args=(c, a, b))
def cast(dtype: Dtype, e: Expr) -> Expr: return Expr(dtype, "cast", args=(e,))
