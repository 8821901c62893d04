"""Reverse-mode AD over the tensor DAG, restating CUDACaml's ``Grad``
(lib/ad/grad.ml). A graph -> graph transform that builds every adjoint from
``dsl`` calls only, so the gradient graph contains no node kind the backend
does not already lower. It is a producer of the graphs the hot path runs (the
Black-Scholes Greeks and the MLP step), not part of the hot path itself.
"""
from __future__ import annotations

from . import deriv as Deriv
from . import dsl as D
from .ir import BOOL, F32, F64, I32, I64, Graph, Tensor, row_length


class NotDifferentiable(Exception):
    pass


def grad_name(output: str, wrt: str) -> str:
    return "d" + output + "/d" + wrt


def _fconst(dt, v):
    if dt not in (F32, F64):
        raise NotDifferentiable(f"dtype {dt.value} carries no gradient")
    return D.const(dt, v)


def _zeros(dt, shape):
    if dt is BOOL:
        raise ValueError("Grad.grad: a bool tensor cannot hold a gradient")
    return D.full(dt, shape, 0.0 if dt.is_float else 0)


class _Tbl:
    def __init__(self):
        self.adj = {}

    def find(self, node: Tensor):
        a = self.adj.get(node.uid)
        if a is not None and a.dtype is not node.dtype:
            raise ValueError("Grad: internal adjoint dtype mismatch")
        return a

    def accumulate(self, node: Tensor, v: Tensor):
        a = self.find(node)
        self.adj[node.uid] = v if a is None else D.map2(D.add, a, v)

    def accum_into(self, tgt: Tensor, v: Tensor):
        # grad.ml:93-100: integer operands carry no adjoint; a float operand of
        # another float dtype takes the adjoint through a cast.
        if tgt.dtype.is_float:
            if tgt.dtype is v.dtype:
                self.accumulate(tgt, v)
            else:
                self.accumulate(tgt, D.map(lambda e: D.cast(tgt.dtype, e), v))


def _dfn1(what, fn):
    try:
        body = Deriv.d(fn.body1, 0)
    except ValueError as e:
        raise NotDifferentiable(f"{what}: {e}")
    return type(fn)(fn.arg1, body)


def _dfn2(what, fn, wrt):
    try:
        body = Deriv.d(fn.body2, wrt)
    except ValueError as e:
        raise NotDifferentiable(f"{what}: {e}")
    return type(fn)(fn.arg_a, fn.arg_b, body)


def _combining_binop(fn):
    """grad.ml:158-166: syntactically one binop over the two placeholders."""
    b = fn.body2
    if b.kind == "binop":
        x, y = b.args

        def is_arg(e, i):
            return e.kind == "arg" and e.value == i

        if (is_arg(x, 0) and is_arg(y, 1)) or (is_arg(x, 1) and is_arg(y, 0)):
            return b.op
    return None


def _rows_of(src_shape, t: Tensor) -> Tensor:
    """out[k] = t[k / n] (grad.ml:184-189)."""
    n = row_length(src_shape)
    ni = D.const(I32, n)
    idx = D.map(lambda k: D.div(k, ni), D.iota(src_shape))
    return D.gather(idx, t)


def _reduce_last(t: Tensor) -> Tensor:
    init = _fconst(t.dtype, 0.0)
    if len(t.shape) <= 1:
        return D.reduce(D.add, init, t)
    return D.reduce_rows(D.add, init, t)


def _scan_last(t: Tensor) -> Tensor:
    init = _fconst(t.dtype, 0.0)
    if len(t.shape) <= 1:
        return D.scan(D.add, init, t)
    return D.scan_rows(D.add, init, t)


def _back_node(tbl: _Tbl, t: Tensor, abar: Tensor) -> None:
    """grad.ml:211-305: push the completed adjoint of t to its operands."""
    k = t.kind
    if k in ("param", "iota"):
        return
    if k == "map":
        (src,) = t.deps
        if src.dtype.is_float:
            df = _dfn1("Map", t.fn)
            tbl.accum_into(src, D.map2(lambda adj, x: D.mul(adj, Deriv.apply1(df, x)), abar, src))
        return
    if k == "map2":
        xa, xb = t.deps
        for wrt, tgt in ((0, xa), (1, xb)):
            if tgt.dtype.is_float:
                df = _dfn2("Map2", t.fn, wrt)
                dk = D.map2(lambda x, y, df=df: Deriv.apply2(df, x, y), xa, xb)
                tbl.accum_into(tgt, D.map2(D.mul, abar, dk))
        return
    if k == "reduce":
        (src,) = t.deps
        op = _combining_binop(t.fn)

        def spread(u):
            return _rows_of(src.shape, u)

        if op == "add":
            tbl.accum_into(src, spread(abar))
        elif op in ("max", "min"):
            m = spread(t)
            one = _fconst(t.dtype, 1.0)
            zero = _fconst(t.dtype, 0.0)
            mask = D.map2(lambda x, mv: D.select(D.eq(x, mv), one, zero), src, m)
            tbl.accum_into(src, D.map2(D.mul, spread(abar), mask))
        elif op == "mul":
            q = D.map2(D.div, spread(t), src)
            tbl.accum_into(src, D.map2(D.mul, spread(abar), q))
        elif op is None:
            raise NotDifferentiable("Reduce <unrecognised operator>")
        else:
            raise NotDifferentiable(f"Reduce {op}")
        return
    if k == "scan":
        (src,) = t.deps
        op = _combining_binop(t.fn)
        if op == "add":
            total = _rows_of(src.shape, _reduce_last(abar))
            prefix = _scan_last(abar)
            tbl.accum_into(src, D.map2(D.add, D.map2(D.sub, total, prefix), abar))
        elif op is None:
            raise NotDifferentiable("Scan <unrecognised operator>")
        else:
            raise NotDifferentiable(f"Scan {op}")
        return
    if k == "gather":
        idx, src = t.deps
        if src.dtype.is_float:
            tbl.accumulate(src, D.scatter_add(idx, abar, src.shape))
        return
    if k == "scatter_add":
        idx, src = t.deps
        tbl.accum_into(src, D.gather(idx, abar))
        return
    if k == "matmul":
        xa, xb = t.deps
        if xa.dtype.is_float:
            tbl.accum_into(xa, D.matmul(abar, D.transpose(xb)))
        if xb.dtype.is_float:
            tbl.accum_into(xb, D.matmul(D.transpose(xa), abar))
        return
    if k == "reshape":
        (src,) = t.deps
        tbl.accum_into(src, D.reshape(src.shape, abar))
        return
    if k == "broadcast":
        (src,) = t.deps
        total = D.reduce(D.add, _fconst(t.dtype, 0.0), abar)
        tbl.accum_into(src, D.reshape(src.shape, total))
        return
    raise AssertionError(k)


def grad(g: Graph, output: str, wrt) -> Graph:
    """grad.ml:334-348: outputs of g plus d<output>/d<p> for every p in wrt."""
    outs = dict(g.outputs)
    params = dict(g.params)
    if output not in outs:
        raise ValueError(f"Grad.grad: no output named {output!r}")
    wrt_nodes = []
    for p in wrt:
        if p not in params:
            raise ValueError(f"Grad.grad: no param named {p!r}")
        wrt_nodes.append((p, params[p]))
    out = outs[output]
    if not out.dtype.is_float:
        raise ValueError(f"Grad.grad: output has dtype {out.dtype.value}, a float dtype is required")
    tbl = _Tbl()
    tbl.accumulate(out, D.full(out.dtype, out.shape, 1.0))
    for t in reversed(g.topological_order()):
        abar = tbl.find(t)
        if abar is not None:
            _back_node(tbl, t, abar)
    grads = []
    for p, node in wrt_nodes:
        a = tbl.find(node)
        grads.append((grad_name(output, p), a if a is not None else _zeros(node.dtype, node.shape)))
    return Graph(g.name + "_grad", list(g.outputs) + grads)
