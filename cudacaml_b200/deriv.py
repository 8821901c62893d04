"""Symbolic differentiation of element expressions, restating CUDACaml's
``Deriv`` (lib/ad/deriv.ml). Graph producer only: it builds the expressions the
gradient graphs carry, so the graphs this backend runs match the reference's.
"""
from __future__ import annotations

import math

from . import dsl as D
from .ir import BOOL, F32, F64, Expr, f32_round

TWO_OVER_SQRT_PI = 2.0 / math.sqrt(math.pi)
SQRT_PI_OVER_TWO = math.sqrt(math.pi) / 2.0


def _fconst(dt, v):
    if dt not in (F32, F64):
        raise ValueError(f"Deriv: dtype {dt.value} is not differentiable")
    return D.const(dt, v)


def _fold_arith(op, x, y):
    # deriv.ml:46-53: arithmetic only; a division by a zero constant is kept.
    if op == "add":
        return x + y
    if op == "sub":
        return x - y
    if op == "mul":
        return x * y
    if op == "div":
        return None if y == 0.0 else x / y
    return None


def _fold_binop(dt, op, x, y):
    if dt is F32:
        r = _fold_arith(op, x, y)
        return None if r is None else f32_round(r)
    if dt is F64:
        return _fold_arith(op, x, y)
    return None


def _is_lit(e: Expr, v: float) -> bool:
    return e.kind == "const" and e.dtype in (F32, F64) and e.value == v


def simplify(e: Expr) -> Expr:
    """deriv.ml:78-141: constant folding and the 0/1 identities, float only."""
    dt = e.dtype
    k = e.kind
    if k in ("const", "arg", "index"):
        return e
    if k == "binop":
        a0, b0 = e.args
        a, b = simplify(a0), simplify(b0)

        def keep():
            return e if (a is a0 and b is b0) else Expr(dt, "binop", op=e.op, args=(a, b))

        if a.kind == "const" and b.kind == "const":
            r = _fold_binop(dt, e.op, a.value, b.value)
            if r is not None:
                return Expr(dt, "const", value=r)
        op = e.op
        if op == "mul":
            if _is_lit(b, 0.0):
                return b
            if _is_lit(a, 0.0):
                return a
            if _is_lit(b, 1.0):
                return a
            if _is_lit(a, 1.0):
                return b
            return keep()
        if op == "add":
            if _is_lit(b, 0.0):
                return a
            if _is_lit(a, 0.0):
                return b
            return keep()
        if op == "sub":
            if _is_lit(b, 0.0):
                return a
            if _is_lit(a, 0.0):
                return Expr(dt, "unop", op="neg", args=(b,))
            return keep()
        return keep()
    if k == "unop":
        (a0,) = e.args
        a = simplify(a0)
        if e.op == "neg" and a.kind == "unop" and a.op == "neg":
            return a.args[0]
        return e if a is a0 else Expr(dt, "unop", op=e.op, args=(a,))
    if k in ("cmp", "logic"):
        a0, b0 = e.args
        a, b = simplify(a0), simplify(b0)
        return e if (a is a0 and b is b0) else Expr(dt, k, op=e.op, args=(a, b))
    if k == "not":
        (a0,) = e.args
        a = simplify(a0)
        return e if a is a0 else Expr(dt, "not", args=(a,))
    if k == "select":
        c0, a0, b0 = e.args
        c, a, b = simplify(c0), simplify(a0), simplify(b0)
        if a.uid == b.uid:
            return a
        if c is c0 and a is a0 and b is b0:
            return e
        return Expr(dt, "select", args=(c, a, b))
    if k == "cast":
        (x0,) = e.args
        x = simplify(x0)
        if x.dtype is dt:
            return x
        return e if x is x0 else Expr(dt, "cast", args=(x,))
    raise AssertionError(k)


def _deriv(e: Expr, wrt: int) -> Expr:
    """deriv.ml:150-207. Kinks take the branch taken at the point, ties to the
    first operand."""
    dt = e.dtype
    k = e.kind
    if k == "const":
        return _fconst(dt, 0.0)
    if k == "arg":
        return _fconst(dt, 1.0 if e.value == wrt else 0.0)
    if k == "index":
        return _fconst(dt, 0.0)
    if k == "binop":
        a, b = e.args
        op = e.op
        if op == "add":
            return D.add(_deriv(a, wrt), _deriv(b, wrt))
        if op == "sub":
            return D.sub(_deriv(a, wrt), _deriv(b, wrt))
        if op == "mul":
            return D.add(D.mul(_deriv(a, wrt), b), D.mul(a, _deriv(b, wrt)))
        if op == "div":
            return D.div(D.sub(D.mul(_deriv(a, wrt), b), D.mul(a, _deriv(b, wrt))), D.mul(b, b))
        if op == "min":
            return D.select(D.le(a, b), _deriv(a, wrt), _deriv(b, wrt))
        if op == "max":
            return D.select(D.ge(a, b), _deriv(a, wrt), _deriv(b, wrt))
        raise ValueError(f"Deriv.d: {op} is integer only")
    if k == "unop":
        (a,) = e.args
        da = _deriv(a, wrt)
        op = e.op
        if op == "neg":
            return D.neg(da)
        if op == "sqrt":
            return D.div(da, D.mul(_fconst(dt, 2.0), D.sqrt(a)))
        if op == "exp":
            return D.mul(D.exp(a), da)
        if op == "log":
            return D.div(da, a)
        if op == "abs":
            return D.select(D.lt(a, _fconst(dt, 0.0)), D.neg(da), da)
        if op == "sin":
            return D.mul(D.cos(a), da)
        if op == "cos":
            return D.mul(D.neg(D.sin(a)), da)
        if op == "erf":
            return D.mul(D.mul(_fconst(dt, TWO_OVER_SQRT_PI), D.exp(D.neg(D.mul(a, a)))), da)
        if op == "erfinv":
            y = D.erfinv(a)
            return D.mul(D.mul(_fconst(dt, SQRT_PI_OVER_TWO), D.exp(D.mul(y, y))), da)
        raise AssertionError(op)
    if k in ("cmp", "logic", "not"):
        raise ValueError("Deriv.d: a boolean expression has dtype bool")
    if k == "select":
        c, a, b = e.args
        return D.select(c, _deriv(a, wrt), _deriv(b, wrt))
    if k == "cast":
        (x,) = e.args
        if x.dtype.is_float:
            return D.cast(dt, _deriv(x, wrt))
        return _fconst(dt, 0.0)
    raise AssertionError(k)


def d(e: Expr, wrt: int) -> Expr:
    if not e.dtype.is_float:
        raise ValueError(f"Deriv.d: expression has dtype {e.dtype.value}, a float dtype is required")
    return simplify(_deriv(e, wrt))


def subst(args: dict, e: Expr) -> Expr:
    """Rebuild with fresh uids, substituting Arg i (deriv.ml:231-255)."""
    memo = {}

    def go(x: Expr) -> Expr:
        if x.uid in memo:
            return memo[x.uid]
        if x.kind == "arg":
            s = args.get(x.value)
            if s is None:
                r = Expr(x.dtype, "arg", value=x.value)
            else:
                if s.dtype is not x.dtype:
                    raise ValueError(
                        f"Deriv.apply: Arg {x.value} has dtype {x.dtype.value} but the substitute has dtype {s.dtype.value}")
                r = s
        elif x.kind == "const":
            r = Expr(x.dtype, "const", value=x.value)
        elif x.kind == "index":
            r = Expr(x.dtype, "index")
        else:
            r = Expr(x.dtype, x.kind, op=x.op, args=tuple(go(a) for a in x.args), value=x.value)
        memo[x.uid] = r
        return r

    return go(e)


def apply1(fn, x: Expr) -> Expr:
    if fn.arg1.dtype is not x.dtype:
        raise ValueError("Deriv.apply1: argument dtype mismatch")
    return subst({0: x}, fn.body1)


def apply2(fn, x: Expr, y: Expr) -> Expr:
    if fn.arg_a.dtype is not x.dtype or fn.arg_b.dtype is not y.dtype:
        raise ValueError("Deriv.apply2: argument dtype mismatch")
    return subst({0: x, 1: y}, fn.body2)
