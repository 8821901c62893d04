"""Deriv (symbolic derivatives of element expressions) against central
differences on the oracle in F64, and structural checks that pin the
simplifier and substitution (the reference's test/unit/test_deriv.ml cases).
The Greeks' adjoint passes are built from these rules. CPU only.
"""
import numpy as np
import pytest

from cudacaml_b200 import deriv as Deriv
from cudacaml_b200 import dsl as D
from cudacaml_b200.ir import F32, F64, I32, Expr, Fn1, Graph, Tensor, Value, make_fn1, make_fn2
from oracle import interp as I

H = 1e-6


def k(v):
    return D.const(F64, v)


def run(g, inputs):
    return dict(I.run(I.compile(g), inputs))


def vec(xs):
    return Value.of_list(F64, (len(xs),), xs)


def eval_f(f, xs):
    x = D.param("x", F64, (len(xs),))
    return run(Graph("f", [("r", D.map(f, x))]), [("x", vec(xs))])["r"].data


def eval_df(f, xs):
    """f' as Deriv builds it, evaluated at every point."""
    x = D.param("x", F64, (len(xs),))
    fn = make_fn1(F64, f)
    dfn = Fn1(fn.arg1, Deriv.d(fn.body1, 0))
    r = Tensor(F64, (len(xs),), "map", deps=(x,), fn=dfn)
    return run(Graph("df", [("r", r)]), [("x", vec(xs))])["r"].data


def fd(f, xs):
    xs = np.array(xs, float)
    return (eval_f(f, list(xs + H)) - eval_f(f, list(xs - H))) / (2 * H)


RULES = [
    ("3x^2 - 2x + 1", lambda x: D.add(D.sub(D.mul(k(3.0), D.mul(x, x)), D.mul(k(2.0), x)), k(1.0)), [-2, -0.5, 0, 1, 3]),
    ("x / (1 + x^2)", lambda x: D.div(x, D.add(k(1.0), D.mul(x, x))), [-2, -0.5, 0, 1, 3]),
    ("sqrt", D.sqrt, [0.5, 1, 4]),
    ("exp", D.exp, [-1, 0, 2]),
    ("log", D.log, [0.5, 1, 3]),
    ("sin", D.sin, [0, 1, -2]),
    ("cos", D.cos, [0, 1, -2]),
    ("erf", D.erf, [-1, 0, 0.5]),
    ("erfinv", D.erfinv, [-0.9, -0.3, 0, 0.5, 0.9]),
    ("abs away from 0", D.abs, [-2, -0.5, 1, 3]),
    ("min(x, 1)", lambda x: D.min(x, k(1.0)), [-1, 0, 2, 3]),
    ("max(x, 1)", lambda x: D.max(x, k(1.0)), [-1, 0, 2, 3]),
    ("select(x<0, x^2, exp x)", lambda x: D.select(D.lt(x, k(0.0)), D.mul(x, x), D.exp(x)), [-2, -1, 1, 2]),
    ("exp(sin x) * log(1 + x^2)", lambda x: D.mul(D.exp(D.sin(x)), D.log(D.add(k(1.0), D.mul(x, x)))), [-1.5, 0.3, 2]),
]


@pytest.mark.parametrize("name,f,xs", RULES, ids=[r[0] for r in RULES])
def test_rule_against_central_difference(name, f, xs):
    xs = [float(v) for v in xs]
    want, got = fd(f, xs), eval_df(f, xs)
    assert np.all(np.abs(want - got) <= 1e-6 * (1 + np.abs(want))), (name, want, got)


def test_fn2_partials():
    fn = make_fn2(F64, F64, lambda a, b: D.add(D.mul(a, b), D.sin(a)))
    xs, ys = [1.0, -0.5], [2.0, 3.0]
    x, y = D.param("x", F64, (2,)), D.param("y", F64, (2,))
    dx = Tensor(F64, (2,), "map2", deps=(x, y), fn=type(fn)(fn.arg_a, fn.arg_b, Deriv.d(fn.body2, 0)))
    dy = Tensor(F64, (2,), "map2", deps=(x, y), fn=type(fn)(fn.arg_a, fn.arg_b, Deriv.d(fn.body2, 1)))
    o = run(Graph("g", [("dx", dx), ("dy", dy)]), [("x", vec(xs)), ("y", vec(ys))])
    assert np.allclose(o["dx"].data, [b + np.cos(a) for a, b in zip(xs, ys)], rtol=0, atol=1e-12)
    assert np.allclose(o["dy"].data, xs, rtol=0, atol=1e-12)


def test_cast_of_integer_index_has_zero_derivative():
    # d/dx (cast index * x) = cast index: the integer part contributes nothing
    got = eval_df(lambda x: D.mul(D.cast(F64, D.index()), x), [5.0, 5.0, 5.0])
    assert np.array_equal(got, [0.0, 1.0, 2.0])


def test_integer_expression_raises():
    fn = make_fn1(I32, lambda x: D.mul(x, x))
    with pytest.raises(ValueError):
        Deriv.d(fn.body1, 0)


def test_structural_constants_and_args():
    def is_const(v, e):
        assert e.kind == "const" and e.value == v

    is_const(0.0, Deriv.d(k(5.0), 0))
    is_const(1.0, Deriv.d(Expr(F64, "arg", value=0), 0))
    is_const(0.0, Deriv.d(Expr(F64, "arg", value=1), 0))


def _has_arg(e):
    return e.kind == "arg" or any(_has_arg(a) for a in e.args)


def _uids(e):
    return [e.uid] + [u for a in e.args for u in _uids(a)]


def test_apply1_substitutes_checks_dtype_and_shares_no_uids():
    fn = make_fn1(F64, lambda x: D.add(D.mul(x, x), k(1.0)))
    assert not _has_arg(Deriv.apply1(fn, k(2.0)))
    with pytest.raises(ValueError):
        Deriv.apply1(fn, D.const(F32, 2.0))
    fresh = Deriv.apply1(fn, Expr(F64, "arg", value=3))
    assert not set(_uids(fresh)) & set(_uids(fn.body1))


def test_apply2_substitutes_both_arguments():
    fn = make_fn2(F64, F64, lambda a, b: D.sub(a, b))
    r = Deriv.apply2(fn, k(5.0), k(3.0))
    assert not _has_arg(r)
    assert np.array_equal(eval_f(lambda _: r, [0.0]), [2.0])


def test_simplify():
    x, y = Expr(F64, "arg", value=0), Expr(F64, "arg", value=1)
    s = Deriv.simplify(D.add(D.mul(x, k(0.0)), D.mul(y, k(1.0))))
    assert s.kind == "arg" and s.value == 1, "x*0 + y*1 simplifies to y"
    s = Deriv.simplify(D.neg(D.neg(x)))
    assert s.kind == "arg" and s.value == 0, "neg neg x"
    s = Deriv.simplify(D.add(k(2.0), k(3.0)))
    assert s.kind == "const" and s.value == 5.0
    s = Deriv.simplify(D.div(k(1.0), k(0.0)))
    assert s.kind == "binop" and s.op == "div", "division by a constant zero must not fold"
