"""Grad.grad against bump-and-revalue on the oracle, in F64 (the reference's
test/unit/test_grad.ml cases). The Greeks and the MLP step on the benchmark
path are Grad-produced graphs, so the adjoint rules are checked here once,
on the host, before the lowering ever sees them. CPU only.
"""
import numpy as np
import pytest

from cudacaml_b200 import dsl as D
from cudacaml_b200 import grad as G
from cudacaml_b200.ir import F64, I32, Graph, Value
from oracle import interp as I

XS4 = [1.0, -2.0, 0.5, 3.0]
YS4 = [0.3, 1.5, -1.0, 2.0]
ZERO = D.const(F64, 0.0)


def run(g, inputs):
    return dict(I.run(I.compile(g), inputs))


def f64(dims, items):
    return Value.of_list(F64, tuple(dims), items)


def p(name, dims):
    return D.param(name, F64, tuple(dims))


def total(g, output, inputs):
    return float(np.sum(run(g, inputs)[output].data))


def fd(g, output, wrt, inputs, h=1e-6):
    """Central difference of sum(output) wrt every element of input `wrt`,
    by rerunning the original graph."""
    base = dict(inputs)[wrt]
    out = []
    for i in range(base.numel):
        def bumped(delta):
            v = base.data.copy()
            v[i] += delta
            return [(nm, Value.of_array(F64, base.shape, v) if nm == wrt else x) for nm, x in inputs]
        out.append((total(g, output, bumped(h)) - total(g, output, bumped(-h))) / (2 * h))
    return np.array(out)


def grad_vs_fd(g, output, wrt, inputs, tol=1e-5):
    gg = G.grad(g, output, wrt)
    o = run(gg, inputs)
    for w in wrt:
        got = o[G.grad_name(output, w)].data
        want = fd(g, output, w, inputs)
        assert np.all(np.abs(want - got) <= tol * (1 + np.abs(want))), (w, want, got)
    return o


def one(name, t):
    return [(name, t)]


def test_sum_square_is_2x():
    x = p("x", [4])
    g = Graph("g", one("s", D.reduce(D.add, ZERO, D.map(lambda e: D.mul(e, e), x))))
    o = grad_vs_fd(g, "s", ["x"], [("x", f64([4], XS4))])
    assert np.allclose(o["ds/dx"].data, 2 * np.array(XS4), rtol=0, atol=1e-9)


def test_sum_product_gives_the_other_factor():
    x, y = p("x", [4]), p("y", [4])
    g = Graph("g", one("s", D.reduce(D.add, ZERO, D.map2(D.mul, x, y))))
    o = grad_vs_fd(g, "s", ["x", "y"], [("x", f64([4], XS4)), ("y", f64([4], YS4))])
    assert np.allclose(o["ds/dx"].data, YS4, rtol=0, atol=1e-9)
    assert np.allclose(o["ds/dy"].data, XS4, rtol=0, atol=1e-9)


def test_chain_exp_sin():
    x, y = p("x", [4]), p("y", [4])
    r = D.map2(lambda a, b: D.add(D.mul(D.exp(a), b), D.sin(D.mul(a, b))), x, y)
    g = Graph("g", one("s", D.reduce(D.add, ZERO, r)))
    grad_vs_fd(g, "s", ["x", "y"], [("x", f64([4], XS4)), ("y", f64([4], YS4))])


def test_reduce_max_is_the_argmax_indicator():
    x = p("x", [4])
    g = Graph("g", one("m", D.reduce(D.max, D.const(F64, -1e300), x)))
    o = grad_vs_fd(g, "m", ["x"], [("x", f64([4], [1.0, 5.0, 3.0, 2.0]))])
    assert np.array_equal(o["dm/dx"].data, [0.0, 1.0, 0.0, 0.0])


def test_reduce_rows_then_weighted_sum():
    x, w = p("x", [2, 3]), p("w", [2])
    g = Graph("g", one("s", D.reduce(D.add, ZERO, D.map2(D.mul, w, D.reduce_rows(D.add, ZERO, x)))))
    ins = [("x", f64([2, 3], [1, 2, 3, 4, 5, 6])), ("w", f64([2], [10.0, 20.0]))]
    o = grad_vs_fd(g, "s", ["x", "w"], ins)
    assert np.allclose(o["ds/dx"].data, [10, 10, 10, 20, 20, 20], rtol=0, atol=1e-9)
    assert o["ds/dx"].shape == (2, 3)


def test_scan_adjoint_is_reverse_cumsum_of_weights():
    x, w = p("x", [4]), p("w", [4])
    g = Graph("g", one("s", D.reduce(D.add, ZERO, D.map2(D.mul, w, D.scan(D.add, ZERO, x)))))
    o = grad_vs_fd(g, "s", ["x"], [("x", f64([4], XS4)), ("w", f64([4], YS4))])
    assert np.allclose(o["ds/dx"].data, np.cumsum(YS4[::-1])[::-1], rtol=0, atol=1e-9)


def test_scan_rows_adjoint_per_row():
    x, w = p("x", [2, 3]), p("w", [2, 3])
    g = Graph("g", one("s", D.reduce(D.add, ZERO, D.map2(D.mul, w, D.scan_rows(D.add, ZERO, x)))))
    vals = [1, 2, 3, 4, 5, 6]
    o = grad_vs_fd(g, "s", ["x"], [("x", f64([2, 3], vals)), ("w", f64([2, 3], vals))])
    assert np.allclose(o["ds/dx"].data, [6, 5, 3, 15, 11, 6], rtol=0, atol=1e-9)


def test_broadcast_scalar_gradient_is_the_sum_with_shape_scalar():
    x, s = p("x", [4]), D.scalar("s", F64)
    g = Graph("g", one("t", D.reduce(D.add, ZERO, D.map2(D.mul, x, D.broadcast((4,), s)))))
    o = grad_vs_fd(g, "t", ["s", "x"], [("x", f64([4], XS4)), ("s", f64([], [1.7]))])
    assert abs(o["dt/ds"].get(0) - sum(XS4)) <= 1e-9
    assert o["dt/ds"].shape == ()


def test_reshape_passes_the_adjoint_with_the_param_shape():
    x = p("x", [2, 3])
    g = Graph("g", one("s", D.reduce(D.add, ZERO, D.map(lambda e: D.mul(e, e), D.reshape((6,), x)))))
    vals = [1, 2, 3, 4, 5, 6]
    o = grad_vs_fd(g, "s", ["x"], [("x", f64([2, 3], vals))])
    assert o["ds/dx"].shape == (2, 3)
    assert np.allclose(o["ds/dx"].data, 2 * np.array(vals, float), rtol=0, atol=1e-9)


def test_non_scalar_output_is_seeded_with_ones():
    x, y = p("x", [4]), p("y", [4])
    g = Graph("g", one("r", D.map2(D.mul, x, y)))
    o = grad_vs_fd(g, "r", ["x"], [("x", f64([4], XS4)), ("y", f64([4], YS4))])
    assert np.allclose(o["dr/dx"].data, YS4, rtol=0, atol=1e-9)


def test_unused_param_gets_zeros_of_its_shape():
    x, y = p("x", [4]), p("y", [2, 2])
    g = Graph("g", [("s", D.reduce(D.add, ZERO, x)), ("y", y)])
    o = run(G.grad(g, "s", ["y"]), [("x", f64([4], XS4)), ("y", f64([2, 2], YS4))])
    assert np.array_equal(o["ds/dy"].data, np.zeros(4))
    assert o["ds/dy"].shape == (2, 2)


def test_unrecognised_reduce_operator_is_not_differentiable():
    x = p("x", [4])
    g = Graph("g", one("s", D.reduce(lambda a, b: D.add(D.mul(a, b), a), ZERO, x)))
    with pytest.raises(G.NotDifferentiable, match="Reduce"):
        G.grad(g, "s", ["x"])


def test_gather_adjoint_accumulates_repeats_and_zeroes_unread():
    x, idx = p("x", [3]), D.param("idx", I32, (3,))
    g = Graph("g", one("s", D.reduce(D.add, ZERO, D.gather(idx, x))))
    ins = [("x", f64([3], [1.0, 2.0, 3.0])), ("idx", Value.of_list(I32, (3,), [0, 0, 1]))]
    o = grad_vs_fd(g, "s", ["x"], ins)
    assert np.array_equal(o["ds/dx"].data, [2.0, 1.0, 0.0])


def test_reverse_gather_with_weights_gives_reversed_weights():
    n = 4
    x, w = p("x", [n]), p("w", [n])
    rev = D.map(lambda i: D.sub(D.const(I32, n - 1), i), D.iota((n,)))
    g = Graph("g", one("s", D.reduce(D.add, ZERO, D.map2(D.mul, w, D.gather(rev, x)))))
    o = grad_vs_fd(g, "s", ["x"], [("x", f64([n], XS4)), ("w", f64([n], YS4))])
    assert np.allclose(o["ds/dx"].data, YS4[::-1], rtol=0, atol=1e-9)


def test_original_outputs_preserved_names_and_count():
    x, y = p("x", [4]), p("y", [4])
    r = D.map2(D.mul, x, y)
    g = Graph("g", [("r", r), ("s", D.reduce(D.add, ZERO, r))])
    ins = [("x", f64([4], XS4)), ("y", f64([4], YS4))]
    o = I.run(I.compile(g), ins)
    og = I.run(I.compile(G.grad(g, "s", ["x", "y"])), ins)
    assert [nm for nm, _ in og] == ["r", "s", G.grad_name("s", "x"), G.grad_name("s", "y")]
    assert np.array_equal(dict(og)["r"].data, dict(o)["r"].data)
    assert np.array_equal(dict(og)["s"].data, dict(o)["s"].data)
    assert G.grad_name("s", "x") == "ds/dx"


def test_unknown_names_raise():
    x = p("x", [4])
    g = Graph("g", one("s", D.reduce(D.add, ZERO, x)))
    with pytest.raises(ValueError):
        G.grad(g, "nope", ["x"])
    with pytest.raises(ValueError):
        G.grad(g, "s", ["nope"])


def test_matmul_and_mlp_gradients_by_bump_and_revalue():
    # the benchmark's MLP step at a few elements: loss and dW1, dW2 from
    # Grad against central differences of the loss graph
    from cudacaml_b200 import examples as X
    bsz, din, hid, dout = 3, 2, 4, 2
    rng = np.random.default_rng(2)
    shapes = {"X": (bsz, din), "W1": (din, hid), "W2": (hid, dout), "T": (bsz, dout)}
    ins = [(nm, Value.of_array(F64, shapes[nm], rng.standard_normal(shapes[nm]) * 0.5)) for nm in ("X", "W1", "W2", "T")]
    g = X.mlp_loss(bsz, din, hid, dout, F64)
    grad_vs_fd(g, "loss", ["W1", "W2"], ins)
