"""The oracle's evaluation rules pinned by the reference interpreter's own
known answers (test/unit/test_interp.ml, test_expr_ops.ml, test_matmul.ml,
test_rows.ml, test_scatter.ml and test_black_scholes.ml, line cited per case):
element maps, index and iota, the sequential left fold from init, empty
reductions, inclusive scans, gathers and their bounds, comparisons and logic
through select, F32 rounding, truncating I32 division, erfinv at the edges,
the input checks, products and their gradients, the DSL's rank and shape
checks, and the multi-step Black-Scholes band. CPU only.
"""
import math

import numpy as np
import pytest

from cudacaml_b200 import dsl as D
from cudacaml_b200 import examples as X
from cudacaml_b200.ir import F32, F64, I32, Graph, Value
from oracle import interp as I


def run(g, inputs=()):
    return I.run(I.compile(g), list(inputs))


def out(g, inputs=(), name="r"):
    return dict(run(g, inputs))[name].to_list()


def f32(xs):
    return Value.of_list(F32, (len(xs),), xs)


def i32(xs):
    return Value.of_list(I32, (len(xs),), xs)


def k(v):
    return D.const(F32, v)


def test_map_and_chain():  # test_interp.ml:29-38
    x, y = D.param("x", F32, (3,)), D.param("y", F32, (3,))
    assert out(Graph("g", [("r", D.map(lambda e: D.mul(e, e), x))]), [("x", f32([1, 2, 3]))]) == [1, 4, 9]
    r = D.map2(D.add, D.map(lambda e: D.mul(k(2.0), e), x), y)
    assert out(Graph("g", [("r", r)]), [("x", f32([1, 2, 3])), ("y", f32([10, 20, 30]))]) == [12, 24, 36]


def test_iota_cast_and_index():  # test_interp.ml:39-47
    assert out(Graph("g", [("r", D.map(lambda i: D.cast(F32, i), D.iota((4,))))])) == [0, 1, 2, 3]
    x = D.param("x", F32, (3,))
    r = D.map(lambda e: D.add(e, D.cast(F32, D.index())), x)
    assert out(Graph("g", [("r", r)]), [("x", f32([10, 10, 10]))]) == [10, 11, 12]


def test_reduce_fold_max_and_empty():  # test_interp.ml:48-59
    x = D.param("x", F32, (4,))
    assert out(Graph("g", [("s", D.reduce(D.add, k(100.0), x))]), [("x", f32([1, 2, 3, 4]))], "s") == [110]
    x3 = D.param("x", F32, (3,))
    assert out(Graph("g", [("m", D.reduce(D.max, k(-1e30), x3))]), [("x", f32([-3, 7, 2]))], "m") == [7]
    x0 = D.param("x", F32, (0,))
    assert out(Graph("g", [("s", D.reduce(D.add, k(5.0), x0))]), [("x", f32([]))], "s") == [5]


def test_scan_inclusive():  # test_interp.ml:60-63
    x = D.param("x", F32, (4,))
    assert out(Graph("g", [("p", D.scan(D.add, k(0.0), x))]), [("x", f32([1, 2, 3, 4]))], "p") == [1, 3, 6, 10]


def test_gather_and_out_of_bounds():  # test_interp.ml:64-72
    x, i = D.param("x", F32, (3,)), D.param("i", I32, (4,))
    g = Graph("g", [("r", D.gather(i, x))])
    assert out(g, [("x", f32([10, 20, 30])), ("i", i32([2, 0, 2, 1]))]) == [30, 10, 30, 20]
    i1 = D.param("i", I32, (1,))
    with pytest.raises(I.InterpError):
        run(Graph("g", [("r", D.gather(i1, x))]), [("x", f32([1, 2, 3])), ("i", i32([3]))])
    with pytest.raises(I.InterpError):
        run(Graph("g", [("r", D.gather(i1, x))]), [("x", f32([1, 2, 3])), ("i", i32([-1]))])


def test_reshape_keeps_data():  # test_interp.ml:73-78
    x = D.param("x", F32, (2, 2))
    o = dict(run(Graph("g", [("r", D.reshape((4,), x))]), [("x", Value.of_list(F32, (2, 2), [1, 2, 3, 4]))]))["r"]
    assert o.to_list() == [1, 2, 3, 4] and o.shape == (4,)


def test_select_comparisons_and_logic():  # test_interp.ml:79-84, test_expr_ops.ml:99-118
    x = D.param("x", F32, (4,))
    r = D.map(lambda e: D.select(D.lt(e, k(0.0)), k(0.0), e), x)
    assert out(Graph("g", [("r", r)]), [("x", f32([-1, 2, -3, 4]))]) == [0, 2, 0, 4]
    x, y = D.param("x", F32, (3,)), D.param("y", F32, (3,))

    def b(c):
        return D.select(c, k(1.0), k(0.0))

    outs = [("ne", D.map2(lambda a, c: b(D.ne(a, c)), x, y)),
            ("gt", D.map2(lambda a, c: b(D.gt(a, c)), x, y)),
            ("ge", D.map2(lambda a, c: b(D.ge(a, c)), x, y)),
            ("and", D.map(lambda a: b(D.and_(D.gt(a, k(1.0)), D.lt(a, k(3.0)))), x)),
            ("or", D.map(lambda a: b(D.or_(D.lt(a, k(2.0)), D.gt(a, k(2.0)))), x)),
            ("not", D.map2(lambda a, c: b(D.not_(D.eq(a, c))), x, y))]
    o = dict(run(Graph("g", outs), [("x", f32([1, 2, 3])), ("y", f32([2, 2, 2]))]))
    want = {"ne": [1, 0, 1], "gt": [0, 0, 1], "ge": [0, 1, 1], "and": [0, 1, 0], "or": [1, 0, 1], "not": [1, 0, 1]}
    for name, w in want.items():
        assert o[name].to_list() == w, name


def test_i32_division_truncates_and_f32_rounds():  # test_interp.ml:85-95
    x = D.param("x", I32, (2,))
    assert out(Graph("g", [("r", D.map(lambda e: D.div(e, D.const(I32, 2)), x))]), [("x", i32([-7, 7]))]) == [-3, 3]
    x = D.param("x", F32, (1,))
    v = out(Graph("g", [("r", D.map(lambda e: D.add(e, k(0.2)), x))]), [("x", f32([0.1]))])[0]
    assert abs(v - 0.300000011920929) <= 1e-9


def test_shared_intermediate_and_output_order():  # test_interp.ml:96-104
    x = D.param("x", F32, (2,))
    s = D.map(lambda e: D.mul(e, e), x)
    o = run(Graph("g", [("a", D.map(D.neg, s)), ("c", D.reduce(D.add, k(0.0), s))]), [("x", f32([3, 4]))])
    assert [n for n, _ in o] == ["a", "c"]
    assert dict(o)["a"].to_list() == [-9, -16] and dict(o)["c"].to_list() == [25]


def test_input_checks():  # test_interp.ml:105-116
    g1 = Graph("g", [("r", D.map(D.neg, D.param("x", F32, (1,))))])
    with pytest.raises(I.InterpError):
        run(g1, [])
    with pytest.raises(I.InterpError):
        run(g1, [("x", i32([1]))])
    g2 = Graph("g", [("r", D.map(D.neg, D.param("x", F32, (2,))))])
    with pytest.raises(I.InterpError):
        run(g2, [("x", f32([1.0]))])


def test_every_registered_example_runs():  # test_interp.ml:117-120
    for p in X.PROGRAMS:
        run(p.graph(), p.inputs())


def _unop_f64(f, xs):
    x = D.param("x", F64, (len(xs),))
    return out(Graph("g", [("r", D.map(f, x))]), [("x", Value.of_list(F64, (len(xs),), xs))])


def test_sin_cos_erf_f64():  # test_expr_ops.ml:80-84
    assert np.allclose(_unop_f64(D.sin, [0.0, math.pi / 2]), [0, 1], rtol=0, atol=1e-12)
    assert np.allclose(_unop_f64(D.cos, [0.0, math.pi / 2]), [1, 0], rtol=0, atol=1e-12)
    assert np.allclose(_unop_f64(D.erf, [0.0, 1.0]), [0, 0.8427007929497149], rtol=0, atol=1e-15)


def test_erfinv_inverts_erf_and_edges():  # test_expr_ops.ml:85-98
    xs = [-2.0, -0.5, 0.0, 0.3, 1.5, 2.5]
    assert np.allclose(_unop_f64(lambda e: D.erfinv(D.erf(e)), xs), xs, rtol=0, atol=1e-12)
    p, z, m = _unop_f64(D.erfinv, [1.0, 0.0, -1.0])
    assert p == math.inf and z == 0.0 and m == -math.inf
    x = D.param("x", F32, (1,))
    v = out(Graph("g", [("r", D.map(D.erfinv, x))]), [("x", f32([0.5]))])[0]
    assert abs(v - 0.4769362762) <= 1e-6


def test_matmul_identity_and_5x7_7x3():  # test_matmul.ml:95-100
    a = [1.0, 2, 3, 4, 5, 6, 7, 8, 9]
    A, B = D.param("a", F64, (3, 3)), D.param("b", F64, (3, 3))
    ident = list(np.eye(3).reshape(-1))
    g = Graph("mm", [("c", D.matmul(A, B))])
    assert out(g, [("a", Value.of_list(F64, (3, 3), a)), ("b", Value.of_list(F64, (3, 3), ident))], "c") == a
    av = [float((i * 7) % 11) - 5.0 for i in range(35)]
    bv = [float((i * 5) % 13) / 4.0 for i in range(21)]
    A, B = D.param("a", F64, (5, 7)), D.param("b", F64, (7, 3))
    got = out(Graph("mm", [("c", D.matmul(A, B))]),
              [("a", Value.of_list(F64, (5, 7), av)), ("b", Value.of_list(F64, (7, 3), bv))], "c")
    want = (np.array(av).reshape(5, 7) @ np.array(bv).reshape(7, 3)).reshape(-1)
    assert np.allclose(got, want, rtol=0, atol=1e-12)


def test_matmul_shape_checks():  # test_matmul.ml:101-104
    with pytest.raises(ValueError):
        D.matmul(D.param("a", F64, (2, 3)), D.param("b", F64, (2, 3)))
    with pytest.raises(ValueError):
        D.matmul(D.param("a", F64, (6,)), D.param("b", F64, (6,)))
    with pytest.raises(ValueError):
        D.matmul(D.param("a", F64, (2, 2, 2)), D.param("b", F64, (2, 2)))


def test_matmul_gradients_by_central_difference():  # test_matmul.ml:140-145
    from cudacaml_b200 import grad as G
    ins = [("a", Value.of_list(F64, (2, 3), [1.0, -2.0, 0.5, 3.0, 1.5, -1.0])),
           ("b", Value.of_list(F64, (3, 2), [0.3, 1.5, -1.0, 2.0, 0.7, -0.2]))]
    zero = D.const(F64, 0.0)
    for wrap in (lambda a: a, lambda a: D.map(D.exp, a)):
        a, b = D.param("a", F64, (2, 3)), D.param("b", F64, (3, 2))
        g = Graph("g", [("s", D.reduce(D.add, zero, D.matmul(wrap(a), b)))])
        o = dict(run(G.grad(g, "s", ["a", "b"]), ins))
        for w in ("a", "b"):
            base = dict(ins)[w]
            h = 1e-6
            for i in range(base.numel):
                def s_at(delta):
                    v = base.data.copy()
                    v[i] += delta
                    bumped = [(n, Value.of_array(F64, base.shape, v) if n == w else x) for n, x in ins]
                    return dict(run(g, bumped))["s"].get(0)
                e = (s_at(h) - s_at(-h)) / (2 * h)
                assert abs(e - o[G.grad_name("s", w)].get(i)) <= 1e-5 * (1 + abs(e)), (w, i)


def test_rows_rank_checks_and_scatter_shapes():  # test_rows.ml:81-87, test_scatter.ml:47-49
    zero = D.const(F32, 0.0)
    v = D.param("v", F32, (5,))
    r3 = D.param("w", F32, (2, 2, 2))
    for bad in (lambda: D.reduce_rows(D.add, zero, v), lambda: D.scan_rows(D.add, zero, v),
                lambda: D.transpose(v), lambda: D.transpose(r3)):
        with pytest.raises(ValueError):
            bad()
    with pytest.raises(ValueError):
        D.scatter_add(D.param("idx", I32, (6,)), D.param("src", F32, (5,)), (4,))


def test_bs_paths_band_and_greeks_graph_structure():  # test_black_scholes.ml:24-43
    from cudacaml_b200 import backend_cuda as B
    cf = X.analytic()
    o = dict(run(X.call_mc_paths(16384, 8, F64), X.bs_inputs(F64, seed=42)))
    assert abs(o["price"].get(0) - cf["price"]) <= 0.5
    g = X.call_greeks(4096, F64)
    assert sorted(n for n, _ in g.params) == ["rate", "s0", "seed", "vol"]
    assert len(g.outputs) == 4
    assert B.lower_info(g)["kernels"] < 40  # the reference's bound; this backend makes one
    for name in ("bs_mc", "bs_paths", "bs_greeks"):
        assert X.find(name) is not None
