"""The oracle (a C++ restatement of the reference interpreter) pinned against
the known answers of the reference's own unit tests (tests/golden/
reference_kats.json, each entry citing its source file:line). CPU only."""
import json
import math
import os

import numpy as np
import pytest

from cudacaml_b200 import dsl as D
from cudacaml_b200 import examples as X
from cudacaml_b200 import rng as Rng
from cudacaml_b200.ir import F32, F64, I32, I64, Graph, Value
from oracle import interp as I

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))


def h(s):
    v = int(s, 16) if isinstance(s, str) else int(s)
    return v


def run(g, inputs):
    return dict(I.run(I.compile(g), inputs))


def seed(k):
    return ("seed", Value.of_list(I32, (), [k]))


@pytest.mark.parametrize("kat", GOLD["philox4x32_10"])
def test_philox_kat_raw(kat):
    got = I.philox4x32_10([h(x) for x in kat["ctr"]], [h(x) for x in kat["key"]])
    assert got == [h(x) for x in kat["out"]]


@pytest.mark.parametrize("kat", GOLD["philox4x32_10"])
def test_philox_kat_through_graph(kat):
    # Rng.Philox.round10 as DSL expressions, evaluated by the oracle.
    def wrap(v):
        return (v + 2**31) % 2**32 - 2**31

    ctr = [D.const(I32, wrap(h(x))) for x in kat["ctr"]]
    key = [D.const(I32, wrap(h(x))) for x in kat["key"]]
    words = Rng.round10(tuple(ctr), tuple(key))
    outs = []
    for k, w in enumerate(words):
        t = D.map(lambda _, w=w: w, D.iota((1,)))
        outs.append((f"w{k}", t))
    o = run(Graph("kat", outs), [])
    assert [o[f"w{k}"].get(0) & 0xFFFFFFFF for k in range(4)] == [h(x) for x in kat["out"]]


def test_u32_element0_and_distinct():
    o = run(Graph("u", [("r", Rng.u32(D.scalar("seed", I32), (4,)))]), [seed(0)])
    l = [x & 0xFFFFFFFF for x in o["r"].to_list()]
    assert l[0] == h(GOLD["u32_key0_elem0"]["value"])
    assert len(set(l)) == 4


def test_reproducible_and_keys_differ():
    def u(k):
        return run(Graph("u", [("r", Rng.u32(D.scalar("seed", I32), (1024,)))]), [seed(k)])["r"].data

    a, b, c = u(42), u(42), u(43)
    assert np.array_equal(a, b)
    assert int(np.sum(a != c)) >= GOLD["keys_differ"]["min_differ"]


def test_counter_is_flat_index():
    a = run(Graph("a", [("r", Rng.u32(D.scalar("seed", I32), (4, 8)))]), [seed(9)])["r"].data
    b = run(Graph("b", [("r", Rng.u32(D.scalar("seed", I32), (32,)))]), [seed(9)])["r"].data
    assert np.array_equal(a, b)


def test_uniform_f64_moments_chi2():
    gd = GOLD["uniform_f64"]
    u = run(Graph("u", [("r", Rng.uniform(F64, D.scalar("seed", I32), (gd["n"],)))]), [seed(gd["key"])])["r"].data
    assert np.all((u > 0) & (u < 1))
    assert abs(u.mean() - gd["mean"]) <= gd["mean_tol"]
    assert abs(u.var() - gd["var"]) <= gd["var_tol"]
    counts = np.bincount((u * 16).astype(int), minlength=16)
    e = gd["n"] / 16
    assert float(((counts - e) ** 2 / e).sum()) < gd["chi2_max"]
    # the numpy restatement used for host inputs agrees bit for bit
    assert np.array_equal(u, X.philox_uniform(gd["key"], gd["n"]))


def test_normal_f64_moments_tail():
    gd = GOLD["normal_f64"]
    z = run(Graph("n", [("r", Rng.normal(F64, D.scalar("seed", I32), (gd["n"],)))]), [seed(gd["key"])])["r"].data
    assert np.all(np.isfinite(z))
    assert abs(z.mean()) <= gd["mean_tol"]
    assert abs(z.var() - 1.0) <= gd["var_tol"]
    assert abs(np.mean(np.abs(z) > 1.96) - gd["tail"]) <= gd["tail_tol"]


def _unop(dt, f, xs):
    x = D.param("x", dt, (len(xs),))
    return run(Graph("g", [("r", D.map(f, x))]), [("x", Value.of_list(dt, (len(xs),), xs))])["r"].data


def test_erf_and_erfinv():
    gd = GOLD["erf_f64"]
    assert np.allclose(_unop(F64, D.erf, gd["x"]), gd["y"], atol=gd["tol"], rtol=0)
    gi = GOLD["erfinv_erf_identity"]
    assert np.allclose(_unop(F64, lambda e: D.erfinv(D.erf(e)), gi["x"]), gi["x"], atol=gi["tol"], rtol=0)
    p, z, m = _unop(F64, D.erfinv, [1.0, 0.0, -1.0])
    assert p == math.inf and z == 0.0 and m == -math.inf
    gh = GOLD["erfinvf_half"]
    assert abs(_unop(F32, D.erfinv, [gh["x"]])[0] - gh["y"]) <= gh["tol"]


@pytest.mark.parametrize("case", GOLD["i32_bitops"])
def test_i32_bitops(case):
    def v(s):
        x = h(s) if isinstance(s, str) else int(s)
        return (x + 2**31) % 2**32 - 2**31

    a = D.param("a", I32, (1,))
    b = D.param("b", I32, (1,))
    op = getattr(D, case["op"])
    r = run(Graph("g", [("r", D.map2(op, a, b))]),
            [("a", Value.of_list(I32, (1,), [v(case["a"])])), ("b", Value.of_list(I32, (1,), [v(case["b"])]))])["r"]
    assert r.get(0) == v(case["r"])


@pytest.mark.parametrize("case", GOLD["i64_shifts"])
def test_i64_shifts(case):
    a = D.param("a", I64, (1,))
    b = D.param("b", I64, (1,))
    r = run(Graph("g", [("r", D.map2(getattr(D, case["op"]), a, b))]),
            [("a", Value.of_list(I64, (1,), [case["a"]])), ("b", Value.of_list(I64, (1,), [case["b"]]))])["r"]
    assert r.get(0) == case["r"]


def test_bitops_on_floats_rejected():
    x = D.param("x", F32, (1,))
    with pytest.raises(I.InterpError):
        run(Graph("g", [("r", D.map2(D.bit_and, x, x))]), [("x", Value.of_list(F32, (1,), [1.0]))])


def test_f32_rounding_and_i32_division():
    gd = GOLD["f32_rounding"]
    x = D.param("x", F32, (1,))
    r = run(Graph("g", [("r", D.map(lambda e: D.add(e, D.const(F32, gd["c"])), x))]),
            [("x", Value.of_list(F32, (1,), [gd["x"]]))])["r"].get(0)
    assert abs(r - gd["r"]) <= gd["tol"]
    gi = GOLD["i32_division"]
    xi = D.param("x", I32, (2,))
    r = run(Graph("g", [("r", D.map(lambda e: D.div(e, D.const(I32, gi["d"])), xi))]),
            [("x", Value.of_list(I32, (2,), gi["x"]))])["r"].to_list()
    assert r == gi["r"]


def test_division_by_zero_raises():
    xi = D.param("x", I32, (1,))
    with pytest.raises(I.InterpDivisionByZero):
        run(Graph("g", [("r", D.map(lambda e: D.div(e, D.const(I32, 0)), xi))]), [("x", Value.of_list(I32, (1,), [3]))])


def test_rows_2x3():
    gd = GOLD["rows_2x3"]
    zero = D.const(F32, 0.0)
    x = D.param("x", F32, (2, 3))
    inp = [("x", Value.of_list(F32, (2, 3), gd["x"]))]
    o = run(Graph("g", [("r", D.reduce_rows(D.add, zero, x)), ("s", D.reduce(D.add, zero, x)),
                        ("rows", D.scan_rows(D.add, zero, x)), ("flat", D.scan(D.add, zero, x)),
                        ("m", D.reduce_rows(D.max, D.const(F32, -1e30), x)), ("t", D.transpose(x)),
                        ("cols", D.reduce_rows(D.add, zero, D.transpose(x)))]), inp)
    assert o["r"].to_list() == gd["reduce_rows_add"] and o["r"].shape == (2,)
    assert o["s"].to_list() == [gd["reduce_all"]] and o["s"].shape == ()
    assert o["rows"].to_list() == gd["scan_rows"] and o["rows"].shape == (2, 3)
    assert o["flat"].to_list() == gd["scan_flat"] and o["flat"].shape == (2, 3)
    assert o["m"].to_list() == gd["reduce_rows_max"]
    assert o["t"].to_list() == gd["transpose"] and o["t"].shape == (3, 2)
    assert o["cols"].to_list() == gd["col_sums"]


def test_scatter_histograms():
    gd = GOLD["scatter"]
    idx = D.param("idx", I32, (6,))
    sf = D.param("src", F32, (6,))
    o = run(Graph("h", [("h", D.scatter_add(idx, sf, (4,)))]),
            [("idx", Value.of_list(I32, (6,), gd["idx"])), ("src", Value.of_list(F32, (6,), [1.0] * 6))])
    assert o["h"].to_list() == gd["f32_hist"]
    si = D.param("src", I32, (6,))
    o = run(Graph("h", [("h", D.scatter_add(idx, si, (4,)))]),
            [("idx", Value.of_list(I32, (6,), gd["idx"])), ("src", Value.of_list(I32, (6,), gd["i32_src"]))])
    assert o["h"].to_list() == gd["i32_hist"]
    with pytest.raises(I.InterpError):
        i1 = D.param("idx", I32, (1,))
        s1 = D.param("src", F32, (1,))
        run(Graph("h", [("h", D.scatter_add(i1, s1, (4,)))]),
            [("idx", Value.of_list(I32, (1,), [4])), ("src", Value.of_list(F32, (1,), [1.0]))])


def test_matmul_2x3_3x2():
    gd = GOLD["matmul_2x3_3x2"]
    a = D.param("a", F64, (2, 3))
    b = D.param("b", F64, (3, 2))
    o = run(Graph("mm", [("c", D.matmul(a, b))]),
            [("a", Value.of_list(F64, (2, 3), gd["a"])), ("b", Value.of_list(F64, (3, 2), gd["b"]))])
    assert o["c"].to_list() == gd["c"] and o["c"].shape == (2, 2)


def test_bs_closed_form():
    gd = GOLD["bs_closed_form"]
    cf = X.analytic()
    for k in ("price", "delta", "vega", "rho"):
        assert abs(cf[k] - gd[k]) <= gd["tol"]


def test_bs_mc_65536_within_band_and_greeks_price_identical():
    cf = X.analytic()
    o = run(X.call_mc(65536, F64), X.bs_inputs(F64, seed=7))
    assert abs(o["price"].get(0) - cf["price"]) <= GOLD["bs_mc_65536_band"]["tol"]
    og = run(X.call_greeks(65536, F64), X.bs_inputs(F64, seed=7))
    assert og["price"].get(0) == o["price"].get(0)
    assert abs(og["dprice/ds0"].get(0) - cf["delta"]) < 0.02
    assert abs(og["dprice/dvol"].get(0) - cf["vega"]) < 1.5
    assert abs(og["dprice/drate"].get(0) - cf["rho"]) < 1.5


def test_programs_registry_runs():
    for p in X.PROGRAMS:
        o = run(p.graph(), p.inputs())
        assert o, p.name


def test_lsm_solve_graph_matches_host_solve():
    # the resident driver's graph solve against the host solve it restates,
    # on the oracle: regular, pivoting, too few paths, singular
    from cudacaml_b200 import lsm as L
    from cudacaml_b200.ir import F64, Value
    g = L.solve_graph(4)
    rng = np.random.default_rng(1)
    for case in range(5):
        x = rng.standard_normal((100, 4)) * (1, 30, 900, 27000)
        y = rng.standard_normal(100)
        xtx, xty = x.T @ x, x.T @ y
        if case == 1:
            xtx[[0, 1]] = xtx[[1, 0]]
        if case == 2:
            xtx[0, 0] = 2.0
        if case == 3:
            xtx = np.zeros((4, 4))
            xtx[0, 0] = 50.0
        want = L._beta(list(xtx.ravel()), list(xty), 4)
        out = dict(I.run(I.compile(g), [("xtx", Value.of_array(F64, (16,), xtx.ravel())),
                                                  ("xty", Value.of_array(F64, (4,), xty))]))
        assert [float(out[f"b{i}"].data[0]) for i in range(4)] == want


def test_lsm_update_regress_graph_is_update_then_regress():
    # the resident driver's fused pass (update date t, normal equations of
    # date t-1 on the updated cash flow) against the two graphs run in turn,
    # on the oracle, bit for bit, both bases
    from cudacaml_b200 import lsm as L
    from cudacaml_b200.ir import F64, I32, Value
    n, ns, t = 512, 8, 5
    rng = np.random.default_rng(4)
    for basis, m in (("poly4", L.BASELINE_MARKET), ("scaled3", L.MARKET)):
        nb = L._nb(basis)
        disc = 0.99
        st = m.strike * np.exp(0.2 * rng.standard_normal((ns, n)))
        cf = np.maximum(m.strike - st[-1], 0.0)
        beta = rng.standard_normal((nb, 1))
        common = [("S", Value.of_array(F64, (ns, n), st)), ("cf", Value.of_array(F64, (n,), cf)),
                  ("beta", Value.of_array(F64, (nb, 1), beta))]
        fused = dict(I.run(I.compile(L.update_regress_graph(n, ns, m.strike, disc, basis)),
                           common + [("t", Value.of_list(I32, (), [t]))]))
        upd = dict(I.run(I.compile(L.update_graph(n, ns, m.strike, disc, basis, "dates")),
                         common + [("t", Value.of_list(I32, (), [t]))]))
        reg = dict(I.run(I.compile(L.regress_graph(n, ns, m.strike, disc, basis, "dates")),
                         [common[0], ("cf", upd["cf"]), ("t", Value.of_list(I32, (), [t - 1]))]))
        assert np.array_equal(fused["cf"].data, upd["cf"].data)
        assert np.array_equal(fused["xtx"].data, reg["xtx"].data)
        assert np.array_equal(fused["xty"].data, reg["xty"].data)


def test_lsm_update_regress_solve_graph_is_the_three_in_turn():
    # one launch per date on the device: update, next normal equations and
    # their solve; on the oracle, bit for bit against the graphs in turn
    from cudacaml_b200 import lsm as L
    from cudacaml_b200.ir import F64, I32, Value
    n, ns, t = 512, 8, 5
    rng = np.random.default_rng(6)
    for basis, m in (("poly4", L.BASELINE_MARKET), ("scaled3", L.MARKET)):
        nb = L._nb(basis)
        st = m.strike * np.exp(0.2 * rng.standard_normal((ns, n)))
        cf = np.maximum(m.strike - st[-1], 0.0)
        beta = rng.standard_normal((nb, 1))
        tv = lambda k: ("t", Value.of_list(I32, (), [k]))  # noqa: E731
        common = [("S", Value.of_array(F64, (ns, n), st)), ("cf", Value.of_array(F64, (n,), cf)),
                  ("beta", Value.of_array(F64, (nb, 1), beta))]
        fused = dict(I.run(I.compile(L.update_regress_solve_graph(n, ns, m.strike, 0.99, basis)), common + [tv(t)]))
        ur = dict(I.run(I.compile(L.update_regress_graph(n, ns, m.strike, 0.99, basis)), common + [tv(t)]))
        sol = dict(I.run(I.compile(L.solve_graph(nb)), [("xtx", Value.of_array(F64, (nb * nb,), ur["xtx"].data)),
                                                         ("xty", Value.of_array(F64, (nb,), ur["xty"].data))]))
        for k in ("cf", "xtx", "xty"):
            assert np.array_equal(fused[k].data, ur[k].data), k
        for i in range(nb):
            assert np.array_equal(fused[f"b{i}"].data, sol[f"b{i}"].data), i
        first = dict(I.run(I.compile(L.regress_solve_graph(n, ns, m.strike, 0.99, basis)), common[:2] + [tv(t)]))
        reg = dict(I.run(I.compile(L.regress_graph(n, ns, m.strike, 0.99, basis, "dates")), common[:2] + [tv(t)]))
        assert np.array_equal(first["xtx"].data, reg["xtx"].data)


def test_lsm_paths_dates_graph_is_the_transpose():
    # the date-major paths program gives paths_graph's S transposed, bit for bit
    from cudacaml_b200 import lsm as L
    from cudacaml_b200.ir import I32, Value
    n, ns = 300, 12
    seed = [("seed", Value.of_list(I32, (), [7]))]
    s = dict(I.run(I.compile(L.paths_graph(n, ns, L.BASELINE_MARKET)), seed))["S"].data.reshape(n, ns)
    st = dict(I.run(I.compile(L.paths_dates_graph(n, ns, L.BASELINE_MARKET)), seed))["ST"].data.reshape(ns, n)
    assert np.array_equal(st, s.T)


def test_lsm_known_answers_on_the_oracle():
    # test_lsm.ml's known answers for the reference market (binomial 6.09,
    # European put 5.5735) and the S17 band: the generic LSM driver over the
    # oracle, 2^14 paths x 50 dates, within 0.15 of the binomial price
    from cudacaml_b200 import lsm as L
    binom = L.binomial_american_put(L.MARKET)
    assert abs(binom - 6.09) < 0.005
    assert abs(L.european_put(L.MARKET) - 5.5735) < 1e-3
    px = L.Make(I, 1 << 14, 50, L.MARKET, "scaled3").price(11)
    assert abs(px - binom) <= 0.15 and px >= L.european_put(L.MARKET) - 0.05
