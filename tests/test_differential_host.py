"""Differential.check (lib/backend/differential.ml) on the CPU: the oracle on
both sides, and candidates with a mistake planted in the oracle's results.
The GPU parity tests judge every kernel with this function. CPU only.
"""
import numpy as np

from cudacaml_b200 import differential as Diff
from cudacaml_b200 import dsl as D
from cudacaml_b200.ir import F32, F64, I32, Graph, Value
from oracle import interp as I


class Planted:
    """The oracle with one output changed after the run."""

    def __init__(self, name, change):
        self.name = name
        self.change = change

    def compile(self, g):
        return I.compile(g)

    def run(self, c, inputs):
        return [self.change(n, v) for n, v in I.run(c, inputs)]


class Raising:
    name = "broken"

    def compile(self, g):
        raise RuntimeError("no device")

    def run(self, c, inputs):
        raise AssertionError("not reached")


def saxpy_graph(dt=F32, n=5):
    x, y = D.param("x", dt, (n,)), D.param("y", dt, (n,))
    r = D.map2(lambda a, b: D.add(D.mul(D.const(dt, 2.0), a), b), x, y)
    return Graph("saxpy", [("r", r), ("s", D.reduce(D.add, D.const(dt, 0.0), r))])


def inputs(dt=F32, n=5):
    return [("x", Value.of_array(dt, (n,), np.arange(n, dtype=dt.np))),
            ("y", Value.of_array(dt, (n,), np.ones(n, dtype=dt.np)))]


def test_identical_backends_agree():
    assert Diff.check(I, I, saxpy_graph(), inputs()) is None


def test_band_is_relative_plus_absolute():
    # |g - e| <= tol * (1 + |e|): at e = 25 a change of 2.5e-4 passes 1e-5, 2.7e-4 does not
    def bump(d):
        def change(n, v):
            return (n, Value.of_array(v.dtype, v.shape, v.data + d)) if n == "s" else (n, v)
        return change
    g, ins = saxpy_graph(F64), inputs(F64)
    assert Diff.check(I, Planted("c", bump(2.5e-4)), g, ins, tolerance=1e-5) is None
    err = Diff.check(I, Planted("c", bump(2.7e-4)), g, ins, tolerance=1e-5)
    assert err == "output s[0]: expected 25, got 25.0003 (tol 1e-05)"


def test_nan_equals_nan_and_integers_are_exact():
    x = D.param("x", F64, (2,))
    g = Graph("g", [("r", D.map(D.log, x))])
    assert Diff.check(I, I, g, [("x", Value.of_list(F64, (2,), [-1.0, 2.0]))]) is None  # log(-1) = NaN both sides
    gi = Graph("g", [("r", D.map(D.neg, D.param("x", I32, (3,))))])
    ins = [("x", Value.of_list(I32, (3,), [1, 2, 3]))]
    off = Planted("c", lambda n, v: (n, Value.of_array(I32, v.shape, v.data + np.int32(1))))
    assert Diff.check(I, off, gi, ins, tolerance=1.0) == "output r[0]: expected -1, got 0 (tol 1)"


def test_dtype_shape_and_missing_outputs():
    g, ins = saxpy_graph(), inputs()
    as_f64 = Planted("c", lambda n, v: (n, Value.of_array(F64, v.shape, v.data.astype(np.float64))))
    assert Diff.check(I, as_f64, g, ins) == "output r: dtype mismatch: expected f32, got f64"
    reshaped = Planted("c", lambda n, v: (n, Value(v.dtype, (1, 5), v.data) if n == "r" else v))
    assert Diff.check(I, reshaped, g, ins) == "output r: shape mismatch: expected [5], got [1,5]"
    renamed = Planted("c", lambda n, v: ("t" if n == "s" else n, v))
    assert Diff.check(I, renamed, g, ins) == "missing output s"
    # by name, not position; extra outputs are not checked
    class Reordered(Planted):
        def run(self, c, inputs):
            return list(reversed(I.run(c, inputs))) + [("extra", Value.of_list(F32, (), [0.0]))]
    assert Diff.check(I, Reordered("c", None), g, ins) is None


def test_a_raising_backend_is_named():
    g, ins = saxpy_graph(), inputs()
    assert Diff.check(I, Raising(), g, ins) == "broken raised: no device"
    assert Diff.check(Raising(), I, g, ins) == "broken raised: no device"
