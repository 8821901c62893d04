"""The restated reference NVRTC backend (baseline/ref_nvrtc.py) on the GPU,
against the oracle: the baseline bench.py times must compute what the
reference computes. Integer results bit-exact; floating point within the
reference's own bands (Differential's 1e-5, S13's 1e-6 for the F64 Greeks).
FMA contraction is on in NVRTC by default, as it is for the reference, so
F32 element results are compared within a band, not bit for bit."""
import numpy as np
import pytest

from baseline import ref_nvrtc as RN
from cudacaml_b200 import examples as X
from cudacaml_b200 import runtime as R
from cudacaml_b200.ir import F32, F64, I32, Value
from oracle import interp

pytestmark = pytest.mark.gpu


def _run(g, inputs):
    R.set_device(0)
    L = RN.Loaded(RN.Program(g))
    try:
        for name, v in inputs:
            L.upload(name, v.data)
        L.launch(0)
        R.check(R.lib().ccb_device_synchronize())
        return {n: L.download(n, t.dtype.np, t.numel) for n, t in g.outputs}
    finally:
        L.release()


def _oracle(g, inputs):
    return {n: v.data for n, v in interp.run(interp.compile(g), inputs)}


def _band(got, want, tol):
    got, want = got.astype(np.float64), want.astype(np.float64)
    assert np.all(np.abs(got - want) <= tol * (1 + np.abs(want))), np.max(np.abs(got - want))


def test_saxpy_sum_two_pass_reduce():
    # positive terms, so the F32 sum does not cancel and a relative band is
    # meaningful for both summation orders (tree here, sequential in the oracle)
    n = 300_007
    x = Value.of_array(F32, (n,), np.linspace(0, 1, n, dtype=np.float32))
    y = Value.of_array(F32, (n,), (1.0 + np.cos(np.arange(n))).astype(np.float32))
    g = X.saxpy(n, 2.0)
    got, want = _run(g, [("x", x), ("y", y)]), _oracle(g, [("x", x), ("y", y)])
    _band(got["r"], want["r"], 1e-6)
    _band(got["s"], want["s"], 1e-3)


def test_i32_scan_three_passes_exact():
    n = (1 << 20) + 77
    g = X.reduce_scan_flat(n, I32)
    x = Value.of_array(I32, (n,), (np.arange(n) % 16).astype(np.int32))
    got, want = _run(g, [("x", x)]), _oracle(g, [("x", x)])
    assert np.array_equal(got["s"], want["s"]) and np.array_equal(got["p"], want["p"])


def test_greeks_f64_25_kernels_vs_oracle():
    g = X.call_greeks(65536, F64)
    got, want = _run(g, X.bs_inputs(F64, seed=42)), _oracle(g, X.bs_inputs(F64, seed=42))
    for k in want:
        _band(got[k], want[k], 1e-6)


def test_scatter_and_product():
    g = X.scatter(100_000, 1000)
    idx = Value.of_array(I32, (100_000,), (np.arange(100_000) * 7919 % 1000).astype(np.int32))
    vals = Value.of_array(F32, (100_000,), np.ones(100_000, np.float32))
    ins = [("idx", idx), ("v", vals)]
    got, want = _run(g, ins), _oracle(g, ins)
    assert np.array_equal(got["h"], want["h"])  # counts of ones: exact in F32
    from cudacaml_b200 import dsl as D
    from cudacaml_b200.ir import Graph
    a, b = D.param("a", F32, (70, 45)), D.param("b", F32, (45, 33))
    g = Graph("mm", [("c", D.matmul(a, b))])
    rng = np.random.default_rng(3)
    ins = [("a", Value.of_array(F32, (70, 45), rng.standard_normal((70, 45)).astype(np.float32))),
           ("b", Value.of_array(F32, (45, 33), rng.standard_normal((45, 33)).astype(np.float32)))]
    got, want = _run(g, ins), _oracle(g, ins)
    _band(got["c"], want["c"], 1e-4)  # S11's F32 band
