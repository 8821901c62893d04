"""F32 products on the tcgen05 tensor cores (graphs compiled with
matmul="tf32"), through libccb.so.

The reference computes F32 products with F32 FMAs in ascending k
(lib/lower/lower.ml:806-958; the interpreter's sequential fold,
lib/backend_interp/cudacaml_backend_interp.ml:407-433). The tensor-core path
reads TF32 operands (10 explicit mantissa bits) and accumulates in F32, so
it is held to the componentwise bound stated with the kernel:

    |C - C_exact| <= (2^-9 + K * 2^-23) * sum_k |A[r,k]| |B[k,c]|

with C_exact the F64 product of the same F32 inputs. Shapes cover whole and
partial 128 x 256 output tiles, a partial 32-wide k-step, all four operand
orders (row-major and transposed views), and more tiles than SMs, so the
persistent CTAs reuse both TMEM accumulators.
"""
import re

import numpy as np
import pytest

from cudacaml_b200 import backend_cuda as cuda
from cudacaml_b200 import dsl as D
from cudacaml_b200 import examples as X
from cudacaml_b200.ir import F32, Graph, Value
from oracle import interp

pytestmark = pytest.mark.gpu


def tf32_bound(c, a, b):
    exact = a.astype(np.float64) @ b.astype(np.float64)
    mag = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    lim = (2.0 ** -9 + a.shape[1] * 2.0 ** -23) * mag + 1e-30
    return np.abs(c.astype(np.float64) - exact) / lim


SHAPES = [(128, 64, 256), (300, 200, 260), (2048, 256, 4096), (4096, 64, 4096)]


@pytest.mark.parametrize("m,k,n", SHAPES, ids=lambda v: str(v))
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)],
                         ids=["AB", "AtB", "ABt", "AtBt"])
def test_tf32_product_within_bound(m, k, n, ta, tb):
    rng = np.random.default_rng(m * 7 + k * 13 + n + 2 * ta + tb)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    pa = D.param("a", F32, (k, m) if ta else (m, k))
    pb = D.param("b", F32, (n, k) if tb else (k, n))
    g = Graph("tc", [("c", D.matmul(D.transpose(pa) if ta else pa, D.transpose(pb) if tb else pb))])
    c = cuda.compile(g, matmul="tf32")
    try:
        assert re.search(r"launch ccb_matmultc2?_", c.plan())
        ins = [("a", Value.of_array(F32, pa.shape, np.ascontiguousarray(a.T if ta else a))),
               ("b", Value.of_array(F32, pb.shape, np.ascontiguousarray(b.T if tb else b)))]
        out = dict(cuda.run(c, ins))["c"].data.reshape(m, n)
        ratio = tf32_bound(out, a, b)
        worst = np.unravel_index(int(np.argmax(ratio)), ratio.shape)
        assert ratio.max() <= 1.0, f"error/bound {ratio.max():.3g} at {worst}"
        # the same graph twice in a row gives the same bits (no stale accumulator)
        again = dict(cuda.run(c, ins))["c"].data.reshape(m, n)
        assert np.array_equal(out, again)
    finally:
        cuda.release(c)


def test_tf32_exact_on_small_integers():
    # integers below 2^10 are exact in TF32 and every partial sum is exact in F32
    m, k, n = 256, 96, 512
    a = (np.arange(m * k) % 13 - 6).astype(np.float32).reshape(m, k)
    b = (np.arange(k * n) % 11 - 5).astype(np.float32).reshape(k, n)
    g = Graph("ti", [("c", D.matmul(D.param("a", F32, (m, k)), D.param("b", F32, (k, n))))])
    c = cuda.compile(g, matmul="tf32")
    out = dict(cuda.run(c, [("a", Value.of_array(F32, (m, k), a)), ("b", Value.of_array(F32, (k, n), b))]))["c"]
    assert np.array_equal(out.data.reshape(m, n), (a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32))
    cuda.release(c)


def test_mlp_step_tf32_vs_interp():
    """The benchmark's MLP step at 1/32 of its size against the F32
    interpreter. Gradient entries are sums of 256 signed products, so near-zero
    entries carry the absolute TF32 error of their large terms: the check is
    normwise, max|g - e| <= 1e-2 * max|e| per output (the elementwise bound is
    tested on the products above)."""
    bsz, din, hid, dout = 256, 128, 256, 32
    g = X.mlp_step(bsz, din, hid, dout)
    rng = np.random.default_rng(3)
    scale = {"X": 1.0, "W1": din ** -0.5, "W2": hid ** -0.5, "T": 1.0}
    shapes = {"X": (bsz, din), "W1": (din, hid), "W2": (hid, dout), "T": (bsz, dout)}
    ins = [(nm, Value.of_array(F32, shapes[nm], (rng.standard_normal(shapes[nm]) * scale[nm]).astype(np.float32)))
           for nm in ("X", "W1", "W2", "T")]
    expected = dict(interp.run(interp.compile(g), ins))
    c = cuda.compile(g, matmul="tf32")
    assert len(re.findall(r"launch ccb_matmultc2?_", c.plan())) == 5
    got = dict(cuda.run(c, ins))
    cuda.release(c)
    for name, e in expected.items():
        ev = e.data.astype(np.float64)
        gv = got[name].data.astype(np.float64)
        rel = np.max(np.abs(gv - ev)) / np.max(np.abs(ev))
        assert rel <= 1e-2, f"{name}: normwise error {rel:.3g}"


def test_mlp_multi_allreduce_sum_one_device():
    # Multi with an explicit row split (X and T, not W2 whose first dimension
    # equals the batch) and an NCCL all-reduce of loss and gradients; on one
    # device the sum is the single-device result itself
    from cudacaml_b200 import multi as M
    bsz, din, hid, dout = 256, 128, 256, 256
    rng = np.random.default_rng(5)
    shapes = {"X": (bsz, din), "W1": (din, hid), "W2": (hid, dout), "T": (bsz, dout)}
    ins = [(nm, Value.of_array(F32, shapes[nm], rng.standard_normal(shapes[nm]).astype(np.float32) * 0.1))
           for nm in ("X", "W1", "W2", "T")]
    c = cuda.compile(X.mlp_step(bsz, din, hid, dout), matmul="tf32")
    want = dict(cuda.run(c, ins))
    cuda.release(c)
    t = M.Multi([0], bsz, lambda k: X.mlp_step(k, din, hid, dout), split=["X", "T"], matmul="tf32")
    got = t.allreduce_sum(["loss", "dloss/dW1", "dloss/dW2"], ins)
    t.release()
    for name, v in got.items():
        assert np.array_equal(v.data, want[name].data), name
    with pytest.raises(ValueError):
        M.Multi([0], bsz, lambda k: X.mlp_step(k, din, hid, dout), split=["W1"]).run(ins)


FUSION_SHAPES = [(256, 2048, 512, False), (300, 2048, 260, False), (256, 2048, 258, True)]


@pytest.mark.parametrize("m,k,n,tb", FUSION_SHAPES, ids=lambda v: str(v))
def test_epilogue_fusion_matches_separate_pass(m, k, n, tb):
    """A map pass fused into the product's epilogue gives the bits of the
    same pass run on the stored product: whole 32-column row chunks (vector
    path), a last chunk of 4 columns, and rows of 258 columns (no 16-byte
    alignment: scalar path). The element function has no multiply feeding
    an add, so FMA contraction cannot differ between the two kernels."""
    rng = np.random.default_rng(m + k + n)
    a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
    b = rng.standard_normal((n, k) if tb else (k, n)).astype(np.float32)
    pa, pb = D.param("a", F32, a.shape), D.param("b", F32, b.shape)
    z = D.matmul(pa, D.transpose(pb) if tb else pb)

    def f(v):
        return D.div(D.const(F32, 1.0), D.add(D.const(F32, 1.0), D.exp(v)))

    ins = [("a", Value.of_array(F32, a.shape, a)), ("b", Value.of_array(F32, b.shape, b))]

    def run(graph, inputs):
        c = cuda.compile(graph, matmul="tf32")
        try:
            return c.plan(), {k_: v.data.reshape(-1) for k_, v in cuda.run(c, inputs)}
        finally:
            cuda.release(c)

    _, prod = run(Graph("p", [("z", z)]), ins)
    pz = D.param("z", F32, (m, n))
    _, sep = run(Graph("q", [("t", D.map(f, pz))]), [("z", Value.of_array(F32, (m, n), prod["z"]))])
    plan, fused = run(Graph("fz", [("t", D.map(f, z))]), ins)
    assert "ccb_mapreduce_" not in plan
    assert np.array_equal(fused["t"].view(np.uint32), sep["t"].view(np.uint32))
    # the product stored beside the pass's result
    plan, both = run(Graph("fb", [("t", D.map(f, z)), ("z", z)]), ins)
    assert "ccb_mapreduce_" not in plan
    assert np.array_equal(both["z"].view(np.uint32), prod["z"].view(np.uint32))
    assert np.array_equal(both["t"].view(np.uint32), sep["t"].view(np.uint32))
