"""Parity at the benchmark configurations' full sizes, where the oracle would
take hours: the MLP training step (8192 x 4096 -> 8192 -> 1024, products on
the tcgen05 tensor cores) against an F64 evaluation of the same step on the
same F32 inputs, and the Longstaff-Schwartz price (2^22 paths x 64 dates,
4-term basis, F64) against the binomial American put.

Tolerances:
* MLP, per output: max |g - e| <= 1e-2 * max |e| (normwise) and
  ||g - e||_F <= 5e-3 * ||e||_F. TF32 rounds every product operand to 10
  explicit mantissa bits (unit roundoff 2^-11 ~ 4.9e-4); the gradients pass
  through up to three products, and entries are sums of signed products, so
  a per-entry relative band is not meaningful. The loss, a sum of 2^23
  squares: relative 1e-3.
* LSM: the reference's S17 band, |price - binomial| <= 0.15
  (test/system/test_system.ml:190-195), and a tighter 0.05 (the regression
  estimator's low bias plus the Monte-Carlo error at 2^22 paths, ~0.003).
"""
import math

import numpy as np
import pytest

from cudacaml_b200 import backend_cuda as cuda
from cudacaml_b200 import examples as X
from cudacaml_b200 import lsm as L
from cudacaml_b200.ir import F32, Value

pytestmark = pytest.mark.gpu


def _mlp_f64(xs, w1, w2, t):
    """The step in F64 on the GPU (torch), from the same F32 inputs: loss =
    sum((tanh_like(X W1) W2 - T)^2) and its gradients wrt W1 and W2."""
    import torch
    dev = torch.device("cuda", 0)
    X_, W1, W2, T = (torch.from_numpy(a).to(dev, torch.float64) for a in (xs, w1, w2, t))
    A1 = 1.0 - 2.0 / (torch.exp(2.0 * (X_ @ W1)) + 1.0)
    Dy = A1 @ W2 - T
    loss = float((Dy * Dy).sum())
    dY = 2.0 * Dy
    dW2 = A1.T @ dY
    dZ1 = (dY @ W2.T) * (1.0 - A1 * A1)
    dW1 = X_.T @ dZ1
    return {"loss": np.array([loss]), "dloss/dW1": dW1.cpu().numpy(), "dloss/dW2": dW2.cpu().numpy()}


def test_mlp_step_full_size_tf32_vs_f64():
    bsz, din, hid, dout = 8192, 4096, 8192, 1024
    rng = np.random.default_rng(2024)
    xs = rng.standard_normal((bsz, din), dtype=np.float32)
    w1 = (rng.standard_normal((din, hid), dtype=np.float32) / np.float32(math.sqrt(din))).astype(np.float32)
    w2 = (rng.standard_normal((hid, dout), dtype=np.float32) / np.float32(math.sqrt(hid))).astype(np.float32)
    t = rng.standard_normal((bsz, dout), dtype=np.float32)
    ins = [("X", Value.of_array(F32, xs.shape, xs)), ("W1", Value.of_array(F32, w1.shape, w1)),
           ("W2", Value.of_array(F32, w2.shape, w2)), ("T", Value.of_array(F32, t.shape, t))]
    c = cuda.compile(X.mlp_step(bsz, din, hid, dout), matmul="tf32")
    assert "ccb_matmultc" in c.plan()
    got = {k: v.data.astype(np.float64).reshape(-1) for k, v in cuda.run(c, ins)}
    cuda.release(c)
    want = {k: v.reshape(-1) for k, v in _mlp_f64(xs, w1, w2, t).items()}
    le, lg = float(want["loss"][0]), float(got["loss"][0])
    print(f"    loss {lg:.6e} vs F64 {le:.6e} (rel {abs(lg - le) / abs(le):.2e})")
    assert abs(lg - le) <= 1e-3 * abs(le)
    for name in ("dloss/dW1", "dloss/dW2"):
        e, g = want[name], got[name]
        norm = np.max(np.abs(g - e)) / np.max(np.abs(e))
        frob = np.linalg.norm(g - e) / np.linalg.norm(e)
        print(f"    {name}: normwise {norm:.2e}, Frobenius {frob:.2e}")
        assert norm <= 1e-2, (name, norm)
        assert frob <= 5e-3, (name, frob)


def test_lsm_full_size_vs_binomial():
    binom = L.binomial_american_put(L.BASELINE_MARKET)
    lp = L.CudaResident(1 << 22, 64, L.BASELINE_MARKET, "poly4")
    try:
        px = lp.price(7)
        px2 = lp.price(7)
    finally:
        lp.release()
    print(f"    lsm 2^22 x 64 poly4 {px:.4f}  binomial {binom:.4f}")
    assert px == px2  # the replayed driver is deterministic
    assert abs(px - binom) <= 0.15
    assert abs(px - binom) <= 0.05
