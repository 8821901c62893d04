"""Workload definitions: the reference's example programs and the graphs of the
benchmark configurations.

* ``saxpy``        -- examples/saxpy.ml:10-17
* Black-Scholes    -- examples/black_scholes.ml (market, closed form, call_mc,
                      call_mc_paths, call_greeks, inputs)
* ``PROGRAMS``     -- the registry of examples/programs.ml:143-148
* configuration graphs for the flat/row reductions and scans, scatter/gather
  with Zipf indices, and seeded Philox inputs, built with the reference's own
  RNG so every synthetic input is reproducible bit for bit.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from . import dsl as D
from . import grad as Grad
from . import rng as Rng
from .ir import F32, F64, I32, Dtype, Graph, Value


# ---------------------------------------------------------------------------
# saxpy (examples/saxpy.ml)
# ---------------------------------------------------------------------------
def saxpy(n: int, a: float, dtype: Dtype = F32) -> Graph:
    """r = a*x + y ; s = sum r (examples/saxpy.ml:10-17)."""
    x = D.param("x", dtype, (n,))
    y = D.param("y", dtype, (n,))
    ax = D.map(lambda xi: D.mul(D.const(dtype, a), xi), x)
    r = D.map2(D.add, ax, y)
    s = D.reduce(D.add, D.const(dtype, 0.0), r)
    return Graph("saxpy", [("r", r), ("s", s)])


# ---------------------------------------------------------------------------
# Black-Scholes (examples/black_scholes.ml)
# ---------------------------------------------------------------------------
@dataclass
class Market:
    s0: float = 100.0
    strike: float = 100.0
    vol: float = 0.2
    rate: float = 0.05
    maturity: float = 1.0


MARKET = Market()


def norm_cdf(x):
    return 0.5 * (1.0 + math.erf(x / math.sqrt(2.0)))


def norm_pdf(x):
    return math.exp(-0.5 * x * x) / math.sqrt(2.0 * math.pi)


def analytic(m: Market = MARKET) -> dict:
    """Closed-form call, delta, vega, rho (black_scholes.ml:61-75)."""
    sqrt_t = math.sqrt(m.maturity)
    d1 = (math.log(m.s0 / m.strike) + (m.rate + 0.5 * m.vol * m.vol) * m.maturity) / (m.vol * sqrt_t)
    d2 = d1 - m.vol * sqrt_t
    disc = math.exp(-m.rate * m.maturity)
    return {
        "price": m.s0 * norm_cdf(d1) - m.strike * disc * norm_cdf(d2),
        "delta": norm_cdf(d1),
        "vega": m.s0 * norm_pdf(d1) * sqrt_t,
        "rho": m.strike * m.maturity * disc * norm_cdf(d2),
    }


def _bs_params(dtype):
    return D.scalar("s0", dtype), D.scalar("vol", dtype), D.scalar("rate", dtype), D.scalar("seed", I32)


def _discounted_mean(dtype, n_paths, m: Market, st, rate):
    """exp(-rT) * mean(max(S_T - K, 0)) (black_scholes.ml:98-104)."""
    kf = lambda v: D.const(dtype, v)  # noqa: E731
    payoff = D.map(lambda s: D.max(D.sub(s, kf(m.strike)), kf(0.0)), st)
    total = D.reduce(D.add, kf(0.0), payoff)
    mean = D.map(lambda s: D.div(s, kf(float(n_paths))), total)
    return D.map2(lambda mu, r: D.mul(mu, D.exp(D.neg(D.mul(r, kf(m.maturity))))), mean, rate)


def call_mc(n_paths: int, dtype: Dtype, m: Market = MARKET) -> Graph:
    """One-step GBM with z = Rng.normal(seed, counter = path index)
    (black_scholes.ml:109-126)."""
    shape = (n_paths,)
    s0, vol, rate, seed = _bs_params(dtype)
    kf = lambda v: D.const(dtype, v)  # noqa: E731
    z = Rng.normal(dtype, seed, shape)
    s0b = D.broadcast(shape, s0)
    volb = D.broadcast(shape, vol)
    rateb = D.broadcast(shape, rate)
    drift = D.map2(lambda r, v: D.mul(D.sub(r, D.mul(kf(0.5), D.mul(v, v))), kf(m.maturity)), rateb, volb)
    diffusion = D.map2(lambda v, zi: D.mul(D.mul(v, kf(math.sqrt(m.maturity))), zi), volb, z)
    st = D.map2(lambda s, e: D.mul(s, D.exp(e)), s0b, D.map2(D.add, drift, diffusion))
    return Graph("bs_mc", [("price", _discounted_mean(dtype, n_paths, m, st, rate))])


def call_mc_paths(n_paths: int, n_steps: int, dtype: Dtype, m: Market = MARKET) -> Graph:
    """n_steps-step paths with scan_rows and a gather of the last column
    (black_scholes.ml:133-152)."""
    grid = (n_paths, n_steps)
    s0, vol, rate, seed = _bs_params(dtype)
    kf = lambda v: D.const(dtype, v)  # noqa: E731
    ki = lambda v: D.const(I32, v)  # noqa: E731
    dt = m.maturity / n_steps
    z = Rng.normal(dtype, seed, grid)
    s0b = D.broadcast(grid, s0)
    volb = D.broadcast(grid, vol)
    rateb = D.broadcast(grid, rate)
    drift = D.map2(lambda r, v: D.mul(D.sub(r, D.mul(kf(0.5), D.mul(v, v))), kf(dt)), rateb, volb)
    diffusion = D.map2(lambda v, zi: D.mul(D.mul(v, kf(math.sqrt(dt))), zi), volb, z)
    cum = D.scan_rows(D.add, kf(0.0), D.map2(D.add, drift, diffusion))
    paths = D.map(D.exp, D.map2(lambda s, c: D.add(D.log(s), c), s0b, cum))
    idx = D.map(lambda p: D.add(D.mul(p, ki(n_steps)), ki(n_steps - 1)), D.iota((n_paths,)))
    st = D.gather(idx, paths)
    return Graph("bs_paths", [("price", _discounted_mean(dtype, n_paths, m, st, rate))])


def call_greeks(n_paths: int, dtype: Dtype, m: Market = MARKET) -> Graph:
    """call_mc plus delta, vega and rho by Grad.grad (black_scholes.ml:157-158)."""
    return Grad.grad(call_mc(n_paths, dtype, m), "price", ["s0", "vol", "rate"])


def bs_inputs(dtype: Dtype, m: Market = MARKET, seed: int = 42):
    """The four scalars (black_scholes.ml:165-172)."""
    f = lambda v: Value.of_list(dtype, (), [v])  # noqa: E731
    return [("s0", f(m.s0)), ("vol", f(m.vol)), ("rate", f(m.rate)), ("seed", Value.of_list(I32, (), [seed]))]


def scalar_out(outs, name: str) -> float:
    return float(dict(outs)[name].data[0])


# ---------------------------------------------------------------------------
# The example registry (examples/programs.ml)
# ---------------------------------------------------------------------------
@dataclass
class Program:
    name: str
    graph: object
    inputs: object


def _f32s(dims, f):
    n = int(np.prod(dims)) if dims else 1
    return Value.of_list(F32, tuple(dims), [f(i) for i in range(n)])


def _x_in(n):
    return ("x", _f32s([n], lambda i: float(i % 17) - 8.0))


def _y_in(n):
    return ("y", _f32s([n], lambda i: float(n - i) / 4.0))


def _saxpy_prog(n):
    return Program("saxpy", lambda: saxpy(n, 2.0), lambda: [_x_in(n), _y_in(n)])


def _sum_prog(n):
    def g():
        x = D.param("x", F32, (n,))
        return Graph("sum", [("s", D.reduce(D.add, D.const(F32, 0.0), x))])
    return Program("sum", g, lambda: [_x_in(n)])


def _maxval_prog(n):
    def g():
        x = D.param("x", F32, (n,))
        return Graph("maxval", [("m", D.reduce(D.max, D.const(F32, -1e30), x))])
    return Program("maxval", g, lambda: [_x_in(n)])


def _prefix_prog(n):
    def g():
        x = D.param("x", F32, (n,))
        return Graph("prefix", [("p", D.scan(D.add, D.const(F32, 0.0), x))])
    return Program("prefix", g, lambda: [_x_in(n)])


def _reverse_prog(n):
    def g():
        x = D.param("x", F32, (n,))
        idx = D.map(lambda i: D.sub(D.const(I32, n - 1), i), D.iota((n,)))
        return Graph("reverse", [("r", D.gather(idx, x))])
    return Program("reverse", g, lambda: [_x_in(n)])


def _clamp_prog(n):
    def g():
        x = D.param("x", F32, (n,))
        zero, one = D.const(F32, 0.0), D.const(F32, 1.0)
        r = D.map(lambda e: D.select(D.lt(e, zero), zero, D.select(D.lt(one, e), one, e)), x)
        return Graph("clamp", [("r", r)])
    return Program("clamp", g, lambda: [_x_in(n)])


def _squares_prog(n):
    def g():
        def body(i):
            f = D.cast(F32, i)
            return D.mul(f, f)
        return Graph("squares", [("r", D.map(body, D.iota((n,))))])
    return Program("squares", g, lambda: [])


def _chain_prog(n):
    def g():
        x = D.param("x", F32, (n,))
        one = D.const(F32, 1.0)
        r = D.map(lambda e: D.add(e, one), x)
        r = D.map(lambda e: D.mul(e, e), r)
        r = D.map(D.neg, r)
        r = D.map(lambda e: D.sub(e, one), r)
        r = D.map(lambda e: D.mul(e, D.const(F32, 0.5)), r)
        return Graph("chain", [("r", r)])
    return Program("chain", g, lambda: [_x_in(n)])


def _fanout_prog(n):
    def g():
        x = D.param("x", F32, (n,))
        s = D.map(lambda e: D.mul(e, e), x)
        return Graph("fanout", [("a", D.map(D.neg, s)), ("b", D.map(D.sqrt, s)),
                                ("c", D.reduce(D.add, D.const(F32, 0.0), s))])
    return Program("fanout", g, lambda: [_x_in(n)])


def _reshape_prog():
    def g():
        x = D.param("x", F32, (4, 8))
        return Graph("reshape_flat", [("r", D.map(D.neg, D.reshape((32,), x)))])
    return Program("reshape_flat", g, lambda: [("x", _f32s([4, 8], float))])


BS_DTYPE = F64
BS_SEED = 7


def _bs_inputs():
    return bs_inputs(BS_DTYPE, MARKET, BS_SEED)


PROGRAMS = [
    _saxpy_prog(1024), _sum_prog(1000), _maxval_prog(257), _prefix_prog(300), _reverse_prog(100),
    _clamp_prog(512), _squares_prog(64), _chain_prog(4096), _fanout_prog(1000), _reshape_prog(),
    Program("bs_mc", lambda: call_mc(4096, BS_DTYPE), _bs_inputs),
    Program("bs_paths", lambda: call_mc_paths(512, 16, BS_DTYPE), _bs_inputs),
    Program("bs_greeks", lambda: call_greeks(4096, BS_DTYPE), _bs_inputs),
]


def find(name: str):
    for p in PROGRAMS:
        if p.name == name:
            return p
    return None


# ---------------------------------------------------------------------------
# Seeded synthetic inputs from the reference's own Philox
# ---------------------------------------------------------------------------
def philox_word0(seed: int, n: int, base: int = 0) -> np.ndarray:
    """Word 0 of Philox4x32-10(ctr=(i,0,0,0), key=(seed,0)) for i in
    [base, base+n), vectorised in numpy (rng.ml:49-59). Used to make
    reproducible host inputs; the graphs themselves use Rng.u32."""
    c0 = (np.arange(base, base + n, dtype=np.uint64) & 0xFFFFFFFF)
    c1 = np.zeros(n, dtype=np.uint64)
    c2 = np.zeros(n, dtype=np.uint64)
    c3 = np.zeros(n, dtype=np.uint64)
    k0 = np.uint64(seed & 0xFFFFFFFF)
    k1 = np.uint64(0)
    M = np.uint64(0xFFFFFFFF)
    for r in range(10):
        p0 = np.uint64(Rng.M0) * c0
        p1 = np.uint64(Rng.M1) * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & M
        hi1, lo1 = p1 >> np.uint64(32), p1 & M
        c0, c1, c2, c3 = (hi1 ^ c1 ^ k0) & M, lo1, (hi0 ^ c3 ^ k1) & M, lo0
        if r < 9:
            k0 = (k0 + np.uint64(Rng.W0)) & M
            k1 = (k1 + np.uint64(Rng.W1)) & M
    return c0.astype(np.uint32)


def philox_uniform(seed: int, n: int, dtype=np.float64, base: int = 0) -> np.ndarray:
    """(w + 0.5) * 2^-32 in F64, then cast (rng.ml:61-67)."""
    w = philox_word0(seed, n, base).astype(np.float64)
    return ((w + 0.5) * 2.3283064365386963e-10).astype(dtype)


def philox_normal(seed: int, n: int, dtype=np.float32, base: int = 0) -> np.ndarray:
    """sqrt(2) * erfinv(2u - 1), computed in float64 with scipy then cast.
    Host input generation only."""
    from scipy.special import erfinv
    u = philox_uniform(seed, n, np.float64, base)
    return (math.sqrt(2.0) * erfinv(2.0 * u - 1.0)).astype(dtype)


def zipf_indices(seed: int, n: int, bins: int, s: float = 1.1) -> np.ndarray:
    """Zipf(s) bin indices on [0, bins) by inverse CDF over a host table,
    driven by the seeded Philox uniform stream."""
    w = 1.0 / np.power(np.arange(1, bins + 1, dtype=np.float64), s)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    u = philox_uniform(seed, n, np.float64)
    return np.minimum(np.searchsorted(cdf, u, side="left"), bins - 1).astype(np.int32)


# ---------------------------------------------------------------------------
# Benchmark-configuration graphs (reductions, scans, rows, scatter, gather)
# ---------------------------------------------------------------------------
def reduce_scan_flat(n: int, dtype: Dtype) -> Graph:
    x = D.param("x", dtype, (n,))
    zero = D.const(dtype, 0.0 if dtype.is_float else 0)
    return Graph("reduce_scan", [("s", D.reduce(D.add, zero, x)), ("p", D.scan(D.add, zero, x))])


def reduce_flat(n: int, dtype: Dtype) -> Graph:
    x = D.param("x", dtype, (n,))
    zero = D.const(dtype, 0.0 if dtype.is_float else 0)
    return Graph("reduce", [("s", D.reduce(D.add, zero, x))])


def scan_flat(n: int, dtype: Dtype) -> Graph:
    x = D.param("x", dtype, (n,))
    zero = D.const(dtype, 0.0 if dtype.is_float else 0)
    return Graph("scan", [("p", D.scan(D.add, zero, x))])


def rows(rows_: int, n: int) -> Graph:
    x = D.param("x", F32, (rows_, n))
    return Graph("rows", [("m", D.reduce_rows(D.max, D.const(F32, -3.0e38), x)),
                          ("p", D.scan_rows(D.add, D.const(F32, 0.0), x))])


def scatter(n: int, bins: int) -> Graph:
    idx = D.param("idx", I32, (n,))
    v = D.param("v", F32, (n,))
    return Graph("scatter", [("h", D.scatter_add(idx, v, (bins,)))])


def gather(n: int, table: int) -> Graph:
    idx = D.param("idx", I32, (n,))
    t = D.param("table", F32, (table,))
    return Graph("gather", [("g", D.gather(idx, t))])


# ---------------------------------------------------------------------------
# Two-layer MLP training step (BASELINE configuration)
# ---------------------------------------------------------------------------
def tanh_like(z):
    """tanh through exp: 1 - 2 / (exp(2z) + 1), saturating cleanly at +-1."""
    d = z.dtype
    return D.sub(D.const(d, 1.0), D.div(D.const(d, 2.0), D.add(D.exp(D.mul(D.const(d, 2.0), z)), D.const(d, 1.0))))


def mlp_loss(batch: int, din: int, hidden: int, dout: int, dtype: Dtype = F32) -> Graph:
    """loss = sum((tanh_like(X W1) W2 - T)^2): matmul -> map -> matmul ->
    squared-error reduce."""
    x = D.param("X", dtype, (batch, din))
    w1 = D.param("W1", dtype, (din, hidden))
    w2 = D.param("W2", dtype, (hidden, dout))
    t = D.param("T", dtype, (batch, dout))
    a1 = D.map(tanh_like, D.matmul(x, w1))
    y = D.matmul(a1, w2)
    d = D.map2(D.sub, y, t)
    loss = D.reduce(D.add, D.const(dtype, 0.0), D.map(lambda e: D.mul(e, e), d))
    return Graph("mlp", [("loss", loss)])


def mlp_step(batch: int, din: int, hidden: int, dout: int, dtype: Dtype = F32) -> Graph:
    """The loss and its gradients wrt W1 and W2 (Grad.grad)."""
    return Grad.grad(mlp_loss(batch, din, hidden, dout, dtype), "loss", ["W1", "W2"])


def mlp_flops(batch: int, din: int, hidden: int, dout: int) -> float:
    """Forward X.W1 and A1.W2, backward dA1 = dY.W2^T, dW2 = A1^T.dY and
    dW1 = X^T.dZ1: 2*B*Din*H * 2 + 2*B*H*Dout * 3."""
    return 2.0 * batch * din * hidden * 2 + 2.0 * batch * hidden * dout * 3
