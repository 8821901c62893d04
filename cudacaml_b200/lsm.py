"""Longstaff-Schwartz American put, restating CUDACaml's examples/lsm.ml.

Three graphs are compiled once and then only run (lsm.ml:126-236):

* ``paths``   -- S : [n_paths; n_steps] of GBM from Rng.normal + scan_rows;
* ``regress`` -- the normal equations X^T X and X^T y of the in-the-money
                 paths at exercise date t (two matmuls of a transposed design
                 matrix; here one split-K pass);
* ``update``  -- the exercise decision and the new cash flow (X . beta is a
                 K = nb dot product, fused inline).

The basis is either the reference's strike-scaled ``[1, S/K, (S/K)^2]``
(``basis="scaled3"``, lsm.ml:170-192) or ``[1, S, S^2, S^3]``
(``basis="poly4"``, the BASELINE configuration). The small dense solve is a
host Gaussian elimination with partial pivoting, as the reference's solve3
(lsm.ml:69-104), generalised to n x n.
"""
from __future__ import annotations

import math

import numpy as np

from . import dsl as D
from . import rng as Rng
from .examples import MARKET, Market, analytic
from .ir import F64, I32, Graph, Value


def binomial_american_put(m: Market = MARKET, steps: int = 500) -> float:
    """Cox-Ross-Rubinstein American put (lsm.ml:40-57)."""
    n = steps
    dt = m.maturity / n
    u = math.exp(m.vol * math.sqrt(dt))
    d = 1.0 / u
    disc = math.exp(-m.rate * dt)
    p = ((1.0 / disc) - d) / (u - d)
    j = np.arange(n + 1)
    v = np.maximum(m.strike - m.s0 * u ** j * d ** (n - j), 0.0)
    for i in range(n - 1, -1, -1):
        j = np.arange(i + 1)
        cont = disc * (p * v[1:i + 2] + (1.0 - p) * v[:i + 1])
        v = np.maximum(cont, m.strike - m.s0 * u ** j * d ** (i - j))
    return float(v[0])


def european_put(m: Market = MARKET) -> float:
    """Put-call parity on the closed-form call (lsm.ml:64-66)."""
    return analytic(m)["price"] - m.s0 + m.strike * math.exp(-m.rate * m.maturity)


def solve(a0, b0):
    """Gaussian elimination with partial pivoting; a singular or non-finite
    system yields zeros ("no usable regression"), as solve3 (lsm.ml:69-104)."""
    a = [list(r) for r in a0]
    b = list(b0)
    n = len(b)
    x = [0.0] * n
    try:
        for k in range(n):
            piv = max(range(k, n), key=lambda i: abs(a[i][k]))
            if not abs(a[piv][k]) > 1e-300:
                raise ZeroDivisionError
            if piv != k:
                a[k], a[piv] = a[piv], a[k]
                b[k], b[piv] = b[piv], b[k]
            for i in range(k + 1, n):
                f = a[i][k] / a[k][k]
                for j in range(k, n):
                    a[i][j] -= f * a[k][j]
                b[i] -= f * b[k]
        for i in range(n - 1, -1, -1):
            s = b[i]
            for j in range(i + 1, n):
                s -= a[i][j] * x[j]
            x[i] = s / a[i][i]
        if not all(math.isfinite(v) for v in x):
            raise ZeroDivisionError
    except ZeroDivisionError:
        x = [0.0] * n
    return x


def _nb(basis: str) -> int:
    return {"scaled3": 3, "poly4": 4}[basis]


def paths_graph(n_paths: int, n_steps: int, m: Market = MARKET) -> Graph:
    """lsm.ml:139-150: column t of S holds time (t+1) dt."""
    grid = (n_paths, n_steps)
    kf = lambda v: D.const(F64, v)  # noqa: E731
    seed = D.scalar("seed", I32)
    dt = m.maturity / n_steps
    drift = (m.rate - 0.5 * m.vol * m.vol) * dt
    vol_dt = m.vol * math.sqrt(dt)
    z = Rng.normal(F64, seed, grid)
    incr = D.map(lambda zi: D.add(kf(drift), D.mul(kf(vol_dt), zi)), z)
    cum = D.scan_rows(D.add, kf(0.0), incr)
    s = D.map(lambda c: D.mul(kf(m.s0), D.exp(c)), cum)
    return Graph("lsm_paths", [("S", s)])


def _basis(n_paths, n_steps, strike, basis):
    """Column t of S, the in-the-money mask and the masked design matrix
    (lsm.ml:170-192)."""
    nb = _nb(basis)
    grid = (n_paths, n_steps)
    gb = (n_paths, nb)
    kf = lambda v: D.const(F64, v)  # noqa: E731
    ki = lambda v: D.const(I32, v)  # noqa: E731
    s = D.param("S", F64, grid)
    cf = D.param("cf", F64, (n_paths,))
    tb = D.broadcast((n_paths,), D.scalar("t", I32))
    idx = D.map2(lambda p, tv: D.add(D.mul(p, ki(n_steps)), tv), D.iota((n_paths,)), tb)
    st = D.gather(idx, s)
    itm = D.map(lambda x: D.select(D.lt(x, kf(strike)), kf(1.0), kf(0.0)), st)
    row = D.map(lambda k: D.div(k, ki(nb)), D.iota(gb))
    st3 = D.gather(row, st)
    itm3 = D.gather(row, itm)

    def phi(k, sv):
        j = D.sub(k, D.mul(D.div(k, ki(nb)), ki(nb)))
        if basis == "scaled3":
            x = D.div(sv, kf(strike))
            return D.select(D.eq(j, ki(0)), kf(1.0), D.select(D.eq(j, ki(1)), x, D.mul(x, x)))
        x = sv
        return D.select(D.eq(j, ki(0)), kf(1.0),
                        D.select(D.eq(j, ki(1)), x, D.select(D.eq(j, ki(2)), D.mul(x, x), D.mul(D.mul(x, x), x))))

    ph = D.map2(phi, D.iota(gb), st3)
    return cf, st, itm, D.map2(D.mul, ph, itm3)


def regress_graph(n_paths, n_steps, strike, disc, basis="scaled3") -> Graph:
    """lsm.ml:201-212."""
    cf, st, itm, xm = _basis(n_paths, n_steps, strike, basis)
    kf = lambda v: D.const(F64, v)  # noqa: E731
    y = D.map2(lambda c, mk: D.mul(D.mul(kf(disc), c), mk), cf, itm)
    xt = D.transpose(xm)
    return Graph("lsm_regress", [("xtx", D.matmul(xt, xm)), ("xty", D.matmul(xt, D.reshape((n_paths, 1), y)))])


def update_graph(n_paths, n_steps, strike, disc, basis="scaled3") -> Graph:
    """lsm.ml:219-234: exercise where intrinsic beats the fitted continuation;
    otherwise keep the realised cash flow, discounted."""
    nb = _nb(basis)
    cf, st, itm, xm = _basis(n_paths, n_steps, strike, basis)
    kf = lambda v: D.const(F64, v)  # noqa: E731
    beta = D.param("beta", F64, (nb, 1))
    cont = D.reshape((n_paths,), D.matmul(xm, beta))

    def exercises(s, c):
        e = D.max(D.sub(kf(strike), s), kf(0.0))
        return D.and_(D.gt(e, kf(0.0)), D.gt(e, c))

    exv = D.map2(lambda s, c: D.select(exercises(s, c), D.sub(kf(strike), s), kf(0.0)), st, cont)
    keep = D.map2(lambda s, c: D.select(exercises(s, c), kf(0.0), kf(1.0)), st, cont)
    held = D.map2(lambda k, c: D.mul(k, D.mul(kf(disc), c)), keep, cf)
    return Graph("lsm_update", [("cf", D.map2(D.add, exv, held))])


def _beta(xtx, xty, nb):
    """lsm.ml:283-294: below nb in-the-money paths the fit is skipped; a
    1e-10 ridge on the diagonal."""
    if xtx[0] < nb:
        return [0.0] * nb
    a = [[xtx[i * nb + j] + (1e-10 if i == j else 0.0) for j in range(nb)] for i in range(nb)]
    return solve(a, list(xty))


class Make:
    """The driver over any Backend.S (lsm.ml:251-305): S crosses to the host
    and back as an ordinary Value each step."""

    def __init__(self, backend, n_paths: int, n_steps: int, m: Market = MARKET, basis: str = "scaled3"):
        if n_paths < 1 or n_steps < 1:
            raise ValueError("Lsm.create: n_paths and n_steps must be >= 1")
        self.B = backend
        self.n_paths, self.n_steps, self.basis = n_paths, n_steps, basis
        self.nb = _nb(basis)
        dt = m.maturity / n_steps
        self.disc = math.exp(-m.rate * dt)
        self.strike = m.strike
        self.paths = backend.compile(paths_graph(n_paths, n_steps, m))
        self.regress = backend.compile(regress_graph(n_paths, n_steps, self.strike, self.disc, basis))
        self.update = backend.compile(update_graph(n_paths, n_steps, self.strike, self.disc, basis))

    def price(self, seed: int, trace=None) -> float:
        B = self.B
        n, ns = self.n_paths, self.n_steps
        s = dict(B.run(self.paths, [("seed", Value.of_list(I32, (), [seed]))]))["S"]
        last = s.data.reshape(n, ns)[:, ns - 1]
        cf = Value.of_array(F64, (n,), np.maximum(self.strike - last, 0.0))
        for step in range(ns - 2, -1, -1):
            tv = Value.of_list(I32, (), [step])
            o = dict(B.run(self.regress, [("S", s), ("cf", cf), ("t", tv)]))
            xtx, xty = o["xtx"].data, o["xty"].data
            if trace is not None:
                trace.append((step, xtx.copy(), xty.copy()))
            beta = _beta(xtx, xty, self.nb)
            bv = Value.of_list(F64, (self.nb, 1), beta)
            cf = dict(B.run(self.update, [("S", s), ("cf", cf), ("t", tv), ("beta", bv)]))["cf"]
        return self.disc * float(np.sum(cf.data)) / n


class CudaResident:
    """The resident CUDA driver (lsm.ml:321-420): S and the running cash flow
    never leave the device; per date only the normal equations (nb^2 + nb
    doubles) come back and beta (nb doubles) goes out."""

    def __init__(self, n_paths: int, n_steps: int, m: Market = MARKET, basis: str = "scaled3", device: int = 0):
        from . import backend_cuda as cuda
        from . import runtime as R
        self.cuda, self.R = cuda, R
        self.n_paths, self.n_steps, self.basis = n_paths, n_steps, basis
        self.nb = _nb(basis)
        dt = m.maturity / n_steps
        self.disc = math.exp(-m.rate * dt)
        self.strike = m.strike
        self.device = device
        self.paths = cuda.compile_on(device, paths_graph(n_paths, n_steps, m))
        self.regress = cuda.compile_on(device, regress_graph(n_paths, n_steps, self.strike, self.disc, basis))
        self.update = cuda.compile_on(device, update_graph(n_paths, n_steps, self.strike, self.disc, basis))
        self.final = cuda.compile_on(device, _final_graph(n_paths, n_steps, self.strike))

    def price(self, seed: int, trace=None) -> float:
        cuda, R = self.cuda, self.R
        n, ns, nb = self.n_paths, self.n_steps, self.nb
        with R.with_device(self.device):
            s_buf = R.Buffer(n * ns * 8)
            cf_a = R.Buffer(n * 8)
            cf_b = R.Buffer(n * 8)
            seed_b = R.Buffer(4)
            seed_b.upload(np.array([seed], np.int32))
            t_b = R.Buffer(4)
            beta_b = R.Buffer(nb * 8)
            xtx_b = R.Buffer(nb * nb * 8)
            xty_b = R.Buffer(nb * 8)
            stream = self.regress.lane_stream(0)
            try:
                def bind(c, **ptrs):  # device pointers in the program's param order
                    return [ptrs[name] for name, _, _ in c.params]

                cuda.run_device_ptrs(self.paths, bind(self.paths, seed=seed_b.ptr), [s_buf.ptr], stream)
                # initial cash flow: intrinsic value at maturity (last column), on the device
                cuda.run_device_ptrs(self.final, bind(self.final, S=s_buf.ptr), [cf_a.ptr], stream)
                cuda.check_device(self.paths, stream)
                xtx = np.empty(nb * nb)
                xty = np.empty(nb)
                cur, nxt = cf_a, cf_b
                for step in range(ns - 2, -1, -1):
                    R.check(R.lib().ccb_memcpy_h2d(t_b.ptr, np.array([step], np.int32).ctypes.data, 4, stream))
                    outs = {"xtx": xtx_b.ptr, "xty": xty_b.ptr}
                    cuda.run_device_ptrs(self.regress, bind(self.regress, S=s_buf.ptr, cf=cur.ptr, t=t_b.ptr),
                                         [outs[name] for name, _, _ in self.regress.outputs], stream)
                    R.check(R.lib().ccb_memcpy_d2h(xtx.ctypes.data, xtx_b.ptr, xtx.nbytes, stream))
                    R.check(R.lib().ccb_memcpy_d2h(xty.ctypes.data, xty_b.ptr, xty.nbytes, stream))
                    cuda.check_device(self.regress, stream)
                    if trace is not None:
                        trace.append((step, xtx.copy(), xty.copy()))
                    beta = np.array(_beta(xtx, xty, nb), np.float64)
                    R.check(R.lib().ccb_memcpy_h2d(beta_b.ptr, beta.ctypes.data, beta.nbytes, stream))
                    cuda.run_device_ptrs(self.update, bind(self.update, S=s_buf.ptr, cf=cur.ptr, t=t_b.ptr, beta=beta_b.ptr),
                                         [nxt.ptr], stream)
                    cur, nxt = nxt, cur
                cfh = np.empty(n)
                R.check(R.lib().ccb_memcpy_d2h(cfh.ctypes.data, cur.ptr, cfh.nbytes, stream))
                cuda.check_device(self.update, stream)
            finally:
                for b in (s_buf, cf_a, cf_b, seed_b, t_b, beta_b, xtx_b, xty_b):
                    b.free()
        return self.disc * float(np.sum(cfh)) / n

    def release(self):
        for c in (self.paths, self.regress, self.update, self.final):
            self.cuda.release(c)


def _final_graph(n_paths, n_steps, strike) -> Graph:
    """max(K - S[:, n_steps - 1], 0): the initial cash flow, on the device."""
    s = D.param("S", F64, (n_paths, n_steps))
    idx = D.map(lambda p: D.add(D.mul(p, D.const(I32, n_steps)), D.const(I32, n_steps - 1)), D.iota((n_paths,)))
    last = D.gather(idx, s)
    return Graph("lsm_final", [("cf", D.map(lambda x: D.max(D.sub(D.const(F64, strike), x), D.const(F64, 0.0)), last))])


BASELINE_MARKET = Market(s0=36.0, strike=40.0, vol=0.2, rate=0.06, maturity=1.0)
