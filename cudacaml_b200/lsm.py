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
Gaussian elimination with partial pivoting, as the reference's solve3
(lsm.ml:69-104), generalised to n x n: on the host in the generic driver
(``Make``), and as a one-launch graph (``solve_graph``) in the resident CUDA
driver.
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


def _cum_log_paths(n_paths: int, n_steps: int, m: Market):
    """lsm.ml:139-150: the running sums of the GBM log-increments, [n_paths;
    n_steps], and the map from them to S."""
    kf = lambda v: D.const(F64, v)  # noqa: E731
    seed = D.scalar("seed", I32)
    dt = m.maturity / n_steps
    drift = (m.rate - 0.5 * m.vol * m.vol) * dt
    vol_dt = m.vol * math.sqrt(dt)
    z = Rng.normal(F64, seed, (n_paths, n_steps))
    incr = D.map(lambda zi: D.add(kf(drift), D.mul(kf(vol_dt), zi)), z)
    return D.scan_rows(D.add, kf(0.0), incr), (lambda c: D.mul(kf(m.s0), D.exp(c)))


def paths_graph(n_paths: int, n_steps: int, m: Market = MARKET) -> Graph:
    """lsm.ml:139-150: column t of S holds time (t+1) dt."""
    cum, to_s = _cum_log_paths(n_paths, n_steps, m)
    return Graph("lsm_paths", [("S", D.map(to_s, cum))])


def paths_dates_graph(n_paths: int, n_steps: int, m: Market = MARKET) -> Graph:
    """The same S stored date-major, [n_steps; n_paths] (row t = date t): the
    map to S applied to the transposed running sums, which the lowering runs
    as one row scan writing the transposed tiles (no [n_paths; n_steps] copy
    is stored). The values are paths_graph's, transposed."""
    cum, to_s = _cum_log_paths(n_paths, n_steps, m)
    return Graph("lsm_paths", [("ST", D.map(to_s, D.transpose(cum)))])


def _basis(n_paths, n_steps, strike, basis, layout="paths", cf=None, tb=None, s=None):
    """Column t of S, the in-the-money mask and the masked design matrix
    (lsm.ml:170-192). ``layout="paths"`` reads S as the reference stores it,
    [n_paths; n_steps]; ``layout="dates"`` reads its transpose [n_steps;
    n_paths], where date t is one contiguous row. The cash flow `cf`, the
    per-path date `tb` and `S` default to the params "cf", "t" (broadcast)
    and "S"."""
    nb = _nb(basis)
    gb = (n_paths, nb)
    kf = lambda v: D.const(F64, v)  # noqa: E731
    ki = lambda v: D.const(I32, v)  # noqa: E731
    if cf is None:
        cf = D.param("cf", F64, (n_paths,))
    if tb is None:
        tb = D.broadcast((n_paths,), D.scalar("t", I32))
    if layout == "paths":
        s = s if s is not None else D.param("S", F64, (n_paths, n_steps))
        idx = D.map2(lambda p, tv: D.add(D.mul(p, ki(n_steps)), tv), D.iota((n_paths,)), tb)
    else:
        s = s if s is not None else D.param("S", F64, (n_steps, n_paths))
        idx = D.map2(lambda p, tv: D.add(D.mul(tv, ki(n_paths)), p), D.iota((n_paths,)), tb)
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


def _regress(n_paths, n_steps, strike, disc, basis, layout, **kw):
    """lsm.ml:201-212: the normal equations X^T X and X^T y of one date."""
    cf, st, itm, xm = _basis(n_paths, n_steps, strike, basis, layout, **kw)
    kf = lambda v: D.const(F64, v)  # noqa: E731
    y = D.map2(lambda c, mk: D.mul(D.mul(kf(disc), c), mk), cf, itm)
    xt = D.transpose(xm)
    return D.matmul(xt, xm), D.matmul(xt, D.reshape((n_paths, 1), y))


def _update(n_paths, n_steps, strike, disc, basis, layout, beta, **kw):
    """lsm.ml:219-234: exercise where intrinsic beats the fitted continuation;
    otherwise keep the realised cash flow, discounted."""
    cf, st, itm, xm = _basis(n_paths, n_steps, strike, basis, layout, **kw)
    kf = lambda v: D.const(F64, v)  # noqa: E731
    cont = D.reshape((n_paths,), D.matmul(xm, beta))

    def exercises(s, c):
        e = D.max(D.sub(kf(strike), s), kf(0.0))
        return D.and_(D.gt(e, kf(0.0)), D.gt(e, c))

    exv = D.map2(lambda s, c: D.select(exercises(s, c), D.sub(kf(strike), s), kf(0.0)), st, cont)
    keep = D.map2(lambda s, c: D.select(exercises(s, c), kf(0.0), kf(1.0)), st, cont)
    held = D.map2(lambda k, c: D.mul(k, D.mul(kf(disc), c)), keep, cf)
    return D.map2(D.add, exv, held)


def regress_graph(n_paths, n_steps, strike, disc, basis="scaled3", layout="paths") -> Graph:
    """lsm.ml:201-212."""
    xtx, xty = _regress(n_paths, n_steps, strike, disc, basis, layout)
    return Graph("lsm_regress", [("xtx", xtx), ("xty", xty)])


def update_graph(n_paths, n_steps, strike, disc, basis="scaled3", layout="paths") -> Graph:
    """lsm.ml:219-234."""
    beta = D.param("beta", F64, (_nb(basis), 1))
    return Graph("lsm_update", [("cf", _update(n_paths, n_steps, strike, disc, basis, layout, beta))])


def update_regress_graph(n_paths, n_steps, strike, disc, basis="scaled3", layout="dates") -> Graph:
    """Date t's update (lsm.ml:219-234) followed by date t-1's normal
    equations (lsm.ml:201-212) on the updated cash flow: the backward loop's
    update and next regression, which the lowering turns into one pass over
    the paths (S rows t and t-1, the cash flow read once and written once).
    The values are those of the two graphs run in turn."""
    beta = D.param("beta", F64, (_nb(basis), 1))
    s = D.param("S", F64, (n_steps, n_paths) if layout == "dates" else (n_paths, n_steps))
    tb = D.broadcast((n_paths,), D.scalar("t", I32))
    cf = _update(n_paths, n_steps, strike, disc, basis, layout, beta, tb=tb, s=s)
    tprev = D.map(lambda v: D.sub(v, D.const(I32, 1)), tb)
    xtx, xty = _regress(n_paths, n_steps, strike, disc, basis, layout, cf=cf, tb=tprev, s=s)
    return Graph("lsm_update_regress", [("cf", cf), ("xtx", xtx), ("xty", xty)])


def _with_solve(name, pairs, nb):
    """Graph of `pairs` (which hold "xtx" [nb; nb] and "xty" [nb; 1]) plus the
    solved beta b0 .. b{nb-1}: the solve becomes scalar tails of the same
    pass, run by its last block once the sums are final."""
    d = dict(pairs)
    bs = _solve(D.reshape((nb * nb,), d["xtx"]), D.reshape((nb,), d["xty"]), nb)
    return Graph(name, list(pairs) + [(f"b{i}", b) for i, b in enumerate(bs)])


def regress_solve_graph(n_paths, n_steps, strike, disc, basis="scaled3", layout="dates") -> Graph:
    """regress_graph and solve_graph in one pass (the first date)."""
    xtx, xty = _regress(n_paths, n_steps, strike, disc, basis, layout)
    return _with_solve("lsm_regress_solve", [("xtx", xtx), ("xty", xty)], _nb(basis))


def update_regress_solve_graph(n_paths, n_steps, strike, disc, basis="scaled3", layout="dates") -> Graph:
    """update_regress_graph and the solve of its normal equations in one
    pass: one launch per date."""
    g = update_regress_graph(n_paths, n_steps, strike, disc, basis, layout)
    return _with_solve("lsm_update_regress_solve", list(g.outputs), _nb(basis))


def solve_graph(nb: int) -> Graph:
    """The normal-equation solve of ``_beta`` as a graph, so that the
    resident driver keeps beta on the device: the ridge and the "fewer than nb
    in-the-money paths" rule of lsm.ml:283-294, and the Gaussian elimination
    with partial pivoting of ``solve`` (solve3, lsm.ml:69-104) in the same
    operation order -- the pivot is the first row of largest magnitude, rows
    are swapped by selects, a pivot not above 1e-300 or a non-finite result
    gives zeros. Every value is a one-element F64 tensor; the graph lowers to
    one single-element pass. Outputs b0 .. b{nb-1}, each [1]."""
    xtx = D.param("xtx", F64, (nb * nb,))
    xty = D.param("xty", F64, (nb,))
    return Graph("lsm_solve", [(f"b{i}", b) for i, b in enumerate(_solve(xtx, xty, nb))])


def _solve(xtx, xty, nb: int):
    """solve_graph's arithmetic on tensors xtx [nb*nb] and xty [nb]: the list
    of the nb one-element beta tensors."""
    one = (1,)
    kf = lambda v: D.const(F64, v)  # noqa: E731

    def el(src, i):
        return D.gather(D.full(I32, one, i), src)

    def f2(op, x, y):
        return D.map2(op, x, y)

    # Flags are F64 0/1 tensors (a graph may not hold Bool tensors: every
    # node of the reference interpreter is a storable value).
    def pick(c, x, y):  # c ? x : y: a select each way, then a sum with +0
        return f2(D.add, D.map2(lambda cc, v: D.select(D.gt(cc, kf(0.5)), v, kf(0.0)), c, x),
                  D.map2(lambda cc, v: D.select(D.gt(cc, kf(0.5)), kf(0.0), v), c, y))

    def absf(x):
        return D.map(D.abs, x)

    def flag2(cmp, x, y):
        return D.map2(lambda u, v: D.select(cmp(u, v), kf(1.0), kf(0.0)), x, y)

    def flag1(pred, x):
        return D.map(lambda u: D.select(pred(u), kf(1.0), kf(0.0)), x)

    def band(x, y):
        return f2(D.mul, x, y)

    def bor(x, y):
        return f2(D.max, x, y)

    def bnot(x):
        return D.map(lambda u: D.sub(kf(1.0), u), x)

    a = [[el(xtx, i * nb + j) for j in range(nb)] for i in range(nb)]
    bv = [el(xty, i) for i in range(nb)]
    few = flag1(lambda e: D.lt(e, kf(float(nb))), a[0][0])
    a = [[D.map(lambda e: D.add(e, kf(1e-10)), a[i][j]) if i == j else a[i][j] for j in range(nb)] for i in range(nb)]
    bad = few
    for k in range(nb):
        best = absf(a[k][k])
        ind = {k: D.full(F64, one, 1.0)}
        for i in range(k + 1, nb):
            take = flag2(D.gt, absf(a[i][k]), best)
            best = pick(take, absf(a[i][k]), best)
            keep = bnot(take)
            for m in list(ind):
                ind[m] = band(ind[m], keep)
            ind[i] = take
        bad = bor(bad, flag1(lambda e: D.not_(D.gt(e, kf(1e-300))), best))
        rowk = []
        for j in range(nb):
            v = a[k][j]
            for i in range(k + 1, nb):
                v = pick(ind[i], a[i][j], v)
            rowk.append(v)
        bk = bv[k]
        for i in range(k + 1, nb):
            bk = pick(ind[i], bv[i], bk)
        for i in range(k + 1, nb):
            a[i] = [pick(ind[i], a[k][j], a[i][j]) for j in range(nb)]
            bv[i] = pick(ind[i], bv[k], bv[i])
        a[k], bv[k] = rowk, bk
        for i in range(k + 1, nb):
            fct = f2(D.div, a[i][k], a[k][k])
            for j in range(k, nb):
                a[i][j] = f2(D.sub, a[i][j], f2(D.mul, fct, a[k][j]))
            bv[i] = f2(D.sub, bv[i], f2(D.mul, fct, bv[k]))
    x = [None] * nb
    for i in range(nb - 1, -1, -1):
        acc = bv[i]
        for j in range(i + 1, nb):
            acc = f2(D.sub, acc, f2(D.mul, a[i][j], x[j]))
        x[i] = f2(D.div, acc, a[i][i])
    for i in range(nb):
        bad = bor(bad, flag1(lambda e: D.not_(D.eq(D.sub(e, e), kf(0.0))), x[i]))
    return [pick(bad, D.full(F64, one, 0.0), x[i]) for i in range(nb)]


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
    """The resident CUDA driver (lsm.ml:321-420): S, the running cash flow,
    the normal equations and beta never leave the device. The reference's
    driver brings the normal equations to the host each date for its solve;
    here the same solve runs as a graph (solve_graph) on the device, so the
    host only launches. S is generated date-major (paths_dates_graph), so
    each date reads one contiguous row; the device buffers are allocated
    once."""

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
        self.paths = cuda.compile_on(device, paths_dates_graph(n_paths, n_steps, m))
        self.update = cuda.compile_on(device, update_graph(n_paths, n_steps, self.strike, self.disc, basis, "dates"))
        self.reg_solve = cuda.compile_on(device, regress_solve_graph(n_paths, n_steps, self.strike, self.disc, basis, "dates"))
        self.upd_reg = cuda.compile_on(device, update_regress_solve_graph(n_paths, n_steps, self.strike, self.disc, basis,
                                                                          "dates"))
        self.final = cuda.compile_on(device, _final_graph(n_paths, n_steps, self.strike))
        cfp = D.param("cf", F64, (n_paths,))
        self.total = cuda.compile_on(device, Graph("lsm_total", [("s", D.reduce(D.add, D.const(F64, 0.0), cfp))]))
        n, ns, nb = n_paths, n_steps, self.nb
        with R.with_device(device):
            self.bufs = {"ST": R.Buffer(n * ns * 8), "cf_a": R.Buffer(n * 8),
                         "cf_b": R.Buffer(n * 8), "seed": R.Buffer(4), "t": R.Buffer(4 * ns), "beta": R.Buffer(nb * 8),
                         "beta_b": R.Buffer(nb * 8),
                         "xtx": R.Buffer(nb * nb * 8), "xty": R.Buffer(nb * 8), "sum": R.Buffer(8)}
            self.bufs["t"].upload(np.arange(ns, dtype=np.int32))  # date t lives at t + 4 t bytes
        self.graph = None  # the captured price, made by the first price()

    def _issue(self, stream, trace=None):
        """The device work of one price on `stream`: generation from the seed
        in bufs["seed"], the transpose, every date (regress, the graph solve
        of the normal equations, update) and the sum of the final cash flows
        into bufs["sum"]. With `trace` the normal equations are also copied
        out each date (which synchronises)."""
        cuda, R = self.cuda, self.R
        ns, nb = self.n_steps, self.nb
        b = self.bufs

        def bind(c, **ptrs):  # device pointers in the program's param order
            return [ptrs[name] for name, _, _ in c.params]

        cuda.run_device_ptrs(self.paths, bind(self.paths, seed=b["seed"].ptr), [b["ST"].ptr], stream)
        # initial cash flow: intrinsic value at maturity (the last date's row), on the device
        cuda.run_device_ptrs(self.final, bind(self.final, S=b["ST"].ptr), [b["cf_a"].ptr], stream)
        xtx = np.empty(nb * nb)
        xty = np.empty(nb)
        cur, nxt = b["cf_a"], b["cf_b"]
        beta, beta_next = b["beta"], b["beta_b"]  # read by this date's update, written for the next

        def outs_of(prog, cf_out, beta_out):
            o = {"cf": cf_out, "xtx": b["xtx"].ptr, "xty": b["xty"].ptr}
            o.update({f"b{j}": beta_out.ptr + 8 * j for j in range(nb)})
            return [o[name] for name, _, _ in prog.outputs]

        def normal_equations(step, prog):
            if trace is not None:
                R.check(R.lib().ccb_memcpy_d2h(xtx.ctypes.data, b["xtx"].ptr, xtx.nbytes, stream))
                R.check(R.lib().ccb_memcpy_d2h(xty.ctypes.data, b["xty"].ptr, xty.nbytes, stream))
                cuda.check_device(prog, stream)
                trace.append((step, xtx.copy(), xty.copy()))

        # Dates ns-2 .. 0 backwards, one launch each: the first date's normal
        # equations and their solve; then per date the update with the last
        # beta, the next date's normal equations from the updated cash flow
        # and their solve; the last date (0) an update alone.
        steps = list(range(ns - 2, -1, -1))
        if steps:
            rs = self.reg_solve
            t0 = b["t"].ptr + 4 * steps[0]
            cuda.run_device_ptrs(rs, bind(rs, S=b["ST"].ptr, cf=cur.ptr, t=t0), outs_of(rs, None, beta), stream)
            normal_equations(steps[0], rs)
        for k, step in enumerate(steps):
            t_ptr = b["t"].ptr + 4 * step
            if k + 1 < len(steps):
                ur = self.upd_reg
                cuda.run_device_ptrs(ur, bind(ur, S=b["ST"].ptr, cf=cur.ptr, t=t_ptr, beta=beta.ptr),
                                     outs_of(ur, nxt.ptr, beta_next), stream)
                normal_equations(step - 1, ur)
                beta, beta_next = beta_next, beta
            else:
                cuda.run_device_ptrs(self.update, bind(self.update, S=b["ST"].ptr, cf=cur.ptr, t=t_ptr, beta=beta.ptr),
                                     [nxt.ptr], stream)
            cur, nxt = nxt, cur
        # the mean of the discounted cash flows (lsm.ml:303-305): summed on the device
        cuda.run_device_ptrs(self.total, [cur.ptr], [b["sum"].ptr], stream)

    def price(self, seed: int, trace=None) -> float:
        """Generation, the transpose and all dates run back to back on one
        stream. The first call captures that work as a CUDA graph (about 190
        program runs); every call then uploads the seed, replays the graph
        with one launch and reads the sum back. With `trace` the work is
        issued run by run instead, copying the normal equations out each
        date."""
        cuda, R = self.cuda, self.R
        b = self.bufs
        stream = self.reg_solve.lane_stream(0)
        progs = (self.paths, self.final, self.reg_solve, self.update, self.upd_reg, self.total)
        with R.with_device(self.device):
            seed_h = np.array([seed], np.int32)
            R.check(R.lib().ccb_memcpy_h2d(b["seed"].ptr, seed_h.ctypes.data, 4, stream))
            if trace is not None:
                self._issue(stream, trace)
            else:
                if self.graph is None:
                    with R.Graph.capture(stream) as g:
                        self._issue(stream)
                    self.graph = g
                self.graph.launch(stream)
            tot = np.empty(1)
            R.check(R.lib().ccb_memcpy_d2h(tot.ctypes.data, b["sum"].ptr, 8, stream))
            for c in progs:  # each program's error word, accumulated over all its runs
                cuda.check_device(c, stream)
        return self.disc * float(tot[0]) / self.n_paths

    def release(self):
        with self.R.with_device(self.device):
            if self.graph is not None:
                self.graph.destroy()
                self.graph = None
            for buf in self.bufs.values():
                buf.free()
        self.bufs = {}
        for c in (self.paths, self.reg_solve, self.update, self.upd_reg, self.final, self.total):
            self.cuda.release(c)


def _final_graph(n_paths, n_steps, strike) -> Graph:
    """max(K - S at maturity, 0): the initial cash flow, on the device, from
    the last row of the date-major S [n_steps; n_paths]."""
    s = D.param("S", F64, (n_steps, n_paths))
    idx = D.map(lambda p: D.add(p, D.const(I32, (n_steps - 1) * n_paths)), D.iota((n_paths,)))
    last = D.gather(idx, s)
    return Graph("lsm_final", [("cf", D.map(lambda x: D.max(D.sub(D.const(F64, strike), x), D.const(F64, 0.0)), last))])


BASELINE_MARKET = Market(s0=36.0, strike=40.0, vol=0.2, rate=0.06, maturity=1.0)
