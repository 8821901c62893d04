"""GPU parity: the CUDA path through libccb.so against the oracle (the C++
restatement of the reference interpreter), in the manner of the reference's
gated system suite (test/system/test_system.ml S1-S19), plus the
benchmark-configuration graphs at sizes the oracle finishes in seconds.

Tolerances are the reference's: Differential's default 1e-5 relative-plus-
absolute band, 1e-3 for long F32 sums (S3, S10), 1e-4/1e-9 for F32/F64
products (S11), 1e-6 for the F64 Greeks (S13). Integer and Philox u32 outputs
are bit-exact.
"""
import json
import os

import numpy as np
import pytest

from cudacaml_b200 import backend_cuda as cuda
from cudacaml_b200 import differential as Diff
from cudacaml_b200 import dsl as D
from cudacaml_b200 import examples as X
from cudacaml_b200 import rng as Rng
from cudacaml_b200 import runtime as R
from cudacaml_b200.ir import F32, F64, I32, Graph, Value
from oracle import interp

pytestmark = pytest.mark.gpu
GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))


def diff(g, inputs, tol=1e-5):
    err = Diff.check(interp, cuda, g, inputs, tolerance=tol)
    assert err is None, err


def f32s(n, f):
    return Value.of_array(F32, (n,), np.array([f(i) for i in range(n)], dtype=np.float32))


def test_native_library_is_the_path():
    assert R.available(), R.lib().ccb_last_error().decode()
    info = R.info(0)
    assert info["compute_capability"][0] >= 10, info


@pytest.mark.parametrize("prog", X.PROGRAMS, ids=lambda p: p.name)
def test_s1_examples(prog):
    diff(prog.graph(), prog.inputs())


@pytest.mark.parametrize("n", GOLD["saxpy_edge_sizes"]["n"])
def test_s2_saxpy_edge_sizes(n):
    x = Value.of_array(F32, (n,), np.arange(n, dtype=np.float32))
    y = Value.of_array(F32, (n,), (n - np.arange(n)).astype(np.float32))
    diff(X.saxpy(n, 3.0), [("x", x), ("y", y)])


def test_s3_sum_4m():
    n = 1 << 22
    x = Value.of_array(F32, (n,), (np.arange(n) % 7 - 3.0).astype(np.float32))
    diff(X.reduce_flat(n, F32), [("x", x)], tol=1e-3)


def test_s6_i32_arithmetic():
    x = D.param("x", I32, (9,))
    r = D.map(lambda e: D.div(D.sub(e, D.const(I32, 4)), D.const(I32, 2)), x)
    diff(Graph("i32", [("r", r)]), [("x", Value.of_array(I32, (9,), np.arange(9, dtype=np.int32)))])


def test_s8_u32_bit_exact():
    g = Graph("u32", [("r", Rng.u32(D.scalar("seed", I32), (1 << 20,)))])
    diff(g, [("seed", Value.of_list(I32, (), [12345]))], tol=0.0)


def test_uniform_f32_f64_bit_exact():
    for dt in (F32, F64):
        g = Graph("u", [("r", Rng.uniform(dt, D.scalar("seed", I32), (1 << 18,)))])
        diff(g, [("seed", Value.of_list(I32, (), [5]))], tol=0.0)


def test_s9_normal_f32_moments_and_parity():
    g = Graph("n", [("z", Rng.normal(F32, D.scalar("seed", I32), (1 << 20,)))])
    c = cuda.compile(g)
    z = dict(cuda.run(c, [("seed", Value.of_list(I32, (), [99]))]))["z"].data
    assert abs(z.mean()) < 0.01 and abs(z.var() - 1.0) < 0.02
    # erfinvf on the device vs the interpreter's Newton-refined erfinv:
    # within a few single-precision ulps
    diff(Graph("n", [("z", Rng.normal(F32, D.scalar("seed", I32), (1 << 16,)))]),
         [("seed", Value.of_list(I32, (), [99]))], tol=2e-6)


def test_s10_rows():
    dims = (1024, 4096)
    x = D.param("x", F32, dims)
    zero = D.const(F32, 0.0)
    g = Graph("rows", [("r", D.reduce_rows(D.add, zero, x)), ("p", D.scan_rows(D.add, zero, x))])
    v = Value.of_array(F32, dims, (np.arange(dims[0] * dims[1]) % 11 - 5.0).astype(np.float32))
    diff(g, [("x", v)], tol=1e-3)


def test_rows_short_and_max_bit_exact():
    x = D.param("x", F32, (300, 16))
    v = Value.of_array(F32, (300, 16), X.philox_normal(3, 300 * 16))
    g = Graph("r", [("m", D.reduce_rows(D.max, D.const(F32, -3e38), x)),
                    ("p", D.scan_rows(D.add, D.const(F32, 0.0), x))])
    diff(g, [("x", v)], tol=1e-5)
    diff(Graph("m", [("m", D.reduce_rows(D.max, D.const(F32, -3e38), x))]), [("x", v)], tol=0.0)


def test_s11_matmul():
    def mm(dt):
        a = D.param("a", dt, (256, 192))
        b = D.param("b", dt, (192, 128))
        return Graph("mm", [("c", D.matmul(a, b))])

    fa = lambda i: (i % 13) / 7.0 - 0.9  # noqa: E731
    fb = lambda i: (i % 17) / 5.0 - 1.6  # noqa: E731
    for dt, tol in ((F32, 1e-4), (F64, 1e-9)):
        a = Value.of_array(dt, (256, 192), np.array([fa(i) for i in range(256 * 192)], dtype=dt.np))
        b = Value.of_array(dt, (192, 128), np.array([fb(i) for i in range(192 * 128)], dtype=dt.np))
        diff(mm(dt), [("a", a), ("b", b)], tol=tol)


def test_matmul_transposed_operands_and_skinny():
    a = D.param("a", F64, (300, 5))
    b = D.param("b", F64, (300, 3))
    g = Graph("t", [("ata", D.matmul(D.transpose(a), a)), ("atb", D.matmul(D.transpose(a), b))])
    va = Value.of_array(F64, (300, 5), X.philox_normal(4, 1500, np.float64))
    vb = Value.of_array(F64, (300, 3), X.philox_normal(5, 900, np.float64))
    diff(g, [("a", va), ("b", vb)], tol=1e-9)
    # the split-K path (k >= 2048, m*n <= 32)
    n = 1 << 14
    a = D.param("a", F64, (n, 4))
    b = D.param("b", F64, (n, 1))
    g = Graph("t", [("xtx", D.matmul(D.transpose(a), a)), ("xty", D.matmul(D.transpose(a), b))])
    va = Value.of_array(F64, (n, 4), X.philox_normal(6, 4 * n, np.float64))
    vb = Value.of_array(F64, (n, 1), X.philox_normal(7, n, np.float64))
    diff(g, [("a", va), ("b", vb)], tol=1e-9)


@pytest.mark.parametrize("dt,m,n", [(F32, 300, 500), (F64, 1000, 37), (I32, 64, 4096 + 3)])
def test_materialised_transpose_tiles(dt, m, n):
    # a materialised Dsl.transpose of a buffer takes the tiled transpose
    # kernel: partial tiles on both axes, bit-exact for every dtype
    a = D.param("a", dt, (m, n))
    g = Graph("tr", [("t", D.transpose(a)), ("s", D.reduce(D.add, D.const(dt, 0), D.transpose(a)))])
    c = cuda.compile(g)
    assert "launch ccb_transpose_" in c.plan()
    x = (np.arange(m * n) % 1000 - 500).astype(dt.np).reshape(m, n)
    got = dict(cuda.run(c, [("a", Value.of_array(dt, (m, n), x))]))
    assert np.array_equal(got["t"].data.reshape(n, m), x.T)
    diff(g, [("a", Value.of_array(dt, (m, n), x))], tol=1e-3 if dt is F32 else 0.0)


def test_s12_scatter():
    n = 100_000
    idx = Value.of_array(I32, (n,), (np.arange(n) % 7).astype(np.int32))
    gi = Graph("hi", [("h", D.scatter_add(D.param("idx", I32, (n,)), D.param("s", I32, (n,)), (7,)))])
    diff(gi, [("idx", idx), ("s", Value.of_array(I32, (n,), np.ones(n, dtype=np.int32)))], tol=0.0)
    gf = Graph("hf", [("h", D.scatter_add(D.param("idx", I32, (n,)), D.param("s", F32, (n,)), (7,)))])
    diff(gf, [("idx", idx), ("s", Value.of_array(F32, (n,), ((np.arange(n) % 13) / 4.0).astype(np.float32)))], tol=1e-4)


def test_scatter_zipf_and_gather_config():
    n, bins = 1 << 20, 1 << 16
    idx = Value.of_array(I32, (n,), X.zipf_indices(4, n, bins))
    v = Value.of_array(F32, (n,), X.philox_uniform(3, n, np.float32))
    diff(X.scatter(n, bins), [("idx", idx), ("v", v)], tol=1e-4)
    tbl = 1 << 16
    gi = Value.of_array(I32, (n,), (X.philox_word0(4, n) % tbl).astype(np.int32))
    t = Value.of_array(F32, (tbl,), X.philox_normal(3, tbl))
    diff(X.gather(n, tbl), [("idx", gi), ("table", t)], tol=0.0)


@pytest.mark.parametrize("n,bins", [(3_000_007, 1 << 20), (12_345, 100), (5, 3)])
def test_scatter_i32_exact_ragged(n, bins):
    # I32 sums are exact in any order: the batched loop's ragged last batch,
    # privatised (low) and global (high) bins against a numpy histogram
    idx = X.zipf_indices(11, n, bins)
    s = (np.arange(n) % 5 - 1).astype(np.int32)
    g = Graph("sc", [("h", D.scatter_add(D.param("idx", I32, (n,)), D.param("s", I32, (n,)), (bins,)))])
    c = cuda.compile(g)
    got = dict(cuda.run(c, [("idx", Value.of_array(I32, (n,), idx)), ("s", Value.of_array(I32, (n,), s))]))["h"].data
    cuda.release(c)
    want = np.bincount(idx, weights=s.astype(np.int64), minlength=bins).astype(np.int64)
    assert np.array_equal(got.astype(np.int64), want)


@pytest.mark.parametrize("bins", [5, 3000, 1 << 16])
def test_scatter_f64_tiers(bins):
    # 8-byte values: 16 per-thread bins, 2048 block-private bins, the rest
    # global; sums of 2^20 F64 updates against an exact F64 histogram
    n = (1 << 20) + 17
    idx = X.zipf_indices(13, n, bins)
    v = np.random.default_rng(bins).random(n)
    g = Graph("s64", [("h", D.scatter_add(D.param("idx", I32, (n,)), D.param("s", F64, (n,)), (bins,)))])
    c = cuda.compile(g)
    got = dict(cuda.run(c, [("idx", Value.of_array(I32, (n,), idx)), ("s", Value.of_array(F64, (n,), v))]))["h"].data
    cuda.release(c)
    want = np.bincount(idx, weights=v, minlength=bins)
    assert np.all(np.abs(got - want) <= 1e-12 * (1 + np.abs(want)))


def test_out_of_bounds_scatter_is_reported():
    idx = D.param("idx", I32, (4,))
    c = cuda.compile(Graph("s", [("h", D.scatter_add(idx, D.param("s", I32, (4,)), (4,)))]))
    ones = Value.of_list(I32, (4,), [1, 1, 1, 1])
    with pytest.raises(R.CcbError):
        cuda.run(c, [("idx", Value.of_list(I32, (4,), [0, 1, 9, 2])), ("s", ones)])
    out = dict(cuda.run(c, [("idx", Value.of_list(I32, (4,), [3, 3, 1, 0])), ("s", ones)]))
    assert out["h"].to_list() == [1, 1, 0, 2]


def test_out_of_bounds_gather_is_reported():
    idx = D.param("idx", I32, (4,))
    t = D.param("t", F32, (4,))
    c = cuda.compile(Graph("g", [("g", D.gather(idx, t))]))
    with pytest.raises(R.CcbError):
        cuda.run(c, [("idx", Value.of_list(I32, (4,), [0, 1, 7, 2])), ("t", Value.of_list(F32, (4,), [1, 2, 3, 4]))])
    # the program stays usable after the error
    out = dict(cuda.run(c, [("idx", Value.of_list(I32, (4,), [3, 2, 1, 0])), ("t", Value.of_list(F32, (4,), [1, 2, 3, 4]))]))
    assert out["g"].to_list() == [4, 3, 2, 1]


def test_s13_greeks_f64_65536():
    diff(X.call_greeks(65536, F64), X.bs_inputs(F64, seed=7), tol=1e-6)


def test_s14_greeks_f32_2p20_vs_closed_form():
    b = GOLD["bs_greeks_f32_2p20_bands"]
    cf = X.analytic()
    c = cuda.compile(X.call_greeks(1 << 20, F32))
    o = cuda.run(c, X.bs_inputs(F32, seed=b["seed"]))
    assert abs(X.scalar_out(o, "price") - cf["price"]) <= b["price"]
    assert abs(X.scalar_out(o, "dprice/ds0") - cf["delta"]) <= b["delta"]
    assert abs(X.scalar_out(o, "dprice/dvol") - cf["vega"]) <= b["vega"]
    assert abs(X.scalar_out(o, "dprice/drate") - cf["rho"]) <= b["rho"]


def test_greeks_f32_vs_oracle():
    diff(X.call_greeks(1 << 18, F32), X.bs_inputs(F32, seed=42), tol=2e-4)


def test_reduce_scan_config_small():
    # F32: a parallel scan and the interpreter's sequential F32 fold round
    # differently, and near a zero crossing of the running sum a relative
    # band is meaningless, so F32 is judged against the exact (F64) prefix
    # sums of the same inputs: the device must be at least as accurate as the
    # reference's own sequential F32 fold. I32 is bit-exact.
    n = 1 << 20
    x = X.philox_normal(3, n)
    g = X.reduce_scan_flat(n, F32)
    got = dict(cuda.run(cuda.compile(g), [("x", Value.of_array(F32, (n,), x))]))
    seq = dict(interp.run(interp.compile(g), [("x", Value.of_array(F32, (n,), x))]))
    exact = np.cumsum(x.astype(np.float64))
    err_dev = float(np.max(np.abs(got["p"].data - exact)))
    err_seq = float(np.max(np.abs(seq["p"].data - exact)))
    assert err_dev <= max(err_seq, 1e-6 * float(np.max(np.abs(exact)))), (err_dev, err_seq)
    assert abs(got["s"].get(0) - exact[-1]) <= max(abs(seq["s"].get(0) - exact[-1]), 1e-5 * (1 + abs(exact[-1])))
    xi = Value.of_array(I32, (n,), (X.philox_word0(3, n) & 15).astype(np.int32))
    diff(X.reduce_scan_flat(n, I32), [("x", xi)], tol=0.0)


def test_reduce_scan_f32_full_size_vs_exact():
    # 2^28 F32 N(0,1) (the config), generated on the device by the
    # reference's own Rng.normal; sums and prefix sums against F64 exact.
    n = 1 << 28
    # (F64 normals cast to F32: the F32 generator itself yields a few +-inf at
    # this size, because (w + 0.5) * 2^-32 rounds to 1.0f for w >= 2^32 - 2^7.)
    gen = cuda.compile(Graph("gen", [("x", D.map(lambda z: D.cast(F32, z),
                                                 Rng.normal(F64, D.scalar("seed", I32), (n,))))]))
    x = dict(cuda.run(gen, [("seed", Value.of_list(I32, (), [3]))]))["x"].data
    cuda.release(gen)
    c = cuda.compile(X.reduce_scan_flat(n, F32))
    o = dict(cuda.run(c, [("x", Value.of_array(F32, (n,), x))]))
    cuda.release(c)
    exact = np.cumsum(x.astype(np.float64))
    scale = float(np.max(np.abs(exact)))
    assert abs(o["s"].get(0) - exact[-1]) <= 1e-5 * (1 + scale)
    assert float(np.max(np.abs(o["p"].data - exact))) <= 1e-5 * (1 + scale)


def test_reduce_scan_i32_full_size_exact():
    # 2^28 I32 U[0,16): exact integer sums, checked against exact host
    # arithmetic (the scan's last element is the total; prefix sums are
    # non-decreasing).
    n = 1 << 28
    gen = cuda.compile(Graph("gen", [("x", D.map(lambda w: D.bit_and(w, D.const(I32, 15)),
                                                 Rng.u32(D.scalar("seed", I32), (n,))))]))
    xi = dict(cuda.run(gen, [("seed", Value.of_list(I32, (), [3]))]))["x"].data
    cuda.release(gen)
    assert xi.min() >= 0 and xi.max() <= 15
    c = cuda.compile(X.reduce_scan_flat(n, I32))
    o = dict(cuda.run(c, [("x", Value.of_array(I32, (n,), xi))]))
    total = int(xi.astype(np.int64).sum())
    assert o["s"].get(0) == total
    p = o["p"].data
    assert int(p[-1]) == total
    assert np.array_equal(p, np.cumsum(xi, dtype=np.int64).astype(np.int32))
    cuda.release(c)


def test_s15_async_streams():
    n = 1 << 16
    g = X.saxpy(n, 2.0)
    c = cuda.compile_with(4, g)

    def inputs(k):
        return [("x", Value.of_array(F32, (n,), ((np.arange(n) + k) % 1000).astype(np.float32))),
                ("y", Value.of_array(F32, (n,), np.ones(n, dtype=np.float32)))]

    jobs = [(k, cuda.run_async(c, inputs(k))) for k in range(16)]
    for k, j in jobs:
        got = dict(cuda.wait(j))
        want = dict(cuda.run(c, inputs(k)))
        assert got["s"].get(0) == want["s"].get(0)
        assert np.array_equal(got["r"].data, want["r"].data)
    cuda.release(c)


def test_s16_resident_chain_sum():
    n = 4096
    chain = X.find("chain")
    gc = chain.graph()
    gs = X.reduce_flat(n, F32)
    cc = cuda.compile(gc)
    cs = cuda.compile(gs)
    rx = cuda.upload(dict(chain.inputs())["x"])
    r = dict(cuda.run_resident(cc, [("x", rx)]))["r"]
    s = dict(cuda.run_resident(cs, [("x", r)]))["s"]
    got = cuda.download(s).get(0)
    ri = dict(interp.run(interp.compile(gc), chain.inputs()))["r"]
    want = dict(interp.run(interp.compile(gs), [("x", ri)]))["s"].get(0)
    assert abs(got - want) <= 1e-5 * (1 + abs(want))
    for v in (rx, r, s):
        cuda.free_resident(v)
    cuda.release(cc)
    cuda.release(cs)


def test_resident_chain_reports_an_error_once():
    # device-resident runs copy no error word; the check after a chain of
    # them reports an out-of-range gather raised in any run, once
    idx = D.param("idx", I32, (4,))
    t = D.param("t", F32, (4,))
    c = cuda.compile(Graph("g", [("g", D.gather(idx, t))]))
    tv = cuda.upload(Value.of_list(F32, (4,), [1, 2, 3, 4]))
    good = cuda.upload(Value.of_list(I32, (4,), [3, 2, 1, 0]))
    bad = cuda.upload(Value.of_list(I32, (4,), [0, 9, 1, 0]))
    out = R.Buffer(16)
    order = [p_ for p_, _, _ in c.params]

    def run(ix):
        ptrs = {"idx": ix.buf.ptr, "t": tv.buf.ptr}
        cuda.run_device_ptrs(c, [ptrs[n_] for n_ in order], [out.ptr], None)

    for ix in (good, bad, good, good):
        run(ix)
    with pytest.raises(R.CcbError):
        cuda.check_device(c, None)
    cuda.check_device(c, None)  # reported once, then cleared
    run(good)
    cuda.check_device(c, None)
    got = np.empty(4, np.float32)
    out.download(got)
    assert got.tolist() == [4, 3, 2, 1]
    for v in (tv, good, bad):
        cuda.free_resident(v)
    out.free()
    cuda.release(c)


def test_graph_capture_replays_resident_runs():
    # two chained resident runs captured once, replayed with new data in the
    # same buffers; a captured gather error is reported by the check after
    # the replay; a flat scan is refused while capturing, and the stream is
    # usable afterwards
    n = 4096
    c = cuda.compile(X.saxpy(n, 2.0))
    s = c.lane_stream(0)
    x, y, r, t = R.Buffer(4 * n), R.Buffer(4 * n), R.Buffer(4 * n), R.Buffer(4)
    order = [p_ for p_, _, _ in c.params]
    outs = [nm for nm, _, _ in c.outputs]
    bufs = {"r": r.ptr, "s": t.ptr}

    def issue(xp, yp):
        ptrs = {"x": xp, "y": yp}
        cuda.run_device_ptrs(c, [ptrs[k] for k in order], [bufs[k] for k in outs], s)

    with R.Graph.capture(s) as g:
        issue(x.ptr, y.ptr)
        issue(r.ptr, y.ptr)  # r = 2 (2x + y) + y
    for k in range(3):
        xv = (np.arange(n) % 7 + k).astype(np.float32)
        yv = (np.arange(n) % 5).astype(np.float32)
        x.upload(xv)
        y.upload(yv)
        g.launch(s)
        cuda.check_device(c, s)
        got = np.empty(n, np.float32)
        r.download(got)
        assert np.array_equal(got, 2 * (2 * xv + yv) + yv)
    g.destroy()
    cuda.release(c)
    for b_ in (x, y, r, t):
        b_.free()

    gi = cuda.compile(Graph("g", [("g", D.gather(D.param("idx", I32, (4,)), D.param("t", F32, (4,))))]))
    tv = cuda.upload(Value.of_list(F32, (4,), [1, 2, 3, 4]))
    ix = cuda.upload(Value.of_list(I32, (4,), [0, 1, 2, 3]))
    o = R.Buffer(16)
    si = gi.lane_stream(0)
    ptrs = {"idx": ix.buf.ptr, "t": tv.buf.ptr}
    with R.Graph.capture(si) as gg:
        cuda.run_device_ptrs(gi, [ptrs[p_] for p_, _, _ in gi.params], [o.ptr], si)
    gg.launch(si)
    cuda.check_device(gi, si)
    ix.buf.upload(np.array([0, 7, 2, 3], np.int32))
    gg.launch(si)
    with pytest.raises(R.CcbError):
        cuda.check_device(gi, si)
    gg.destroy()
    for v in (tv, ix):
        cuda.free_resident(v)
    o.free()
    cuda.release(gi)

    cs = cuda.compile(X.scan_flat(1 << 20, F32))
    ss = cs.lane_stream(0)
    xb, ob = R.Buffer(4 << 20), R.Buffer(4 << 20)
    with pytest.raises(R.CcbError, match="flat scan"):
        with R.Graph.capture(ss):
            cuda.run_device_ptrs(cs, [xb.ptr], [ob.ptr], ss)
    R.check(R.lib().ccb_memset_d8(xb.ptr, 0, 4 << 20, ss))
    cuda.run_device_ptrs(cs, [xb.ptr], [ob.ptr], ss)
    cuda.check_device(cs, ss)
    xb.free()
    ob.free()
    cuda.release(cs)


@pytest.mark.parametrize("dt,rows,n", [(F64, 1000, 64), (F32, 300, 4096 + 5), (F64, 1, 100003)],
                         ids=["rows-warp-f64", "rows-block-f32", "flat-f64"])
def test_scan_store_fusion_matches_separate(dt, rows, n):
    # a map over a scan's output, run in the scan's stores, gives the bits of
    # the separate pass on the stored scan (no multiply feeding an add)
    shape = (n,) if rows == 1 else (rows, n)
    x = ((np.arange(rows * n) % 17 - 8) / 64.0).astype(dt.np).reshape(shape)
    px = D.param("x", dt, shape)
    scan = (lambda f, i, s: D.scan(f, i, s)) if rows == 1 else (lambda f, i, s: D.scan_rows(f, i, s))
    c = scan(D.add, D.const(dt, 0.0), px)

    def f(v):
        return D.mul(D.const(dt, 1.5), D.exp(v))

    def run(graph, ins):
        cc = cuda.compile(graph)
        try:
            return cc.plan(), {k: v.data for k, v in cuda.run(cc, ins)}
        finally:
            cuda.release(cc)

    ins = [("x", Value.of_array(dt, shape, x))]
    _, sc = run(Graph("s", [("c", c)]), ins)
    pc = D.param("c", dt, shape)
    _, sep = run(Graph("m", [("y", D.map(f, pc))]), [("c", Value.of_array(dt, shape, sc["c"].reshape(shape)))])
    plan, fused = run(Graph("fz", [("y", D.map(f, c))]), ins)
    assert "ccb_mapreduce_" not in plan
    assert np.array_equal(fused["y"], sep["y"])
    plan, both = run(Graph("fb", [("y", D.map(f, c)), ("c", c)]), ins)
    assert np.array_equal(both["c"], sc["c"]) and np.array_equal(both["y"], sep["y"])


def test_output_events_order_a_second_stream():
    # each output's event fires once the output is final: a second stream
    # that waits on it and copies the output sees the final values, for an
    # output of the first pass (a reduction) and one of the last (a scan);
    # all partial sums below 2^24, so exact in F32
    n = 1 << 20
    x = D.param("x", F32, (n,))
    g = Graph("ev", [("s", D.reduce(D.add, D.const(F32, 0.0), x)),
                     ("p", D.scan(D.add, D.const(F32, 0.0), D.map(lambda v: D.mul(v, D.const(F32, 2.0)), x)))])
    c = cuda.compile(g)
    st = c.lane_stream(0)
    other = R.Stream()
    xv = (np.arange(n) % 7).astype(np.float32)
    xb = R.Buffer(4 * n)
    xb.upload(xv)
    names = [nm for nm, _, _ in c.outputs]
    outs = {"s": R.Buffer(4), "p": R.Buffer(4 * n)}
    copies = {"s": R.Buffer(4), "p": R.Buffer(4 * n)}
    evs = [R.Event() for _ in names]
    for _ in range(3):
        cuda.run_device_ptrs_events(c, [xb.ptr], [outs[nm].ptr for nm in names], evs, st)
        for j, nm in enumerate(names):
            R.check(R.lib().ccb_stream_wait_event(other.h, evs[j].h))
            R.check(R.lib().ccb_memcpy_d2d(copies[nm].ptr, outs[nm].ptr, outs[nm].nbytes, other.h))
        other.synchronize()
        cuda.check_device(c, st)
        got_s, got_p = np.empty(1, np.float32), np.empty(n, np.float32)
        copies["s"].download(got_s)
        copies["p"].download(got_p)
        assert got_s[0] == float(xv.astype(np.float64).sum())
        assert np.array_equal(got_p, np.cumsum(2 * xv.astype(np.float64)).astype(np.float32))
    for b_ in list(outs.values()) + list(copies.values()) + [xb]:
        b_.free()
    other.destroy()
    cuda.release(c)


@pytest.mark.parametrize("dt,rows,n", [(F64, 1000, 64), (F32, 70, 100), (F64, 4096 + 3, 31), (F32, 33, 1000)],
                         ids=["f64-1000x64", "f32-70x100", "f64-4099x31", "f32-33x1000"])
def test_row_scan_transposed_store_matches_separate(dt, rows, n):
    # a row scan whose result is read only transposed writes the transpose
    # through shared-memory tiles: ragged row tiles (rows % 32) and column
    # chunks (n % 32), bare and with a map over the transpose, against the
    # scan stored and transposed by separate launches
    x = ((np.arange(rows * n) % 23 - 11) / 32.0).astype(dt.np).reshape(rows, n)
    px = D.param("x", dt, (rows, n))
    c = D.scan_rows(D.add, D.const(dt, 0.0), px)

    def f(v):
        return D.mul(D.const(dt, 1.5), D.exp(v))

    def run(graph, ins):
        cc = cuda.compile(graph)
        try:
            return cc.plan(), {k: v.data for k, v in cuda.run(cc, ins)}
        finally:
            cuda.release(cc)

    ins = [("x", Value.of_array(dt, (rows, n), x))]
    _, sc = run(Graph("s", [("c", c)]), ins)
    ref_t = sc["c"].reshape(rows, n).T.copy()
    _, sep = run(Graph("m", [("y", D.map(f, D.param("t", dt, (n, rows))))]), [("t", Value.of_array(dt, (n, rows), ref_t))])
    plan, tr = run(Graph("t", [("t", D.transpose(c))]), ins)
    assert plan.count("launch") == 1
    assert np.array_equal(tr["t"].reshape(n, rows), ref_t)
    plan, fused = run(Graph("fy", [("y", D.map(f, D.transpose(c)))]), ins)
    assert plan.count("launch") == 1
    assert np.array_equal(fused["y"], sep["y"])


@pytest.mark.parametrize("m,k,n", [(128, 16, 128), (300, 200, 260), (256, 1000, 384), (1024, 777, 512)],
                         ids=lambda v: str(v))
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)],
                         ids=["AB", "AtB", "ABt", "AtBt"])
def test_f32_product_register_blocked(m, k, n, ta, tb):
    # the CUDA-core product of 128 x 128 tiles (F32, matmul="f32"): ragged
    # tiles and k-steps, every operand order, within the F32 summation bound
    # k * 2^-24 * sum|a||b| of the F64 product of the same inputs
    rng = np.random.default_rng(m + 3 * k + 7 * n + 2 * ta + tb)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    pa = D.param("a", F32, (k, m) if ta else (m, k))
    pb = D.param("b", F32, (n, k) if tb else (k, n))
    g = Graph("mm128", [("c", D.matmul(D.transpose(pa) if ta else pa, D.transpose(pb) if tb else pb))])
    c = cuda.compile(g)
    assert "matmul_tiled128" in cuda.source(g)
    out = dict(cuda.run(c, [("a", Value.of_array(F32, pa.shape, np.ascontiguousarray(a.T if ta else a))),
                            ("b", Value.of_array(F32, pb.shape, np.ascontiguousarray(b.T if tb else b)))]))["c"]
    cuda.release(c)
    got = out.data.reshape(m, n).astype(np.float64)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    mag = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    assert np.all(np.abs(got - exact) <= (k + 2) * 2.0 ** -24 * mag + 1e-30)


def test_s5_pool_stable():
    n = 4096
    c = cuda.compile(X.saxpy(n, 2.0))
    live = R.live_count()
    for k in range(1, 51):
        x = Value.of_array(F32, (n,), (np.arange(n) + k).astype(np.float32))
        y = Value.of_array(F32, (n,), np.ones(n, dtype=np.float32))
        s = X.scalar_out(cuda.run(c, [("x", x), ("y", y)]), "s")
        expect = float(np.sum(2.0 * (np.arange(n) + k) + 1.0))
        assert abs(s - expect) <= expect * 1e-4
        assert R.live_count() == live
    cuda.release(c)


def test_s19_multi_same_device_and_counter_split():
    from cudacaml_b200 import multi as M
    n = 1 << 16
    saxpy = lambda n: X.saxpy(n, 2.0)  # noqa: E731
    x = Value.of_array(F32, (n,), np.arange(n, dtype=np.float32))
    y = Value.of_array(F32, (n,), np.ones(n, dtype=np.float32))
    c = cuda.compile(saxpy(n))
    single = dict(cuda.run(c, [("x", x), ("y", y)]))
    cuda.release(c)
    devices = [0, 0] if R.count() < 2 else [0, 1]
    for devs in ([0, 0], devices):
        t = M.Multi(devs, n, saxpy)
        per = t.run([("x", x), ("y", y)])
        assert np.array_equal(M.concat([dict(o)["r"] for o in per]).data, single["r"].data)
        t.release()
    # same seed, split counter range: D devices compute one device's paths
    m = 1 << 18
    g1 = cuda.compile(X.call_mc(m, F64))
    p1 = X.scalar_out(cuda.run(g1, X.bs_inputs(F64, seed=42)), "price")
    cuda.release(g1)
    t = M.Multi([0, 0, 0, 0], m, lambda k: X.call_mc(k, F64), counter_key="seed")
    per = t.run(X.bs_inputs(F64, seed=42))
    pm = M.mean_scalar([dict(o)["price"] for o in per])
    t.release()
    assert abs(pm - p1) <= 1e-9 * (1 + abs(p1))


def test_s19_multi_counter_split_multistep_grid():
    # (paths, steps) draws: the counter base is scaled by the steps per path,
    # so two programs draw exactly the unsplit program's words
    from cudacaml_b200 import multi as M
    n, steps = 1 << 12, 8
    key = D.scalar("seed", I32)
    words = lambda k: Graph("w", [("w", Rng.u32(key, (k, steps)))])  # noqa: E731
    c = cuda.compile(words(n))
    w1 = dict(cuda.run(c, [("seed", Value.of_list(I32, (), [42]))]))["w"].data
    cuda.release(c)
    t = M.Multi([0, 0], n, words, counter_key="seed")
    per = t.run([("seed", Value.of_list(I32, (), [42]))])
    t.release()
    assert np.array_equal(M.concat([dict(o)["w"] for o in per]).data, w1)
    g1 = cuda.compile(X.call_mc_paths(n, steps, F64))
    p1 = X.scalar_out(cuda.run(g1, X.bs_inputs(F64, seed=42)), "price")
    cuda.release(g1)
    t = M.Multi([0, 0], n, lambda k: X.call_mc_paths(k, steps, F64), counter_key="seed")
    pm = M.mean_scalar([dict(o)["price"] for o in t.run(X.bs_inputs(F64, seed=42))])
    t.release()
    assert abs(pm - p1) <= 1e-9 * (1 + abs(p1))


@pytest.mark.parametrize("n", [1, 4, 6143, 6144, 6145, 8192, 3 * 6144 + 5, 1 << 16, (1 << 20) + 7])
def test_flat_scan_tile_edges_i32_exact(n):
    # the staged scan's 6144-element tiles: ragged last tiles, one-tile and
    # multi-tile cases, bit-exact for I32 (wrapping add)
    x = (X.philox_word0(9, n) & 1023).astype(np.int32)
    g = X.scan_flat(n, I32)
    got = dict(cuda.run(cuda.compile(g), [("x", Value.of_array(I32, (n,), x))]))["p"].data
    assert np.array_equal(got, np.cumsum(x, dtype=np.int64).astype(np.int32))
    diff(g, [("x", Value.of_array(I32, (n,), x))], tol=0.0)


def test_flat_scan_max_and_repeat_runs():
    # a non-add combiner through the staged path, and repeated launches of one
    # program (epoch-tagged status words, counters re-armed by the kernel)
    n = 100_003
    x = X.philox_normal(12, n)
    v = D.param("x", F32, (n,))
    g = Graph("m", [("p", D.scan(D.max, D.const(F32, -3e38), v))])
    c = cuda.compile(g)
    for _ in range(3):
        got = dict(cuda.run(c, [("x", Value.of_array(F32, (n,), x))]))["p"].data
        assert np.array_equal(got, np.maximum.accumulate(x))


@pytest.mark.parametrize("n", [1 << 20, (1 << 20) + 32, 3 * 444 * 6144 + 96, (1 << 24) + 4096])
def test_flat_scan_large_i32_exact(n):
    # larger flat scans: a partial last tile, a few hundred tiles, thousands of
    # tiles; bit-exact I32, three launches of one program (epoch-tagged
    # statuses, re-armed counters)
    x = (X.philox_word0(13, n) & 1023).astype(np.int32)
    c = cuda.compile(X.scan_flat(n, I32))
    want = np.cumsum(x, dtype=np.int64).astype(np.int32)
    for _ in range(3):
        got = dict(cuda.run(c, [("x", Value.of_array(I32, (n,), x))]))["p"].data
        assert np.array_equal(got, want)


def test_flat_scan_large_max_f32():
    # a non-add combiner with a non-zero identity over many tiles
    n = (1 << 21) + 4064
    x = X.philox_normal(14, n)
    v = D.param("x", F32, (n,))
    c = cuda.compile(Graph("m", [("p", D.scan(D.max, D.const(F32, -3e38), v))]))
    got = dict(cuda.run(c, [("x", Value.of_array(F32, (n,), x))]))["p"].data
    assert np.array_equal(got, np.maximum.accumulate(x))


@pytest.mark.parametrize("basis", ["scaled3", "poly4"])
def test_lsm_drivers_match_interp(basis):
    # the generic driver over the CUDA backend, the resident CUDA driver and
    # the generic driver over the oracle: same normal equations every date,
    # same price (examples/lsm.ml:251-420)
    from cudacaml_b200 import lsm as L
    m = X.MARKET if basis == "scaled3" else L.BASELINE_MARKET
    n, ns = 4096, 16
    ti, tc, tr = [], [], []
    pi = L.Make(interp, n, ns, m, basis).price(11, trace=ti)
    pc = L.Make(cuda, n, ns, m, basis).price(11, trace=tc)
    res = L.CudaResident(n, ns, m, basis)
    pr = res.price(11, trace=tr)
    # the captured graph (first untraced call) and its replays: the same bits
    pg = [res.price(11) for _ in range(3)]
    assert res.graph is not None
    assert pg == [pr] * 3
    assert res.price(12) != pr  # a new seed reaches the replayed generator
    res.release()
    for (si, ai, bi), (sc, ac, bc), (sr, ar, br) in zip(ti, tc, tr):
        assert si == sc == sr
        for e, g in ((ai, ac), (bi, bc), (ai, ar), (bi, br)):
            assert np.all(np.abs(g - e) <= 1e-9 * (1 + np.abs(e))), (si, e, g)
    assert abs(pc - pi) <= 1e-9 * (1 + abs(pi))
    assert abs(pr - pi) <= 1e-9 * (1 + abs(pi))


def test_s17_lsm_vs_binomial():
    # S17: the resident driver against the binomial price (band 0.15), on the
    # reference market (3-term basis) and the BASELINE market (4-term basis)
    from cudacaml_b200 import lsm as L
    for m, basis in ((X.MARKET, "scaled3"), (L.BASELINE_MARKET, "poly4")):
        res = L.CudaResident(1 << 16, 50, m, basis)
        px = res.price(11)
        res.release()
        assert abs(px - L.binomial_american_put(m)) <= 0.15, (basis, px)
        assert px >= L.european_put(m) - 0.05
