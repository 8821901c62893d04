"""The TMA-staged row kernels (rows_staged: reduce_rows and scan_rows of a
4-byte buffer with rows of >= 1024 elements, a multiple of 4; selected with
CCB_ROWS_STAGED=1) against the oracle and against the default
register-streaming row kernels (CCB_ROWS_STAGED=0). Integer results bit-exact; F32 max bit-exact; F32 sums
within the reference's row band (S10's 1e-3). Row lengths cover one chunk,
a ragged last chunk and several chunks; row counts cover fewer rows than
CTAs and many rows per CTA; a caller pointer that is not 16-byte aligned
takes the in-kernel plain-load path."""
import os

import numpy as np
import pytest

from cudacaml_b200 import backend_cuda as cuda
from cudacaml_b200 import differential as Diff
from cudacaml_b200 import dsl as D
from cudacaml_b200 import examples as X
from cudacaml_b200 import runtime as R
from cudacaml_b200.ir import F32, I32, Graph, Value
from oracle import interp

pytestmark = pytest.mark.gpu


def rows_graph(dt, rows, n, op="add"):
    x = D.param("x", dt, (rows, n))
    zero = D.const(dt, 0.0 if dt is F32 else 0)
    red = D.reduce_rows(D.max, D.const(dt, -3e38 if dt is F32 else -(2 ** 31)), x) if op == "max" else \
        D.reduce_rows(D.add, zero, x)
    return Graph("rows", [("r", red), ("p", D.scan_rows(D.add, zero, x))])


def compiled(g, staged=True):
    old = os.environ.get("CCB_ROWS_STAGED")
    os.environ["CCB_ROWS_STAGED"] = "1" if staged else "0"
    try:
        return cuda.compile(g)
    finally:
        if old is None:
            del os.environ["CCB_ROWS_STAGED"]
        else:
            os.environ["CCB_ROWS_STAGED"] = old


@pytest.mark.parametrize("rows,n", [(7, 1024), (300, 4100), (5, 12288 + 4), (2000, 4096)])
def test_i32_rows_exact_vs_oracle_and_unstaged(rows, n):
    g = rows_graph(I32, rows, n)
    v = Value.of_array(I32, (rows, n), ((np.arange(rows * n) * 7) % 23 - 11).astype(np.int32))
    c = compiled(g)
    assert "rowsstaged" in c.plan(), c.plan()
    got = dict(cuda.run(c, [("x", v)]))
    cuda.release(c)
    want = dict(interp.run(interp.compile(g), [("x", v)]))
    c0 = compiled(g, staged=False)
    assert "rowsstaged" not in c0.plan()
    plain = dict(cuda.run(c0, [("x", v)]))
    cuda.release(c0)
    for k in ("r", "p"):
        assert np.array_equal(got[k].data, want[k].data), k
        assert np.array_equal(got[k].data, plain[k].data), k


def test_f32_rows_max_exact_and_sum_band():
    rows, n = 1000, 4096 + 1024
    v = Value.of_array(F32, (rows, n), X.philox_normal(5, rows * n))
    g = rows_graph(F32, rows, n, op="max")
    os.environ["CCB_ROWS_STAGED"] = "1"
    try:
        assert "rowsstaged" in cuda.lower_info(g)["plan"]
        err = Diff.check(interp, cuda, Graph("m", [("m", g.outputs[0][1])]), [("x", v)], tolerance=0.0)
        assert err is None, err
        err = Diff.check(interp, cuda, rows_graph(F32, rows, n), [("x", v)], tolerance=1e-3)
        assert err is None, err
    finally:
        del os.environ["CCB_ROWS_STAGED"]


def test_unaligned_caller_pointer_takes_plain_loads():
    rows, n = 64, 2048
    g = rows_graph(I32, rows, n)
    host = ((np.arange(rows * n) * 5) % 17).astype(np.int32)
    c = compiled(g)
    big = R.Buffer(4 * rows * n + 16)
    r_out, p_out = R.Buffer(4 * rows), R.Buffer(4 * rows * n + 16)
    try:
        R.check(R.lib().ccb_memcpy_h2d(big.ptr + 4, host.ctypes.data, host.nbytes, None))
        R.check(R.lib().ccb_stream_synchronize(None))
        names = [nm for nm, _, _ in c.outputs]
        outs = {"r": r_out.ptr, "p": p_out.ptr + 4}
        cuda.run_device_ptrs(c, [big.ptr + 4], [outs[nm] for nm in names], None)
        cuda.check_device(c, None)
        got_r = np.empty(rows, np.int32)
        got_p = np.empty(rows * n, np.int32)
        R.check(R.lib().ccb_memcpy_d2h(got_r.ctypes.data, r_out.ptr, 4 * rows, None))
        R.check(R.lib().ccb_memcpy_d2h(got_p.ctypes.data, p_out.ptr + 4, 4 * rows * n, None))
        R.check(R.lib().ccb_stream_synchronize(None))
    finally:
        for b in (big, r_out, p_out):
            b.free()
        cuda.release(c)
    m = host.reshape(rows, n).astype(np.int64)
    assert np.array_equal(got_r, m.sum(axis=1).astype(np.int32))
    assert np.array_equal(got_p, np.cumsum(m, axis=1).astype(np.int32).reshape(-1))
