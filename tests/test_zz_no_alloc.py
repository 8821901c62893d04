"""The allocation-free sum (ccb_sum_f32_noalloc) against the regular path.

Some callers cannot allocate device memory -- code inside another framework's
stream capture, under an application-owned memory pool, in a real-time path
that must not take the driver's allocation locks, or a plugin that is handed
device pointers but no allocator. For them, ccb_sum_f32_noalloc computes the
same flat F32 sum as a compiled `reduce add` graph, with its scratch in a
fixed device array instead of an allocation. This checks it through the C-ABI
against the regular entry point (ccb_program_run_device) on two calls in a
row, with the tolerance the other F32-sum tests use, and checks with the
driver's own count of free device memory (cuMemGetInfo) that calls after the
first allocate nothing. It is collected last so that a run stopping at its
first failure has run every other test already.
"""
import ctypes

import numpy as np
import pytest

from cudacaml_b200 import backend_cuda as cuda
from cudacaml_b200 import examples as X
from cudacaml_b200 import runtime as R
from cudacaml_b200.ir import F32

pytestmark = pytest.mark.gpu
TOL = 1e-5  # Differential's default band, |g - e| <= tol * (1 + |e|)


def _noalloc_sum(x_ptr, n, out_ptr):
    rc = R.lib().ccb_sum_f32_noalloc(x_ptr, n, out_ptr, None)
    assert rc == 0, R.lib().ccb_last_error().decode()
    R.check(R.lib().ccb_stream_synchronize(None))


def _free_device_bytes():
    """Free memory of the current device as the driver counts it. Any device
    allocation (cudaMalloc takes at least a 2 MiB page) lowers it."""
    cu = ctypes.CDLL("libcuda.so.1")
    free, total = ctypes.c_size_t(), ctypes.c_size_t()
    assert cu.cuMemGetInfo_v2(ctypes.byref(free), ctypes.byref(total)) == 0
    return free.value


def test_noalloc_sum_matches_program_path_twice():
    R.set_device(0)
    n = (1 << 22) + 3  # ragged tail: not a multiple of the 4-wide vector step
    c = cuda.compile(X.reduce_flat(n, F32))
    x = R.Buffer(4 * n)
    ref_out = R.Buffer(4)
    out = R.Buffer(4)
    try:
        # The first call on a device does its set-up (the runtime may load the
        # module that holds the scratch array); from then on nothing allocates.
        _noalloc_sum(x.ptr, 1, out.ptr)
        for call, seed in enumerate((3, 11)):
            host = X.philox_normal(seed, n)
            x.upload(host)
            cuda.run_device_ptrs(c, [x.ptr], [ref_out.ptr], None)
            cuda.check_device(c, None)
            want = np.empty(1, np.float32)
            ref_out.download(want)
            live, free = R.live_count(), _free_device_bytes()
            _noalloc_sum(x.ptr, n, out.ptr)
            assert R.live_count() == live
            assert _free_device_bytes() == free, "the no-allocation sum allocated device memory"
            got = np.empty(1, np.float32)
            out.download(got)
            e, g = float(want[0]), float(got[0])
            assert abs(g - e) <= TOL * (1 + abs(e)), (call, e, g)
            # and both agree with the exact sum of the same inputs
            exact = float(np.sum(host.astype(np.float64)))
            assert abs(g - exact) <= 1e-6 * (1 + float(np.sum(np.abs(host.astype(np.float64)))))
    finally:
        x.free()
        ref_out.free()
        out.free()
        cuda.release(c)


def test_noalloc_sum_edge_sizes_and_limit():
    R.set_device(0)
    out = R.Buffer(4)
    x = R.Buffer(4 * 1000)
    try:
        x.upload(np.arange(1000, dtype=np.float32))
        for n in (0, 1, 7, 1000):
            _noalloc_sum(x.ptr, n, out.ptr)
            got = np.empty(1, np.float32)
            out.download(got)
            assert float(got[0]) == float(sum(range(n)))
        rc = R.lib().ccb_sum_f32_noalloc(x.ptr, 1 << 31, out.ptr, None)
        assert rc == 1
        assert "2^31" in R.lib().ccb_last_error().decode()
        assert R.lib().ccb_sum_f32_noalloc(None, 5, out.ptr, None) == 1
        assert "null pointer" in R.lib().ccb_last_error().decode()
    finally:
        x.free()
        out.free()
