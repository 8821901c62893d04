"""GPU tests of the runtime half of the C-ABI: pinned host memory (the
reference's S18), the bounded device waits of the skeletons, the launch
entry point's argument check, and Multi over distinct GPUs with its NCCL
recombination (S19's [0;1] case, test/system/test_system.ml:210-224).

The bounded-wait tests make each wait run out the way a stuck predecessor
would leave it: a flag that nothing sets. The kernels are compiled from the
shipped skeleton header with small poll limits, wait, give up, raise their
error bit and return; the context stays usable, which the tests check by
running a program afterwards. No kernel here faults, traps or hangs.
"""
import ctypes
import time

import numpy as np
import pytest

from cudacaml_b200 import backend_cuda as cuda
from cudacaml_b200 import examples as X
from cudacaml_b200 import runtime as R
from cudacaml_b200.ir import F32, F64, Value

pytestmark = pytest.mark.gpu

ERR_LOOKBACK, ERR_TMA, ERR_TC_WAIT = 4, 8, 16


def test_s18_pinned_round_trip_and_bandwidth():
    """64 MiB through page-locked host memory and back, bit for bit, with the
    pinned and pageable upload rates printed (test_system.ml:196-209; the
    allocator is lib/runtime/pinned.ml:76-108)."""
    n = 16 * 1024 * 1024
    src = R.pinned_empty((n,), np.float32)
    dst = R.pinned_empty((n,), np.float32)
    assert not dst.any()  # ccb_host_alloc zero-fills, as Pinned.alloc does
    src[:] = (np.arange(n) & 1023).astype(np.float32)
    b = R.Buffer(4 * n)
    try:
        b.upload(src)  # first touch of the buffer, untimed
        t0 = time.perf_counter()
        b.upload(src)
        tp = time.perf_counter() - t0
        b.download(dst)
        pageable = np.zeros(n, np.float32)
        t0 = time.perf_counter()
        b.upload(pageable)
        tg = time.perf_counter() - t0
    finally:
        b.free()
    print(f"    H->D pinned {4 * n / tp / 1e9:.1f} GB/s   pageable {4 * n / tg / 1e9:.1f} GB/s")
    assert np.array_equal(src.view(np.uint32), dst.view(np.uint32))


WAIT_SRC = r"""
#define CCB_LOOKBACK_SPIN_LIMIT 64u
#define CCB_MBAR_SPIN_LIMIT 256u
#include "ccb_skel.cuh"

// The flat scan's look-back interface over I32 add.
struct LbI32 {
  typedef int T;
  struct P {
    unsigned long long* status;
    unsigned* err;
    unsigned epoch;
  };
  static __device__ __forceinline__ T identity() { return 0; }
  static __device__ __forceinline__ T combine(T a, T b) { return a + b; }
};

// Tile 1 of launch epoch 1 whose tile 0 never publishes: status[0] keeps
// epoch 0, so no poll can fold it.
extern "C" __global__ void wait_lookback(unsigned long long* status, unsigned* err, int* out) {
  LbI32::P p{status, err, 1u};
  const int v = ccb::lookback<LbI32>(p, 1u, 5, threadIdx.x & 31);
  if (threadIdx.x == 0) out[0] = v;
}
extern "C" __global__ void wait_walk_back(unsigned long long* status, unsigned* err, int* out) {
  LbI32::P p{status, err, 1u};
  const int v = ccb::walk_back<LbI32>(p, 1u, 5, threadIdx.x & 31);
  if (threadIdx.x == 0) out[0] = v;
}
// A bulk-copy barrier whose phase nothing completes.
extern "C" __global__ void wait_bulk_copy(unsigned* err) {
  __shared__ __align__(8) unsigned long long bar;
  if (threadIdx.x == 0) {
    ccb::mbar_init(&bar, 1);
    ccb::mbar_fence_init();
  }
  __syncthreads();
  ccb::mbar_wait(&bar, 0u, err);
}
// The tensor-core pipeline's wait on a stage barrier nothing arrives on.
extern "C" __global__ void wait_tc_pipeline(unsigned* err) {
  __shared__ __align__(8) unsigned long long bar;
  if (threadIdx.x == 0) {
    ccb::mbar_init(&bar, 1);
    ccb::mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) ccb::tc::wait(&bar, 0u, err);
}
"""


def _module(src, name):
    L = R.lib()
    mod = ctypes.c_void_p()
    log = ctypes.c_void_p()
    rc = L.ccb_module_compile(src.encode(), name.encode(), ctypes.byref(mod), ctypes.byref(log))
    text = ctypes.string_at(log.value).decode() if log.value else ""
    if log.value:
        L.ccb_free_string(log)
    assert rc == 0, (L.ccb_last_error().decode(), text)
    return mod.value


def _function(mod, name):
    fn = ctypes.c_void_p()
    R.check(R.lib().ccb_module_get_function(mod, name.encode(), ctypes.byref(fn)))
    return fn.value


def _launch(fn, threads, *ptrs):
    vals = [ctypes.c_void_p(p) for p in ptrs]
    args = (ctypes.c_void_p * len(vals))(*[ctypes.cast(ctypes.byref(v), ctypes.c_void_p) for v in vals])
    return R.lib().ccb_launch(fn, 1, 1, 1, threads, 1, 1, 0, None, args, len(vals))


@pytest.mark.parametrize("kernel,bit", [("wait_lookback", ERR_LOOKBACK), ("wait_walk_back", ERR_LOOKBACK),
                                        ("wait_bulk_copy", ERR_TMA), ("wait_tc_pipeline", ERR_TC_WAIT)])
def test_bounded_wait_gives_up_and_reports(kernel, bit):
    R.set_device(0)
    L = R.lib()
    mod = _module(WAIT_SRC, "waits")
    status, err, out = R.Buffer(16), R.Buffer(4), R.Buffer(4)
    try:
        for b in (status, err, out):
            R.check(L.ccb_memset_d8(b.ptr, 0, b.nbytes, None))
        ptrs = (status.ptr, err.ptr, out.ptr) if "walk" in kernel or "lookback" in kernel else (err.ptr,)
        R.check(_launch(_function(mod, kernel), 32, *ptrs))
        R.check(L.ccb_stream_synchronize(None))
        word = np.empty(1, np.uint32)
        err.download(word)
        assert int(word[0]) == bit, (kernel, int(word[0]))
        if len(ptrs) == 3:
            got = np.empty(1, np.int32)
            out.download(got)
            assert int(got[0]) == 0  # a walk that gives up returns the identity
    finally:
        for b in (status, err, out):
            b.free()
        R.check(L.ccb_module_unload(mod))
    # the context is still usable
    n = 1000
    c = cuda.compile(X.saxpy(n, 2.0))
    x = Value.of_array(F32, (n,), np.arange(n, dtype=np.float32))
    y = Value.of_array(F32, (n,), np.ones(n, np.float32))
    r = dict(cuda.run(c, [("x", x), ("y", y)]))["r"].data
    cuda.release(c)
    assert np.array_equal(r, 2.0 * np.arange(n, dtype=np.float32) + 1.0)


def test_launch_checks_the_argument_count():
    R.set_device(0)
    L = R.lib()
    mod = _module(WAIT_SRC, "waits")
    try:
        fn = _function(mod, "wait_lookback")
        buf = R.Buffer(16)
        try:
            assert _launch(fn, 32, buf.ptr, buf.ptr) == 1  # three parameters, two given
            assert "takes 3 arguments, 2 given" in L.ccb_last_error().decode()
        finally:
            buf.free()
    finally:
        R.check(L.ccb_module_unload(mod))


def test_s19_multi_distinct_devices_nccl():
    """Multi over GPUs 0 and 1: the counter-split Greeks recombined by one NCCL
    all-reduce equal the single-device run up to summation order, and the
    row-split MLP gradients all-reduced on the devices equal the full batch's."""
    if R.count() < 2:
        pytest.skip("one device: [0;1] not run")
    from cudacaml_b200 import multi as M
    m = 1 << 20
    g = X.call_greeks(m, F64)
    c = cuda.compile(g)
    single = {k: float(v.data[0]) for k, v in cuda.run(c, X.bs_inputs(F64, seed=42))}
    cuda.release(c)
    t = M.Multi([0, 1], m, lambda k: X.call_greeks(k, F64), counter_key="seed")
    names = list(single)
    got = t.allreduce_mean(names, X.bs_inputs(F64, seed=42))
    host = {k: M.mean_scalar([dict(o)[k] for o in t.run(X.bs_inputs(F64, seed=42))]) for k in names}
    t.release()
    for k in names:
        assert abs(got[k] - single[k]) <= 1e-9 * (1 + abs(single[k])), (k, got[k], single[k])
        assert abs(host[k] - got[k]) <= 1e-12 * (1 + abs(got[k])), (k, host[k], got[k])

    bsz, din, hid, dout = 512, 256, 512, 256
    rng = np.random.default_rng(9)
    shapes = {"X": (bsz, din), "W1": (din, hid), "W2": (hid, dout), "T": (bsz, dout)}
    ins = [(nm, Value.of_array(F32, shapes[nm], rng.standard_normal(shapes[nm]).astype(np.float32) * 0.1))
           for nm in ("X", "W1", "W2", "T")]
    c = cuda.compile(X.mlp_step(bsz, din, hid, dout), matmul="tf32")
    want = dict(cuda.run(c, ins))
    cuda.release(c)
    t = M.Multi([0, 1], bsz, lambda k: X.mlp_step(k, din, hid, dout), split=["X", "T"], matmul="tf32")
    got = t.allreduce_sum(["loss", "dloss/dW1", "dloss/dW2"], ins)
    t.release()
    for name, v in got.items():
        e = want[name].data.astype(np.float64)
        rel = np.max(np.abs(v.data.astype(np.float64) - e)) / np.max(np.abs(e))
        assert rel <= 1e-5, (name, rel)  # same TF32 operands; only the F32 summation order differs
