"""Sharded Monte-Carlo programs on the GPU (include/ccb.h, sharded programs).

One GPU: a run before the mailboxes are bound is refused on the host; a rank
whose peer never runs gives up its bounded wait, reports it through the
program's error word and leaves its outputs untouched (both mailboxes live on
one GPU and no second rank runs: the flag nothing sets), and the context stays
usable. Two GPUs (skipped on one): Multi(sharded=True) over devices 0 and 1
gives the same bits on both devices, run after run, within 1e-12 of the
unsplit single-device program in F64 (only the summation order differs) and
within the reference's F32 band of the oracle in F32. Ranks never share a GPU
here."""
import numpy as np
import pytest

from cudacaml_b200 import backend_cuda as B
from cudacaml_b200 import examples as X
from cudacaml_b200 import multi as M
from cudacaml_b200 import runtime as R
from cudacaml_b200.ir import F32, F64
from oracle import interp

pytestmark = pytest.mark.gpu


def _resident(c, dt):
    ins = {"s0": np.array([100.0], dt.np), "vol": np.array([0.2], dt.np), "rate": np.array([0.05], dt.np),
           "seed": np.array([42], np.int32)}
    bufs = []
    for name, _, _ in c.params:
        b = R.Buffer(ins[name].nbytes)
        b.upload(ins[name])
        bufs.append(b)
    outs = [R.Buffer(dt.size_in_bytes) for _ in c.outputs]
    return bufs, outs


def test_run_before_bind_is_refused():
    R.set_device(0)
    c = B.compile_on(0, X.call_greeks(1 << 12, F64), shard=(0, 2))
    ins, outs = _resident(c, F64)
    try:
        with pytest.raises(ValueError, match="bind_peers"):
            B.run_device_ptrs(c, [b.ptr for b in ins], [b.ptr for b in outs], None)
    finally:
        for b in ins + outs:
            b.free()
        B.release(c)


def test_missing_peer_gives_up_and_reports():
    R.set_device(0)
    c = B.compile_on(0, X.call_greeks(1 << 16, F64), shard=(0, 2))
    nb = B.mailbox_bytes(c)
    mine, theirs = R.Buffer(nb), R.Buffer(nb)
    ins, outs = _resident(c, F64)
    try:
        for b in (mine, theirs):
            R.check(R.lib().ccb_memset_d8(b.ptr, 0, nb, None))
        for b in outs:
            b.upload(np.array([-7.0]))
        R.check(R.lib().ccb_stream_synchronize(None))
        B.bind_peers(c, [mine.ptr, theirs.ptr])  # rank 1 never runs
        B.run_device_ptrs(c, [b.ptr for b in ins], [b.ptr for b in outs], None)
        with pytest.raises(R.CcbError, match="cross-rank combine gave up"):
            B.check_device(c, None)
        for b in outs:  # the scalar tails were skipped
            h = np.empty(1)
            b.download(h)
            assert h[0] == -7.0
        # the context is still usable, and the program's error word was cleared
        x = R.Buffer(8)
        x.upload(np.array([3.0]))
        x.free()
    finally:
        for b in ins + outs + [mine, theirs]:
            b.free()
        B.release(c)


def _two():
    if R.count() < 2:
        pytest.skip("one device: ranks need distinct GPUs")


def test_two_gpus_same_bits_and_unsplit_result_f64():
    _two()
    n = 1 << 20
    c = B.compile(X.call_greeks(n, F64))
    single = {k: float(v.data[0]) for k, v in B.run(c, X.bs_inputs(F64, seed=42))}
    B.release(c)
    t = M.Multi([0, 1], n, lambda k: X.call_greeks(k, F64), sharded=True)
    try:
        assert all(s.num_launches() == 1 for s in t.slots)
        first = None
        for _ in range(3):  # epochs alternate the two mailbox halves
            per_dev = [{k: v.data.copy() for k, v in o} for o in t.run(X.bs_inputs(F64, seed=42))]
            for k in single:
                a, b = per_dev[0][k], per_dev[1][k]
                assert np.array_equal(a.view(np.uint64), b.view(np.uint64)), (k, a, b)
                assert abs(float(a[0]) - single[k]) <= 1e-12 * (1 + abs(single[k])), (k, float(a[0]), single[k])
            if first is None:
                first = per_dev[0]
            else:
                for k in single:
                    assert np.array_equal(first[k], per_dev[0][k])
        got = t.allreduce_mean(list(single), X.bs_inputs(F64, seed=42))
        for k in single:
            assert got[k] == float(first[k][0])
    finally:
        t.release()


def test_two_gpus_f32_against_the_oracle():
    _two()
    n = 1 << 18
    g = X.call_greeks(n, F32)
    want = {k: float(v.data[0]) for k, v in interp.run(interp.compile(g), X.bs_inputs(F32, seed=42))}
    t = M.Multi([0, 1], n, lambda k: X.call_greeks(k, F32), sharded=True)
    try:
        got = dict(t.run(X.bs_inputs(F32, seed=42))[1])
    finally:
        t.release()
    for k, e in want.items():
        v = float(got[k].data[0])
        assert abs(v - e) <= 2e-4 * (1 + abs(e)), (k, v, e)  # the F32 Greeks band of the single-device test
