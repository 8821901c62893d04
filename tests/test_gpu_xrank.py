"""The cross-rank scalar sum over peer memory (ccb_xrank_sum, multi.PeerSum):
one rank alone returns its own values for every dtype and every epoch; a
peer that never publishes makes the bounded wait give up, raise its error
bit and leave the output untouched (the flag nothing sets: both mailboxes
live on one GPU and no second kernel runs); two GPUs driven from one process
sum to the same bits on both. Ranks never share a GPU here."""
import ctypes

import numpy as np
import pytest

from cudacaml_b200 import multi as M
from cudacaml_b200 import runtime as R

pytestmark = pytest.mark.gpu

DTYPES = [(np.float32, 0), (np.float64, 1), (np.int32, 2), (np.int64, 3)]


def test_single_rank_is_identity_for_every_dtype():
    R.set_device(0)
    ps = M.PeerSum(1, 0, lambda h: [h])
    try:
        for npdt, code in DTYPES:
            vals = (np.arange(1, 9) * 3 - 7).astype(npdt)
            src, dst = R.Buffer(vals.nbytes), R.Buffer(vals.nbytes)
            src.upload(vals)
            for _ in range(3):  # successive epochs reuse the two mailbox halves
                ps.sum(src.ptr, dst.ptr, 8, code, None)
                ps.check(None)
                got = np.empty(8, npdt)
                dst.download(got)
                assert np.array_equal(got, vals)
            src.free()
            dst.free()
    finally:
        ps.close()


def test_missing_peer_gives_up_and_reports():
    R.set_device(0)
    L = R.lib()
    size = ctypes.c_size_t()
    R.check(L.ccb_xrank_mailbox_bytes(2, ctypes.byref(size)))
    mine, theirs, err, buf = R.Buffer(size.value), R.Buffer(size.value), R.Buffer(4), R.Buffer(32)
    try:
        for b in (mine, theirs, err):
            R.check(L.ccb_memset_d8(b.ptr, 0, b.nbytes, None))
        buf.upload(np.array([1.0, 2.0, 3.0, 4.0]))
        boxes = (ctypes.c_void_p * 2)(mine.ptr, theirs.ptr)
        # rank 0 of 2: rank 1 never writes into `mine`
        R.check(L.ccb_xrank_sum(buf.ptr, buf.ptr, 4, 1, 2, 0, boxes, 1, err.ptr, None))
        R.check(L.ccb_stream_synchronize(None))
        w = np.empty(1, np.uint32)
        err.download(w)
        assert int(w[0]) == M.PeerSum.ERR_XRANK
        got = np.empty(4)
        buf.download(got)
        assert np.array_equal(got, [1.0, 2.0, 3.0, 4.0])
    finally:
        for b in (mine, theirs, err, buf):
            b.free()
    # the context is still usable
    x = R.Buffer(4)
    x.upload(np.array([5], np.int32))
    x.free()


def test_argument_checks():
    R.set_device(0)
    L = R.lib()
    b = R.Buffer(64)
    boxes = (ctypes.c_void_p * 1)(b.ptr)
    try:
        for args in ((0, 1, 1, 0, 1), (9, 1, 1, 0, 1), (1, 7, 1, 0, 1), (1, 1, 17, 0, 1), (1, 1, 1, 1, 1),
                     (1, 1, 1, 0, 0)):
            count, dtype, nranks, rank, epoch = args
            assert L.ccb_xrank_sum(b.ptr, b.ptr, count, dtype, nranks, rank, boxes, epoch, b.ptr, None) == 1, args
    finally:
        b.free()


def test_two_gpus_in_one_process_sum_to_the_same_bits():
    if R.count() < 2:
        pytest.skip("one device")
    ranks = M.PeerSum.in_process([0, 1])
    vals = [np.array([0.1, 1e16, -1e16, 3.0], np.float64), np.array([0.2, 1.0, 1.0, -3.0], np.float64)]
    bufs, streams = [], []
    try:
        for d in (0, 1):
            with R.with_device(d):
                b = R.Buffer(32)
                b.upload(vals[d])
                bufs.append(b)
        for step in range(4):
            for d in (0, 1):
                with R.with_device(d):
                    ranks[d].sum(bufs[d].ptr, bufs[d].ptr, 4, 1, None)
            got = []
            for d in (0, 1):
                with R.with_device(d):
                    ranks[d].check(None)
                    h = np.empty(4)
                    bufs[d].download(h)
                    got.append(h)
            assert np.array_equal(got[0].view(np.uint64), got[1].view(np.uint64)), got
            want = vals[0] + vals[1]  # rank order: rank 0's value first
            assert np.array_equal(got[0], want)
            vals = [want, want]
    finally:
        for d, b in enumerate(bufs):
            with R.with_device(d):
                b.free()
        for d, ps in enumerate(ranks):
            with R.with_device(d):
                ps.close()
