"""Sharded programs on the CPU (no device): the wire option, the slices the
lowering gives each rank (they partition the index space, so the ranks draw
exactly the unsplit program's Philox counters), the sm_100a compile of a
sharded pass, the programs that cannot be sharded, and the argument checks
of the C-ABI entry points and of Multi(sharded=True)."""
import ctypes
import re

import pytest

from cudacaml_b200 import backend_cuda as B
from cudacaml_b200 import dsl as D
from cudacaml_b200 import examples as X
from cudacaml_b200 import multi as M
from cudacaml_b200 import rng as Rng
from cudacaml_b200 import runtime as R
from cudacaml_b200.ir import F32, F64, I32, Graph
from cudacaml_b200.wire import to_wire

from test_lower_abi import nvrtc_ok


def _slice(src):
    lo = int(re.search(r"XLO = (-?\d+)LL", src).group(1))
    hi = int(re.search(r"XHI = (-?\d+)LL", src).group(1))
    w, r = (int(x) for x in re.search(r"XWORLD = (\d+), XRANK = (\d+)", src).groups())
    return lo, hi, r, w


def test_wire_option():
    g = X.call_greeks(1 << 10, F64)
    assert "opt shard 3 8\n" in to_wire(g, shard=(3, 8))
    assert "opt shard" not in to_wire(g, shard=(0, 1))  # one rank: the plain program
    for bad in ((2, 2), (-1, 2), (0, 0), (0, 33)):
        with pytest.raises(ValueError):
            to_wire(g, shard=bad)


@pytest.mark.parametrize("n,world", [(1 << 28, 8), (1 << 28, 2), (1000003, 3), (7, 4)])
def test_rank_slices_partition_the_index_space(n, world):
    covered = 0
    for r in range(world):
        src = B.source(X.call_greeks(n, F64), shard=(r, world))
        lo, hi, rank, w = _slice(src)
        assert (rank, w) == (r, world)
        assert lo == covered and hi >= lo
        covered = hi
    assert covered == n
    if n % world == 0:  # the counters Multi's split gives rank r
        assert [_slice(B.source(X.call_greeks(n, F64), shard=(r, world)))[:2] for r in range(world)] == \
            [(b, b + p) for b, p in (M.path_range(n, world, r) for r in range(world))]


def test_sharded_pass_is_one_launch_and_compiles_for_sm100a():
    for dt in (F64, F32):
        info = B.lower_info(X.call_greeks(1 << 28, dt), shard=(5, 8))
        assert info["launches"] == 1, info["plan"]
        src = info["source"]
        assert "unsigned long long* xmb[8];" in src and "unsigned long long xepoch;" in src
        assert nvrtc_ok(src, "greeks_shard") > 0
    # an MC estimator with an I32 reduction (max) shards too: the combiner is the pass's own
    n = 1 << 12
    w = D.map(lambda v: D.bit_and(v, D.const(I32, 1023)), Rng.u32(D.scalar("seed", I32), (n,)))
    g = Graph("umax", [("m", D.reduce(D.max, D.const(I32, -1), w))])
    assert nvrtc_ok(B.lower_info(g, shard=(1, 2))["source"], "umax_shard") > 0


@pytest.mark.parametrize("graph,why", [
    (lambda: X.saxpy(1 << 12, 2.0), "stores elements"),
    (lambda: X.reduce_flat(1 << 12, F32), "loads elements by index"),
    (lambda: X.call_mc_paths(64, 16, F32), "scan"),
    (lambda: X.rows(64, 128), "scan"),
])
def test_programs_that_cannot_be_sharded(graph, why):
    with pytest.raises(R.CcbError) as e:
        B.lower_info(graph(), shard=(0, 2))
    assert e.value.code == 7 and why in str(e.value)


def test_two_reduction_passes_are_refused():
    n = 1 << 10
    u = Rng.uniform(F64, D.scalar("seed", I32), (n,))
    s = D.reduce(D.add, D.const(F64, 0.0), u)
    # the second reduction needs the first one's result for every element
    dev = D.map2(D.sub, u, D.broadcast((n,), s))
    g = Graph("two", [("s", s), ("v", D.reduce(D.add, D.const(F64, 0.0), D.map2(D.mul, dev, dev)))])
    info = B.lower_info(g)
    if info["launches"] < 2:
        pytest.skip("the lowering fused both reductions into one pass")
    with pytest.raises(R.CcbError) as e:
        B.lower_info(g, shard=(0, 2))
    assert e.value.code == 7


def test_mailbox_and_bind_argument_checks():
    L = R.lib()
    h = ctypes.c_void_p()
    R.check(L.ccb_program_lower(to_wire(X.call_greeks(1 << 12, F64), shard=(1, 3)).encode(), ctypes.byref(h)))
    try:
        rank, world = ctypes.c_int(), ctypes.c_int()
        R.check(L.ccb_program_shard(h, ctypes.byref(rank), ctypes.byref(world)))
        assert (rank.value, world.value) == (1, 3)
        size = ctypes.c_size_t()
        R.check(L.ccb_program_mailbox_bytes(h, ctypes.byref(size)))
        assert size.value == 2 * 3 * 33 * 8
        boxes = (ctypes.c_void_p * 3)(0x1000, 0x2000, 0x3000)
        assert L.ccb_program_bind_peers(h, boxes, 2) == 1  # three ranks
        assert L.ccb_program_bind_peers(h, (ctypes.c_void_p * 3)(0x1000, None, 0x3000), 3) == 1
        assert L.ccb_program_bind_peers(h, (ctypes.c_void_p * 3)(0x1000, 0x2004, 0x3000), 3) == 1  # unaligned
        assert "aligned" in L.ccb_last_error().decode()
        assert L.ccb_program_bind_peers(h, boxes, 3) == 0
    finally:
        L.ccb_program_destroy(h)
    R.check(L.ccb_program_lower(to_wire(X.call_greeks(1 << 12, F64)).encode(), ctypes.byref(h)))
    try:
        size = ctypes.c_size_t(99)
        R.check(L.ccb_program_mailbox_bytes(h, ctypes.byref(size)))
        assert size.value == 0
        assert L.ccb_program_bind_peers(h, (ctypes.c_void_p * 1)(0x1000), 1) == 1
        assert "not sharded" in L.ccb_last_error().decode()
    finally:
        L.ccb_program_destroy(h)


def test_multi_sharded_argument_checks():
    build = lambda k: X.call_greeks(k, F64)  # noqa: E731
    with pytest.raises(ValueError):
        M.Multi([0, 0], 1 << 12, build, sharded=True)  # two ranks on one GPU would wait on each other
    with pytest.raises(ValueError):
        M.Multi([0, 1], 1 << 12, build, counter_key="seed", sharded=True)
