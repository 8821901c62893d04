"""The multi-GPU host logic on the CPU.

* ``Multi`` (lib/backend_cuda/multi.ml:123-174): input slicing, the explicit
  ``split=`` list, the counter-range split of a Monte-Carlo graph and the host
  combines, with the oracle standing in for the devices (``compile_on``,
  ``run_async``, ``wait`` and ``release`` evaluate on the host).
* The process-per-GPU split ``bench.py`` runs under torchrun, as world_size-2
  ``gloo`` ranks: rank r computes paths [r*per, (r+1)*per) of the same seed
  and the four Greeks are summed by an all-reduce and divided by the world
  size; per-path draws gathered from the ranks are the unsplit draws bit for
  bit; the MLP batch split by rows sums to the full-batch loss and gradients.

CPU only; the oracle is the checker and the executor here, nothing runs on a
GPU.
"""
import datetime
import multiprocessing as mp
import queue
import socket
import time

import numpy as np
import pytest

from cudacaml_b200 import dsl as D
from cudacaml_b200 import examples as X
from cudacaml_b200 import multi as M
from cudacaml_b200 import rng as Rng
from cudacaml_b200.ir import F32, F64, I32, Graph, Value
from oracle import interp as I

SEED = 42


class OracleDevices:
    """Stands in for backend_cuda inside Multi: every 'device' evaluates its
    program with the oracle on the host."""

    def __init__(self):
        self.compiled = []

    def compile_on(self, ordinal, g, matmul=None):
        self.compiled.append((ordinal, g))
        return I.compile(g)

    def run_async(self, c, inputs):
        return I.run(c, list(inputs))

    def wait(self, job):
        return job

    def release(self, c):
        pass


@pytest.fixture
def devices(monkeypatch):
    fake = OracleDevices()
    monkeypatch.setattr(M, "B", fake)
    return fake


def run(g, inputs):
    return dict(I.run(I.compile(g), inputs))


def seed_in(k=SEED):
    return ("seed", Value.of_list(I32, (), [k]))


def draws(k: int) -> Graph:
    """Per-path draws of three shapes: one normal per path, a 5-step grid of
    raw words per path, and a 7-element draw shared by every path."""
    key = D.scalar("seed", I32)
    return Graph("draws", [("z", Rng.normal(F64, key, (k,))),
                           ("w", Rng.u32(key, (k, 5))),
                           ("shared", Rng.u32(key, (7,)))])


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-300))


# ---------------------------------------------------------------------------
# Multi, with the oracle in place of the devices
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("devs", [[0, 1], [0, 0, 0, 0]])
def test_multi_slices_inputs_like_one_device(devices, devs):
    n = 1024
    x = Value.of_array(F32, (n,), np.arange(n, dtype=np.float32))
    y = Value.of_array(F32, (n,), np.ones(n, dtype=np.float32))
    single = run(X.saxpy(n, 2.0), [("x", x), ("y", y)])
    t = M.Multi(devs, n, lambda k: X.saxpy(k, 2.0))
    assert [o for o, _ in devices.compiled] == devs
    per = t.run([("x", x), ("y", y)])
    assert np.array_equal(M.concat([dict(o)["r"] for o in per]).data, single["r"].data)
    t.release()
    with pytest.raises(RuntimeError):
        t.run([("x", x), ("y", y)])


def test_multi_mean_scalar_and_i32_across_device_lists(devices):
    # test/unit/test_multigpu.ml: 2 * mean of the per-device sums is the
    # single sum; an I32 program with negative division splits the same on
    # [0; 0] and [0; 1]
    n = 8192
    x = Value.of_array(F32, (n,), np.arange(n, dtype=np.float32))
    y = Value.of_array(F32, (n,), (n - np.arange(n)).astype(np.float32))
    s = run(X.saxpy(n, 2.0), [("x", x), ("y", y)])["s"].get(0)
    t = M.Multi([0, 0], n, lambda k: X.saxpy(k, 2.0))
    per = t.run([("x", x), ("y", y)])
    assert len(per) == 2
    assert abs(2.0 * M.mean_scalar([dict(o)["s"] for o in per]) - s) <= 1e-5 * abs(s)
    t.release()

    def i32_prog(k):
        e = D.param("x", I32, (k,))
        return Graph("i32", [("r", D.map(lambda v: D.div(D.sub(v, D.const(I32, 4)), D.const(I32, 2)), e))])

    xi = Value.of_array(I32, (n,), np.arange(n, dtype=np.int32) - 100)
    want = run(i32_prog(n), [("x", xi)])["r"].data
    for devs in ([0, 0], [0, 1]):
        t = M.Multi(devs, n, i32_prog)
        got = M.concat([dict(o)["r"] for o in t.run([("x", xi)])]).data
        t.release()
        assert np.array_equal(got, want)
    # truncating division, as the reference's Int32.div: (-101 - 4) / 2 = -52
    assert want[0] == -52


def test_multi_run_per_device_one_seed_each(devices):
    # test/unit/test_multigpu.ml "per-device inputs": the reference's way to
    # decorrelate devices is one seed per device; prices differ and each is
    # within the reference's band of the closed form
    n = 1 << 14
    t = M.Multi([0, 0], n, lambda k: X.call_mc(k, F32))
    per = t.run_per_device(lambda d: X.bs_inputs(F32, seed=d + 1))
    t.release()
    prices = [dict(o)["price"].get(0) for o in per]
    cf = X.analytic()["price"]
    assert all(abs(p - cf) <= 1.0 for p in prices)
    assert prices[0] != prices[1]


@pytest.mark.parametrize("d", [2, 4])
def test_multi_counter_split_draws_bit_exact(devices, d):
    # rank-1 and multi-step draws split by path; the shared draw stays whole
    n = 64
    single = run(draws(n), [seed_in()])
    t = M.Multi(list(range(d)), n, draws, counter_key="seed")
    per = [dict(o) for o in t.run([seed_in()])]
    assert np.array_equal(M.concat([o["z"] for o in per]).data, single["z"].data)
    assert np.array_equal(M.concat([o["w"] for o in per]).data, single["w"].data)
    for o in per:
        assert np.array_equal(o["shared"].data, single["shared"].data)
    t.release()


def test_offset_counters_base_is_first_path():
    # a 1-D draw counts from the base itself, a (paths, 5) grid from 5 * base
    n = 16
    g = M.offset_counters(draws(n), "seed")
    out = run(g, [seed_in(), (M.CTR_BASE, Value.of_list(I32, (), [3]))])
    full = run(draws(n + 3), [seed_in()])
    assert np.array_equal(out["z"].data, full["z"].data[3:])
    assert np.array_equal(out["w"].data, full["w"].data[3 * 5:])
    # rows=None moves every draw keyed by the seed: the 7-element one too
    words = run(Graph("u", [("u", Rng.u32(D.scalar("seed", I32), (10,)))]), [seed_in()])["u"].data
    assert np.array_equal(out["shared"].data, words[3:])
    # rows=n leaves it where the unsplit program has it
    g = M.offset_counters(draws(n), "seed", rows=n)
    out = run(g, [seed_in(), (M.CTR_BASE, Value.of_list(I32, (), [3]))])
    assert np.array_equal(out["shared"].data, words[:7])
    assert np.array_equal(out["w"].data, full["w"].data[3 * 5:])


def test_split_graphs_lower_and_compile_for_sm100a():
    # the counter base is a scalar parameter folded into the counter: the
    # split program has the unsplit program's kernels and compiles with NVRTC
    import ctypes
    from cudacaml_b200 import backend_cuda as B
    from cudacaml_b200 import runtime as R
    for name, g0, g1 in [
            ("paths", X.call_mc_paths(512, 16, F64), M.offset_counters(X.call_mc_paths(512, 16, F64), "seed", rows=512)),
            ("greeks", X.call_greeks(4096, F64), M.offset_counters(X.call_greeks(4096, F64), "seed")),
            ("draws", draws(512), M.offset_counters(draws(512), "seed", rows=512))]:
        info = B.lower_info(g1)
        assert info["kernels"] == B.lower_info(g0)["kernels"], name
        sz = ctypes.c_size_t()
        log = ctypes.c_void_p()
        rc = R.lib().ccb_nvrtc_check(info["source"].encode(), name.encode(), ctypes.byref(sz), ctypes.byref(log))
        if log.value:
            R.lib().ccb_free_string(log)
        assert rc == 0 and sz.value > 0, R.lib().ccb_last_error().decode()[:2000]


def test_multi_counter_split_multistep_price(devices):
    # call_mc_paths: (paths, steps) normals, scan_rows, gather of the last
    # column; D devices' mean equals the one-device price
    n, steps = 256, 8
    p1 = X.scalar_out(list(run(X.call_mc_paths(n, steps, F64), X.bs_inputs(F64, seed=SEED)).items()), "price")
    t = M.Multi([0, 1, 2, 3], n, lambda k: X.call_mc_paths(k, steps, F64), counter_key="seed")
    pm = M.mean_scalar([dict(o)["price"] for o in t.run(X.bs_inputs(F64, seed=SEED))])
    t.release()
    assert abs(pm - p1) <= 1e-12 * abs(p1)


def test_multi_split_names_row_split_gradients(devices):
    # W2's first dimension equals the batch: slicing by leading dimension
    # alone would cut it, the explicit split keeps it whole
    bsz, din, hid, dout = 8, 4, 8, 3
    rng = np.random.default_rng(3)
    shapes = {"X": (bsz, din), "W1": (din, hid), "W2": (hid, dout), "T": (bsz, dout)}
    ins = [(nm, Value.of_array(F64, shapes[nm], rng.standard_normal(shapes[nm]) * 0.5))
           for nm in ("X", "W1", "W2", "T")]
    want = run(X.mlp_step(bsz, din, hid, dout, F64), ins)
    build = lambda k: X.mlp_step(k, din, hid, dout, F64)  # noqa: E731
    t = M.Multi([0, 1], bsz, build, split=["X", "T"])
    per = [dict(o) for o in t.run(ins)]
    t.release()
    for name in ("loss", "dloss/dW1", "dloss/dW2"):
        got = sum(o[name].data for o in per)
        assert rel(got, want[name].data) <= 1e-12, name
    with pytest.raises(I.InterpError):
        M.Multi([0, 1], bsz, build).run(ins)  # W2 sliced to 4 rows
    with pytest.raises(ValueError):
        M.Multi([0, 1], bsz, build, split=["W1"]).run(ins)


def test_multi_create_and_combine_errors(devices):
    with pytest.raises(ValueError):
        M.Multi([], 8, lambda k: X.saxpy(k, 1.0))
    with pytest.raises(ValueError):
        M.Multi([0, 1, 2], 8, lambda k: X.saxpy(k, 1.0))
    with pytest.raises(ValueError):
        M.concat([])
    with pytest.raises(ValueError):
        M.concat([Value.of_list(F32, (), [1.0])])
    with pytest.raises(ValueError):
        M.concat([Value.of_list(F32, (2,), [1.0, 2.0]), Value.of_list(F64, (2,), [1.0, 2.0])])
    with pytest.raises(ValueError):
        M.concat([Value.of_list(F32, (1, 2), [1.0, 2.0]), Value.of_list(F32, (1, 3), [1.0, 2.0, 3.0])])
    with pytest.raises(ValueError):
        M.mean_scalar([])
    with pytest.raises(ValueError):
        M.mean_scalar([Value.of_list(F32, (2,), [1.0, 2.0])])
    assert M.mean_scalar([Value.of_list(F64, (), [1.0]), Value.of_list(F64, (), [2.0])]) == 1.5


# ---------------------------------------------------------------------------
# One process per rank over gloo: the split bench.py runs under torchrun
# ---------------------------------------------------------------------------
GREEKS_N = 1 << 12
MLP = (16, 6, 8, 4)  # batch, din, hidden, dout


def _mlp_inputs():
    bsz, din, hid, dout = MLP
    rng = np.random.default_rng(11)
    shapes = {"X": (bsz, din), "W1": (din, hid), "W2": (hid, dout), "T": (bsz, dout)}
    return {nm: rng.standard_normal(shapes[nm]) * 0.5 for nm in ("X", "W1", "W2", "T")}


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        res = {}
        # Greeks, split as bench.py splits its headline (strong scaling):
        # counter range [rank*per, (rank+1)*per) of one seed, Multi's
        # path_range and offset_counters; every output is a mean over paths,
        # so the ranks' sum / world is the mean
        first, per = M.path_range(GREEKS_N, world, rank)
        g = M.offset_counters(X.call_greeks(per, F64), "seed", rows=per)
        base = (M.CTR_BASE, Value.of_list(I32, (), [first]))
        out = run(g, X.bs_inputs(F64, seed=SEED) + [base])
        names = [nm for nm, _ in g.outputs]
        s = torch.tensor([out[nm].get(0) for nm in names], dtype=torch.float64)
        dist.all_reduce(s, op=dist.ReduceOp.SUM)
        res["greeks"] = {nm: float(v) / world for nm, v in zip(names, s.tolist())}
        # per-path draws: gathered from the ranks in rank order
        dg = M.offset_counters(draws(per), "seed", rows=per)
        o = run(dg, [seed_in(), base])
        for nm in ("z", "w"):
            mine = torch.from_numpy(np.ascontiguousarray(o[nm].data))
            parts = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(parts, mine)
            res[nm] = torch.cat(parts).numpy()
        # MLP: rows [rank*rows, (rank+1)*rows) of X and T, whole weights;
        # loss and gradients are sums over rows, all-reduced by sum
        bsz, din, hid, dout = MLP
        rows = bsz // world
        full = _mlp_inputs()
        ins = [("X", Value.of_array(F64, (rows, din), full["X"][rank * rows:(rank + 1) * rows])),
               ("W1", Value.of_array(F64, (din, hid), full["W1"])),
               ("W2", Value.of_array(F64, (hid, dout), full["W2"])),
               ("T", Value.of_array(F64, (rows, dout), full["T"][rank * rows:(rank + 1) * rows]))]
        mo = run(X.mlp_step(rows, din, hid, dout, F64), ins)
        for nm in ("loss", "dloss/dW1", "dloss/dW2"):
            t = torch.from_numpy(np.ascontiguousarray(mo[nm].data, dtype=np.float64))
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
            res[nm] = t.numpy()
        # the slowest rank's time is the job's: max over ranks
        tm = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        res["max_over_ranks"] = float(tm.item())
        q.put((rank, res))
    except Exception as e:  # reported to the parent instead of a silent exit
        q.put((rank, {"error": repr(e)}))
    finally:
        dist.destroy_process_group()


def test_path_range_split_and_counter_limit():
    assert [M.path_range(1 << 28, 8, i) for i in (0, 1, 7)] == [(0, 1 << 25), (1 << 25, 1 << 25), (7 << 25, 1 << 25)]
    assert M.path_range(1 << 31, 8, 7) == (7 << 28, 1 << 28)  # weak scaling at 8 GPUs: counters up to 2^31 - 1
    with pytest.raises(ValueError):
        M.path_range((1 << 31) + 8, 8, 0)  # would wrap the I32 counters
    with pytest.raises(ValueError):
        M.path_range(100, 3, 0)
    with pytest.raises(ValueError):
        M.Multi([0, 0], (1 << 31) + 2, lambda k: X.call_mc(k, F64), counter_key="seed")


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_gloo_world2_counter_split_and_row_split():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.monotonic() + 240
    try:
        while len(got) < world and time.monotonic() < deadline:
            try:
                r, res = q.get(timeout=1)
            except queue.Empty:
                gone = [r for r, p in enumerate(procs) if p.exitcode is not None and r not in got]
                if gone and q.empty():
                    break  # a rank ended without a result
                continue
            got[r] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    errors = {r: res["error"] for r, res in got.items() if "error" in res}
    assert not errors, errors
    assert len(got) == world, f"ranks with results: {sorted(got)}, exit codes {[p.exitcode for p in procs]}"
    assert all(p.exitcode == 0 for p in procs)

    want = run(X.call_greeks(GREEKS_N, F64), X.bs_inputs(F64, seed=SEED))
    for r in range(world):
        for nm, v in got[r]["greeks"].items():
            assert abs(v - want[nm].get(0)) <= 1e-12 * max(abs(want[nm].get(0)), 1e-12), nm
        assert got[r]["max_over_ranks"] == float(world)
    wd = run(draws(GREEKS_N), [seed_in()])
    for nm in ("z", "w"):
        assert np.array_equal(got[0][nm], wd[nm].data), nm
        assert np.array_equal(got[1][nm], wd[nm].data), nm

    bsz, din, hid, dout = MLP
    full = _mlp_inputs()
    shapes = {"X": (bsz, din), "W1": (din, hid), "W2": (hid, dout), "T": (bsz, dout)}
    wm = run(X.mlp_step(bsz, din, hid, dout, F64), [(nm, Value.of_array(F64, shapes[nm], full[nm])) for nm in full])
    for nm in ("loss", "dloss/dW1", "dloss/dW2"):
        for r in range(world):
            assert rel(got[r][nm], wm[nm].data) <= 1e-12, (r, nm)
