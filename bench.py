#!/usr/bin/env python3
"""Benchmark: Black-Scholes Monte-Carlo price with pathwise Greeks (Grad.grad
wrt s0, vol, rate) over 2^28 paths, F64 (F32 reported alongside) -- the
configuration the reference metric "MC paths/s" is quoted on (BASELINE
configs[1]). F64 is the headline because at 2^28 paths the reference's own F32
normal generator produces a few infinite normals (see "secondary"). One step =
one run of the Greeks graph (one fused forward+adjoint launch) plus, on N > 1
GPUs, the cross-rank sum that recombines the four scalar outputs over NVLink
peer memory inside that same kernel.

Scaling is strong, as BASELINE configs[1] states it: on N > 1 GPUs every rank
compiles the unsplit 2^28-path graph as one rank of a sharded program
(compile_on(..., shard=(r, N))): rank r prices counters
[r*2^28/N, (r+1)*2^28/N) with the same seed -- the split
Multi(..., counter_key="seed") makes (multi.path_range) -- and the kernel's
last block combines the four totals of all ranks over NVLink peer memory
(multi.ShardPeers), so each step is one launch per GPU and every rank ends it
with the whole run's results. Weak scaling (2^28 paths per rank, the results
summed after the kernel by multi.PeerSum) is reported under "secondary" for
N > 1.

`value` is device-timed with the inputs resident; `e2e` is the same metric
through the plugin call a user makes, ccb_program_enqueue + ccb_program_wait
with page-locked host inputs and outputs (Backend_cuda.run_async/wait), every
step (on N > 1 the results it downloads are already the whole run's).

Also measured in the same run (reported under "secondary"): the flat reduce
and inclusive scan over 2^28 values, F32 ~N(0,1) and I32 U[0,16) (HBM GB/s as
a fraction of the measured copy peak), and every other BASELINE
configuration. L2 is flushed before every timed step by a read-only pass over
256 MiB (twice the L2).

--impl reference times the reference algorithm on the host cores: the oracle
(the C++ restatement of the reference interpreter, the only runnable form of
the reference here -- OCaml is not installed) with one process per core.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PATHS = 1 << 28
SEED = 42
# Warp instructions executed per path by the fused F64 Greeks kernel, from
# ncu's smsp__inst_executed.sum over 2^26 paths (539,122,169 / 2^26; 443
# paths per thread, the steady state of the 2^28-path launch):
# profiles/mapreduce_bs_greeks_f64_2p26_instructions.md.
INST_PER_PATH_F64 = 539122169 / (1 << 26)
# DRAM bytes per launch of the same kernel (read 55,040, write 0; constant in
# the path count), same capture.
DRAM_BYTES_GREEKS_F64 = 55040


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d.get("bf16_tflops", 1590.0), "sm_max_mhz": d.get("sm_max_mhz", 1965.0),
                "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "sm_max_mhz": 1965.0, "src": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# reference arm: the oracle on the host cores
# ---------------------------------------------------------------------------
def _oracle_worker(args):
    n, base, dts = args
    sys.path.insert(0, ROOT)
    from cudacaml_b200 import examples as X
    from cudacaml_b200 import multi as M
    from cudacaml_b200.ir import F32, I32, Value
    from oracle import interp as I
    from cudacaml_b200.ir import F64
    dt = F64 if dts == "f64" else F32
    g = M.offset_counters(X.call_greeks(n, dt), "seed")
    c = I.compile(g)
    ins = X.bs_inputs(dt, seed=SEED) + [(M.CTR_BASE, Value.of_list(I32, (), [base]))]
    t = time.perf_counter()
    out = dict(I.run(c, ins))
    return time.perf_counter() - t, out["price"].get(0)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import multiprocessing as mp
    cores = os.cpu_count() or 1
    per = 1 << 17
    ctx = mp.get_context("spawn")
    times = []
    with ctx.Pool(cores) as pool:
        for step in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            pool.map(_oracle_worker, [(per, (step * cores + w) * per, "f64") for w in range(cores)])
            dt = time.perf_counter() - t0
            if step >= args.warmup:
                times.append(dt)
    total = sum(times)
    value = args.steps * cores * per / total
    line = {
        "impl": "reference", "metric": "MC paths/s (Black-Scholes price + pathwise Greeks)", "value": value,
        "unit": "paths/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f64", "data": "synthetic (Philox normals, seed 42)",
        "config": {"workload": "bs_greeks_f64 (BASELINE configs[1]; F32 under secondary)", "paths_total": PATHS,
                   "paths_per_step": cores * per,
                   "note": "bounded host sample of the same workload: paths/s is linear in the path count"},
        "cpu_baseline": {"value": value, "unit": "paths/s", "cores": cores, "kind": "port",
                         "sample": f"{cores} processes x {per} paths per step, oracle (C++ restatement of the reference interpreter)"},
        "e2e": {"value": value, "unit": "paths/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def cpu_baseline_sample():
    """The oracle (port) on one core over a bounded sample of the workload."""
    n = 1 << 20
    t, _ = _oracle_worker((n, 0, "f64"))
    return {"value": n / t, "unit": "paths/s", "cores": 1, "kind": "port",
            "sample": f"{n} paths of the same Greeks graph (F64, seed {SEED}) on 1 core, oracle = C++ restatement of the reference interpreter"}


def secondary_hbm(dev, stream_h, flush, pk):
    """Flat reduce and inclusive scan over 2^28 values (config (a): F32
    ~N(0,1); config (b): I32 U[0,16)), and saxpy + sum at 2^28 (F32 and F64,
    x, y = 2U - 1), all larger than L2, device timed (median of 5 after 3
    warm-ups, L2 flushed before each). Inputs are generated on the device by
    the reference's own Rng graphs: seeds 3 (data), 1 (x), 2 (y)."""
    import numpy as np
    from cudacaml_b200 import backend_cuda as B
    from cudacaml_b200 import dsl as D
    from cudacaml_b200 import rng as Rng
    from cudacaml_b200 import runtime as R
    from cudacaml_b200 import examples as X
    from cudacaml_b200.ir import F32, F64, I32, Graph
    n = 1 << 28
    res = {}
    seed_buf = R.Buffer(4)

    def gen(expr, nbytes, seed):
        c = B.compile_on(dev, Graph("gen", [("x", expr)]))
        out = R.Buffer(nbytes)
        seed_buf.upload(np.array([seed], np.int32))
        B.run_device_ptrs(c, [seed_buf.ptr], [out.ptr], None)
        B.check_device(c, None)
        B.release(c)
        return out

    def time_prog(c, ins, outs):
        s = c.lane_stream(0)
        e0, e1 = R.Event(), R.Event()
        ts = []
        for k in range(8):
            flush(s)
            e0.record(s)
            B.run_device_ptrs(c, [b.ptr for b in ins], [b.ptr for b in outs], s)
            e1.record(s)
            e1.synchronize()
            if k >= 3:
                ts.append(e0.elapsed_ms(e1))
        B.check_device(c, s)
        return statistics.median(ts) * 1e-3

    key = D.scalar("seed", I32)
    inputs = (("f32", F32, 4, D.map(lambda v: D.cast(F32, v), Rng.normal(F64, key, (n,))), "~N(0,1)"),
              ("i32", I32, 4, D.map(lambda w: D.bit_and(w, D.const(I32, 15)), Rng.u32(key, (n,))), "U[0,16)"))
    for tag, dt, esz, expr, dist in inputs:
        x = gen(expr, esz * n, 3)
        for name, g, out_bytes, alg_bytes in ((f"reduce_{tag}_2p28", X.reduce_flat(n, dt), esz, esz * n),
                                              (f"scan_{tag}_2p28", X.scan_flat(n, dt), esz * n, 2 * esz * n)):
            c = B.compile_on(dev, g)
            o = R.Buffer(out_bytes)
            t = time_prog(c, [x], [o])
            gbs = alg_bytes / t / 1e9
            res[name] = {"gbs": gbs, "frac_of_measured_hbm": gbs / pk["hbm_gbs"], "ms": t * 1e3, "alg_bytes": alg_bytes,
                         "input": f"{dist}, Rng seed 3"}
            o.free()
            B.release(c)
        x.free()
    for dt, esz in ((F32, 4), (F64, 8)):
        u2 = lambda v: D.cast(dt, D.sub(D.mul(D.const(F64, 2.0), v), D.const(F64, 1.0)))  # noqa: E731
        xs = gen(D.map(u2, Rng.uniform(F64, key, (n,))), esz * n, 1)
        ys = gen(D.map(u2, Rng.uniform(F64, key, (n,))), esz * n, 2)
        c = B.compile_on(dev, X.saxpy(n, 2.0, dt))
        rb, sb = R.Buffer(esz * n), R.Buffer(esz)
        t = time_prog(c, [xs, ys], [rb, sb])
        gbs = 3 * esz * n / t / 1e9
        res[f"saxpy_sum_2p28_{dt.value}"] = {"gbs": gbs, "frac_of_measured_hbm": gbs / pk["hbm_gbs"], "ms": t * 1e3,
                                             "alg_bytes": 3 * esz * n, "launches": c.num_launches(),
                                             "note": "r = 2x + y and s = sum(r) in one pass: read x, y, write r"}
        for b in (xs, ys, rb, sb):
            b.free()
        B.release(c)
    seed_buf.free()
    return res


def secondary_configs(dev, flush, pk, quick=False):
    """The other BASELINE configurations, each device-timed (median of 5 after
    2 warm-ups, L2 flushed before each): rows (65536 x 4096 F32 reduce_rows max
    and scan_rows add), scatter_add of 2^27 Zipf(1.1) updates into 2^20 bins,
    gather of 2^27 from a 2^24 table, saxpy+sum at 2^20 (F32, F64), the
    Longstaff-Schwartz price (2^22 paths x 64 dates, 4-term basis, F64) and the
    MLP training step (8192 x 4096 -> 8192 -> 1024, F32). Inputs are generated
    on the device by the reference's own Rng graphs (Zipf indices by a host
    inverse-CDF table over device-generated uniforms)."""
    import numpy as np
    from cudacaml_b200 import backend_cuda as B
    from cudacaml_b200 import dsl as D
    from cudacaml_b200 import examples as X
    from cudacaml_b200 import lsm as L
    from cudacaml_b200 import rng as Rng
    from cudacaml_b200 import runtime as R
    from cudacaml_b200.ir import F32, F64, I32, Graph, Value

    res = {}
    seed_buf = R.Buffer(4)

    def gen(graph, nbytes, seed):
        c = B.compile_on(dev, graph)
        out = R.Buffer(nbytes)
        seed_buf.upload(np.array([seed], np.int32))
        B.run_device_ptrs(c, [seed_buf.ptr], [out.ptr], None)
        B.check_device(c, None)
        B.release(c)
        return out

    def normal_f32(shape, seed, scale=1.0):
        z = D.map(lambda v: D.cast(F32, D.mul(v, D.const(F64, scale))), Rng.normal(F64, D.scalar("seed", I32), shape))
        return gen(Graph("gen", [("x", z)]), 4 * int(np.prod(shape)), seed)

    def time_prog(c, ins, outs, reps=5):
        s = c.lane_stream(0)
        e0, e1 = R.Event(), R.Event()
        ts = []
        for k in range(2 + reps):
            flush(s)
            e0.record(s)
            B.run_device_ptrs(c, [b.ptr for b in ins], [b.ptr for b in outs], s)
            e1.record(s)
            e1.synchronize()
            if k >= 2:
                ts.append(e0.elapsed_ms(e1) * 1e-3)
        B.check_device(c, s)
        return statistics.median(ts)

    def hbm(t, alg):
        return {"ms": t * 1e3, "gbs": alg / t / 1e9, "frac_of_measured_hbm": alg / t / 1e9 / pk["hbm_gbs"], "alg_bytes": alg}

    # rows
    rows, n = 65536, 4096
    x = normal_f32((rows, n), 3)
    for name, g, ob, alg in (("reduce_rows_max_65536x4096", Graph("rmax", [("m", D.reduce_rows(D.max, D.const(F32, -3e38), D.param("x", F32, (rows, n))))]), 4 * rows, 4 * rows * n + 4 * rows),
                             ("scan_rows_add_65536x4096", Graph("rscan", [("p", D.scan_rows(D.add, D.const(F32, 0.0), D.param("x", F32, (rows, n))))]), 4 * rows * n, 8 * rows * n)):
        c = B.compile_on(dev, g)
        o = R.Buffer(ob)
        res[name] = hbm(time_prog(c, [x], [o]), alg)
        o.free()
        B.release(c)
    x.free()

    # scatter (Zipf) and gather
    m = 1 << 27
    bins = 1 << 20
    u = gen(Graph("u", [("u", Rng.uniform(F64, D.scalar("seed", I32), (m,)))]), 8 * m, 4)
    uh = np.empty(m, np.float64)
    u.download(uh)
    u.free()
    w = 1.0 / np.power(np.arange(1, bins + 1, dtype=np.float64), 1.1)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    idx = np.minimum(np.searchsorted(cdf, uh, side="left"), bins - 1).astype(np.int32)
    del uh
    ib = R.Buffer(4 * m)
    ib.upload(idx)
    vb = gen(Graph("v", [("v", Rng.uniform(F32, D.scalar("seed", I32), (m,)))]), 4 * m, 3)
    c = B.compile_on(dev, X.scatter(m, bins))
    o = R.Buffer(4 * bins)
    r = hbm(time_prog(c, [ib, vb], [o]), 8 * m)
    r["updates_per_s"] = m / (r["ms"] * 1e-3)
    r["hot_bin_share"] = float(np.mean(idx == 0))
    res["scatter_add_zipf_2p27_into_2p20"] = r
    o.free()
    B.release(c)
    tbl = 1 << 24
    gi = gen(Graph("gi", [("i", D.map(lambda w_: D.bit_and(w_, D.const(I32, tbl - 1)), Rng.u32(D.scalar("seed", I32), (m,))))]), 4 * m, 4)
    tb = normal_f32((tbl,), 3)
    c = B.compile_on(dev, X.gather(m, tbl))
    o = R.Buffer(4 * m)
    res["gather_2p27_from_2p24"] = hbm(time_prog(c, [gi, tb], [o]), 12 * m)
    for b in (o, gi, tb, ib, vb):
        b.free()
    B.release(c)

    # saxpy + sum
    for dt, esz in ((F32, 4), (F64, 8)):
        k = 1 << 20
        xs = gen(Graph("x", [("x", D.map(lambda v: D.cast(dt, D.sub(D.mul(D.const(F64, 2.0), v), D.const(F64, 1.0))),
                                          Rng.uniform(F64, D.scalar("seed", I32), (k,))))]), esz * k, 1)
        ys = gen(Graph("y", [("y", D.map(lambda v: D.cast(dt, D.sub(D.mul(D.const(F64, 2.0), v), D.const(F64, 1.0))),
                                          Rng.uniform(F64, D.scalar("seed", I32), (k,))))]), esz * k, 2)
        c = B.compile_on(dev, X.saxpy(k, 2.0, dt))
        rb, sb = R.Buffer(esz * k), R.Buffer(esz)
        t = time_prog(c, [xs, ys], [rb, sb], reps=20)
        r = hbm(t, 3 * esz * k)
        r["note"] = "12.6/25.2 MB: launch-latency bound at this size"
        res[f"saxpy_sum_2p20_{dt.value}"] = r
        for b in (xs, ys, rb, sb):
            b.free()
        B.release(c)

    # Longstaff-Schwartz, BASELINE configuration
    if not quick:
        lp = L.CudaResident(1 << 22, 64, L.BASELINE_MARKET, "poly4", device=dev)
        lp.price(7)
        t0 = time.perf_counter()
        px = lp.price(7)
        t = time.perf_counter() - t0
        lp.release()
        res["lsm_2p22x64_poly4_f64"] = {"ms": t * 1e3, "price": px, "binomial": L.binomial_american_put(L.BASELINE_MARKET),
                                         "note": "wall time of one full price, device-resident: paths graph, one transpose to date-major S, then 63 dates of regress + on-device 4x4 solve + update launched back to back, the mean summed on the device"}

    # MLP training step
    if not quick:
        bsz, din, hid, dout = 8192, 4096, 8192, 1024
        xb = normal_f32((bsz, din), 5)
        w1 = normal_f32((din, hid), 6, 1.0 / math.sqrt(din))
        w2 = normal_f32((hid, dout), 7, 1.0 / math.sqrt(hid))
        tt = normal_f32((bsz, dout), 8)
        named = {"X": xb, "W1": w1, "W2": w2, "T": tt}
        fl = X.mlp_flops(bsz, din, hid, dout)
        tf32_peak = pk["bf16_tflops"] / 2.0
        for prec, reps in (("tf32", 10), ("f32", 3)):
            c = B.compile_on(dev, X.mlp_step(bsz, din, hid, dout), matmul=prec)
            outs = [R.Buffer(4 * int(np.prod(shape)) if shape else 4) for _, _, shape in c.outputs]
            t = time_prog(c, [named[nm] for nm, _, _ in c.params], outs, reps=reps)
            line = {"ms": t * 1e3, "tflops": fl / t / 1e12, "flops": fl, "launches": c.num_launches()}
            if prec == "tf32":
                line["frac_of_tf32_peak"] = fl / t / 1e12 / tf32_peak
                line["note"] = ("matmuls on tcgen05 tensor cores (kind::tf32, TMEM accumulators, TMA operands); "
                                "TF32 peak taken as half the measured dense bf16 %.0f TFLOP/s" % pk["bf16_tflops"])
            else:
                line["note"] = "F32 precision mode: matmuls on CUDA cores (FP32 FMA)"
            res[f"mlp_step_8192x4096x8192x1024_{prec}"] = line
            for b in outs:
                b.free()
            B.release(c)
        for b in (xb, w1, w2, tt):
            b.free()
    seed_buf.free()
    return res


def secondary_reference_nvrtc(dev, flush, ours):
    """The reference's NVRTC backend, restated (baseline/ref_nvrtc.py: the
    reference's buffer plan, kernel templates, launch geometry and C
    spellings, compiled by NVRTC with no options and JIT-loaded), timed on the
    same GPU, on the same synthetic inputs, device-resident, L2 flushed before
    each run, median of 3 after 1 warm-up. `ours` holds this backend's
    numbers from the same run; speedup = reference time / ours."""
    import numpy as np
    from baseline import ref_nvrtc as RN
    from cudacaml_b200 import backend_cuda as B
    from cudacaml_b200 import dsl as D
    from cudacaml_b200 import examples as X
    from cudacaml_b200 import rng as Rng
    from cudacaml_b200 import runtime as R
    from cudacaml_b200.ir import F32, F64, I32, Graph
    from cuda.bindings import driver as cu

    res = {}
    seed_buf = R.Buffer(4)
    key = D.scalar("seed", I32)

    def gen(expr, nbytes, seed):
        c = B.compile_on(dev, Graph("gen", [("x", expr)]))
        out = R.Buffer(nbytes)
        seed_buf.upload(np.array([seed], np.int32))
        B.run_device_ptrs(c, [seed_buf.ptr], [out.ptr], None)
        B.check_device(c, None)
        B.release(c)
        return out

    stream = R.Stream()
    e0, e1 = R.Event(), R.Event()

    def time_ref(g, inputs, reps=3):
        L = RN.Loaded(RN.Program(g))
        try:
            for name, buf in inputs.items():
                RN._ck(cu.cuMemcpyDtoD(L.param_buffer(name), buf.ptr, buf.nbytes), "cuMemcpyDtoD")
            ts = []
            for k in range(1 + reps):
                flush(stream.h)
                e0.record(stream)
                L.launch(stream.h)
                e1.record(stream)
                e1.synchronize()
                if k >= 1:
                    ts.append(e0.elapsed_ms(e1))
            return statistics.median(ts), len(L.prog.kernels)
        finally:
            L.release()

    def put(name, g, inputs, ours_ms, reps=3):
        try:
            ms, nk = time_ref(g, inputs, reps)
            res[name] = {"ms": ms, "kernels": nk, "ours_ms": ours_ms,
                         "speedup": (ms / ours_ms) if ours_ms else None}
        except Exception as e:  # noqa: BLE001 - a baseline failure is reported, not fatal
            res[name] = {"error": f"{type(e).__name__}: {e}"}

    def ours_ms(k):
        v = ours.get(k) or {}
        return v.get("ms")

    n = 1 << 28
    u2 = lambda dt: (lambda v: D.cast(dt, D.sub(D.mul(D.const(F64, 2.0), v), D.const(F64, 1.0))))  # noqa: E731
    xs = gen(D.map(u2(F32), Rng.uniform(F64, key, (n,))), 4 * n, 1)
    ys = gen(D.map(u2(F32), Rng.uniform(F64, key, (n,))), 4 * n, 2)
    put("saxpy_sum_2p28_f32", X.saxpy(n, 2.0), {"x": xs, "y": ys}, ours_ms("saxpy_sum_2p28_f32"))
    xs.free()
    ys.free()
    xf = gen(D.map(lambda v: D.cast(F32, v), Rng.normal(F64, key, (n,))), 4 * n, 3)
    put("reduce_f32_2p28", X.reduce_flat(n, F32), {"x": xf}, ours_ms("reduce_f32_2p28"))
    put("scan_f32_2p28", X.scan_flat(n, F32), {"x": xf}, ours_ms("scan_f32_2p28"))
    xf.free()
    xi = gen(D.map(lambda w: D.bit_and(w, D.const(I32, 15)), Rng.u32(key, (n,))), 4 * n, 3)
    put("reduce_i32_2p28", X.reduce_flat(n, I32), {"x": xi}, ours_ms("reduce_i32_2p28"))
    put("scan_i32_2p28", X.scan_flat(n, I32), {"x": xi}, ours_ms("scan_i32_2p28"))
    xi.free()
    rows, rn = 65536, 4096
    xr = gen(D.map(lambda v: D.cast(F32, v), Rng.normal(F64, key, (rows, rn))), 4 * rows * rn, 3)
    xp = D.param("x", F32, (rows, rn))
    put("reduce_rows_max_65536x4096", Graph("rmax", [("m", D.reduce_rows(D.max, D.const(F32, -3e38), xp))]), {"x": xr},
        ours_ms("reduce_rows_max_65536x4096"))
    put("scan_rows_add_65536x4096", Graph("rscan", [("p", D.scan_rows(D.add, D.const(F32, 0.0), xp))]), {"x": xr},
        ours_ms("scan_rows_add_65536x4096"))
    xr.free()
    m, bins, tbl = 1 << 27, 1 << 20, 1 << 24
    vb = gen(Rng.uniform(F32, key, (m,)), 4 * m, 3)
    ib = gen(D.map(lambda w: D.bit_and(w, D.const(I32, bins - 1)), Rng.u32(key, (m,))), 4 * m, 4)
    # Zipf indices as bench's own scatter line uses them (host inverse CDF)
    u = gen(Rng.uniform(F64, key, (m,)), 8 * m, 4)
    uh = np.empty(m, np.float64)
    u.download(uh)
    u.free()
    w = 1.0 / np.power(np.arange(1, bins + 1, dtype=np.float64), 1.1)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    ib.upload(np.minimum(np.searchsorted(cdf, uh, side="left"), bins - 1).astype(np.int32))
    del uh
    put("scatter_add_zipf_2p27_into_2p20", X.scatter(m, bins), {"idx": ib, "v": vb},
        ours_ms("scatter_add_zipf_2p27_into_2p20"))
    ib.free()
    vb.free()
    gi = gen(D.map(lambda w_: D.bit_and(w_, D.const(I32, tbl - 1)), Rng.u32(key, (m,))), 4 * m, 4)
    tb = gen(D.map(lambda v: D.cast(F32, v), Rng.normal(F64, key, (tbl,))), 4 * tbl, 3)
    put("gather_2p27_from_2p24", X.gather(m, tbl), {"idx": gi, "table": tb}, ours_ms("gather_2p27_from_2p24"))
    gi.free()
    tb.free()
    for dt, esz in ((F64, 8), (F32, 4)):
        ins = {}
        for name, val in (("s0", 100.0), ("vol", 0.2), ("rate", 0.05)):
            b = R.Buffer(esz)
            b.upload(np.array([val], dt.np))
            ins[name] = b
        sb = R.Buffer(4)
        sb.upload(np.array([42], np.int32))
        ins["seed"] = sb
        put(f"bs_greeks_{dt.value}_2p28", X.call_greeks(PATHS, dt), ins, ours_ms(f"bs_greeks_{dt.value}_2p28"))
        for b in ins.values():
            b.free()
    bsz, din, hid, dout = 8192, 4096, 8192, 1024
    named = {"X": gen(D.map(lambda v: D.cast(F32, v), Rng.normal(F64, key, (bsz, din))), 4 * bsz * din, 5),
             "W1": gen(D.map(lambda v: D.cast(F32, D.mul(v, D.const(F64, 1 / math.sqrt(din)))),
                             Rng.normal(F64, key, (din, hid))), 4 * din * hid, 6),
             "W2": gen(D.map(lambda v: D.cast(F32, D.mul(v, D.const(F64, 1 / math.sqrt(hid)))),
                             Rng.normal(F64, key, (hid, dout))), 4 * hid * dout, 7),
             "T": gen(D.map(lambda v: D.cast(F32, v), Rng.normal(F64, key, (bsz, dout))), 4 * bsz * dout, 8)}
    put("mlp_step_8192x4096x8192x1024_f32", X.mlp_step(bsz, din, hid, dout), named,
        ours_ms("mlp_step_8192x4096x8192x1024_tf32"), reps=1)
    if "ms" in res["mlp_step_8192x4096x8192x1024_f32"]:
        res["mlp_step_8192x4096x8192x1024_f32"]["ours_f32_ms"] = ours_ms("mlp_step_8192x4096x8192x1024_f32")
        res["mlp_step_8192x4096x8192x1024_f32"]["note"] = ("ours_ms is this backend's tf32 step (tensor cores), "
                                                            "ours_f32_ms its F32 (CUDA-core) step")
    for b in named.values():
        b.free()
    seed_buf.free()
    stream.destroy()
    return res


def sharded_probe(rank, world, local, dist, exchange):
    """A small sharded Greeks run (2^20 paths, two runs, checked) before the
    headline relies on sharded programs. Every rank reaches the same
    collectives whatever fails, and learns whether all ranks succeeded (MIN
    all-reduces), so a failure on any rank sends every rank to the split-then-
    sum path instead of leaving ranks waiting on each other. Returns
    (ok, reason)."""
    import numpy as np
    import torch
    from cudacaml_b200 import backend_cuda as B
    from cudacaml_b200 import examples as X
    from cudacaml_b200 import multi as M
    from cudacaml_b200 import runtime as R
    from cudacaml_b200.ir import F64

    dev = f"cuda:{local}" if dist.get_backend() == "nccl" else "cpu"

    def agree(ok):
        t = torch.tensor([1.0 if ok else 0.0], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return float(t[0]) > 0.5

    why, c, sp, bufs = None, None, None, []
    try:
        c = B.compile_on(local, X.call_greeks(1 << 20, F64), shard=(rank, world))
    except Exception as e:  # noqa: BLE001 - reported, the headline falls back
        why = f"compile: {type(e).__name__}: {e}"
    if agree(why is None):
        try:
            sp = M.ShardPeers(c, exchange)  # a collective: every rank calls it
            host = {"s0": 100.0, "vol": 0.2, "rate": 0.05}
            for name, dt, _ in c.params:
                b = R.Buffer(8 if dt.value == "f64" else 4)
                b.upload(np.array([host[name]]) if name in host else np.array([SEED], np.int32))
                bufs.append(b)
            out = R.Buffer(32)
            bufs.append(out)
            for _ in range(2):
                B.run_device_ptrs(c, [b.ptr for b in bufs[:-1]], [out.ptr + 8 * j for j in range(4)], None)
            B.check_device(c, None)
        except Exception as e:  # noqa: BLE001
            why = f"run: {type(e).__name__}: {e}"
    elif why is None:
        why = "another rank failed"
    ok = agree(why is None)
    dist.barrier()
    if sp is not None:
        sp.close()
    for b in bufs:
        b.free()
    if c is not None:
        B.release(c)
    return ok, why or ("" if ok else "another rank failed")


def measure_greeks(args, dtype, rank, world, local, dist, peer, flush, weak=False, exchange=None, sharded_ok=True):
    """Device-timed and end-to-end paths/s of the Greeks graph in `dtype`.

    Strong scaling (default): the unsplit 2^28-path graph compiled as rank r
    of a sharded program (shard=(r, world)): the kernel walks paths
    [r*PATHS/world, (r+1)*PATHS/world) -- the counters Multi's split gives
    rank r -- and its last block combines all ranks' totals over NVLink peer
    memory (multi.ShardPeers), so every rank ends each step with the whole
    run's results and no collective follows. weak=True gives every rank
    PATHS paths of its own (counters [r*PATHS, (r+1)*PATHS), which must stay
    below 2^31, offset_counters) and sums the four results across the ranks
    after the kernel (multi.PeerSum)."""
    import numpy as np
    from cudacaml_b200 import backend_cuda as B
    from cudacaml_b200 import examples as X
    from cudacaml_b200 import multi as M
    from cudacaml_b200 import runtime as R

    sharded = world > 1 and not weak and sharded_ok
    total = PATHS * world if weak else PATHS
    base, per = M.path_range(total, world, rank)
    shard_peers = None
    if sharded:
        c = B.compile_on(local, X.call_greeks(PATHS, dtype), shard=(rank, world))
        shard_peers = M.ShardPeers(c, exchange)
        peer = None
    else:
        g = X.call_greeks(per, dtype)
        if world > 1:
            g = M.offset_counters(g, "seed", rows=per)
        c = B.compile_on(local, g)
    stream = c.lane_stream(0)
    fnp = dtype.np
    esz = np.dtype(fnp).itemsize
    host_in = {"s0": np.array([100.0], fnp), "vol": np.array([0.2], fnp), "rate": np.array([0.05], fnp),
               "seed": np.array([SEED], np.int32), M.CTR_BASE: np.array([base], np.int32)}
    in_bufs = []
    for name, _, _ in c.params:
        b = R.Buffer(host_in[name].nbytes)
        b.upload(host_in[name])
        in_bufs.append(b)
    red = R.Buffer(4 * esz)  # the four scalar outputs, contiguous: one all-reduce
    out_ptrs = [red.ptr + j * esz for j in range(len(c.outputs))]
    dt_code = R.DT_CODE[dtype.value]

    def step():
        B.run_device_ptrs(c, [b.ptr for b in in_bufs], out_ptrs, stream)
        if peer is not None:
            peer.sum(red.ptr, red.ptr, 4, dt_code, stream)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(t):
        if dist is None:
            return t
        import torch
        x = torch.tensor([t], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(x, op=dist.ReduceOp.MAX)
        return float(x.item())

    for _ in range(args.warmup):
        flush(stream)
        step()
    B.check_device(c, stream)
    evs = [(R.Event(), R.Event()) for _ in range(args.steps)]
    barrier()
    R.check(R.lib().ccb_stream_synchronize(stream))
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    # The ranks' steps are coupled (each step's cross-rank combine waits for
    # every rank), so a rank whose host starts the timed loop late stalls
    # the others' first timed step (on 8 GPUs the sampler's start-up skew
    # once added ~2 ms per step on average). Every rank leaves one barrier
    # right before the loop, and one untimed step on every GPU lines the
    # GPUs up before the first timed one.
    barrier()
    if world > 1:
        flush(stream)
        step()
    for k in range(args.steps):
        flush(stream)
        evs[k][0].record(stream)
        step()
        evs[k][1].record(stream)
    R.check(R.lib().ccb_stream_synchronize(stream))
    clk = clocks.stop()
    barrier()
    B.check_device(c, stream)
    t_dev = max_over_ranks(sum(a.elapsed_ms(b) for a, b in evs) * 1e-3)
    h = np.empty(4, fnp)
    red.download(h)
    if peer is not None:
        peer.check(stream)
    div = world if peer is not None else 1
    outs = {name: float(v) / div for (name, _, _), v in zip(c.outputs, h)}

    # e2e through the plugin call (Backend_cuda.run_async + wait): the
    # program uploads the page-locked host inputs, runs and downloads its four
    # results into page-locked host memory on its lane's stream; on N > 1 the
    # downloaded results are then all-reduced (uploaded, NCCL, read back) on
    # the same stream. Device-timed on that stream, every step.
    L = R.lib()
    pin_in = [R.pinned_empty(host_in[name].shape, host_in[name].dtype) for name, _, _ in c.params]
    for a, (name, _, _) in zip(pin_in, c.params):
        a[...] = host_in[name]
    pin_out = R.pinned_empty((4,), fnp)
    pin_res = R.pinned_empty((4,), fnp)
    in_arr = B._ptr_array([a.ctypes.data for a in pin_in])
    out_arr = B._ptr_array([pin_out.ctypes.data + j * esz for j in range(len(c.outputs))])
    h2d = sum(a.nbytes for a in pin_in)
    e2e_evs = [(R.Event(), R.Event()) for _ in range(args.steps)]
    barrier()
    for k in range(args.warmup + args.steps):
        flush(stream)
        timed = k >= args.warmup
        if timed:
            e2e_evs[k - args.warmup][0].record(stream)
        R.check(L.ccb_program_enqueue(c.h, 0, in_arr, out_arr))
        if peer is not None:
            R.check(L.ccb_memcpy_h2d(red.ptr, pin_out.ctypes.data, 4 * esz, stream))
            peer.sum(red.ptr, red.ptr, 4, dt_code, stream)
            R.check(L.ccb_memcpy_d2h(pin_res.ctypes.data, red.ptr, 4 * esz, stream))
        if timed:
            e2e_evs[k - args.warmup][1].record(stream)
        R.check(L.ccb_program_wait(c.h, 0))
        R.check(L.ccb_stream_synchronize(stream))
    B.check_device(c, stream)
    t_e2e = max_over_ranks(sum(a.elapsed_ms(b) for a, b in e2e_evs) * 1e-3)
    # the plugin call computed the same bits as the device-resident runs
    if peer is not None:
        peer.check(stream)
    e2e_res = pin_res if peer is not None else pin_out
    assert np.array_equal(e2e_res, h, equal_nan=True), (e2e_res, h)
    n_launch = c.num_launches()
    for b in in_bufs:
        b.free()
    red.free()
    if shard_peers is not None:
        barrier()  # every rank finished its last run before a mailbox goes away
        shard_peers.close()
    B.release(c)
    paths_all = per * world
    return {"value": paths_all * args.steps / t_dev, "t_dev": t_dev, "ms_per_step": 1e3 * t_dev / args.steps,
            "e2e": paths_all * args.steps / t_e2e, "h2d": h2d + (4 * esz if peer is not None else 0),
            # the four results, the program's 4-byte error word, and on N > 1 the all-reduced results
            "d2h": 4 * esz + 4 + (4 * esz if peer is not None else 0), "outs": outs, "clocks": clk,
            "launches": n_launch, "paths_per_rank": per}


def measure_mlp_dp(rank, world, local, dist, comm, flush, pk):
    """The MLP training step data-parallel over `world` GPUs (BASELINE
    configs: global batch 8192 split by rows, gradients combined by NCCL
    all-reduce): per rank the tf32 step on 8192/world rows; the NCCL
    all-reduces (sum) of loss, dW2 and dW1 run on a second stream, each as
    soon as its output is final, so dW2's overlaps the dA1, dZ1 and dW1 work. Device
    time per step, max over ranks; inputs device-generated, rank-specific
    rows."""
    import math
    import numpy as np
    import torch
    from cudacaml_b200 import backend_cuda as B
    from cudacaml_b200 import dsl as D
    from cudacaml_b200 import examples as X
    from cudacaml_b200 import rng as Rng
    from cudacaml_b200 import runtime as R
    from cudacaml_b200.ir import F32, F64, I32, Graph, numel

    L = R.lib()
    bsz, din, hid, dout = 8192, 4096, 8192, 1024
    per = bsz // world
    seed_buf = R.Buffer(4)

    def normal_f32(shape, seed, scale=1.0):
        z = D.map(lambda v: D.cast(F32, D.mul(v, D.const(F64, scale))), Rng.normal(F64, D.scalar("seed", I32), shape))
        c = B.compile_on(local, Graph("gen", [("x", z)]))
        out = R.Buffer(4 * int(np.prod(shape)))
        seed_buf.upload(np.array([seed], np.int32))
        B.run_device_ptrs(c, [seed_buf.ptr], [out.ptr], None)
        B.check_device(c, None)
        B.release(c)
        return out

    # Set-up first; every rank agrees it succeeded before any NCCL call, so a
    # failing rank cannot leave the others waiting inside a collective.
    err = None
    try:
        named = {"X": normal_f32((per, din), 5 + 1000 * rank), "W1": normal_f32((din, hid), 6, 1.0 / math.sqrt(din)),
                 "W2": normal_f32((hid, dout), 7, 1.0 / math.sqrt(hid)), "T": normal_f32((per, dout), 8 + 1000 * rank)}
        c = B.compile_on(local, X.mlp_step(per, din, hid, dout), matmul="tf32")
        outs = [R.Buffer(4 * numel(shape) if shape else 4) for _, _, shape in c.outputs]
    except Exception as e:  # noqa: BLE001
        err = f"{type(e).__name__}: {e}"
    ok = torch.tensor([0.0 if err else 1.0], device=f"cuda:{local}")
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if float(ok[0]) < 1.0:
        return {"error": err or "set-up failed on another rank"}
    ins = [named[nm].ptr for nm, _, _ in c.params]
    s = c.lane_stream(0)
    ar_bytes = sum(4 * numel(shape) for _, _, shape in c.outputs)

    # Each output's all-reduce runs on a communication stream as soon as the
    # output is final (an event recorded right after the kernel that writes
    # it), in production order -- the launch scheduler runs dW2's product
    # right after the dY/loss pass: the loss, dW2 while dA1, dZ1 and dW1 are
    # computed, then dW1 (collectives on one communicator run in issue order,
    # so the issue order must follow production). Every rank issues the same
    # collectives in the same order.
    cs = R.Stream()
    ev_out = [R.Event() for _ in c.outputs]
    ev_join = R.Event()
    produced = ["loss", "dloss/dW2", "dloss/dW1"]
    pos = {nm: j for j, (nm, _, _) in enumerate(c.outputs)}
    e0, e1, e2 = R.Event(), R.Event(), R.Event()
    t_step, t_comp = [], []
    for k in range(3 + 10):
        flush(s)
        e0.record(s)
        B.run_device_ptrs_events(c, ins, [b.ptr for b in outs], ev_out, s)
        e1.record(s)
        for nm in produced:
            j = pos[nm]
            _, dt, shape = c.outputs[j]
            R.check(L.ccb_stream_wait_event(cs.h, ev_out[j].h))
            R.check(L.ccb_allreduce(comm, outs[j].ptr, outs[j].ptr, numel(shape), R.DT_CODE[dt.value], 0, cs.h))
        ev_join.record(cs)
        R.check(L.ccb_stream_wait_event(s, ev_join.h))
        e2.record(s)
        e2.synchronize()
        if k >= 3:
            t_step.append(e0.elapsed_ms(e2))
            t_comp.append(e0.elapsed_ms(e1))
    B.check_device(c, s)
    ts = torch.tensor([float(np.median(t_step)), float(np.median(t_comp))], device=f"cuda:{local}")
    dist.all_reduce(ts, op=dist.ReduceOp.MAX)
    ms, ms_comp = float(ts[0]), float(ts[1])
    for b in outs + list(named.values()) + [seed_buf]:
        b.free()
    cs.destroy()
    B.release(c)
    fl = X.mlp_flops(bsz, din, hid, dout)
    return {"ms": ms, "tflops": fl / ms / 1e9, "compute_ms": ms_comp, "allreduce_ms": ms - ms_comp,
            "allreduce_bytes_per_rank": ar_bytes, "rows_per_gpu": per,
            "note": "global batch 8192 split by rows; per rank the tf32 step; NCCL all-reduces (sum) of loss, dW2, "
                    "dW1 on a second stream, each started when its output is final (dW2's overlaps dA1, dZ1, dW1); "
                    "compute_ms = the step's own kernels, allreduce_ms = what the collectives add; device time, max "
                    "over ranks, median of 10 after 3 warm-ups"}


def run_ours(args):
    from cudacaml_b200 import examples as X
    from cudacaml_b200 import multi as M
    from cudacaml_b200 import runtime as R
    from cudacaml_b200.ir import F32, F64

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    # NCCL may print its version banner on stdout when a communicator is
    # created; stdout carries only the JSON line, so the set-up below runs
    # with stdout pointed at stderr.
    saved_stdout = os.dup(1) if world > 1 else None
    if world > 1:
        sys.stdout.flush()
        os.dup2(2, 1)
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    R.set_device(local)
    pk = peaks()
    comm = None
    if world > 1:
        import ctypes
        uid = (ctypes.c_ubyte * 128)()
        if rank == 0:
            R.check(R.lib().ccb_comm_unique_id(uid))
        obj = [bytes(uid)]
        dist.broadcast_object_list(obj, src=0)
        uid = (ctypes.c_ubyte * 128).from_buffer_copy(obj[0])
        h = ctypes.c_void_p()
        R.check(R.lib().ccb_comm_init_rank(world, uid, rank, ctypes.byref(h)))
        comm = h.value
        dist.barrier()
        sys.stdout.flush()
        os.dup2(saved_stdout, 1)
        os.close(saved_stdout)
    # L2 flush between timed steps: a read-only pass over 256 MiB (twice the
    # 126 MB L2) with the allocation-free sum kernel. A write-based flush (a
    # memset) would leave ~126 MB of dirty lines whose write-back then
    # competes with the next timed kernel.
    flush_n = 64 << 20
    flush_buf = R.Buffer(4 * flush_n)
    R.check(R.lib().ccb_memset_d8(flush_buf.ptr, 0, 4 * flush_n, None))
    flush_out = R.Buffer(4)
    R.check(R.lib().ccb_stream_synchronize(None))

    def flush(s):
        rc = R.lib().ccb_sum_f32_noalloc(flush_buf.ptr, flush_n, flush_out.ptr, s)
        if rc != 0:
            raise RuntimeError(R.lib().ccb_last_error().decode())

    # Mailboxes are mapped between the ranks through CUDA IPC (`exchange`
    # trades the handles): the headline's sharded program combines its four
    # totals in its own last block (ShardPeers); the weak-scaling line sums
    # its four results after the kernel (PeerSum, one 32-thread kernel per
    # rank); NCCL stays for the MLP step's gradients.
    peer = None
    if world > 1:
        def exchange(h):
            got = [None] * world
            dist.all_gather_object(got, h)
            return got
        peer = M.PeerSum(world, rank, exchange)
    sharded_ok, sharded_why = True, ""
    if world > 1:
        sharded_ok, sharded_why = sharded_probe(rank, world, local, dist, exchange)
    head = measure_greeks(args, F64, rank, world, local, dist, peer, flush, exchange=exchange if world > 1 else None,
                          sharded_ok=sharded_ok)
    cf = X.analytic()
    ok = abs(head["outs"]["price"] - cf["price"]) < 0.02
    f32 = None
    if world == 1 and not args.no_secondary:
        f32 = measure_greeks(args, F32, rank, world, local, dist, peer, flush)
    secondary = None
    if world > 1 and not args.no_secondary:
        weak = measure_greeks(args, F64, rank, world, local, dist, peer, flush, weak=True)
        try:
            mlp = measure_mlp_dp(rank, world, local, dist, comm, flush, pk)
        except Exception as e:  # noqa: BLE001 - reported, not fatal to the headline
            mlp = {"error": f"{type(e).__name__}: {e}"}
        if rank == 0:
            secondary = {
                "bs_greeks_f64_weak": {"value": weak["value"], "unit": "paths/s", "e2e": weak["e2e"],
                                       "ms_per_step": weak["ms_per_step"], "paths_per_gpu": weak["paths_per_rank"],
                                       "result": weak["outs"],
                                       "note": "weak scaling: every rank prices 2^28 paths of its own "
                                               "(counters [r*2^28, (r+1)*2^28)), 4 scalars summed across ranks per step"},
                f"mlp_step_8192x4096x8192x1024_tf32_dp{world}": mlp}
    if rank == 0 and world == 1 and not args.no_secondary:
        secondary = secondary_hbm(local, None, flush, pk)
        try:
            secondary.update(secondary_configs(local, flush, pk))
        except Exception as e:  # keep the headline line; report what failed
            secondary["configs_error"] = f"{type(e).__name__}: {e}"
        secondary["bs_greeks_f32_2p28"] = {
            "value": f32["value"], "unit": "paths/s", "e2e": f32["e2e"], "ms_per_step": f32["ms_per_step"],
            "ms": f32["ms_per_step"], "result": f32["outs"],
            "note": "the reference's F32 generator rounds (w + 0.5) * 2^-32 to 1.0f for w >= 2^32 - 2^7 "
                    "(expected ~8 of 2^28 paths) and erfinv(1) = inf, so the F32 price is inf at this size in the "
                    "reference interpreter too (cudacaml_backend_interp.ml:130); throughput only"}
        secondary["bs_greeks_f64_2p28"] = {"ms": head["ms_per_step"]}
        try:
            secondary["reference_nvrtc_restated"] = secondary_reference_nvrtc(local, flush, secondary)
        except Exception as e:  # noqa: BLE001 - the baseline is reported, not fatal
            secondary["reference_nvrtc_restated"] = {"error": f"{type(e).__name__}: {e}"}

    # Issue roofline from the measured instruction count: warp instructions
    # per launch / launch time against 148 SMs x 4 sub-partitions x 1 warp
    # instruction per cycle at the measured maximum SM clock.
    avg_launch = head["t_dev"] / args.steps
    issue_peak = 148 * 4 * pk["sm_max_mhz"] * 1e6
    achieved = INST_PER_PATH_F64 * head["paths_per_rank"] / avg_launch
    roofline = {"bound": "issue", "achieved": achieved / 1e9, "peak": issue_peak / 1e9, "unit": "Gwarp-inst/s",
                "frac": achieved / issue_peak, "traffic": DRAM_BYTES_GREEKS_F64,
                "note": f"Monte Carlo moves ~0 algorithmic bytes; {INST_PER_PATH_F64:.3f} warp instructions per path "
                        f"(ncu smsp__inst_executed.sum over 2^26 paths, 443 per thread: the steady state of this "
                        f"launch; profiles/mapreduce_bs_greeks_f64_2p26_instructions.md) x "
                        f"{head['paths_per_rank']} paths per launch / the average step, against 148 SMs x 4 "
                        f"sub-partitions x 1 warp instruction/cycle x {pk['sm_max_mhz']:.0f} MHz ({pk['src']} max "
                        f"clock); ncu's issue-active on the same capture is 75 %; traffic = DRAM bytes per launch "
                        f"from the same ncu capture"
                        + ("; the step includes the cross-rank combine of the 4 totals inside the kernel"
                           if world > 1 else "")}
    if rank == 0:
        line = {
            "metric": "MC paths/s (Black-Scholes price + pathwise Greeks)", "value": head["value"], "unit": "paths/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (Philox normals generated in registers, seed 42)",
            "config": {"workload": "bs_greeks_f64 (BASELINE configs[1]; F32 under secondary)", "paths_total": PATHS,
                       "paths_per_gpu": head["paths_per_rank"],
                       "parallelism": ((f"dp{world} (sharded program: rank r walks paths [r*2^28/{world}, "
                                        f"(r+1)*2^28/{world}), the 4 reductions combined across ranks in the kernel's "
                                        f"last block over NVLink peer memory)") if sharded_ok else
                                       (f"dp{world} (counter range split {world} ways, the 4 results summed across "
                                        f"ranks after the kernel over NVLink peer memory; the sharded program's probe "
                                        f"failed: {sharded_why})")) if world > 1 else "dp1",
                       "l2": "flushed before every timed step (read-only pass over 256 MiB, twice L2)",
                       "market": "S0=100 K=100 r=0.05 sigma=0.2 T=1"},
            "result": head["outs"], "result_ok_vs_closed_form": ok, "closed_form": cf,
            "gpu_launches": head["launches"] * args.steps,
            "roofline": roofline,
            "clocks": head["clocks"],
            "e2e": {"value": head["e2e"], "unit": "paths/s", "h2d_bytes_per_step": head["h2d"],
                    "d2h_bytes_per_step": head["d2h"],
                    "path": "ccb_program_enqueue + ccb_program_wait with page-locked host buffers"
                            + (" (the cross-rank combine runs inside the kernel)" if world > 1 else "")},
        }
        if world == 1:
            line["cpu_baseline"] = cpu_baseline_sample()
        if secondary:
            line["secondary"] = secondary
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        if peer is not None:
            peer.close()
        if comm is not None:
            R.lib().ccb_comm_destroy(comm)
        dist.destroy_process_group()
    return 0 if ok else 1


def run_profile_case(args):
    """A small fixed case for ncu captures: a couple of launches of one kernel."""
    import numpy as np
    from cudacaml_b200 import backend_cuda as B
    from cudacaml_b200 import examples as X
    from cudacaml_b200 import runtime as R
    from cudacaml_b200.ir import F32, F64
    from cudacaml_b200 import dsl as D
    from cudacaml_b200.ir import I32, Graph, Value
    R.set_device(0)
    n = args.size
    if args.profile in ("greeks64", "greeks32"):
        dt = F64 if args.profile == "greeks64" else F32
        c = B.compile(X.call_greeks(n, dt))
        ins = X.bs_inputs(dt, seed=SEED)
    elif args.profile in ("reduce", "scan"):
        g = {"reduce": X.reduce_flat(n, F32), "scan": X.scan_flat(n, F32)}[args.profile]
        c = B.compile(g)
        ins = [("x", Value.of_array(F32, (n,), np.full(n, 0.5, np.float32)))]
    elif args.profile in ("rows_reduce", "rows_scan"):
        rows = n // 4096
        x = D.param("x", F32, (rows, 4096))
        op = (D.reduce_rows(D.max, D.const(F32, -3e38), x) if args.profile == "rows_reduce"
              else D.scan_rows(D.add, D.const(F32, 0.0), x))
        c = B.compile(Graph("rows", [("r", op)]))
        ins = [("x", Value.of_array(F32, (rows, 4096), np.full(rows * 4096, 0.5, np.float32)))]
    elif args.profile == "scatter":
        bins = 1 << 20
        c = B.compile(X.scatter(n, bins))
        ins = [("idx", Value.of_array(I32, (n,), X.zipf_indices(4, n, bins))),
               ("v", Value.of_array(F32, (n,), np.full(n, 0.5, np.float32)))]
    elif args.profile == "gather":
        tbl = 1 << 24
        c = B.compile(X.gather(n, tbl))
        ins = [("idx", Value.of_array(I32, (n,), (X.philox_word0(4, n) & (tbl - 1)).astype(np.int32))),
               ("table", Value.of_array(F32, (tbl,), np.full(tbl, 0.5, np.float32)))]
    elif args.profile == "lsm":  # the resident LSM driver: n paths x 64 dates, 4-term basis, F64
        from cudacaml_b200 import lsm as L
        lp = L.CudaResident(n, 64, L.BASELINE_MARKET, "poly4")
        for _ in range(2):
            px = lp.price(7)
        lp.release()
        print(json.dumps({"price": px}))
        return 0
    elif args.profile == "mm_tf32":  # one square tensor-core product
        a = D.param("a", F32, (n, n))
        bm = D.param("b", F32, (n, n))
        c = B.compile(Graph("mm", [("c", D.matmul(a, bm))]), matmul="tf32")
        rng = np.random.default_rng(0)
        ins = [(nm, Value.of_array(F32, (n, n), rng.standard_normal(n * n).astype(np.float32))) for nm in ("a", "b")]
    else:  # mlp at a reduced size
        b = n
        c = B.compile(X.mlp_step(b, b // 2, b, b // 8), matmul="tf32" if args.profile == "mlp_tf32" else "f32")
        rng = np.random.default_rng(0)
        ins = [(nm, Value.of_array(F32, shape, rng.standard_normal(int(np.prod(shape))).astype(np.float32) * 0.05))
               for nm, _, shape in c.params]
    for _ in range(3):
        out = B.run(c, ins)
    print(json.dumps({k: float(v.data[0]) for k, v in out if v.numel == 1}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--profile", default=None,
                    choices=["greeks64", "greeks32", "reduce", "scan", "rows_reduce", "rows_scan", "scatter", "gather", "mlp",
                             "mlp_tf32", "mm_tf32", "lsm"],
                    help="run a small fixed case (3 launches) for an ncu capture, no timing")
    ap.add_argument("--size", type=int, default=1 << 24, help="paths/elements of the --profile case")
    args = ap.parse_args()
    if args.profile:
        return run_profile_case(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
