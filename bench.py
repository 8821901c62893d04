#!/usr/bin/env python3
"""Benchmark: Black-Scholes Monte-Carlo price with pathwise Greeks (Grad.grad
wrt s0, vol, rate), 2^28 paths per GPU, F32 -- the configuration the reference
metric "MC paths/s" is quoted on. One step = one run of
the Greeks graph (one fused forward+adjoint launch) over 2^28 paths, plus, on
N > 1 GPUs, the NCCL all-reduce that recombines the four scalar outputs.

Scaling is weak: rank r draws Philox counters [r*2^28, (r+1)*2^28) with the
same seed, so N GPUs price N*2^28 distinct paths.

Also measured in the same run (reported under "secondary"): the flat reduce
and inclusive scan over 2^28 F32 values (HBM GB/s as a fraction of the
measured copy peak), the other half of the reference metric.

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
SLOTS_PER_PATH = 150  # algorithmic issue slots per path (Philox, uniform, erfinv, exp, adjoint, sums)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "sm_max_mhz": d.get("sm_max_mhz", 1965.0), "src": "measured"}
    return {"hbm_gbs": 6650.0, "sm_max_mhz": 1965.0, "src": "fallback"}


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
    n, base = args
    sys.path.insert(0, ROOT)
    from cudacaml_b200 import examples as X
    from cudacaml_b200 import multi as M
    from cudacaml_b200.ir import F32, I32, Value
    from oracle import interp as I
    g = M.offset_counters(X.call_greeks(n, F32), "seed")
    c = I.compile(g)
    ins = X.bs_inputs(F32, seed=SEED) + [(M.CTR_BASE, Value.of_list(I32, (), [base]))]
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
            pool.map(_oracle_worker, [(per, (step * cores + w) * per) for w in range(cores)])
            dt = time.perf_counter() - t0
            if step >= args.warmup:
                times.append(dt)
    total = sum(times)
    value = args.steps * cores * per / total
    line = {
        "impl": "reference", "metric": "MC paths/s (Black-Scholes price + pathwise Greeks)", "value": value,
        "unit": "paths/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (Philox normals, seed 42)",
        "config": {"workload": "bs_greeks_f32", "paths_per_step": cores * per, "note": "bounded host sample"},
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
    t, _ = _oracle_worker((n, 0))
    return {"value": n / t, "unit": "paths/s", "cores": 1, "kind": "port",
            "sample": f"{n} paths of the same Greeks graph (F32, seed {SEED}) on 1 core, oracle = C++ restatement of the reference interpreter"}


def secondary_hbm(dev, stream_h, flush, pk):
    """Flat reduce and inclusive scan over 2^28 F32 (1 GiB, > L2), device timed."""
    import numpy as np
    from cudacaml_b200 import backend_cuda as B
    from cudacaml_b200 import runtime as R
    from cudacaml_b200 import examples as X
    from cudacaml_b200.ir import F32
    n = 1 << 28
    res = {}
    x = R.Buffer(4 * n)
    R.check(R.lib().ccb_memset_d8(x.ptr, 0x3c, 4 * n, None))  # 0x3c3c3c3c = 0.0115 in every lane
    R.check(R.lib().ccb_stream_synchronize(None))
    for name, g, out_bytes, alg_bytes in (("reduce_f32_2p28", X.reduce_flat(n, F32), 4, 4 * n),
                                          ("scan_f32_2p28", X.scan_flat(n, F32), 4 * n, 8 * n)):
        c = B.compile_on(dev, g)
        o = R.Buffer(out_bytes)
        s = c.lane_stream(0)
        e0, e1 = R.Event(), R.Event()
        ts = []
        for k in range(8):
            flush(s)
            e0.record(s)
            B.run_device_ptrs(c, [x.ptr], [o.ptr], s)
            e1.record(s)
            e1.synchronize()
            if k >= 3:
                ts.append(e0.elapsed_ms(e1))
        B.check_device(c, s)
        t = statistics.median(ts) * 1e-3
        gbs = alg_bytes / t / 1e9
        res[name] = {"gbs": gbs, "frac_of_measured_hbm": gbs / pk["hbm_gbs"], "ms": t * 1e3, "alg_bytes": alg_bytes}
        o.free()
        B.release(c)
    x.free()
    return res


def run_ours(args):
    import numpy as np
    from cudacaml_b200 import backend_cuda as B
    from cudacaml_b200 import examples as X
    from cudacaml_b200 import multi as M
    from cudacaml_b200 import runtime as R
    from cudacaml_b200.ir import F32, I32

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    R.set_device(local)
    pk = peaks()

    g = X.call_greeks(PATHS, F32)
    if world > 1:
        g = M.offset_counters(g, "seed")
    c = B.compile_on(local, g)
    n_launch = c.num_launches()
    stream = c.lane_stream(0)

    # resident inputs (param order) and outputs
    host_in = {"s0": np.array([100.0], np.float32), "vol": np.array([0.2], np.float32),
               "rate": np.array([0.05], np.float32), "seed": np.array([SEED], np.int32),
               M.CTR_BASE: np.array([rank * PATHS], np.int32)}
    in_bufs = []
    for name, dt, shape in c.params:
        b = R.Buffer(host_in[name].nbytes)
        b.upload(host_in[name])
        in_bufs.append(b)
    out_bufs = [R.Buffer(4) for _ in c.outputs]
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
    red = R.Buffer(16)  # the 4 F32 outputs gathered contiguously for one all-reduce

    def step():
        B.run_device_ptrs(c, [b.ptr for b in in_bufs], [b.ptr for b in out_bufs], stream)
        if comm is not None:
            for j, ob in enumerate(out_bufs):
                R.check(R.lib().ccb_memcpy_d2d(red.ptr + 4 * j, ob.ptr, 4, stream))
            R.check(R.lib().ccb_allreduce(comm, red.ptr, red.ptr, 4, 0, 0, stream))

    flush_buf = R.Buffer(256 << 20)

    def flush(s):
        R.check(R.lib().ccb_memset_d8(flush_buf.ptr, 0, 256 << 20, s))

    def barrier():
        if dist is not None:
            dist.barrier()

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
    for k in range(args.steps):
        flush(stream)
        evs[k][0].record(stream)
        step()
        evs[k][1].record(stream)
    R.check(R.lib().ccb_stream_synchronize(stream))
    clk = clocks.stop()
    barrier()
    B.check_device(c, stream)
    t_dev = sum(a.elapsed_ms(b) for a, b in evs) * 1e-3
    if dist is not None:
        import torch
        t = torch.tensor([t_dev], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_dev = float(t.item())
    value = world * PATHS * args.steps / t_dev

    # read the result once (correctness guard on the timed configuration)
    outs = {}
    for (name, _, _), ob in zip(c.outputs, out_bufs):
        h = np.empty(1, np.float32)
        ob.download(h)
        outs[name] = float(h[0])
    if comm is not None:
        h = np.empty(4, np.float32)
        red.download(h)
        outs = {name: float(v) / world for (name, _, _), v in zip(c.outputs, h)}
    cf = X.analytic()
    assert abs(outs["price"] - cf["price"]) < 0.05, outs

    # e2e: host inputs in pinned memory -> H2D, launch, (all-reduce), D2H of
    # the four results, every step, device-timed on the launching stream.
    pin_in = [R.pinned_empty(host_in[name].shape, host_in[name].dtype) for name, _, _ in c.params]
    for a, (name, _, _) in zip(pin_in, c.params):
        a[...] = host_in[name]
    pin_out = R.pinned_empty((4,), np.float32)
    h2d = sum(a.nbytes for a in pin_in)
    e2e_evs = [(R.Event(), R.Event()) for _ in range(args.steps)]
    for k in range(args.warmup + args.steps):
        flush(stream)
        if k >= args.warmup:
            e2e_evs[k - args.warmup][0].record(stream)
        for a, b in zip(pin_in, in_bufs):
            R.check(R.lib().ccb_memcpy_h2d(b.ptr, a.ctypes.data, a.nbytes, stream))
        step()
        src = red if comm is not None else None
        for j, ob in enumerate(out_bufs):
            R.check(R.lib().ccb_memcpy_d2h(pin_out.ctypes.data + 4 * j, (src.ptr + 4 * j) if src else ob.ptr, 4, stream))
        if k >= args.warmup:
            e2e_evs[k - args.warmup][1].record(stream)
    R.check(R.lib().ccb_stream_synchronize(stream))
    t_e2e = sum(a.elapsed_ms(b) for a, b in e2e_evs) * 1e-3
    if dist is not None:
        import torch
        t = torch.tensor([t_e2e], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_e2e = float(t.item())
    e2e = world * PATHS * args.steps / t_e2e

    avg_launch = t_dev / args.steps
    issue_peak = 148 * 128 * pk["sm_max_mhz"] * 1e6
    achieved = SLOTS_PER_PATH * PATHS / avg_launch
    roofline = {"bound": "issue", "achieved": achieved / 1e9, "peak": issue_peak / 1e9, "unit": "Gslot/s",
                "frac": achieved / issue_peak, "traffic": None,
                "note": f"MC moves ~0 algorithmic bytes; {SLOTS_PER_PATH} issue slots/path x 2^28 paths per launch "
                        f"against 148 SMs x 128 lanes x {pk['sm_max_mhz']:.0f} MHz ({pk['src']} clock)"}

    secondary = None
    if rank == 0 and world == 1 and not args.no_secondary:
        secondary = secondary_hbm(local, stream, flush, pk)

    if rank == 0:
        line = {
            "metric": "MC paths/s (Black-Scholes price + pathwise Greeks)", "value": value, "unit": "paths/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t_dev / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (Philox normals generated in registers, seed 42)",
            "config": {"workload": "bs_greeks_f32 (BASELINE configs[1])", "paths_per_gpu": PATHS,
                       "parallelism": f"dp{world} (counter-range split, NCCL all-reduce of 4 scalars)" if world > 1 else "dp1",
                       "l2": "flushed (256 MiB memset) before every timed step", "market": "S0=100 K=100 r=0.05 sigma=0.2 T=1"},
            "result": outs, "closed_form": cf,
            "gpu_launches": n_launch * args.steps,
            "roofline": roofline,
            "clocks": clk,
            "e2e": {"value": e2e, "unit": "paths/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 16},
        }
        if world == 1:
            line["cpu_baseline"] = cpu_baseline_sample()
        if secondary:
            line["secondary"] = secondary
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        if comm is not None:
            R.lib().ccb_comm_destroy(comm)
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-secondary", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
