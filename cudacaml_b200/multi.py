"""Data-parallel runs across the GPUs of one box, restating CUDACaml's
``Multi`` (lib/backend_cuda/multi.mli:14-64, multi.ml:123-174).

``Multi(devices, n, build)`` compiles ``build(n // d)`` once per device;
``run`` slices every input whose leading dimension is ``n`` (a view, no host
copy), issues all devices before waiting on any, and returns one output list
per device. ``concat`` and ``mean_scalar`` combine on the host as the
reference does.

Additions, all opt-in:

* ``counter_key="seed"`` splits a Monte-Carlo graph by *counter range* with the
  same seed (device d draws Philox counters [d*n/D, (d+1)*n/D)), so D devices
  compute exactly the paths one device would. The reference instead asks the
  caller to reseed each device (multi.mli:39-44). The graph is rewritten to
  add a scalar ``__ctr_base`` parameter (the device's first path) to every
  per-path Rng counter, scaled by the draw's elements per path, so
  multi-step grids split correctly too.
* ``allreduce_mean(names, inputs)`` recombines scalar outputs on the devices
  with a cross-device sum over NVLink peer memory (``PeerSum``) instead of a
  host loop.
* ``sharded=True`` compiles the unsplit graph on every device as one rank of
  a sharded program: each device walks its slice of the paths and the
  kernel's last block combines all devices' totals over NVLink, so the
  recombination is part of the kernel (``ShardPeers`` does the same for one
  process per GPU).
* ``allreduce_sum(names, inputs)`` sums whole outputs across the devices on
  the devices (one NCCL all-reduce per output, grouped): a loss and the weight
  gradients of a batch split by rows, as in the MLP training step.
* ``split=[names]`` limits slicing to the named inputs (the reference slices
  every input whose leading dimension is n, which also cuts a weight matrix
  whose first dimension happens to equal the batch size); ``matmul=`` is the
  F32 product precision each device program is compiled with.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import backend_cuda as B
from . import dsl as D
from . import runtime as R
from .ir import I32, Graph, Tensor, Value, numel

CTR_BASE = "__ctr_base"


def offset_counters(g: Graph, key: str, rows: int | None = None) -> Graph:
    """Rewrite every Rng.u32 counter ``map2 f (iota s) (broadcast s key)`` to
    count from a scalar parameter ``__ctr_base`` (rng.ml:49-59).

    ``__ctr_base`` is the first *path* (leading-axis row) the program
    computes. Rng.u32's counter is the flat element index (the iota of the
    draw's shape), so a draw of shape ``(paths, k1, ...)`` counts from
    ``__ctr_base * k1 * ...``: a program built for rows [b, b + paths) draws
    the same counters as those rows of the unsplit program, also for
    multi-step grids. A 1-D draw counts from ``__ctr_base`` itself.

    ``rows=None`` offsets every draw keyed by ``key``; with ``rows`` set only
    draws whose leading dimension equals ``rows`` (the per-device path count)
    move, and any other draw is shared, as it is in the unsplit program."""
    base = D.scalar(CTR_BASE, I32)
    memo = {}

    def is_counter(t: Tensor) -> bool:
        if t.kind != "map2":
            return False
        i, k = t.deps
        if not (i.kind == "iota" and k.kind == "broadcast" and k.deps[0].kind == "param"
                and k.deps[0].name == key):
            return False
        return rows is None or (len(i.shape) > 0 and i.shape[0] == rows)

    def go(t: Tensor) -> Tensor:
        if t.uid in memo:
            return memo[t.uid]
        deps = [go(d) for d in t.deps]
        if is_counter(t):
            it = t.deps[0]
            row = numel(it.shape[1:])
            start = base if row == 1 else D.map(lambda b: D.mul(b, D.const(I32, row)), base)
            deps[0] = D.map2(D.add, it, D.broadcast(it.shape, start))
        if all(a is b for a, b in zip(deps, t.deps)):
            new = t
        else:
            new = Tensor(t.dtype, t.shape, t.kind, deps=deps, name=t.name, fn=t.fn, init=t.init)
        memo[t.uid] = new
        return new

    return Graph(g.name, [(n, go(t)) for n, t in g.outputs])


def path_range(n: int, d: int, i: int) -> tuple[int, int]:
    """Device ``i`` of ``d``'s share of ``n`` paths: ``(first path, count)``,
    the counters ``[i*n/d, (i+1)*n/d)``. Rng counters are I32 element indices,
    so the whole range must stay below 2^31; a larger one would wrap and
    repeat draws, and is refused instead."""
    if d <= 0 or not 0 <= i < d:
        raise ValueError(f"Multi: device {i} of {d}")
    if n % d != 0:
        raise ValueError(f"Multi.create: n = {n} is not divisible by {d} devices")
    per = n // d
    if n > 1 << 31:
        raise ValueError(f"Multi: {n} paths exceed the I32 counter range (2^31)")
    return i * per, per


def concat(values):
    """Concatenate along the leading axis (multi.ml:51-92)."""
    if not values:
        raise ValueError("Multi.concat: no values to concatenate")
    first = values[0]
    if len(first.shape) == 0:
        raise ValueError("Multi.concat: a rank-0 value has no leading axis")
    rest = first.shape[1:]
    for v in values:
        if v.dtype is not first.dtype:
            raise ValueError(f"Multi.concat: dtype {v.dtype.value} does not match {first.dtype.value}")
        if len(v.shape) == 0 or v.shape[1:] != rest:
            raise ValueError(f"Multi.concat: shape {list(v.shape)} does not match {list(first.shape)} outside the leading axis")
    lead = sum(v.shape[0] for v in values)
    return Value(first.dtype, (lead,) + tuple(rest), np.concatenate([v.data for v in values]))


def mean_scalar(values) -> float:
    """Plain mean of per-device scalars (multi.ml:105-109)."""
    if not values:
        raise ValueError("Multi.mean_scalar: no values to average")
    for v in values:
        if v.numel != 1:
            raise ValueError(f"Multi.mean_scalar: {list(v.shape)} is not a scalar")
    return sum(float(v.data[0]) for v in values) / len(values)


def _ipc_mailbox(nbytes, nranks, rank, exchange):
    """Allocate and zero-fill this rank's mailbox, then trade IPC handles with
    ``exchange`` (a collective returning every rank's 64-byte handle in rank
    order, so no rank can write into a mailbox its owner has not zeroed yet)
    and map every peer's. Returns (own buffer, pointers in rank order, the
    mapped peer pointers to close)."""
    L = R.lib()
    own = R.Buffer(nbytes)
    R.check(L.ccb_memset_d8(own.ptr, 0, nbytes, None))
    R.check(L.ccb_stream_synchronize(None))
    h = (ctypes.c_ubyte * 64)()
    R.check(L.ccb_ipc_mem_handle(own.ptr, h))
    handles = exchange(bytes(h))
    ptrs, opened = [], []
    for q, hq in enumerate(handles):
        if q == rank:
            ptrs.append(own.ptr)
            continue
        p = ctypes.c_void_p()
        R.check(L.ccb_ipc_mem_open((ctypes.c_ubyte * 64).from_buffer_copy(hq), ctypes.byref(p)))
        opened.append(p.value)
        ptrs.append(p.value)
    return own, ptrs, opened


def _peer_mailboxes(devices, nbytes):
    """One zero-filled mailbox on each of ``devices`` (distinct ordinals, one
    process), with peer access enabled between all of them."""
    if len(set(devices)) != len(devices):
        raise ValueError("every rank needs its own GPU")
    L = R.lib()
    own = []
    for d in devices:
        with R.with_device(d):
            for q in devices:
                if q != d:
                    R.check(L.ccb_peer_access_enable(q))
            b = R.Buffer(nbytes)
            R.check(L.ccb_memset_d8(b.ptr, 0, nbytes, None))
            R.check(L.ccb_stream_synchronize(None))
            own.append(b)
    return own


class ShardPeers:
    """The mailboxes of a sharded program (compiled with ``shard=(rank,
    world)``) in a process-per-GPU job: this rank's mailbox is allocated and
    zero-filled here, mapped by every peer through CUDA IPC (``exchange`` as
    for PeerSum), and all of them are bound to the program. Every rank then
    runs the program the same number of times in the same order; each run's
    last block combines the ranks' totals over NVLink, so no collective
    follows the kernel."""

    def __init__(self, c, exchange):
        rank, world = B.shard_of(c)
        if world < 2:
            raise ValueError("ShardPeers: the program is not sharded")
        self.own, ptrs, self._opened = _ipc_mailbox(B.mailbox_bytes(c), world, rank, exchange)
        B.bind_peers(c, ptrs)

    def close(self):
        """Unmap the peers' mailboxes and free this rank's; every rank must
        have finished its last run (synchronised) first."""
        for p in self._opened:
            R.lib().ccb_ipc_mem_close(p)
        self._opened = []
        if self.own is not None:
            self.own.free()
            self.own = None


class PeerSum:
    """Cross-rank sum of a few scalars over NVLink peer memory
    (ccb_xrank_sum), for ranks on distinct GPUs of one box: one 32-thread
    kernel per rank writes its values into every rank's mailbox and sums
    what arrives, in rank order, so every rank gets the same bits. It
    replaces a library all-reduce of the 4 scalars a split Monte-Carlo run
    recombines per step, whose launch and protocol latency grows with the
    rank count.

    ``PeerSum(nranks, rank, exchange)``: one process per rank. The mailbox is
    allocated and zero-filled here, then ``exchange(handle_bytes)`` must
    return every rank's 64-byte IPC handle in rank order (for example
    ``torch.distributed.all_gather_object``); it is a collective, so no rank
    can write into a mailbox that its owner has not zeroed yet.
    ``PeerSum.in_process(devices)``: one process driving several GPUs, each
    device a rank, peer access enabled between them.
    """

    ERR_XRANK = 32

    def __init__(self, nranks, rank, exchange=None, _devices=None):
        L = R.lib()
        self.nranks, self.rank = nranks, rank
        self.epoch = 0
        size = ctypes.c_size_t()
        R.check(L.ccb_xrank_mailbox_bytes(nranks, ctypes.byref(size)))
        self._opened = []
        if _devices is None:
            self.err = R.Buffer(4)
            R.check(L.ccb_memset_d8(self.err.ptr, 0, 4, None))
            self.own, ptrs, self._opened = _ipc_mailbox(size.value, nranks, rank, exchange)
            self.mailboxes = (ctypes.c_void_p * nranks)(*ptrs)
            self.devices = None

    @classmethod
    def in_process(cls, devices):
        """One PeerSum per device of ``devices`` (distinct ordinals), sharing
        mailboxes through peer access; returns the list, rank = position."""
        devices = list(devices)
        if len(set(devices)) != len(devices):
            raise ValueError("PeerSum: every rank needs its own GPU")
        L = R.lib()
        n = len(devices)
        size = ctypes.c_size_t()
        R.check(L.ccb_xrank_mailbox_bytes(n, ctypes.byref(size)))
        own = _peer_mailboxes(devices, size.value)
        errs = []
        for d in devices:
            with R.with_device(d):
                e = R.Buffer(4)
                R.check(L.ccb_memset_d8(e.ptr, 0, 4, None))
                R.check(L.ccb_stream_synchronize(None))
                errs.append(e)
        out = []
        for r, d in enumerate(devices):
            ps = cls(n, r, _devices=devices)
            ps.own, ps.err, ps.devices = own[r], errs[r], devices
            ps.mailboxes = (ctypes.c_void_p * n)(*[b.ptr for b in own])
            out.append(ps)
        return out

    def sum(self, in_ptr, out_ptr, count, dtype_code, stream=None):
        """Issue one sum on ``stream`` (the current device must be this
        rank's); every rank must issue the same sums in the same order."""
        self.epoch += 1
        R.check(R.lib().ccb_xrank_sum(in_ptr, out_ptr, count, dtype_code, self.nranks, self.rank, self.mailboxes,
                                      self.epoch, self.err.ptr, stream))

    def check(self, stream=None):
        """Synchronise ``stream`` and raise if a wait gave up."""
        R.check(R.lib().ccb_stream_synchronize(stream))
        w = np.empty(1, np.uint32)
        self.err.download(w)
        if int(w[0]) & self.ERR_XRANK:
            raise R.CcbError("cross-rank sum: a peer did not publish its values (bounded wait gave up)")

    def close(self):
        """Unmap the peers' mailboxes and free this rank's. Every rank must
        have finished its last sum (synchronised) first."""
        for p in self._opened:
            R.lib().ccb_ipc_mem_close(p)
        self._opened = []
        if getattr(self, "own", None) is not None:
            self.own.free()
            self.err.free()
            self.own = None


class Multi:
    """``sharded=True`` (Monte-Carlo estimators): every device compiles the
    unsplit graph ``build(n)`` as one rank of a sharded program
    (include/ccb.h, sharded programs): device i walks paths
    [i*n/D, (i+1)*n/D) and the kernel's last block combines the devices'
    totals over NVLink peer memory, so each device's outputs are already the
    whole run's (the same bits on every device) and no recombination step
    follows. Needs distinct devices; inputs are not sliced."""

    def __init__(self, devices, n: int, build, counter_key: str | None = None, split=None, matmul=None,
                 sharded: bool = False):
        devices = list(devices)
        d = len(devices)
        if d == 0:
            raise ValueError("Multi.create: devices must not be empty")
        if n % d != 0:
            raise ValueError(f"Multi.create: n = {n} is not divisible by {d} devices")
        if sharded and (counter_key is not None or split is not None):
            raise ValueError("Multi.create: a sharded Multi splits the index space itself (no counter_key, no split)")
        if sharded and len(set(devices)) != d:
            raise ValueError("Multi.create: a sharded Multi needs distinct devices (its ranks wait on each other)")
        if counter_key is not None:
            path_range(n, d, 0)  # the split counter range must fit the I32 counters
        self.devices = devices
        self.n = n
        self.per = n // d
        self.counter_key = counter_key
        self.split = None if split is None else set(split)
        self.sharded = sharded and d > 1
        self.released = False
        self.slots = []
        self._mailboxes = []
        for i, ordinal in enumerate(devices):
            if self.sharded:
                self.slots.append(B.compile_on(ordinal, build(n), matmul=matmul, shard=(i, d)))
                continue
            g = build(self.per)
            if counter_key is not None:
                g = offset_counters(g, counter_key, rows=self.per)
            self.slots.append(B.compile_on(ordinal, g, matmul=matmul))
        if self.sharded:
            self._mailboxes = _peer_mailboxes(devices, B.mailbox_bytes(self.slots[0]))
            for c in self.slots:
                B.bind_peers(c, [b.ptr for b in self._mailboxes])
        self._comms = None

    def _splits(self, name, v) -> bool:
        if self.split is not None:
            if name in self.split and (not len(v.shape) or v.shape[0] != self.n):
                raise ValueError(f"Multi.run: input {name} has shape {list(v.shape)}, leading dimension {self.n} expected")
            return name in self.split
        return bool(len(v.shape)) and v.shape[0] == self.n

    def _inputs_for(self, i: int, inputs):
        if self.sharded:
            return list(inputs)
        out = []
        for name, v in inputs:
            if self._splits(name, v):
                rest = v.shape[1:]
                stride = numel(rest)
                data = v.data[i * self.per * stride:(i + 1) * self.per * stride]
                out.append((name, Value(v.dtype, (self.per,) + tuple(rest), data)))
            else:
                out.append((name, v))
        if self.counter_key is not None:
            base, _ = path_range(self.n, len(self.devices), i)
            out.append((CTR_BASE, Value.of_list(I32, (), [base])))
        return out

    def run_per_device(self, inputs_fn):
        if self.released:
            raise RuntimeError("Multi.run: this Multi.t has been released")
        if self.sharded:
            # A sharded kernel's last block waits for every device's totals, so
            # every device's run is issued before the host waits on any of them
            # (a host-buffer run would block in its pageable download first).
            keep = self._issue_resident(inputs_fn)
            out = []
            for i, c in enumerate(self.slots):
                with R.with_device(c.device):
                    B.check_device(c, c.lane_stream(0))
                    vals = []
                    for (name, dt, shape), buf in zip(c.outputs, keep[i][1]):
                        host = np.empty(numel(shape), dtype=dt.np)
                        buf.download(host)
                        vals.append((name, Value(dt, tuple(shape), host)))
                    out.append(vals)
            self._free_resident(keep)
            return out
        jobs = [B.run_async(c, inputs_fn(i)) for i, c in enumerate(self.slots)]
        return [B.wait(j) for j in jobs]

    def run(self, inputs):
        inputs = list(inputs)
        return self.run_per_device(lambda i: self._inputs_for(i, inputs))

    def allreduce_mean(self, names, inputs):
        """Run every device resident, sum the named scalar outputs across the
        devices on the devices, and return {name: sum / d}. The sum runs over
        NVLink peer memory (PeerSum: one small kernel per device, every
        device gets the same bits). Needs distinct device ordinals."""
        if self.released:
            raise RuntimeError("Multi.run: this Multi.t has been released")
        if len(set(self.devices)) != len(self.devices):
            raise ValueError("Multi.allreduce: a cross-device sum needs distinct devices; use mean_scalar for repeats")
        outs = self.slots[0].outputs
        for name in names:
            js = [k for k, (n, _, shape) in enumerate(outs) if n == name]
            if not js:
                raise ValueError(f"Multi.allreduce: no output named {name}")
            if numel(outs[js[0]][2]) != 1:
                raise ValueError(f"Multi.allreduce_mean: output {name} is not a scalar")
        d = len(self.devices)
        inputs = list(inputs)
        if self.sharded:  # every device's outputs are already the whole run's
            keep = self._run_all_resident(inputs)
            for c in self.slots:
                B.check_device(c, c.lane_stream(0))
            result = {}
            for name in names:
                j = [k for k, (n, _, _) in enumerate(outs) if n == name][0]
                host = np.empty(1, dtype=outs[j][1].np)
                with R.with_device(self.slots[0].device):
                    keep[0][1][j].download(host)
                result[name] = float(host[0])
            self._free_resident(keep)
            return result
        if getattr(self, "_peer", None) is None:
            self._peer = PeerSum.in_process(self.devices)
        keep = self._run_all_resident(inputs)
        for name in names:
            j = [k for k, (n, _, _) in enumerate(outs) if n == name][0]
            dt = outs[j][1]
            for i, c in enumerate(self.slots):
                with R.with_device(c.device):
                    ptr = keep[i][1][j].ptr
                    self._peer[i].sum(ptr, ptr, 1, R.DT_CODE[dt.value], c.lane_stream(0))
        result = {}
        for i, c in enumerate(self.slots):
            with R.with_device(c.device):
                self._peer[i].check(c.lane_stream(0))
                B.check_device(c, c.lane_stream(0))
        for name in names:
            j = [k for k, (n, _, _) in enumerate(outs) if n == name][0]
            dt = outs[j][1]
            host = np.empty(1, dtype=dt.np)
            with R.with_device(self.slots[0].device):
                keep[0][1][j].download(host)
            result[name] = float(host[0]) / d
        self._free_resident(keep)
        return result

    def _run_all_resident(self, inputs):
        return self._issue_resident(lambda i: self._inputs_for(i, inputs))

    def _issue_resident(self, inputs_fn):
        """Upload every device's inputs and run it resident on its lane
        stream, without waiting on any; returns [(input buffers, output
        buffers)] per device."""
        keep = []
        for i, c in enumerate(self.slots):
            with R.with_device(c.device):
                bound = dict(inputs_fn(i))
                in_bufs = []
                for pname, dt, shape in c.params:
                    buf = R.Buffer(bound[pname].byte_size)
                    buf.upload(bound[pname].data)
                    in_bufs.append(buf)
                out_bufs = [R.Buffer(numel(shape) * dt.size_in_bytes) for _, dt, shape in c.outputs]
                B.run_device_ptrs(c, [b.ptr for b in in_bufs], [b.ptr for b in out_bufs], c.lane_stream(0))
                keep.append((in_bufs, out_bufs))
        return keep

    def _free_resident(self, keep):
        for c, (ib, ob) in zip(self.slots, keep):
            with R.with_device(c.device):
                for b in ib + ob:
                    b.free()

    def allreduce_sum(self, names, inputs):
        """Run every device resident, all-reduce the named outputs with NCCL
        (sum) across the devices, on the devices, and return {name: Value}
        (the sum, read back from the first device). Needs distinct device
        ordinals (NCCL puts one rank on each GPU)."""
        if self.released:
            raise RuntimeError("Multi.run: this Multi.t has been released")
        if len(set(self.devices)) != len(self.devices):
            raise ValueError("Multi.allreduce: NCCL needs distinct devices; use mean_scalar for repeats")
        out_names = [n for n, _, _ in self.slots[0].outputs]
        for name in names:
            if name not in out_names:
                raise ValueError(f"Multi.allreduce: no output named {name}")
        L = R.lib()
        d = len(self.devices)
        if self._comms is None:
            arr = (ctypes.c_int * d)(*self.devices)
            comms = (ctypes.c_void_p * d)()
            R.check(L.ccb_comm_init_all(d, arr, comms))
            self._comms = [comms[i] for i in range(d)]
        inputs = list(inputs)
        keep = self._run_all_resident(inputs)
        outs_dev = [ob for _, ob in keep]
        result = {}
        for name in names:
            j = [k for k, (n, _, _) in enumerate(self.slots[0].outputs) if n == name][0]
            _, dt, shape = self.slots[0].outputs[j]
            R.check(L.ccb_group_start())
            for i, c in enumerate(self.slots):
                R.check(L.ccb_allreduce(self._comms[i], outs_dev[i][j].ptr, outs_dev[i][j].ptr, numel(shape),
                                        R.DT_CODE[dt.value], 0, c.lane_stream(0)))
            R.check(L.ccb_group_end())
        for i, c in enumerate(self.slots):
            B.check_device(c, c.lane_stream(0))
        for name in names:
            j = [k for k, (n, _, _) in enumerate(self.slots[0].outputs) if n == name][0]
            _, dt, shape = self.slots[0].outputs[j]
            host = np.empty(numel(shape), dtype=dt.np)
            with R.with_device(self.slots[0].device):
                outs_dev[0][j].download(host)
            result[name] = Value(dt, tuple(shape), host)
        self._free_resident(keep)
        return result

    def release(self):
        if not self.released:
            self.released = True
            for c in self.slots:
                B.release(c)
            for i, b in enumerate(self._mailboxes):
                with R.with_device(self.devices[i]):
                    b.free()
            self._mailboxes = []
            for ps in getattr(self, "_peer", None) or []:
                with R.with_device(self.devices[ps.rank]):
                    ps.close()
            self._peer = None
            if self._comms:
                for h in self._comms:
                    R.lib().ccb_comm_destroy(h)
                self._comms = None
