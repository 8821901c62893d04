"""The CUDA backend: the Python mirror of CUDACaml's ``Cudacaml_backend_cuda``
(lib/backend_cuda/cudacaml_backend_cuda.mli:1-84) over libccb.so.

``compile`` lowers the graph natively (fusion, skeleton selection, emission),
compiles it with NVRTC for sm_100a and allocates one buffer pool per stream;
``run`` uploads, launches and downloads on that stream. The same names and
semantics as the reference: ``compile``/``run``/``source``/``release``/
``compile_with``/``compile_on``/``device_of``/``run_async``/``wait`` and the
device-resident ``upload``/``download``/``free_resident``/``run_resident``.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import runtime as R
from .ir import Dtype, Graph, Value, numel
from .wire import to_wire

name = "cuda"

# Precision of F32 matmul nodes for graphs compiled without an explicit
# choice: "f32" (F32 arithmetic, as the reference) or "tf32" (tcgen05 tensor
# cores, TF32 operands, F32 accumulation). Like torch's allow_tf32 switch.
matmul_precision = "f32"


def set_matmul_precision(p: str) -> None:
    global matmul_precision
    to_wire(Graph("probe", []), p)  # validates the name
    matmul_precision = p


def _wire(graph: Graph, matmul, shard=None) -> bytes:
    return to_wire(graph, matmul or matmul_precision, shard).encode()

_CODE_DT = {0: Dtype.F32, 1: Dtype.F64, 2: Dtype.I32, 3: Dtype.I64}


def _io_specs(h, count_fn, get_fn):
    L = R.lib()
    n = ctypes.c_int()
    R.check(getattr(L, count_fn)(h, ctypes.byref(n)))
    out = []
    for i in range(n.value):
        nm = ctypes.c_char_p()
        dt = ctypes.c_int()
        rk = ctypes.c_int()
        dims = ctypes.POINTER(ctypes.c_longlong)()
        R.check(getattr(L, get_fn)(h, i, ctypes.byref(nm), ctypes.byref(dt), ctypes.byref(rk), ctypes.byref(dims)))
        shape = tuple(dims[k] for k in range(rk.value))
        out.append((nm.value.decode(), _CODE_DT[dt.value], shape))
    return out


class Compiled:
    """A program compiled for one device, with ``streams`` executors."""

    def __init__(self, graph: Graph, device: int, streams: int, matmul=None, shard=None):
        if streams < 1:
            raise ValueError("Backend_cuda.compile_on: streams must be >= 1")
        self.graph = graph
        self.device = device
        self.streams = streams
        self.next = 0
        h = ctypes.c_void_p()
        R.check(R.lib().ccb_program_create(_wire(graph, matmul, shard), device, streams, ctypes.byref(h)))
        self.h = h.value
        self.params = _io_specs(self.h, "ccb_program_num_params", "ccb_program_param")
        self.outputs = _io_specs(self.h, "ccb_program_num_outputs", "ccb_program_output")
        self.released = False

    def _check_live(self):
        if self.released:
            raise RuntimeError("Executor.run: this executor has been released")

    def __del__(self):
        try:
            release(self)
        except Exception:
            pass

    # -- introspection ------------------------------------------------------
    def num_kernels(self) -> int:
        n = ctypes.c_int()
        R.check(R.lib().ccb_program_num_kernels(self.h, ctypes.byref(n)))
        return n.value

    def num_launches(self) -> int:
        n = ctypes.c_int()
        R.check(R.lib().ccb_program_num_launches(self.h, ctypes.byref(n)))
        return n.value

    def plan(self) -> str:
        s = ctypes.c_char_p()
        R.check(R.lib().ccb_program_plan(self.h, ctypes.byref(s)))
        return s.value.decode()

    def lane_stream(self, lane: int = 0):
        s = ctypes.c_void_p()
        R.check(R.lib().ccb_program_lane_stream(self.h, lane, ctypes.byref(s)))
        return s.value


def _bind_inputs(c: Compiled, inputs):
    """Every param must be present with its dtype and shape before a byte is
    moved (lib/backend_cuda/executor.ml:14-21)."""
    got = dict(inputs)
    arrs = []
    for pname, dt, shape in c.params:
        if pname not in got:
            raise ValueError(f"Executor.run: missing input {pname}")
        v = got[pname]
        if v.dtype is not dt:
            raise ValueError(f"Executor.run: input {pname} has dtype {v.dtype.value}, expected {dt.value}")
        if tuple(v.shape) != tuple(shape):
            raise ValueError(f"Executor.run: input {pname} has shape {list(v.shape)}, expected {list(shape)}")
        arrs.append(np.ascontiguousarray(v.data))
    return arrs


def _ptr_array(ptrs):
    n = max(len(ptrs), 1)
    a = (ctypes.c_void_p * n)()
    for i, p in enumerate(ptrs):
        a[i] = p
    return a


def source(graph: Graph, matmul=None, shard=None) -> str:
    """The generated CUDA C++ for a graph, without compiling it."""
    h = ctypes.c_void_p()
    R.check(R.lib().ccb_program_lower(_wire(graph, matmul, shard), ctypes.byref(h)))
    try:
        s = ctypes.c_char_p()
        R.check(R.lib().ccb_program_source(h.value, ctypes.byref(s)))
        return s.value.decode()
    finally:
        R.lib().ccb_program_destroy(h.value)


def lower_info(graph: Graph, matmul=None, shard=None) -> dict:
    """Kernel count, launches per run and the host plan, without a device."""
    L = R.lib()
    h = ctypes.c_void_p()
    R.check(L.ccb_program_lower(_wire(graph, matmul, shard), ctypes.byref(h)))
    try:
        k = ctypes.c_int()
        n = ctypes.c_int()
        s = ctypes.c_char_p()
        src = ctypes.c_char_p()
        R.check(L.ccb_program_num_kernels(h.value, ctypes.byref(k)))
        R.check(L.ccb_program_num_launches(h.value, ctypes.byref(n)))
        R.check(L.ccb_program_plan(h.value, ctypes.byref(s)))
        R.check(L.ccb_program_source(h.value, ctypes.byref(src)))
        return {"kernels": k.value, "launches": n.value, "plan": s.value.decode(), "source": src.value.decode()}
    finally:
        L.ccb_program_destroy(h.value)


def compile_on(device: int, graph: Graph, streams: int = 1, matmul=None, shard=None) -> Compiled:
    """``shard=(rank, world)``: rank ``rank`` of a sharded Monte-Carlo
    program (bind_peers before the first run)."""
    return Compiled(graph, device, streams, matmul, shard)


def shard_of(c: Compiled) -> tuple[int, int]:
    """(rank, world) of a sharded program; (0, 1) otherwise."""
    r, w = ctypes.c_int(), ctypes.c_int()
    R.check(R.lib().ccb_program_shard(c.h, ctypes.byref(r), ctypes.byref(w)))
    return r.value, w.value


def mailbox_bytes(c: Compiled) -> int:
    """Bytes of one rank's mailbox for a sharded program (0 otherwise)."""
    n = ctypes.c_size_t()
    R.check(R.lib().ccb_program_mailbox_bytes(c.h, ctypes.byref(n)))
    return n.value


def bind_peers(c: Compiled, mailboxes) -> None:
    """Bind every rank's mailbox (device pointers as this rank addresses
    them, rank order) to a sharded program; each owner zero-fills its own
    before any rank's first run."""
    arr = (ctypes.c_void_p * max(len(mailboxes), 1))(*mailboxes)
    R.check(R.lib().ccb_program_bind_peers(c.h, arr, len(mailboxes)))


def compile_with(streams: int, graph: Graph, matmul=None) -> Compiled:
    return Compiled(graph, 0, streams, matmul)


def compile(graph: Graph, matmul=None) -> Compiled:  # noqa: A001 - Backend.S.compile
    return Compiled(graph, 0, 1, matmul)


def device_of(c: Compiled) -> int:
    return c.device


def release(c: Compiled) -> None:
    """Frees the device buffers; idempotent; run after it raises."""
    if not getattr(c, "released", True) and R._LIB is not None:
        c.released = True
        R.lib().ccb_program_destroy(c.h)
        c.h = None


class Job:
    """An issued run; ``wait`` blocks and returns its outputs (the job keeps
    its host inputs and outputs alive until then)."""

    def __init__(self, c: Compiled, lane: int, keep, outs):
        self.c = c
        self.lane = lane
        self.keep = keep
        self.outs = outs
        self.done = None


def run_async(c: Compiled, inputs) -> Job:
    c._check_live()
    arrs = _bind_inputs(c, inputs)
    outs = [(n, Value(dt, shape, np.empty(numel(shape), dtype=dt.np))) for n, dt, shape in c.outputs]
    lane = c.next
    c.next = (c.next + 1) % c.streams
    ins = _ptr_array([a.ctypes.data for a in arrs])
    ops = _ptr_array([v.data.ctypes.data for _, v in outs])
    R.check(R.lib().ccb_program_enqueue(c.h, lane, ins, ops))
    return Job(c, lane, (arrs, ins, ops), outs)


def wait(j: Job):
    if j.done is None:
        R.check(R.lib().ccb_program_wait(j.c.h, j.lane))
        j.done = j.outs
        j.keep = None
    return j.done


def run(c: Compiled, inputs):
    """Synchronous, on lane 0 (Backend.S.run)."""
    c._check_live()
    arrs = _bind_inputs(c, inputs)
    outs = [(n, Value(dt, shape, np.empty(numel(shape), dtype=dt.np))) for n, dt, shape in c.outputs]
    ins = _ptr_array([a.ctypes.data for a in arrs])
    ops = _ptr_array([v.data.ctypes.data for _, v in outs])
    R.check(R.lib().ccb_program_run(c.h, ins, ops))
    return outs


# ---------------------------------------------------------------------------
# Device-resident values
# ---------------------------------------------------------------------------
@dataclass
class Resident:
    buf: R.Buffer
    dtype: Dtype
    shape: tuple
    device: int = 0


def upload(v: Value, device: int = 0) -> Resident:
    with R.with_device(device):
        b = R.Buffer(v.byte_size)
        b.upload(v.data)
    return Resident(b, v.dtype, tuple(v.shape), device)


def download(r: Resident) -> Value:
    out = Value.create(r.dtype, r.shape)
    with R.with_device(r.device):
        r.buf.download(out.data)
    return out


def free_resident(r: Resident) -> None:
    with R.with_device(r.device):
        r.buf.free()


def run_resident(c: Compiled, inputs):
    """Device in, device out, zero-copy; synchronises before returning."""
    c._check_live()
    got = dict(inputs)
    ptrs = []
    for pname, dt, shape in c.params:
        if pname not in got:
            raise ValueError(f"Executor.run_resident: missing input {pname}")
        r = got[pname]
        want = numel(shape) * dt.size_in_bytes
        if r.buf.nbytes != want:
            raise ValueError(f"Executor.run_resident: input {pname} is {r.buf.nbytes} bytes, parameter needs {want}")
        ptrs.append(r.buf.ptr)
    with R.with_device(c.device):
        outs = [(n, Resident(R.Buffer(numel(shape) * dt.size_in_bytes), dt, shape, c.device)) for n, dt, shape in c.outputs]
        ins = _ptr_array(ptrs)
        ops = _ptr_array([r.buf.ptr for _, r in outs])
        R.check(R.lib().ccb_program_run_device(c.h, 0, ins, ops, None))
        R.check(R.lib().ccb_program_check(c.h, 0, None))
    return outs


def run_device_ptrs(c: Compiled, in_ptrs, out_ptrs, stream=None, lane: int = 0) -> None:
    """Lowest-level resident run on raw device pointers (param order in,
    output order out), issued on ``stream`` without synchronising."""
    R.check(R.lib().ccb_program_run_device(c.h, lane, _ptr_array(in_ptrs), _ptr_array(out_ptrs), stream))


def run_device_ptrs_events(c: Compiled, in_ptrs, out_ptrs, events, stream=None, lane: int = 0) -> None:
    """run_device_ptrs, recording events[j] (an R.Event or None) on `stream`
    as soon as output j is final, so that another stream can wait on it."""
    hs = [e.h if e is not None else None for e in events]
    R.check(R.lib().ccb_program_run_device_events(c.h, lane, _ptr_array(in_ptrs), _ptr_array(out_ptrs), stream,
                                                  _ptr_array(hs)))


def check_device(c: Compiled, stream=None, lane: int = 0) -> None:
    R.check(R.lib().ccb_program_check(c.h, lane, stream))
