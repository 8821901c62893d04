"""ORACLE -- test infrastructure only. The product never imports this module;
tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline leg use it
as the checker.

``Backend.S`` instance "interp" over liboracle.so, the C++ restatement of the
reference interpreter (lib/backend_interp/cudacaml_backend_interp.ml:3-7,
452-457). ``compile`` parses the graph, ``run`` evaluates it single-threaded,
element at a time, exactly as the reference interpreter does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

from cudacaml_b200.ir import Dtype, Graph, Value
from cudacaml_b200.wire import to_wire

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_DT_CODE = {Dtype.F32: 0, Dtype.F64: 1, Dtype.I32: 2, Dtype.I64: 3}
_CODE_DT = {v: k for k, v in _DT_CODE.items()}


class InterpError(ValueError):
    """Invalid_argument from the interpreter (missing input, bad index...)."""


class InterpDivisionByZero(ArithmeticError):
    pass


def build() -> str:
    """Compile liboracle.so in place (g++ is part of the image)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return os.path.join(_HERE, "liboracle.so")


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(os.path.join(_HERE, "interp.cpp")):
            build()
        L = ctypes.CDLL(path)
        L.ccbo_load.restype = ctypes.c_void_p
        L.ccbo_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
        L.ccbo_free.argtypes = [ctypes.c_void_p]
        L.ccbo_run.restype = ctypes.c_int
        L.ccbo_run.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                               ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                               ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_void_p),
                               ctypes.c_char_p, ctypes.c_int]
        for f, r in (("ccbo_num_outputs", ctypes.c_int), ("ccbo_output_name", ctypes.c_char_p),
                     ("ccbo_output_dtype", ctypes.c_int), ("ccbo_output_rank", ctypes.c_int),
                     ("ccbo_output_data", ctypes.c_void_p), ("ccbo_output_bytes", ctypes.c_longlong)):
            getattr(L, f).restype = r
        L.ccbo_num_outputs.argtypes = [ctypes.c_void_p]
        for f in ("ccbo_output_name", "ccbo_output_dtype", "ccbo_output_rank", "ccbo_output_data",
                  "ccbo_output_bytes"):
            getattr(L, f).argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.ccbo_output_dim.restype = ctypes.c_longlong
        L.ccbo_output_dim.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.ccbo_philox4x32_10.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32),
                                         ctypes.POINTER(ctypes.c_uint32)]
        L.ccbo_erfinv.restype = ctypes.c_double
        L.ccbo_erfinv.argtypes = [ctypes.c_double]
        _LIB = L
    return _LIB


class Compiled:
    def __init__(self, graph: Graph):
        self.graph = graph
        err = ctypes.create_string_buffer(1024)
        h = lib().ccbo_load(to_wire(graph).encode(), err, 1024)
        if not h:
            raise InterpError(err.value.decode())
        self.h = h

    def __del__(self):
        h = getattr(self, "h", None)
        if h and _LIB is not None:
            _LIB.ccbo_free(h)
            self.h = None


name = "interp"


def compile(graph: Graph) -> Compiled:  # noqa: A001 - Backend.S.compile
    return Compiled(graph)


def run(c: Compiled, inputs):
    """Inputs keyed by param name; outputs in Graph.outputs order."""
    L = lib()
    inputs = list(inputs)
    n = len(inputs)
    names = (ctypes.c_char_p * max(n, 1))()
    dts = (ctypes.c_int * max(n, 1))()
    ranks = (ctypes.c_int * max(n, 1))()
    dims = []
    ptrs = (ctypes.c_void_p * max(n, 1))()
    keep = []
    for k, (nm, v) in enumerate(inputs):
        names[k] = nm.encode()
        dts[k] = _DT_CODE[v.dtype]
        ranks[k] = len(v.shape)
        dims.extend(v.shape)
        a = np.ascontiguousarray(v.data)
        keep.append(a)
        ptrs[k] = a.ctypes.data
    cdims = (ctypes.c_longlong * max(len(dims), 1))(*dims)
    err = ctypes.create_string_buffer(2048)
    rc = L.ccbo_run(c.h, n, names, dts, ranks, cdims, ptrs, err, 2048)
    if rc == 1:
        raise InterpError(err.value.decode())
    if rc == 2:
        raise InterpDivisionByZero(err.value.decode())
    if rc != 0:
        raise RuntimeError(err.value.decode())
    outs = []
    for i in range(L.ccbo_num_outputs(c.h)):
        dt = _CODE_DT[L.ccbo_output_dtype(c.h, i)]
        shape = tuple(L.ccbo_output_dim(c.h, i, k) for k in range(L.ccbo_output_rank(c.h, i)))
        nbytes = L.ccbo_output_bytes(c.h, i)
        buf = ctypes.string_at(L.ccbo_output_data(c.h, i), nbytes) if nbytes else b""
        arr = np.frombuffer(buf, dtype=dt.np).copy()
        outs.append((L.ccbo_output_name(c.h, i).decode(), Value(dt, shape, arr)))
    return outs


def philox4x32_10(ctr, key):
    L = lib()
    c = (ctypes.c_uint32 * 4)(*[x & 0xFFFFFFFF for x in ctr])
    k = (ctypes.c_uint32 * 2)(*[x & 0xFFFFFFFF for x in key])
    o = (ctypes.c_uint32 * 4)()
    L.ccbo_philox4x32_10(c, k, o)
    return list(o)


def erfinv(x: float) -> float:
    return lib().ccbo_erfinv(float(x))
