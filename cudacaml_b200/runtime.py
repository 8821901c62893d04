"""ctypes bindings to libccb.so, the C-ABI of this backend (include/ccb.h).

The Python mirror of the reference's ``lib/runtime`` modules
(device/buffer/stream/event/jit/launch/pinned): every call goes straight to
the C-ABI, which is what an OCaml ``ctypes`` binding of the same library would
call. There is no fallback: if the library is missing, importing the backend
fails loudly.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libccb.so")
_LIB = None

CCB_OK = 0
ERR_NAMES = {1: "invalid", 2: "no device", 3: "driver", 4: "compile", 5: "nccl", 6: "device check", 7: "unsupported"}

DT_CODE = {"f32": 0, "f64": 1, "i32": 2, "i64": 3}


class CcbError(RuntimeError):
    """A failing libccb call; ``code`` is the CCB_ERR_* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{ERR_NAMES.get(code, code)}] {msg}")
        self.code = code


class CcbInvalid(CcbError, ValueError):
    """Caller mistakes map to ValueError, like the reference's Invalid_argument."""


def build(force: bool = False) -> str:
    """Compile libccb.so in place with the committed Makefile."""
    csrc = os.path.join(_HERE, "csrc")
    args = ["make", "-s", "-C", csrc]
    if force:
        subprocess.run(args + ["clean"], check=True)
    subprocess.run(args, check=True)
    return LIB_PATH


def _declare(L):
    c = ctypes
    P = c.c_void_p
    I = c.c_int
    SZ = c.c_size_t
    sigs = {
        "ccb_last_error": (c.c_char_p, []),
        "ccb_version": (c.c_char_p, []),
        "ccb_available": (I, []),
        "ccb_init": (I, []),
        "ccb_device_count": (I, [c.POINTER(I)]),
        "ccb_set_device": (I, [I]),
        "ccb_get_device": (I, [c.POINTER(I)]),
        "ccb_device_info": (I, [I, P]),
        "ccb_device_synchronize": (I, []),
        "ccb_malloc": (I, [SZ, c.POINTER(P)]),
        "ccb_free": (I, [P]),
        "ccb_live_count": (I, [c.POINTER(c.c_longlong)]),
        "ccb_memcpy_h2d": (I, [P, P, SZ, P]),
        "ccb_memcpy_d2h": (I, [P, P, SZ, P]),
        "ccb_memcpy_d2d": (I, [P, P, SZ, P]),
        "ccb_memset_d8": (I, [P, c.c_ubyte, SZ, P]),
        "ccb_host_alloc": (I, [SZ, c.POINTER(P)]),
        "ccb_host_free": (I, [P]),
        "ccb_stream_create": (I, [c.POINTER(P)]),
        "ccb_stream_destroy": (I, [P]),
        "ccb_stream_synchronize": (I, [P]),
        "ccb_stream_query": (I, [P, c.POINTER(I)]),
        "ccb_event_create": (I, [c.POINTER(P)]),
        "ccb_event_destroy": (I, [P]),
        "ccb_event_record": (I, [P, P]),
        "ccb_event_synchronize": (I, [P]),
        "ccb_event_elapsed_ms": (I, [P, P, c.POINTER(c.c_float)]),
        "ccb_stream_wait_event": (I, [P, P]),
        "ccb_module_compile": (I, [c.c_char_p, c.c_char_p, c.POINTER(P), c.POINTER(c.c_void_p)]),
        "ccb_module_unload": (I, [P]),
        "ccb_module_get_function": (I, [P, c.c_char_p, c.POINTER(P)]),
        "ccb_launch": (I, [P, c.c_uint, c.c_uint, c.c_uint, c.c_uint, c.c_uint, c.c_uint, c.c_uint, P, c.POINTER(P), I]),
        "ccb_nvrtc_check": (I, [c.c_char_p, c.c_char_p, c.POINTER(SZ), c.POINTER(c.c_void_p)]),
        "ccb_free_string": (None, [c.c_void_p]),
        "ccb_program_create": (I, [c.c_char_p, I, I, c.POINTER(P)]),
        "ccb_program_lower": (I, [c.c_char_p, c.POINTER(P)]),
        "ccb_program_destroy": (I, [P]),
        "ccb_program_source": (I, [P, c.POINTER(c.c_char_p)]),
        "ccb_program_device": (I, [P, c.POINTER(I)]),
        "ccb_program_num_kernels": (I, [P, c.POINTER(I)]),
        "ccb_program_num_launches": (I, [P, c.POINTER(I)]),
        "ccb_program_plan": (I, [P, c.POINTER(c.c_char_p)]),
        "ccb_program_num_params": (I, [P, c.POINTER(I)]),
        "ccb_program_param": (I, [P, I, c.POINTER(c.c_char_p), c.POINTER(I), c.POINTER(I),
                                  c.POINTER(c.POINTER(c.c_longlong))]),
        "ccb_program_num_outputs": (I, [P, c.POINTER(I)]),
        "ccb_program_output": (I, [P, I, c.POINTER(c.c_char_p), c.POINTER(I), c.POINTER(I),
                                   c.POINTER(c.POINTER(c.c_longlong))]),
        "ccb_program_enqueue": (I, [P, I, c.POINTER(P), c.POINTER(P)]),
        "ccb_program_wait": (I, [P, I]),
        "ccb_program_run": (I, [P, c.POINTER(P), c.POINTER(P)]),
        "ccb_program_run_device": (I, [P, I, c.POINTER(P), c.POINTER(P), P]),
        "ccb_program_check": (I, [P, I, P]),
        "ccb_program_run_device_events": (I, [P, I, c.POINTER(P), c.POINTER(P), P, c.POINTER(P)]),
        "ccb_program_lane_stream": (I, [P, I, c.POINTER(P)]),
        "ccb_program_shard": (I, [P, c.POINTER(I), c.POINTER(I)]),
        "ccb_program_mailbox_bytes": (I, [P, c.POINTER(SZ)]),
        "ccb_program_bind_peers": (I, [P, c.POINTER(P), I]),
        "ccb_comm_init_all": (I, [I, c.POINTER(I), c.POINTER(P)]),
        "ccb_comm_unique_id": (I, [c.POINTER(c.c_ubyte)]),
        "ccb_comm_init_rank": (I, [I, c.POINTER(c.c_ubyte), I, c.POINTER(P)]),
        "ccb_comm_destroy": (I, [P]),
        "ccb_allreduce": (I, [P, P, P, SZ, I, I, P]),
        "ccb_sum_f32_noalloc": (I, [P, c.c_longlong, P, P]),
        "ccb_ipc_mem_handle": (I, [P, c.POINTER(c.c_ubyte)]),
        "ccb_ipc_mem_open": (I, [c.POINTER(c.c_ubyte), c.POINTER(P)]),
        "ccb_ipc_mem_close": (I, [P]),
        "ccb_peer_access_enable": (I, [I]),
        "ccb_xrank_mailbox_bytes": (I, [I, c.POINTER(SZ)]),
        "ccb_xrank_sum": (I, [P, P, I, I, I, I, c.POINTER(P), c.c_ulonglong, P, P]),
        "ccb_group_start": (I, []),
        "ccb_group_end": (I, []),
        "ccb_graph_begin": (I, [P]),
        "ccb_graph_end": (I, [P, c.POINTER(P)]),
        "ccb_graph_launch": (I, [P, P]),
        "ccb_graph_destroy": (I, [P]),
    }
    for name, (res, args) in sigs.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    return sigs


def lib():
    """The loaded library. Raises if libccb.so has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libccb.so is not built at {LIB_PATH}; run cudacaml_b200.runtime.build()")
        _preload_nccl()
        L = ctypes.CDLL(LIB_PATH)
        _declare(L)
        _LIB = L
    return _LIB


def _preload_nccl():
    """Load the NCCL that torch links against (the nvidia-nccl wheel), if it is
    installed, before libccb.so opens one: libccb.so then reuses it, and a
    later `import torch` in the same process does not find an older system
    libnccl.so.2 already bound to the name."""
    try:
        import importlib.util
        spec = importlib.util.find_spec("nvidia.nccl")
    except (ImportError, ValueError):
        return
    for d in (spec.submodule_search_locations or []) if spec else []:
        path = os.path.join(d, "lib", "libnccl.so.2")
        if os.path.exists(path):
            try:
                ctypes.CDLL(path, mode=ctypes.RTLD_GLOBAL)
            except OSError:
                pass
            return


def exported_symbols():
    """Names this module binds (every entry point of include/ccb.h)."""
    lib()
    return list(_declare(_LIB).keys())


def check(rc: int) -> None:
    if rc != CCB_OK:
        msg = lib().ccb_last_error().decode(errors="replace")
        if rc == 1:
            raise CcbInvalid(rc, msg)
        raise CcbError(rc, msg)


# ---------------------------------------------------------------------------
# Device (lib/runtime/device.mli)
# ---------------------------------------------------------------------------
class DeviceInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 256), ("cc_major", ctypes.c_int), ("cc_minor", ctypes.c_int),
                ("multiprocessors", ctypes.c_int), ("total_memory_bytes", ctypes.c_longlong)]


def available() -> bool:
    return bool(lib().ccb_available())


def init() -> None:
    check(lib().ccb_init())


def count() -> int:
    n = ctypes.c_int()
    check(lib().ccb_device_count(ctypes.byref(n)))
    return n.value


def set_device(ordinal: int) -> None:
    check(lib().ccb_set_device(ordinal))


def current() -> int:
    n = ctypes.c_int()
    check(lib().ccb_get_device(ctypes.byref(n)))
    return n.value


class with_device:
    """Context manager: make ``ordinal``'s primary context current, restore the
    previous device afterwards (lib/runtime/device.ml:68-79)."""

    def __init__(self, ordinal: int):
        self.ordinal = ordinal

    def __enter__(self):
        self.prev = current()
        set_device(self.ordinal)
        return self

    def __exit__(self, *exc):
        set_device(self.prev)
        return False


def info(ordinal: int = 0) -> dict:
    d = DeviceInfo()
    check(lib().ccb_device_info(ordinal, ctypes.byref(d)))
    return {"name": d.name.decode(), "compute_capability": (d.cc_major, d.cc_minor),
            "multiprocessors": d.multiprocessors, "total_memory_bytes": d.total_memory_bytes}


def info_to_string(i: dict) -> str:
    """The reference's grep-able format (lib/runtime/device.mli)."""
    ma, mi = i["compute_capability"]
    return (f"device: {i['name']}\ncompute: sm_{ma}{mi}\nmultiprocessors: {i['multiprocessors']}\n"
            f"memory_mib: {i['total_memory_bytes'] // 1048576}\n")


def synchronize() -> None:
    check(lib().ccb_device_synchronize())


def live_count() -> int:
    n = ctypes.c_longlong()
    check(lib().ccb_live_count(ctypes.byref(n)))
    return n.value


# ---------------------------------------------------------------------------
# Streams and events (lib/runtime/stream.mli, event.mli)
# ---------------------------------------------------------------------------
class Stream:
    def __init__(self):
        h = ctypes.c_void_p()
        check(lib().ccb_stream_create(ctypes.byref(h)))
        self.h = h.value

    def synchronize(self):
        check(lib().ccb_stream_synchronize(self.h))

    def is_idle(self) -> bool:
        i = ctypes.c_int()
        check(lib().ccb_stream_query(self.h, ctypes.byref(i)))
        return bool(i.value)

    def destroy(self):
        if self.h:
            check(lib().ccb_stream_destroy(self.h))
            self.h = None


class Graph:
    """Work captured from a stream and replayed with one launch (a CUDA
    graph). ``with Graph.capture(stream) as g: ...issue work on stream...``
    then ``g.launch(stream)`` any number of times; ``destroy`` frees it."""

    def __init__(self, h):
        self.h = h

    @staticmethod
    def capture(stream):
        return _Capture(stream)

    def launch(self, stream):
        check(lib().ccb_graph_launch(self.h, stream.h if isinstance(stream, Stream) else stream))

    def destroy(self):
        if self.h:
            check(lib().ccb_graph_destroy(self.h))
            self.h = None


class _Capture:
    def __init__(self, stream):
        self.stream = stream.h if isinstance(stream, Stream) else stream
        self.graph = None

    def __enter__(self):
        check(lib().ccb_graph_begin(self.stream))
        self.graph = Graph(None)
        return self.graph

    def __exit__(self, et, ev, tb):
        h = ctypes.c_void_p()
        rc = lib().ccb_graph_end(self.stream, ctypes.byref(h))
        if et is None:
            check(rc)
            self.graph.h = h.value
        elif rc == 0 and h.value:  # the capture ended; drop what it held
            lib().ccb_graph_destroy(h.value)
        return False


class Event:
    def __init__(self):
        h = ctypes.c_void_p()
        check(lib().ccb_event_create(ctypes.byref(h)))
        self.h = h.value

    def record(self, stream=None):
        check(lib().ccb_event_record(self.h, stream.h if isinstance(stream, Stream) else stream))

    def synchronize(self):
        check(lib().ccb_event_synchronize(self.h))

    def elapsed_ms(self, end: "Event") -> float:
        f = ctypes.c_float()
        check(lib().ccb_event_elapsed_ms(self.h, end.h, ctypes.byref(f)))
        return f.value

    def destroy(self):
        if self.h:
            check(lib().ccb_event_destroy(self.h))
            self.h = None


# ---------------------------------------------------------------------------
# Memory (lib/runtime/buffer.mli, pinned.mli)
# ---------------------------------------------------------------------------
class Buffer:
    """Device memory on the current device: an opaque pointer plus a byte count."""

    def __init__(self, nbytes: int):
        p = ctypes.c_void_p()
        check(lib().ccb_malloc(nbytes, ctypes.byref(p)))
        self.ptr = p.value
        self.nbytes = nbytes

    def free(self):
        if self.ptr:
            check(lib().ccb_free(self.ptr))
            self.ptr = None

    def upload(self, arr, stream=None):
        import numpy as np
        a = np.ascontiguousarray(arr)
        if a.nbytes != self.nbytes:
            raise ValueError(f"Buffer.upload: {a.nbytes} bytes into a {self.nbytes}-byte buffer")
        check(lib().ccb_memcpy_h2d(self.ptr, a.ctypes.data, a.nbytes, stream))
        if stream is None:
            check(lib().ccb_stream_synchronize(None))

    def download(self, arr, stream=None):
        if arr.nbytes != self.nbytes:
            raise ValueError(f"Buffer.download: {self.nbytes} bytes into a {arr.nbytes}-byte array")
        check(lib().ccb_memcpy_d2h(arr.ctypes.data, self.ptr, self.nbytes, stream))
        if stream is None:
            check(lib().ccb_stream_synchronize(None))


def pinned_empty(shape, dtype):
    """A numpy array in page-locked memory (cuMemHostAlloc PORTABLE), freed
    when the array is garbage collected (lib/runtime/pinned.ml:76-108)."""
    import numpy as np
    dt = np.dtype(dtype)
    n = int(np.prod(shape)) if len(shape) else 1
    nbytes = max(n * dt.itemsize, 1)
    p = ctypes.c_void_p()
    check(lib().ccb_host_alloc(nbytes, ctypes.byref(p)))
    buf = (ctypes.c_byte * nbytes).from_address(p.value)
    arr = np.frombuffer(buf, dtype=dt, count=n).reshape(shape)
    holder = _PinnedHolder(p.value)
    arr_base = arr
    # keep the holder alive as long as the array lives
    _PINNED_OWNERS[id(buf)] = holder
    import weakref
    weakref.finalize(buf, _release_pinned, id(buf))
    return arr_base


class _PinnedHolder:
    def __init__(self, ptr):
        self.ptr = ptr


_PINNED_OWNERS = {}


def _release_pinned(key):
    h = _PINNED_OWNERS.pop(key, None)
    if h is not None and _LIB is not None:
        _LIB.ccb_host_free(h.ptr)
