"""Seeded random graphs and zero-size tensors through the native lowering,
NVRTC for sm_100a and the oracle, and mutated wire text through both parsers.

Every random graph must lower; a sample of them must compile for sm_100a;
the oracle must evaluate them, outputs in the graph's order. Mutated graph
text must come back as either a lowered program or an error status, never a
crash. CPU only.
"""
import ctypes
import random

import numpy as np
import pytest

from cudacaml_b200 import backend_cuda as B
from cudacaml_b200 import dsl as D
from cudacaml_b200 import runtime as R
from cudacaml_b200.ir import F32, F64, I32, Graph, Value
from cudacaml_b200.wire import to_wire
from oracle import interp as I

UNARY = [D.neg, D.sqrt, D.exp, D.log, D.sin, D.cos, D.erf]
BINARY_F = [D.add, D.sub, D.mul, D.div, D.min, D.max]
BINARY_I = [D.add, D.sub, D.mul, D.bit_and, D.bit_or, D.bit_xor, D.min, D.max]


def element(rnd, dt, a, b=None):
    if dt is I32:
        if b is None:
            return D.add(D.mul(a, D.const(I32, rnd.randint(-3, 3))), D.index())
        return rnd.choice(BINARY_I)(a, b)
    if b is None:
        r = rnd.random()
        if r < 0.3:
            return D.select(D.lt(a, D.const(dt, 0.0)), D.neg(a), a)
        if r < 0.7:
            return rnd.choice(UNARY)(D.abs(a))
        return D.mul(a, D.const(dt, rnd.uniform(-2.0, 2.0)))
    return rnd.choice(BINARY_F)(a, b)


def random_graph(rnd, gi):
    """Maps, map2s, flat and row reductions and scans, broadcasts of
    reductions, transposes, gathers, scatters, small products and reshapes
    over one dtype, with several outputs."""
    dt = rnd.choice([F32, F64, I32])
    rows, cols = rnd.choice([1, 2, 3, 7, 33, 100]), rnd.choice([1, 4, 5, 31, 64, 129])
    n = rows * cols
    params = {}

    def param(name, shape):
        t = D.param(name, dt, shape)
        params[name] = shape
        return t

    zero = D.const(dt, 0)
    pool = [param("x", (n,)), param("y", (n,)), param("m", (rows, cols))]
    outs = []
    for step in range(rnd.randint(1, 6)):
        src = rnd.choice(pool)
        flat = src if len(src.shape) == 1 else D.reshape((int(np.prod(src.shape)),), src)
        k = rnd.random()
        if k < 0.25:
            t = D.map(lambda a: element(rnd, dt, a), src)
        elif k < 0.45:
            other = rnd.choice([p for p in pool if p.shape == src.shape])
            t = D.map2(lambda a, b: element(rnd, dt, a, b), src, other)
        elif k < 0.55:
            t = D.reduce(D.add if rnd.random() < 0.7 else D.max, zero, src)
            if rnd.random() < 0.5:
                t = D.broadcast((n,), t)
        elif k < 0.63:
            t = D.scan(D.add, zero, src)
        elif k < 0.71 and len(src.shape) == 2:
            t = (D.reduce_rows if rnd.random() < 0.5 else D.scan_rows)(D.add, zero, src)
        elif k < 0.77 and len(src.shape) == 2:
            t = D.transpose(src)
        elif k < 0.83:
            m = flat.shape[0]
            t = D.gather(D.map(lambda i: D.sub(D.const(I32, m - 1), i), D.iota((min(m, 17),))), flat)
        elif k < 0.88:
            t = D.scatter_add(D.map(lambda i: D.bit_and(i, D.const(I32, 7)), D.iota(flat.shape)), flat, (8,))
        elif k < 0.94 and dt is not I32 and len(src.shape) == 2:
            t = D.matmul(src, param(f"w{step}", (src.shape[1], rnd.choice([1, 3, 16, 33]))))
        else:
            t = flat if len(src.shape) == 2 else D.reshape((rows, cols), src) if src.shape == (n,) else src
        pool.append(t)
        if rnd.random() < 0.6:
            outs.append((f"o{step}", t))
    if not outs:
        outs.append(("o", pool[-1]))
    return Graph(f"rand{gi}", outs), params, dt


def random_inputs(rnd, params, dt):
    r = np.random.default_rng(rnd.randint(0, 1 << 30))
    ins = []
    for name, shape in params.items():
        k = int(np.prod(shape))
        a = r.integers(-50, 50, size=k).astype(np.int32) if dt is I32 else r.uniform(-2, 2, size=k).astype(dt.np)
        ins.append((name, Value.of_array(dt, shape, a)))
    return ins


def mutate(rnd, text: str) -> bytes:
    b = bytearray(text.encode())
    for _ in range(rnd.randint(1, 4)):
        if not b:
            break
        i = rnd.randrange(len(b))
        r = rnd.random()
        if r < 0.3:
            b[i] = rnd.randrange(32, 127)
        elif r < 0.5:
            del b[i:i + rnd.randint(1, 20)]
        elif r < 0.7:
            b[i:i] = rnd.choice([b" -1", b" 999999999999", b"%", b"\n", b" 0", b" nan", b"t 1 f32 1 4 param x\n"])
        else:
            j = rnd.randrange(len(b))
            b[i], b[j] = b[j], b[i]
    return bytes(b)


def nvrtc_compiles(g):
    L = R.lib()
    h = ctypes.c_void_p()
    R.check(L.ccb_program_lower(to_wire(g).encode(), ctypes.byref(h)))
    try:
        src = ctypes.c_char_p()
        R.check(L.ccb_program_source(h, ctypes.byref(src)))
        sz, log = ctypes.c_size_t(), ctypes.c_void_p()
        rc = L.ccb_nvrtc_check(src.value, g.name.encode(), ctypes.byref(sz), ctypes.byref(log))
        if log.value:
            L.ccb_free_string(log)
        assert rc == 0, L.ccb_last_error().decode()[:3000]
        assert sz.value > 0
    finally:
        L.ccb_program_destroy(h)


@pytest.mark.parametrize("seed", [11, 12, 13])
def test_random_graphs_lower_compile_and_evaluate(seed):
    rnd = random.Random(seed)
    for gi in range(40):
        g, params, dt = random_graph(rnd, gi)
        info = B.lower_info(g)
        assert info["kernels"] >= 0 and info["plan"].rstrip().endswith(tuple(f"-> {n}" for n, _ in g.outputs))
        if gi % 10 == 0:
            nvrtc_compiles(g)
        try:
            out = I.run(I.compile(g), random_inputs(rnd, params, dt))
            assert [n for n, _ in out] == [n for n, _ in g.outputs]
        except I.InterpDivisionByZero:
            pass


@pytest.mark.parametrize("seed", [21, 22])
def test_mutated_wire_text_is_lowered_or_refused(seed):
    rnd = random.Random(seed)
    L = R.lib()
    refused = 0
    for gi in range(30):
        text = to_wire(random_graph(rnd, gi)[0])
        for _ in range(10):
            m = mutate(rnd, text)
            h = ctypes.c_void_p()
            rc = L.ccb_program_lower(m, ctypes.byref(h))
            if rc == 0:
                L.ccb_program_destroy(h)
            else:
                refused += 1
                assert L.ccb_last_error()  # every refusal carries a message
            err = ctypes.create_string_buffer(1024)
            p = I.lib().ccbo_load(m, err, 1024)
            if p:
                I.lib().ccbo_free(p)
            else:
                assert err.value
    assert refused > 0


def zero_size_graphs():
    z = D.const(F32, 0.0)
    x0 = D.param("x", F32, (0,))
    out = [("map", Graph("g", [("r", D.map(D.neg, x0)), ("s", D.reduce(D.add, D.const(F32, 5.0), x0))])),
           ("scan", Graph("g", [("p", D.scan(D.add, z, x0))])),
           ("gather", Graph("g", [("r", D.gather(D.param("i", I32, (0,)), D.param("x", F32, (5,))))])),
           ("scatter", Graph("g", [("h", D.scatter_add(D.param("i", I32, (0,)), x0, (4,)))]))]
    for r, c in ((0, 4), (4, 0), (0, 0)):
        m = D.param("m", F32, (r, c))
        out.append((f"rows{r}x{c}", Graph("g", [("r", D.reduce_rows(D.add, D.const(F32, 2.0), m)),
                                                  ("q", D.scan_rows(D.add, z, m)), ("t", D.transpose(m))])))
    for mm, k, n in ((0, 4, 3), (3, 0, 3), (3, 4, 0), (256, 0, 256)):
        out.append((f"matmul{mm}x{k}x{n}", Graph("g", [("c", D.matmul(D.param("a", F32, (mm, k)),
                                                                      D.param("b", F32, (k, n))))])))
    return out


@pytest.mark.parametrize("name,g", zero_size_graphs(), ids=[n for n, _ in zero_size_graphs()])
def test_zero_size_tensors_lower_compile_and_evaluate(name, g):
    # the reference's rules at size 0: a reduction is its init (row by row
    # for [rows; 0]), a product over K = 0 is zeros, everything else is empty
    assert B.lower_info(g)["kernels"] >= 1
    nvrtc_compiles(g)
    out = dict(I.run(I.compile(g), [(n, Value.create(t.dtype, t.shape)) for n, t in g.params]))
    if name == "map":
        assert out["r"].shape == (0,) and out["s"].to_list() == [5.0]
    if name == "rows4x0":
        assert out["r"].to_list() == [2.0] * 4 and out["q"].shape == (4, 0) and out["t"].shape == (0, 4)
    if name.startswith("matmul"):
        assert not np.any(out["c"].data)


def _kernel_io(src):
    """{kernel: (nodes it reads, nodes it writes)} from the generated source:
    a pass reads node t through a `const T* b<t>` field of its parameter
    block and writes it through a `T* o<t>` field."""
    import re
    io, cur, fields = {}, None, {}
    for line in src.splitlines():
        m = re.match(r"struct (F\d+) \{", line)
        if m:
            cur = m.group(1)
            fields[cur] = (set(), set())
            continue
        m = re.match(r"\s+const \w[\w ]*\* __restrict__ b(\d+);", line)
        if m and cur:
            fields[cur][0].add(int(m.group(1)))
            continue
        m = re.match(r"\s+\w[\w ]*\* __restrict__ o(\d+);", line)
        if m and cur:
            fields[cur][1].add(int(m.group(1)))
            continue
        m = re.search(r'extern "C" __global__ .* (ccb_\w+)\(const (?:__grid_constant__ )?(F\d+)::P p\)', line)
        if m:
            io[m.group(1)] = fields.get(m.group(2), (set(), set()))
    return io


@pytest.mark.parametrize("seed", range(0, 400, 7))
def test_launch_order_keeps_every_producer_before_its_consumers(seed):
    """The launch scheduler may move a launch that writes a program output
    ahead of others; on random graphs every launch still comes after the
    launch that writes each node it reads."""
    rnd = random.Random(seed)
    g, _, _ = random_graph(rnd, seed)
    info = B.lower_info(g)
    order = [ln.split()[1] for ln in info["plan"].splitlines() if ln.startswith("launch")]
    io = _kernel_io(info["source"])
    writer = {}
    for k, fn in enumerate(order):
        for t in io.get(fn, (set(), set()))[1]:
            writer.setdefault(t, k)
    for k, fn in enumerate(order):
        for t in io.get(fn, (set(), set()))[0]:
            if t in writer:
                assert writer[t] < k, (fn, t, order)
