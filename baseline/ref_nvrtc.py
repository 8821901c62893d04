"""A labelled RESTATEMENT of the reference's NVRTC backend, used only as a
timed baseline beside this backend.

The reference compiles a graph in three steps, all OCaml: Fusion.plan picks
the nodes that own a global buffer (params, barriers, outputs, fan-out >= 2;
lib/lower/fusion.ml:41-73), Lower.program turns every other node into an
inlined element expression and every buffer-owning node into one to three
kernels from a fixed set of templates with fixed geometry
(lib/lower/lower.ml:232-1012, lib/lower/schedule.ml:8-84), and Emit prints
them as CUDA C (lib/backend_cuda/emit.ml:58-367). Jit compiles that text with
NVRTC and no options at all -- no -arch, so PTX for NVRTC's default virtual
architecture, JIT-compiled by the driver at load (lib/runtime/jit.ml:11-25).

OCaml is not installed here, so the reference cannot run. This module
produces the same kernels from this repository's restatement of the
reference IR (cudacaml_b200.ir): the same buffer plan, the same templates
(K1 grid-stride element-wise, K2/K3 shared-memory tree reduce with an extra
partials pass for long rows, K4/K5 Hillis-Steele chunk scan with a serial
pass over chunk totals, K6 zero-fill + atomicAdd scatter, K8 16x16 shared
tiled product), the same launch geometry, the same C spellings (integers
wrapped through unsigned, masked shifts, float math names), compiled the same
way (NVRTC, no options, PTX loaded by cuModuleLoadData). It runs the plan
device-resident: every buffer (scratch included) is allocated once, as the
reference's Executor does at create, and a run is the launch sequence.

It is a baseline, not part of the backend: nothing under cudacaml_b200/
imports it, and the NVRTC and driver calls go through cuda-python, not
through libccb.so.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np

from cudacaml_b200.ir import F32, F64, I32, I64, BOOL, numel, row_length

BLOCK = 256  # Schedule.block_size
REDUCE_THRESHOLD = 4096  # Schedule.reduce_threshold
SCAN_CHUNK = 256  # Schedule.scan_chunk
TILE = 16  # Schedule.tile


# ---------------------------------------------------------------- geometry (lib/lower/schedule.ml)
def grid_stride(n):
    return (max(1, min(1024, (n + 255) // 256)), 1, BLOCK, 1)


def rows_block(rows):
    return (max(1, rows), 1, BLOCK, 1)


def rows_thread(rows):
    return (max(1, rows), 1, 1, 1)


def reduce_blocks(row_len):
    if row_len <= REDUCE_THRESHOLD:
        return 1
    per = BLOCK * 8
    return min(128, (row_len + per - 1) // per)


# ---------------------------------------------------------------- C spellings (lib/backend_cuda/emit.ml)
CTYPE = {F32: "float", F64: "double", I32: "int", I64: "long long", BOOL: "bool"}


def float_lit(dt, v):
    sfx = "" if dt is F64 else "f"
    if math.isnan(v):
        return f"(0.0{sfx}/0.0{sfx})"
    if v == math.inf:
        return f"(1.0{sfx}/0.0{sfx})"
    if v == -math.inf:
        return f"(-1.0{sfx}/0.0{sfx})"
    s = "%.9g" % v
    if not any(c in s for c in ".en"):
        s += ".0"
    return s + sfx


def lit(dt, v):
    if dt is BOOL:
        return "true" if v else "false"
    if dt.is_float:
        return float_lit(dt, float(v))
    return f"{int(v)}LL" if dt is I64 else f"{int(v)}"


def ilit(n):
    return str(int(n))


def wrap(dt, sym, a, b):
    if dt is I32:
        return f"((int)((unsigned int)({a}) {sym} (unsigned int)({b})))"
    if dt is I64:
        return f"((long long)((unsigned long long)({a}) {sym} (unsigned long long)({b})))"
    return f"({a} {sym} {b})"


def iadd(a, b):
    return wrap(I32, "+", a, b)


def isub(a, b):
    return wrap(I32, "-", a, b)


def imul(a, b):
    return wrap(I32, "*", a, b)


def idiv(a, b):
    return f"({a} / {b})"


def binop(dt, op, a, b):
    if op == "add":
        return wrap(dt, "+", a, b)
    if op == "sub":
        return wrap(dt, "-", a, b)
    if op == "mul":
        return wrap(dt, "*", a, b)
    if op == "div":
        return f"({a} / {b})"
    if op in ("min", "max"):
        if dt is F32:
            return f"f{op}f({a}, {b})"
        if dt is F64:
            return f"f{op}({a}, {b})"
        c = "<" if op == "min" else ">"
        return f"(({a} {c} {b}) ? {a} : {b})"
    if op in ("bit_and", "bit_or", "bit_xor"):
        return f"({a} {dict(bit_and='&', bit_or='|', bit_xor='^')[op]} {b})"
    if op in ("shl", "shr"):
        sym = "<<" if op == "shl" else ">>"
        if dt is I32:
            return f"((int)((unsigned int)({a}) {sym} (({b}) & 31)))"
        return f"((long long)((unsigned long long)({a}) {sym} (({b}) & 63)))"
    raise ValueError(op)


def neg(dt, a):
    if dt is I32:
        return f"((int)(0u - (unsigned int)({a})))"
    if dt is I64:
        return f"((long long)(0ull - (unsigned long long)({a})))"
    return f"(- {a})" if a[:1] in "-+" else f"(-{a})"


MATH = {"sqrt": ("sqrtf", "sqrt"), "exp": ("expf", "exp"), "log": ("logf", "log"), "sin": ("sinf", "sin"),
        "cos": ("cosf", "cos"), "erf": ("erff", "erf"), "erfinv": ("erfinvf", "erfinv")}
CMP = {"eq": "==", "ne": "!=", "lt": "<", "le": "<=", "gt": ">", "ge": ">="}


def unop(dt, op, a):
    if op == "neg":
        return neg(dt, a)
    if op == "abs":
        if dt is F32:
            return f"fabsf({a})"
        if dt is F64:
            return f"fabs({a})"
        return f"(({a} < 0) ? {neg(dt, a)} : {a})"
    f32, f64 = MATH[op]
    return f"{f32 if dt is F32 else f64}({a})"


def expr_text(e, env, index):
    """Lower.expr_of + Emit.expr: an element function's body as C text with
    [Arg i] bound to env[i] and [Index] to `index`. Shared expression nodes
    are printed once per use, as the reference's tree printer does; the memo
    only saves Python the work of printing them again."""
    memo = {}

    def go(x):
        s = memo.get(x.uid)
        if s is not None:
            return s
        k = x.kind
        if k == "const":
            s = lit(x.dtype, x.value)
        elif k == "arg":
            s = env[x.value]
        elif k == "index":
            s = index
        elif k == "binop":
            s = binop(x.dtype, x.op, go(x.args[0]), go(x.args[1]))
        elif k == "unop":
            s = unop(x.dtype, x.op, go(x.args[0]))
        elif k == "cmp":
            s = f"({go(x.args[0])} {CMP[x.op]} {go(x.args[1])})"
        elif k == "logic":
            s = f"({go(x.args[0])} {'&&' if x.op == 'and' else '||'} {go(x.args[1])})"
        elif k == "not":
            s = f"(!{go(x.args[0])})"
        elif k == "select":
            s = f"({go(x.args[0])} ? {go(x.args[1])} : {go(x.args[2])})"
        elif k == "cast":
            s = f"(({CTYPE[x.dtype]})({go(x.args[0])}))"
        else:
            raise ValueError(k)
        memo[x.uid] = s
        return s

    return go(e)


# ---------------------------------------------------------------- the buffer plan (Fusion.plan)
BARRIERS = ("reduce", "scan", "scatter_add", "matmul")


class Plan:
    def __init__(self, g):
        self.g = g
        outs = {t.uid for _, t in g.outputs}
        self.mat = {}
        self.roots = []
        for t in g.order:
            if t.kind == "param" or t.kind in BARRIERS or t.uid in outs or g.fan_out(t) >= 2:
                self.mat[t.uid] = (f"p{len(self.mat)}" if t.kind == "param" else f"t{t.uid}")
                if t.kind != "param":
                    self.roots.append(t)

    def elem(self, t, index):
        """Lower.elem: a load of a materialised node, else the node inlined."""
        if t.uid in self.mat:
            return f"{self.mat[t.uid]}[{index}]"
        return self.inline(t, index)

    def inline(self, t, index):
        k = t.kind
        if k == "iota":
            return index
        if k == "map":
            return expr_text(t.fn.body1, [self.elem(t.deps[0], index)], index)
        if k == "map2":
            return expr_text(t.fn.body2, [self.elem(t.deps[0], index), self.elem(t.deps[1], index)], index)
        if k == "gather":
            return self.elem(t.deps[1], self.elem(t.deps[0], index))
        if k == "reshape":
            return self.elem(t.deps[0], index)
        if k == "broadcast":
            return self.elem(t.deps[0], "0")
        raise ValueError(f"{k} must be materialised")

    def inputs_of(self, root):
        seen, acc = set(), []

        def visit(t):
            if t.uid in seen:
                return
            seen.add(t.uid)
            if t.uid in self.mat:
                acc.append(t)
            else:
                for d in t.deps:
                    visit(d)

        for d in root.deps:
            visit(d)
        return acc


class Kernel:
    def __init__(self, name, params, body, launch, shared=()):
        self.name, self.params, self.body, self.launch, self.shared = name, params, body, launch, shared

    def text(self):
        ps = ", ".join(f"{CTYPE[dt]}* {nm}" for nm, dt, _ in self.params)
        sh = "".join(f"  __shared__ {CTYPE[dt]} {nm}[{n}];\n" for nm, dt, n in self.shared)
        return f'extern "C" __global__ void {self.name}({ps}) {{\n{sh}{self.body}}}\n'


def _tree(combine, dt):
    out = []
    for k in range(8):
        s = BLOCK >> (k + 1)
        out.append(f"  if ((threadIdx.x < {s})) {{\n    sdata[threadIdx.x] = "
                   f"{combine('sdata[threadIdx.x]', f'sdata[{iadd('threadIdx.x', ilit(s))}]')};\n  }}\n"
                   f"  __syncthreads();\n")
    return "".join(out)


def _reduction(prelude, lo, hi, step, load, dst, dst_index, combine, identity, dt):
    return (prelude + f"  {CTYPE[dt]} acc = {identity};\n"
            f"  for (int i = {lo}; i < {hi}; i += {step}) {{\n    acc = {combine('acc', load('i'))};\n  }}\n"
            f"  sdata[threadIdx.x] = acc;\n  __syncthreads();\n" + _tree(combine, dt)
            + f"  if ((threadIdx.x == 0)) {{\n    {dst}[{dst_index}] = sdata[0];\n  }}\n")


def kernels_of(plan, root):
    """Lower.kernels_of: the kernels of one buffer-owning node, plus its
    scratch buffers (name, dtype, numel)."""
    out = plan.mat[root.uid]
    dt = root.dtype
    ins = [(plan.mat[t.uid], t.dtype, t.numel) for t in plan.inputs_of(root)]
    outp = (out, dt, root.numel)
    params = ins + [outp]
    name = f"k_{root.uid}"
    k = root.kind
    if k in ("map", "map2", "iota", "gather", "reshape", "broadcast"):
        n = root.numel
        body = (f"  for (int i = (blockIdx.x * blockDim.x + threadIdx.x); i < {ilit(n)}; i += (gridDim.x * blockDim.x)) {{\n"
                f"    {out}[i] = {plan.inline(root, 'i')};\n  }}\n")
        return [Kernel(name, params, body, grid_stride(n))], []
    if k == "reduce":
        src = root.deps[0]
        n = row_length(src.shape)
        rows = root.numel
        g = reduce_blocks(n)

        def combine(a, b):
            return expr_text(root.fn.body2, [a, b], "0")

        ident = expr_text(root.init, [], "0")
        sdata = [("sdata", dt, BLOCK)]

        def load(i):
            return plan.elem(src, i)

        if g == 1:
            rb = imul("blockIdx.x", ilit(n))
            body = _reduction("", iadd(rb, "threadIdx.x"), iadd(rb, ilit(n)), "blockDim.x", load, out, "blockIdx.x",
                              combine, ident, dt)
            return [Kernel(name, params, body, rows_block(rows), sdata)], []
        part = (f"t{root.uid}_partials", dt, rows * g)
        pre = (f"  int row = {idiv('blockIdx.x', ilit(g))};\n"
               f"  int blk = {isub('blockIdx.x', imul('row', ilit(g)))};\n")
        rb = imul("row", ilit(n))
        body1 = _reduction(pre, iadd(rb, iadd(imul("blk", ilit(BLOCK)), "threadIdx.x")), iadd(rb, ilit(n)),
                           ilit(g * BLOCK), load, part[0], "blockIdx.x", combine, ident, dt)
        pb = imul("blockIdx.x", ilit(g))
        body2 = _reduction("", iadd(pb, "threadIdx.x"), iadd(pb, ilit(g)), "blockDim.x", lambda i: f"{part[0]}[{i}]",
                           out, "blockIdx.x", combine, ident, dt)
        return [Kernel(name + "_partial", ins + [part], body1, rows_block(rows * g), sdata),
                Kernel(name, [part, outp], body2, rows_block(rows), sdata)], [part]
    if k == "scan":
        src = root.deps[0]
        n = row_length(src.shape)
        rows = 0 if n == 0 else src.numel // n
        c = SCAN_CHUNK
        nb = 1 if n <= 0 else (n + c - 1) // c

        def combine(a, b):
            return expr_text(root.fn.body2, [a, b], "0")

        ident = expr_text(root.init, [], "0")
        T = CTYPE[dt]
        offsets = []
        o = 1
        while o < c:
            offsets.append(o)
            o *= 2
        hs = "".join(f"  __syncthreads();\n  {T} v{o} = ((threadIdx.x >= {o}) ? "
                     f"{combine(f'sdata[{isub('threadIdx.x', ilit(o))}]', 'sdata[threadIdx.x]')} : sdata[threadIdx.x]);\n"
                     f"  __syncthreads();\n  sdata[threadIdx.x] = v{o};\n" for o in offsets) + "  __syncthreads();\n"

        def chunk(base, ln):
            return (f"  sdata[threadIdx.x] = ((threadIdx.x < {ln}) ? {plan.elem(src, iadd(base, 'threadIdx.x'))} : {ident});\n"
                    + hs + f"  if ((threadIdx.x < {ln})) {{\n    {out}[{iadd(base, 'threadIdx.x')}] = sdata[threadIdx.x];\n  }}\n")

        sdata = [("sdata", dt, c)]
        launch = lambda blocks: (max(1, blocks), 1, c, 1)  # noqa: E731
        if nb == 1:
            return [Kernel(name, params, chunk(imul("blockIdx.x", ilit(n)), ilit(n)), launch(rows), sdata)], []
        sums = (f"t{root.uid}_sums", dt, rows * nb)
        rest = isub(ilit(n), imul("blk", ilit(c)))
        body1 = (f"  int row = {idiv('blockIdx.x', ilit(nb))};\n"
                 f"  int blk = {isub('blockIdx.x', imul('row', ilit(nb)))};\n"
                 f"  int base = {iadd(imul('row', ilit(n)), imul('blk', ilit(c)))};\n"
                 f"  int len = (({rest} < {c}) ? {rest} : {c});\n"
                 + chunk("base", "len")
                 + f"  if ((threadIdx.x == 0)) {{\n    {sums[0]}[blockIdx.x] = sdata[{isub('len', '1')}];\n  }}\n")
        sb = imul("blockIdx.x", ilit(nb))
        body2 = (f"  {T} acc = {ident};\n  for (int i = {sb}; i < {iadd(sb, ilit(nb))}; i += 1) {{\n"
                 f"    acc = {combine('acc', f'{sums[0]}[i]')};\n    {sums[0]}[i] = acc;\n  }}\n")
        blk3 = idiv(isub("i", imul("row", ilit(n))), ilit(c))
        body3 = (f"  for (int i = (blockIdx.x * blockDim.x + threadIdx.x); i < {ilit(rows * n)}; i += (gridDim.x * blockDim.x)) {{\n"
                 f"    int row = {idiv('i', ilit(n))};\n    int blk = {blk3};\n"
                 f"    if ((blk > 0)) {{\n      {out}[i] = "
                 f"{combine(f'{sums[0]}[{isub(iadd(imul('row', ilit(nb)), 'blk'), '1')}]', f'{out}[i]')};\n    }}\n  }}\n")
        return [Kernel(name + "_chunks", ins + [sums, outp], body1, launch(rows * nb), sdata),
                Kernel(name + "_sums", [sums], body2, rows_thread(rows)),
                Kernel(name, [sums, outp], body3, grid_stride(rows * n))], [sums]
    if k == "scatter_add":
        m = root.numel
        idx, src = root.deps
        n = src.numel
        zero = lit(dt, 0)
        body0 = (f"  for (int i = (blockIdx.x * blockDim.x + threadIdx.x); i < {ilit(m)}; i += (gridDim.x * blockDim.x)) {{\n"
                 f"    {out}[i] = {zero};\n  }}\n")
        body1 = (f"  for (int i = (blockIdx.x * blockDim.x + threadIdx.x); i < {ilit(n)}; i += (gridDim.x * blockDim.x)) {{\n"
                 f"    atomicAdd(&{out}[{plan.elem(idx, 'i')}], {plan.elem(src, 'i')});\n  }}\n")
        return [Kernel(name + "_zero", [outp], body0, grid_stride(m)), Kernel(name, params, body1, grid_stride(n))], []
    if k == "matmul":
        a, b = root.deps
        m, n = root.shape
        kk = row_length(a.shape)
        nt = (kk + TILE - 1) // TILE
        zero = lit(dt, 0)
        T = CTYPE[dt]
        slot = iadd(imul("threadIdx.y", ilit(TILE)), "threadIdx.x")
        fma = binop(dt, "add", "acc", binop(dt, "mul", f"sa[{iadd(imul('threadIdx.y', ilit(TILE)), 'p')}]",
                                            f"sb[{iadd(imul('p', ilit(TILE)), 'threadIdx.x')}]"))
        body = (f"  int row = {iadd(imul('blockIdx.y', ilit(TILE)), 'threadIdx.y')};\n"
                f"  int col = {iadd(imul('blockIdx.x', ilit(TILE)), 'threadIdx.x')};\n"
                f"  {T} acc = {zero};\n"
                f"  for (int kt = 0; kt < {nt}; kt += 1) {{\n"
                f"    int ka = {iadd(imul('kt', ilit(TILE)), 'threadIdx.x')};\n"
                f"    int kb = {iadd(imul('kt', ilit(TILE)), 'threadIdx.y')};\n"
                f"    sa[{slot}] = (((row < {m}) && (ka < {kk})) ? {plan.elem(a, iadd(imul('row', ilit(kk)), 'ka'))} : {zero});\n"
                f"    sb[{slot}] = (((kb < {kk}) && (col < {n})) ? {plan.elem(b, iadd(imul('kb', ilit(n)), 'col'))} : {zero});\n"
                f"    __syncthreads();\n"
                f"    for (int p = 0; p < {TILE}; p += 1) {{\n"
                f"      acc = {fma};\n"
                f"    }}\n    __syncthreads();\n  }}\n"
                f"  if (((row < {m}) && (col < {n}))) {{\n    {out}[{iadd(imul('row', ilit(n)), 'col')}] = acc;\n  }}\n")
        launch = (max(1, (n + TILE - 1) // TILE), max(1, (m + TILE - 1) // TILE), TILE, TILE)
        return [Kernel(name, params, body, launch, [("sa", dt, TILE * TILE), ("sb", dt, TILE * TILE)])], []
    raise ValueError(k)


class Program:
    """Lower.program + Emit.program: the kernels in launch order, the buffers
    (params, computed nodes, scratch) and the CUDA text."""

    def __init__(self, g):
        self.g = g
        self.plan = Plan(g)
        self.kernels = []
        self.scratch = []
        for r in self.plan.roots:
            ks, sc = kernels_of(self.plan, r)
            self.kernels += ks
            self.scratch += sc
        self.source = f"// generated by cudacaml: {g.name}\n" + "\n".join(k.text() for k in self.kernels)

    def buffers(self):
        """(name, dtype, numel) of every buffer the plan allocates."""
        out = []
        for t in self.g.order:
            if t.uid in self.plan.mat:
                out.append((self.plan.mat[t.uid], t.dtype, t.numel))
        return out + list(self.scratch)


# ---------------------------------------------------------------- NVRTC (no options) + driver JIT, via cuda-python
def _ck(res, what):
    err = res[0]
    if int(err) != 0:
        raise RuntimeError(f"{what}: {err}")
    return res[1:] if len(res) > 2 else (res[1] if len(res) == 2 else None)


class Loaded:
    """The program compiled as the reference's Jit.compile does
    (nvrtcCompileProgram with no options -> PTX -> cuModuleLoadData), its
    buffers allocated once on the current device, launchable as a unit."""

    def __init__(self, prog: Program):
        from cuda.bindings import driver as cu
        from cuda.bindings import nvrtc
        self.cu = cu
        self.prog = prog
        p = _ck(nvrtc.nvrtcCreateProgram(prog.source.encode(), f"{prog.g.name}.cu".encode(), 0, [], []), "nvrtcCreateProgram")
        res = nvrtc.nvrtcCompileProgram(p, 0, [])
        if int(res[0]) != 0:
            size = _ck(nvrtc.nvrtcGetProgramLogSize(p), "log size")
            log = b" " * size
            nvrtc.nvrtcGetProgramLog(p, log)
            raise RuntimeError("nvrtc: " + log.decode(errors="replace")[:4000])
        size = _ck(nvrtc.nvrtcGetPTXSize(p), "ptx size")
        ptx = b" " * size
        _ck(nvrtc.nvrtcGetPTX(p, ptx), "ptx")
        nvrtc.nvrtcDestroyProgram(p)
        self.ptx = ptx
        self.module = _ck(cu.cuModuleLoadData(ptx), "cuModuleLoadData")
        self.fns = [_ck(cu.cuModuleGetFunction(self.module, k.name.encode()), "cuModuleGetFunction") for k in prog.kernels]
        self.bufs = {}
        for name, dt, n in prog.buffers():
            self.bufs[name] = (_ck(cu.cuMemAlloc(max(1, n * dt.size_in_bytes)), "cuMemAlloc"), dt, n)
        self.args = []
        for k in prog.kernels:
            vals = [ctypes.c_void_p(int(self.bufs[nm][0])) for nm, _, _ in k.params]
            arr = (ctypes.c_void_p * len(vals))(*[ctypes.addressof(v) for v in vals])
            self.args.append((vals, arr))

    def param_buffer(self, name):
        for t in self.prog.g.order:
            if t.kind == "param" and t.name == name:
                return int(self.bufs[self.prog.plan.mat[t.uid]][0])
        raise KeyError(name)

    def output_buffer(self, name):
        t = self.prog.g.output(name)
        return int(self.bufs[self.prog.plan.mat[t.uid]][0])

    def upload(self, name, arr):
        a = np.ascontiguousarray(arr)
        _ck(self.cu.cuMemcpyHtoD(self.param_buffer(name), a.ctypes.data, a.nbytes), "cuMemcpyHtoD")

    def download(self, name, dtype, count):
        out = np.empty(count, dtype)
        _ck(self.cu.cuMemcpyDtoH(out.ctypes.data, self.output_buffer(name), out.nbytes), "cuMemcpyDtoH")
        return out

    def launch(self, stream):
        """One run: every kernel of the plan, in order, on `stream`."""
        for k, f, (_, arr) in zip(self.prog.kernels, self.fns, self.args):
            gx, gy, bx, by = k.launch
            _ck(self.cu.cuLaunchKernel(f, gx, gy, 1, bx, by, 1, 0, stream, ctypes.addressof(arr), 0), "cuLaunchKernel")

    def release(self):
        for p, _, _ in self.bufs.values():
            self.cu.cuMemFree(p)
        self.bufs = {}
        self.cu.cuModuleUnload(self.module)
