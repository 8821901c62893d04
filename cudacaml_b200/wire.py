"""The graph wire format: how a ``Graph`` crosses the C-ABI.

The reference hands its graph to OCaml code in the same process. This backend
lowers graphs natively inside ``libccb.so``, so the graph travels as a small,
line-oriented text that any host language can print (the OCaml printer a
maintainer would add is ocaml/wire.ml). Expression DAGs keep their sharing:
every expression node is written once, before its users, under its own id.

    ccbgraph 1
    name <graph name>
    opt matmul <f32|tf32>                optional; F32 product precision (default f32)
    opt shard <rank> <world>             optional; rank's slice of a sharded Monte-Carlo program
    e <eid> <dtype> const <value>        f32/f64 value = IEEE-754 double bits (hex)
    e <eid> <dtype> arg <i>
    e <eid> i32 index
    e <eid> <dtype> binop <op> <a> <b>
    e <eid> <dtype> unop <op> <a>
    e <eid> bool cmp <op> <a> <b>
    e <eid> bool logic <op> <a> <b>
    e <eid> bool not <a>
    e <eid> <dtype> select <c> <a> <b>
    e <eid> <dtype> cast <a>
    t <tid> <dtype> <rank> <d0> .. <dk-1> <kind> <operands>
        param <name> | iota | map <src> <arg> <body> | map2 <a> <b> <arga> <argb> <body>
        reduce <src> <arga> <argb> <body> <init> | scan <src> <arga> <argb> <body> <init>
        gather <idx> <src> | scatter_add <idx> <src> | matmul <a> <b>
        reshape <src> | broadcast <src>
    o <output name> <tid>
    end

Tensor lines are in the graph's topological order. Names (graph, params,
outputs) are one token each: '%', whitespace and control characters are
escaped as %XX per UTF-8 byte, and the empty name is the lone token %, so
any name crosses unchanged.
"""
from __future__ import annotations

from .ir import Expr, Graph, f64_bits


def _const_text(e: Expr) -> str:
    if e.dtype.is_float:
        return "%016x" % f64_bits(e.value)
    if e.dtype.value == "bool":
        return "1" if e.value else "0"
    return str(int(e.value))


MATMUL_PRECISIONS = ("f32", "tf32")


def to_wire(g: Graph, matmul: str = "f32", shard=None) -> str:
    """``matmul`` selects how F32 products are computed: "f32" keeps F32
    arithmetic (the reference's), "tf32" runs them on the tensor cores with
    TF32 operands and F32 accumulation (error bound in ccb_skel.cuh).
    ``shard=(rank, world)`` lowers the graph as rank ``rank`` of a sharded
    Monte-Carlo program (include/ccb.h, sharded programs)."""
    if matmul not in MATMUL_PRECISIONS:
        raise ValueError(f"matmul precision must be one of {MATMUL_PRECISIONS}, got {matmul!r}")
    lines = ["ccbgraph 1", f"name {_check_name(g.name)}"]
    if matmul != "f32":
        lines.append(f"opt matmul {matmul}")
    if shard is not None:
        rank, world = (int(x) for x in shard)
        if not (1 <= world <= 32 and 0 <= rank < world):
            raise ValueError(f"shard must be (rank, world) with 0 <= rank < world <= 32, got {shard!r}")
        if world > 1:
            lines.append(f"opt shard {rank} {world}")
    written = set()

    def emit_expr(root: Expr):
        # Iterative post-order so deep Philox trees cannot hit the recursion
        # limit; sharing is preserved by the uid set.
        stack = [(root, False)]
        while stack:
            e, expanded = stack.pop()
            if e.uid in written:
                continue
            if not expanded:
                stack.append((e, True))
                for a in reversed(e.args):
                    if a.uid not in written:
                        stack.append((a, False))
                continue
            written.add(e.uid)
            dt = e.dtype.value
            k = e.kind
            if k == "const":
                lines.append(f"e {e.uid} {dt} const {_const_text(e)}")
            elif k == "arg":
                lines.append(f"e {e.uid} {dt} arg {e.value}")
            elif k == "index":
                lines.append(f"e {e.uid} {dt} index")
            elif k in ("binop", "cmp", "logic"):
                lines.append(f"e {e.uid} {dt} {k} {e.op} {e.args[0].uid} {e.args[1].uid}")
            elif k == "unop":
                lines.append(f"e {e.uid} {dt} unop {e.op} {e.args[0].uid}")
            elif k in ("not", "cast"):
                lines.append(f"e {e.uid} {dt} {k} {e.args[0].uid}")
            elif k == "select":
                c, a, b = e.args
                lines.append(f"e {e.uid} {dt} select {c.uid} {a.uid} {b.uid}")
            else:
                raise AssertionError(k)

    for t in g.order:
        k = t.kind
        head = f"t {t.uid} {t.dtype.value} {len(t.shape)}" + "".join(f" {d}" for d in t.shape)
        if k == "param":
            lines.append(f"{head} param {_check_name(t.name)}")
        elif k == "iota":
            lines.append(f"{head} iota")
        elif k == "map":
            emit_expr(t.fn.arg1)
            emit_expr(t.fn.body1)
            lines.append(f"{head} map {t.deps[0].uid} {t.fn.arg1.uid} {t.fn.body1.uid}")
        elif k == "map2":
            for e in (t.fn.arg_a, t.fn.arg_b, t.fn.body2):
                emit_expr(e)
            lines.append(f"{head} map2 {t.deps[0].uid} {t.deps[1].uid} {t.fn.arg_a.uid} {t.fn.arg_b.uid} {t.fn.body2.uid}")
        elif k in ("reduce", "scan"):
            for e in (t.fn.arg_a, t.fn.arg_b, t.fn.body2, t.init):
                emit_expr(e)
            lines.append(f"{head} {k} {t.deps[0].uid} {t.fn.arg_a.uid} {t.fn.arg_b.uid} {t.fn.body2.uid} {t.init.uid}")
        elif k in ("gather", "scatter_add", "matmul"):
            lines.append(f"{head} {k} {t.deps[0].uid} {t.deps[1].uid}")
        elif k in ("reshape", "broadcast"):
            lines.append(f"{head} {k} {t.deps[0].uid}")
        else:
            raise AssertionError(k)
    for n, t in g.outputs:
        lines.append(f"o {_check_name(n)} {t.uid}")
    lines.append("end")
    return "\n".join(lines) + "\n"


def _check_name(n: str) -> str:
    """A name as one whitespace-free token: '%', whitespace and control
    characters are written as %XX (each UTF-8 byte), every other character
    as itself, so ordinary names read the same in the text. The empty name
    is the lone token '%' (a literal '%' is always '%25')."""
    if not n:
        return "%"
    out = []
    for c in n:
        if c == "%" or c.isspace() or ord(c) < 0x20 or ord(c) == 0x7F:
            out.extend("%%%02X" % b for b in c.encode("utf-8"))
        else:
            out.append(c)
    return "".join(out)
