"""The OCaml binding sources under ocaml/ (not compiled here: the image has
no OCaml toolchain) against what they must cover: one ctypes binding per
entry point declared in include/ccb.h, and a wire printer that writes every
expression and tensor node kind the C parser reads. CPU only."""
import os
import re

from cudacaml_b200 import ir

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _read(*p):
    with open(os.path.join(ROOT, *p)) as f:
        return f.read()


def test_every_header_entry_point_has_an_ocaml_binding():
    declared = set(re.findall(r"\b(ccb_[a-z0-9_]+)\s*\(", _read("include", "ccb.h")))
    bound = re.findall(r'fn "(ccb_[a-z0-9_]+)"', _read("ocaml", "ccb.ml"))
    assert len(bound) == len(set(bound)), "a symbol is bound twice"
    assert declared == set(bound), (sorted(declared - set(bound)), sorted(set(bound) - declared))


def test_wire_printer_names_every_node_kind():
    src = _read("ocaml", "wire.ml")
    for op in ir.BINOPS + ir.UNOPS + ir.CMPS + ir.LOGICS:
        assert f'"{op}"' in src, op
    for kind in ("const", "arg", "index", "binop", "unop", "cmp", "logic", "not", "select", "cast"):
        assert re.search(rf'"e %d [^"]*{kind}\b', src), kind
    for kind in ("param", "iota", "map", "map2", "reduce", "scan", "gather", "scatter_add", "matmul", "reshape",
                 "broadcast"):
        assert re.search(rf'"%s {kind}\b', src), kind
    for ctor in ("Tensor.Param", "Tensor.Iota", "Tensor.Map ", "Tensor.Map2", "Tensor.Reduce", "Tensor.Scan",
                 "Tensor.Gather", "Tensor.Scatter_add", "Tensor.Matmul", "Tensor.Reshape", "Tensor.Broadcast"):
        assert ctor in src, ctor


def test_sources_say_they_are_not_built_here():
    for name in sorted(os.listdir(os.path.join(ROOT, "ocaml"))):
        assert "NOT BUILT HERE" in _read("ocaml", name), name
