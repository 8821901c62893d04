"""The types that cross the boundary, on the host: Graph construction and
validation, Value storage, and Broadcast / full / scalar (the reference's
test/unit/test_graph.ml, test_value.ml and test_broadcast.ml cases; the
structural ones asked of this backend's lowering). CPU only.
"""
import numpy as np
import pytest

from cudacaml_b200 import backend_cuda as B
from cudacaml_b200 import dsl as D
from cudacaml_b200.ir import BOOL, F32, F64, I32, I64, Graph, Value
from oracle import interp as I

SHAPE = (8,)


def run(g, inputs):
    return dict(I.run(I.compile(g), inputs))


def uids(g):
    return [t.uid for t in g.topological_order()]


# ---------------------------------------------------------------------------
# Graph
# ---------------------------------------------------------------------------
def test_params_in_first_use_order_deduped():
    x, y = D.param("x", F32, SHAPE), D.param("y", F32, SHAPE)
    r = D.map2(D.add, D.map(lambda e: D.mul(e, e), x), y)
    assert [n for n, _ in Graph("g", [("r", r)]).params] == ["x", "y"]


def test_topological_order_deps_first_no_duplicates():
    x = D.param("x", F32, SHAPE)
    a = D.map(D.neg, x)
    b = D.map(D.neg, a)
    o = uids(Graph("g", [("b", b)]))
    assert len(o) == 3
    assert o.index(x.uid) < o.index(a.uid) < o.index(b.uid)


def test_shared_node_once_and_fan_out():
    x = D.param("x", F32, SHAPE)
    s = D.map(lambda e: D.mul(e, e), x)
    a, b = D.map(D.neg, s), D.map(D.sqrt, s)
    g = Graph("g", [("a", a), ("b", b)])
    assert len(uids(g)) == 4
    assert (g.fan_out(s), g.fan_out(x), g.fan_out(a)) == (2, 1, 0)
    r = D.map2(D.add, s, s)
    assert Graph("h", [("r", r)]).fan_out(s) == 2  # one consumer, used twice


def test_outputs_in_order_and_name():
    x = D.param("x", F32, SHAPE)
    g = Graph("g", [("b", D.map(D.neg, x)), ("a", x)])
    assert [n for n, _ in g.outputs] == ["b", "a"]
    assert g.name == "g"


def test_construction_errors():
    x1, x2 = D.param("x", F32, SHAPE), D.param("x", F32, SHAPE)
    with pytest.raises(ValueError):
        Graph("g", [("r", D.map2(D.add, x1, x2))])  # two Params named x
    with pytest.raises(ValueError):
        Graph("g", [("r", x1), ("r", x1)])
    with pytest.raises(ValueError):
        Graph("g", [])
    with pytest.raises(ValueError):
        D.map2(D.add, x1, D.param("y", F32, (9,)))
    with pytest.raises(ValueError):
        D.reshape((3, 3), x1)
    assert D.reshape((2, 4), x1).shape == (2, 4)


def test_gather_and_reduce_shapes():
    x = D.param("x", F32, SHAPE)
    assert D.gather(D.iota((3,)), x).shape == (3,)
    assert D.reduce(D.add, D.const(F32, 0.0), x).shape == ()


def test_to_dot_names_the_graph_and_every_node():
    x = D.param("x", F32, SHAPE)
    r = D.map(D.neg, x)
    dot = Graph("mygraph", [("r", r)]).to_dot()
    for sub in ("digraph", "mygraph", f"n{x.uid}", f"n{r.uid}", "->", "Param x", "Map [8] f32"):
        assert sub in dot, sub
    assert '\\"' in Graph('a"b', [("r", r)]).to_dot()  # names are escaped


# ---------------------------------------------------------------------------
# Value
# ---------------------------------------------------------------------------
def test_value_create_zero_fills_and_sizes():
    v = Value.create(F32, (4,))
    assert (v.numel, v.byte_size, v.to_list()) == (4, 16, [0.0] * 4)
    s = Value.create(F32, ())
    assert (s.numel, s.byte_size) == (1, 4)
    assert Value.create(F64, (3,)).byte_size == 24
    assert Value.create(I64, (3,)).byte_size == 24


def test_value_get_set_roundtrip_and_bounds():
    v = Value.of_list(I32, (3,), [1, 2, 3])
    assert v.get(2) == 3
    v.set(0, 9)
    assert v.to_list() == [9, 2, 3]
    with pytest.raises(ValueError):
        Value.of_list(F32, (2,), [1.0])
    w = Value.create(F64, (2,))
    with pytest.raises(IndexError):
        w.get(2)
    with pytest.raises(IndexError):
        w.get(-1)
    with pytest.raises(IndexError):
        w.set(-1, 1.0)
    with pytest.raises(ValueError):
        Value.create(BOOL, ())


def test_value_storage_is_shared_row_major_and_f32_rounds():
    v = Value.of_list(I64, (2, 3), [1, 2, 3, 4, 5, 6])
    a = v.array()
    assert a.shape == (2, 3) and a[1, 2] == 6
    a[0, 0] = 42  # the array view shares the value's storage
    assert v.get(0) == 42
    m = Value.of_list(I32, (2, 2), [1, 2, 3, 4])
    assert m.get(2) == 3 and m.shape == (2, 2)
    f = Value.of_list(F32, (1,), [0.1])
    assert f.get(0) != 0.1
    assert abs(f.get(0) - 0.100000001490116) <= 1e-9


# ---------------------------------------------------------------------------
# Broadcast, full, scalar
# ---------------------------------------------------------------------------
def test_broadcast_a_scalar_param():
    s = D.scalar("s", F32)
    r = run(Graph("b", [("r", D.broadcast((4,), s))]), [("s", Value.of_list(F32, (), [2.5]))])["r"]
    assert r.to_list() == [2.5] * 4


def test_x_times_broadcast_sum_x():
    x = D.param("x", F32, (3,))
    total = D.reduce(D.add, D.const(F32, 0.0), x)
    g = Graph("b", [("r", D.map2(D.mul, x, D.broadcast(x.shape, total)))])
    assert run(g, [("x", Value.of_list(F32, (3,), [1.0, 2.0, 3.0]))])["r"].to_list() == [6.0, 12.0, 18.0]
    # the reduce, then one pass that reads its result: two kernels
    assert B.lower_info(g)["kernels"] == 2


def test_broadcast_rejects_a_source_with_more_than_one_element():
    with pytest.raises(ValueError):
        D.broadcast((6,), D.param("x", F32, (3,)))


def test_full_has_no_params_and_uploads_nothing():
    g = Graph("f", [("r", D.full(F32, (3,), 7.0))])
    assert g.params == []
    assert run(g, [])["r"].to_list() == [7.0, 7.0, 7.0]
    assert not any(line.startswith("upload") for line in B.lower_info(g)["plan"].splitlines())


def test_scalar_is_a_scalar_param():
    s = D.scalar("s", F64)
    assert s.shape == () and s.kind == "param"


def test_broadcast_with_fan_out_one_is_inlined():
    x, s = D.param("x", F32, (8,)), D.scalar("s", F32)
    b = D.broadcast((8,), s)
    g = Graph("b", [("r", D.map2(D.mul, x, b))])
    assert B.lower_info(g)["kernels"] == 1


def test_broadcast_deps_and_dot_name():
    s = D.scalar("s", F32)
    b = D.broadcast((4,), s)
    assert len(b.deps) == 1 and b.deps[0].uid == s.uid
    assert "Broadcast" in Graph("b", [("r", b)]).to_dot()


# ---------------------------------------------------------------------------
# Names cross the wire unchanged
# ---------------------------------------------------------------------------
ODD_NAMES = ["spot price", "a%b", "tab\there", "two\nlines", "prix €", "dloss/dW1", "%", ""]


def test_wire_escapes_only_what_must_be_escaped():
    from cudacaml_b200.wire import to_wire
    x = D.param("spot price", F32, (2,))
    text = to_wire(Graph("my graph", [("dloss/dW1", D.map(D.neg, x)), ("50%", x)]))
    assert "name my%20graph" in text.splitlines()
    assert any(line.endswith("param spot%20price") for line in text.splitlines())
    assert any(line.startswith("o dloss/dW1 ") for line in text.splitlines())
    assert any(line.startswith("o 50%25 ") for line in text.splitlines())
    assert any(line.startswith("o % ") for line in to_wire(Graph("g", [("", x)])).splitlines())


@pytest.mark.parametrize("name", ODD_NAMES)
def test_any_name_round_trips_through_the_oracle_and_lowering(name):
    x = D.param(name, F32, (3,))
    g = Graph(name, [("out " + name, D.map(D.neg, x)), (name + " sum", D.reduce(D.add, D.const(F32, 0.0), x))])
    o = I.run(I.compile(g), [(name, Value.of_list(F32, (3,), [1.0, 2.0, 3.0]))])
    assert [n for n, _ in o] == ["out " + name, name + " sum"]
    assert dict(o)["out " + name].to_list() == [-1.0, -2.0, -3.0]
    info = B.lower_info(g)
    assert info["kernels"] == 1
    assert f"upload {name} ->" in info["plan"]


def test_malformed_escapes_are_rejected():
    import ctypes
    from cudacaml_b200 import runtime as R
    for bad in (b"x%G1", b"x%4", b"x%", b"%%"):
        text = b"ccbgraph 1\nname g\nt 1 f32 1 4 param " + bad + b"\no r 1\nend\n"
        h = ctypes.c_void_p()
        assert R.lib().ccb_program_lower(text, ctypes.byref(h)) != 0
        assert "escape" in R.lib().ccb_last_error().decode()
        err = ctypes.create_string_buffer(1024)
        assert not I.lib().ccbo_load(text, err, 1024)
        assert "escape" in err.value.decode()
