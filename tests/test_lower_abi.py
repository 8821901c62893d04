"""CPU-only checks of the product: libccb.so loads and exports every entry
point include/ccb.h declares; lowering makes the expected kernels (the
reference's structural tests, test/unit/test_lower.ml, test_multikernel.ml);
every generated program compiles under NVRTC for sm_100a; errors surface as
the reference's exception classes."""
import ctypes
import os
import re

import pytest

from cudacaml_b200 import backend_cuda as B
from cudacaml_b200 import dsl as D
from cudacaml_b200 import examples as X
from cudacaml_b200 import runtime as R
from cudacaml_b200.ir import BOOL, F32, F64, I32, Graph

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "ccb.h")).read()
    return sorted(set(re.findall(r"\b(ccb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    L = ctypes.CDLL(R.LIB_PATH)
    missing = [s for s in header_symbols() if not hasattr(L, s)]
    assert not missing, missing
    assert set(header_symbols()) <= set(R.exported_symbols())


def test_library_loads_without_gpu():
    assert R.lib().ccb_version().decode().startswith("ccb")
    # no crash, a clean status, whatever the machine
    assert R.lib().ccb_available() in (0, 1)


def nvrtc_ok(src: str, name: str) -> int:
    sz = ctypes.c_size_t()
    log = ctypes.c_void_p()
    rc = R.lib().ccb_nvrtc_check(src.encode(), name.encode(), ctypes.byref(sz), ctypes.byref(log))
    if log.value:
        R.lib().ccb_free_string(log)
    assert rc == 0, R.lib().ccb_last_error().decode()[:4000]
    return sz.value


@pytest.mark.parametrize("prog", X.PROGRAMS, ids=lambda p: p.name)
def test_examples_compile_for_sm100a(prog):
    info = B.lower_info(prog.graph())
    assert nvrtc_ok(info["source"], prog.name) > 0


def test_config_graphs_compile():
    for g in (X.call_greeks(1 << 20, F32), X.call_greeks(1 << 20, F64), X.reduce_scan_flat(1 << 20, F32),
              X.reduce_scan_flat(1 << 20, I32), X.reduce_scan_flat(1 << 20, F64), X.rows(64, 4096), X.rows(100, 16), X.scatter(1000, 7),
              X.gather(1000, 100), X.saxpy(1000, 2.0, F64)):
        assert nvrtc_ok(B.lower_info(g)["source"], g.name) > 0


def test_structure():
    k = lambda g: B.lower_info(g)["kernels"]  # noqa: E731
    # saxpy: the map, the stored r and the sum share one pass (12 B/elem)
    assert k(X.saxpy(4096, 2.0)) == 1
    # five chained maps: one kernel (S4)
    assert k(X.find("chain").graph()) == 1
    # s = x*x used three times: recomputed, one pass for a, b and c
    assert k(X.find("fanout").graph()) == 1
    # Grad-produced Greeks: forward sum, three adjoint sums, four scalar
    # outputs -- one launch (the reference makes 25)
    assert k(X.call_greeks(1 << 20, F32)) == 1
    assert k(X.call_greeks(4096, F64)) == 1
    # scan_rows then gather-of-last-column into the mean: 2
    assert k(X.call_mc_paths(512, 16, F64)) == 2
    # reduce + scan over one vector: a pass and a look-back scan
    assert k(X.reduce_scan_flat(1 << 20, F32)) == 2
    # a skinny product (LSM normal equations) is a one-pass split-K reduction
    a = D.param("a", F64, (4, 1 << 14))
    b = D.param("b", F64, (1 << 14, 4))
    assert k(Graph("mm", [("c", D.matmul(a, b))])) == 1
    assert "ccb_mapreduce_0_mm" in B.lower_info(Graph("mm", [("c", D.matmul(a, b))]))["source"]


def test_plan_mentions_params_and_outputs():
    plan = B.lower_info(X.saxpy(8, 2.0))["plan"]
    assert "upload x" in plan and "upload y" in plan
    assert "-> r" in plan and "-> s" in plan


def test_uniform_graph_has_one_param():
    from cudacaml_b200 import rng as Rng
    g = Graph("u", [("r", Rng.uniform(F32, D.scalar("seed", I32), (16,)))])
    assert [n for n, _ in g.params] == ["seed"]
    assert B.lower_info(g)["plan"].count("upload") == 1


def test_bool_output_rejected():
    x = D.param("x", F32, (4,))
    g = Graph("b", [("r", D.map(lambda e: D.lt(e, D.const(F32, 0.0)), x))])
    with pytest.raises(ValueError):
        B.lower_info(g)


def test_malformed_wire_rejected():
    h = ctypes.c_void_p()
    rc = R.lib().ccb_program_lower(b"ccbgraph 1\nname x\nt 1 f32 1 4 frobnicate\nend\n", ctypes.byref(h))
    assert rc == 1
    assert "unknown tensor kind" in R.lib().ccb_last_error().decode()


def test_no_device_is_reported_not_crashed():
    if R.available():
        pytest.skip("a device is present")
    with pytest.raises(R.CcbError):
        B.compile(X.saxpy(8, 2.0))


# ---------------------------------------------------------------- tensor-core products
def _tc_lines(info):
    return [ln for ln in info["source"].splitlines() if ln.startswith("// matmul") and "tensor cores" in ln]


def test_matmul_precision_option_and_default():
    g = X.mlp_step(512, 256, 512, 128)
    assert "matmultc" not in B.lower_info(g)["plan"]  # F32 arithmetic unless asked
    info = B.lower_info(g, matmul="tf32")
    assert len(re.findall(r"launch ccb_matmultc2?_", info["plan"])) == 5
    # 5 products + the dY(+loss) and dZ1 passes; A1 = tanh_like(Z1) runs in
    # the epilogue of the Z1 product (K = 256 here is below the fusion bound)
    assert info["launches"] == 8
    assert B.lower_info(X.mlp_step(512, 2048, 512, 128), matmul="tf32")["launches"] == 7
    with pytest.raises(ValueError):
        B.lower_info(g, matmul="bf16")
    assert nvrtc_ok(info["source"], "mlp_tf32") > 0


def test_tensor_core_operand_views():
    a = D.param("a", F32, (256, 512))   # used transposed: A^T is [512 x 256], stored [K][M]
    b = D.param("b", F32, (256, 384))   # B [K][N] row-major
    w = D.param("w", F32, (256, 384))   # used transposed as B: stored [N][K]
    g = Graph("v", [("c", D.matmul(D.transpose(a), b)), ("d", D.matmul(b, D.transpose(w)))])
    lines = _tc_lines(B.lower_info(g, matmul="tf32"))
    assert len(lines) == 2
    assert f"A MN-major from n{a.uid}" in lines[0] and f"B MN-major from n{b.uid}" in lines[0]
    assert f"A K-major from n{b.uid}" in lines[1] and f"B K-major from n{w.uid}" in lines[1]


def test_tensor_core_operand_expression_is_materialised():
    a = D.param("a", F32, (256, 256))
    b = D.param("b", F32, (256, 256))
    e = D.map(lambda v: D.exp(v), a)
    g = Graph("m", [("c", D.matmul(D.transpose(e), b))])
    info = B.lower_info(g, matmul="tf32")
    # exp(a) is written once by an element pass, then read transposed by TMA
    assert info["plan"].count("launch ccb_mapreduce_") == 1
    assert len(_tc_lines(info)) == 1 and "A MN-major" in _tc_lines(info)[0]


def test_tensor_core_eligibility():
    def mm(dt, m, k, n):
        return Graph("e", [("c", D.matmul(D.param("a", dt, (m, k)), D.param("b", dt, (k, n))))])
    assert _tc_lines(B.lower_info(mm(F32, 256, 256, 256), matmul="tf32"))
    assert not _tc_lines(B.lower_info(mm(F64, 256, 256, 256), matmul="tf32"))   # no f64 kind
    assert not _tc_lines(B.lower_info(mm(F32, 16, 16, 16), matmul="tf32"))      # tiny: exact kernel
    assert not _tc_lines(B.lower_info(mm(F32, 256, 255, 256), matmul="tf32"))   # 1020-byte rows: no TMA
    assert not _tc_lines(B.lower_info(mm(F32, 4, 4096, 4), matmul="tf32"))      # split-K reduction


def test_tensor_core_epilogue_fusion():
    a = D.param("a", F32, (256, 2048))
    b = D.param("b", F32, (2048, 512))
    z = D.matmul(a, b)
    t = D.map(lambda v: D.exp(v), z)
    # the product read by nothing else: the pass runs in the epilogue, the
    # product is not stored
    info = B.lower_info(Graph("f", [("t", t)]), matmul="tf32")
    assert "launch ccb_mapreduce_" not in info["plan"] and info["launches"] == 1
    assert "pass 1 in the epilogue, product not stored" in _tc_lines(info)[0]
    assert info["plan"].count("alloc t") == 1
    # the product is also an output: stored beside the pass's result
    info = B.lower_info(Graph("f", [("t", t), ("z", z)]), matmul="tf32")
    assert info["launches"] == 1 and _tc_lines(info)[0].endswith("pass 1 in the epilogue")
    assert nvrtc_ok(info["source"], "fused") > 0
    # passes that stay apart: a reduction, a second input, a neighbour of
    # element i, a short inner dimension
    s = D.reduce(D.add, D.const(F32, 0.0), D.reshape((256 * 512,), t))
    assert B.lower_info(Graph("f", [("s", s)]), matmul="tf32")["launches"] == 2
    w = D.param("w", F32, (256, 512))
    two = D.map2(lambda u, v: D.mul(u, v), z, w)
    assert B.lower_info(Graph("f", [("s", two)]), matmul="tf32")["launches"] == 2
    sq = D.matmul(a, D.param("c", F32, (2048, 256)))
    sym = D.map2(lambda u, v: D.add(u, v), sq, D.transpose(sq))
    assert B.lower_info(Graph("f", [("s", sym)]), matmul="tf32")["launches"] == 2
    short = D.map(lambda v: D.exp(v), D.matmul(D.param("d", F32, (256, 1024)), D.param("e", F32, (1024, 512))))
    assert B.lower_info(Graph("f", [("s", short)]), matmul="tf32")["launches"] == 2


def test_scan_store_fusion():
    from cudacaml_b200 import lsm as L
    # LSM's S = S0 exp(cumsum): one row-scan launch, the cumulative sums never stored
    info = B.lower_info(L.paths_graph(1 << 12, 64, L.BASELINE_MARKET))
    assert info["launches"] == 1 and "pass 1 in the store, scan not stored" in info["source"]
    x = D.param("x", F64, (1 << 20,))
    c = D.scan(D.add, D.const(F64, 0.0), x)
    y = D.map(lambda v: D.exp(v), c)
    # flat 8-byte scan: fused; the scan kept when it is an output too
    assert B.lower_info(Graph("f", [("y", y)]))["launches"] == 1
    info = B.lower_info(Graph("f", [("y", y), ("c", c)]))
    assert info["launches"] == 1 and "pass 1 in the store\n" in info["source"]
    # the staged 4-byte flat scan writes its destination directly: apart
    x32 = D.param("x", F32, (1 << 20,))
    y32 = D.map(lambda v: D.exp(v), D.scan(D.add, D.const(F32, 0.0), x32))
    assert B.lower_info(Graph("f", [("y", y32)]))["launches"] == 2
    assert nvrtc_ok(info["source"], "scanfused") > 0


def test_row_scan_writes_its_transpose():
    from cudacaml_b200 import lsm as L
    # LSM's date-major S: one row-scan launch writes the transposed tiles
    info = B.lower_info(L.paths_dates_graph(1 << 12, 64, L.BASELINE_MARKET))
    assert info["launches"] == 1 and "scan_rows_warp_t" in info["source"]
    assert info["plan"].count("alloc t") == 1  # only the [64; 4096] result
    x = D.param("x", F32, (1000, 40))
    c = D.scan_rows(D.add, D.const(F32, 0.0), x)
    # a materialised transpose (an output) and a transpose used by the map
    # over it both fuse; a map that uses the element index does not
    t = D.transpose(c)
    assert B.lower_info(Graph("t", [("t", t)]))["launches"] == 1
    assert B.lower_info(Graph("t", [("y", D.map(lambda v: D.exp(v), t))]))["launches"] == 1
    idx_map = D.map(lambda v: D.add(v, D.cast(F32, D.index())), t)
    assert B.lower_info(Graph("t", [("y", idx_map)]))["launches"] == 2
    # the scan itself also an output: stored, then transposed apart
    assert B.lower_info(Graph("t", [("t", t), ("c", c)]))["launches"] == 2
    assert nvrtc_ok(B.lower_info(L.paths_dates_graph(1 << 12, 64, L.BASELINE_MARKET))["source"], "pt") > 0


def test_cuda_core_product_kernels():
    # 4-byte products of at least 128 x 128 take the register-blocked kernel,
    # with tiles loaded along each operand's contiguous dimension; smaller
    # ones and F64 keep the 64 x 64 kernel
    def mm(dt, m, k, n, ta=False, tb=False):
        a = D.param("a", dt, (k, m) if ta else (m, k))
        b = D.param("b", dt, (n, k) if tb else (k, n))
        return Graph("m", [("c", D.matmul(D.transpose(a) if ta else a, D.transpose(b) if tb else b))])

    src = B.lower_info(mm(F32, 256, 64, 256))["source"]
    assert "matmul_tiled128" in src and "A_MN = false, B_KM = false" in src
    assert "A_MN = true, B_KM = true" in B.lower_info(mm(F32, 256, 64, 256, True, True))["source"]
    assert "matmul_tiled128" not in B.lower_info(mm(F32, 100, 64, 256))["source"]
    assert "matmul_tiled128" not in B.lower_info(mm(F64, 256, 64, 256))["source"]
    # an operand expression is stored once before the product reads it
    x = D.param("x", F32, (256, 64))
    e = D.map(lambda v: D.exp(v), D.param("w", F32, (64, 256)))
    info = B.lower_info(Graph("m", [("c", D.matmul(x, e))]))
    assert info["launches"] == 2 and "launch ccb_mapreduce_" in info["plan"]
    # the F32-mode MLP step: the TF32 step's structure, 5 products + 3 passes
    info = B.lower_info(X.mlp_step(512, 256, 512, 128))
    assert info["launches"] == 8 and info["source"].count("matmul_tiled128<") == 5
    assert nvrtc_ok(info["source"], "mlp_f32") > 0


def test_offset_streams_are_vector_loads():
    # row t of a [rows; n] buffer, t a scalar: read as one 16-byte stream,
    # checked once (range and alignment) by vec_ok; a row index that is not
    # uniform (i-dependent) stays a checked scalar gather
    rows, n = 64, 4096
    m = D.param("m", F32, (rows, n))
    tb = D.broadcast((n,), D.scalar("t", I32))
    idx = D.map2(lambda p, tv: D.add(D.mul(tv, D.const(I32, n)), p), D.iota((n,)), tb)
    src = B.lower_info(Graph("row", [("r", D.gather(idx, m))]))["source"]
    assert "K0 = ccb::ld4(p.b" in src and "u + p.n <= " in src
    rev = D.map(lambda p: D.sub(D.const(I32, n - 1), p), D.iota((n,)))
    src = B.lower_info(Graph("rev", [("r", D.gather(rev, D.reshape((rows * n,), m)))]))["source"]
    assert "K0 = " not in src


def test_staged_row_kernels_are_opt_in_and_compile(monkeypatch):
    """rows_staged (TMA-staged row tiles) is selected only with
    CCB_ROWS_STAGED=1, only for 4-byte rows of >= 1024 elements and a multiple
    of 4 read straight from a buffer, and its source compiles for sm_100a."""
    from cudacaml_b200 import dsl as D
    from cudacaml_b200.ir import F64, Graph
    g = X.rows(256, 4096)
    assert "rowsstaged" not in B.lower_info(g)["plan"]
    monkeypatch.setenv("CCB_ROWS_STAGED", "1")
    info = B.lower_info(g)
    assert "ccb_redrowsstaged_" in info["plan"] and "ccb_scanrowsstaged_" in info["plan"]
    assert nvrtc_ok(info["source"], "rows_staged") > 0
    for dt, n in ((F64, 4096), (F32, 1022), (F32, 512)):  # 8-byte, ragged, short rows keep the plain kernels
        x = D.param("x", dt, (64, n))
        assert "rowsstaged" not in B.lower_info(Graph("r", [("r", D.reduce_rows(D.add, D.const(dt, 0.0), x))]))["plan"]
    x = D.param("x", F32, (64, 4096))
    mapped = Graph("r", [("r", D.reduce_rows(D.add, D.const(F32, 0.0), D.map(D.exp, x)))])
    assert "rowsstaged" not in B.lower_info(mapped)["plan"]  # the source is an expression, not a buffer


def test_output_products_are_launched_as_soon_as_their_inputs_are_ready():
    """The MLP step's dW2 = A1^T dY needs only the forward pass and dY, so it
    is launched right after the dY/loss pass, ahead of dA1, dZ1 and dW1 (an
    all-reduce of dW2 on another stream then overlaps them); every launch
    still follows the ones whose buffers it reads."""
    for prec in ("tf32", "f32"):
        plan = B.lower_info(X.mlp_step(256, 128, 256, 64), matmul=prec)["plan"]
        launches = [ln.split()[1] for ln in plan.splitlines() if ln.startswith("launch")]
        idx = [int(re.match(r"ccb_[a-z0-9]+_(\d+)_", f).group(1)) for f in launches]
        w2 = idx.index(max(idx))  # dW2: the last group of the graph
        assert "mapreduce" in launches[w2 - 1], launches  # right after the dY / loss pass
        assert "matmul" in launches[w2 + 1] and "mapreduce" in launches[w2 + 2], launches  # then dA1, dZ1
        rest = [k for k in idx if k != max(idx)]
        assert rest == sorted(rest), launches  # the others keep graph order


def test_one_nccl_per_process():
    """libccb.so binds the NCCL that torch links against when that wheel is
    installed, so a test that imports torch after a collective of this
    library does not meet an older libnccl.so.2 bound to the same name."""
    import importlib.util
    spec = importlib.util.find_spec("nvidia.nccl")
    if spec is None:
        pytest.skip("no nvidia-nccl wheel")
    R.lib()
    maps = [ln.split()[-1] for ln in open("/proc/self/maps") if "libnccl.so" in ln]
    assert maps and all("nvidia/nccl/lib" in m for m in maps), sorted(set(maps))
