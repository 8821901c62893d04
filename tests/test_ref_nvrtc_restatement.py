"""The restated reference NVRTC backend (baseline/ref_nvrtc.py), the timed
"reference NVRTC" baseline of bench.py, checked on the CPU: it plans the
buffers and kernels the reference's compiler does -- the Greeks graph lowers
to the reference's 25 kernels (README.md:151-152 of the reference), saxpy
to a map plus the two-pass reduce (16 bytes per element), a flat scan of
2^28 to the three-pass chunk scan with 2^20 chunks -- and its CUDA text
compiles with NVRTC and no options, as the reference's Jit does."""
import pytest

from baseline import ref_nvrtc as RN
from cudacaml_b200 import examples as X
from cudacaml_b200.ir import F32, F64

nvrtc = pytest.importorskip("cuda.bindings.nvrtc")


def _compiles(src):
    p = RN._ck(nvrtc.nvrtcCreateProgram(src.encode(), b"ref.cu", 0, [], []), "nvrtcCreateProgram")
    try:
        res = nvrtc.nvrtcCompileProgram(p, 0, [])
        size = RN._ck(nvrtc.nvrtcGetProgramLogSize(p), "log size")
        log = b" " * size
        nvrtc.nvrtcGetProgramLog(p, log)
        return int(res[0]) == 0, log.decode(errors="replace")
    finally:
        nvrtc.nvrtcDestroyProgram(p)


def test_kernel_plans_follow_the_reference():
    greeks = RN.Program(X.call_greeks(1 << 20, F64))
    assert len(greeks.kernels) == 25
    saxpy = RN.Program(X.saxpy(1 << 20, 2.0))
    assert len(saxpy.kernels) == 3 and saxpy.kernels[1].name.endswith("_partial")
    assert saxpy.kernels[0].launch == (1024, 1, 256, 1)  # grid-stride, capped at 1024 blocks
    assert saxpy.kernels[1].launch == (128, 1, 256, 1)  # reduce_blocks caps at 128
    scan = RN.Program(X.scan_flat(1 << 28, F32))
    assert [k.launch for k in scan.kernels] == [(1 << 20, 1, 256, 1), (1, 1, 1, 1), (1024, 1, 256, 1)]
    mm = RN.Program(X.mlp_step(256, 128, 256, 64))
    assert any(k.launch[2:] == (16, 16) for k in mm.kernels)


@pytest.mark.parametrize("name,g", [("saxpy", X.saxpy(1 << 20, 2.0)), ("scan", X.scan_flat(1 << 20, F32)),
                                    ("rows", X.rows(64, 4096)), ("scatter", X.scatter(1 << 20, 1 << 16)),
                                    ("greeks", X.call_greeks(1 << 16, F32)), ("mlp", X.mlp_step(64, 32, 64, 16))],
                         ids=lambda v: v if isinstance(v, str) else "")
def test_restated_source_compiles_with_no_options(name, g):
    ok, log = _compiles(RN.Program(g).source)
    assert ok, log[:2000]
