"""cudacaml_b200 -- a B200-native execution backend for CUDACaml graphs.

The package mirrors the reference's public surface (``Dsl``, ``Graph``,
``Rng``, ``Grad``, ``Backend.S``, ``Multi``, ``Differential``) in Python and
runs graphs through libccb.so: native lowering to hand-written sm_100a kernel
skeletons, NVRTC, and a stream-ordered executor.
"""
from . import dsl, grad, ir, rng, wire  # noqa: F401
from .ir import BOOL, F32, F64, I32, I64, SCALAR, Dtype, Graph, Tensor, Value  # noqa: F401

__all__ = ["dsl", "grad", "ir", "rng", "wire", "Graph", "Tensor", "Value", "Dtype",
           "F32", "F64", "I32", "I64", "BOOL", "SCALAR"]
