"""``Differential.check``: run a graph on a reference backend and a candidate
and compare every output by name (lib/backend/differential.ml:80-88), with
the reference's mismatch messages (differential.ml:36-61).

Floats use the relative-plus-absolute band |g - e| <= tol * (1 + |e|) with
NaN == NaN (differential.ml:6-8); integers must be exactly equal
(differential.ml:17-19). The default tolerance is 1e-5.
"""
from __future__ import annotations

import numpy as np

from .ir import shape_to_string


def float_close(tolerance: float, e, g):
    e = np.asarray(e, dtype=np.float64)
    g = np.asarray(g, dtype=np.float64)
    both_nan = np.isnan(e) & np.isnan(g)
    with np.errstate(invalid="ignore"):
        ok = np.abs(g - e) <= tolerance * (1.0 + np.abs(e))
    return both_nan | ok


def compare_one(tolerance, output, e, g):
    if e.dtype is not g.dtype:
        return f"output {output}: dtype mismatch: expected {e.dtype.value}, got {g.dtype.value}"
    if tuple(e.shape) != tuple(g.shape):
        return (f"output {output}: shape mismatch: expected {shape_to_string(e.shape)}, "
                f"got {shape_to_string(g.shape)}")
    if e.dtype.is_float:
        ok = float_close(tolerance, e.data, g.data)
    else:
        ok = e.data == g.data
    if not np.all(ok):
        i = int(np.argmin(ok))
        return f"output {output}[{i}]: expected {float(e.data[i]):g}, got {float(g.data[i]):g} (tol {tolerance:g})"
    return None


def compare_all(tolerance, expected, got):
    got = dict(got)
    for output, e in expected:
        if output not in got:
            return f"missing output {output}"
        err = compare_one(tolerance, output, e, got[output])
        if err:
            return err
    return None


def check(reference, candidate, graph, inputs, tolerance: float = 1e-5):
    """Returns None when the candidate agrees, else the first mismatch as a
    string (the reference's [Error msg])."""
    try:
        expected = reference.run(reference.compile(graph), inputs)
    except Exception as e:  # noqa: BLE001 - mirrors "<name> raised: <exn>"
        return f"{reference.name} raised: {e}"
    try:
        got = candidate.run(candidate.compile(graph), inputs)
    except Exception as e:  # noqa: BLE001
        return f"{candidate.name} raised: {e}"
    return compare_all(tolerance, expected, got)
