"""Counter-based random numbers built out of the DSL, restating CUDACaml's
``Rng`` (lib/rng/rng.ml:1-74, lib/rng/rng.mli).

Philox-4x32-10 (Salmon, Moraes, Dror, Shaw 2011): a pure function from a
128-bit counter and a 64-bit key to four 32-bit words. Element ``i`` of a random
tensor uses counter ``(i, 0, 0, 0)`` and key ``(seed, 0)`` and keeps word 0
only (rng.ml:49-59). The multipliers and Weyl constants are the published
Philox parameters (rng.ml:8-15). Because the generator is an expression tree,
it fuses into whatever consumes it and is never materialised.
"""
from __future__ import annotations

import math

from . import dsl as D
from .ir import F64, I32, I64, Dtype, Tensor

# Philox-4x32 round multipliers and key-schedule (Weyl) increments.
M0 = 0xD2511F53
M1 = 0xCD9E8D57
W0 = 0x9E3779B9
W1 = 0xBB67AE85


def _wide(x):
    """Zero-extend an I32 word into I64 (rng.ml:20-21)."""
    return D.bit_and(D.cast(I64, x), D.const(I64, 0xFFFFFFFF))


def mulhilo32(a, b):
    """The full 64-bit product split into (hi, lo) words (rng.ml:26-29)."""
    lo = D.mul(a, b)
    hi = D.cast(I32, D.shr(D.mul(_wide(a), _wide(b)), D.const(I64, 32)))
    return hi, lo


def _round(ctr, key):
    c0, c1, c2, c3 = ctr
    k0, k1 = key
    hi0, lo0 = mulhilo32(D.const(I32, M0), c0)
    hi1, lo1 = mulhilo32(D.const(I32, M1), c2)
    return (D.bit_xor(D.bit_xor(hi1, c1), k0), lo1, D.bit_xor(D.bit_xor(hi0, c3), k1), lo0)


def _bump(key):
    k0, k1 = key
    return D.add(k0, D.const(I32, W0)), D.add(k1, D.const(I32, W1))


def round10(ctr, key):
    """Ten rounds; the key is bumped after each of the first nine only
    (rng.ml:41-46)."""
    for n in range(1, 11):
        ctr = _round(ctr, key)
        if n < 10:
            key = _bump(key)
    return ctr


def u32(key: Tensor, shape) -> Tensor:
    """Element i = word 0 of Philox(ctr=(i,0,0,0), key=(key,0)) (rng.ml:49-59)."""
    i = D.iota(shape)
    k = D.broadcast(shape, key)
    z = D.const(I32, 0)

    def body(ii, kk):
        w0, _, _, _ = round10((ii, z, z, z), (kk, z))
        return w0

    return D.map2(body, i, k)


def to_unit_interval(dtype: Dtype, w):
    """Read the word as unsigned, map to (0,1) as (u + 0.5) * 2^-32 in F64,
    then cast (rng.ml:61-67)."""
    f = D.cast(F64, w)
    u = D.select(D.lt(w, D.const(I32, 0)), D.add(f, D.const(F64, 4294967296.0)), f)
    return D.cast(dtype, D.mul(D.add(u, D.const(F64, 0.5)), D.const(F64, 2.3283064365386963e-10)))


def normal_inv_cdf(u):
    """sqrt 2 * erfinv (2u - 1) (rng.ml:69-71)."""
    d = u.dtype
    return D.mul(D.const(d, math.sqrt(2.0)), D.erfinv(D.sub(D.mul(D.const(d, 2.0), u), D.const(d, 1.0))))


def uniform(dtype: Dtype, key: Tensor, shape) -> Tensor:
    return D.map(lambda w: to_unit_interval(dtype, w), u32(key, shape))


def normal(dtype: Dtype, key: Tensor, shape) -> Tensor:
    return D.map(normal_inv_cdf, uniform(dtype, key, shape))
