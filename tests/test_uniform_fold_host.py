"""The lowering's exact fold of Rng's word-to-float chain (CPU only).

Rng reads a Philox word as unsigned through a select on its sign, maps it to
(u + 0.5) * 2^-32 in F64, and Rng.normal takes 2u - 1 (rng.ml:61-74). The
lowering emits that chain as one unsigned conversion and one FMA. It is the
same function bit for bit because every intermediate value of the chain is
exact in F64: checked here in exact rational arithmetic for edge and random
words, against the chain evaluated step by step in IEEE doubles (Python
floats), for both forms the lowering emits. The GPU suite checks the device's
uniform and normal streams against the oracle bit for bit."""
from fractions import Fraction

import numpy as np

from cudacaml_b200 import backend_cuda as B
from cudacaml_b200 import examples as X
from cudacaml_b200.ir import F32, F64


def _chain(w: int):
    """The reference chain in IEEE doubles for the signed I32 word w."""
    f = float(w)
    u = f + 4294967296.0 if w < 0 else f
    uni = (u + 0.5) * 2.3283064365386963e-10
    return uni, uni * 2.0 - 1.0


def test_chain_is_exact_so_one_fma_equals_it():
    rng = np.random.default_rng(5)
    words = [0, 1, -1, 2**31 - 1, -(2**31), 12345, -12345] + [int(x) for x in rng.integers(-(2**31), 2**31, 5000)]
    for w in words:
        uw = w % (1 << 32)
        uni, nrm = _chain(w)
        # the values the two FMAs compute, exactly (an FMA rounds once; an exact value is returned as is)
        assert Fraction(uni) == Fraction(uw) * Fraction(1, 2**32) + Fraction(1, 2**33), w
        assert Fraction(nrm) == Fraction(uw) * Fraction(1, 2**31) + (Fraction(1, 2**32) - 1), w


def test_greeks_source_uses_the_folded_form():
    for dt in (F64, F32):
        src = B.source(X.call_greeks(1 << 20, dt))
        assert "(double)(unsigned int)(" in src and "fma(" in src, dt
        assert "0x1p+32" not in src  # the sign fix-up select is gone


def test_philox_high_and_low_words_share_one_product():
    """Each Philox multiply whose high and low words are both used is
    emitted once, as a 64-bit product both words are read from."""
    src = B.source(X.call_greeks(1 << 20, F64))
    body = src[src.find("void elem(const P& p, int i"):src.find("void elem4(")]
    # 20 products per draw; the last round's feed only word 0 through their high words
    assert body.count("const unsigned long long w") >= 12
    assert body.count("__umulhi") <= 4
