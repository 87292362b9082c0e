"""The restatement's float32 fused multiply-add (oracle/kernel_order.py: fma32), which the routing
proxy's partial sums use (fma.rn.f32x2 on the GPU), against exact rational arithmetic rounded
once to the nearest float32 (ties to even): random operands over wide exponent ranges and
constructed cases whose float64 sum lands exactly on a float32 midpoint (where a float64
evaluation rounded twice would be wrong)."""

from fractions import Fraction

import numpy as np

from oracle.kernel_order import fma32

F32 = np.float32


def _round32(x: Fraction) -> np.float32:
    f = F32(float(x))  # within one float32 step of the exact value
    cands = [np.nextafter(f, F32(-np.inf)), f, np.nextafter(f, F32(np.inf))]
    return min(cands, key=lambda v: (abs(Fraction(float(v)) - x),
                                     int(np.array(v, F32).view(np.uint32)) & 1))


def _exact(a, b, c):
    return np.array([_round32(Fraction(float(x)) * Fraction(float(y)) + Fraction(float(z)))
                     for x, y, z in zip(a, b, c)], F32)


def _check(a, b, c):
    a, b, c = (np.asarray(v, F32) for v in (a, b, c))
    got = fma32(a, b, c)
    want = _exact(a, b, c)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, [(a[i], b[i], c[i], got[i], want[i]) for i in bad[:5]]


def test_random_operands():
    rng = np.random.default_rng(0)
    n = 4000
    a = (rng.standard_normal(n) * np.exp2(rng.integers(-20, 20, n))).astype(F32)
    b = (rng.standard_normal(n) * np.exp2(rng.integers(-20, 20, n))).astype(F32)
    c = (rng.standard_normal(n) * np.exp2(rng.integers(-40, 40, n))).astype(F32)
    _check(a, b, c)
    # the routing proxy's own range: means of O(1) values, partial sums of a few units
    _check(rng.standard_normal(n).astype(F32) * F32(0.05), rng.standard_normal(n).astype(F32),
           rng.standard_normal(n).astype(F32) * F32(2))


def test_float64_sum_on_a_float32_midpoint():
    # a * b = 2^-24 (1 - 2^-30) exactly; c + a * b lies 2^-54 below the midpoint of c and its
    # upper neighbour, and the float64 sum rounds onto that midpoint.
    a = F32(2.0 ** -12 * (1 + 2.0 ** -15))
    b = F32(2.0 ** -12 * (1 - 2.0 ** -15))
    cs = [F32(1.0), F32(1 + 2.0 ** -23), F32(1 + 3 * 2.0 ** -23), F32(1.5), F32(1.75 + 2.0 ** -22)]
    _check([a] * len(cs), [b] * len(cs), cs)
    # and below zero, mirrored
    _check([-a] * len(cs), [b] * len(cs), [-x for x in cs])
    # a midpoint reached exactly (a tie: even wins) and one float64 step above it
    half = F32(2.0 ** -24)
    _check([half, half], [F32(1.0), F32(1.0)], [F32(1.0), F32(1 + 2.0 ** -23)])
    rng = np.random.default_rng(1)
    # products just under / over half a step of random c
    c = (1 + rng.integers(0, 2 ** 23, 500) * 2.0 ** -23).astype(F32)
    _check(np.full(500, a), np.full(500, b), c)
