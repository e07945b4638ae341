"""The corrected-reciprocal quotient used by the exact-settle kernel (``quot_rn`` in
``fracture_b200/csrc/tq_umma.cu``), checked with exact rational arithmetic.

For fp16 numerators x and denominators den = norm + 1e-8 with |x| <= den <= 2^20, the
sequence r = RN(1/den), q0 = RN(x r), q1 = RN(q0 + RN(x - den q0) r) [FMA],
q = RN(q1 + (x - den q1) r) [FMA] must equal RN(x / den), the correctly rounded
quotient of the float32 statement, and the second remainder must be exact. Float32
round-to-nearest-even is emulated exactly with Fractions.
"""

import struct
from fractions import Fraction as F

import numpy as np


def _rn32(x: F) -> F:
    if x == 0:
        return F(0)
    sign = -1 if x < 0 else 1
    x = abs(x)
    e = x.numerator.bit_length() - x.denominator.bit_length()
    while F(2) ** e > x:
        e -= 1
    while F(2) ** (e + 1) <= x:
        e += 1
    ulp = F(2) ** (e - 23)
    m = x / ulp
    fl = m.numerator // m.denominator
    rem = m - fl
    if rem > F(1, 2) or (rem == F(1, 2) and fl % 2 == 1):
        fl += 1
    return sign * fl * ulp


def _cases(n, seed):
    rng = np.random.default_rng(seed)
    out = []
    while len(out) < n:
        a = float(np.float16(rng.standard_normal() * 10.0 ** rng.uniform(-5, 4.5)))
        if not np.isfinite(a):
            continue
        k = rng.random()
        if k < 0.6:
            b = float(np.float32(abs(a) * rng.uniform(1.0, 60.0) + 1e-8))
        elif k < 0.8:  # all-ones mantissas
            ex = int(rng.integers(-20, 20))
            b = struct.unpack("<f", struct.pack("<I", ((ex + 127) << 23) | 0x7FFFFF))[0]
        else:
            b = float(np.float32(rng.uniform(1e-8, 7.5e5)))
        if b < abs(a):
            b = float(np.float32(abs(a) * 1.0000001 + 1e-8))
        out.append((a, b))
    out += [(0.0, 1e-8), (-0.0, 3.0), (65504.0, 65504.0), (-65504.0, 741000.0), (2.0 ** -24, 2.0 ** -24),
            (2.0 ** -24, 741000.0), (1.0, 3.0), (-1.0, 3.0)]
    return out


def test_corrected_reciprocal_quotient_is_correctly_rounded():
    for a, b in _cases(6000, 3):
        A, B = F(a), F(b)
        r = _rn32(1 / B)
        q0 = _rn32(A * r)
        q1 = _rn32(q0 + _rn32(A - q0 * B) * r)
        rem = A - q1 * B
        assert _rn32(rem) == rem, (a, b)
        assert _rn32(q1 + rem * r) == _rn32(A / B), (a, b)


def _divu32_params(d):
    """Multiplier and shifts of the round-up method (``make_divu32`` in
    ``fracture_b200/csrc/tq_sm100.cuh``): Granlund and Montgomery, PLDI 1994, section 4."""
    l = 0
    while (1 << l) < d:
        l += 1
    m = ((1 << 32) * ((1 << l) - d)) // d + 1
    assert 0 < m < (1 << 32)
    return m, min(l, 1), max(l - 1, 0)


def _divu32(n, params):
    m, s1, s2 = params
    t = (m * n) >> 32
    return (t + ((n - t) >> s1)) >> s2


def test_invariant_divisor_quotient_is_exact():
    """n / d by multiply-high and shifts equals floor division for every divisor tried, at the
    dividends where a wrong multiplier would show first (around multiples of d and at 2^32 - 1)."""
    rng = np.random.default_rng(7)
    divisors = list(range(1, 300)) + [2 ** k for k in range(32)] + [2 ** k - 1 for k in range(2, 33)] + \
        [2 ** k + 1 for k in range(2, 32)] + [int(x) for x in rng.integers(1, 2 ** 32, 200)]
    for d in divisors:
        p = _divu32_params(d)
        ns = [0, 1, d - 1, d, d + 1, 2 ** 31 - 1, 2 ** 31, 2 ** 32 - 1] + \
            [int(x) for x in rng.integers(0, 2 ** 32, 64)]
        q = (2 ** 32 - 1) // d
        ns += [q * d, q * d - 1, min(q * d + d - 1, 2 ** 32 - 1)]
        for n in ns:
            if 0 <= n < 2 ** 32:
                assert _divu32(n, p) == n // d, (d, n)
