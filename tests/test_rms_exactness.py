"""The exactness argument behind the tree-summed RMS partials (CPU only).

For bf16-valued elements whose nonzero biased exponents span at most 15, every partial sum of at
most 128 squares is an integer multiple of 2^(2 e_min - 268) below 2^53 of those units, so the
sequential double sum equals the exact sum in any order.  Checked here against exact rational
sums, together with a case just outside the bound where the sequential sum does round."""
from fractions import Fraction

import numpy as np

from oracle_lib import bf16_bits, bf16_to_f32


def r16(a):
    return bf16_to_f32(bf16_bits(np.ascontiguousarray(a, np.float32)))


def r16s(v):
    return r16(np.array([v], np.float32))[0]


def seq_sum(xs):
    s = 0.0
    for v in xs:
        s = s + float(v) * float(v)  # the square of a float is exact in double
    return s


def span(xs):
    e = [max(int((np.float32(v).view(np.uint32) >> 23) & 0xFF), 1) for v in xs if v != 0]
    return (max(e) - min(e)) if e else 0


def test_sequential_sum_is_exact_within_span_15():
    rng = np.random.default_rng(0)
    checked = 0
    for trial in range(400):
        scale = np.float32(2.0) ** rng.integers(-60, 60)
        xs = r16(rng.standard_normal(128, dtype=np.float32) * scale)
        # force the span to exactly 15 binades in half the trials
        if trial % 2 == 0:
            xs[0] = r16s(np.float32(1.5) * scale * np.float32(2.0 ** 8))
            xs[1] = r16s(np.float32(1.0) * scale * np.float32(2.0 ** -7))
        if span(xs) > 15:
            continue
        exact = sum((Fraction(float(v)) ** 2 for v in xs), Fraction(0))
        assert Fraction(seq_sum(xs)) == exact
        assert Fraction(seq_sum(xs[::-1])) == exact
        checked += 1
    assert checked > 150


def test_sum_can_round_outside_the_bound():
    xs = np.zeros(128, np.float32)
    xs[0] = r16s(np.float32(1.9921875) * np.float32(2.0 ** 30))
    xs[1:] = r16s(np.float32(1.0078125))
    assert span(xs) == 30
    exact = sum((Fraction(float(v)) ** 2 for v in xs), Fraction(0))
    assert Fraction(seq_sum(xs)) != exact
