"""Exhaustive proof of the quantize kernel's division-free code formula.

An element's code depends only on the pair (x, amax), both bf16, so all finite
pairs can be enumerated (about 5e8 per qmax). The kernel computes
s = amax / qmax (IEEE), r = 1/s (correctly rounded) and the Markstein-refined
quotient y = fma(fma(-x*r, s, x), r, x*r), code = rne(y), with the exact IEEE
divide for groups with amax < 2^-100. This test checks that formula against
the reference's rne(x / s) (quant_kv.py:151-153) on every pair.
"""
from oracle import c_oracle


def test_fast_code_formula_is_exact_int4():
    n, first = c_oracle.check_fast_codes(7, 2.0 ** -100)
    assert n == 0, f"{n} mismatches, first (amax, x) bf16 bits = {first}"


def test_fast_code_formula_is_exact_int8():
    n, first = c_oracle.check_fast_codes(127, 2.0 ** -100)
    assert n == 0, f"{n} mismatches, first (amax, x) bf16 bits = {first}"


def test_plain_reciprocal_is_not_exact():
    # Without the guard the formula breaks on tiny scales; this pins that the
    # guard (and the check itself) is doing work.
    n, _ = c_oracle.check_fast_codes(7, 0.0)
    assert n > 0


def test_group_scale_without_divide_is_exact():
    # s = fma(fma(-amax*r, qmax, amax), r, amax*r), r = RN(1/qmax), equals the
    # IEEE amax / qmax for every positive finite bf16 amax
    assert c_oracle.check_scale_div(7) == 0
    assert c_oracle.check_scale_div(127) == 0


def test_fast_code_formula_holds_for_any_one_ulp_reciprocal():
    # the kernel's reciprocal is an approximation refined by one Newton step,
    # within one ulp of 1/s: the formula must hold for RN(1/s) and both neighbours
    for qmax in (7, 127):
        n, first = c_oracle.check_fast_codes_any_rcp(qmax, 2.0 ** -100)
        assert n == 0, f"qmax {qmax}: {n} mismatches, first {first}"
