"""FP16 values summed in FP16 (the reference's SPMV_HALF_ACCUMULATE control build, value_types.cuh:7-33):
the oracle's FP16 fma (a*b + c rounded once, round to nearest even, what __hfma computes) checked
against exact rational arithmetic, including exact ties and the overflow boundary, and the FP16-sum
product order (every entry one fma, every tree step one FP16 add)."""
import bisect
from fractions import Fraction

import numpy as np

import oracle

# every finite FP16 value, ascending, as exact fractions
_BITS = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
_ALL = _BITS.view(np.float16)
_FINITE = np.unique(_ALL[np.isfinite(_ALL)].astype(np.float64))
_FRACTIONS = [Fraction(v) for v in _FINITE]
_LARGEST = Fraction(65504)


def round_to_half(exact: Fraction, sign_if_zero: float) -> np.float16:
    """exact rounded to FP16, to nearest with ties to even (binary16 significands)."""
    if exact >= _LARGEST + 16:          # 65520 and above (the tie at 65520 goes to the even 2^16): inf
        return np.float16(np.inf)
    if exact <= -_LARGEST - 16:
        return np.float16(-np.inf)
    if exact > _LARGEST:                 # (65504, 65520): below the midpoint to infinity
        return np.float16(65504)
    if exact < -_LARGEST:
        return np.float16(-65504)
    i = bisect.bisect_left(_FRACTIONS, exact)
    if i < len(_FRACTIONS) and _FRACTIONS[i] == exact:
        value = _FINITE[i]
    else:
        low, high = _FINITE[i - 1], _FINITE[i]
        below, above = exact - _FRACTIONS[i - 1], _FRACTIONS[i] - exact
        if below != above:
            value = low if below < above else high
        else:                            # the one with the even significand
            low_bits = int(np.float16(low).view(np.uint16))
            value = low if low_bits % 2 == 0 else high
    if value == 0:
        return np.float16(np.copysign(0.0, sign_if_zero))
    return np.float16(value)


def reference_fma(a, b, c):
    out = np.zeros(a.size, np.float16)
    for k in range(a.size):
        exact = Fraction(float(a[k])) * Fraction(float(b[k])) + Fraction(float(c[k]))
        if exact == 0:                   # an exact zero sum is +0, unless both addends are -0
            product_negative_zero = (float(a[k]) * float(b[k]) == 0) and np.signbit(np.float64(a[k]) * np.float64(b[k]))
            sign = -1.0 if (product_negative_zero and np.signbit(c[k])) else 1.0
        else:
            sign = float(exact)
        out[k] = round_to_half(exact, sign)
    return out


def samples(rng, count):
    groups = []
    # random finite values across the range
    bits = rng.integers(0, 1 << 16, 3 * count).astype(np.uint16).view(np.float16)
    bits = bits[np.isfinite(bits)][:3 * (count // 3) * 1]
    a, b, c = bits[:count // 3], bits[count // 3:2 * (count // 3)], bits[2 * (count // 3):3 * (count // 3)]
    groups.append((a, b, c))
    # short significands: products land exactly on FP16 midpoints (ties)
    small = lambda n: (rng.integers(-64, 64, n) * 2.0 ** rng.integers(-6, 6, n)).astype(np.float16)  # noqa: E731
    groups.append((small(count), small(count), (rng.integers(-4096, 4096, count) * 2.0 ** -4).astype(np.float16)))
    # near the overflow boundary
    big = np.float16(255.875)
    groups.append((np.full(count // 4, big), (rng.integers(250, 257, count // 4)).astype(np.float16),
                   (rng.integers(-64, 64, count // 4) * 1.0).astype(np.float16)))
    return groups


def test_half_fma_is_rounded_once_to_nearest_even():
    rng = np.random.default_rng(11)
    for a, b, c in samples(rng, 9000):
        got = oracle.half_fma(a, b, c)
        want = reference_fma(a, b, c)
        assert np.array_equal(got.view(np.uint16), want.view(np.uint16)), \
            [(float(a[k]), float(b[k]), float(c[k]), float(got[k]), float(want[k]))
             for k in np.nonzero(got.view(np.uint16) != want.view(np.uint16))[0][:5]]


def test_half_sum_product_order():
    """A row of FP16 sums: lane L's fmas over entries L, L+T, ... then the FP16 tree (T/2, ..., 1)."""
    rng = np.random.default_rng(12)
    n, tpr = 40, 8
    row_ptr = np.array([0, 37], dtype=np.int32)
    col_ind = np.sort(rng.choice(n, 37, replace=False)).astype(np.int32)
    values = rng.uniform(-1, 1, 37)
    x = rng.uniform(-1, 1, n).astype(np.float16)
    y = oracle.spmv_csr(row_ptr, col_ind, values, x, oracle.F16_HALF_SUMS, 0, tpr)
    v = oracle.convert_values(values, oracle.F16)
    lanes = []
    for lane in range(tpr):
        acc = np.float16(0)
        for e in range(lane, 37, tpr):
            acc = oracle.half_fma(np.array([v[e]]), np.array([x[col_ind[e]]]), np.array([acc]))[0]
        lanes.append(acc)
    offset = tpr // 2
    while offset:
        for lane in range(offset):
            lanes[lane] = np.float16(np.float64(lanes[lane]) + np.float64(lanes[lane + offset]))
        offset //= 2
    assert y.view(np.uint16)[0] == np.float16(lanes[0]).view(np.uint16)


def test_half_sums_need_fp16_values():
    """SPMV_ACCUMULATE_HALF is refused for FP64 and FP32 operators, and unknown values are refused, before any
    device is touched."""
    import pytest
    import spmvb200 as spmv
    matrix = spmv.synth_laplacian2d(16)
    for dtype, accumulate in ((spmv.F64, spmv.ACCUMULATE_HALF), (spmv.F32, spmv.ACCUMULATE_HALF), (spmv.F16, 2)):
        with pytest.raises(spmv.SpmvError) as error:
            spmv.Operator(matrix, spmv.I32, dtype, 4, accumulate=accumulate)
        assert error.value.status == spmv.ERR_INVALID_ARGUMENT
