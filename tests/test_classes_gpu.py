"""GPU parity of the rows-by-length schedule (SPMV_SCHEDULE_CLASSES): short rows one per thread, listed
rows on groups of P threads (P per row, from 1 to T), long rows one per CTA, all straight from global
memory. Every class must give the reference's CSR-i32 results bit for bit."""
import numpy as np
import pytest

import oracle
import spmvb200 as spmv
from conftest import random_csr

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DTYPES = (spmv.F64, spmv.F32, spmv.F16)
TORCH = {spmv.F64: torch.float64, spmv.F32: torch.float32, spmv.F16: torch.float16}


def bits(array):
    return np.ascontiguousarray(array).view(np.uint8)


def device_run(op, x):
    x_device = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    y_device = torch.full((op.rows,), float("nan"), dtype=TORCH[op.dtype], device="cuda")
    op.run(x_device.data_ptr(), y_device.data_ptr(), 0)
    torch.cuda.synchronize()
    op.check()
    return y_device.cpu().numpy()


def skewed_lengths(rng):
    """Mostly rows of 0..8 entries, some of 9..128, a few of 129..1500 (a power-law-like mix)."""
    draw = rng.random()
    if draw < 0.80:
        return rng.integers(0, 9)
    if draw < 0.97:
        return rng.integers(9, 129)
    return rng.integers(129, 1500)


@pytest.fixture(scope="module")
def skewed():
    rows, cols = 5000, 6000
    row_ptr, col_ind, values = random_csr(rows, cols, skewed_lengths, 21, empty_every=31,
                                          long_rows={3: 4100, 777: 2049, 4999: 6000})
    return spmv.CsrMatrix.from_arrays(rows, cols, row_ptr, col_ind, values, name="skewed")


def oracle_product(matrix, x, dtype, layout, tpr):
    row_ptr, col_ind, values = matrix.arrays()
    return oracle.spmv_csr(row_ptr, col_ind, values, x, dtype, layout, tpr)


def test_skewed_rows_choose_classes(skewed):
    with spmv.Operator(skewed, spmv.I32, spmv.F32, 32) as op:
        info = op.info()
    assert info.schedule == spmv.SCHEDULE_CLASSES
    assert info.listed_rows > 0 and info.long_rows > 0 and info.tiles == 0
    regular = spmv.synth_stencil27(20)
    with spmv.Operator(regular, spmv.I32, spmv.F64, 8) as op:
        assert op.info().schedule == spmv.SCHEDULE_TILES


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("tpr", spmv.THREADS_PER_ROW)
def test_classes_match_oracle_every_layout(skewed, dtype, tpr):
    x = spmv.fill_uniform(dtype, skewed.cols, 13)
    for layout in (spmv.I32, spmv.I16, spmv.R16, spmv.LP):
        if not spmv.configuration_admissible(skewed, None, spmv.Configuration.of(layout, dtype, tpr)):
            continue
        expected = oracle_product(skewed, x, dtype, layout, tpr)
        for schedule in (spmv.SCHEDULE_CLASSES, spmv.SCHEDULE_TILES):
            with spmv.Operator(skewed, layout, dtype, tpr, schedule=schedule) as op:
                assert op.info().schedule == schedule
                y = device_run(op, x)
            assert np.array_equal(bits(y), bits(expected)), (spmv.LAYOUT_NAMES[layout], tpr, schedule)


@pytest.mark.parametrize("dtype", DTYPES)
def test_classes_narrow_8bit_and_empty(dtype):
    """8-bit layouts, an all-empty matrix and a matrix of only short rows under the class schedule."""
    rows, cols = 900, 256
    row_ptr, col_ind, values = random_csr(rows, cols, lambda rng: rng.integers(0, 12), 4, empty_every=5,
                                          long_rows={10: 256, 11: 200})
    matrix = spmv.CsrMatrix.from_arrays(rows, cols, row_ptr, col_ind, values)
    x = spmv.fill_uniform(dtype, cols, 8)
    for tpr in spmv.THREADS_PER_ROW:
        for layout in (spmv.I8, spmv.R8):
            with spmv.Operator(matrix, layout, dtype, tpr, schedule=spmv.SCHEDULE_CLASSES) as op:
                y = device_run(op, x)
            assert np.array_equal(bits(y), bits(oracle_product(matrix, x, dtype, spmv.I32, tpr)))
    empty = spmv.CsrMatrix.from_arrays(300, 40, np.zeros(301, np.int32), np.zeros(0, np.int32), np.zeros(0))
    with spmv.Operator(empty, spmv.LP, dtype, 8, schedule=spmv.SCHEDULE_CLASSES) as op:
        y = device_run(op, spmv.fill_uniform(dtype, 40, 1))
    assert np.all(bits(y) == 0)


def test_underflow_signs_in_short_rows():
    """Products that underflow to -0 in every lane of short rows: y is -0 where the full T-lane tree adds
    only -0 lane sums (T = 2, 4, 8) and +0 where it adds an empty (+0) lane first (T = 16, 32)."""
    rows, cols = 64, 8
    lengths = np.arange(rows) % 8 + 1                        # rows of 1..8 entries, every lane sum -0
    row_ptr = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    col_ind = np.concatenate([np.arange(length) for length in lengths]).astype(np.int32)
    values = np.full(col_ind.size, -1e-300)
    matrix = spmv.CsrMatrix.from_arrays(rows, cols, row_ptr, col_ind, values)
    x = np.full(cols, 1e-300)
    for tpr in spmv.THREADS_PER_ROW:
        with spmv.Operator(matrix, spmv.I32, spmv.F64, tpr, schedule=spmv.SCHEDULE_CLASSES, value_rounding=1) as op:
            y = device_run(op, x)
        expected = oracle.spmv(spmv.F64, spmv.I32, tpr, row_ptr, values, x, columns=col_ind)
        assert np.array_equal(bits(y), bits(expected)), tpr
