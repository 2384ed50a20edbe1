"""FP16 values summed in FP16 on the GPU (SPMV_ACCUMULATE_HALF, the reference's SPMV_HALF_ACCUMULATE
control build): every schedule and layout bit-identical to the oracle's FP16-sum restatement, and
different from the FP32-sum products (so the FP16 kernels are the ones that ran)."""
import numpy as np
import pytest

import oracle
import spmvb200 as spmv
from conftest import random_csr

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def run(op, x):
    x_device = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    y_device = torch.full((op.rows,), float("nan"), dtype=torch.float16, device="cuda")
    op.run(x_device.data_ptr(), y_device.data_ptr())
    torch.cuda.synchronize()
    op.check()
    return y_device.cpu().numpy()


@pytest.fixture(scope="module")
def ragged():
    rows, cols = 3000, 2500
    row_ptr, col_ind, values = random_csr(rows, cols, lambda rng: rng.integers(0, 60), 7, empty_every=23,
                                          long_rows={11: 2400, 1500: 2049, 2999: 2500})
    return spmv.CsrMatrix.from_arrays(rows, cols, row_ptr, col_ind, values, name="ragged")


@pytest.mark.parametrize("tpr", spmv.THREADS_PER_ROW)
def test_half_sums_match_the_oracle(ragged, tpr):
    row_ptr, col_ind, values = ragged.arrays()
    x = spmv.fill_uniform(spmv.F16, ragged.cols, 13)
    for layout in (spmv.I32, spmv.I16, spmv.R16, spmv.LP):
        if not spmv.configuration_admissible(ragged, None, spmv.Configuration.of(layout, spmv.F16, tpr)):
            continue
        expected = oracle.spmv_csr(row_ptr, col_ind, values, x, oracle.F16_HALF_SUMS, layout, tpr)
        wide = oracle.spmv_csr(row_ptr, col_ind, values, x, spmv.F16, layout, tpr)
        assert not np.array_equal(expected.view(np.uint16), wide.view(np.uint16))
        for options in ({"tile_nnz": 2048}, {}, {"schedule": spmv.SCHEDULE_CLASSES}):
            with spmv.Operator(ragged, layout, spmv.F16, tpr, accumulate=spmv.ACCUMULATE_HALF, **options) as op:
                y = run(op, x)
            assert np.array_equal(y.view(np.uint16), expected.view(np.uint16)), (spmv.LAYOUT_NAMES[layout], tpr, options)


def test_half_sums_dense_variant():
    """Rows of column runs with one thread per lane: the dense FP16-sum tile variant."""
    matrix = spmv.synth_block_fem(20000, 8, 8, 2000, 4, 0, 20000)
    row_ptr, col_ind, values = matrix.arrays()
    x = spmv.fill_uniform(spmv.F16, matrix.cols, 14)
    for layout, tpr in ((spmv.I32, 8), (spmv.LP, 16)):
        with spmv.Operator(matrix, layout, spmv.F16, tpr, accumulate=spmv.ACCUMULATE_HALF) as op:
            assert op.info().physical_tpr == tpr
            y = run(op, x)
        expected = oracle.spmv_csr(row_ptr, col_ind, values, x, oracle.F16_HALF_SUMS, layout, tpr)
        assert np.array_equal(y.view(np.uint16), expected.view(np.uint16)), (spmv.LAYOUT_NAMES[layout], tpr)
