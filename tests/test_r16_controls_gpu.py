"""The reference's control builds of CSR-r16 (bench_csr_width.cu:34-42, :343-432): lane-major offsets with
16-bit loads (LANE), the same stream two offsets to a 32-bit load (PAIR), 32-bit offsets (WIDE) and the
16-bit loop unrolled 16 times at FP16 (UNROLL16), each on the r16 operator's own row_ptr, row_base and values
through spmv_launch_r16_control, bit for bit against the oracle's CSR-i32 product at the same T."""
import numpy as np
import pytest

import oracle
import spmvb200 as spmv
from conftest import random_csr

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TORCH = {spmv.F64: torch.float64, spmv.F32: torch.float32, spmv.F16: torch.float16}


@pytest.mark.parametrize("dtype", (spmv.F64, spmv.F32, spmv.F16))
def test_every_control_matches_oracle(dtype):
    rows, cols = 2500, 3000
    row_ptr, col_ind, values = random_csr(rows, cols, lambda rng: rng.integers(0, 70), 23, empty_every=31,
                                          long_rows={4: 2000, 1000: 2900})
    matrix = spmv.CsrMatrix.from_arrays(rows, cols, row_ptr, col_ind, values)
    x = spmv.fill_uniform(dtype, cols, 5)
    x_device = torch.from_numpy(x).cuda()
    wide = torch.from_numpy(spmv.encode_relative(matrix, 4).view(np.int32)).cuda()
    for tpr in spmv.THREADS_PER_ROW:
        want = oracle.spmv_csr(row_ptr, col_ind, values, x, dtype, oracle.I32, tpr)
        lane = torch.from_numpy(spmv.encode_relative_lane(matrix, tpr).view(np.int16)).cuda()
        with spmv.Operator(matrix, spmv.R16, dtype, tpr) as op:
            arrays = op.arrays()
            for name, control in spmv.R16_CONTROLS.items():
                offsets = {"lane": lane, "pair": lane, "wide": wide}.get(name)
                y = torch.full((rows,), float("nan"), dtype=TORCH[dtype], device="cuda")
                device = spmv.DeviceMatrix(rows=rows, cols=cols, nnz=matrix.nnz, row_ptr=arrays.row_ptr,
                                           columns=offsets.data_ptr() if offsets is not None else arrays.columns,
                                           row_base=arrays.row_base, values=arrays.values, x=x_device.data_ptr(),
                                           y=y.data_ptr())
                spmv.launch_r16_control(control, dtype, tpr, device)
                torch.cuda.synchronize()
                got = y.cpu().numpy()
                assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), (name, tpr)


def test_unknown_control_is_refused():
    device = spmv.DeviceMatrix(rows=0, cols=0, nnz=0)
    with pytest.raises(spmv.SpmvError):
        spmv.launch_r16_control(9, spmv.F64, 8, device)
