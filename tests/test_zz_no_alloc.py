"""The allocation-free CSR-lp encoder (spmv_encode_lane_packed_device_noalloc), for callers that must not
allocate device memory while they encode, against the allocating GPU encoder
(spmv_encode_lane_packed_device) through the C ABI: two different matrices encoded in a row (so that
anything the first call leaves in the shared scratch array would show in the second), then the first again;
every row word, width and stream word must be the same bits. Kept in a file of its own, collected last."""
import numpy as np
import pytest

import spmvb200 as spmv
from conftest import random_csr

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def encode(build, matrix, tpr):
    row_ptr, col_ind, _ = matrix.arrays()
    device_row_ptr = torch.from_numpy(row_ptr.astype(np.int32)).cuda()
    device_col = torch.from_numpy(col_ind.astype(np.int32) if col_ind.size else np.zeros(1, np.int32)).cuda()
    row_word = torch.full((max(matrix.rows, 1),), -7, dtype=torch.int32, device="cuda")
    row_width = torch.full((max(matrix.rows, 1),), 99, dtype=torch.uint8, device="cuda")
    count = build(device_row_ptr.data_ptr(), device_col.data_ptr(), matrix.rows, tpr, row_word.data_ptr(),
                  row_width.data_ptr())
    words = torch.full((count,), -1, dtype=torch.int32, device="cuda")
    assert build(device_row_ptr.data_ptr(), device_col.data_ptr(), matrix.rows, tpr, row_word.data_ptr(),
                 row_width.data_ptr(), words.data_ptr(), count) == count
    torch.cuda.synchronize()
    return row_word.cpu().numpy()[:matrix.rows], row_width.cpu().numpy()[:matrix.rows], words.cpu().numpy()


def test_two_calls_in_a_row_match_the_allocating_encoder():
    first = spmv.CsrMatrix.from_arrays(3000, 4000, *random_csr(3000, 4000, lambda rng: rng.integers(0, 80), 31,
                                                               empty_every=17, long_rows={5: 3000}))
    second = spmv.CsrMatrix.from_arrays(70000, 9000, *random_csr(70000, 9000, 6.0, 32, empty_every=101))
    for tpr in (2, 8, 32):
        for matrix in (first, second, first):
            mine = encode(spmv.build_packed_deltas_device_noalloc, matrix, tpr)
            theirs = encode(spmv.build_packed_deltas_device, matrix, tpr)
            for a, b in zip(mine, theirs):
                assert np.array_equal(a, b), (tpr, matrix.rows)


def test_edge_matrices_match_the_allocating_encoder():
    """Deltas of 31 bits, a matrix with no rows, and 1.1 M short rows: 1075 scan blocks, so the sums of the
    blocks are scanned across more than one chunk of 1024."""
    wide = spmv.CsrMatrix.from_arrays(3, (1 << 31) - 1, [0, 3, 3, 5], [0, 1 << 30, (1 << 31) - 2, 5, 7])
    empty = spmv.CsrMatrix.from_arrays(0, 10, [0], [], [])
    many = spmv.synth_random_band(1_100_000, 40, 3.0, 9)
    for tpr in (2, 32):
        for matrix in (wide, empty, many, wide):
            mine = encode(spmv.build_packed_deltas_device_noalloc, matrix, tpr)
            theirs = encode(spmv.build_packed_deltas_device, matrix, tpr)
            for a, b in zip(mine, theirs):
                assert np.array_equal(a, b), (tpr, matrix.rows)


def test_rows_beyond_the_fixed_scratch_are_refused():
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    with pytest.raises(spmv.SpmvError) as failure:
        spmv.build_packed_deltas_device_noalloc(dummy.data_ptr(), dummy.data_ptr(), (1 << 26) + 1, 8,
                                                dummy.data_ptr(), dummy.data_ptr())
    assert failure.value.status == spmv.ERR_TOO_LARGE
