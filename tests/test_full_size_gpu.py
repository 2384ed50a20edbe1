"""Parity on the benchmarked inputs at their full sizes: every product bit for bit against the CPU oracle's
reference-order CSR-i32 product at the same T (the reference's acceptance rule, max_abs_diff = 0 against
CSR-i32, src/bench_csr_width.cu:14-16, 1205-1210).

  * the random band, n = 1M (FP32): every admissible layout at T = 2, 4, 8, 16, 32;
  * the 27-point stencil on 160^3, RCM-permuted (FP64, 109 M nonzeros): CSR-i32 and CSR-lp at T = 8 and 32;
  * the power-law matrix, n = 8M (FP16, rows of up to 100,000 entries on the class schedule): CSR-i32 and
    CSR-lp at T = 32;
  * a 4M-row range of the block-FEM matrix of n = 32M (256 M nonzeros, FP32): CSR-i32 and CSR-lp at T = 8;
  * an operator whose row_ptr ends above 2^30 (the first 16.8M rows of the block-FEM matrix, 1.07 G
    nonzeros): CSR-i32 at T = 8, its last rows (entries above 2^30) checked against the oracle.
"""
import numpy as np
import pytest

import oracle
import spmvb200 as spmv

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TORCH = {spmv.F64: torch.float64, spmv.F32: torch.float32, spmv.F16: torch.float16}


def device_product(op, x_device, rows, dtype):
    y = torch.full((rows,), float("nan"), dtype=TORCH[dtype], device="cuda")
    op.run(x_device.data_ptr(), y.data_ptr())
    torch.cuda.synchronize()
    op.check()
    return y.cpu().numpy()


def reference_product(row_ptr, col_ind, values, x, dtype, tpr):
    return oracle.spmv_csr(row_ptr, col_ind, values, x, dtype, oracle.I32, tpr)


def assert_bits(got, want, label):
    got, want = np.ascontiguousarray(got), np.ascontiguousarray(want)
    assert got.shape == want.shape, label
    differ = got.view(np.uint8).reshape(got.size, -1) != want.view(np.uint8).reshape(want.size, -1)
    bad = np.flatnonzero(differ.any(axis=1))
    assert bad.size == 0, f"{label}: {bad.size} rows differ, first {bad[:5].tolist()}"


def check_matrix(matrix, dtype, layouts, tprs, seed):
    row_ptr, col_ind, values = matrix.arrays()
    x = spmv.fill_uniform(dtype, matrix.cols, seed)
    x_device = torch.from_numpy(x).cuda()
    facts = spmv.facts_of(matrix)
    checked = 0
    for tpr in tprs:
        want = reference_product(row_ptr, col_ind, values, x, dtype, tpr)
        for layout in layouts:
            if not spmv.configuration_admissible(matrix, facts, spmv.Configuration.of(layout, dtype, tpr)):
                continue
            with spmv.Operator(matrix, layout, dtype, tpr) as op:
                got = device_product(op, x_device, matrix.rows, dtype)
            assert_bits(got, want, f"{matrix.name} {spmv.LAYOUT_NAMES[layout]} T={tpr}")
            checked += 1
    return checked


def test_random_band_every_layout_and_t():
    matrix = spmv.synth_random_band(1_000_000, 2000, 32.0, 1)
    checked = check_matrix(matrix, spmv.F32, (spmv.I32, spmv.I16, spmv.R16, spmv.LP), spmv.THREADS_PER_ROW, 1)
    assert checked == 3 * len(spmv.THREADS_PER_ROW)   # i16 is not admissible at n = 1M


def test_stencil_rcm_i32_and_lp():
    matrix = spmv.synth_stencil27(160)
    matrix = spmv.apply_symmetric_permutation(matrix, spmv.reverse_cuthill_mckee(matrix))
    matrix.name = "stencil27_160_rcm"
    assert matrix.nnz == 109_215_352
    assert check_matrix(matrix, spmv.F64, (spmv.I32, spmv.LP), (8, 32), 2) == 4


def test_power_law_i32_and_lp_with_long_rows():
    matrix = spmv.synth_power_law(8_000_000, 1.8, 100_000, 12.0, 3)
    row_ptr, _, _ = matrix.arrays()
    assert int(np.diff(row_ptr).max()) > 40_000   # rows far longer than a tile or a class chunk
    with spmv.Operator(matrix, spmv.I32, spmv.F16, 32) as op:
        assert op.info().schedule == spmv.SCHEDULE_CLASSES
    assert check_matrix(matrix, spmv.F16, (spmv.I32, spmv.LP), (32,), 3) == 2


def test_block_fem_range_of_256m_nonzeros():
    first, last = 12_000_000, 16_000_000
    matrix = spmv.synth_block_fem(32_000_000, 8, 8, 50_000, 4, first, last)
    assert matrix.nnz == 64 * (last - first) >= 256_000_000
    assert check_matrix(matrix, spmv.F32, (spmv.I32, spmv.LP), (8,), 4) == 2


def test_row_pointer_above_2_to_the_30():
    rows = 16_800_000
    matrix = spmv.synth_block_fem(32_000_000, 8, 8, 50_000, 4, 0, rows)
    assert matrix.nnz > (1 << 30)
    row_ptr, col_ind, values = matrix.arrays(copy=False)   # views into the matrix (12.9 GB not copied)
    x = spmv.fill_uniform(spmv.F32, matrix.cols, 5)
    with spmv.Operator(matrix, spmv.I32, spmv.F32, 8) as op:
        got = device_product(op, torch.from_numpy(x).cuda(), matrix.rows, spmv.F32)
    # the rows whose entries lie above 2^30, and a block at the start
    tail = int(np.searchsorted(row_ptr, 1 << 30)) - 1
    for begin, end in ((0, 65_536), (tail, rows)):
        want = oracle.spmv(spmv.F32, oracle.I32, 8, row_ptr[begin:end + 1], oracle.convert_values(values, spmv.F32), x,
                           columns=col_ind)
        assert_bits(got[begin:end], want, f"rows [{begin}, {end})")
