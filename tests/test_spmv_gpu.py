"""GPU parity: the library's sm_100a kernels against the CPU oracle (bit for bit), against the reference's own
kernels rebuilt for sm_100a (bit for bit), and against cuSPARSE (within the north-star tolerance). Every
product goes through the C ABI (spmv_operator_run / spmv_launch)."""
import numpy as np
import pytest

import oracle
import spmvb200 as spmv
from conftest import random_csr

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

LAYOUTS = (spmv.I32, spmv.I16, spmv.R16, spmv.LP, spmv.I8, spmv.R8)
DTYPES = (spmv.F64, spmv.F32, spmv.F16)
TORCH = {spmv.F64: torch.float64, spmv.F32: torch.float32, spmv.F16: torch.float16}


def bits(array):
    return np.ascontiguousarray(array).view(np.uint8)


def device_run(op, x, stream=0):
    x_device = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    y_device = torch.full((op.rows,), float("nan"), dtype=TORCH[op.dtype], device="cuda")
    op.run(x_device.data_ptr(), y_device.data_ptr(), stream)
    torch.cuda.synchronize()
    op.check()
    return y_device.cpu().numpy()


def oracle_product(matrix, x, dtype, layout, tpr):
    row_ptr, col_ind, values = matrix.arrays()
    return oracle.spmv_csr(row_ptr, col_ind, values, x, dtype, layout, tpr)


def admissible(matrix, layout, tpr):
    return spmv.configuration_admissible(matrix, None, spmv.Configuration.of(layout, spmv.F64, tpr))


def physical_variants(tpr):
    return [tpr // slots for slots in (1, 2, 4, 8, 16) if tpr // slots >= 1 and tpr % slots == 0]


@pytest.fixture(scope="module")
def ragged():
    """Ragged rows: empty rows, rows of 0..59 entries and three rows of 2049..2500 entries."""
    rows, cols = 3000, 2500
    row_ptr, col_ind, values = random_csr(rows, cols, lambda rng: rng.integers(0, 60), 7, empty_every=23,
                                          long_rows={11: 2400, 1500: 2049, 2999: 2500})
    return spmv.CsrMatrix.from_arrays(rows, cols, row_ptr, col_ind, values, name="ragged")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("tpr", spmv.THREADS_PER_ROW)
def test_operator_matches_oracle_every_layout(ragged, dtype, tpr):
    x = spmv.fill_uniform(dtype, ragged.cols, 11)
    for layout in (spmv.I32, spmv.I16, spmv.R16, spmv.LP):
        if not admissible(ragged, layout, tpr):
            continue
        expected = oracle_product(ragged, x, dtype, layout, tpr)
        # 2048-nonzero tiles leave the three rows of 2049..2500 entries to the long-row path
        with spmv.Operator(ragged, layout, dtype, tpr, tile_nnz=2048) as op:
            assert op.info().long_rows == 3
            y = device_run(op, x)
        assert np.array_equal(bits(y), bits(expected)), (spmv.LAYOUT_NAMES[layout], tpr)
        with spmv.Operator(ragged, layout, dtype, tpr) as op:   # the library's own tile plan
            y = device_run(op, x)
        assert np.array_equal(bits(y), bits(expected)), (spmv.LAYOUT_NAMES[layout], tpr)


@pytest.mark.parametrize("tpr", spmv.THREADS_PER_ROW)
def test_every_physical_mapping_and_tile_size(ragged, tpr):
    """The result must not depend on how many threads run a row nor on the tile size."""
    dtype = spmv.F32
    x = spmv.fill_uniform(dtype, ragged.cols, 5)
    for layout in (spmv.I32, spmv.R16, spmv.LP):
        expected = oracle_product(ragged, x, dtype, layout, tpr)
        for physical in physical_variants(tpr):
            for tile_nnz in (64, 700, 2048, 8192):
                with spmv.Operator(ragged, layout, dtype, tpr, physical_tpr=physical, tile_nnz=tile_nnz) as op:
                    y = device_run(op, x)
                assert np.array_equal(bits(y), bits(expected)), (spmv.LAYOUT_NAMES[layout], tpr, physical, tile_nnz)


@pytest.mark.parametrize("dtype", DTYPES)
def test_narrow_8bit_layouts(dtype):
    rows, cols = 700, 256
    row_ptr, col_ind, values = random_csr(rows, cols, 20, 3, empty_every=9, long_rows={4: 256})
    matrix = spmv.CsrMatrix.from_arrays(rows, cols, row_ptr, col_ind, values)
    x = spmv.fill_uniform(dtype, cols, 2)
    for tpr in spmv.THREADS_PER_ROW:
        for layout in (spmv.I8, spmv.R8):
            assert admissible(matrix, layout, tpr)
            with spmv.Operator(matrix, layout, dtype, tpr, tile_nnz=128) as op:
                y = device_run(op, x)
            assert np.array_equal(bits(y), bits(oracle_product(matrix, x, dtype, spmv.I32, tpr)))


def test_inadmissible_layouts_are_refused():
    matrix = spmv.synth_random_band(70000, 2000, 8.0, 1)      # n > 2^16: i16 not admissible
    with pytest.raises(spmv.SpmvError) as failure:
        spmv.Operator(matrix, spmv.I16, spmv.F32, 8)
    assert failure.value.status == spmv.ERR_NOT_ADMISSIBLE
    wide = spmv.CsrMatrix.from_arrays(2, 100000, [0, 2, 3], [0, 99999, 5])
    with pytest.raises(spmv.SpmvError) as failure:
        spmv.Operator(wide, spmv.R16, spmv.F32, 8)
    assert failure.value.status == spmv.ERR_NOT_ADMISSIBLE


@pytest.mark.parametrize("dtype", DTYPES)
def test_degenerate_matrices(dtype):
    cases = [
        spmv.CsrMatrix.from_arrays(5, 7, [0, 0, 0, 0, 0, 0], []),                       # no nonzeros
        spmv.CsrMatrix.from_arrays(1, 1, [0, 1], [0], [2.5]),                           # 1 x 1
        spmv.CsrMatrix.from_arrays(3, 40000, [0, 0, 40000, 40000], np.arange(40000)),    # one row wider than tiles
        spmv.CsrMatrix.from_arrays(4, 3, [0, 1, 2, 3, 3], [2, 1, 0], [-0.0, 1.0, -1.0]),  # -0 product, rectangular
    ]
    for matrix in cases:
        x = spmv.fill_uniform(dtype, matrix.cols, 9)
        for tpr in (2, 32):
            for layout in (spmv.I32, spmv.LP):
                with spmv.Operator(matrix, layout, dtype, tpr) as op:
                    y = device_run(op, x)
                assert np.array_equal(bits(y), bits(oracle_product(matrix, x, dtype, layout, tpr)))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("tpr", spmv.THREADS_PER_ROW)
def test_raw_launch_matches_oracle(ragged, dtype, tpr):
    """spmv_launch over caller-owned device arrays (the launch<T> shape, no preprocessing)."""
    row_ptr, col_ind, values = ragged.arrays()
    x = spmv.fill_uniform(dtype, ragged.cols, 4)
    typed = oracle.convert_values(values, dtype)
    for layout in (spmv.I32, spmv.I16, spmv.R16, spmv.LP):
        if not admissible(ragged, layout, tpr):
            continue
        streams = oracle.encode(row_ptr, col_ind, layout, tpr)
        dev = {key: torch.from_numpy(np.ascontiguousarray(value)).cuda() for key, value in streams.items()}
        d_row_ptr = torch.from_numpy(row_ptr).cuda()
        d_values = torch.from_numpy(typed).cuda()
        d_x = torch.from_numpy(x).cuda()
        d_y = torch.zeros(ragged.rows, dtype=TORCH[dtype], device="cuda")
        matrix = spmv.DeviceMatrix(ragged.rows, ragged.cols, col_ind.size, d_row_ptr.data_ptr(),
                                   dev["columns"].data_ptr() if "columns" in dev else None,
                                   dev["row_base"].data_ptr() if "row_base" in dev else None,
                                   dev["row_word"].data_ptr() if "row_word" in dev else None,
                                   dev["row_width"].data_ptr() if "row_width" in dev else None,
                                   dev["words"].data_ptr() if "words" in dev else None,
                                   d_values.data_ptr(), d_x.data_ptr(), d_y.data_ptr())
        spmv.launch(layout, dtype, tpr, matrix)
        torch.cuda.synchronize()
        expected = oracle.spmv(dtype, layout, tpr, row_ptr, typed, x, **streams)
        assert np.array_equal(bits(d_y.cpu().numpy()), bits(expected))


@pytest.mark.parametrize("dtype", DTYPES)
def test_reference_kernels_agree_bit_for_bit(ragged, reference, dtype):
    """The reference's kernels (launch<T>, bench_csr_width.cu:607) rebuilt for sm_100a on the operator's own
    device arrays give the same bits as the library and as the oracle."""
    x = spmv.fill_uniform(dtype, ragged.cols, 21)
    d_x = torch.from_numpy(x).cuda()
    for tpr in spmv.THREADS_PER_ROW:
        for layout in (spmv.I32, spmv.I16, spmv.R16, spmv.LP):
            if not admissible(ragged, layout, tpr):
                continue
            with spmv.Operator(ragged, layout, dtype, tpr) as op:
                arrays = op.arrays()
                d_y = torch.zeros(ragged.rows, dtype=TORCH[dtype], device="cuda")
                status = reference.launch(dtype, layout, tpr, ragged.rows, ragged.cols, ragged.nnz, arrays.row_ptr,
                                          arrays.columns, arrays.row_base, arrays.row_word, arrays.row_width,
                                          arrays.words, arrays.values, d_x.data_ptr(), d_y.data_ptr())
                assert status == 0
                theirs = d_y.cpu().numpy()
                mine = device_run(op, x)
            assert np.array_equal(bits(mine), bits(theirs)), (spmv.LAYOUT_NAMES[layout], tpr)
            assert np.array_equal(bits(mine), bits(oracle_product(ragged, x, dtype, layout, tpr)))


def l2_relative(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300)


# tolerances of the cuSPARSE comparison (relative, L2 norm): FP64 1e-12, FP32 1e-5, FP16 1e-2
CUSPARSE_TOLERANCE = {spmv.F64: 1e-12, spmv.F32: 1e-5, spmv.F16: 1e-2}


@pytest.mark.parametrize("dtype", DTYPES)
def test_cusparse_agrees_within_tolerance(ragged, dtype):
    """torch's CSR product (cuSPARSE) on the same values; FP16 computed in FP32 as the reference does (:1066)."""
    row_ptr, col_ind, values = ragged.arrays()
    x = spmv.fill_uniform(dtype, ragged.cols, 8)
    compute = torch.float32 if dtype == spmv.F16 else TORCH[dtype]
    typed = torch.from_numpy(oracle.convert_values(values, dtype)).to(compute)
    a = torch.sparse_csr_tensor(torch.from_numpy(row_ptr.astype(np.int64)), torch.from_numpy(col_ind.astype(np.int64)),
                                typed, size=(ragged.rows, ragged.cols)).cuda()
    reference_y = (a @ torch.from_numpy(x).to(compute).cuda().unsqueeze(1)).squeeze(1).cpu().numpy()
    with spmv.Operator(ragged, spmv.LP, dtype, 8) as op:
        y = device_run(op, x)
    assert l2_relative(y, reference_y) <= CUSPARSE_TOLERANCE[dtype]


def test_misaligned_vectors_are_refused(ragged):
    with spmv.Operator(ragged, spmv.I32, spmv.F64, 8) as op:
        x = torch.zeros(ragged.cols + 1, dtype=torch.float64, device="cuda")
        y = torch.zeros(ragged.rows + 1, dtype=torch.float64, device="cuda")
        with pytest.raises(spmv.SpmvError) as failure:
            op.run(x.data_ptr() + 4, y.data_ptr())
        assert failure.value.status == spmv.ERR_INVALID_ARGUMENT
    with spmv.Operator(ragged, spmv.I32, spmv.F16, 8) as op:
        x = torch.zeros(ragged.cols + 1, dtype=torch.float16, device="cuda")
        y = torch.zeros(ragged.rows, dtype=torch.float16, device="cuda")
        with pytest.raises(spmv.SpmvError):
            op.run(x.data_ptr() + 2, y.data_ptr())


def test_streams_and_repeated_runs(ragged):
    """Products on a side stream, repeated, with the same bits every time."""
    x = spmv.fill_uniform(spmv.F64, ragged.cols, 1)
    stream = torch.cuda.Stream()
    with spmv.Operator(ragged, spmv.R16, spmv.F64, 16) as op:
        first = device_run(op, x, stream.cuda_stream)
        for _ in range(3):
            assert np.array_equal(bits(device_run(op, x, stream.cuda_stream)), bits(first))


def test_run_host_round_trip(ragged):
    x = spmv.fill_uniform(spmv.F32, ragged.cols, 3)
    with spmv.Operator(ragged, spmv.I32, spmv.F32, 4) as op:
        y = np.zeros(ragged.rows, np.float32)
        x_device = torch.empty(ragged.cols, dtype=torch.float32, device="cuda")
        y_device = torch.empty(ragged.rows, dtype=torch.float32, device="cuda")
        op.run_host(x, y, x_device.data_ptr(), y_device.data_ptr())
    assert np.array_equal(bits(y), bits(oracle_product(ragged, x, spmv.F32, spmv.I32, 4)))


def test_laplacian_config_bit_identical():
    """The 5-point Laplacian on 256 x 256, FP64, x uniform from seed 0, CSR-i32/i16/r16 at T = 4: every
    layout bit-identical to the CPU CSR-i32 product."""
    matrix = spmv.synth_laplacian2d(256)
    x = spmv.fill_uniform(spmv.F64, matrix.cols, 0)
    expected = oracle_product(matrix, x, spmv.F64, spmv.I32, 4)
    for layout in (spmv.I32, spmv.I16, spmv.R16):
        with spmv.Operator(matrix, layout, spmv.F64, 4) as op:
            assert np.array_equal(bits(device_run(op, x)), bits(expected))


def test_read_bandwidth_is_a_device_memory_rate():
    """The read roof behind epsilon: a streaming read of 1 GiB (past the 126 MB L2), between 1 TB/s and the
    nominal 8 TB/s of HBM3e on this device."""
    rate = spmv.read_bandwidth(1 << 30, 5)
    assert 1000.0 < rate < 8200.0
    with pytest.raises(spmv.SpmvError):
        spmv.read_bandwidth(0, 5)


def test_gather_rate_is_below_the_sector_rate():
    """The random-gather ceiling: single 2-, 4- and 8-byte elements at random positions of a 16 MB array;
    each costs a 32-byte L2 sector, so the rate times 32 bytes stays under 40 TB/s and above 1 TB/s."""
    for value_bytes in (2, 4, 8):
        rate = spmv.gather_rate((16 << 20) // value_bytes, value_bytes, 3)
        assert 1e12 / 32 < rate < 40e12 / 32, (value_bytes, rate)
    with pytest.raises(spmv.SpmvError):
        spmv.gather_rate(1 << 20, 3, 3)


@pytest.mark.parametrize("tpr", spmv.THREADS_PER_ROW)
def test_device_lane_packed_encoder_matches_host(ragged, tpr):
    """The GPU CSR-lp encoder gives the host encoder's row words, widths and words (empty rows, rows of
    2000+ entries, 12-bit and 31-bit deltas, a matrix with no rows)."""
    wide = spmv.CsrMatrix.from_arrays(3, (1 << 31) - 1, [0, 3, 3, 5], [0, 1 << 30, (1 << 31) - 2, 5, 7])
    empty = spmv.CsrMatrix.from_arrays(0, 10, [0], [], [])
    for matrix in (ragged, wide, empty):
        row_ptr, col_ind, _ = matrix.arrays()
        host_word, host_width, host_words = spmv.build_packed_deltas(matrix, tpr)
        device_row_ptr = torch.from_numpy(row_ptr.astype(np.int32)).cuda()
        device_col = torch.from_numpy(col_ind.astype(np.int32) if col_ind.size else np.zeros(1, np.int32)).cuda()
        row_word = torch.zeros(max(matrix.rows, 1), dtype=torch.int32, device="cuda")
        row_width = torch.zeros(max(matrix.rows, 1), dtype=torch.uint8, device="cuda")
        count = spmv.build_packed_deltas_device(device_row_ptr.data_ptr(), device_col.data_ptr(), matrix.rows, tpr,
                                                row_word.data_ptr(), row_width.data_ptr())
        assert count == host_words.size
        words = torch.full((count,), -1, dtype=torch.int32, device="cuda")
        spmv.build_packed_deltas_device(device_row_ptr.data_ptr(), device_col.data_ptr(), matrix.rows, tpr,
                                        row_word.data_ptr(), row_width.data_ptr(), words.data_ptr(), count)
        assert np.array_equal(row_word.cpu().numpy()[:matrix.rows], host_word)
        assert np.array_equal(row_width.cpu().numpy()[:matrix.rows], host_width)
        assert np.array_equal(words.cpu().numpy().view(np.uint32), host_words)


def test_large_lp_operator_encodes_on_the_device():
    """An operator over more than 2^20 nonzeros encodes CSR-lp on the GPU; its products stay bit-identical
    to the oracle's."""
    matrix = spmv.synth_random_band(60000, 3000, 24.0, 5)
    assert matrix.nnz > (1 << 20)
    for tpr in (8, 32):
        x = spmv.fill_uniform(spmv.F32, matrix.cols, 3)
        with spmv.Operator(matrix, spmv.LP, spmv.F32, tpr) as op:
            y = device_run(op, x)
        assert np.array_equal(bits(y), bits(oracle_product(matrix, x, spmv.F32, spmv.LP, tpr))), tpr


@pytest.mark.parametrize("dtype", DTYPES)
def test_x_windows_of_banded_tiles(dtype):
    """A banded matrix: its tiles stage their window of x and gather from shared memory; every layout stays
    bit-identical to the oracle, with x 16-byte aligned (windows on) and x offset by one element (windows off
    for that launch)."""
    matrix = spmv.synth_random_band(30000, 700, 20.0, 8)
    x = spmv.fill_uniform(dtype, matrix.cols + 8, 4)
    for layout, tpr in ((spmv.I32, 8), (spmv.R16, 32), (spmv.I16, 4), (spmv.I32, 2)):
        with spmv.Operator(matrix, layout, dtype, tpr) as op:
            assert op.info().window_elements > 0
            x_device = torch.from_numpy(x).cuda()
            for shift in (0, 2 if dtype == spmv.F16 else 1):
                y_device = torch.full((op.rows,), float("nan"), dtype=TORCH[dtype], device="cuda")
                op.run(x_device[shift:].data_ptr(), y_device.data_ptr(), 0)
                torch.cuda.synchronize()
                op.check()
                expected = oracle_product(matrix, x[shift:shift + matrix.cols], dtype, layout, tpr)
                assert np.array_equal(bits(y_device.cpu().numpy()), bits(expected)), (spmv.LAYOUT_NAMES[layout], tpr, shift)


def test_run_host_batch_pipelines_a_stream_of_vectors(ragged):
    """Five different x vectors through host buffers with overlapped copies: every y as run() gives it."""
    dtype = spmv.F64
    count = 5
    xs = np.stack([spmv.fill_uniform(dtype, ragged.cols, 20 + i) for i in range(count)])
    ys = np.full((count, ragged.rows), np.nan)
    x_pinned = torch.from_numpy(xs).pin_memory()
    y_pinned = torch.from_numpy(ys).pin_memory()
    pitch = lambda n: (n * 8 + 15) // 16 * 16 // 8  # noqa: E731
    x_device = torch.empty(2 * pitch(ragged.cols), dtype=torch.float64, device="cuda")
    y_device = torch.empty(2 * pitch(ragged.rows), dtype=torch.float64, device="cuda")
    with spmv.Operator(ragged, spmv.LP, dtype, 8) as op:
        op.run_host_batch(x_pinned.data_ptr(), ragged.cols * 8, y_pinned.data_ptr(), ragged.rows * 8, count,
                          x_device.data_ptr(), y_device.data_ptr())
        for i in range(count):
            assert np.array_equal(bits(y_pinned[i].numpy()), bits(device_run(op, xs[i]))), i


@pytest.mark.parametrize("dtype", DTYPES)
def test_dense_variants_one_thread_per_lane(dtype):
    """One thread per lane (P = T) on gathers in runs: the dense tile variants (4 CTAs a multiprocessor, 3
    for FP64, 8 gathers at once) at every T, bit-identical to the oracle, with more persistent CTAs than
    the 2 a multiprocessor of the other variants."""
    matrix = spmv.synth_block_fem(60000, 8, 8, 2000, 4, 0, 60000)   # i16: at most 65536 columns
    x = spmv.fill_uniform(dtype, matrix.cols, 8)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for layout in (spmv.I32, spmv.I16, spmv.R16, spmv.LP):
        for tpr in spmv.THREADS_PER_ROW:
            with spmv.Operator(matrix, layout, dtype, tpr, physical_tpr=tpr) as op:
                info = op.info()
                assert info.tile_ctas == min(info.tiles, (3 if dtype == spmv.F64 else 4) * sms), (layout, tpr)
                y = device_run(op, x)
            assert np.array_equal(bits(y), bits(oracle_product(matrix, x, dtype, layout, tpr))), \
                (spmv.LAYOUT_NAMES[layout], tpr)


@pytest.mark.parametrize("dtype", DTYPES)
def test_block_rows_of_column_runs(dtype):
    """8x8-block rows (64 nonzeros in runs of 8 columns): one thread per lane up to T = 16, else 8 threads a
    row (not CSR-lp), at least two passes a tile; every layout bit-identical to the oracle."""
    matrix = spmv.synth_block_fem(20000, 8, 8, 2000, 4, 0, 20000)
    x = spmv.fill_uniform(dtype, matrix.cols, 6)
    for layout, tpr in ((spmv.I32, 8), (spmv.R16, 16), (spmv.I16, 32), (spmv.LP, 8), (spmv.LP, 16), (spmv.LP, 32)):
        with spmv.Operator(matrix, layout, dtype, tpr) as op:
            if tpr <= 16:
                assert op.info().physical_tpr == tpr and op.info().tile_rows == 64
            elif layout != spmv.LP:
                assert op.info().physical_tpr == 8 and op.info().tile_rows == 64
            y = device_run(op, x)
        assert np.array_equal(bits(y), bits(oracle_product(matrix, x, dtype, layout, tpr))), (spmv.LAYOUT_NAMES[layout], tpr)


@pytest.mark.parametrize("dtype", DTYPES)
def test_long_rows_on_the_class_schedule_at_segment_and_chunk_edges(dtype):
    """Rows above 64*T entries run one CTA each; for CSR-lp every gatherer decodes 16 deltas of one lane from
    that lane's column mark. Lengths just around 16*T*k and around the class chunk (1024, 2048 or 3584 entries)
    leave lanes with fewer deltas than a segment, segments cut by the row's end and rows over several chunks;
    every layout must give the oracle's CSR-i32 bits."""
    for tpr in spmv.THREADS_PER_ROW:
        chunk = {spmv.F64: 1024, spmv.F32: 2048, spmv.F16: 3584}[dtype]
        lengths = [64 * tpr + 1, 16 * tpr * 5 - 1, 16 * tpr * 5 + 1, chunk - 1, chunk + 1, 3 * chunk + 16 * tpr - 3,
                   7 * tpr + 64 * tpr + 5]
        rows, cols = 400, 12000
        long_rows = {5 + 37 * i: n for i, n in enumerate(lengths)}
        row_ptr, col_ind, values = random_csr(rows, cols, lambda rng: rng.integers(0, 12), 41 + tpr, empty_every=13,
                                              long_rows=long_rows)
        matrix = spmv.CsrMatrix.from_arrays(rows, cols, row_ptr, col_ind, values, name="long-edges")
        x = spmv.fill_uniform(dtype, cols, 3)
        expected = oracle_product(matrix, x, dtype, spmv.I32, tpr)
        for layout in (spmv.I32, spmv.LP):
            with spmv.Operator(matrix, layout, dtype, tpr, schedule=spmv.SCHEDULE_CLASSES) as op:
                assert op.info().long_rows == sum(n > 64 * tpr for n in lengths), (tpr, op.info().long_rows)
                y = device_run(op, x)
                op.check()
            assert np.array_equal(bits(y), bits(expected)), (spmv.LAYOUT_NAMES[layout], tpr)
