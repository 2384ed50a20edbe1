"""The library's host side against the reference's own code (oracle/_ref) and the golden fixtures: the CSR
reader, RCM and its permutation file, characterization, the layout encoders and byte model, the synthetic
generators and the row sharding. No GPU is used."""
import csv
import io
import os

import numpy as np
import pytest

import oracle
import spmvb200 as spmv
from conftest import GOLDEN, random_csr


def csr_of(matrix):
    return matrix.arrays()


def assert_same_matrix(matrix, reference, handle):
    rows, cols, row_ptr, col_ind, values = reference.arrays(handle)
    mine = matrix.arrays()
    assert (matrix.rows, matrix.cols) == (rows, cols)
    assert np.array_equal(mine[0], row_ptr)
    assert np.array_equal(mine[1], col_ind)
    assert np.array_equal(mine[2].view(np.int64), values.view(np.int64))


def write_mtx(path, banner, size_line, entries, comments=("% a comment",), newline="\n"):
    with open(path, "w", newline="") as out:
        out.write(banner + newline)
        for line in comments:
            out.write(line + newline)
        out.write(size_line + newline)
        for entry in entries:
            out.write(" ".join(str(token) for token in entry) + newline)
    return str(path)


# ---- reader ------------------------------------------------------------------------------------------
def test_reader_matches_reference_on_smoke_matrices(smoke_matrix_paths, reference):
    for name, path in smoke_matrix_paths.items():
        matrix = spmv.read_matrix_market(path)
        handle = reference.read_matrix_market(path)
        assert_same_matrix(matrix, reference, handle)
        info = matrix.info()
        stats = reference.stats(handle)
        assert [info.nnz_per_row_mean, info.nnz_per_row_max, info.nnz_per_row_min, info.nnz_per_row_std,
                info.dynamic_range, info.norm_inf, info.max_abs, info.min_abs] == stats.tolist()
        assert matrix.name == name
        reference.free(handle)


MTX_CASES = {
    "symmetric": ("%%MatrixMarket matrix coordinate real symmetric", "5 5 6",
                  [(1, 1, 2.0), (2, 1, -1.5), (3, 2, 4.0), (5, 1, 1e-3), (4, 4, 7.0), (5, 3, -2.0)]),
    "skew": ("%%MatrixMarket matrix coordinate real skew-symmetric", "4 4 3",
             [(2, 1, 1.0), (3, 1, -2.0), (4, 3, 0.5)]),
    "pattern": ("%%MatrixMarket matrix coordinate pattern general", "3 6 4", [(1, 6), (2, 2), (3, 1), (3, 5)]),
    "integer_upper": ("%%MatrixMarket MATRIX Coordinate INTEGER General", "4 4 5",
                      [(1, 2, 3), (4, 4, -9), (2, 1, 5), (1, 1, 1), (3, 4, 2)]),
    "out_of_range": ("%%MatrixMarket matrix coordinate real general", "3 3 4",
                     [(1, 1, 1.0), (4, 1, 2.0), (2, 0, 3.0), (3, 3, 4.0)]),
    "duplicates": ("%%MatrixMarket matrix coordinate real general", "3 3 5",
                   [(1, 2, 1.0), (1, 2, 2.0), (1, 1, 3.0), (1, 2, 4.0), (3, 3, 5.0)]),
    "hermitian_as_symmetric": ("%%MatrixMarket matrix coordinate real hermitian", "3 3 2", [(2, 1, 1.0), (3, 3, 2.0)]),
    "short_file": ("%%MatrixMarket matrix coordinate real general", "4 4 10", [(1, 1, 1.0), (4, 2, 2.0)]),
    "empty_rows": ("%%MatrixMarket matrix coordinate real general", "6 6 2", [(6, 6, 1.0), (2, 3, -1.0)]),
}


@pytest.mark.parametrize("case", sorted(MTX_CASES))
@pytest.mark.parametrize("newline", ["\n", "\r\n"])
def test_reader_edge_cases_match_reference(tmp_path, reference, case, newline):
    banner, size_line, entries = MTX_CASES[case]
    path = write_mtx(tmp_path / f"{case}.mtx", banner, size_line, entries, newline=newline)
    matrix = spmv.read_matrix_market(path)
    handle = reference.read_matrix_market(path)
    assert_same_matrix(matrix, reference, handle)
    reference.free(handle)


def test_reader_symmetric_expansion_by_hand(tmp_path):
    path = write_mtx(tmp_path / "s.mtx", *MTX_CASES["skew"])
    matrix = spmv.read_matrix_market(path)
    row_ptr, col_ind, values = matrix.arrays()
    dense = np.zeros((4, 4))
    for row in range(4):
        for entry in range(row_ptr[row], row_ptr[row + 1]):
            dense[row, col_ind[entry]] = values[entry]
    assert np.array_equal(dense, -dense.T)
    assert matrix.info().symmetric_expanded == 1


@pytest.mark.parametrize("content,status", [
    ("", spmv.ERR_FORMAT),
    ("hello\n1 1 1\n1 1 1\n", spmv.ERR_FORMAT),
    ("%%MatrixMarket matrix array real general\n2 2\n1\n2\n3\n4\n", spmv.ERR_FORMAT),
    ("%%MatrixMarket matrix coordinate real general\n0 3 0\n", spmv.ERR_FORMAT),
])
def test_reader_errors(tmp_path, content, status):
    path = tmp_path / "bad.mtx"
    path.write_text(content)
    with pytest.raises(spmv.SpmvError) as failure:
        spmv.read_matrix_market(str(path))
    assert failure.value.status == status


def test_reader_missing_file():
    with pytest.raises(spmv.SpmvError) as failure:
        spmv.read_matrix_market("/nonexistent/matrix.mtx")
    assert failure.value.status == spmv.ERR_IO


def test_create_sorts_columns_and_validates():
    matrix = spmv.CsrMatrix.from_arrays(2, 5, [0, 3, 4], [4, 0, 2, 1], [1.0, 2.0, 3.0, 4.0])
    row_ptr, col_ind, values = matrix.arrays()
    assert col_ind.tolist() == [0, 2, 4, 1]
    assert values.tolist() == [2.0, 3.0, 1.0, 4.0]
    for bad in ([0, 3, 2], [1, 3, 4]):
        with pytest.raises(spmv.SpmvError):
            spmv.CsrMatrix.from_arrays(2, 5, bad, [4, 0, 2, 1])
    with pytest.raises(spmv.SpmvError):
        spmv.CsrMatrix.from_arrays(2, 3, [0, 3, 4], [4, 0, 2, 1])


# ---- RCM ------------------------------------------------------------------------------------------------
def test_rcm_matches_reference_on_smoke_matrices(smoke_matrix_paths, reference):
    for path in smoke_matrix_paths.values():
        matrix = spmv.read_matrix_market(path)
        handle = reference.read_matrix_market(path)
        order = spmv.reverse_cuthill_mckee(matrix)
        assert np.array_equal(order, reference.rcm_order(handle, matrix.rows))
        permuted = spmv.apply_symmetric_permutation(matrix, order)
        theirs = reference.permute(handle, order)
        assert_same_matrix(permuted, reference, theirs)
        reference.free(theirs)
        reference.free(handle)


@pytest.mark.parametrize("seed", range(6))
def test_rcm_matches_reference_on_random(reference, seed):
    n = 500 + 37 * seed
    # several components, unsymmetric patterns, isolated nodes, duplicate-degree ties
    row_ptr, col_ind, values = random_csr(n, n, 2 + seed % 3, seed, empty_every=17 if seed % 2 else 0)
    matrix = spmv.CsrMatrix.from_arrays(n, n, row_ptr, col_ind, values)
    handle = reference.from_arrays(n, n, row_ptr, col_ind, values)
    order = spmv.reverse_cuthill_mckee(matrix)
    assert np.array_equal(order, reference.rcm_order(handle, n))
    assert_same_matrix(spmv.apply_symmetric_permutation(matrix, order), reference, reference.permute(handle, order))
    reference.free(handle)


def test_rcm_matches_golden_order():
    data = np.load(os.path.join(GOLDEN, "reference_streams.npz"))
    row_ptr, col_ind = data["ragged300/row_ptr"], data["ragged300/col_ind"]
    matrix = spmv.CsrMatrix.from_arrays(300, 300, row_ptr, col_ind)
    assert np.array_equal(spmv.reverse_cuthill_mckee(matrix), data["ragged300/rcm"])


def test_rcm_rejects_rectangular():
    matrix = spmv.CsrMatrix.from_arrays(2, 3, [0, 1, 2], [0, 2])
    with pytest.raises(spmv.SpmvError):
        spmv.reverse_cuthill_mckee(matrix)


def test_permutation_file_round_trip_and_validation(tmp_path, reference):
    laplacian = spmv.synth_laplacian2d(20)
    row_ptr, col_ind, values = laplacian.arrays()
    path = write_mtx(tmp_path / "grid.mtx", "%%MatrixMarket matrix coordinate real general", f"400 400 {col_ind.size}",
                     [(r + 1, col_ind[e] + 1, values[e]) for r in range(400) for e in range(row_ptr[r], row_ptr[r + 1])])
    matrix = spmv.read_matrix_market(path)
    assert spmv.permutation_path_for(path) == str(tmp_path / "grid.rcm.perm")
    reordered, seconds = spmv.reorder_with_rcm(path, matrix)
    assert os.path.exists(tmp_path / "grid.rcm.perm") and not os.path.exists(tmp_path / "grid.rcm.perm.partial")
    raw = open(tmp_path / "grid.rcm.perm", "rb").read()
    assert raw[:8] == b"RCMPERM1" and int.from_bytes(raw[8:16], "little") == 400 and len(raw) == 24 + 4 * 400
    order, stored_seconds = spmv.read_permutation(str(tmp_path / "grid.rcm.perm"), 400)
    assert stored_seconds == seconds
    # the reference reads the same file and reorders identically
    handle = reference.read_matrix_market(path)
    theirs, their_seconds = reference.reorder_with_rcm(path, handle)
    assert their_seconds == seconds
    assert_same_matrix(reordered, reference, theirs)
    # a second call loads the cache instead of recomputing
    again, seconds_again = spmv.reorder_with_rcm(path, matrix)
    assert seconds_again == seconds
    # invalid files: wrong magic, wrong size, not a bijection
    bad = tmp_path / "bad.perm"
    for blob in (b"XXXXXXXX" + raw[8:], raw[:8] + (401).to_bytes(8, "little") + raw[16:],
                 raw[:24] + (0).to_bytes(4, "little") * 400, raw[:30]):
        bad.write_bytes(blob)
        with pytest.raises(spmv.SpmvError) as failure:
            spmv.read_permutation(str(bad), 400)
        assert failure.value.status == spmv.ERR_FORMAT
    assert spmv.read_permutation(str(tmp_path / "missing.perm"), 400) is None


# ---- characterization ---------------------------------------------------------------------------------
def characterization_fields(text):
    rows = list(csv.DictReader(io.StringIO(text)))
    assert len(rows) == 1
    row = rows[0]
    row.pop("ordering_seconds")
    return row


def test_characterization_matches_reference_tool(smoke_matrix_paths, tmp_path):
    if not os.path.exists(oracle.REFERENCE_CHARACTERIZE):
        pytest.skip("reference characterize_matrix not built")
    for name, path in smoke_matrix_paths.items():
        matrix = spmv.read_matrix_market(path)
        expected = characterization_fields(oracle.reference_characterize(path, "original"))
        assert characterization_fields(spmv.characterize(matrix, "original")) == expected
        local = tmp_path / os.path.basename(path)
        os.symlink(path, local)
        expected = characterization_fields(oracle.reference_characterize(str(local), "rcm"))
        reordered, seconds = spmv.reorder_with_rcm(str(local), matrix)
        assert characterization_fields(spmv.characterize(reordered, "rcm", seconds)) == expected


def test_characterization_matches_published_rows(smoke_matrix_paths, tmp_path):
    """matrices/characterization_rcm/{dawson5,rim}.csv: the 35 columns that file carries."""
    published = {row["name"]: row for row in csv.DictReader(open(os.path.join(GOLDEN, "characterization_rcm.csv")))}
    for name, path in smoke_matrix_paths.items():
        local = tmp_path / os.path.basename(path)
        os.symlink(path, local)
        reordered, seconds = spmv.reorder_with_rcm(str(local), spmv.read_matrix_market(path))
        mine = characterization_fields(spmv.characterize(reordered, "rcm", seconds))
        expected = dict(published[name])
        expected.pop("ordering_seconds")
        for key, value in expected.items():
            assert mine[key] == value, (name, key)


def test_characterization_on_synthetic_against_reference(tmp_path):
    if not os.path.exists(oracle.REFERENCE_CHARACTERIZE):
        pytest.skip("reference characterize_matrix not built")
    for seed in range(3):
        n = 3000
        row_ptr, col_ind, values = random_csr(n, n, 6 + 10 * seed, seed, empty_every=0 if seed else 9)
        path = write_mtx(tmp_path / f"r{seed}.mtx", "%%MatrixMarket matrix coordinate real general", f"{n} {n} {col_ind.size}",
                         [(r + 1, col_ind[e] + 1, repr(values[e])) for r in range(n) for e in range(row_ptr[r], row_ptr[r + 1])])
        matrix = spmv.read_matrix_market(path)
        assert characterization_fields(spmv.characterize(matrix)) == \
            characterization_fields(oracle.reference_characterize(path))


# ---- layouts: encoders, facts, admissibility, byte model -------------------------------------------------------
def test_encoders_match_oracle_and_golden():
    data = np.load(os.path.join(GOLDEN, "reference_streams.npz"))
    for name in ("ragged300", "wide64"):
        row_ptr, col_ind = data[f"{name}/row_ptr"], data[f"{name}/col_ind"]
        rows, cols = row_ptr.size - 1, int(data[f"{name}/cols"][0])
        matrix = spmv.CsrMatrix.from_arrays(rows, cols, row_ptr, col_ind)
        facts = spmv.facts_of(matrix)
        assert facts.widest_row_span == int(data[f"{name}/widest_row_span"][0])
        assert list(facts.lane_packed_words)[1:] == data[f"{name}/lane_packed_words"][1:].tolist()
        for tpr in (2, 4, 8, 16, 32):
            row_word, row_width, words = spmv.build_packed_deltas(matrix, tpr)
            assert np.array_equal(row_word, data[f"{name}/lp{tpr}/row_word"])
            assert np.array_equal(row_width, data[f"{name}/lp{tpr}/row_width"])
            assert np.array_equal(words, data[f"{name}/lp{tpr}/words"])
        assert np.array_equal(spmv.encode_row_base(matrix), oracle.row_bases(row_ptr, col_ind))
        for column_bytes in (2, 1):
            assert np.array_equal(spmv.encode_relative(matrix, column_bytes), oracle.relative_columns(row_ptr, col_ind, column_bytes))
            assert np.array_equal(spmv.encode_absolute(matrix, column_bytes), oracle.narrow_columns(col_ind, column_bytes))
        for layout, label in ((0, "i32"), (1, "i16"), (2, "r16"), (3, "lp"), (4, "i8"), (5, "r8")):
            for value_bytes in (8, 4, 2):
                configuration = spmv.Configuration.of(layout, {8: spmv.F64, 4: spmv.F32, 2: spmv.F16}[value_bytes], 4)
                memory = spmv.memory_of(matrix, facts, configuration)
                expected = data[f"{name}/memory/{label}/{value_bytes}"]
                assert [memory.values, memory.columns, memory.column_bases, memory.row_pointer, memory.vectors,
                        memory.total] == expected.tolist()
            configuration = spmv.Configuration.of(layout, spmv.F64, 4)
            assert spmv.configuration_admissible(matrix, facts, configuration) == bool(data[f"{name}/admissible/{label}"][0])


@pytest.mark.parametrize("seed", range(3))
def test_lane_packed_encoder_matches_reference_at_scale(reference, seed):
    rows, cols = 20000, 3_000_000
    row_ptr, col_ind, values = random_csr(rows, cols, 30, seed, empty_every=101, long_rows={3: 5000})
    matrix = spmv.CsrMatrix.from_arrays(rows, cols, row_ptr, col_ind, values)
    handle = reference.from_arrays(rows, cols, row_ptr, col_ind, values)
    for tpr in (2, 8, 32):
        mine = spmv.build_packed_deltas(matrix, tpr)
        theirs = reference.build_packed_deltas(handle, rows, tpr)
        for a, b in zip(mine, theirs):
            assert np.array_equal(a, b)
    reference.free(handle)


def test_published_bytes_through_library(smoke_matrix_paths, tmp_path):
    """memory_of of the library on the RCM-ordered smoke matrices equals the published bytes_total."""
    rows = list(csv.DictReader(open(os.path.join(GOLDEN, "published_bytes.csv"))))
    for name, path in smoke_matrix_paths.items():
        local = tmp_path / os.path.basename(path)
        os.symlink(path, local)
        matrix, _ = spmv.reorder_with_rcm(str(local), spmv.read_matrix_market(path))
        facts = spmv.facts_of(matrix)
        for row in rows:
            if row["matrix"] != name:
                continue
            configuration = spmv.Configuration({"fp64": 8, "fp32": 4, "fp16": 2}[row["prec"]], int(row["column_bytes"]),
                                               row["column_mode"], int(row["best_tpr"]) if row["column_mode"] == "lane-packed" else 0)
            assert spmv.memory_of(matrix, facts, configuration).total == float(row["bytes_total"])
            assert spmv.configuration_admissible(matrix, facts, configuration) == (row["status"] == "ok")


# ---- synthetic inputs ------------------------------------------------------------------------------------------
def test_laplacian_and_stencil_shapes():
    laplacian = spmv.synth_laplacian2d(256)
    assert (laplacian.rows, laplacian.nnz) == (65536, 326656)
    row_ptr, col_ind, values = laplacian.arrays()
    assert values[row_ptr[300]:row_ptr[301]].tolist() == [-1.0, -1.0, 4.0, -1.0, -1.0]
    stencil = spmv.synth_stencil27(10)
    assert (stencil.rows, stencil.nnz) == (1000, 28 ** 3)
    row_ptr, col_ind, values = stencil.arrays()
    assert np.all(np.diff(col_ind[row_ptr[555]:row_ptr[556]]) > 0)
    assert sorted(values[row_ptr[555]:row_ptr[556]].tolist()) == [-1.0] * 26 + [26.0]


def test_random_band_properties():
    band = spmv.synth_random_band(20000, 2000, 32.0, 1)
    row_ptr, col_ind, _ = band.arrays()
    rows = np.repeat(np.arange(20000), np.diff(row_ptr))
    assert np.all(np.abs(col_ind - rows) <= 2000)
    lengths = np.diff(row_ptr)
    assert abs(lengths.mean() - 33.0) < 0.3 and lengths.min() >= 2
    has_diagonal = np.zeros(20000, bool)
    has_diagonal[rows[col_ind == rows]] = True
    assert has_diagonal.all()
    again = spmv.synth_random_band(20000, 2000, 32.0, 1)
    assert all(np.array_equal(a, b) for a, b in zip(band.arrays(), again.arrays()))


def test_power_law_properties():
    matrix = spmv.synth_power_law(400000, 1.8, 100000, 12.0, 3)
    row_ptr, col_ind, values = matrix.arrays()
    lengths = np.diff(row_ptr)
    assert abs(lengths.mean() - 12.0) < 1.5
    assert lengths.min() >= 1 and lengths.max() > 1000
    assert np.all(np.abs(values) <= 1.0)
    for row in np.argsort(lengths)[-3:]:
        segment = col_ind[row_ptr[row]:row_ptr[row + 1]]
        assert np.all(np.diff(segment) > 0)


def test_block_fem_shards_equal_whole():
    n = 8 * 5000
    whole = spmv.synth_block_fem(n, 8, 8, 8000, 4)
    row_ptr, col_ind, values = whole.arrays()
    assert whole.nnz == 64 * n
    for begin, end in ((0, 8000), (12345, 20000), (39992, n)):
        shard = spmv.synth_block_fem(n, 8, 8, 8000, 4, begin, end)
        s_ptr, s_col, s_val = shard.arrays()
        assert np.array_equal(s_ptr, row_ptr[begin:end + 1] - row_ptr[begin])
        assert np.array_equal(s_col, col_ind[row_ptr[begin]:row_ptr[end]])
        assert np.array_equal(s_val, values[row_ptr[begin]:row_ptr[end]])
    # diagonal dominance
    rows = np.repeat(np.arange(n), 64)
    diagonal = values[col_ind == rows]
    off = np.abs(values).reshape(n, 64).sum(axis=1) - np.abs(diagonal)
    assert np.all(diagonal > off)


def test_fill_uniform_and_reference_x():
    x64 = spmv.fill_uniform(spmv.F64, 1000, 0)
    x16 = spmv.fill_uniform(spmv.F16, 1000, 0)
    assert np.all(np.abs(x64) <= 1.0) and np.array_equal(x16, x64.astype(np.float16))
    assert np.array_equal(x64, x64.astype(np.float32).astype(np.float64))
    ref = spmv.fill_reference_x(spmv.F32, 5)
    # std::mt19937(7) + uniform_real_distribution<double>(-1, 1), the reference's x (bench_csr_width.cu:923)
    import random
    assert ref.dtype == np.float32 and np.all(np.abs(ref) <= 1)


def test_shard_rows_balances_nonzeros():
    matrix = spmv.synth_random_band(100000, 2000, 32.0, 1)
    row_ptr = matrix.arrays()[0]
    for shards in (1, 2, 3, 8):
        bounds = spmv.shard_rows(matrix, shards)
        assert bounds[0] == 0 and bounds[-1] == matrix.rows and np.all(np.diff(bounds) >= 0)
        counts = np.diff(row_ptr[bounds])
        assert counts.max() - counts.min() <= 2 * np.diff(row_ptr).max()


def test_slice_rows_matches_arrays():
    matrix = spmv.synth_laplacian2d(30)
    row_ptr, col_ind, values = matrix.arrays()
    part = matrix.slice_rows(100, 700)
    p_ptr, p_col, p_val = part.arrays()
    assert part.cols == matrix.cols
    assert np.array_equal(p_ptr, row_ptr[100:701] - row_ptr[100])
    assert np.array_equal(p_col, col_ind[row_ptr[100]:row_ptr[700]])


def test_r16_control_encoders():
    """The control builds' offset streams (bench_csr_width.cu:838-855, :944): lane L's 16-bit offsets of a row
    come next to each other from position L * (length // T) + min(L, length % T) of the row's own positions,
    padded to whole 32-bit words; the WIDE offsets are the r16 offsets in 32 bits."""
    row_ptr, col_ind, values = random_csr(300, 5000, lambda rng: rng.integers(0, 70), 17, empty_every=9)
    matrix = spmv.CsrMatrix.from_arrays(300, 5000, row_ptr, col_ind, values)
    relative = spmv.encode_relative(matrix, 2)
    assert np.array_equal(spmv.encode_relative(matrix, 4), relative.astype(np.uint32))
    for tpr in spmv.THREADS_PER_ROW:
        want = np.zeros((col_ind.size + 1) // 2 * 2, np.uint16)
        for row in range(300):
            begin, end = int(row_ptr[row]), int(row_ptr[row + 1])
            length = end - begin
            quotient, remainder = divmod(length, tpr)
            for offset in range(length):
                lane, k = offset % tpr, offset // tpr
                want[begin + lane * quotient + min(lane, remainder) + k] = relative[begin + offset]
        assert np.array_equal(spmv.encode_relative_lane(matrix, tpr), want), tpr
