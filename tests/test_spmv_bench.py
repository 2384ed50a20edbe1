"""The benchmark program (spmv_bench): the reference's command line and CSV files, on the library.

The reference program is src/bench_csr_width.cu; its result rows (ResultRow, :99-125) and its
per-threads-per-row rows (append_thread_samples, :990-1005) are what analysis/compare_campaign.py reads.
The GPU test runs the program on the RCM-ordered smoke matrices and checks the rows the reference
checks: every layout bit-identical to CSR-i32 at the same T (max_abs_diff 0), byte counts equal to the
published ones, cuSPARSE within floating-point tolerance of CSR-i32.
"""
import csv
import os
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
BINARY = os.path.join(ROOT, "spmv-index-compression_b200", "spmvb200", "spmv_bench")
GOLDEN = os.path.join(HERE, "golden")

HEADER = ("matrix,prec,row_encoding,value_bytes,column_bytes,length_bytes,status,rows,cols,nnz,"
          "bytes_values,bytes_columns,bytes_row_pointer,bytes_vectors,bytes_total,bytes_per_nnz,"
          "best_tpr,t_ms,gflops,bw_gbs,epsilon,speedup_meas,speedup_pred,max_abs_diff,column_mode,bytes_column_bases,"
          "kernel,bytes_workspace,max_rel_diff,ordering,batch")
TPR_HEADER = "matrix,ordering,prec,layout,tpr,t_ms,batch,bytes_total,nnz,max_abs_diff"
LABELS = {("absolute", "4"): "i32", ("absolute", "2"): "i16", ("absolute", "1"): "i8",
          ("row-base", "2"): "r16", ("row-base", "1"): "r8", ("lane-packed", "0"): "lp"}
# cuSPARSE sums in its own order: max |dy| / max |y| against CSR-i32 at T = 8
CUSPARSE_TOLERANCE = {"fp64": 1e-12, "fp32": 1e-5, "fp16": 1e-2}


def built():
    if not os.path.exists(BINARY):
        pytest.skip("spmv_bench is not built (make -C spmv-index-compression_b200)")
    return BINARY


def test_help_and_argument_errors():
    """--help prints the reference's usage line and exits 0; bad options exit 1 (no GPU is touched)."""
    binary = built()
    done = subprocess.run([binary, "--help"], capture_output=True, text=True, timeout=60)
    assert done.returncode == 0 and done.stdout.startswith("usage: spmv_bench --matrix A.mtx")
    for arguments in (["--bogus", "1"], [], ["--matrix", "a.mtx", "--ordering", "amd"],
                      ["--matrix", "a.mtx", "--precision", "bf16"], ["--matrix", "a.mtx", "--accumulate", "fp8"]):
        assert subprocess.run([binary] + arguments, capture_output=True, timeout=60).returncode == 1


@pytest.mark.gpu
def test_campaign_rows_on_smoke_matrices(smoke_matrix_paths, tmp_path):
    binary = built()
    results, per_tpr = tmp_path / "results.csv", tmp_path / "tpr.csv"
    matrices = []
    for name, path in smoke_matrix_paths.items():
        local = tmp_path / os.path.basename(path)
        os.symlink(path, local)
        matrices += ["--matrix", str(local)]
    done = subprocess.run([binary] + matrices + ["--ordering", "rcm", "--reps", "3", "--warmup", "1",
                                                 "--csv", str(results), "--tpr-csv", str(per_tpr)],
                          capture_output=True, text=True, timeout=900)
    assert done.returncode == 0, done.stdout[-2000:] + done.stderr[-2000:]
    lines = open(results).read().splitlines()
    assert lines[0] == HEADER and len(lines[1].split(",")) == 31
    assert open(per_tpr).readline().strip() == TPR_HEADER
    rows = list(csv.DictReader(open(results)))
    samples = list(csv.DictReader(open(per_tpr)))
    published = {(r["matrix"], r["prec"], r["column_mode"], r["column_bytes"]): r
                 for r in csv.DictReader(open(os.path.join(GOLDEN, "published_bytes.csv")))}
    published_tpr = {(r["matrix"], r["prec"], r["layout"], r["tpr"]): float(r["bytes_total"])
                     for r in csv.DictReader(open(os.path.join(GOLDEN, "published_tpr_bytes.csv")))}

    custom = [r for r in rows if r["kernel"] == "custom"]
    assert len(custom) == 2 * 3 * 6
    for row in custom:
        assert row["ordering"] == "rcm" and row["row_encoding"] == "cumulative"
        key = (row["matrix"], row["prec"], row["column_mode"], row["column_bytes"])
        expected = published[key]
        assert row["status"] == expected["status"], key
        label = LABELS[(row["column_mode"], row["column_bytes"])]
        if label != "lp":
            assert float(row["bytes_total"]) == float(expected["bytes_total"]), key
        if row["status"] != "ok":
            continue
        assert float(row["max_abs_diff"]) == 0.0, key
        if label == "lp":
            assert float(row["bytes_total"]) == published_tpr[(row["matrix"], row["prec"], "lp", row["best_tpr"])]
        assert float(row["t_ms"]) > 0 and float(row["epsilon"]) > 0 and int(row["best_tpr"]) in (2, 4, 8, 16, 32)
    for sample in samples:
        assert float(sample["max_abs_diff"]) == 0.0, sample
        assert float(sample["bytes_total"]) == published_tpr[(sample["matrix"], sample["prec"], sample["layout"], sample["tpr"])]
    library = [r for r in rows if r["kernel"].startswith("cusparse")]
    assert len(library) == 2 * 3 * 2
    for row in library:
        assert row["status"] == "ok", row
        assert float(row["max_rel_diff"]) <= CUSPARSE_TOLERANCE[row["prec"]], row


@pytest.mark.gpu
def test_half_sums_campaign_rows(smoke_matrix_paths, tmp_path):
    """--accumulate half (the reference's bench_csr_width_fp16acc): FP16 rows only, every layout still
    bit-identical to CSR-i32 at the same T (all of them sum in FP16 in the same order)."""
    binary = built()
    results = tmp_path / "results.csv"
    name, path = sorted(smoke_matrix_paths.items())[0]
    local = tmp_path / os.path.basename(path)
    os.symlink(path, local)
    done = subprocess.run([binary, "--matrix", str(local), "--reps", "2", "--warmup", "1", "--accumulate", "half",
                           "--csv", str(results)], capture_output=True, text=True, timeout=900)
    assert done.returncode == 0, done.stdout[-2000:] + done.stderr[-2000:]
    rows = [r for r in csv.DictReader(open(results)) if r["kernel"] == "custom"]
    assert len(rows) == 6 and all(r["prec"] == "fp16" for r in rows)
    for row in rows:
        if row["status"] == "ok":
            assert float(row["max_abs_diff"]) == 0.0, row


@pytest.mark.gpu
def test_r16_control_campaign_rows(smoke_matrix_paths, tmp_path):
    """--r16-control (the reference's bench_csr_width_r16{lane,pair,wide,unroll16} builds): the r16 rows are the
    control kernels', still bit-identical to CSR-i32; WIDE counts 4 bytes an offset."""
    binary = built()
    name, path = sorted(smoke_matrix_paths.items())[0]
    local = tmp_path / os.path.basename(path)
    os.symlink(path, local)
    bytes_of = {}
    for control in ("lane", "pair", "wide", "unroll16"):
        results = tmp_path / f"{control}.csv"
        done = subprocess.run([binary, "--matrix", str(local), "--reps", "2", "--warmup", "1", "--precision", "fp64",
                               "--ordering", "rcm", "--r16-control", control, "--csv", str(results)],
                              capture_output=True, text=True, timeout=900)
        assert done.returncode == 0, done.stdout[-2000:] + done.stderr[-2000:]
        rows = [r for r in csv.DictReader(open(results)) if r["kernel"] == "custom" and r["column_mode"] == "row-base"
                and r["column_bytes"] == "2"]
        assert len(rows) == 1, control
        if rows[0]["status"] == "ok":
            assert float(rows[0]["max_abs_diff"]) == 0.0, (control, rows[0])
        bytes_of[control] = float(rows[0]["bytes_total"])
    nnz = float(rows[0]["nnz"])
    assert bytes_of["wide"] == pytest.approx(bytes_of["lane"] + 2 * nnz)
