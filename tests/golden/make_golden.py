#!/usr/bin/env python3
"""Regenerates the golden fixtures of tests/golden/ from the reference (HERMES-TorVerLab/spmv-index-compression).

    python tests/golden/make_golden.py --reference <reference tree>   (or SPMV_REFERENCE_ROOT set)

Reads the reference tree as text and data, and runs the reference's own code compiled from its sources
(oracle/_ref, `make -C oracle ref`). Writes:

  published_bytes.csv     the published byte counts of dawson5 and rim (data/results/a100/csr_layouts_rcm.csv,
                          kernel "custom"): every layout's memory_of, the numbers compare_campaign.py gates on
  published_tpr_bytes.csv the per-T byte counts (data/results/a100/csr_layouts_rcm_tpr.csv): CSR-lp at every T
  characterization_rcm.csv  the published characterization rows of dawson5 and rim (matrices/characterization_rcm)
  lp_worked_example.json  the 10-entry row of analysis/make_layout_figure.py:22 encoded by the reference's
                          build_packed_deltas at T = 2 and 4
  reference_streams.npz   small matrices (ragged, empty rows, wide deltas) with the reference's RCM order,
                          CSR-lp streams at T = 2..32, facts and memory_of, for checks without the reference
"""
import argparse
import csv
import json
import os
import re
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def published_rows(reference):
    keep = ("matrix", "prec", "column_mode", "column_bytes", "status", "rows", "cols", "nnz", "bytes_values",
            "bytes_columns", "bytes_column_bases", "bytes_row_pointer", "bytes_vectors", "bytes_total", "best_tpr",
            "max_abs_diff")
    source = os.path.join(reference, "data/results/a100/csr_layouts_rcm.csv")
    with open(source) as handle, open(os.path.join(HERE, "published_bytes.csv"), "w", newline="") as out:
        writer = csv.writer(out)
        writer.writerow(keep)
        for row in csv.DictReader(handle):
            if row["matrix"] in ("dawson5", "rim") and row["kernel"] == "custom":
                writer.writerow([row[key] for key in keep])
    source = os.path.join(reference, "data/results/a100/csr_layouts_rcm_tpr.csv")
    with open(source) as handle, open(os.path.join(HERE, "published_tpr_bytes.csv"), "w", newline="") as out:
        writer = csv.writer(out)
        writer.writerow(("matrix", "prec", "layout", "tpr", "bytes_total", "nnz", "max_abs_diff"))
        for row in csv.DictReader(handle):
            if row["matrix"] in ("dawson5", "rim"):
                writer.writerow([row[k] for k in ("matrix", "prec", "layout", "tpr", "bytes_total", "nnz", "max_abs_diff")])


def characterization_rows(reference):
    with open(os.path.join(HERE, "characterization_rcm.csv"), "w") as out:
        for index, name in enumerate(("dawson5", "rim")):
            lines = open(os.path.join(reference, "matrices/characterization_rcm", name + ".csv")).read().splitlines()
            out.write("\n".join(lines if index == 0 else lines[1:]) + "\n")


def lp_worked_example(reference, ref):
    text = open(os.path.join(reference, "analysis/make_layout_figure.py")).read()
    columns = [int(value) for value in re.search(r"COLUMNS\s*=\s*\[([^\]]*)\]", text).group(1).split(",")]
    n = max(columns) + 1
    row_ptr = np.array([0, len(columns)], np.int32)
    handle = ref.from_arrays(1, n, row_ptr, np.array(columns, np.int32))
    example = {"columns": columns, "cols": n, "encodings": {}}
    for tpr in (2, 4, 8, 16, 32):
        row_word, row_width, words = ref.build_packed_deltas(handle, 1, tpr)
        example["encodings"][str(tpr)] = {"width": int(row_width[0]), "row_word": int(row_word[0]),
                                          "words": [int(w) for w in words]}
    ref.free(handle)
    with open(os.path.join(HERE, "lp_worked_example.json"), "w") as out:
        json.dump(example, out, indent=1)


def small_matrices():
    """A few deterministic small square matrices exercising the encoders' edge cases."""
    rng = np.random.default_rng(20240601)
    cases = {}
    # ragged rows, empty rows, a long row, wide deltas near 2^16 and beyond
    n = 300
    rows = []
    for r in range(n):
        kind = r % 7
        if kind == 0:
            cols = []
        elif kind == 1:
            cols = [r]
        elif kind == 2:
            cols = sorted(set(rng.integers(0, n, size=rng.integers(1, 40)).tolist()))
        elif kind == 3:
            cols = list(range(max(0, r - 3), min(n, r + 4)))
        elif kind == 4:
            cols = sorted(set([0, n - 1, r]))
        else:
            cols = sorted(set(rng.integers(max(0, r - 20), min(n, r + 20), size=8).tolist()))
        rows.append(cols)
    rows[150] = list(range(0, n, 2))    # one long row of 150 entries
    cases["ragged300"] = rows
    # wide columns: n = 200000, rows with spans beyond 2^16
    n2 = 200000
    rows2 = []
    for r in range(64):
        k = int(rng.integers(0, 60))
        rows2.append(sorted(set(rng.integers(0, n2, size=k).tolist())))
    cases["wide64"] = (rows2, n2)
    return cases


def reference_streams(ref):
    arrays = {}
    for name, case in small_matrices().items():
        rows_list, cols = (case, len(case)) if isinstance(case, list) else case
        nrows = len(rows_list)
        row_ptr = np.zeros(nrows + 1, np.int32)
        row_ptr[1:] = np.cumsum([len(r) for r in rows_list])
        col_ind = np.array([c for r in rows_list for c in r], np.int32)
        values = np.linspace(-1.0, 1.0, max(col_ind.size, 1))[:col_ind.size]
        handle = ref.from_arrays(nrows, cols, row_ptr, col_ind, values)
        arrays[f"{name}/row_ptr"] = row_ptr
        arrays[f"{name}/col_ind"] = col_ind
        arrays[f"{name}/cols"] = np.array([cols])
        span, lane_words = ref.facts(handle)
        arrays[f"{name}/widest_row_span"] = np.array([span])
        arrays[f"{name}/lane_packed_words"] = lane_words
        for tpr in (2, 4, 8, 16, 32):
            row_word, row_width, words = ref.build_packed_deltas(handle, nrows, tpr)
            arrays[f"{name}/lp{tpr}/row_word"] = row_word
            arrays[f"{name}/lp{tpr}/row_width"] = row_width
            arrays[f"{name}/lp{tpr}/words"] = words
        for layout, label in ((0, "i32"), (1, "i16"), (2, "r16"), (3, "lp"), (4, "i8"), (5, "r8")):
            for value_bytes in (8, 4, 2):
                arrays[f"{name}/memory/{label}/{value_bytes}"] = ref.memory_of(handle, value_bytes, layout, 4)
            arrays[f"{name}/admissible/{label}"] = np.array([ref.admissible(handle, layout, 4)])
        if nrows == cols:
            arrays[f"{name}/rcm"] = ref.rcm_order(handle, nrows)
        ref.free(handle)
    np.savez_compressed(os.path.join(HERE, "reference_streams.npz"), **arrays)


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("SPMV_REFERENCE_ROOT", ""))
    args = parser.parse_args()
    if not args.reference:
        parser.error("name the reference tree with --reference or SPMV_REFERENCE_ROOT")
    import oracle
    oracle.build(reference=True, reference_root=args.reference)
    ref = oracle.Reference()
    published_rows(args.reference)
    characterization_rows(args.reference)
    lp_worked_example(args.reference, ref)
    reference_streams(ref)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
