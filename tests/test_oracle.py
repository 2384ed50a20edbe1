"""Pins the CPU oracle (oracle/spmv_oracle.c) before anything is checked against it: its encoders and byte
model against the reference's own code (oracle/_ref) and the published numbers (tests/golden/), and its
SpMV against the reference's acceptance rule (every layout bit-identical to CSR-i32 at the same T)."""
import csv
import json
import os

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, random_csr

LAYOUTS = (oracle.I32, oracle.I16, oracle.R16, oracle.LP, oracle.I8, oracle.R8)


def golden_streams():
    data = np.load(os.path.join(GOLDEN, "reference_streams.npz"))
    names = sorted({key.split("/")[0] for key in data.files})
    return data, names


def test_lp_worked_example_matches_reference_encoder():
    """analysis/make_layout_figure.py:22: the 10-entry row encoded by build_packed_deltas."""
    example = json.load(open(os.path.join(GOLDEN, "lp_worked_example.json")))
    columns = np.array(example["columns"], np.int32)
    row_ptr = np.array([0, columns.size], np.int32)
    for tpr, expected in example["encodings"].items():
        row_word, row_width, words = oracle.build_lane_packed(row_ptr, columns, int(tpr))
        assert int(row_width[0]) == expected["width"]
        assert int(row_word[0]) == expected["row_word"]
        assert words.tolist() == expected["words"]
    # the figure's own arithmetic: deltas from the entry T back, width = bits of the widest delta
    deltas4 = [c - columns[0] if i < 4 else c - columns[i - 4] for i, c in enumerate(columns)]
    assert example["encodings"]["4"]["width"] == int(max(deltas4)).bit_length() == 4
    assert len(example["encodings"]["4"]["words"]) == -(-columns.size * 4 // 32) + 2


def test_encoders_match_reference_fixtures():
    data, names = golden_streams()
    for name in names:
        row_ptr, col_ind = data[f"{name}/row_ptr"], data[f"{name}/col_ind"]
        cols = int(data[f"{name}/cols"][0])
        rows = row_ptr.size - 1
        assert oracle.widest_row_span(row_ptr, col_ind) == int(data[f"{name}/widest_row_span"][0])
        words_by_slot = oracle.lane_words_by_slot(row_ptr, col_ind)
        assert np.array_equal(words_by_slot[1:], data[f"{name}/lane_packed_words"][1:])
        for tpr in (2, 4, 8, 16, 32):
            row_word, row_width, words = oracle.build_lane_packed(row_ptr, col_ind, tpr)
            assert np.array_equal(row_word, data[f"{name}/lp{tpr}/row_word"]), (name, tpr)
            assert np.array_equal(row_width, data[f"{name}/lp{tpr}/row_width"]), (name, tpr)
            assert np.array_equal(words, data[f"{name}/lp{tpr}/words"]), (name, tpr)
        for layout, label in ((0, "i32"), (1, "i16"), (2, "r16"), (3, "lp"), (4, "i8"), (5, "r8")):
            for value_bytes in (8, 4, 2):
                memory = oracle.memory_of(rows, cols, row_ptr, col_ind, layout, value_bytes, 4, words_by_slot)
                assert np.array_equal(memory, data[f"{name}/memory/{label}/{value_bytes}"]), (name, label)
            assert oracle.admissible(rows, cols, row_ptr, col_ind, layout, 4, words_by_slot) == \
                bool(data[f"{name}/admissible/{label}"][0])


def test_encoders_match_reference_on_random(reference):
    for seed in range(4):
        rows, cols = 257 + seed, 70000 if seed % 2 else 513
        row_ptr, col_ind, values = random_csr(rows, cols, 9 + 5 * seed, seed, empty_every=11,
                                              long_rows={5: 400} if seed == 3 else ())
        handle = reference.from_arrays(rows, cols, row_ptr, col_ind, values)
        try:
            span, lane_words = reference.facts(handle)
            assert oracle.widest_row_span(row_ptr, col_ind) == span
            assert np.array_equal(oracle.lane_words_by_slot(row_ptr, col_ind)[1:], lane_words[1:])
            for tpr in (2, 4, 8, 16, 32):
                mine = oracle.build_lane_packed(row_ptr, col_ind, tpr)
                theirs = reference.build_packed_deltas(handle, rows, tpr)
                for a, b in zip(mine, theirs):
                    assert np.array_equal(a, b)
            for layout in (0, 1, 2, 3, 4, 5):
                for value_bytes in (8, 4, 2):
                    for tpr in (0, 2, 32):
                        assert np.array_equal(oracle.memory_of(rows, cols, row_ptr, col_ind, layout, value_bytes, tpr),
                                              reference.memory_of(handle, value_bytes, layout, tpr))
                assert oracle.admissible(rows, cols, row_ptr, col_ind, layout, 8) == reference.admissible(handle, layout, 8)
        finally:
            reference.free(handle)


def published(prec=None):
    rows = list(csv.DictReader(open(os.path.join(GOLDEN, "published_bytes.csv"))))
    return [row for row in rows if prec is None or row["prec"] == prec]


def test_memory_of_matches_published_bytes(smoke_matrix_paths, reference):
    """The byte counts compare_campaign.py gates on (data/results/a100/csr_layouts_rcm.csv), from the
    RCM-ordered matrices, for every layout and precision (CSR-lp at its published best T)."""
    for name, path in smoke_matrix_paths.items():
        handle = reference.read_matrix_market(path)
        order = reference.rcm_order(handle, reference.arrays(handle)[0])
        permuted = reference.permute(handle, order)
        rows, cols, row_ptr, col_ind, _ = reference.arrays(permuted)
        lane_words = oracle.lane_words_by_slot(row_ptr, col_ind)
        checked = 0
        for row in published():
            if row["matrix"] != name:
                continue
            mode = {"absolute": {"4": 0, "2": 1, "1": 4}, "row-base": {"2": 2, "1": 5},
                    "lane-packed": {"0": 3}}[row["column_mode"]][row["column_bytes"]]
            value_bytes = {"fp64": 8, "fp32": 4, "fp16": 2}[row["prec"]]
            tpr = int(row["best_tpr"]) if mode == 3 else 0
            memory = oracle.memory_of(rows, cols, row_ptr, col_ind, mode, value_bytes, tpr, lane_words)
            assert memory[5] == float(row["bytes_total"]), (name, row["prec"], row["column_mode"], row["column_bytes"])
            assert memory[1] == float(row["bytes_columns"])
            assert memory[2] == float(row["bytes_column_bases"])
            admissible = oracle.admissible(rows, cols, row_ptr, col_ind, mode, tpr, lane_words)
            assert admissible == (row["status"] == "ok")
            checked += 1
        assert checked == 18
        # CSR-lp at every T (csr_layouts_rcm_tpr.csv)
        for row in csv.DictReader(open(os.path.join(GOLDEN, "published_tpr_bytes.csv"))):
            if row["matrix"] == name and row["layout"] == "lp":
                value_bytes = {"fp64": 8, "fp32": 4, "fp16": 2}[row["prec"]]
                memory = oracle.memory_of(rows, cols, row_ptr, col_ind, 3, value_bytes, int(row["tpr"]), lane_words)
                assert memory[5] == float(row["bytes_total"])
        reference.free(permuted)
        reference.free(handle)


@pytest.mark.parametrize("dtype", [oracle.F64, oracle.F32, oracle.F16])
@pytest.mark.parametrize("tpr", [2, 4, 8, 16, 32])
def test_layouts_bit_identical_to_i32(dtype, tpr):
    """The reference's acceptance rule (bench_csr_width.cu:14-16): every admissible layout at the same T
    sums in the same order as CSR-i32, so max |dy| = 0."""
    rows, cols = 400, 250
    row_ptr, col_ind, values = random_csr(rows, cols, 14, 100 + tpr, empty_every=13, long_rows={7: 200})
    x = oracle.convert_values(np.random.default_rng(tpr).uniform(-1, 1, cols), dtype)
    base = oracle.spmv_csr(row_ptr, col_ind, values, x, dtype, oracle.I32, tpr)
    for layout in LAYOUTS:
        if not oracle.admissible(rows, cols, row_ptr, col_ind, layout, tpr):
            continue
        y = oracle.spmv_csr(row_ptr, col_ind, values, x, dtype, layout, tpr)
        assert np.array_equal(y.view(np.uint8), base.view(np.uint8)), oracle.MODE_OF[layout]


def test_spmv_sums_in_lane_then_tree_order():
    """A hand-worked row: T=2, entries v0..v4, x = 1: lane 0 sums v0, v2, v4 and lane 1 sums v1, v3 (fma
    chains from +0), then lane0 + lane1. Float values chosen so that the order changes the rounding."""
    row_ptr = np.array([0, 5], np.int32)
    col_ind = np.arange(5, dtype=np.int32)
    values = np.array([1.0, 1e8, -1.0, -1e8, 3.0])
    x = np.ones(5, np.float32)
    y = oracle.spmv_csr(row_ptr, col_ind, values, x, oracle.F32, oracle.I32, 2)
    lane0 = np.float32(np.float32(np.float32(1.0) + np.float32(-1.0)) + np.float32(3.0))
    lane1 = np.float32(np.float32(1e8) + np.float32(-1e8))
    assert y[0] == np.float32(lane0 + lane1) == np.float32(3.0)
    # T=4: lanes {v0, v4}, {v1}, {v2}, {v3}; tree ((l0 + l2) + (l1 + l3))
    y4 = oracle.spmv_csr(row_ptr, col_ind, values, x, oracle.F32, oracle.I32, 4)
    l0, l1, l2, l3 = np.float32(4.0), np.float32(1e8), np.float32(-1.0), np.float32(-1e8)
    assert y4[0] == np.float32(np.float32(l0 + l2) + np.float32(l1 + l3))


def test_fp64_uses_fused_multiply_add():
    """sum += v * x is one fused multiply-add (nvcc contracts it): a chain fma(1+e, 1+e, -1) keeps the e^2
    that a separate multiply would round away."""
    e = 2.0 ** -30
    row_ptr = np.array([0, 3], np.int32)
    col_ind = np.array([0, 2, 1], np.int32)
    values = np.array([-1.0, 0.0, 1.0 + e])
    x = np.array([1.0, 1.0 + e, 0.0])
    # T=2: lane 0 chains entries 0 and 2: fma(1+e, 1+e, fma(-1, 1, 0)) = 2e + e^2 exactly; lane 1 = 0
    y = oracle.spmv(oracle.F64, oracle.I32, 2, row_ptr, values, x, columns=col_ind)
    assert y[0] == 2 * e + e * e
    assert y[0] != ((1.0 + e) * (1.0 + e)) - 1.0


def test_fp16_accumulates_in_fp32_and_narrows_once():
    row_ptr = np.array([0, 3], np.int32)
    col_ind = np.arange(3, dtype=np.int32)
    values = np.array([2048.0, 1.0, 1.0])
    x = np.ones(3, np.float16)
    # at T=2 lane 0 = 2048 + 1 in FP32 = 2049 and lane 1 = 1; sum 2050 -> FP16 2050 (FP16 steps are 2 there)
    y = oracle.spmv_csr(row_ptr, col_ind, values, x, oracle.F16, oracle.I32, 2)
    assert y[0] == np.float16(2050.0)
    # FP16 accumulation would give 2048 + 1 = 2048 (ties to even), then + 1 = 2048
    assert y[0] != np.float16(2048.0)


def test_empty_and_degenerate_rows():
    row_ptr = np.array([0, 0, 1, 1, 3, 3], np.int32)
    col_ind = np.array([2, 0, 4], np.int32)
    values = np.array([-0.0, 1.0, 2.0])
    x = np.array([1.0, 1.0, 1.0, 1.0, 1.0])
    for tpr in (2, 32):
        for layout in (oracle.I32, oracle.R16, oracle.LP):
            y = oracle.spmv_csr(row_ptr, col_ind, values, x, oracle.F64, layout, tpr)
            assert y.tolist() == [0.0, 0.0, 0.0, 3.0, 0.0]
            # an empty row and a row whose only product is -0 both give +0, as fma(., ., +0) does
            assert not np.signbit(y).any()
