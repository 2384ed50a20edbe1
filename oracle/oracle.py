"""oracle.py — TEST INFRASTRUCTURE ONLY: ctypes bindings to the CPU oracle (liboracle.so, the C restatement
in spmv_oracle.c) and to the reference's own code compiled from its sources (_ref/libspmvref.so and
_ref/characterize_matrix, built by `make -C oracle ref` where the reference tree is present).

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline / reference arm use this module, as the
checker or as the timed CPU baseline. The product never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIBRARY = os.path.join(HERE, "liboracle.so")
REFERENCE_LIBRARY = os.path.join(HERE, "_ref", "libspmvref.so")
REFERENCE_CHARACTERIZE = os.path.join(HERE, "_ref", "characterize_matrix")

I32, I16, R16, LP, I8, R8 = 0, 1, 2, 3, 4, 5
F64, F32, F16 = 0, 1, 2
# F16_HALF_SUMS: FP16 values summed in FP16 (the reference's SPMV_HALF_ACCUMULATE control build)
F16_HALF_SUMS = 3
NUMPY = {F64: np.float64, F32: np.float32, F16: np.float16, F16_HALF_SUMS: np.float16}


def build(reference: bool = False, reference_root: str = ""):
    """Builds liboracle.so (and, with reference=True, the _ref checkers from the reference sources under
    reference_root, or under SPMV_REFERENCE_ROOT when that is empty)."""
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    if reference:
        extra = [f"REFERENCE_ROOT={reference_root}"] if reference_root else []
        subprocess.run(["make", "-s", "-C", HERE, "ref"] + extra, check=True)


def _load_oracle():
    if not os.path.exists(ORACLE_LIBRARY):
        build()
    lib = ctypes.CDLL(ORACLE_LIBRARY)
    v, i, i64, d = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_double
    lib.oracle_spmv.restype = i
    lib.oracle_spmv.argtypes = [i, i, i, i, v, v, v, v, v, v, v, v, v, i]
    lib.oracle_half_fma_array.argtypes = [i64, v, v, v, v]
    lib.oracle_lane_packed_words.restype = i64
    lib.oracle_lane_packed_words.argtypes = [i, v, v, i]
    lib.oracle_build_lane_packed.restype = i
    lib.oracle_build_lane_packed.argtypes = [i, v, v, i, i64, v, v, v]
    lib.oracle_row_bases.restype = None
    lib.oracle_row_bases.argtypes = [i, v, v, v]
    lib.oracle_relative_columns.restype = None
    lib.oracle_relative_columns.argtypes = [i, v, v, i, v]
    lib.oracle_narrow_columns.restype = None
    lib.oracle_narrow_columns.argtypes = [i64, v, i, v]
    lib.oracle_widest_row_span.restype = i
    lib.oracle_widest_row_span.argtypes = [i, v, v]
    lib.oracle_admissible.restype = i
    lib.oracle_admissible.argtypes = [i, i, v, i, i, i]
    lib.oracle_memory_of.restype = None
    lib.oracle_memory_of.argtypes = [i, i, i64, v, i, i, i, i, v]
    lib.oracle_convert_values.restype = None
    lib.oracle_convert_values.argtypes = [i, i64, v, v]
    lib.oracle_max_threads.restype = i
    lib.oracle_set_threads.restype = None
    lib.oracle_set_threads.argtypes = [i]
    lib.oracle_tpr_slot.restype = i
    lib.oracle_tpr_slot.argtypes = [i]
    return lib


_oracle = _load_oracle()


def _p(array: Optional[np.ndarray]):
    if array is None:
        return None
    return array.ctypes.data if array.size else None


def max_threads() -> int:
    return _oracle.oracle_max_threads()


def set_threads(count: int) -> None:
    """Sets the threads the oracle's products use by default. A launcher such as torch.distributed.run
    exports OMP_NUM_THREADS=1, which would otherwise hold the oracle to one core."""
    _oracle.oracle_set_threads(int(count))


# ---- encoders (bench_csr_width.cu:149-285, 795-917) --------------------------------------------------------
def lane_packed_words(row_ptr, col_ind, tpr: int) -> int:
    row_ptr = np.ascontiguousarray(row_ptr, np.int32)
    col_ind = np.ascontiguousarray(col_ind, np.int32)
    return _oracle.oracle_lane_packed_words(row_ptr.size - 1, _p(row_ptr), _p(col_ind), tpr)


def build_lane_packed(row_ptr, col_ind, tpr: int):
    row_ptr = np.ascontiguousarray(row_ptr, np.int32)
    col_ind = np.ascontiguousarray(col_ind, np.int32)
    rows = row_ptr.size - 1
    count = lane_packed_words(row_ptr, col_ind, tpr)
    row_word = np.zeros(max(rows, 1), np.int32)
    row_width = np.zeros(max(rows, 1), np.uint8)
    words = np.zeros(count, np.uint32)
    status = _oracle.oracle_build_lane_packed(rows, _p(row_ptr), _p(col_ind), tpr, count, _p(row_word), _p(row_width),
                                              _p(words))
    assert status == 0, "oracle lane-packed encoder overflowed its words"
    return row_word[:rows], row_width[:rows], words


def row_bases(row_ptr, col_ind) -> np.ndarray:
    row_ptr = np.ascontiguousarray(row_ptr, np.int32)
    col_ind = np.ascontiguousarray(col_ind, np.int32)
    rows = row_ptr.size - 1
    out = np.zeros(max(rows, 1), np.int32)
    _oracle.oracle_row_bases(rows, _p(row_ptr), _p(col_ind), _p(out))
    return out[:rows]


def relative_columns(row_ptr, col_ind, column_bytes: int) -> np.ndarray:
    row_ptr = np.ascontiguousarray(row_ptr, np.int32)
    col_ind = np.ascontiguousarray(col_ind, np.int32)
    out = np.zeros(max(col_ind.size, 1), np.uint16 if column_bytes == 2 else np.uint8)
    _oracle.oracle_relative_columns(row_ptr.size - 1, _p(row_ptr), _p(col_ind), column_bytes, _p(out))
    return out[:col_ind.size]


def narrow_columns(col_ind, column_bytes: int) -> np.ndarray:
    col_ind = np.ascontiguousarray(col_ind, np.int32)
    out = np.zeros(max(col_ind.size, 1), np.uint16 if column_bytes == 2 else np.uint8)
    _oracle.oracle_narrow_columns(col_ind.size, _p(col_ind), column_bytes, _p(out))
    return out[:col_ind.size]


def widest_row_span(row_ptr, col_ind) -> int:
    row_ptr = np.ascontiguousarray(row_ptr, np.int32)
    col_ind = np.ascontiguousarray(col_ind, np.int32)
    return _oracle.oracle_widest_row_span(row_ptr.size - 1, _p(row_ptr), _p(col_ind))


def lane_words_by_slot(row_ptr, col_ind) -> np.ndarray:
    words = np.zeros(6, np.int64)
    for slot in range(1, 6):
        words[slot] = lane_packed_words(row_ptr, col_ind, 1 << slot)
    return words


MODE_OF = {I32: (0, 4), I16: (0, 2), I8: (0, 1), R16: (1, 2), R8: (1, 1), LP: (2, 0)}


def admissible(rows, cols, row_ptr, col_ind, layout: int, tpr: int = 0, lane_words=None) -> bool:
    mode, column_bytes = MODE_OF[layout]
    lane_words = lane_words_by_slot(row_ptr, col_ind) if lane_words is None else np.asarray(lane_words, np.int64)
    span = widest_row_span(row_ptr, col_ind)
    return bool(_oracle.oracle_admissible(cols, span, _p(lane_words), mode, column_bytes, tpr))


def memory_of(rows, cols, row_ptr, col_ind, layout: int, value_bytes: int, tpr: int = 0, lane_words=None) -> np.ndarray:
    """values, columns, column_bases, row_pointer, vectors, total."""
    mode, column_bytes = MODE_OF[layout]
    lane_words = lane_words_by_slot(row_ptr, col_ind) if lane_words is None else np.asarray(lane_words, np.int64)
    out = np.zeros(6)
    _oracle.oracle_memory_of(rows, cols, int(np.asarray(col_ind).size), _p(lane_words), value_bytes, column_bytes, mode,
                             tpr, _p(out))
    return out


def convert_values(values, dtype: int) -> np.ndarray:
    values = np.ascontiguousarray(values, np.float64)
    out = np.zeros(max(values.size, 1), NUMPY[dtype])
    _oracle.oracle_convert_values(dtype, values.size, _p(values), _p(out))
    return out[:values.size]


# ---- the SpMV in reference order ------------------------------------------------------------------------------
def spmv(dtype: int, layout: int, tpr: int, row_ptr, values, x, columns=None, row_base=None, row_word=None,
         row_width=None, words=None, threads: int = 0) -> np.ndarray:
    """y = A x summed as the reference kernels sum (lane chains of fma, then the shuffle tree)."""
    row_ptr = np.ascontiguousarray(row_ptr, np.int32)
    rows = row_ptr.size - 1
    values = np.ascontiguousarray(values, NUMPY[dtype])
    x = np.ascontiguousarray(x, NUMPY[dtype])
    y = np.zeros(max(rows, 1), NUMPY[dtype])
    if columns is not None:
        columns = np.ascontiguousarray(columns)
    status = _oracle.oracle_spmv(dtype, layout, tpr, rows, _p(row_ptr), _p(columns), _p(row_base), _p(row_word),
                                 _p(row_width), _p(words), _p(values), _p(x), _p(y), threads)
    assert status == 0, "oracle_spmv rejected its arguments"
    return y[:rows]


def encode(row_ptr, col_ind, layout: int, tpr: int) -> dict:
    """The reference's streams of one layout, as keyword arguments of spmv()."""
    if layout == I32:
        return {"columns": np.ascontiguousarray(col_ind, np.int32)}
    if layout in (I16, I8):
        return {"columns": narrow_columns(col_ind, 2 if layout == I16 else 1)}
    if layout in (R16, R8):
        return {"columns": relative_columns(row_ptr, col_ind, 2 if layout == R16 else 1),
                "row_base": row_bases(row_ptr, col_ind)}
    row_word, row_width, words = build_lane_packed(row_ptr, col_ind, tpr)
    return {"row_base": row_bases(row_ptr, col_ind), "row_word": row_word, "row_width": row_width, "words": words}


def half_fma(a, b, c) -> np.ndarray:
    """a*b + c of FP16 arrays, rounded once to FP16 (what __hfma computes), element by element."""
    a, b, c = (np.ascontiguousarray(t, np.float16) for t in (a, b, c))
    out = np.zeros(max(a.size, 1), np.float16)
    _oracle.oracle_half_fma_array(a.size, _p(a), _p(b), _p(c), _p(out))
    return out[:a.size]


def spmv_csr(row_ptr, col_ind, values64, x, dtype: int, layout: int, tpr: int, threads: int = 0) -> np.ndarray:
    """Reference-order product of a CSR matrix (FP64 values, converted as upload_matrix does) in one layout."""
    return spmv(dtype, layout, tpr, row_ptr, convert_values(values64, dtype), x, threads=threads,
                **encode(row_ptr, col_ind, layout, tpr))


# ---- the reference itself, compiled from its sources --------------------------------------------------------
class Reference:
    """The reference's reader, RCM, encoders, byte model and kernels (oracle/_ref/libspmvref.so)."""

    def __init__(self, path: str = REFERENCE_LIBRARY):
        lib = ctypes.CDLL(path)
        v, i, d, s = ctypes.c_void_p, ctypes.c_int, ctypes.c_double, ctypes.c_char_p
        ll = ctypes.c_longlong
        lib.ref_read_matrix_market.restype = v
        lib.ref_read_matrix_market.argtypes = [s, s, i]
        lib.ref_matrix_from_arrays.restype = v
        lib.ref_matrix_from_arrays.argtypes = [i, i, v, v, v]
        lib.ref_matrix_free.argtypes = [v]
        lib.ref_matrix_shape.argtypes = [v, v, v, v]
        lib.ref_matrix_copy.argtypes = [v, v, v, v]
        lib.ref_matrix_stats.argtypes = [v, v]
        lib.ref_rcm_order.restype = i
        lib.ref_rcm_order.argtypes = [v, v]
        lib.ref_permute.restype = v
        lib.ref_permute.argtypes = [v, v]
        lib.ref_reorder_with_rcm.restype = v
        lib.ref_reorder_with_rcm.argtypes = [s, v, ctypes.POINTER(d)]
        lib.ref_packed_word_count.restype = ll
        lib.ref_packed_word_count.argtypes = [v, i]
        lib.ref_build_packed_deltas.argtypes = [v, i, ll, v, v, v]
        lib.ref_facts.argtypes = [v, v, v]
        lib.ref_memory_of.argtypes = [v, i, i, i, i, v]
        lib.ref_admissible.restype = i
        lib.ref_admissible.argtypes = [v, i, i, i]
        lib.ref_launch.restype = i
        lib.ref_launch.argtypes = [i, i, i, i, i, ll, v, v, v, v, v, v, v, v, v]
        self.has_async = hasattr(lib, "ref_launch_async")
        if self.has_async:
            lib.ref_launch_async.restype = i
            lib.ref_launch_async.argtypes = [i, i, i, i, i, ll, v, v, v, v, v, v, v, v, v]
        self.lib = lib

    @staticmethod
    def available() -> bool:
        return os.path.exists(REFERENCE_LIBRARY)

    # matrices are opaque handles freed with free()
    def read_matrix_market(self, path: str):
        error = ctypes.create_string_buffer(512)
        handle = self.lib.ref_read_matrix_market(os.fsencode(path), error, 512)
        if not handle:
            raise RuntimeError(error.value.decode())
        return handle

    def from_arrays(self, rows, cols, row_ptr, col_ind, values=None):
        row_ptr = np.ascontiguousarray(row_ptr, np.int32)
        col_ind = np.ascontiguousarray(col_ind, np.int32)
        values = None if values is None else np.ascontiguousarray(values, np.float64)
        return self.lib.ref_matrix_from_arrays(rows, cols, _p(row_ptr), _p(col_ind), _p(values))

    def free(self, handle):
        self.lib.ref_matrix_free(handle)

    def arrays(self, handle):
        rows, cols, nnz = ctypes.c_int(), ctypes.c_int(), ctypes.c_longlong()
        self.lib.ref_matrix_shape(handle, ctypes.byref(rows), ctypes.byref(cols), ctypes.byref(nnz))
        row_ptr = np.zeros(rows.value + 1, np.int32)
        col_ind = np.zeros(max(nnz.value, 1), np.int32)
        values = np.zeros(max(nnz.value, 1), np.float64)
        self.lib.ref_matrix_copy(handle, _p(row_ptr), _p(col_ind), _p(values))
        return rows.value, cols.value, row_ptr, col_ind[:nnz.value], values[:nnz.value]

    def stats(self, handle) -> np.ndarray:
        out = np.zeros(8)
        self.lib.ref_matrix_stats(handle, _p(out))
        return out

    def rcm_order(self, handle, rows: int) -> np.ndarray:
        order = np.zeros(rows, np.int32)
        assert self.lib.ref_rcm_order(handle, _p(order)) == 0
        return order

    def permute(self, handle, new_to_old):
        order = np.ascontiguousarray(new_to_old, np.int32)
        return self.lib.ref_permute(handle, _p(order))

    def reorder_with_rcm(self, matrix_path: str, handle):
        seconds = ctypes.c_double()
        result = self.lib.ref_reorder_with_rcm(os.fsencode(matrix_path), handle, ctypes.byref(seconds))
        if not result:
            raise RuntimeError("reference reorder_with_rcm failed")
        return result, seconds.value

    def packed_word_count(self, handle, tpr: int) -> int:
        return self.lib.ref_packed_word_count(handle, tpr)

    def build_packed_deltas(self, handle, rows: int, tpr: int):
        count = self.packed_word_count(handle, tpr)
        row_word = np.zeros(max(rows, 1), np.int32)
        row_width = np.zeros(max(rows, 1), np.uint8)
        words = np.zeros(count, np.uint32)
        self.lib.ref_build_packed_deltas(handle, tpr, count, _p(row_word), _p(row_width), _p(words))
        return row_word[:rows], row_width[:rows], words

    def facts(self, handle):
        span = ctypes.c_int()
        words = np.zeros(6, np.int64)
        self.lib.ref_facts(handle, ctypes.byref(span), _p(words))
        return span.value, words

    def memory_of(self, handle, value_bytes: int, layout: int, tpr: int = 0) -> np.ndarray:
        mode, column_bytes = MODE_OF[layout]
        out = np.zeros(6)
        self.lib.ref_memory_of(handle, value_bytes, column_bytes, mode, tpr, _p(out))
        return out

    def admissible(self, handle, layout: int, tpr: int = 0) -> bool:
        mode, column_bytes = MODE_OF[layout]
        return bool(self.lib.ref_admissible(handle, column_bytes, mode, tpr))

    def launch(self, dtype, layout, tpr, rows, cols, nnz, row_ptr, columns, row_base, row_word, row_width, words, values,
               x, y) -> int:
        """The reference kernels on device pointers (integers); returns the cudaError_t."""
        return self.lib.ref_launch(dtype, layout, tpr, rows, cols, nnz, row_ptr, columns, row_base, row_word, row_width,
                                   words, values, x, y)

    def launch_async(self, dtype, layout, tpr, rows, cols, nnz, row_ptr, columns, row_base, row_word, row_width, words,
                     values, x, y) -> int:
        """The reference kernels on the default stream without waiting (back-to-back timing); returns the
        launch's cudaError_t."""
        call = self.lib.ref_launch_async if self.has_async else self.lib.ref_launch
        return call(dtype, layout, tpr, rows, cols, nnz, row_ptr, columns, row_base, row_word, row_width, words,
                    values, x, y)


def reference_characterize(matrix_path: str, ordering: str = "original") -> str:
    """Runs the reference's characterize_matrix on a .mtx and returns its CSV text."""
    result = subprocess.run([REFERENCE_CHARACTERIZE, matrix_path, "--ordering", ordering], check=True,
                            capture_output=True, text=True)
    return result.stdout
