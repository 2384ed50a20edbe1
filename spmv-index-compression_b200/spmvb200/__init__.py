"""spmvb200 — ctypes shim over libspmvb200.so, the B200 CSR SpMV library with compressed column indices.

The names mirror the reference benchmark's own host and operator functions (HERMES-TorVerLab/
spmv-index-compression: include/csr.hpp, include/rcm.hpp, src/characterize_matrix.cpp and
src/bench_csr_width.cu), so code written against that program reads the same here:

    matrix = read_matrix_market("A.mtx")                      # csr.hpp:232
    matrix = reorder_with_rcm("A.mtx", matrix)                # rcm.hpp:306
    facts = facts_of(matrix)                                  # bench_csr_width.cu:223
    configuration = Configuration(value_bytes=8, column_bytes=2, column_mode="row-base")
    configuration_admissible(matrix, facts, configuration)    # :246
    memory_of(matrix, facts, configuration)                   # :258
    op = Operator(matrix, layout=R16, dtype=F64, tpr=8)        # upload_matrix + launch<T>, :920 / :607
    op.run(x_device_pointer, y_device_pointer, stream)

Every failure raises SpmvError carrying the library status. There is no CPU fallback: the products run
only through the CUDA library, and creating an Operator without a GPU raises.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.environ.get("SPMVB200_LIBRARY", os.path.join(_HERE, "libspmvb200.so"))

# layouts (Configuration column_mode x column_bytes, bench_csr_width.cu:88)
I32, I16, R16, LP, I8, R8 = 0, 1, 2, 3, 4, 5
LAYOUT_NAMES = {I32: "i32", I16: "i16", R16: "r16", LP: "lp", I8: "i8", R8: "r8"}
LAYOUT_BY_NAME = {name: code for code, name in LAYOUT_NAMES.items()}
# value types
F64, F32, F16 = 0, 1, 2
DTYPE_NAMES = {F64: "fp64", F32: "fp32", F16: "fp16"}
DTYPE_BY_NAME = {name: code for code, name in DTYPE_NAMES.items()}
NUMPY_DTYPES = {F64: np.float64, F32: np.float32, F16: np.float16}
VALUE_BYTES = {F64: 8, F32: 4, F16: 2}
THREADS_PER_ROW = (2, 4, 8, 16, 32)
SCHEDULE_AUTO, SCHEDULE_TILES, SCHEDULE_CLASSES = 0, 1, 2
# the type FP16 values are summed in (SPMV_ACCUMULATE_*): FP32, or FP16 (the half-accumulate control build)
ACCUMULATE_WIDE, ACCUMULATE_HALF = 0, 1

OK = 0
ERR_INVALID_ARGUMENT, ERR_IO, ERR_FORMAT, ERR_NOT_ADMISSIBLE, ERR_OUT_OF_MEMORY = 1, 2, 3, 4, 5
ERR_CUDA, ERR_UNSUPPORTED, ERR_NCCL, ERR_TIMEOUT, ERR_TOO_LARGE = 6, 7, 8, 9, 10


class SpmvError(RuntimeError):
    """A failing library call; .status is the SPMV_ERR_* code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status


def _load():
    if not os.path.exists(LIBRARY_PATH):
        raise ImportError(f"libspmvb200.so is not built ({LIBRARY_PATH}); run `make -C spmv-index-compression_b200`")
    return ctypes.CDLL(LIBRARY_PATH, mode=ctypes.RTLD_GLOBAL)


_lib = _load()
_c_int_p = ctypes.POINTER(ctypes.c_int)
_c_void_pp = ctypes.POINTER(ctypes.c_void_p)


class CsrInfo(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int), ("cols", ctypes.c_int), ("nnz", ctypes.c_int64),
                ("nnz_per_row_mean", ctypes.c_double), ("nnz_per_row_max", ctypes.c_int),
                ("nnz_per_row_min", ctypes.c_int), ("nnz_per_row_std", ctypes.c_double),
                ("dynamic_range", ctypes.c_double), ("norm_inf", ctypes.c_double), ("max_abs", ctypes.c_double),
                ("min_abs", ctypes.c_double), ("symmetric_expanded", ctypes.c_int)]


class Facts(ctypes.Structure):
    """MatrixFacts (bench_csr_width.cu:160)."""
    _fields_ = [("widest_row_span", ctypes.c_int), ("lane_packed_words", ctypes.c_int64 * 6)]


class MemoryBreakdown(ctypes.Structure):
    """MemoryBreakdown (bench_csr_width.cu:95)."""
    _fields_ = [("values", ctypes.c_double), ("columns", ctypes.c_double), ("column_bases", ctypes.c_double),
                ("row_pointer", ctypes.c_double), ("vectors", ctypes.c_double), ("total", ctypes.c_double)]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


class OperatorConfig(ctypes.Structure):
    _fields_ = [("layout", ctypes.c_int), ("dtype", ctypes.c_int), ("tpr", ctypes.c_int),
                ("physical_tpr", ctypes.c_int), ("tile_nnz", ctypes.c_int), ("value_rounding", ctypes.c_int),
                ("device", ctypes.c_int), ("stages", ctypes.c_int), ("tile_rows", ctypes.c_int),
                ("schedule", ctypes.c_int), ("accumulate", ctypes.c_int)]


class OperatorInfo(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int), ("cols", ctypes.c_int), ("nnz", ctypes.c_int64), ("layout", ctypes.c_int),
                ("dtype", ctypes.c_int), ("tpr", ctypes.c_int), ("physical_tpr", ctypes.c_int),
                ("tile_nnz", ctypes.c_int), ("tiles", ctypes.c_int64), ("tile_ctas", ctypes.c_int64),
                ("stages", ctypes.c_int), ("tile_rows", ctypes.c_int), ("long_rows", ctypes.c_int64),
                ("device_bytes", ctypes.c_int64), ("memory", MemoryBreakdown), ("schedule", ctypes.c_int),
                ("listed_rows", ctypes.c_int64), ("blocks", ctypes.c_int64),
                ("window_elements", ctypes.c_int)]


class OperatorArrays(ctypes.Structure):
    _fields_ = [("row_ptr", ctypes.c_void_p), ("columns", ctypes.c_void_p), ("row_base", ctypes.c_void_p),
                ("row_word", ctypes.c_void_p), ("row_width", ctypes.c_void_p), ("words", ctypes.c_void_p),
                ("values", ctypes.c_void_p)]


class DeviceMatrix(ctypes.Structure):
    """DeviceMatrix<T> (bench_csr_width.cu:128) restricted to one layout: device pointers."""
    _fields_ = [("rows", ctypes.c_int), ("cols", ctypes.c_int), ("nnz", ctypes.c_int64),
                ("row_ptr", ctypes.c_void_p), ("columns", ctypes.c_void_p), ("row_base", ctypes.c_void_p),
                ("row_word", ctypes.c_void_p), ("row_width", ctypes.c_void_p), ("words", ctypes.c_void_p),
                ("values", ctypes.c_void_p), ("x", ctypes.c_void_p), ("y", ctypes.c_void_p)]


def _sig(name, restype, *argtypes):
    function = getattr(_lib, name)
    function.restype = restype
    function.argtypes = list(argtypes)
    return function


_v = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_d = ctypes.c_double
_s = ctypes.c_char_p
_sz = ctypes.c_size_t

_sig("spmv_version", _s)
_sig("spmv_status_string", _s, _i)
_sig("spmv_last_error", _s)
_sig("spmv_csr_read_matrix_market", _i, _s, _c_void_pp)
_sig("spmv_csr_create", _i, _i, _i, _v, _v, _v, _s, _c_void_pp)
_sig("spmv_csr_get_info", _i, _v, ctypes.POINTER(CsrInfo))
_sig("spmv_csr_get_arrays", _i, _v, _c_void_pp, _c_void_pp, _c_void_pp)
_sig("spmv_csr_name", _s, _v)
_sig("spmv_csr_set_name", _i, _v, _s)
_sig("spmv_csr_destroy", None, _v)
_sig("spmv_csr_slice_rows", _i, _v, _i, _i, _c_void_pp)
_sig("spmv_rcm_order", _i, _v, _v)
_sig("spmv_csr_permute", _i, _v, _v, _c_void_pp)
_sig("spmv_permutation_path", _i, _s, _s, _v, _sz)
_sig("spmv_permutation_write", _i, _s, _v, _i64, _d)
_sig("spmv_permutation_read", _i, _s, _i, _v, ctypes.POINTER(_d), _c_int_p)
_sig("spmv_csr_reorder_rcm", _i, _s, _v, _c_void_pp, ctypes.POINTER(_d))
_sig("spmv_characterize", _i, _v, _s, _d, _v, _sz, ctypes.POINTER(_sz))
_sig("spmv_characterize_device", _i, _v, _s, _d, _i, _v, _sz, ctypes.POINTER(_sz))
_sig("spmv_matrix_facts", _i, _v, ctypes.POINTER(Facts))
_sig("spmv_admissible", _i, _v, ctypes.POINTER(Facts), _i, _i, _c_int_p)
_sig("spmv_memory_of", _i, _v, ctypes.POINTER(Facts), _i, _i, _i, ctypes.POINTER(MemoryBreakdown))
_sig("spmv_encode_absolute", _i, _v, _i, _v)
_sig("spmv_encode_row_base", _i, _v, _v)
_sig("spmv_encode_relative", _i, _v, _i, _v)
_sig("spmv_lane_packed_word_count", _i, _v, _i, ctypes.POINTER(_i64))
_sig("spmv_encode_lane_packed", _i, _v, _i, _i64, _v, _v, _v)
_sig("spmv_encode_lane_packed_device", _i, _v, _v, _i, _i, _v, _v, _v, _i64, ctypes.POINTER(_i64), _v)
_sig("spmv_encode_lane_packed_device_noalloc", _i, _v, _v, _i, _i, _v, _v, _v, _i64, ctypes.POINTER(_i64), _v)
_sig("spmv_operator_config_init", None, ctypes.POINTER(OperatorConfig), _i, _i, _i)
_sig("spmv_operator_create", _i, _v, ctypes.POINTER(OperatorConfig), _c_void_pp)
_sig("spmv_operator_get_info", _i, _v, ctypes.POINTER(OperatorInfo))
_sig("spmv_operator_run", _i, _v, _v, _v, _v)
_sig("spmv_operator_run_host", _i, _v, _v, _v, _v, _v, _v)
_sig("spmv_operator_run_host_batch", _i, _v, _v, _i64, _v, _i64, _i, _v, _v, _v)
_sig("spmv_operator_check", _i, _v)
_sig("spmv_operator_get_arrays", _i, _v, ctypes.POINTER(OperatorArrays))
_sig("spmv_operator_destroy", None, _v)
_sig("spmv_launch", _i, _i, _i, _i, ctypes.POINTER(DeviceMatrix), _v)
_sig("spmv_launch_r16_control", _i, _i, _i, _i, ctypes.POINTER(DeviceMatrix), _v)
_sig("spmv_encode_relative_lane", _i, _v, _i, _v)
_sig("spmv_synth_laplacian2d", _i, _i, _c_void_pp)
_sig("spmv_synth_random_band", _i, _i, _i, _d, _u64, _c_void_pp)
_sig("spmv_synth_stencil27", _i, _i, _c_void_pp)
_sig("spmv_synth_power_law", _i, _i, _d, _i, _d, _u64, _c_void_pp)
_sig("spmv_synth_block_fem", _i, _i, _i, _i, _i, _u64, _i, _i, _c_void_pp)
_sig("spmv_fill_uniform", _i, _i, _i64, _u64, _v)
_sig("spmv_fill_reference_x", _i, _i, _i64, _v)
_sig("spmv_shard_rows", _i, _v, _i, _v)
_sig("spmv_read_bandwidth", _i, _i64, _i, ctypes.POINTER(_d))
_sig("spmv_gather_rate", _i, _i64, _i, _i, ctypes.POINTER(_d))
_sig("spmv_comm_unique_id", _i, _v)
_sig("spmv_comm_create", _i, _i, _i, _v, _i, _c_void_pp)
_sig("spmv_comm_destroy", None, _v)
_sig("spmv_comm_check", _i, _v, _v, _i)
_sig("spmv_chain_run", _i, _v, _v, _v, _v, _v, _i, _v)
_sig("spmv_chain_run_blocks", _i, _v, _i, _i, _v, _v, _v, _i, _v)
_sig("spmv_shard_run_host_batch", _i, _v, _v, _v, _i64, _v, _i64, _i, _v, _v, _v)
_sig("spmv_peer_group_create", _i, _i, _i, _i64, _i, _c_void_pp)
_sig("spmv_peer_group_handle", _i, _v, _v)
_sig("spmv_peer_group_open", _i, _v, _v)
_sig("spmv_peer_group_x", _i, _v, _i, _c_void_pp)
_sig("spmv_peer_group_barrier", _i, _v, _i, _v)
_sig("spmv_peer_group_copy_x", _i, _v, _i, _v, _i64, _v)
_sig("spmv_peer_group_check", _i, _v)
_sig("spmv_chain_run_peer", _i, _v, _v, _v, _i, _i, _v)
_sig("spmv_peer_group_set_halo", _i, _v, _v, _v)
_sig("spmv_peer_group_halo_entries", _i, _v, ctypes.POINTER(_i64))
_sig("spmv_peer_group_destroy", None, _v)


def _check(status: int):
    if status != OK:
        message = _lib.spmv_last_error().decode(errors="replace")
        raise SpmvError(status, f"{_lib.spmv_status_string(status).decode()}: {message}")


def version() -> str:
    return _lib.spmv_version().decode()


def _pointer(array: np.ndarray) -> int:
    return array.ctypes.data


# ---------------------------------------------------------------------------------------------------
# CsrMatrix (include/csr.hpp:33)
# ---------------------------------------------------------------------------------------------------
class CsrMatrix:
    """A host CSR matrix held by the library: int32 row pointer and columns, FP64 values, columns sorted
    within rows (the CsrMatrix of include/csr.hpp)."""

    def __init__(self, handle: int):
        if not handle:
            raise SpmvError(ERR_INVALID_ARGUMENT, "null matrix handle")
        self._handle = ctypes.c_void_p(handle)

    @classmethod
    def from_arrays(cls, rows: int, cols: int, row_ptr, col_ind, values=None, name: Optional[str] = None):
        row_ptr = np.ascontiguousarray(row_ptr, dtype=np.int32)
        col_ind = np.ascontiguousarray(col_ind, dtype=np.int32)
        values_array = None if values is None else np.ascontiguousarray(values, dtype=np.float64)
        handle = ctypes.c_void_p()
        _check(_lib.spmv_csr_create(rows, cols, _pointer(row_ptr), _pointer(col_ind) if col_ind.size else None,
                                    _pointer(values_array) if values_array is not None and values_array.size else None,
                                    name.encode() if name else None, ctypes.byref(handle)))
        return cls(handle.value)

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if _lib is not None and handle is not None and handle.value:   # _lib may be gone at interpreter exit
            _lib.spmv_csr_destroy(handle)
            self._handle = None

    @property
    def handle(self):
        return self._handle

    def info(self) -> CsrInfo:
        info = CsrInfo()
        _check(_lib.spmv_csr_get_info(self._handle, ctypes.byref(info)))
        return info

    @property
    def rows(self) -> int:
        return self.info().rows

    @property
    def cols(self) -> int:
        return self.info().cols

    @property
    def nnz(self) -> int:
        return self.info().nnz

    @property
    def name(self) -> str:
        return _lib.spmv_csr_name(self._handle).decode()

    @name.setter
    def name(self, value: str):
        _check(_lib.spmv_csr_set_name(self._handle, value.encode()))

    def arrays(self, copy: bool = True):
        """(row_ptr int32[rows+1], col_ind int32[nnz], values float64[nnz]) as numpy arrays."""
        info = self.info()
        row_ptr, col_ind, values = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        _check(_lib.spmv_csr_get_arrays(self._handle, ctypes.byref(row_ptr), ctypes.byref(col_ind), ctypes.byref(values)))

        def view(pointer, count, ctype, dtype):
            if count == 0:
                return np.zeros(0, dtype=dtype)
            array = np.ctypeslib.as_array(ctypes.cast(pointer, ctypes.POINTER(ctype)), shape=(count,))
            return array.copy() if copy else array

        return (view(row_ptr, info.rows + 1, ctypes.c_int32, np.int32),
                view(col_ind, info.nnz, ctypes.c_int32, np.int32),
                view(values, info.nnz, ctypes.c_double, np.float64))

    def slice_rows(self, row_begin: int, row_end: int) -> "CsrMatrix":
        handle = ctypes.c_void_p()
        _check(_lib.spmv_csr_slice_rows(self._handle, row_begin, row_end, ctypes.byref(handle)))
        return CsrMatrix(handle.value)


def read_matrix_market(path: str) -> CsrMatrix:
    """read_matrix_market (include/csr.hpp:232)."""
    handle = ctypes.c_void_p()
    _check(_lib.spmv_csr_read_matrix_market(os.fsencode(path), ctypes.byref(handle)))
    return CsrMatrix(handle.value)


# ---------------------------------------------------------------------------------------------------
# RCM (include/rcm.hpp)
# ---------------------------------------------------------------------------------------------------
def reverse_cuthill_mckee(matrix: CsrMatrix) -> np.ndarray:
    """reverse_cuthill_mckee (rcm.hpp:199): new_to_old."""
    order = np.zeros(matrix.rows, dtype=np.int32)
    _check(_lib.spmv_rcm_order(matrix.handle, _pointer(order)))
    return order


def apply_symmetric_permutation(matrix: CsrMatrix, new_to_old) -> CsrMatrix:
    """apply_symmetric_permutation (rcm.hpp:219): P A P^T."""
    order = np.ascontiguousarray(new_to_old, dtype=np.int32)
    if order.size != matrix.rows:
        raise SpmvError(ERR_INVALID_ARGUMENT, "permutation size does not match the matrix")
    handle = ctypes.c_void_p()
    _check(_lib.spmv_csr_permute(matrix.handle, _pointer(order), ctypes.byref(handle)))
    return CsrMatrix(handle.value)


def permutation_path_for(matrix_path: str, ordering: str = "rcm") -> str:
    buffer = ctypes.create_string_buffer(len(os.fsencode(matrix_path)) + len(ordering) + 16)
    _check(_lib.spmv_permutation_path(os.fsencode(matrix_path), ordering.encode(), buffer, len(buffer)))
    return buffer.value.decode()


def write_permutation(path: str, new_to_old, seconds: float):
    order = np.ascontiguousarray(new_to_old, dtype=np.int32)
    _check(_lib.spmv_permutation_write(os.fsencode(path), _pointer(order), order.size, seconds))


def read_permutation(path: str, expected_rows: int):
    """(new_to_old, seconds), or None when the file does not exist; raises on an invalid file."""
    order = np.zeros(expected_rows, dtype=np.int32)
    seconds = ctypes.c_double()
    found = ctypes.c_int()
    _check(_lib.spmv_permutation_read(os.fsencode(path), expected_rows, _pointer(order), ctypes.byref(seconds),
                                      ctypes.byref(found)))
    return (order, seconds.value) if found.value else None


def reorder_with_rcm(matrix_path: str, matrix: CsrMatrix):
    """reorder_with_rcm (rcm.hpp:306): (P A P^T, seconds the ordering took when computed)."""
    handle = ctypes.c_void_p()
    seconds = ctypes.c_double()
    _check(_lib.spmv_csr_reorder_rcm(os.fsencode(matrix_path), matrix.handle, ctypes.byref(handle), ctypes.byref(seconds)))
    return CsrMatrix(handle.value), seconds.value


def characterize_device(matrix: CsrMatrix, ordering: str = "original", ordering_seconds: float = 0.0,
                        device: int = -1) -> str:
    """characterize() computed on the GPU (the FIFO gather model on host threads beside it); the same text."""
    capacity = ctypes.c_size_t(8192 + 2 * len(matrix.name.encode()))
    buffer = ctypes.create_string_buffer(capacity.value)
    _check(_lib.spmv_characterize_device(matrix.handle, ordering.encode(), ordering_seconds, device, buffer,
                                         capacity.value, None))
    return buffer.value.decode()


def characterize(matrix: CsrMatrix, ordering: str = "original", ordering_seconds: float = 0.0) -> str:
    """The header and value line of src/characterize_matrix.cpp:253 (write_csv)."""
    needed = ctypes.c_size_t()
    status = _lib.spmv_characterize(matrix.handle, ordering.encode(), ordering_seconds, None, 0, ctypes.byref(needed))
    if status not in (OK, ERR_TOO_LARGE):
        _check(status)
    buffer = ctypes.create_string_buffer(needed.value)
    _check(_lib.spmv_characterize(matrix.handle, ordering.encode(), ordering_seconds, buffer, needed.value, None))
    return buffer.value.decode()


# ---------------------------------------------------------------------------------------------------
# Configurations, admissibility and byte model (bench_csr_width.cu:88, :223-276)
# ---------------------------------------------------------------------------------------------------
@dataclass
class Configuration:
    """Configuration (bench_csr_width.cu:88): value_bytes 8/4/2, column_bytes 4/2/1 (0 for lane-packed),
    column_mode "absolute" | "row-base" | "lane-packed", fixed_tpr (lane-packed: the T it was built for)."""
    value_bytes: int = 8
    column_bytes: int = 4
    column_mode: str = "absolute"
    fixed_tpr: int = 0

    @property
    def layout(self) -> int:
        if self.column_mode == "lane-packed":
            return LP
        if self.column_mode == "row-base":
            return {2: R16, 1: R8}[self.column_bytes]
        return {4: I32, 2: I16, 1: I8}[self.column_bytes]

    @property
    def dtype(self) -> int:
        return {8: F64, 4: F32, 2: F16}[self.value_bytes]

    @classmethod
    def of(cls, layout: int, dtype: int, tpr: int = 0) -> "Configuration":
        mode = "lane-packed" if layout == LP else ("row-base" if layout in (R16, R8) else "absolute")
        column_bytes = {I32: 4, I16: 2, I8: 1, R16: 2, R8: 1, LP: 0}[layout]
        return cls(VALUE_BYTES[dtype], column_bytes, mode, tpr if layout == LP else 0)


def facts_of(matrix: CsrMatrix) -> Facts:
    facts = Facts()
    _check(_lib.spmv_matrix_facts(matrix.handle, ctypes.byref(facts)))
    return facts


def configuration_admissible(matrix: CsrMatrix, facts: Optional[Facts], configuration: Configuration) -> bool:
    result = ctypes.c_int()
    _check(_lib.spmv_admissible(matrix.handle, ctypes.byref(facts) if facts is not None else None,
                                configuration.layout, configuration.fixed_tpr, ctypes.byref(result)))
    return bool(result.value)


def memory_of(matrix: CsrMatrix, facts: Optional[Facts], configuration: Configuration) -> MemoryBreakdown:
    memory = MemoryBreakdown()
    _check(_lib.spmv_memory_of(matrix.handle, ctypes.byref(facts) if facts is not None else None,
                               configuration.layout, configuration.dtype, configuration.fixed_tpr, ctypes.byref(memory)))
    return memory


def encode_absolute(matrix: CsrMatrix, column_bytes: int) -> np.ndarray:
    """upload_columns<T, I> (bench_csr_width.cu:796) on the host."""
    out = np.zeros(matrix.nnz, dtype=np.uint16 if column_bytes == 2 else np.uint8)
    _check(_lib.spmv_encode_absolute(matrix.handle, column_bytes, _pointer(out) if out.size else _pointer(np.zeros(1, out.dtype))))
    return out


def encode_row_base(matrix: CsrMatrix) -> np.ndarray:
    """upload_row_bases (bench_csr_width.cu:807) on the host."""
    out = np.zeros(max(matrix.rows, 1), dtype=np.int32)
    _check(_lib.spmv_encode_row_base(matrix.handle, _pointer(out)))
    return out[:matrix.rows]


def encode_relative(matrix: CsrMatrix, column_bytes: int) -> np.ndarray:
    """upload_relative_columns<I> (bench_csr_width.cu:820) on the host; column_bytes 4 gives the 32-bit
    offsets of the SPMV_R16_WIDE control build."""
    dtype = {4: np.uint32, 2: np.uint16}.get(column_bytes, np.uint8)
    out = np.zeros(max(matrix.nnz, 1), dtype=dtype)
    _check(_lib.spmv_encode_relative(matrix.handle, column_bytes, _pointer(out)))
    return out[:matrix.nnz]


def encode_relative_lane(matrix: CsrMatrix, tpr: int) -> np.ndarray:
    """upload_lane_major_offsets (bench_csr_width.cu:838): the 16-bit offsets of every row in lane-major order
    for tpr, (nnz + 1) // 2 * 2 entries (the SPMV_R16_LANE / SPMV_R16_PAIR control builds)."""
    out = np.zeros(max((matrix.nnz + 1) // 2 * 2, 2), dtype=np.uint16)
    _check(_lib.spmv_encode_relative_lane(matrix.handle, tpr, _pointer(out)))
    return out[:(matrix.nnz + 1) // 2 * 2]


def packed_word_count(matrix: CsrMatrix, tpr: int) -> int:
    """packed_word_count (bench_csr_width.cu:206)."""
    count = ctypes.c_int64()
    _check(_lib.spmv_lane_packed_word_count(matrix.handle, tpr, ctypes.byref(count)))
    return count.value


def build_packed_deltas(matrix: CsrMatrix, tpr: int, word_count: Optional[int] = None):
    """build_packed_deltas (bench_csr_width.cu:861): (row_word int32, row_width uint8, words uint32)."""
    if word_count is None:
        word_count = packed_word_count(matrix, tpr)
    rows = matrix.rows
    row_word = np.zeros(max(rows, 1), dtype=np.int32)
    row_width = np.zeros(max(rows, 1), dtype=np.uint8)
    words = np.zeros(word_count, dtype=np.uint32)
    _check(_lib.spmv_encode_lane_packed(matrix.handle, tpr, word_count, _pointer(row_word), _pointer(row_width),
                                        _pointer(words)))
    return row_word[:rows], row_width[:rows], words


def build_packed_deltas_device(row_ptr: int, col_ind: int, rows: int, tpr: int, row_word: int, row_width: int,
                               words: int = 0, word_capacity: int = 0, stream: int = 0) -> int:
    """build_packed_deltas on the GPU from device pointers (row_ptr int32[rows+1], col_ind int32[nnz]) into
    device row_word int32[rows] and row_width uint8[rows], and words uint32 when given; returns the word
    count (2 spare words included)."""
    count = ctypes.c_int64()
    _check(_lib.spmv_encode_lane_packed_device(row_ptr, col_ind, rows, tpr, row_word, row_width, words or None,
                                               word_capacity, ctypes.byref(count), stream or None))
    return count.value


def build_packed_deltas_device_noalloc(row_ptr: int, col_ind: int, rows: int, tpr: int, row_word: int, row_width: int,
                                       words: int = 0, word_capacity: int = 0, stream: int = 0) -> int:
    """build_packed_deltas_device without allocating device memory (a fixed scratch array inside the
    library; at most 2^26 rows; calls that overlap on the GPU race on that array)."""
    count = ctypes.c_int64()
    _check(_lib.spmv_encode_lane_packed_device_noalloc(row_ptr, col_ind, rows, tpr, row_word, row_width, words or None,
                                                       word_capacity, ctypes.byref(count), stream or None))
    return count.value


# ---------------------------------------------------------------------------------------------------
# Synthetic inputs
# ---------------------------------------------------------------------------------------------------
def _synth(function, *args) -> CsrMatrix:
    handle = ctypes.c_void_p()
    _check(function(*args, ctypes.byref(handle)))
    return CsrMatrix(handle.value)


def synth_laplacian2d(grid: int) -> CsrMatrix:
    return _synth(_lib.spmv_synth_laplacian2d, grid)


def synth_random_band(n: int, half_bandwidth: int, mean: float, seed: int) -> CsrMatrix:
    return _synth(_lib.spmv_synth_random_band, n, half_bandwidth, mean, seed)


def synth_stencil27(grid: int) -> CsrMatrix:
    return _synth(_lib.spmv_synth_stencil27, grid)


def synth_power_law(n: int, alpha: float, max_length: int, mean: float, seed: int) -> CsrMatrix:
    return _synth(_lib.spmv_synth_power_law, n, alpha, max_length, mean, seed)


def synth_block_fem(n: int, block: int, blocks_per_row: int, offset_range: int, seed: int,
                    row_begin: int = 0, row_end: Optional[int] = None) -> CsrMatrix:
    return _synth(_lib.spmv_synth_block_fem, n, block, blocks_per_row, offset_range, seed, row_begin,
                  n if row_end is None else row_end)


def fill_uniform(dtype: int, count: int, seed: int) -> np.ndarray:
    out = np.zeros(max(count, 1), dtype=NUMPY_DTYPES[dtype])
    _check(_lib.spmv_fill_uniform(dtype, count, seed, _pointer(out)))
    return out[:count]


def fill_reference_x(dtype: int, count: int) -> np.ndarray:
    """The x of upload_matrix (bench_csr_width.cu:923-928): mt19937(7), uniform(-1, 1), through float."""
    out = np.zeros(max(count, 1), dtype=NUMPY_DTYPES[dtype])
    _check(_lib.spmv_fill_reference_x(dtype, count, _pointer(out)))
    return out[:count]


def convert_values(values: np.ndarray, dtype: int) -> np.ndarray:
    """(T)(float)val, the device values of upload_matrix (bench_csr_width.cu:927)."""
    return np.asarray(values, dtype=np.float64).astype(np.float32).astype(NUMPY_DTYPES[dtype])


def shard_rows(matrix: CsrMatrix, nshards: int) -> np.ndarray:
    """Row boundaries of nshards row blocks balanced by nonzeros (nshards + 1 entries)."""
    bounds = np.zeros(nshards + 1, dtype=np.int32)
    _check(_lib.spmv_shard_rows(matrix.handle, nshards, _pointer(bounds)))
    return bounds


# ---------------------------------------------------------------------------------------------------
# Device operator: DeviceMatrix<T> + launch<T> (bench_csr_width.cu:128, :607)
# ---------------------------------------------------------------------------------------------------
class Operator:
    """A matrix encoded in one layout and uploaded to a GPU; run() is launch<T> at the operator's T."""

    def __init__(self, matrix: CsrMatrix, layout: int, dtype: int, tpr: int, physical_tpr: int = 0,
                 tile_nnz: int = 0, value_rounding: int = 0, device: int = -1, stages: int = 0, tile_rows: int = 0,
                 schedule: int = 0, accumulate: int = 0):
        config = OperatorConfig()
        _lib.spmv_operator_config_init(ctypes.byref(config), layout, dtype, tpr)
        config.physical_tpr = physical_tpr
        config.tile_nnz = tile_nnz
        config.value_rounding = value_rounding
        config.device = device
        config.stages = stages
        config.tile_rows = tile_rows
        config.schedule = schedule
        config.accumulate = accumulate
        handle = ctypes.c_void_p()
        _check(_lib.spmv_operator_create(matrix.handle, ctypes.byref(config), ctypes.byref(handle)))
        self._handle = handle
        self.layout, self.dtype, self.tpr = layout, dtype, tpr
        info = self.info()
        self.rows, self.cols, self.nnz = info.rows, info.cols, info.nnz

    def close(self):
        if getattr(self, "_handle", None) is not None and self._handle.value:
            _lib.spmv_operator_destroy(self._handle)
            self._handle = None

    def __del__(self):
        if _lib is not None:   # at interpreter exit the module's globals may already be gone
            self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self):
        return self._handle

    def info(self) -> OperatorInfo:
        info = OperatorInfo()
        _check(_lib.spmv_operator_get_info(self._handle, ctypes.byref(info)))
        return info

    def arrays(self) -> OperatorArrays:
        arrays = OperatorArrays()
        _check(_lib.spmv_operator_get_arrays(self._handle, ctypes.byref(arrays)))
        return arrays

    def run(self, x_ptr: int, y_ptr: int, stream: int = 0):
        """y = A x on a CUDA stream (device pointers as integers, e.g. torch tensor.data_ptr())."""
        _check(_lib.spmv_operator_run(self._handle, x_ptr, y_ptr, stream or None))

    def run_host(self, x_host, y_host, x_device: int, y_device: int, stream: int = 0):
        """Copies x in, multiplies, copies y out and waits (result_at_fixed_tpr, bench_csr_width.cu:779).
        x_host / y_host are numpy arrays or host pointers (e.g. of pinned torch tensors)."""
        host = lambda array: array if isinstance(array, int) else _pointer(array)  # noqa: E731
        _check(_lib.spmv_operator_run_host(self._handle, host(x_host), host(y_host), x_device, y_device,
                                           stream or None))

    def run_host_batch(self, x_host, x_stride: int, y_host, y_stride: int, count: int, x_device: int, y_device: int,
                       stream: int = 0):
        """count products through host buffers with the copies in, the products and the copies out overlapped;
        x_device / y_device hold two vectors each (the second 16-byte aligned after the first)."""
        host = lambda array: array if isinstance(array, int) else _pointer(array)  # noqa: E731
        _check(_lib.spmv_operator_run_host_batch(self._handle, host(x_host), x_stride, host(y_host), y_stride, count,
                                                 x_device, y_device, stream or None))

    def check(self):
        """Raises SpmvError(ERR_TIMEOUT) if a bounded device-side wait gave up since the last check."""
        _check(_lib.spmv_operator_check(self._handle))


def read_bandwidth(bytes_: int = 4 << 30, reps: int = 20) -> float:
    """Measured streaming read bandwidth of the current device in GB/s (measure_read_bandwidth,
    roofline.cuh:101)."""
    result = ctypes.c_double()
    _check(_lib.spmv_read_bandwidth(bytes_, reps, ctypes.byref(result)))
    return result.value


def gather_rate(elements: int, value_bytes: int, reps: int = 10) -> float:
    """Measured rate (elements/s) of random single-element reads from an array of `elements` elements of
    value_bytes each: the ceiling of the x gathers of a matrix with scattered columns."""
    result = ctypes.c_double()
    _check(_lib.spmv_gather_rate(elements, value_bytes, reps, ctypes.byref(result)))
    return result.value


def launch(layout: int, dtype: int, tpr: int, device_matrix: DeviceMatrix, stream: int = 0):
    """launch<T> (bench_csr_width.cu:607) on caller-owned device arrays (no preprocessing)."""
    _check(_lib.spmv_launch(layout, dtype, tpr, ctypes.byref(device_matrix), stream or None))


R16_CONTROL_LANE, R16_CONTROL_PAIR, R16_CONTROL_WIDE, R16_CONTROL_UNROLL16 = 1, 2, 3, 4
R16_CONTROLS = {"lane": R16_CONTROL_LANE, "pair": R16_CONTROL_PAIR, "wide": R16_CONTROL_WIDE,
                "unroll16": R16_CONTROL_UNROLL16}


def launch_r16_control(control: int, dtype: int, tpr: int, device_matrix: DeviceMatrix, stream: int = 0):
    """A control build of the reference's CSR-r16 kernel (bench_csr_width.cu:34-42) on caller arrays:
    device_matrix.columns is the lane-major stream (LANE, PAIR), the 32-bit offsets (WIDE) or the 16-bit
    offsets (UNROLL16)."""
    _check(_lib.spmv_launch_r16_control(control, dtype, tpr, ctypes.byref(device_matrix), stream or None))


# ---------------------------------------------------------------------------------------------------
# Multi-GPU: NCCL communicator and chained products over row shards
# ---------------------------------------------------------------------------------------------------
def comm_unique_id() -> bytes:
    """The 128-byte NCCL id rank 0 creates and the other ranks receive (e.g. by torch.distributed)."""
    buffer = ctypes.create_string_buffer(128)
    _check(_lib.spmv_comm_unique_id(buffer))
    return buffer.raw


class Comm:
    """An NCCL communicator of one rank (one process per GPU)."""

    def __init__(self, nranks: int, rank: int, unique_id: bytes, device: int = -1):
        handle = ctypes.c_void_p()
        _check(_lib.spmv_comm_create(nranks, rank, ctypes.create_string_buffer(unique_id, 128), device,
                                     ctypes.byref(handle)))
        self._handle = handle
        self.nranks, self.rank = nranks, rank

    @property
    def handle(self):
        return self._handle

    def check(self, stream: int = 0, timeout_ms: int = 30000):
        _check(_lib.spmv_comm_check(self._handle, stream or None, timeout_ms))

    def close(self):
        if getattr(self, "_handle", None) is not None and self._handle.value:
            _lib.spmv_comm_destroy(self._handle)
            self._handle = None

    def __del__(self):
        if _lib is not None:   # at interpreter exit the module's globals may already be gone
            self.close()


def chain_run(shard_op: "Operator", comm: Comm, shard_row_begin, x_current: int, x_next: int, products: int,
              stream: int = 0):
    """products chained y -> x: each rank's shard product into its slice of the next x, then the slices
    all-gathered. The result is in x_current for an even count of products, in x_next for an odd one."""
    bounds = np.ascontiguousarray(shard_row_begin, dtype=np.int32)
    _check(_lib.spmv_chain_run(shard_op.handle, comm.handle, _pointer(bounds), x_current, x_next, products,
                               stream or None))


def shard_run_host_batch(shard_op: "Operator", comm: Comm, x_host: int, x_stride: int, y_host: int, y_stride: int,
                         count: int, x_device: int, y_device: int, stream: int = 0):
    """count products of this rank's shard from host memory: each rank copies its 1/nranks slice of every
    x in, the slices are all-gathered over NCCL, the product runs and the shard's rows of y go out.
    x_device holds two buffers of nranks * ceil(cols / nranks) entries (each rounded up to 16 bytes),
    y_device two of the shard's rows."""
    _check(_lib.spmv_shard_run_host_batch(shard_op.handle, comm.handle, x_host, x_stride, y_host, y_stride, count,
                                          x_device, y_device, stream or None))


def chain_run_blocks(block_ops: Sequence["Operator"], block_rows: int, comm: Comm, x_current: int, x_next: int,
                     products: int, stream: int = 0):
    """products chained y -> x over interleaved row blocks: block_ops[c] holds rows of block
    c * nranks + rank (block_rows rows, all n columns); each round's all-gather runs beside the next
    block's product. Results, and where they are left, as chain_run's."""
    handles = (ctypes.c_void_p * len(block_ops))(*[op.handle.value for op in block_ops])
    _check(_lib.spmv_chain_run_blocks(handles, len(block_ops), block_rows, comm.handle, x_current, x_next, products,
                                      stream or None))


class PeerGroup:
    """One rank's share of chained products over peer memory: two x buffers and barrier flags, mapped by
    every other rank (CUDA IPC), so that each product stores its rows straight into every rank's next x."""

    HANDLE_BYTES = 64

    def __init__(self, nranks: int, rank: int, x_bytes: int, device: int = -1):
        handle = ctypes.c_void_p()
        _check(_lib.spmv_peer_group_create(nranks, rank, x_bytes, device, ctypes.byref(handle)))
        self._handle = handle
        self.nranks, self.rank = nranks, rank

    @property
    def handle(self):
        return self._handle

    def export(self) -> bytes:
        """This rank's allocation handle, to be gathered by every rank in rank order."""
        out = ctypes.create_string_buffer(self.HANDLE_BYTES)
        _check(_lib.spmv_peer_group_handle(self._handle, out))
        return out.raw

    def open(self, handles: Sequence[bytes]):
        blob = b"".join(handles)
        if len(blob) != self.HANDLE_BYTES * self.nranks:
            raise ValueError("one handle per rank is required")
        _check(_lib.spmv_peer_group_open(self._handle, ctypes.create_string_buffer(blob, len(blob))))

    def x(self, which: int = 0) -> int:
        """Device pointer of the current x (which=0) or of the other buffer (which=1)."""
        pointer = ctypes.c_void_p()
        _check(_lib.spmv_peer_group_x(self._handle, which, ctypes.byref(pointer)))
        return pointer.value

    def write_x(self, pointer: int, nbytes: int, stream: int = 0):
        """Copies nbytes from pointer (host or device memory) into this rank's current x."""
        _check(_lib.spmv_peer_group_copy_x(self._handle, 0, pointer, nbytes, stream or None))

    def read_x(self, pointer: int, nbytes: int, stream: int = 0):
        """Copies nbytes of this rank's current x to pointer (host or device memory)."""
        _check(_lib.spmv_peer_group_copy_x(self._handle, 1, pointer, nbytes, stream or None))

    def set_halo(self, shard: "CsrMatrix", shard_row_begin):
        """Halo mode for this rank's row shard: each chained product pulls only the entries of x that other
        ranks own and these rows read. Returns the number of entries pulled per product."""
        bounds = np.ascontiguousarray(shard_row_begin, dtype=np.int32)
        _check(_lib.spmv_peer_group_set_halo(self._handle, shard.handle, _pointer(bounds)))
        count = ctypes.c_int64()
        _check(_lib.spmv_peer_group_halo_entries(self._handle, ctypes.byref(count)))
        return count.value

    def barrier(self, timeout_ms: int = 5000, stream: int = 0):
        _check(_lib.spmv_peer_group_barrier(self._handle, timeout_ms, stream or None))

    def check(self):
        _check(_lib.spmv_peer_group_check(self._handle))

    def close(self):
        if getattr(self, "_handle", None) is not None and self._handle.value:
            _lib.spmv_peer_group_destroy(self._handle)
            self._handle = None

    def __del__(self):
        if _lib is not None:   # at interpreter exit the module's globals may already be gone
            self.close()


def chain_run_peer(shard_op: "Operator", group: PeerGroup, shard_row_begin, products: int, stream: int = 0,
                   timeout_ms: int = 5000):
    """products chained y -> x over the row shards, each product storing its rows into every rank's next x
    over peer memory, then a barrier of the ranks' GPUs. The result is the group's current x."""
    bounds = np.ascontiguousarray(shard_row_begin, dtype=np.int32)
    _check(_lib.spmv_chain_run_peer(shard_op.handle, group.handle, _pointer(bounds), products, timeout_ms,
                                    stream or None))


def interleaved_block_rows(row_ptr, col_ind, values, nranks: int, blocks_per_rank: int, rank: int):
    """The CSR arrays (row_ptr, col_ind, values) of each of rank's interleaved row blocks, in the order
    chain_run_blocks takes them: block c * nranks + rank for c = 0 .. blocks_per_rank - 1. The rows must
    divide into nranks * blocks_per_rank blocks of equal size."""
    row_ptr = np.asarray(row_ptr, dtype=np.int64)
    rows = row_ptr.size - 1
    blocks = nranks * blocks_per_rank
    if rows % blocks:
        raise ValueError(f"{rows} rows do not divide into {blocks} equal blocks")
    block_rows = rows // blocks
    out = []
    for c in range(blocks_per_rank):
        first = (c * nranks + rank) * block_rows
        begin, end = int(row_ptr[first]), int(row_ptr[first + block_rows])
        out.append(((row_ptr[first:first + block_rows + 1] - begin).astype(np.int32), col_ind[begin:end],
                    values[begin:end]))
    return out


def exported_symbols() -> Sequence[str]:
    """Names of every spmv_* entry point the header declares that the loaded library exports."""
    header = os.path.join(_HERE, "..", "..", "include", "spmvb200.h")
    import re
    names = re.findall(r"\b(spmv_[a-z0-9_]+)\s*\(", open(header).read())
    return [name for name in dict.fromkeys(names) if hasattr(_lib, name)]
