"""The C ABI itself: the library loads, exports every entry point include/spmvb200.h declares, and reports
errors as statuses (no compute call needs a GPU here)."""
import ctypes
import re

import numpy as np
import pytest

import spmvb200 as spmv
from conftest import ROOT


def declared():
    header = open(f"{ROOT}/include/spmvb200.h").read()
    return sorted(set(re.findall(r"\b(spmv_[a-z0-9_]+)\s*\(", header)))


def test_every_declared_symbol_is_exported():
    names = declared()
    assert len(names) >= 40
    assert sorted(spmv.exported_symbols()) == names


def test_status_strings_and_last_error():
    assert spmv._lib.spmv_status_string(spmv.ERR_NOT_ADMISSIBLE) == b"not admissible"
    with pytest.raises(spmv.SpmvError) as failure:
        spmv.read_matrix_market("/does/not/exist.mtx")
    assert "cannot open" in str(failure.value)
    assert b"cannot open" in spmv._lib.spmv_last_error()


def test_bad_arguments_are_statuses_not_crashes():
    matrix = spmv.synth_laplacian2d(8)
    with pytest.raises(spmv.SpmvError) as failure:
        spmv.packed_word_count(matrix, 3)
    assert failure.value.status == spmv.ERR_INVALID_ARGUMENT
    memory = spmv.MemoryBreakdown()
    assert spmv._lib.spmv_memory_of(matrix.handle, None, spmv.I32, 7, 0, ctypes.byref(memory)) == spmv.ERR_INVALID_ARGUMENT
    with pytest.raises(spmv.SpmvError):
        spmv.apply_symmetric_permutation(matrix, np.zeros(64, np.int32))   # not a permutation
    assert spmv._lib.spmv_csr_get_info(None, None) == spmv.ERR_INVALID_ARGUMENT


def test_operator_without_device_fails_cleanly():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(spmv.SpmvError) as failure:
        spmv.Operator(spmv.synth_laplacian2d(8), spmv.I32, spmv.F64, 8)
    assert failure.value.status == spmv.ERR_UNSUPPORTED


def test_nccl_unique_id_without_gpu():
    assert len(spmv.comm_unique_id()) == 128
