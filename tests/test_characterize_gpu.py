"""Characterization on the GPU (spmv_characterize_device) against the host characterization, which the CPU
tests hold field for field to the reference's own tool (src/characterize_matrix.cpp) and its published
rows: the same CSV text, byte for byte, on the reference's smoke matrices in both orderings and on
synthetic matrices with empty rows, rows of 40,000+ entries, spans beyond 2^16 and the 27-point stencil."""
import numpy as np
import pytest

import spmvb200 as spmv
from conftest import random_csr

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_smoke_matrices_both_orderings(smoke_matrix_paths):
    for name, path in smoke_matrix_paths.items():
        matrix = spmv.read_matrix_market(path)
        assert spmv.characterize_device(matrix, "original") == spmv.characterize(matrix, "original"), name
        reordered = spmv.apply_symmetric_permutation(matrix, spmv.reverse_cuthill_mckee(matrix))
        reordered.name = matrix.name
        assert spmv.characterize_device(reordered, "rcm", 0.125) == spmv.characterize(reordered, "rcm", 0.125), name


def test_synthetic_matrices():
    ragged = spmv.CsrMatrix.from_arrays(4000, 4000, *random_csr(4000, 4000, lambda rng: rng.integers(0, 90), 12,
                                                                 empty_every=13, long_rows={3: 3900}), name="ragged")
    stencil = spmv.synth_stencil27(48)
    stencil = spmv.apply_symmetric_permutation(stencil, spmv.reverse_cuthill_mckee(stencil))
    stencil.name = "stencil27_48_rcm"
    for matrix in (ragged, spmv.synth_random_band(200_000, 90_000, 6.0, 2), stencil,
                   spmv.synth_power_law(400_000, 1.8, 40_000, 12.0, 5), spmv.synth_laplacian2d(64)):
        assert spmv.characterize_device(matrix) == spmv.characterize(matrix), matrix.name


def test_single_row_and_refusals():
    one = spmv.CsrMatrix.from_arrays(1, 1, np.array([0, 1], np.int32), np.array([0], np.int32), np.array([2.0]), name="one")
    assert spmv.characterize_device(one) == spmv.characterize(one)
    rectangular = spmv.CsrMatrix.from_arrays(2, 3, np.array([0, 1, 2], np.int32), np.array([0, 2], np.int32),
                                             np.array([1.0, 1.0]), name="rect")
    with pytest.raises(spmv.SpmvError):
        spmv.characterize_device(rectangular)
