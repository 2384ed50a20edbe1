"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on a CPU-only machine.

Matrices of the reference's smoke test (dawson5, rim) are read from tests/_data/ (copied there by
__graft_entry__.build() when the reference tree is present; git-ignored) or straight from the reference
tree; tests that need them skip when neither exists.
"""
import gzip
import os
import shutil
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "spmv-index-compression_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

# the reference tree, when the environment names one (SPMV_REFERENCE_ROOT); tests that need it skip otherwise
REFERENCE_ROOT = os.environ.get("SPMV_REFERENCE_ROOT", "")
DATA = os.path.join(ROOT, "tests", "_data")
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (the B200 box)")


def smoke_matrix_archive(name):
    candidates = [os.path.join(DATA, name + ".mtx.gz")]
    if REFERENCE_ROOT:
        candidates.append(os.path.join(REFERENCE_ROOT, "data", "smoke_matrices", name + ".mtx.gz"))
    for candidate in candidates:
        if os.path.exists(candidate):
            return candidate
    return None


@pytest.fixture(scope="session")
def smoke_matrix_paths(tmp_path_factory):
    """{'dawson5': path, 'rim': path} of the decompressed .mtx files."""
    directory = tmp_path_factory.mktemp("smoke_matrices")
    paths = {}
    for name in ("dawson5", "rim"):
        archive = smoke_matrix_archive(name)
        if archive is None:
            pytest.skip("smoke matrices (dawson5, rim) are not available")
        target = directory / (name + ".mtx")
        with gzip.open(archive, "rb") as source, open(target, "wb") as out:
            shutil.copyfileobj(source, out)
        paths[name] = str(target)
    return paths


@pytest.fixture(scope="session")
def reference():
    """The reference's own code compiled from its sources, or skip."""
    import oracle
    if not oracle.Reference.available():
        pytest.skip("oracle/_ref is not built (needs the reference sources)")
    return oracle.Reference()


def random_csr(rows, cols, density_or_lengths, seed, empty_every=0, long_rows=()):
    """A random CSR (row_ptr, col_ind, values) with sorted unique columns per row."""
    rng = np.random.default_rng(seed)
    lists = []
    for row in range(rows):
        if empty_every and row % empty_every == 0:
            lists.append(np.zeros(0, np.int64))
            continue
        if row in long_rows:
            length = min(cols, long_rows[row] if isinstance(long_rows, dict) else cols // 2)
        elif callable(density_or_lengths):
            length = min(cols, int(density_or_lengths(rng)))
        else:
            length = min(cols, int(rng.poisson(density_or_lengths)))
        lists.append(np.sort(rng.choice(cols, size=length, replace=False)))
    row_ptr = np.zeros(rows + 1, np.int32)
    row_ptr[1:] = np.cumsum([len(item) for item in lists])
    col_ind = np.concatenate(lists).astype(np.int32) if rows else np.zeros(0, np.int32)
    values = rng.standard_normal(col_ind.size)
    return row_ptr, col_ind, values
