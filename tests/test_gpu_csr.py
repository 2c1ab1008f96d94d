"""Sparse rows emitted on the device (C ABI mdsoap_compute_csr) against the
representation OutputOptions(sparse=True) gives in the reference
(scipy.sparse.csr_matrix of the dense rows, src/mdescriptor/core/result.py:64-84):
identical row offsets, column indices and values to the GPU's own dense rows,
and the CPU checker's rows (oracle/) in CSR form: the same nonzero pattern
(structural zeros of absent species pairs are exact zeros in both) and values
within the float32 bound (float32 rows) or the two-implementation agreement
bound (float64 rows; float64 accuracy itself is tested against the exact
value in test_gpu_f64_reference.py), for batches whose environments miss some
species (zero blocks) and for every average."""

from __future__ import annotations

import numpy as np
import pytest
import scipy.sparse

from _util import AGREE_FLOOR, AGREE_TOL, assert_features_close, max_rel_err
from mdescriptor_b200 import workloads
from mdescriptor_b200.basis import basis_gto
from mdescriptor_b200.soap import Soap

pytestmark = pytest.mark.gpu


def sparse_batch(seed: int, structures: int = 9) -> workloads.Batch:
    """Isolated clusters drawing from a few of the species each, so many
    species-pair blocks of a row are exactly zero; one structure is empty."""
    rng = np.random.default_rng(seed)
    numbers, positions, offsets = [], [], [0]
    for s in range(structures):
        n = 0 if s == 4 else int(rng.integers(1, 24))
        pool = rng.choice([1, 6, 7, 8, 16], size=2, replace=False)
        numbers.append(rng.choice(pool, n).astype(np.int32))
        positions.append(rng.uniform(-4.0, 4.0, (n, 3)))
        offsets.append(offsets[-1] + n)
    return workloads.Batch(np.concatenate(numbers), np.concatenate(positions), np.zeros((structures, 3, 3)),
                           np.zeros((structures, 3), np.int32), np.array(offsets, np.int64))


@pytest.mark.parametrize("dtype", ["float32", "float64"])
@pytest.mark.parametrize("average", ["off", "inner", "outer"])
@pytest.mark.parametrize("n_max", [8, 4])
def test_csr_rows_match_dense_rows(oracle, cuda_device, dtype, average, n_max):
    species = (1, 6, 7, 8, 16)
    alphas, betas = basis_gto(4.0, n_max, 4)
    soap = Soap(species, r_cut=4.0, n_max=n_max, l_max=4, sigma=0.7, average=average, dtype=dtype,
                alphas=alphas, betas=betas)
    batch = sparse_batch(3 + n_max)
    dense = soap.compute(batch, devices=[0])
    want = scipy.sparse.csr_matrix(dense)
    got = soap.compute_csr(batch, device=0)
    assert got.shape == dense.shape and got.dtype == dense.dtype
    assert got.nnz == want.nnz < dense.size  # zero blocks were dropped
    np.testing.assert_array_equal(got.indptr, want.indptr)
    np.testing.assert_array_equal(got.indices, want.indices)
    np.testing.assert_array_equal(got.data, want.data)
    # A second call reuses the plan's device state.
    again = soap.compute_csr(batch, device=0)
    assert (again != got).nnz == 0
    # The checker's rows in CSR form: same nonzero pattern, values within tolerance.
    checker = scipy.sparse.csr_matrix(oracle.soap(batch, species, 4.0, n_max, 4, 0.7, alphas, betas, average))
    np.testing.assert_array_equal(got.indptr, checker.indptr)
    np.testing.assert_array_equal(got.indices, checker.indices)
    if dtype == "float32":
        assert_features_close(got.toarray(), checker.toarray(), "float32")
    else:
        assert max_rel_err(got.toarray(), checker.toarray(), AGREE_FLOOR) <= AGREE_TOL


def test_csr_empty_batch_and_periodic_rows(cuda_device):
    soap = Soap((1, 6, 7, 8), r_cut=5.0, n_max=8, l_max=6, sigma=1.0, average="off", dtype="float32")
    empty = workloads.Batch(np.zeros(0, np.int32), np.zeros((0, 3)), np.zeros((0, 3, 3)),
                            np.zeros((0, 3), np.int32), np.array([0], np.int64))
    got = soap.compute_csr(empty, device=0)
    assert got.shape == (0, soap.feature_count) and got.nnz == 0
    batch = workloads.config2(structures=3, seed=11)
    dense = soap.compute(batch, devices=[0])
    got = soap.compute_csr(batch, device=0)
    want = scipy.sparse.csr_matrix(dense)
    np.testing.assert_array_equal(got.indptr, want.indptr)
    np.testing.assert_array_equal(got.indices, want.indices)
    np.testing.assert_array_equal(got.data, want.data)
