"""Pins the CPU checker's compression layouts and radial weighting against the
reference's own compute_soap (oracle/_ref, compiled from the reference sources):
every compression mode, every weighting function and w0, species weights,
and the three averages, on small mixed periodic / isolated batches."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from _util import AGREE_FLOOR, AGREE_TOL, max_rel_err
from mdescriptor_b200 import workloads
from mdescriptor_b200.basis import basis_gto, feature_count, labels

REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libref_soap.so"
pytestmark = pytest.mark.skipif(not REF_LIB.is_file(), reason="reference library not built in this tree")

WEIGHTINGS = {
    "none": None,
    "poly": {"function": "poly", "r0": 4.2, "c": 1.3, "m": 2.0},
    "pow": {"function": "pow", "r0": 1.7, "c": 0.9, "d": 0.4, "m": 3.0},
    "exp": {"function": "exp", "r0": 1.1, "c": 2.0, "d": 0.25},
    "w0": {"w0": 0.35},
    "poly+w0": {"function": "poly", "r0": 5.5, "c": 1.0, "m": 1.5, "w0": 0.0},
}


def mixed_batch(seed: int) -> workloads.Batch:
    rng = np.random.default_rng(seed)
    numbers, positions, cells, pbc, offsets = [], [], [], [], [0]
    for s in range(4):
        n = int(rng.integers(2, 14))
        periodic = s != 2
        cell = np.diag(rng.uniform(4.0, 7.0, 3)) + np.triu(rng.uniform(-0.6, 0.6, (3, 3)), 1)
        frac = rng.uniform(-0.2, 1.2, (n, 3))
        positions.append(frac @ cell)
        numbers.append(rng.choice([1, 6, 8], n).astype(np.int32))
        cells.append(cell if periodic else np.zeros((3, 3)))
        pbc.append([1, 1, 1] if periodic else [0, 0, 0])
        offsets.append(offsets[-1] + n)
    return workloads.Batch(np.concatenate(numbers), np.concatenate(positions), np.array(cells),
                           np.array(pbc, np.int32), np.array(offsets, np.int64))


@pytest.mark.parametrize("compression", ["off", "mu2", "mu1nu1", "crossover"])
@pytest.mark.parametrize("weighting", sorted(WEIGHTINGS))
def test_checker_matches_reference_options(oracle, compression, weighting):
    from oracle import RefLib

    ref = RefLib()
    species, r_cut, n_max, l_max, sigma = (1, 6, 8), 3.6, 4, 3, 0.8
    alphas, betas = basis_gto(r_cut, n_max, l_max)
    weights = np.array([1.0, 0.7, 1.9])
    batch = mixed_batch(7 * sorted(WEIGHTINGS).index(weighting) + ["off", "mu2", "mu1nu1", "crossover"].index(compression))
    for average in ("off", "inner", "outer"):
        kwargs = dict(average=average, species_weights=weights, compression=compression,
                      weighting=WEIGHTINGS[weighting])
        got = oracle.soap(batch, species, r_cut, n_max, l_max, sigma, alphas, betas, **kwargs)
        want = ref.soap_ex(batch, species, r_cut, n_max, l_max, sigma, alphas, betas, **kwargs)
        assert got.shape == want.shape
        assert got.shape[1] == feature_count(len(species), n_max, l_max, compression)
        assert np.isfinite(want).all()
        err = max_rel_err(got, want, AGREE_FLOOR)
        assert err <= AGREE_TOL, f"{compression}/{weighting}/{average}: {err:.3e}"


def test_labels_follow_reference_layouts():
    """Label order of every compression mode (_kernels/core.py:306-329)."""
    species, n_max, l_max = (8, 1), 3, 2
    for compression in ("off", "mu2", "mu1nu1", "crossover"):
        names = labels(species, n_max, l_max, compression)
        assert len(names) == feature_count(len(species), n_max, l_max, compression)
        assert len(set(names)) == len(names)
    assert labels(species, n_max, l_max, "mu2")[:3] == (
        "soap:compression=mu2,l=0,n1=0,n2=0", "soap:compression=mu2,l=0,n1=0,n2=1",
        "soap:compression=mu2,l=0,n1=0,n2=2")
    assert labels(species, n_max, l_max, "mu1nu1")[0] == "soap:compression=mu1nu1,z1=8,l=0,n1=0,n2=0"
    assert labels(species, n_max, l_max, "crossover")[-1] == "soap:z1=1,z2=1,l=2,n1=2,n2=2"


@pytest.mark.parametrize("l_max", [0, 1, 3, 6])
@pytest.mark.parametrize("compression", ["off", "mu2", "mu1nu1", "crossover"])
def test_checker_matches_reference_polynomial_basis(oracle, l_max, compression):
    """rbf="polynomial": the checker's flir recurrence, integrand and projection
    (soap.cpp:450-492, 799-857) against compute_soap, with weighting and w0
    (the exact self pair takes the r <= 1e-14 branch)."""
    from oracle import RefLib
    from mdescriptor_b200.basis import basis_polynomial

    ref = RefLib()
    species, r_cut, n_max, sigma = (1, 6, 8), 3.6, 4, 0.8
    grid, grid_weights, values = basis_polynomial(r_cut, n_max)
    batch = mixed_batch(31 + l_max)
    for average in ("off", "inner", "outer"):
        kwargs = dict(average=average, species_weights=np.array([1.0, 0.7, 1.9]), compression=compression,
                      weighting={"function": "poly", "r0": 4.2, "c": 1.3, "m": 2.0, "w0": 0.3})
        got = oracle.soap_poly(batch, species, r_cut, n_max, l_max, sigma, grid, grid_weights, values, **kwargs)
        want = ref.soap_poly(batch, species, r_cut, n_max, l_max, sigma, grid, grid_weights, values, **kwargs)
        assert got.shape == want.shape == (want.shape[0], feature_count(3, n_max, l_max, compression))
        assert np.isfinite(want).all() and np.abs(want).max() > 0
        err = max_rel_err(got, want, AGREE_FLOOR)
        assert err <= AGREE_TOL, f"{compression}/{average}: {err:.3e}"


def test_polynomial_basis_matches_reference_construction():
    """basis_polynomial restates _basis_polynomial (_kernels/core.py:79-95): the
    values are orthonormal under the quadrature weight r^2 (to the conditioning
    of the monomial overlap, which grows quickly with n_max)."""
    from mdescriptor_b200.basis import basis_polynomial

    grid, weights, values = basis_polynomial(5.0, 4)
    assert grid.shape == weights.shape == (100,) and values.shape == (4, 100)
    assert grid.min() > 0.0 and grid.max() < 5.0
    gram = (values * (weights * grid**2)) @ values.T
    np.testing.assert_allclose(gram, np.eye(4), atol=1e-8)


def test_flir_conditioning_probe(oracle):
    """The probe that moves every polynomial-basis exponential by one ulp
    changes the checker's rows by a small, nonzero amount, and switching it
    off restores the reference-matching rows bit for bit."""
    from mdescriptor_b200.basis import basis_polynomial

    species, r_cut, n_max, l_max, sigma = (1, 6, 8), 3.6, 4, 3, 0.8
    grid, grid_weights, values = basis_polynomial(r_cut, n_max)
    batch = mixed_batch(5)
    base = oracle.soap_poly(batch, species, r_cut, n_max, l_max, sigma, grid, grid_weights, values)
    try:
        oracle.lib.oracle_set_flir_exp_ulp(1)
        moved = oracle.soap_poly(batch, species, r_cut, n_max, l_max, sigma, grid, grid_weights, values)
    finally:
        oracle.lib.oracle_set_flir_exp_ulp(0)
    again = oracle.soap_poly(batch, species, r_cut, n_max, l_max, sigma, grid, grid_weights, values)
    assert np.array_equal(again, base)
    assert 0.0 < max_rel_err(moved, base, AGREE_FLOOR) < 1e-6
