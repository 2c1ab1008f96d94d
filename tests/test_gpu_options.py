"""GPU parity of compression layouts and radial weighting (paired-channel
kernel and, for the shapes outside it, the centre kernel) against the CPU
checker, which tests/test_oracle_options.py pins to the reference's own
compute_soap."""

from __future__ import annotations

import numpy as np
import pytest

from _util import AGREE_FLOOR, AGREE_TOL, F32_FLOOR, F32_TOL, assert_features_close, max_rel_err
from mdescriptor_b200 import workloads
from mdescriptor_b200.basis import basis_gto
from mdescriptor_b200.soap import Soap
from test_oracle_options import WEIGHTINGS, mixed_batch

pytestmark = pytest.mark.gpu

SHAPES = {
    # species, r_cut, n_max, l_max, sigma
    "n8l6": ((1, 6, 7, 8), 4.0, 8, 6, 1.0),   # register tail (n_max = 8)
    "n4l3": ((1, 6, 8), 3.6, 4, 3, 0.8),      # tensor-core / generic tails
    "n6l4": ((1, 6, 8), 3.8, 6, 4, 1.0),
}


def cluster_batch(seed: int, structures: int = 6) -> workloads.Batch:
    rng = np.random.default_rng(seed)
    numbers, positions, offsets = [], [], [0]
    for _ in range(structures):
        n = int(rng.integers(3, 30))
        positions.append(rng.uniform(-3.0, 3.0, (n, 3)))
        numbers.append(rng.choice([1, 6, 7, 8], n).astype(np.int32))
        offsets.append(offsets[-1] + n)
    return workloads.Batch(np.concatenate(numbers), np.concatenate(positions), np.zeros((structures, 3, 3)),
                           np.zeros((structures, 3), np.int32), np.array(offsets, np.int64))


def assert_close(got, want, dtype):
    """float32 rows: the float32 bound; float64 rows: the agreement bound of two
    fp64 implementations that sum in different orders (the l = 6 cancellations
    of the harmonic recurrences differ by up to ~5e-10 at floor 1e-4)."""
    if dtype == "float32":
        assert_features_close(got, want, dtype)
    else:
        err = max_rel_err(got, want, AGREE_FLOOR)
        assert err <= AGREE_TOL, f"float64 max rel err {err:.3e} > {AGREE_TOL}"


def run_both(oracle, shape, batch, average, dtype, compression, weighting, species_weights=None):
    species, r_cut, n_max, l_max, sigma = SHAPES[shape]
    alphas, betas = basis_gto(r_cut, n_max, l_max)
    soap = Soap(species, r_cut=r_cut, n_max=n_max, l_max=l_max, sigma=sigma, average=average, dtype=dtype,
                species_weights=species_weights, alphas=alphas, betas=betas, compression=compression,
                weighting=weighting)
    got = soap.compute(batch, devices=[0])
    want = oracle.soap(batch, species, r_cut, n_max, l_max, sigma, alphas, betas, average=average,
                       species_weights=species_weights, compression=compression, weighting=weighting)
    return soap, got, want


@pytest.mark.parametrize("shape", sorted(SHAPES))
@pytest.mark.parametrize("compression", ["off", "mu2", "mu1nu1", "crossover"])
@pytest.mark.parametrize("average", ["off", "inner", "outer"])
def test_compression_layouts(oracle, cuda_device, shape, compression, average):
    batch = cluster_batch(11) if shape == "n8l6" else mixed_batch(3)
    species = SHAPES[shape][0]
    weights = list(np.linspace(0.6, 1.8, len(species)))
    for dtype in ("float64", "float32"):
        soap, got, want = run_both(oracle, shape, batch, average, dtype, compression, None, weights)
        assert "soap_paired_kernel" in soap.kernel()
        assert_close(got, want, dtype)


@pytest.mark.parametrize("weighting", sorted(WEIGHTINGS))
@pytest.mark.parametrize("shape", ["n8l6", "n4l3"])
def test_weighting_functions(oracle, cuda_device, weighting, shape):
    batch = cluster_batch(5) if shape == "n8l6" else mixed_batch(9)
    for compression, average in (("off", "off"), ("mu2", "inner"), ("crossover", "outer")):
        _, got, want = run_both(oracle, shape, batch, average, "float64", compression, WEIGHTINGS[weighting])
        assert_close(got, want, "float64")


def test_config2_rows_with_weighting(oracle, cuda_device):
    """A full config-2 structure slice (the benchmark shape) under poly weighting and mu1nu1."""
    cfg = workloads.CONFIGS[2]
    batch = workloads.config2(structures=3)
    alphas, betas = basis_gto(cfg.r_cut, cfg.n_max, cfg.l_max)
    weighting = {"function": "poly", "r0": 7.0, "c": 1.0, "m": 2.0, "w0": 0.5}
    for compression in ("off", "mu1nu1"):
        soap = Soap(cfg.species, r_cut=cfg.r_cut, n_max=cfg.n_max, l_max=cfg.l_max, average="off",
                    dtype="float32", alphas=alphas, betas=betas, compression=compression, weighting=weighting)
        got = soap.compute(batch, devices=[0])
        want = oracle.soap(batch, cfg.species, cfg.r_cut, cfg.n_max, cfg.l_max, cfg.sigma, alphas, betas,
                           compression=compression, weighting=weighting)
        assert_features_close(got, want, "float32")


# Shapes outside the paired-channel kernel: the one-warp centre kernel with
# the tensor-core tail (n_max <= 8, l_max 8, config 3's shape) and with the
# scalar tail (n_max > 8).
CENTER_SHAPES = {
    "n8l8": ((1, 6, 8), 4.5, 8, 8, 1.0),
    "n10l4": ((1, 6, 8), 6.0, 10, 4, 1.0),
}


@pytest.mark.parametrize("shape", sorted(CENTER_SHAPES))
@pytest.mark.parametrize("compression", ["off", "mu2", "mu1nu1", "crossover"])
def test_center_kernel_compression_and_weighting(oracle, cuda_device, shape, compression):
    """Compression layouts, radial weighting (with w0) and species weights on
    the centre kernel, every average, both dtypes, against the checker."""
    species, r_cut, n_max, l_max, sigma = CENTER_SHAPES[shape]
    alphas, betas = basis_gto(r_cut, n_max, l_max)
    batch = mixed_batch(31)
    weights = list(np.linspace(0.6, 1.8, len(species)))
    cases = (("off", None), ("outer", WEIGHTINGS["poly+w0"]), ("inner", WEIGHTINGS["pow"]), ("off", WEIGHTINGS["exp"]),
             ("off", WEIGHTINGS["w0"]))
    for average, weighting in cases:
        want = oracle.soap(batch, species, r_cut, n_max, l_max, sigma, alphas, betas, average=average,
                           species_weights=weights, compression=compression, weighting=weighting)
        for dtype in ("float64", "float32"):
            soap = Soap(species, r_cut=r_cut, n_max=n_max, l_max=l_max, sigma=sigma, average=average, dtype=dtype,
                        species_weights=weights, alphas=alphas, betas=betas, compression=compression,
                        weighting=weighting)
            assert "soap_center_kernel" in soap.kernel()
            got = soap.compute(batch, devices=[0])
            if dtype == "float32":
                assert_features_close(got, want, dtype)
            else:
                # The agreement bound, widened for the worse-conditioned radial
                # bases of larger n_max (|beta| up to 6e3 here).
                bound = AGREE_TOL * max(1.0, float(np.abs(betas).max()) / 2e3)
                err = max_rel_err(got, want, AGREE_FLOOR)
                assert err <= bound, f"float64 max rel err {err:.3e} > {bound:.3e}"


def test_polynomial_basis_needs_paired_kernel_shape():
    """The polynomial radial basis runs on the paired kernel only: other
    shapes (here l_max = 8) reject it with a clear error instead of computing
    something else."""
    from mdescriptor_b200.basis import basis_polynomial

    grid, grid_weights, values = basis_polynomial(5.0, 8)
    with pytest.raises(ValueError, match="paired-channel kernel"):
        Soap((13, 29), r_cut=5.0, n_max=8, l_max=8, average="off", dtype="float64", rbf="polynomial",
             radial_grid=grid, radial_weights=grid_weights, radial_values=values)


@pytest.mark.parametrize("shape", sorted(SHAPES))
@pytest.mark.parametrize("compression", ["off", "mu2", "mu1nu1", "crossover"])
def test_polynomial_basis(oracle, cuda_device, shape, compression):
    """rbf="polynomial" on the paired kernel's POLY instantiation (per-edge
    flir on the quadrature nodes) against the checker."""
    from mdescriptor_b200.basis import basis_polynomial

    species, r_cut, n_max, l_max, sigma = SHAPES[shape]
    grid, grid_weights, values = basis_polynomial(r_cut, n_max)
    batch = cluster_batch(17) if shape == "n8l6" else mixed_batch(21)
    weights = list(np.linspace(0.6, 1.8, len(species)))
    weighting = WEIGHTINGS["poly+w0"] if compression == "mu2" else None
    for average in ("off", "inner", "outer"):
        kwargs = dict(average=average, species_weights=weights, compression=compression, weighting=weighting)
        want = oracle.soap_poly(batch, species, r_cut, n_max, l_max, sigma, grid, grid_weights, values, **kwargs)
        # The reference's upward flir recurrence amplifies last-bit differences
        # of its exponentials (at n_max = 8 up to ~1e-6 relative at floor 1e-3
        # and ~6e-4 at floor 1e-6); each bound is four times the spread the
        # checker itself shows at that floor when every exponential moves by
        # one ulp, and never below the usual bound for the dtype.
        try:
            oracle.lib.oracle_set_flir_exp_ulp(1)
            moved = oracle.soap_poly(batch, species, r_cut, n_max, l_max, sigma, grid, grid_weights, values,
                                     **kwargs)
        finally:
            oracle.lib.oracle_set_flir_exp_ulp(0)
        bound = {"float64": max(AGREE_TOL, 4.0 * max_rel_err(moved, want, AGREE_FLOOR)),
                 "float32": max(F32_TOL, 4.0 * max_rel_err(moved, want, F32_FLOOR))}
        floor = {"float64": AGREE_FLOOR, "float32": F32_FLOOR}
        for dtype in ("float64", "float32"):
            soap = Soap(species, r_cut=r_cut, n_max=n_max, l_max=l_max, sigma=sigma, average=average, dtype=dtype,
                        species_weights=weights, compression=compression, weighting=weighting, rbf="polynomial",
                        radial_grid=grid, radial_weights=grid_weights, radial_values=values)
            assert soap.kernel().endswith("true, 2, false, true>")
            got = soap.compute(batch, devices=[0])
            err = max_rel_err(got, want, floor[dtype])
            assert err <= bound[dtype], f"{dtype} max rel err {err:.3e} > {bound[dtype]:.3e}"
