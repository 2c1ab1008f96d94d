"""Local spherical spectra (SphericalExpansion, SoapRadialSpectrum,
SoapPowerSpectrum) on the GPU against the reference's own values.

* the checker is the reference's compiled ``compute_spherical_expansion``
  (the staged reference package in baseline/_ref), pinned to the reference's own committed goldens
  for this family (its CPU output and the Featomic 0.6.6 external golden);
* committed fixtures (tests/golden/local_spectra.npz, made by
  tests/golden/make_local_golden.py): the reference goldens and seeded
  synthetic cases;
* where ``_native`` is present, larger seeded batches against it live,
  including triclinic cells, atoms outside the cell, an isolated cluster and
  an empty structure;
* without a GPU: feature counts, option validation and the empty batch
  through the C ABI.

Float64 bound of the generated cases: 1e-10 relative with floor 1e-4 x row
max (the SOAP float64 bound); the reference goldens keep their manifests'
rtol / atol.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

from _reference import reference_native
from _util import F64_FLOOR, F64_TOL, max_rel_err
from mdescriptor_b200 import workloads
from mdescriptor_b200.soap import LOCAL_KINDS, local_feature_count, local_spectrum

LOCAL_TOL, LOCAL_FLOOR = F64_TOL, F64_FLOOR

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden" / "local_spectra.npz"
NAMES = {v: k for k, v in LOCAL_KINDS.items()}


def golden_cases():
    data = np.load(GOLDEN)
    names = sorted({key.split("/")[0] for key in data.files})
    return data, names


def golden_batch(data, name):
    return workloads.Batch(data[f"{name}/numbers"], data[f"{name}/positions"], data[f"{name}/cells"],
                           data[f"{name}/pbc"], data[f"{name}/offsets"])


def native_values(nat, b, species, cutoff, width, nr, na, kind):
    return np.asarray(nat.compute_spherical_expansion(b.numbers, b.positions, b.cells, b.pbc, b.offsets,
                                                      [int(z) for z in species], float(cutoff), float(width),
                                                      int(nr), int(na), int(kind), 2.5, 1, float(cutoff), 0, None))


def test_feature_counts_follow_reference_layout():
    # local_layout.hpp:115-130
    for S, nr, na in [(1, 0, 0), (2, 6, 4), (5, 4, 6), (3, 7, 8)]:
        species = list(range(1, S + 1))
        n, A = nr + 1, na + 1
        assert local_feature_count("SphericalExpansion", species, nr, na) == S * S * n * A * A
        assert local_feature_count("SoapRadialSpectrum", species, nr, na) == S * S * n
        assert local_feature_count("SoapPowerSpectrum", species, nr, na) == S * (S + 1) // 2 * S * A * n * n


def test_invalid_options_rejected():
    for species, nr, na in [([], 6, 4), ([1, 1], 6, 4), ([1], -1, 4), ([1], 16, 4)]:
        with pytest.raises(ValueError):
            local_feature_count("SphericalExpansion", species, nr, na)
    with pytest.raises(ValueError):  # above the kernel's l <= 8
        local_feature_count("SoapPowerSpectrum", [1], 6, 9)
    with pytest.raises(ValueError):
        local_feature_count("Unknown", [1], 6, 4)
    b = workloads.make(1, structures=1)
    with pytest.raises(ValueError):
        local_spectrum("SphericalExpansion", b, [1, 8], cutoff=-1.0)
    with pytest.raises(ValueError):
        local_spectrum("SphericalExpansion", b, [1, 8], density_width=0.0)
    with pytest.raises(ValueError):  # atomic number 8 outside the species
        local_spectrum("SphericalExpansion", b, [1])


def test_empty_batch():
    empty = workloads.Batch(np.zeros(0, np.int32), np.zeros((0, 3)), np.zeros((0, 3, 3)), np.zeros((0, 3), np.int32),
                            np.zeros(1, np.int64))
    out = local_spectrum("SoapPowerSpectrum", empty, [1, 8], max_radial=3, max_angular=2)
    assert out.shape == (0, local_feature_count("SoapPowerSpectrum", [1, 8], 3, 2))


def test_reference_build_reproduces_reference_goldens():
    """Pin the checker: the compiled reference reproduces the reference's own
    committed goldens within their manifests' tolerances."""
    nat = reference_native()
    data, names = golden_cases()
    gold = [n for n in names if n.startswith("refgold_")]
    assert len(gold) == 4
    for name in gold:
        rtol, atol = data[f"{name}/tolerance"]
        got = native_values(nat, golden_batch(data, name), data[f"{name}/species"], *data[f"{name}/options"])
        np.testing.assert_allclose(got, data[f"{name}/values"], rtol=rtol, atol=atol, err_msg=name)


def test_golden_fixtures_are_reference_values():
    """The generated fixture rows are the reference's own values."""
    nat = reference_native()
    data, names = golden_cases()
    for name in [n for n in names if not n.startswith("refgold_")]:
        got = native_values(nat, golden_batch(data, name), data[f"{name}/species"], *data[f"{name}/options"])
        np.testing.assert_array_equal(got[data[f"{name}/rows"]], data[f"{name}/values"], err_msg=name)


@pytest.mark.gpu
def test_gpu_matches_golden_fixtures():
    data, names = golden_cases()
    assert len(names) == 11
    for name in names:
        b = golden_batch(data, name)
        cutoff, width, nr, na, kind = data[f"{name}/options"]
        got = local_spectrum(NAMES[int(kind)], b, [int(z) for z in data[f"{name}/species"]], cutoff=float(cutoff),
                             density_width=float(width), max_radial=int(nr), max_angular=int(na))
        want = data[f"{name}/values"]
        got = got[data[f"{name}/rows"]]
        if name.startswith("refgold_"):
            rtol, atol = data[f"{name}/tolerance"]
            np.testing.assert_allclose(got, want, rtol=rtol, atol=atol, err_msg=name)
            continue
        err = max_rel_err(got, want, LOCAL_FLOOR)
        assert err <= LOCAL_TOL, f"{name}: max rel err {err:.3e}"
        # entries outside the centre species' block are exactly zero, as in the reference
        np.testing.assert_array_equal(got == 0.0, want == 0.0)


def varied_batch(seed: int) -> workloads.Batch:
    """Triclinic cells (one small enough for several images per axis), atoms
    outside the cell, an isolated cluster, an empty structure."""
    rng = np.random.default_rng(seed)
    numbers, positions, cells, pbc, offsets = [], [], [], [], [0]
    for s in range(5):
        n = 0 if s == 3 else int(rng.integers(1, 24))
        periodic = s != 2
        scale = 2.2 if s == 4 else rng.uniform(4.0, 8.0)
        cell = np.diag(rng.uniform(0.9, 1.2, 3) * scale) + np.triu(rng.uniform(-0.5, 0.5, (3, 3)), 1)
        frac = rng.uniform(-0.4, 1.4, (n, 3))
        positions.append(frac @ cell if n else np.zeros((0, 3)))
        numbers.append(rng.choice([1, 8], n).astype(np.int32))
        cells.append(cell if periodic else np.zeros((3, 3)))
        pbc.append([1, 1, 1] if periodic else [0, 0, 0])
        offsets.append(offsets[-1] + n)
    return workloads.Batch(np.concatenate(numbers), np.concatenate(positions), np.array(cells),
                           np.array(pbc, np.int32), np.array(offsets, np.int64))


LIVE = [
    ("cfg4", 4, 12, [1, 6, 7, 8, 16], 5.0, 0.3, 6, 4),
    ("cfg2", 2, 2, [1, 6, 7, 8], 5.0, 0.3, 7, 5),
    ("cfg3", 3, 1, [13, 29], 4.0, 0.25, 5, 3),
    ("varied", 0, 0, [1, 8], 3.5, 0.3, 5, 4),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", LIVE, ids=[c[0] for c in LIVE])
@pytest.mark.parametrize("name", sorted(LOCAL_KINDS))
def test_gpu_matches_reference_live(case, name):
    nat = reference_native()
    label, config, structures, species, cutoff, width, nr, na = case
    if config == 0:
        b = varied_batch(7)
    elif config == 3:
        b = workloads.config3(structures=1, reps=(4, 4, 2))
    else:
        b = workloads.make(config, structures=structures)
    want = native_values(nat, b, species, cutoff, width, nr, na, LOCAL_KINDS[name])
    got = local_spectrum(name, b, species, cutoff=cutoff, density_width=width, max_radial=nr, max_angular=na)
    err = max_rel_err(got, want, LOCAL_FLOOR)
    assert err <= LOCAL_TOL, f"{label}/{name}: max rel err {err:.3e}"
