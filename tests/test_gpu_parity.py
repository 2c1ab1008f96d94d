"""GPU parity of the B200 engine through its C ABI (libmdsoap.so).

Neighbour graphs must equal the CPU checker's bit for bit (same pair set, same
fp64 displacement / squared-distance bits); features must match the
reference's own outputs (committed goldens) and the checker within the
tolerances of tests/_util.py.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from _util import (AGREE_FLOOR, AGREE_TOL, F32_FLOOR, F32_TOL, F64_FLOOR, F64_TOL, assert_features_close,
                   assert_graph_bit_exact, max_rel_err)
from mdescriptor_b200 import workloads
from mdescriptor_b200.basis import basis_gto, graph_cutoff
from mdescriptor_b200.soap import Soap, neighbor_graph

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
REF = np.load(GOLDEN / "reference_goldens.npz")
REF_META = json.loads((GOLDEN / "reference_goldens.json").read_text())
CFG = np.load(GOLDEN / "config_goldens.npz")
CFG_META = json.loads((GOLDEN / "config_goldens.json").read_text())


def batch_from(arrays, prefix):
    return workloads.Batch(*(arrays[f"{prefix}/{key}"] for key in ("numbers", "positions", "cells", "pbc", "offsets")))


def soap_for(meta, average, dtype=None, **extra):
    return Soap(meta["species"], r_cut=meta["r_cut"], n_max=meta["n_max"], l_max=meta["l_max"],
                sigma=meta["sigma"], average=average, dtype=dtype or meta["dtype"], **extra)


# --------------------------------------------------------------------- graph


@pytest.mark.parametrize("name", sorted(CFG_META))
def test_graph_bit_exact_config_slices(oracle, cuda_device, name):
    meta = CFG_META[name]
    batch = batch_from(CFG, f"{name}/input")
    cutoff = graph_cutoff(meta["r_cut"], meta["sigma"])
    gpu = neighbor_graph(batch, cutoff, cuda_device)
    assert_graph_bit_exact(gpu, oracle.graph(batch, cutoff))
    assert len(gpu[1]) == meta["graph_pairs"]


def test_graph_triclinic_many_images(oracle, cuda_device):
    cell = np.array([[1.8, 0.0, 0.0], [0.25, 1.7, 0.0], [0.1, 0.2, 1.9]])
    batch = workloads.Batch(np.array([8, 14], np.int32), np.array([[0.18, 0.29, 0.41], [0.96, 0.85, 1.12]]),
                            cell[None], np.ones((1, 3), np.int32), np.array([0, 2], np.int64))
    for cutoff in (2.3, 4.1):
        assert_graph_bit_exact(neighbor_graph(batch, cutoff, cuda_device), oracle.graph(batch, cutoff))


def test_graph_reference_golden_inputs(oracle, cuda_device):
    batch = batch_from(REF, "soap/input")
    for cutoff in (3.5, graph_cutoff(3.5, 1.0)):
        assert_graph_bit_exact(neighbor_graph(batch, cutoff, cuda_device), oracle.graph(batch, cutoff))


def random_mixed_batch(seed, structures=6, frac_range=(-0.4, 1.4)):
    rng = np.random.default_rng(seed)
    numbers, positions, cells, pbc, offsets = [], [], [], [], [0]
    for s in range(structures):
        n = 0 if s == 3 else int(rng.integers(1, 40))
        periodic = s % 3 != 2
        cell = np.diag(rng.uniform(3.0, 9.0, 3)) + np.triu(rng.uniform(-1.5, 1.5, (3, 3)), 1)
        frac = rng.uniform(*frac_range, (n, 3))  # by default unwrapped: some atoms outside the cell
        positions.append(frac @ cell)
        numbers.append(rng.choice([1, 6, 8], n).astype(np.int32))
        cells.append(cell if periodic else np.zeros((3, 3)))
        pbc.append([1, 1, 1] if periodic else [0, 0, 0])
        offsets.append(offsets[-1] + n)
    return workloads.Batch(np.concatenate(numbers), np.concatenate(positions).reshape(-1, 3), np.array(cells),
                           np.array(pbc, np.int32), np.array(offsets, np.int64))


@pytest.mark.parametrize("seed", range(6))
def test_graph_random_cells_bit_exact(oracle, cuda_device, seed):
    batch = random_mixed_batch(seed)
    cutoff = float(np.random.default_rng(100 + seed).uniform(2.0, 9.0))
    assert_graph_bit_exact(neighbor_graph(batch, cutoff, cuda_device), oracle.graph(batch, cutoff))


def test_graph_full_size_fcc_sampled(oracle, cuda_device):
    """Full 32768-atom config-3 cell: pair count per centre and sampled centres bit-exact."""
    batch = workloads.config3(structures=1)
    cutoff = graph_cutoff(6.0, 1.0)
    gpu = neighbor_graph(batch, cutoff, cuda_device)
    offsets = gpu[0]
    counts = np.diff(offsets)
    assert counts.min() > 150 and counts.max() < 320
    # exact-self present once per centre
    centers = np.repeat(np.arange(batch.atoms), counts)
    self_pairs = (gpu[1] == centers) & (gpu[2] == 0).all(axis=1)
    assert self_pairs.sum() == batch.atoms
    # a sub-batch re-indexed ordering check: sampled rows of the oracle graph
    cpu = oracle.graph(batch, cutoff)
    assert_graph_bit_exact(gpu, cpu)


# ------------------------------------------------------------------ features


@pytest.mark.parametrize("name", sorted(CFG_META))
def test_features_match_reference_config_slices(cuda_device, name):
    meta = CFG_META[name]
    batch = batch_from(CFG, f"{name}/input")
    for average in meta["outputs"]:
        soap = soap_for(meta, average, alphas=CFG[f"{name}/alphas"], betas=CFG[f"{name}/betas"])
        values = soap.compute(batch, devices=[cuda_device])
        assert values.dtype == np.dtype(meta["dtype"])
        rows = CFG[f"{name}/{average}/rows"]
        assert values.shape == (meta["outputs"][average]["rows_total"], soap.feature_count)
        assert_features_close(values[rows], CFG[f"{name}/{average}/values"], meta["dtype"])


@pytest.mark.parametrize("name", sorted(CFG_META))
@pytest.mark.parametrize("dtype", ["float32", "float64"])
def test_features_match_oracle_both_dtypes(oracle, cuda_device, name, dtype):
    meta = CFG_META[name]
    batch = batch_from(CFG, f"{name}/input")
    alphas, betas = CFG[f"{name}/alphas"], CFG[f"{name}/betas"]
    for average in ("off", "inner", "outer"):
        expected = oracle.soap(batch, meta["species"], meta["r_cut"], meta["n_max"], meta["l_max"], meta["sigma"],
                               alphas, betas, average)
        got = soap_for(meta, average, dtype, alphas=alphas, betas=betas).compute(batch, devices=[cuda_device])
        if dtype == "float32":
            assert_features_close(got, expected, "float32")
        else:
            err = max_rel_err(got, expected, 1e-3)
            assert err <= 1e-9, f"{name}/{average} float64: {err:.3e}"


def test_reference_soap_golden(cuda_device):
    meta = REF_META["soap"]
    p = meta["parameters"]
    batch = batch_from(REF, "soap/input")
    soap = Soap(p["species"], r_cut=p["r_cut"], n_max=p["n_max"], l_max=p["l_max"], sigma=p["sigma"],
                average=p["average"], dtype="float64")
    values = soap.compute(batch, devices=[cuda_device])
    np.testing.assert_allclose(values, REF["soap/expected/values"], rtol=meta["tolerance"]["rtol"],
                               atol=meta["tolerance"]["atol"])


def test_dscribe_static_golden(cuda_device):
    meta = REF_META["soap_dscribe"]
    p = meta["parameters"]
    batch = batch_from(REF, "soap_dscribe/input")
    soap = Soap(p["species"], r_cut=p["r_cut"], n_max=p["n_max"], l_max=p["l_max"], sigma=p["sigma"],
                average=p["average"], dtype="float64")
    np.testing.assert_allclose(soap.compute(batch, devices=[cuda_device]), REF["soap_dscribe/expected/values"],
                               rtol=meta["tolerance"]["rtol"], atol=meta["tolerance"]["atol"])


def test_full_size_config3_sampled_rows(oracle, cuda_device):
    """Full 32768-atom fcc cell (float64 output): sampled rows vs the checker at 1e-10."""
    cfg = workloads.CONFIGS[3]
    batch = workloads.config3(structures=1)
    alphas, betas = basis_gto(cfg.r_cut, cfg.n_max, cfg.l_max)
    soap = Soap(cfg.species, r_cut=cfg.r_cut, n_max=cfg.n_max, l_max=cfg.l_max, average="off", dtype="float64",
                alphas=alphas, betas=betas)
    values = soap.compute(batch, devices=[cuda_device])
    rows = np.random.default_rng(7).choice(batch.atoms, 96, replace=False)
    expected = oracle.soap_rows(batch, rows, cfg.species, cfg.r_cut, cfg.n_max, cfg.l_max, 1.0, alphas, betas)
    err = max_rel_err(values[rows], expected, F64_FLOOR)
    assert err <= F64_TOL, f"{err:.3e}"
    assert np.isfinite(values).all()


def test_mixed_batch_with_empty_structure_all_averages(oracle, cuda_device):
    batch = random_mixed_batch(11)
    assert (np.diff(batch.offsets) == 0).any()
    species = (1, 6, 8)
    alphas, betas = basis_gto(4.0, 5, 4)
    for average in ("off", "inner", "outer"):
        expected = oracle.soap(batch, species, 4.0, 5, 4, 0.7, alphas, betas, average)
        got = Soap(species, r_cut=4.0, n_max=5, l_max=4, sigma=0.7, average=average, dtype="float64",
                   alphas=alphas, betas=betas).compute(batch, devices=[cuda_device])
        assert max_rel_err(got, expected, 1e-3) <= 1e-9


def test_species_weights(oracle, cuda_device):
    meta = CFG_META["cfg4"]
    batch = batch_from(CFG, "cfg4/input")
    weights = {1: 0.5, 6: 1.25, 7: 2.0, 8: 0.75, 16: 3.0}
    expected = oracle.soap(batch, meta["species"], meta["r_cut"], meta["n_max"], meta["l_max"], 1.0,
                           CFG["cfg4/alphas"], CFG["cfg4/betas"], "off",
                           species_weights=[weights[z] for z in meta["species"]])
    got = soap_for(meta, "off", "float64", species_weights=weights, alphas=CFG["cfg4/alphas"],
                   betas=CFG["cfg4/betas"]).compute(batch, devices=[cuda_device])
    assert max_rel_err(got, expected, 1e-3) <= 1e-9


@pytest.mark.parametrize("frac_range", [(-0.4, 1.4), (0.0, 0.999)], ids=["unwrapped", "inside"])
@pytest.mark.parametrize("seed", range(3))
def test_float32_rows_certified_pairs(oracle, cuda_device, seed, frac_range):
    """float32 plans take candidates well inside the cutoff without the exact
    test when every atom of a structure lies inside its cell: random triclinic
    cells (some with atoms outside the cell), isolated and empty structures,
    radial weighting with a self weight, species-pooled compression."""
    from test_oracle_options import WEIGHTINGS

    batch = random_mixed_batch(seed, structures=8, frac_range=frac_range)
    species = (1, 6, 8)
    weights = [0.7, 1.3, 1.9]
    for n_max, l_max, r_cut in ((8, 6, 4.0), (4, 3, 3.6)):
        alphas, betas = basis_gto(r_cut, n_max, l_max)
        for compression, weighting in (("off", None), ("mu2", WEIGHTINGS["poly+w0"]),
                                       ("crossover", WEIGHTINGS["w0"])):
            for average in ("off", "outer"):
                want = oracle.soap(batch, species, r_cut, n_max, l_max, 0.8, alphas, betas, average=average,
                                   species_weights=weights, compression=compression, weighting=weighting)
                soap = Soap(species, r_cut=r_cut, n_max=n_max, l_max=l_max, sigma=0.8, average=average,
                            dtype="float32", species_weights=weights, alphas=alphas, betas=betas,
                            compression=compression, weighting=weighting)
                assert "soap_paired_kernel" in soap.kernel()
                assert_features_close(soap.compute(batch, devices=[cuda_device]), want, "float32")


@pytest.mark.parametrize("l_max,n_max", [(0, 1), (1, 3), (2, 2), (5, 7), (7, 6), (9, 4), (12, 3), (6, 12)])
def test_other_basis_sizes(oracle, cuda_device, l_max, n_max):
    batch = random_mixed_batch(3, structures=4)
    species = (1, 6, 8)
    alphas, betas = basis_gto(3.5, n_max, l_max)
    expected = oracle.soap(batch, species, 3.5, n_max, l_max, 1.0, alphas, betas, "off")
    got = Soap(species, r_cut=3.5, n_max=n_max, l_max=l_max, average="off", dtype="float64", alphas=alphas,
               betas=betas).compute(batch, devices=[cuda_device])
    # Nearly dependent Gaussians (many n over a short r_cut) give large beta
    # entries that amplify fp64 rounding in any implementation; scale the bound
    # by |beta| relative to the well-conditioned configs (|beta| ~ 2e3).
    tol = 1e-9 * max(1.0, float(np.abs(betas).max()) / 2e3)
    assert max_rel_err(got, expected, 1e-3) <= tol


def test_empty_and_degenerate_batches(cuda_device):
    soap = Soap((1, 8), r_cut=4.5, n_max=4, l_max=3, average="off", dtype="float32")
    empty = workloads.Batch(np.zeros(0, np.int32), np.zeros((0, 3)), np.zeros((0, 3, 3)), np.zeros((0, 3), np.int32),
                            np.zeros(1, np.int64))
    assert soap.compute(empty, devices=[cuda_device]).shape == (0, soap.feature_count)
    one = workloads.Batch(np.array([8], np.int32), np.zeros((1, 3)), (np.eye(3) * 2.0)[None],
                          np.ones((1, 3), np.int32), np.array([0, 1], np.int64))
    values = soap.compute(one, devices=[cuda_device])
    assert values.shape == (1, soap.feature_count) and np.isfinite(values).all()
    inner = Soap((1, 8), r_cut=4.5, n_max=4, l_max=3, average="inner", dtype="float64")
    hollow = workloads.Batch(np.zeros(0, np.int32), np.zeros((0, 3)), (np.eye(3) * 5.0)[None],
                             np.ones((1, 3), np.int32), np.array([0, 0], np.int64))
    np.testing.assert_array_equal(inner.compute(hollow, devices=[cuda_device]), 0.0)


def test_invalid_inputs_raise(cuda_device):
    soap = Soap((1, 8), r_cut=4.5, n_max=4, l_max=3, average="off", dtype="float32")
    batch = workloads.config1(structures=1)
    bad_species = workloads.Batch(np.where(batch.numbers == 1, 6, 8).astype(np.int32), batch.positions, batch.cells,
                                  batch.pbc, batch.offsets)
    with pytest.raises(ValueError, match="outside calculator species"):
        soap.compute(bad_species, devices=[cuda_device])
    mixed = workloads.Batch(batch.numbers, batch.positions, batch.cells, np.array([[1, 0, 1]], np.int32),
                            batch.offsets)
    with pytest.raises(ValueError, match="mixed periodicity"):
        soap.compute(mixed, devices=[cuda_device])
    singular = workloads.Batch(batch.numbers, batch.positions, np.zeros((1, 3, 3)), batch.pbc, batch.offsets)
    with pytest.raises(ValueError, match="nonsingular"):
        soap.compute(singular, devices=[cuda_device])


def test_deterministic_and_dtype_consistent(cuda_device):
    """Repeated runs give the same bits; float32 rows agree with the float64
    rows within the float32 bound (float32 plans evaluate the radial factors
    to a few 1e-14 instead of full fp64 accuracy, so a row can differ from the
    rounded float64 row in its last bit)."""
    meta = CFG_META["cfg2"]
    batch = batch_from(CFG, "cfg2/input")
    soap64 = soap_for(meta, "off", "float64")
    a = soap64.compute(batch, devices=[cuda_device])
    b = soap64.compute(batch, devices=[cuda_device])
    np.testing.assert_array_equal(a, b)
    soap32 = soap_for(meta, "off", "float32")
    f32 = soap32.compute(batch, devices=[cuda_device])
    np.testing.assert_array_equal(f32, soap32.compute(batch, devices=[cuda_device]))
    assert max_rel_err(f32, a, F32_FLOOR) <= F32_TOL


def test_blocked_pipeline_matches_single_block(cuda_device, monkeypatch):
    """Many small output blocks (copy/compute overlap path) give the same bits."""
    meta = CFG_META["cfg1"]
    batch = workloads.config1(structures=16)
    whole = soap_for(meta, "off").compute(batch, devices=[cuda_device])
    monkeypatch.setenv("MDSOAP_BLOCK_BYTES", str(64 * 144 * 4 * 3))
    blocked = soap_for(meta, "off").compute(batch, devices=[cuda_device])
    np.testing.assert_array_equal(whole, blocked)


def test_device_api_matches_host_api(cuda_device):
    torch = pytest.importorskip("torch")
    from mdescriptor_b200.soap import device_view

    meta = CFG_META["cfg2"]
    batch = batch_from(CFG, "cfg2/input")
    soap = soap_for(meta, "off")
    host = soap.compute(batch, devices=[cuda_device])
    dev = torch.device("cuda", cuda_device)
    tensors = [torch.from_numpy(np.ascontiguousarray(getattr(batch, k))).to(dev)
               for k in ("numbers", "positions", "cells", "pbc", "offsets")]
    out = torch.empty((batch.atoms, soap.feature_count), dtype=torch.float32, device=dev)
    view = device_view(*(t.data_ptr() for t in tensors), batch.structures, batch.atoms)
    stream = torch.cuda.current_stream(dev)
    soap.compute_device(view, out.data_ptr(), cuda_device, stream.cuda_stream)
    soap.check(cuda_device, stream.cuda_stream)
    np.testing.assert_array_equal(out.cpu().numpy(), host)


def test_multi_device_sharding_matches_single(cuda_device):
    from mdescriptor_b200.soap import device_count

    if device_count() < 2:
        pytest.skip("one visible device: the multi-device host path is covered by the CPU sharding tests")
    meta = CFG_META["cfg1"]
    batch = workloads.config1(structures=32)
    single = soap_for(meta, "off").compute(batch, devices=[0])
    multi = soap_for(meta, "off").compute(batch, devices=list(range(device_count())))
    np.testing.assert_array_equal(single, multi)


@pytest.mark.parametrize("config,variant", [(c, k) for c in (1, 2, 3, 4) for k in (1, 2)])
def test_alternative_kernel_variants_match(cuda_device, monkeypatch, config, variant):
    """Every alternative kernel of a class (selected with MDSOAP_VARIANT: the
    scalar centre kernel where the paired kernel is the default, other
    register-bank splits; an index past the class gives the default) matches
    the default kernel's features within the agreement bound of two fp64
    implementations that sum in different orders."""
    name = f"cfg{config}"
    meta = CFG_META[name]
    batch = batch_from(CFG, f"{name}/input")
    default = soap_for(meta, "off", "float64").compute(batch, devices=[cuda_device])
    monkeypatch.setenv("MDSOAP_VARIANT", str(variant))
    alt = soap_for(meta, "off", "float64").compute(batch, devices=[cuda_device])
    assert max_rel_err(alt, default, AGREE_FLOOR) <= AGREE_TOL
