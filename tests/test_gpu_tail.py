"""The n_max = 8 tail as its own persistent kernel (soap_tail_kernel: bulk-copied,
double-buffered coefficient blocks; float64 rows of four species, whose sums
take two register banks each, run soap_tail_generic_kernel) against the tail fused into the expansion
kernel (MDSOAP_SPLIT_TAIL=0) and against chunked expansion / tail launches
(MDSOAP_TAIL_CHUNK), and the persistent expansion kernel against one CTA per
four centres (MDSOAP_PERSISTENT=0): the same per-centre arithmetic in every
mode, so the rows agree bit for bit, and with the CPU checker within the float
tolerances."""

from __future__ import annotations

import numpy as np
import pytest

from test_gpu_options import assert_close
from mdescriptor_b200 import workloads
from mdescriptor_b200.basis import basis_gto
from mdescriptor_b200.soap import Soap

pytestmark = pytest.mark.gpu

SPECIES, R_CUT, N_MAX, L_MAX, SIGMA = (1, 6, 7, 8), 5.0, 8, 6, 1.0


def make(average, dtype, compression="off"):
    return Soap(SPECIES, r_cut=R_CUT, n_max=N_MAX, l_max=L_MAX, sigma=SIGMA, average=average, dtype=dtype,
                compression=compression)


@pytest.mark.parametrize("average", ["off", "outer"])
@pytest.mark.parametrize("dtype", ["float32", "float64"])
def test_split_fused_and_chunked_tails_agree(oracle, cuda_device, monkeypatch, average, dtype):
    # Walk and expansion in one kernel throughout (the edge-list split, which
    # regroups float32 sums, has its own test: test_gpu_edge_lists.py).
    monkeypatch.setenv("MDSOAP_EDGE_CAP", "0")
    batch = workloads.config2(structures=12, seed=5)
    split = make(average, dtype)
    # float64 plans split each neighbour sum over two register banks, so four
    # species no longer fit the register tail and soap_tail_generic_kernel runs.
    assert ("soap_tail_kernel" if dtype == "float32" else "soap_tail_generic_kernel") in split.kernel()
    want = split.compute(batch, devices=[0])
    # Repeated calls reuse the device state (barriers re-initialised per launch).
    assert np.array_equal(split.compute(batch, devices=[0]), want)

    monkeypatch.setenv("MDSOAP_SPLIT_TAIL", "0")
    fused = make(average, dtype)
    assert "soap_tail" not in fused.kernel()
    assert np.array_equal(fused.compute(batch, devices=[0]), want)
    monkeypatch.delenv("MDSOAP_SPLIT_TAIL")

    monkeypatch.setenv("MDSOAP_PERSISTENT", "0")  # one CTA per four centres instead of resident CTAs
    assert np.array_equal(make(average, dtype).compute(batch, devices=[0]), want)
    monkeypatch.delenv("MDSOAP_PERSISTENT")

    for chunk in ("37", "200"):  # ragged chunks; more centres than some grids
        monkeypatch.setenv("MDSOAP_TAIL_CHUNK", chunk)
        chunked = make(average, dtype)
        assert np.array_equal(chunked.compute(batch, devices=[0]), want), chunk
    monkeypatch.delenv("MDSOAP_TAIL_CHUNK")

    alphas, betas = basis_gto(R_CUT, N_MAX, L_MAX)
    ref = oracle.soap(batch, SPECIES, R_CUT, N_MAX, L_MAX, SIGMA, alphas, betas, average=average)
    assert_close(want, ref, dtype)


def test_split_tail_single_centre_and_empty(cuda_device):
    """Fewer centres than resident CTAs (one structure of one atom) and an empty batch."""
    soap = make("off", "float64")
    one = workloads.Batch(np.array([8], np.int32), np.zeros((1, 3)), np.zeros((1, 3, 3)),
                          np.zeros((1, 3), np.int32), np.array([0, 1], np.int64))
    rows = soap.compute(one, devices=[0])
    assert rows.shape == (1, soap.feature_count) and np.isfinite(rows).all() and rows.any()
    empty = workloads.Batch(np.zeros(0, np.int32), np.zeros((0, 3)), np.zeros((0, 3, 3)),
                            np.zeros((0, 3), np.int32), np.array([0], np.int64))
    assert soap.compute(empty, devices=[0]).shape == (0, soap.feature_count)


@pytest.mark.parametrize("shape", [((1, 6, 7, 8, 16), 5.0, 6, 4, "off"),      # more species than banks
                                   ((1, 8), 4.5, 4, 3, "off"),                # n_max < 8
                                   ((1, 6, 8), 3.8, 6, 4, "mu1nu1"),          # power_generic layouts
                                   ((1, 6, 8), 3.8, 8, 6, "crossover")])
@pytest.mark.parametrize("average", ["off", "outer"])
def test_generic_split_tail_matches_fused(oracle, cuda_device, monkeypatch, shape, average):
    """Plans whose coefficients do not stay in registers hand their raw-sum
    blocks to soap_tail_generic_kernel; the rows equal the fused kernel's bit
    for bit (the same tail code on the same blocks) and the checker's."""
    species, r_cut, n_max, l_max, compression = shape
    batch = workloads.config4(structures=40, seed=9)
    batch = workloads.Batch(np.where(np.isin(batch.numbers, species), batch.numbers, species[0]).astype(np.int32),
                            batch.positions, batch.cells, batch.pbc, batch.offsets)

    def make_plan():
        return Soap(species, r_cut=r_cut, n_max=n_max, l_max=l_max, sigma=1.0, average=average, dtype="float64",
                    compression=compression)

    split = make_plan()
    assert "soap_tail_generic_kernel" in split.kernel() or "soap_tail_kernel" in split.kernel()
    want = split.compute(batch, devices=[0])
    monkeypatch.setenv("MDSOAP_SPLIT_TAIL", "0")
    fused = make_plan()
    assert "soap_tail" not in fused.kernel()
    assert np.array_equal(fused.compute(batch, devices=[0]), want)
    monkeypatch.delenv("MDSOAP_SPLIT_TAIL")
    monkeypatch.setenv("MDSOAP_TAIL_CHUNK", "29")
    assert np.array_equal(make_plan().compute(batch, devices=[0]), want)
    monkeypatch.delenv("MDSOAP_TAIL_CHUNK")
    alphas, betas = basis_gto(r_cut, n_max, l_max)
    ref = oracle.soap(batch, species, r_cut, n_max, l_max, 1.0, alphas, betas, average=average,
                      compression=compression)
    assert_close(want, ref, "float64")
