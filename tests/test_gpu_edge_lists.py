"""The edge-list split of the split-tail path (MDSOAP_EDGE_CAP > 0): a
walk-only kernel writes each centre's accepted edges to a slot of edge_cap
edges, an expansion-only kernel reads them back, and the fused kernel redoes
the centres whose slot overflowed: with slots large enough for every centre,
with some centres overflowing (cap 64, 200) and with every centre
overflowing (cap 1), in both dtypes, with weighting, pooled species and
compression layouts.  The edges reach the expansion in the order the fused
kernel accepts them and float64 plans add them in that order, so float64
rows must equal the fused kernel's bit for bit.  For float32 rows the
expansion kernel lets the two half warps take alternate edges and adds the
two partial sums at the end, so the fp64 sums may differ from the fused
kernel's in their last bits: those rows are held to the float32 bound (and
are mostly identical)."""

from __future__ import annotations

import numpy as np
import pytest

from _util import assert_features_close
from mdescriptor_b200 import workloads
from mdescriptor_b200.basis import basis_gto
from mdescriptor_b200.soap import Soap

pytestmark = pytest.mark.gpu

CASES = {
    # name: (config, structures, dtype, average, weighting, compression)
    "cfg5-f32": (5, 48, "float32", "off", None, "off"),
    "cfg5-f64": (5, 16, "float64", "off", None, "off"),
    "cfg2-f32-outer": (2, 12, "float32", "outer", None, "off"),
    "cfg2-f64-poly-mu2": (2, 6, "float64", "off", {"function": "poly", "r0": 7.0, "c": 1.0, "m": 2.0, "w0": 0.5},
                          "mu2"),
    "cfg4-f32": (4, 48, "float32", "off", None, "off"),
    "cfg1-f64-w0-crossover": (1, 16, "float64", "outer", {"w0": 0.3}, "crossover"),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_edge_lists_match_the_fused_kernel_bitwise(cuda_device, monkeypatch, name):
    config, structures, dtype, average, weighting, compression = CASES[name]
    cfg = workloads.CONFIGS[config]
    batch = workloads.make(config, structures)
    alphas, betas = basis_gto(cfg.r_cut, cfg.n_max, cfg.l_max)

    def rows(cap):
        monkeypatch.setenv("MDSOAP_EDGE_CAP", cap)
        soap = Soap(cfg.species, r_cut=cfg.r_cut, n_max=cfg.n_max, l_max=cfg.l_max, sigma=cfg.sigma,
                    average=average, dtype=dtype, alphas=alphas, betas=betas, weighting=weighting,
                    compression=compression)
        return soap.kernel(), soap.compute(batch, devices=[cuda_device])

    fused_kernel, fused = rows("0")
    assert "edge lists" not in fused_kernel
    for cap in ("512", "200", "64", "1"):
        kernel, got = rows(cap)
        assert "edge lists" in kernel
        if dtype == "float64":
            assert np.array_equal(got.view(np.uint8), fused.view(np.uint8)), f"cap {cap}: rows differ from the fused kernel"
        else:
            assert_features_close(got, fused, dtype)


CENTER_CASES = {
    # name: (batch, species, r_cut, n_max, l_max, dtype, average, weighting, compression)
    "cfg3-l8-f64": ("cfg3", (13, 29), 6.0, 8, 8, "float64", "off", None, "off"),
    "cfg3-l8-f64-outer-mu1nu1": ("cfg3", (13, 29), 6.0, 8, 8, "float64", "outer", None, "mu1nu1"),
    "cfg2-l8-f64-inner-poly-mu2": ("cfg2", (1, 6, 7, 8), 5.0, 8, 8, "float64", "inner",
                                   {"function": "poly", "r0": 7.0, "c": 1.0, "m": 2.0, "w0": 0.5}, "mu2"),
    "cfg2-n10-f64-w0-crossover": ("cfg2", (1, 6, 7, 8), 5.0, 10, 4, "float64", "off", {"w0": 0.3}, "crossover"),
    "cfg2-n10-f32-outer": ("cfg2", (1, 6, 7, 8), 5.0, 10, 4, "float32", "outer", None, "off"),
}


@pytest.mark.parametrize("name", sorted(CENTER_CASES))
def test_centre_kernel_on_edge_lists_matches_its_own_walk(cuda_device, monkeypatch, name):
    """Shapes outside the paired kernel (l_max > 6, n_max > 8): the walk-only
    kernel fills the edge slots and the centre kernel reads them instead of
    walking (a centre whose slot overflowed walks itself).  For float64 rows
    the accepted edges arrive in the order of the centre kernel's own walk, so
    the rows equal those of MDSOAP_EDGE_CAP=0 bit for bit; float32 rows take
    the certified pairs' displacements (last bits) and are held to the float32
    bound."""
    bname, species, r_cut, n_max, l_max, dtype, average, weighting, compression = CENTER_CASES[name]
    batch = workloads.config3(structures=1, reps=(6, 6, 4)) if bname == "cfg3" else workloads.config2(structures=4)
    alphas, betas = basis_gto(r_cut, n_max, l_max)

    def rows(cap):
        monkeypatch.setenv("MDSOAP_EDGE_CAP", cap)
        soap = Soap(species, r_cut=r_cut, n_max=n_max, l_max=l_max, average=average, dtype=dtype, alphas=alphas,
                    betas=betas, weighting=weighting, compression=compression)
        return soap.kernel(), soap.compute(batch, devices=[cuda_device])

    own_kernel, own = rows("0")
    assert "soap_center_kernel" in own_kernel and "edge lists" not in own_kernel
    for cap in ("512", "64", "1"):
        kernel, got = rows(cap)
        assert "soap_center_kernel" in kernel and "edge lists" in kernel
        if dtype == "float64":
            assert np.array_equal(got.view(np.uint8), own.view(np.uint8)), f"cap {cap}: rows differ"
        else:
            assert_features_close(got, own, dtype)

