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
