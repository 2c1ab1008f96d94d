"""Comparison helpers for the parity tests.

Error metric: per element |a - b| / max(|b|, floor * max_row |b|).  With the
engine computing in fp64 and rounding once at the store, the bound is
1e-5 for float32 output (floor 1e-6) and 1e-10 for float64 output with
floor 1e-4 (fp64 rounding noise between two fp64 implementations that sum in
different orders is ~1e-14 x row max, so a 1e-10 relative bound is only
meaningful above 1e-4 x row max; below it the bound reads as 1e-14 x row max
absolute).
"""

from __future__ import annotations

import numpy as np

F32_TOL, F32_FLOOR = 1e-5, 1e-6
F64_TOL, F64_FLOOR = 1e-10, 1e-4
# Two independent fp64 implementations (the oracle's harmonic recurrence vs the
# reference's literal l<=4 / l=6 polynomials, different summation orders)
# agree to ~3e-13 x row max; power-spectrum entries built from nearly
# orthogonal coefficient vectors amplify that to ~2e-10 relative at l = 6.
AGREE_TOL, AGREE_FLOOR = 1e-9, 1e-3


def max_rel_err(actual, expected, floor):
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    assert actual.shape == expected.shape, (actual.shape, expected.shape)
    if expected.size == 0:
        return 0.0
    scale = np.abs(expected).max(axis=1, keepdims=True)
    denom = np.maximum(np.abs(expected), floor * scale)
    denom[denom == 0] = 1.0
    return float((np.abs(actual - expected) / denom).max())


def assert_features_close(actual, expected, dtype):
    if np.dtype(dtype) == np.float32:
        err = max_rel_err(actual, expected, F32_FLOOR)
        assert err <= F32_TOL, f"float32 max rel err {err:.3e} > {F32_TOL}"
    else:
        err = max_rel_err(actual, expected, F64_FLOOR)
        assert err <= F64_TOL, f"float64 max rel err {err:.3e} > {F64_TOL}"
    return err


def canonical_graph(graph):
    """Sort a CSR graph into (center, atom, shift) order; returns a dict of arrays."""
    offsets, atoms, shifts, disp, d2 = graph
    centers = np.repeat(np.arange(len(offsets) - 1, dtype=np.int64), np.diff(offsets))
    order = np.lexsort((shifts[:, 2], shifts[:, 1], shifts[:, 0], atoms, centers))
    return {
        "centers": centers[order],
        "atoms": atoms[order],
        "shifts": shifts[order],
        "disp_bits": np.ascontiguousarray(disp[order]).view(np.uint64),
        "d2_bits": np.ascontiguousarray(d2[order]).view(np.uint64),
        "offsets": offsets,
    }


def assert_graph_bit_exact(actual, expected):
    a, b = canonical_graph(actual), canonical_graph(expected)
    assert np.array_equal(a["offsets"], b["offsets"]), "per-centre pair counts differ"
    for key in ("centers", "atoms", "shifts", "disp_bits", "d2_bits"):
        assert np.array_equal(a[key], b[key]), f"graph field {key} differs"
