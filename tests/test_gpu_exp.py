"""The engine's exp() against CUDA's exp().

Every radial factor exp(-a r^2) goes through exp_nonpositive
(mdescriptor_b200/csrc/expneg.cuh), written from Tang's table-driven method
(ACM TOMS 15(2), 1989) rather than calling CUDA's exp().  This checks it
against CUDA's exp() and numpy's exp() on the same arguments: within 1 ulp
over the whole range the kernels use (x in [-708, 0]), and exactly 0 below
-708, where the true value is under exp(-708) = 3.31e-308 (far below every
other term of a SOAP sum).
"""

from __future__ import annotations

import numpy as np
import pytest

from mdescriptor_b200.soap import probe_exp


def _ulps(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a.view(np.int64) - b.view(np.int64))


@pytest.mark.gpu
def test_exp_matches_cuda_within_one_ulp(cuda_device):
    rng = np.random.default_rng(7)
    x = np.concatenate([
        -np.linspace(0.0, 708.0, 400_001),
        -rng.exponential(2.0, 400_000),                         # the SOAP range: a r^2 of a few units
        -rng.uniform(0.0, 0.05, 100_000),                       # near 0 (self pair, tiny exponents)
        -np.abs(rng.standard_normal(100_000)) * 1e-12,
        np.array([0.0, -0.0, -1e-300, -np.log(2.0) / 64, -np.log(2.0) / 32, -707.9, -708.0]),
    ])
    ours, cuda = probe_exp(x, cuda_device)
    assert np.isfinite(ours).all()
    assert _ulps(ours, cuda).max() <= 1
    assert _ulps(ours, np.exp(x)).max() <= 1
    assert ours[x == 0.0].tolist() == [1.0] * int((x == 0.0).sum())


@pytest.mark.gpu
def test_exp_flushes_below_the_double_range(cuda_device):
    x = -np.linspace(708.0001, 800.0, 10_001)
    ours, cuda = probe_exp(x, cuda_device)
    assert (ours == 0.0).all()
    assert (cuda <= 3.31e-308).all()


def _radial_args(seed):
    """Arguments spanning what the plans allow: exponents e of the GTO channels
    (0.01 .. 3 per A^2), r^2 = u up to the padded cutoff^2 and beyond, e u up
    to 700, prefactors over many decades; results kept normal doubles."""
    rng = np.random.default_rng(seed)
    n = 600_000
    e = np.exp(rng.uniform(np.log(0.01), np.log(3.0), n))
    u = np.concatenate([rng.uniform(0.0, 100.0, n // 2), rng.uniform(0.0, 700.0, n - n // 2) / e[n // 2:]])
    u[:1000] = 0.0                                            # the exact self pair
    pref = np.exp(rng.uniform(np.log(1e-6), np.log(1e6), n))
    keep = (e * u <= 700.0) & (pref * np.exp(-e * u) >= 1e-300)
    return u[keep], e[keep], pref[keep]


@pytest.mark.gpu
@pytest.mark.parametrize("form,bound", [(0, 1e-15), (1, 1e-13), (2, 2e-13)],
                         ids=["float64-rows", "float32-rows-fused", "float32-rows-folded"])
def test_radial_factor_forms_against_cuda_exp(cuda_device, form, bound):
    """The kernels' radial factors pref * exp(-e u) (Tang's method with the
    prefactor folded into the table factor) against pref * CUDA's exp(-e u):
    the float64-row form within a few ulp; the float32-row forms (one series
    term and one reduction step fewer; the expansion-only kernel's form also
    folds e into the reduction and uses a 64-entry table) within a few 1e-14
    relative, bounded here at 1e-13 and 2e-13 -- far below what a float32
    row resolves."""
    from mdescriptor_b200.soap import probe_radial

    u, e, pref = _radial_args(11 + form)
    ours, cuda = probe_radial(form, u, e, pref, cuda_device)
    assert np.isfinite(ours).all()
    rel = np.abs(ours - cuda) / np.abs(cuda)
    assert rel.max() <= bound, f"max relative error {rel.max():.3e}"
    assert np.array_equal(ours[u == 0.0], pref[u == 0.0])    # exp(0) exactly: the self pair
