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
