"""GTO radial basis and feature layout of MDescriptor's SOAP, restated.

The drop-in plugin never calls these: MDescriptor's adapter hands the plugin
the basis it built itself (``_cuda_payload``).  They exist so that the C ABI
can be driven without MDescriptor installed (benchmarks, GPU tests).
"""

from __future__ import annotations

from math import gamma, log, sqrt

import numpy as np


def basis_gto(r_cut: float, n_max: int, l_max: int) -> tuple[np.ndarray, np.ndarray]:
    """Orthonormalised GTO radial basis (alphas (L+1, n), betas (L+1, n, n)).

    Restates ``_basis_gto`` (src/mdescriptor/descriptors/_kernels/core.py:60-76):
    r_k = linspace(1, r_cut, n); alpha_{lk} = -ln(1e-3 / r_k^l) / r_k^2; the
    Gaussian overlap S_l = 0.5 Gamma(l + 3/2) (alpha_k + alpha_k')^(-l-3/2) is
    inverted-square-rooted through its eigendecomposition, beta_l = S_l^(-1/2).
    """
    radii = np.linspace(1.0, r_cut, n_max)
    alphas = np.empty((l_max + 1, n_max), dtype=np.float64)
    betas = np.empty((l_max + 1, n_max, n_max), dtype=np.float64)
    for degree in range(l_max + 1):
        alpha = -np.log(1e-3 / radii**degree) / radii**2
        overlap = 0.5 * gamma(degree + 1.5) * (alpha[:, None] + alpha[None, :]) ** (-degree - 1.5)
        values, vectors = np.linalg.eigh(overlap)
        if np.any(values <= 0):
            raise ValueError("could not normalize the SOAP GTO radial basis")
        betas[degree] = (vectors * (1.0 / np.sqrt(values))) @ vectors.T
        alphas[degree] = alpha
    return alphas, betas


def basis_polynomial(r_cut: float, n_max: int, nodes: int = 100) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Polynomial radial basis on a Gauss-Legendre grid (grid (Q,), weights (Q,),
    values (n, Q)).

    Restates ``_basis_polynomial`` (src/mdescriptor/descriptors/_kernels/core.py:79-95):
    Q = 100 Gauss-Legendre nodes mapped to [0, r_cut]; the monomials
    (r_cut - r)^(n + 3), n = 0..n_max-1, have the overlap
    S_ij = 2 r_cut^(7+i+j) / ((5+i+j)(6+i+j)(7+i+j)) (i, j = 1..n_max), and the
    orthonormal basis on the nodes is S^(-1/2) applied to the monomials.
    """
    x, w = np.polynomial.legendre.leggauss(nodes)
    grid = 0.5 * r_cut * (x + 1.0)
    weights = 0.5 * r_cut * w
    overlap = np.empty((n_max, n_max), dtype=np.float64)
    for i in range(1, n_max + 1):
        for j in range(1, n_max + 1):
            overlap[i - 1, j - 1] = (2.0 * r_cut ** (7 + i + j)) / ((5 + i + j) * (6 + i + j) * (7 + i + j))
    values, vectors = np.linalg.eigh(overlap)
    if np.any(values <= 0.0):
        raise ValueError("could not normalize the SOAP polynomial radial basis")
    betas = (vectors * (1.0 / np.sqrt(values))) @ vectors.T
    powers = np.asarray([(r_cut - np.clip(grid, 0.0, r_cut)) ** (n + 3) for n in range(n_max)])
    return grid, weights, betas @ powers


def feature_count(n_species: int, n_max: int, l_max: int, compression: str = "off") -> int:
    """Features per row by compression mode (_kernels/core.py:272-284; soap.cpp:373-387)."""
    if compression == "mu2":
        return n_max * (n_max + 1) // 2 * (l_max + 1)
    if compression == "mu1nu1":
        return n_species * n_max * n_max * (l_max + 1)
    if compression == "crossover":
        return n_species * n_max * (n_max + 1) // 2 * (l_max + 1)
    width = n_species * n_max
    return width * (width + 1) // 2 * (l_max + 1)


def labels(species, n_max: int, l_max: int, compression: str = "off") -> tuple[str, ...]:
    """Feature labels in output order (_kernels/core.py:306-329).

    Species pairs follow the declared (not sorted) species order, z1 <= z2 by
    position; then l, then n1, then n2 (n2 >= n1 within a species).  mu2 has
    one pooled density; mu1nu1 pairs each species with it (all n2); crossover
    keeps same-species pairs only.
    """
    species = list(species)
    out = []
    if compression == "mu2":
        for degree in range(l_max + 1):
            for n1 in range(n_max):
                for n2 in range(n1, n_max):
                    out.append(f"soap:compression=mu2,l={degree},n1={n1},n2={n2}")
        return tuple(out)
    if compression == "mu1nu1":
        for first in species:
            for degree in range(l_max + 1):
                for n1 in range(n_max):
                    for n2 in range(n_max):
                        out.append(f"soap:compression=mu1nu1,z1={first},l={degree},n1={n1},n2={n2}")
        return tuple(out)
    if compression == "crossover":
        pairs = [(first, first) for first in species]
    else:
        pairs = [(first, second) for i, first in enumerate(species) for second in species[i:]]
    for first, second in pairs:
        for degree in range(l_max + 1):
            for n1 in range(n_max):
                for n2 in range(n1 if first == second else 0, n_max):
                    out.append(f"soap:z1={first},z2={second},l={degree},n1={n1},n2={n2}")
    return tuple(out)


def graph_cutoff(r_cut: float, sigma: float) -> float:
    """Neighbour cutoff of the GTO SOAP: r_cut + sigma sqrt(-2 ln 1e-3) (soap.cpp:1214,1234).

    Evaluated with the C library's log/sqrt (as the reference's C++ does), not
    numpy's vectorised ones, so the last bit of the cutoff matches.  The C ABI
    computes the same value itself; this copy is for reporting only.
    """
    return r_cut + sigma * sqrt(-2.0 * log(1e-3))
