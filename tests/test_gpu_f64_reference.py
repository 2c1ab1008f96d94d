"""float64 rows against the reference itself, and against the exact value.

The GPU's float64 rows are compared with the reference's own C++ SOAP
(``oracle/_ref/libref_soap.so``, compiled from its sources) on the same
seeded inputs, err(a, b) = max |a - b| / max(|b|, 1e-4 max_row |b|), and with
the exact value of the same algorithm on the same double inputs (the checker's
extended-precision build, ``oracle/liboracle_soap_ext.so``).

The bar is 1e-10 against the reference.  It applies wherever the reference's
own rows are within 1e-10 of the exact value, which holds for the l_max 2, 3,
4, 6 and 8 harmonic branches at n_max <= 6.  With n_max = 8 and r_cut 5-5.5
the orthonormalisation beta (entries up to 1.7e3) amplifies last-bit
rounding, and the reference's own rows stray 5-6e-10 from the exact value
(merely reversing the neighbour summation order of the C restatement moves
its rows by 5.9e-10).  No double implementation that rounds differently can
then meet 1e-10 against the reference.  There the test requires instead that
the GPU rows be about as close to the exact value as the reference's (within
2x of the reference's own error) and within 1e-10 of the exact value's
distance to the reference plus the GPU's own (the triangle bound).  Each case
prints err at floors 1e-4 and 1e-6, the unfloored maximum and the maximum
absolute error over the row maximum (``pytest -s``).
"""

from __future__ import annotations

import numpy as np
import pytest

from _util import F64_FLOOR, F64_TOL, max_rel_err
from mdescriptor_b200 import workloads
from mdescriptor_b200.basis import basis_gto
from mdescriptor_b200.soap import Soap

pytestmark = pytest.mark.gpu

CASES = {
    # name: (config, structures, species, r_cut, n_max, l_max, average, compression)
    "cfg2-l6": (2, 3, (1, 6, 7, 8), 5.0, 8, 6, "off", "off"),
    "cfg5-l6": (5, 2, (1, 6, 8), 5.5, 8, 6, "off", "off"),
    "cfg2-l4": (2, 3, (1, 6, 7, 8), 5.0, 8, 4, "off", "off"),
    "cfg2-l2": (2, 3, (1, 6, 7, 8), 5.0, 8, 2, "off", "off"),
    "cfg1-l3": (1, 6, (1, 8), 4.5, 4, 3, "off", "off"),
    "cfg4-l4": (4, 24, (1, 6, 7, 8, 16), 5.0, 6, 4, "off", "off"),
    "cfg3-l8": (3, 1, (13, 29), 6.0, 8, 8, "off", "off"),
    "cfg1-inner": (1, 6, (1, 8), 4.5, 4, 3, "inner", "off"),
    "cfg2-outer": (2, 3, (1, 6, 7, 8), 5.0, 8, 6, "outer", "off"),
    "cfg2-mu1nu1": (2, 3, (1, 6, 7, 8), 5.0, 8, 6, "off", "mu1nu1"),
    "cfg2-crossover": (2, 3, (1, 6, 7, 8), 5.0, 8, 6, "off", "crossover"),
    "cfg2-mu2": (2, 3, (1, 6, 7, 8), 5.0, 8, 6, "off", "mu2"),
}


@pytest.fixture(scope="module")
def ref():
    from oracle import RefLib, reference_available

    if not reference_available():
        pytest.fail("oracle/_ref/libref_soap.so (the compiled reference) is missing")
    return RefLib()


@pytest.fixture(scope="module")
def exact():
    from oracle import ExtendedLib

    return ExtendedLib()


def figures(got, want):
    scale = np.abs(want).max(axis=1, keepdims=True)
    scale[scale == 0] = 1.0
    return {"floor1e-4": max_rel_err(got, want, F64_FLOOR), "floor1e-6": max_rel_err(got, want, 1e-6),
            "unfloored": max_rel_err(got, want, 0.0),
            "max_abs/rowmax": float((np.abs(got - want) / scale).max())}


def _batch(config, structures):
    if config == 3:
        return workloads.config3(structures=structures, reps=(8, 8, 4))
    return workloads.make(config, structures)


@pytest.mark.parametrize("name", sorted(CASES))
def test_float64_rows_match_the_compiled_reference(ref, exact, cuda_device, name):
    config, structures, species, r_cut, n_max, l_max, average, compression = CASES[name]
    batch = _batch(config, structures)
    alphas, betas = basis_gto(r_cut, n_max, l_max)
    soap = Soap(species, r_cut=r_cut, n_max=n_max, l_max=l_max, average=average, dtype="float64",
                alphas=alphas, betas=betas, compression=compression)
    got = soap.compute(batch, devices=[cuda_device])
    args = (batch, species, r_cut, n_max, l_max, 1.0, alphas, betas)
    want = ref.soap_ex(*args, average=average, compression=compression)
    truth = exact.soap(*args, average=average, compression=compression)
    vs_ref, gpu_exact, ref_exact = figures(got, want), figures(got, truth), figures(want, truth)
    print(f"\n{name}: GPU vs reference " + ", ".join(f"{k} {v:.2e}" for k, v in vs_ref.items())
          + f"; vs exact: GPU {gpu_exact['floor1e-4']:.2e}, reference {ref_exact['floor1e-4']:.2e}")
    if ref_exact["floor1e-4"] <= F64_TOL:
        assert vs_ref["floor1e-4"] <= F64_TOL, vs_ref
    else:
        assert gpu_exact["floor1e-4"] <= 2.0 * ref_exact["floor1e-4"], (gpu_exact, ref_exact)
        assert vs_ref["floor1e-4"] <= F64_TOL + gpu_exact["floor1e-4"] + ref_exact["floor1e-4"], (vs_ref, ref_exact)
