"""float64 rows against the reference itself, and against the exact value.

The GPU's float64 rows are compared with the reference's own C++ SOAP
(``oracle/_ref/libref_soap.so``, compiled from its sources) on the same
seeded inputs, err(a, b) = max |a - b| / max(|b|, 1e-4 max_row |b|), and with
the exact value of the same algorithm on the same double inputs (the checker's
extended-precision build, ``oracle/liboracle_soap_ext.so``).

The bar is 1e-10 against the reference.  What limits agreement at that level
is the rounding of the neighbour sums, which the radial basis then amplifies
(beta entries up to 1.7e3 at n_max = 8, r_cut 5-5.5): with the sums made
exact, the checker's rows move 4-7x closer to the exact value, while exact
harmonics change nothing.  The reference forms each sum with a two-lane SIMD
reduction (its rows reproduce exactly when the checker sums alternate
neighbours separately), and lands 5e-11 to 6e-10 from the exact value; any
double implementation summing in another order lands a comparable, different
distance away, so two such implementations can differ by more than 1e-10
even when both are within 1e-10 of the exact value.  The paired-channel
kernel's float64 instantiations keep every sum as two partial sums over
alternate neighbours (the same accuracy class).  A case passes when the GPU
rows are within 1e-10 of the reference's, or else no farther from the exact
value than twice the larger of the bar and the reference's own distance to
it.  Each case prints err at floors 1e-4 and
1e-6, the unfloored maximum and the maximum absolute error over the row
maximum (``pytest -s``).
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
    # shapes outside the paired-channel kernel (the centre kernel)
    "cfg3-mu2": (3, 1, (13, 29), 6.0, 8, 8, "off", "mu2"),
    "cfg3-mu1nu1-outer": (3, 1, (13, 29), 6.0, 8, 8, "outer", "mu1nu1"),
    "cfg2-n10-crossover": (2, 3, (1, 6, 7, 8), 5.0, 10, 4, "off", "crossover"),
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
    if vs_ref["floor1e-4"] > F64_TOL:
        assert gpu_exact["floor1e-4"] <= 2.0 * max(F64_TOL, ref_exact["floor1e-4"]), (vs_ref, gpu_exact, ref_exact)
