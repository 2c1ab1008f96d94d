"""The reference's unchanged public API computing on the GPU.

``SOAP(..., execution=ExecutionOptions(device="cuda")).compute(StructureBatch)``
from the reference package (staged in baseline/_ref) reaches this
repository's ``mdescriptor._cuda`` plugin through MDESCRIPTOR_CUDA_PLUGIN_DIR
and runs the adapter's whole chain: the 32-structure block loop, the block
combiner and the result normalisation
(src/mdescriptor/core/backends.py:192-249, 412-467, 470-522).  Its
``DescriptorResult`` must equal the same call with ``device="cpu"`` (the
reference's own C++ path): the same labels, level, row offsets and sample
identities, and values within the float32 / float64 bounds of tests/_util.py.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

from _plugin import PLUGIN_DIR
from _reference import reference_package
from _util import assert_features_close
from mdescriptor_b200 import workloads

pytestmark = pytest.mark.gpu

CASES = [
    # config, structures, species, r_cut, n_max, l_max, average, dtype
    (1, 72, (1, 8), 4.5, 4, 3, "off", "float32"),
    (1, 72, (1, 8), 4.5, 4, 3, "inner", "float32"),
    (1, 40, (1, 8), 4.5, 4, 3, "outer", "float32"),
    (2, 66, (1, 6, 7, 8), 5.0, 8, 6, "off", "float32"),
    (2, 34, (1, 6, 7, 8), 5.0, 8, 6, "inner", "float32"),
]


@pytest.fixture()
def api(monkeypatch, cuda_device):
    reference_package()
    monkeypatch.setenv("MDESCRIPTOR_CUDA_PLUGIN_DIR", str(PLUGIN_DIR))
    monkeypatch.setenv("MDSOAP_DEVICES", str(cuda_device))
    import mdescriptor
    from mdescriptor import ExecutionOptions, OutputOptions, StructureBatch
    from mdescriptor._cuda_loader import load_cuda_plugin
    from mdescriptor.descriptors import SOAP

    # The reference's own loader (what its tests and benchmarks call); it
    # accepts a plugin already imported from the same directory.
    assert load_cuda_plugin() == PLUGIN_DIR.resolve()

    return mdescriptor, SOAP, StructureBatch, OutputOptions, ExecutionOptions


@pytest.mark.parametrize("case", CASES, ids=[f"cfg{c[0]}-{c[6]}-{c[7]}-{c[1]}" for c in CASES])
def test_public_api_on_the_gpu_equals_the_reference_cpu_path(api, case):
    _, SOAP, StructureBatch, OutputOptions, ExecutionOptions = api
    config, structures, species, r_cut, n_max, l_max, average, dtype = case
    batch = workloads.make(config, structures)
    sb = StructureBatch(batch.numbers, batch.positions, batch.cells, batch.pbc, batch.offsets,
                        tuple(f"s{i}" for i in range(structures)))
    kw = dict(species=list(species), r_cut=r_cut, n_max=n_max, l_max=l_max, average=average,
              output=OutputOptions(dtype=dtype))
    gpu = SOAP(**kw, execution=ExecutionOptions(device="cuda")).compute(sb)
    cpu = SOAP(**kw, execution=ExecutionOptions(device="cpu")).compute(sb)
    assert Path(sys.modules["mdescriptor._cuda"].__file__).parent.resolve() == PLUGIN_DIR.resolve()
    assert gpu.metadata["backend"] == "mdescriptor-cuda" and gpu.metadata["execution"]["device"] == "cuda"
    assert gpu.level == cpu.level
    assert tuple(gpu.labels) == tuple(cpu.labels)
    assert gpu.values.dtype == cpu.values.dtype == np.dtype(dtype)
    assert gpu.values.shape == cpu.values.shape
    if cpu.row_offsets is None:
        assert gpu.row_offsets is None
    else:
        np.testing.assert_array_equal(gpu.row_offsets, cpu.row_offsets)
    np.testing.assert_array_equal(np.asarray(gpu.samples), np.asarray(cpu.samples))
    assert_features_close(gpu.values, cpu.values, dtype)


def test_public_api_sparse_output_on_the_gpu(api):
    """OutputOptions(sparse=True): the adapter builds the CSR from the plugin's
    dense blocks; the matrix equals the CPU path's."""
    _, SOAP, StructureBatch, OutputOptions, ExecutionOptions = api
    batch = workloads.make(1, 36)
    sb = StructureBatch(batch.numbers, batch.positions, batch.cells, batch.pbc, batch.offsets,
                        tuple(f"s{i}" for i in range(36)))
    kw = dict(species=[1, 8], r_cut=4.5, n_max=4, l_max=3, average="off",
              output=OutputOptions(dtype="float32", sparse=True))
    gpu = SOAP(**kw, execution=ExecutionOptions(device="cuda")).compute(sb).values
    cpu = SOAP(**kw, execution=ExecutionOptions(device="cpu")).compute(sb).values
    assert gpu.shape == cpu.shape
    assert_features_close(gpu.toarray(), cpu.toarray(), "float32")
