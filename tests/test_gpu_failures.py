"""Failure detection on a GPU box without faulting a GPU.

* Out of memory: MDSOAP_TEST_FAIL_ALLOC makes the engine's device allocator
  return cudaErrorMemoryAllocation on the host (no real exhaustion).  The
  status is MDSOAP_OUT_OF_MEMORY, the plugin raises CudaOutOfMemory
  (MemoryError, cpp/cuda/include/mdescriptor/cuda/error.hpp:15-28 and
  cpp/cuda/src/bindings.cu:18-20), and the reference's adapter turns that into
  MDescriptorError(code="backend_out_of_memory")
  (src/mdescriptor/core/errors.py:83-113).  The engine computes normally once
  the hook is cleared.
* Bounded waits: the tail kernel's wait for its bulk copies gives up after a
  time limit, sets an error bit and returns.  mdsoap_probe_bounded_wait makes
  that exact wait run out (an mbarrier armed for a copy that is never issued,
  1 ms limit); the call reports MDSOAP_INTERNAL with the tail-timeout message
  and the device stays usable.
"""

from __future__ import annotations

import numpy as np
import pytest

from _plugin import PLUGIN_DIR
from _reference import reference_package
from mdescriptor_b200 import _lib, workloads
from mdescriptor_b200.soap import Soap

pytestmark = pytest.mark.gpu


def _soap():
    return Soap((1, 8), r_cut=4.5, n_max=4, l_max=3, average="off", dtype="float32")


def test_injected_allocation_failure_is_out_of_memory_and_recoverable(cuda_device, monkeypatch):
    batch = workloads.config1(structures=3)
    expected = _soap().compute(batch, devices=[cuda_device])
    monkeypatch.setenv("MDSOAP_TEST_FAIL_ALLOC", "1")
    soap = _soap()
    with pytest.raises(_lib.CudaOutOfMemory, match="out of memory|allocation"):
        soap.compute(batch, devices=[cuda_device])
    # a large-block threshold: the plan's small tables allocate, the rows' block does not
    monkeypatch.setenv("MDSOAP_TEST_FAIL_ALLOC", str(1 << 16))
    with pytest.raises(MemoryError):
        _soap().compute(batch, devices=[cuda_device])
    monkeypatch.delenv("MDSOAP_TEST_FAIL_ALLOC")
    np.testing.assert_array_equal(soap.compute(batch, devices=[cuda_device]), expected)


def test_out_of_memory_reaches_the_public_api_as_backend_out_of_memory(cuda_device, monkeypatch):
    reference_package()
    monkeypatch.setenv("MDESCRIPTOR_CUDA_PLUGIN_DIR", str(PLUGIN_DIR))
    monkeypatch.setenv("MDSOAP_DEVICES", str(cuda_device))
    from mdescriptor import ExecutionOptions, MDescriptorError, OutputOptions, StructureBatch
    from mdescriptor._cuda_loader import load_cuda_plugin
    from mdescriptor.descriptors import SOAP

    load_cuda_plugin()
    batch = workloads.config1(structures=2)
    sb = StructureBatch(batch.numbers, batch.positions, batch.cells, batch.pbc, batch.offsets, ("a", "b"))
    soap = SOAP(species=[1, 8], r_cut=4.5, n_max=4, l_max=3, average="off", output=OutputOptions(dtype="float32"),
                execution=ExecutionOptions(device="cuda"))
    monkeypatch.setenv("MDSOAP_TEST_FAIL_ALLOC", "1")
    with pytest.raises(MDescriptorError) as info:
        soap.compute(sb)
    assert info.value.code == "backend_out_of_memory"
    monkeypatch.delenv("MDSOAP_TEST_FAIL_ALLOC")
    assert soap.compute(sb).values.shape == (128, 144)


def test_bounded_wait_runs_out_and_reports_internal(cuda_device):
    status = _lib.lib.mdsoap_probe_bounded_wait(cuda_device, 1_000_000)
    assert status == _lib.INTERNAL
    assert "did not complete in time" in _lib.last_error()
    # the context is intact: a normal computation follows
    values = _soap().compute(workloads.config1(structures=1), devices=[cuda_device])
    assert np.isfinite(values).all()
    assert _lib.lib.mdsoap_probe_bounded_wait(cuda_device, 0) == _lib.INVALID_ARGUMENT
