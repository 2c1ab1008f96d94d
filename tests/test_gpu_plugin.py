"""The drop-in plugin contract on a GPU.

The options MDescriptor's unchanged adapter hands to
``mdescriptor._cuda.create_backend`` (captured from the live adapter into
tests/golden/adapter_options.json) are replayed into this plugin, and the
result dictionary is checked field by field against what the adapter's
``_cuda_result`` consumes (src/mdescriptor/core/backends.py:134-190) and
against the reference's own CPU result for the same options and batch
(tests/golden/adapter_expected.npz).  The control object follows the
reference's ComputeControl protocol (src/mdescriptor/core/control.py:47-73):
``reset(total)``, ``cancelled()``, ``mark_completed()``.
"""

from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import pytest

from _plugin import adapter_cases, load_plugin
from _util import assert_features_close

GOLDEN = Path(__file__).resolve().parent / "golden"


class Batch:
    def __init__(self, arrays):
        for key in ("numbers", "positions", "cells", "pbc", "offsets"):
            setattr(self, key, arrays[f"input/{key}"])

    @property
    def structures(self):
        return len(self.offsets) - 1


class Control:
    """Counts the protocol calls; cancels once cancelled() has been asked
    `cancel_after` times (None: never)."""

    def __init__(self, cancel_after=None):
        self.total = None
        self.completed = 0
        self.asked = 0
        self.cancel_after = cancel_after

    def reset(self, total):
        self.total = total
        self.completed = 0

    def cancelled(self):
        self.asked += 1
        return self.cancel_after is not None and self.asked > self.cancel_after

    def mark_completed(self):
        self.completed += 1


@pytest.fixture(scope="module")
def expected():
    return dict(np.load(GOLDEN / "adapter_expected.npz"))


@pytest.mark.gpu
@pytest.mark.parametrize("index", [0, 1, 2, 3, 4])
def test_adapter_options_replayed_into_the_plugin(cuda_device, expected, index):
    plugin = load_plugin()
    name, options, kwargs = adapter_cases()[index]
    batch = Batch(expected)
    backend = plugin.create_backend(name, options)
    control = Control()
    result = backend.compute(batch, control)
    assert control.total == batch.structures and control.completed == batch.structures

    values = result["values"]
    assert isinstance(values, np.ndarray) and values.dtype == np.float32 and values.flags.c_contiguous
    # owned (no snapshot copy in the adapter) exactly when NumPy owns the rows;
    # rows in a recycled page-locked buffer are not
    assert result["_mdescriptor_owned_values"] is bool(values.flags.owndata)
    assert values.shape[1] == backend.feature_count == options["_cuda_feature_count"]
    assert_features_close(values, expected[f"case{index}/values"], np.float32)
    if kwargs["average"] == "off":
        assert result["level"] == "atom"
        np.testing.assert_array_equal(result["row_offsets"], expected[f"case{index}/row_offsets"])
    else:
        assert result["level"] == "structure"
        assert values.shape[0] == batch.structures
    assert tuple(tuple(x) if isinstance(x, list) else x for x in result["labels"]) == tuple(options["_cuda_labels"])
    assert result["metadata"] == {"descriptor": "SOAP", "backend": "mdescriptor-cuda",
                                  "execution": {"device": "cuda", "num_threads": None}}

    # A second call on the same backend (device state reused) gives the same bytes.
    again = backend.compute(batch, None)["values"]
    assert np.array_equal(again, values)
    backend.close()


@pytest.mark.gpu
def test_adapter_block_slicing_matches_one_call(cuda_device, expected):
    """The adapter submits 32-structure blocks (backends.py:192-249); a block
    call gives the same rows as the whole-batch call."""
    plugin = load_plugin()
    name, options, _ = adapter_cases()[0]
    batch = Batch(expected)
    backend = plugin.create_backend(name, options)
    whole = backend.compute(batch, None)["values"]
    offsets = batch.offsets
    for s in range(batch.structures):
        block = Batch({
            "input/numbers": batch.numbers[offsets[s]:offsets[s + 1]],
            "input/positions": batch.positions[offsets[s]:offsets[s + 1]],
            "input/cells": batch.cells[s:s + 1],
            "input/pbc": batch.pbc[s:s + 1],
            "input/offsets": offsets[s:s + 2] - offsets[s],
        })
        part = backend.compute(block, None)
        assert np.array_equal(part["values"], whole[offsets[s]:offsets[s + 1]])
    backend.close()


@pytest.mark.gpu
def test_cancellation_before_and_during_the_run(cuda_device, expected, monkeypatch):
    plugin = load_plugin()
    name, options, _ = adapter_cases()[0]
    batch = Batch(expected)
    backend = plugin.create_backend(name, options)

    control = Control(cancel_after=0)
    with pytest.raises(plugin.CudaCancelledError):
        backend.compute(batch, control)
    assert control.completed == 0

    # Tiny output blocks: the engine asks between blocks, so a cancel that
    # arrives after the first question stops the run part-way.
    monkeypatch.setenv("MDSOAP_BLOCK_BYTES", "4096")
    control = Control(cancel_after=2)
    with pytest.raises(plugin.CudaCancelledError):
        backend.compute(batch, control)
    assert control.completed == 0
    assert control.asked >= 3

    # The backend stays usable after a cancelled run.
    monkeypatch.delenv("MDSOAP_BLOCK_BYTES")
    result = backend.compute(batch, Control())
    assert_features_close(result["values"], expected["case0/values"], np.float32)
    backend.close()


@pytest.mark.gpu
def test_invalid_batch_is_rejected_and_backend_survives(cuda_device, expected):
    plugin = load_plugin()
    name, options, _ = adapter_cases()[0]
    good = Batch(expected)
    backend = plugin.create_backend(name, options)
    bad = Batch(expected)
    bad.numbers = bad.numbers.copy()
    bad.numbers[5] = 6  # carbon is not a configured species
    with pytest.raises(ValueError, match="species"):
        backend.compute(bad, None)
    result = backend.compute(good, None)
    assert_features_close(result["values"], expected["case0/values"], np.float32)
    backend.close()


@pytest.mark.gpu
def test_devices_environment_variable(cuda_device, expected, monkeypatch):
    """MDSOAP_DEVICES picks the devices a backend shards over; a single listed
    device gives the same rows as the default."""
    plugin = load_plugin()
    name, options, _ = adapter_cases()[0]
    batch = Batch(expected)
    backend = plugin.create_backend(name, options)
    reference = backend.compute(batch, None)["values"]
    backend.close()
    monkeypatch.setenv("MDSOAP_DEVICES", str(cuda_device))
    backend = plugin.create_backend(name, options)
    assert np.array_equal(backend.compute(batch, None)["values"], reference)
    backend.close()
    assert os.environ["MDSOAP_DEVICES"] == str(cuda_device)


@pytest.mark.gpu
def test_recycled_page_locked_result_buffers(cuda_device, expected, monkeypatch):
    """The plugin returns rows in recycled page-locked buffers
    (mdsoap_host_buffer_acquire): a result the caller still holds is never
    handed out again, a freed one is reused, results stay writable NumPy
    arrays, and with the pool's cache disabled the rows are the same."""
    import gc

    plugin = load_plugin()
    name, options, _ = adapter_cases()[0]
    batch = Batch(expected)
    backend = plugin.create_backend(name, options)
    first = backend.compute(batch, None)["values"]
    snapshot = first.copy()
    held = [backend.compute(batch, None)["values"] for _ in range(3)]
    for values in held:
        assert values.ctypes.data != first.ctypes.data
        assert np.array_equal(values, snapshot)
    assert np.array_equal(first, snapshot)  # untouched by the later calls
    address = held[0].ctypes.data
    del held
    gc.collect()
    reused = backend.compute(batch, None)["values"]
    assert np.array_equal(reused, snapshot)
    assert reused.ctypes.data in (address, first.ctypes.data) or reused.base is not None
    reused[0, 0] = 1.0  # writable
    monkeypatch.setenv("MDSOAP_HOST_POOL_BYTES", "0")
    del reused
    gc.collect()
    assert np.array_equal(backend.compute(batch, None)["values"], snapshot)
    backend.close()
