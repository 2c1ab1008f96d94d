"""The allocation-free entry point, mdsoap_compute_device_noalloc.

Callers whose framework allocator already owns the GPU's memory, or whose
latency-critical loop must not synchronise the device through cudaMalloc or
cudaFree, use this entry point: it runs the same kernels as
mdsoap_compute_device but keeps every working buffer in one fixed 32 MiB
device array instead of allocating.  This file is collected last on purpose:
the GPU test must pass both after the rest of the suite and alone in a fresh
process (`pytest tests/test_zz_no_alloc.py -m gpu`).
"""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

from _util import assert_features_close
from mdescriptor_b200 import _lib, workloads
from mdescriptor_b200.soap import Soap, device_view

GOLDEN = Path(__file__).resolve().parent / "golden"


def _case(name):
    meta = json.loads((GOLDEN / "config_goldens.json").read_text())[name]
    arrays = np.load(GOLDEN / "config_goldens.npz")
    batch = workloads.Batch(*(arrays[f"{name}/input/{k}"] for k in ("numbers", "positions", "cells", "pbc", "offsets")))
    return meta, batch


def test_noalloc_rejects_batches_beyond_its_scratch_without_touching_the_gpu():
    """The size check comes before any CUDA call, so it also runs without a GPU."""
    soap = Soap((1, 8), r_cut=4.5, n_max=4, l_max=3, average="off", dtype="float32")
    huge = device_view(0, 0, 0, 0, 0, 1000, 2_000_000)  # 2 M atoms: far beyond 32 MiB of bins
    status = _lib.lib.mdsoap_compute_device_noalloc(soap._plan, ctypes.byref(huge), None, 0, None)
    assert status == _lib.CAPACITY_OVERFLOW
    assert "scratch" in _lib.last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("name,average", [("cfg2", "off"), ("cfg3", "off"), ("cfg4", "inner"), ("cfg1", "outer")])
def test_noalloc_matches_device_entry_point_on_two_calls(cuda_device, name, average):
    torch = pytest.importorskip("torch")
    meta, batch = _case(name)
    soap = Soap(meta["species"], r_cut=meta["r_cut"], n_max=meta["n_max"], l_max=meta["l_max"],
                sigma=meta["sigma"], average=average, dtype=meta["dtype"])
    dev = torch.device("cuda", cuda_device)
    tensors = [torch.from_numpy(np.ascontiguousarray(getattr(batch, k))).to(dev)
               for k in ("numbers", "positions", "cells", "pbc", "offsets")]
    view = device_view(*(t.data_ptr() for t in tensors), batch.structures, batch.atoms)
    dtype = torch.float32 if meta["dtype"] == "float32" else torch.float64
    shape = (soap.rows(batch), soap.feature_count)
    stream = torch.cuda.current_stream(dev)

    expected = torch.empty(shape, dtype=dtype, device=dev)
    soap.compute_device(view, expected.data_ptr(), cuda_device, stream.cuda_stream)
    soap.check(cuda_device, stream.cuda_stream)
    expected = expected.cpu().numpy()

    for call in range(2):
        out = torch.full(shape, float("nan"), dtype=dtype, device=dev)
        status = _lib.lib.mdsoap_compute_device_noalloc(soap._plan, ctypes.byref(view), ctypes.c_void_p(out.data_ptr()),
                                                        cuda_device, ctypes.c_void_p(stream.cuda_stream))
        _lib.raise_for(status)
        got = out.cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}: unwritten rows"
        assert_features_close(got, expected, meta["dtype"])
