"""The drop-in boundary, checked without a GPU.

* libmdsoap.so exports every function include/mdsoap.h declares;
* the ``mdescriptor._cuda`` plugin has the attributes MDescriptor's lazy
  loader looks up (src/mdescriptor/_runtime.py:78-125) and registers the
  reference's exception classes (cpp/cuda/src/bindings.cu:15-57);
* option validation and the "unsupported" answers raise the classes the
  adapter maps (src/mdescriptor/core/errors.py:83-113);
* building a backend touches no GPU, and computing without one raises
  CudaUnavailable (ImportError) -- never a silent CPU result;
* when the reference package is staged (baseline/_ref), the reference's own
  public API, pointed at the plugin through MDESCRIPTOR_CUDA_PLUGIN_DIR,
  reaches it and reports device_unavailable.
"""

from __future__ import annotations

import ctypes
import re
import sys
from pathlib import Path

import numpy as np
import pytest

from _plugin import PLUGIN_DIR, adapter_cases, load_plugin
from _reference import reference_package
from mdescriptor_b200 import _lib, workloads

ROOT = Path(__file__).resolve().parents[1]


def test_library_exports_every_declared_symbol():
    header = (ROOT / "include" / "mdsoap.h").read_text()
    declared = set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(mdsoap_\w+)\s*\(", header, re.M))
    assert declared == set(_lib.EXPORTED), sorted(declared ^ set(_lib.EXPORTED))
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared:
        assert hasattr(lib, name), name
    assert _lib.lib.mdsoap_abi_version() == 3


def test_plugin_module_attributes():
    plugin = load_plugin()
    assert plugin.MODEL_SNAPSHOT_ABI == 1
    assert callable(plugin.create_backend)
    assert issubclass(plugin.CudaUnavailable, ImportError)
    assert issubclass(plugin.CudaOutOfMemory, MemoryError)
    assert issubclass(plugin.CudaCancelledError, RuntimeError)
    assert Path(plugin.__file__).parent.resolve() == PLUGIN_DIR.resolve()


def test_backend_construction_touches_no_gpu_and_compute_fails_loudly():
    plugin = load_plugin()
    name, options, _ = adapter_cases()[0]
    backend = plugin.create_backend(name, options)
    assert backend.feature_count == options["_cuda_feature_count"] == 144
    meta = backend.metadata()
    assert meta == {"descriptor": "SOAP", "backend": "mdescriptor-cuda",
                    "execution": {"device": "cuda", "num_threads": None}}
    from mdescriptor_b200.soap import device_count

    if device_count() == 0:
        batch = workloads.config1(structures=1)
        with pytest.raises(ImportError, match="CUDA"):
            backend.compute(batch, None)
    backend.close()
    backend.close()  # idempotent
    with pytest.raises(RuntimeError, match="closed"):
        backend.compute(workloads.config1(structures=1), None)


def test_unsupported_descriptors_and_options_raise_mapped_errors():
    plugin = load_plugin()
    name, options, _ = adapter_cases()[0]
    with pytest.raises(ImportError, match="SOAP, NeighborList, SphericalExpansion"):
        plugin.create_backend("ACSF", {"species": [1, 8]})
    # local spectra: reference option names, defaults and layout
    # (cpp/cuda/src/backend.cu:108-131, 590-602)
    for local, features in [("SphericalExpansion", 2 * 2 * 7 * 25), ("SoapRadialSpectrum", 2 * 2 * 7),
                            ("SoapPowerSpectrum", 3 * 2 * 5 * 49)]:
        backend = plugin.create_backend(local, {"species": [1, 8]})
        assert backend.feature_count == features
        backend.close()
        backend.close()
    with pytest.raises(ValueError):
        plugin.create_backend("SphericalExpansion", {"species": [1, 8], "density_width": -1.0})
    for key, value, match in [
        ("rbf", "bessel", "radial basis"),
        ("rbf", "polynomial", "polynomial payload"),
        ("compression", {"mode": "mu3"}, "compression"),
        ("weighting", {"function": "gauss", "r0": 3.0, "c": 1.0}, "weighting"),
        ("average", "median", "average"),
        ("_cuda_feature_count", 7, "feature count"),
        ("n_max", 40, "invalid CUDA SOAP parameters"),
    ]:
        bad = dict(options)
        bad[key] = value
        with pytest.raises(ValueError, match=match):
            plugin.create_backend(name, bad)
    bad = dict(options)
    bad["_cuda_payload"] = {"radial_basis": {"alphas": np.zeros((2, 2)), "betas": np.zeros((2, 2, 2))}}
    with pytest.raises(ValueError, match="payload"):
        plugin.create_backend(name, bad)


def test_species_weighting_keys_follow_the_reference_lookup():
    """Int key, then decimal string, then element symbol; missing species weigh
    1.0 (cpp/cuda/src/extended_descriptors_common.cuh:257-294).  The weights a
    plan holds are visible through the feature values only, so this checks that
    every key form is accepted; the GPU suite checks the values."""
    plugin = load_plugin()
    name, options, _ = adapter_cases()[1]
    for weights in ({1: 0.5, 8: 2.0}, {"1": 0.5, "8": 2.0}, {"H": 0.5, "O": 2.0}, {8: 2.0}, {}):
        ok = dict(options)
        ok["compression"] = {"mode": "off", "species_weighting": weights}
        plugin.create_backend(name, ok).close()
    bad = dict(options)
    bad["compression"] = {"mode": "off", "species_weighting": [0.5, 2.0]}
    with pytest.raises(Exception):
        plugin.create_backend(name, bad)


def test_labels_follow_declared_species_order():
    from mdescriptor_b200.basis import labels

    for _, options, _ in adapter_cases():
        mode = (options.get("compression") or {}).get("mode", "off")
        assert tuple(options["_cuda_labels"]) == labels(options["species"], options["n_max"], options["l_max"], mode)


def _reference_api():
    return reference_package()


def test_adapter_options_fixture_matches_live_adapter():
    """The committed options equal what the live adapter builds today."""
    mdescriptor = _reference_api()
    from mdescriptor import ExecutionOptions, OutputOptions, StructureBatch
    from mdescriptor.descriptors import SOAP
    import mdescriptor._runtime as runtime

    seen = []

    class Recorder:
        feature_count = None

        def __init__(self, name, options):
            seen.append((name, options))

        def compute(self, batch, control=None):
            raise ImportError("recorder")

    original = runtime.create_cuda_backend
    runtime.create_cuda_backend = lambda name, options: Recorder(name, options)
    try:
        batch = workloads.config1(structures=1)
        sb = StructureBatch(batch.numbers, batch.positions, batch.cells, batch.pbc, batch.offsets, ("s0",))
        for name, options, kwargs in adapter_cases():
            kwargs = dict(kwargs)
            if "compression" in kwargs and kwargs["compression"].get("species_weighting"):
                kwargs["compression"] = dict(kwargs["compression"])
                kwargs["compression"]["species_weighting"] = {
                    int(k): v for k, v in kwargs["compression"]["species_weighting"].items()}
            soap = SOAP(**kwargs, output=OutputOptions(dtype="float32"), execution=ExecutionOptions(device="cuda"))
            with pytest.raises(Exception):
                soap.compute(sb)
            live_name, live = seen[-1]
            assert live_name == name
            assert set(live) == set(options)
            for key in options:
                if key == "_cuda_payload":
                    assert set(live[key]["radial_basis"]) == set(options[key]["radial_basis"])
                    for arr in options[key]["radial_basis"]:
                        np.testing.assert_array_equal(live[key]["radial_basis"][arr],
                                                      options[key]["radial_basis"][arr])
                else:
                    assert live[key] == options[key], key
    finally:
        runtime.create_cuda_backend = original


def test_reference_public_api_reaches_the_plugin(monkeypatch):
    """SOAP(..., device="cuda") through MDescriptor's unchanged API loads this
    plugin via MDESCRIPTOR_CUDA_PLUGIN_DIR; without a GPU the public error is
    device_unavailable (no silent CPU fallback)."""
    mdescriptor = _reference_api()
    from mdescriptor_b200.soap import device_count

    if device_count() > 0:
        pytest.skip("a GPU is visible: the GPU suite covers the computing path")
    from mdescriptor import ExecutionOptions, MDescriptorError, OutputOptions, StructureBatch
    from mdescriptor._cuda_loader import load_cuda_plugin
    from mdescriptor.descriptors import SOAP

    monkeypatch.setenv("MDESCRIPTOR_CUDA_PLUGIN_DIR", str(PLUGIN_DIR))
    load_plugin()
    assert load_cuda_plugin() == PLUGIN_DIR.resolve()
    batch = workloads.config1(structures=2)
    sb = StructureBatch(batch.numbers, batch.positions, batch.cells, batch.pbc, batch.offsets, ("a", "b"))
    soap = SOAP(species=[1, 8], r_cut=4.5, n_max=4, l_max=3, average="off",
                output=OutputOptions(dtype="float32"), execution=ExecutionOptions(device="cuda"))
    with pytest.raises(MDescriptorError) as info:
        soap.compute(sb)
    assert info.value.code == "device_unavailable"
    assert Path(sys.modules["mdescriptor._cuda"].__file__).parent.resolve() == PLUGIN_DIR.resolve()


def test_golden_archives_load_without_pickle():
    golden = Path(__file__).resolve().parent / "golden"
    for path in sorted(golden.glob("*.npz")):
        with np.load(path) as archive:
            for key in archive.files:
                assert archive[key].dtype != object, (path.name, key)


def test_checker_reproduces_the_reference_public_api_for_every_adapter_case(oracle):
    """The CPU checker, fed the adapter's own options and payload (GTO and
    polynomial bases, compression, weighting), reproduces the reference's
    public-API CPU rows committed beside them (float32 output)."""
    from _util import assert_features_close
    from mdescriptor_b200.soap import options_from_payload

    expected = dict(np.load(ROOT / "tests" / "golden" / "adapter_expected.npz"))
    batch = workloads.Batch(*(expected[f"input/{k}"] for k in ("numbers", "positions", "cells", "pbc", "offsets")))
    for index, (_, options, _) in enumerate(adapter_cases()):
        kw = options_from_payload(options)
        weights = kw["species_weights"]
        if weights is not None:
            weights = [float(weights.get(str(z), weights.get(z, 1.0))) for z in kw["species"]]
        common = dict(average=kw["average"], species_weights=weights, compression=kw["compression"],
                      weighting=kw["weighting"])
        args = (batch, kw["species"], kw["r_cut"], kw["n_max"], kw["l_max"], kw["sigma"])
        if kw["rbf"] == "polynomial":
            got = oracle.soap_poly(*args, kw["radial_grid"], kw["radial_weights"], kw["radial_values"], **common)
        else:
            got = oracle.soap(*args, kw["alphas"], kw["betas"], **common)
        assert_features_close(got.astype(np.float32), expected[f"case{index}/values"], np.float32)
