"""Generate ``local_spectra.npz``: reference values of the local spherical
spectra (SphericalExpansion, SoapRadialSpectrum, SoapPowerSpectrum) for the
GPU parity tests.

Run in the build container, where the reference tree is present and its
``_native`` module has been built from its sources by
``oracle/build_oracle.py``:

    python tests/golden/make_local_golden.py

Each generated case is a seeded synthetic batch (slices of the benchmark
config generators: periodic cells and isolated clusters) and one option set;
the stored values are ``_native.compute_spherical_expansion`` (the
reference's cpp/src/standalone/spherical_expansion.cpp:124-206 through its
pybind binding), float64 rows of every ``stride``-th atom (``rows``).  The
``refgold_*`` cases are the reference's own committed goldens for
SphericalExpansion and SoapPowerSpectrum (tests/golden/sphericalexpansion,
tests/golden/soappowerspectrum: its CPU output and the Featomic 0.6.6
external golden), copied as data with their manifests' options and
tolerances (``tolerance`` = rtol, atol).
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
if not os.environ.get("MDSOAP_REFERENCE_ROOT"):
    raise SystemExit("set MDSOAP_REFERENCE_ROOT to the reference source tree")
REFERENCE = Path(os.environ["MDSOAP_REFERENCE_ROOT"])
sys.path.insert(0, str(ROOT))

from mdescriptor_b200 import workloads  # noqa: E402

KINDS = {"SphericalExpansion": 0, "SoapRadialSpectrum": 2, "SoapPowerSpectrum": 3}

# name -> (config, structures, descriptor, cutoff, density_width, max_radial,
# max_angular, stride of the stored rows)
CASES = {
    "se_cfg1_default": (1, 2, "SphericalExpansion", 6.0, 0.3, 6, 4, 4),
    "ps_cfg1_default": (1, 2, "SoapPowerSpectrum", 6.0, 0.3, 6, 4, 4),
    "rs_cfg1_default": (1, 2, "SoapRadialSpectrum", 6.0, 0.3, 6, 4, 1),
    "se_cfg4_wide": (4, 3, "SphericalExpansion", 5.0, 0.5, 4, 6, 8),
    "ps_cfg4_wide": (4, 2, "SoapPowerSpectrum", 5.0, 0.5, 4, 6, 16),
    "ps_cfg2_l8": (2, 1, "SoapPowerSpectrum", 4.5, 0.4, 5, 8, 32),
    "se_cfg1_short": (1, 1, "SphericalExpansion", 3.0, 0.2, 3, 2, 1),
}

REFERENCE_GOLDENS = {
    "refgold_se": ("sphericalexpansion", "SphericalExpansion", ""),
    "refgold_ps": ("soappowerspectrum", "SoapPowerSpectrum", ""),
    "refgold_se_featomic": ("sphericalexpansion", "SphericalExpansion", "external_"),
    "refgold_ps_featomic": ("soappowerspectrum", "SoapPowerSpectrum", "external_"),
}


def native():
    sys.path.insert(0, str(ROOT / "oracle" / "_ref" / "pkg"))
    import _native  # noqa: PLC0415

    return _native


def copy_reference_goldens(out: dict) -> None:
    for name, (folder, desc, prefix) in REFERENCE_GOLDENS.items():
        base = REFERENCE / "tests" / "golden" / folder
        manifest = json.loads((base / f"{prefix}manifest.json").read_text())
        params = manifest["configuration"]["parameters"]
        inputs = np.load(base / f"{prefix}input.npz")
        expected = np.load(base / f"{prefix}expected_output.npz")
        for key in ("numbers", "positions", "cells", "pbc", "offsets"):
            out[f"{name}/{key}"] = inputs[key]
        out[f"{name}/species"] = np.asarray(params["species"], np.int32)
        out[f"{name}/options"] = np.asarray([params["cutoff"], params["density_width"], params["max_radial"],
                                             params["max_angular"], KINDS[desc]], np.float64)
        out[f"{name}/rows"] = np.arange(expected["values"].shape[0], dtype=np.int64)
        out[f"{name}/values"] = np.asarray(expected["values"], np.float64)
        out[f"{name}/tolerance"] = np.asarray([manifest["tolerance"]["rtol"], manifest["tolerance"]["atol"]])
        print(name, expected["values"].shape, manifest["tolerance"])


def main() -> None:
    nat = native()
    out: dict[str, np.ndarray] = {}
    for name, (config, structures, desc, cutoff, width, nr, na, stride) in CASES.items():
        b = workloads.make(config, structures=structures)
        species = list(workloads.CONFIGS[config].species)
        values = nat.compute_spherical_expansion(b.numbers, b.positions, b.cells, b.pbc, b.offsets, species, cutoff,
                                                 width, nr, na, KINDS[desc], 2.5, 1, cutoff, 1, None)
        rows = np.arange(0, b.numbers.shape[0], stride, dtype=np.int64)
        out[f"{name}/rows"] = rows
        out[f"{name}/values"] = np.asarray(values, dtype=np.float64)[rows]
        for key in ("numbers", "positions", "cells", "pbc", "offsets"):
            out[f"{name}/{key}"] = getattr(b, key)
        out[f"{name}/species"] = np.asarray(species, np.int32)
        out[f"{name}/options"] = np.asarray([cutoff, width, nr, na, KINDS[desc]], np.float64)
        print(name, out[f"{name}/values"].shape)
    copy_reference_goldens(out)
    np.savez_compressed(HERE / "local_spectra.npz", **out)


if __name__ == "__main__":
    main()
