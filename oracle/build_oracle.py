"""Build recipe for the test-only checkers under ``oracle/``.

Two things are built here, neither of which is part of the product:

* ``oracle/liboracle_soap.so`` -- the plain-C restatement of the reference's
  SOAP hot path (``oracle/soap_oracle.c``).  It travels with the repository
  snapshot and is what the GPU parity tests and ``smoke()`` check against.
  ``oracle/liboracle_soap_ext.so`` is the same source with its SOAP stage in
  extended precision: the exact-value yardstick for float64 parity.
* ``oracle/_ref/`` -- the reference's own CPU path compiled from its sources
  where they lie (never copied into this repository):
  - ``libref_soap.so``: ``cpp/src/standalone/soap.cpp``,
    ``cpp/src/standalone/neighbor_list.cpp``,
    ``cpp/src/common/neighbor.cpp``, ``cpp/src/common/control.cpp`` plus the
    C entry layer ``oracle/ref_shim.cpp``.  This is the "reference" CPU
    baseline timed by ``bench.py --impl reference`` and the pin for the C
    restatement.
  - ``pkg/_native<EXT_SUFFIX>``: the reference's full pybind11 ``_native``
    module (every source of ``CMakeLists.txt:92-120``), linked against the
    local sgemm stand-in in ``oracle/ref_cblas``.  Only used in the build
    container, to run the reference's unchanged Python API when generating
    golden fixtures and when checking the drop-in plugin boundary.

* ``baseline/_ref/mdescriptor/`` -- the reference's Python package, staged
  from ``src/mdescriptor`` with the ``_native`` build above beside it (the
  offline ``pip install --target baseline/_ref`` of the reference fails here:
  its build backend needs ``setuptools_scm`` and ``scipy-openblas32``, neither
  of which is installed).  Its unchanged public API is what the GPU tests and
  ``bench.py``'s API-path figure drive, with ``MDESCRIPTOR_CUDA_PLUGIN_DIR``
  pointing at this repository's plugin.  The model weight files are left out
  (no SOAP path reads them).

The reference tree is only present in the build container, named by the
``MDSOAP_REFERENCE_ROOT`` environment variable; without it the reference steps
are skipped (with a message) and the prebuilt files are used.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
REF_OUT = ORACLE_DIR / "_ref"
BASELINE_REF = ORACLE_DIR.parent / "baseline" / "_ref"

# CMakeLists.txt:92-120 (MDESCRIPTOR_CPP_SOURCES)
_NATIVE_SOURCES = [
    "cpp/src/common/control.cpp",
    "cpp/src/common/neighbor.cpp",
    "cpp/src/standalone/soap.cpp",
    "cpp/src/standalone/soap_turbo.cpp",
    "cpp/src/standalone/acsf.cpp",
    "cpp/src/standalone/c00ps_mlff.cpp",
    "cpp/src/standalone/coulomb_matrix.cpp",
    "cpp/src/standalone/sine_matrix.cpp",
    "cpp/src/standalone/ewald_sum_matrix.cpp",
    "cpp/src/standalone/matrix_dispatch.cpp",
    "cpp/src/common/matrix_output.cpp",
    "cpp/src/standalone/mbtr.cpp",
    "cpp/src/standalone/ead.cpp",
    "cpp/src/standalone/ace.cpp",
    "cpp/src/standalone/mtp.cpp",
    "cpp/src/standalone/mtp4.cpp",
    "cpp/src/standalone/rotational_descriptors.cpp",
    "cpp/src/common/nep.cpp",
    "cpp/src/model_backed/dpa4.cpp",
    "cpp/src/model_backed/dpa4_wigner.cpp",
    "cpp/src/model_backed/dpa4c.cpp",
    "cpp/src/standalone/atomic_composition.cpp",
    "cpp/src/standalone/sorted_distances.cpp",
    "cpp/src/standalone/neighbor_list.cpp",
    "cpp/src/standalone/spherical_expansion.cpp",
    "cpp/src/standalone/spherical_expansion_by_pair.cpp",
    "cpp/src/bindings/module.cpp",
]
_SOAP_SOURCES = [
    "cpp/src/standalone/soap.cpp",
    "cpp/src/standalone/neighbor_list.cpp",
    "cpp/src/common/neighbor.cpp",
    "cpp/src/common/control.cpp",
]
# scikit-build-core builds the reference in Release mode: -O3 -DNDEBUG, no -march.
_REF_FLAGS = ["-std=c++17", "-O3", "-DNDEBUG", "-fopenmp", "-fPIC"]


def reference_root() -> Path | None:
    """The reference source tree named by MDSOAP_REFERENCE_ROOT, or None when
    the variable is unset; a set variable that names no reference tree is an
    error."""
    value = os.environ.get("MDSOAP_REFERENCE_ROOT")
    if not value:
        return None
    root = Path(value)
    if not (root / "cpp" / "src" / "standalone" / "soap.cpp").is_file():
        raise RuntimeError(f"MDSOAP_REFERENCE_ROOT={value} is not a reference source tree "
                           "(cpp/src/standalone/soap.cpp missing)")
    return root


def _run(cmd: list[str]) -> None:
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{result.stdout}\n{result.stderr}")


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(source.stat().st_mtime > mtime for source in sources)


def build_c_oracle(force: bool = False) -> Path:
    """Compile the plain-C restatement (no FMA contraction, like the reference
    build), and the same source with its SOAP stage in x87 extended precision
    (liboracle_soap_ext.so, -DORACLE_EXTENDED): the exact-value yardstick of
    the float64 parity tests."""
    source = ORACLE_DIR / "soap_oracle.c"
    target = ORACLE_DIR / "liboracle_soap.so"
    flags = ["gcc", "-std=c11", "-O2", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared", "-Wall"]
    if force or _stale(target, [source]):
        _run([*flags, str(source), "-o", str(target), "-lm"])
    extended = ORACLE_DIR / "liboracle_soap_ext.so"
    if force or _stale(extended, [source]):
        _run([*flags, "-DORACLE_EXTENDED", str(source), "-o", str(extended), "-lm"])
    return target


def _includes(root: Path) -> list[str]:
    return [f"-I{root / 'cpp' / 'include'}", f"-I{root / 'cpp' / 'src'}",
            f"-I{root / 'cpp' / 'src' / 'common'}", f"-I{root / 'cpp' / 'src' / 'standalone'}"]


def build_ref_soap(root: Path, force: bool = False) -> Path:
    target = REF_OUT / "libref_soap.so"
    sources = [root / s for s in _SOAP_SOURCES] + [ORACLE_DIR / "ref_shim.cpp", Path(__file__).resolve()]
    if force or _stale(target, sources):
        REF_OUT.mkdir(parents=True, exist_ok=True)
        _run(["g++", *_REF_FLAGS, "-shared", *_includes(root), *map(str, sources[:-1]),
              "-o", str(target)])
    return target


def build_ref_native(root: Path, force: bool = False) -> Path:
    import pybind11

    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    target = REF_OUT / "pkg" / f"_native{suffix}"
    sources = [root / s for s in _NATIVE_SOURCES] + [ORACLE_DIR / "ref_cblas" / "cblas_shim.cpp"]
    if not force and not _stale(target, sources):
        return target
    obj_dir = REF_OUT / "obj"
    obj_dir.mkdir(parents=True, exist_ok=True)
    target.parent.mkdir(parents=True, exist_ok=True)
    flags = [*_REF_FLAGS, *_includes(root), f"-I{ORACLE_DIR / 'ref_cblas'}",
             f"-I{pybind11.get_include()}", f"-I{sysconfig.get_paths()['include']}",
             "-fvisibility=hidden"]

    def compile_one(source: Path) -> Path:
        obj = obj_dir / (source.stem + ".o")
        if force or _stale(obj, [source]):
            _run(["g++", *flags, "-c", str(source), "-o", str(obj)])
        return obj

    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        objects = list(pool.map(compile_one, sources))
    _run(["g++", "-shared", "-fopenmp", *map(str, objects), "-o", str(target)])
    return target


def stage_reference_package(root: Path, native: Path) -> Path:
    """Copy the reference's Python package into baseline/_ref with its compiled
    ``_native`` beside it (weights and caches left out)."""
    dest = BASELINE_REF / "mdescriptor"
    if dest.exists():
        shutil.rmtree(dest)
    shutil.copytree(root / "src" / "mdescriptor", dest,
                    ignore=shutil.ignore_patterns("__pycache__", "*.pyc", "*.pt", "nep89*.txt"))
    # The source placeholder would shadow nothing once the extension sits beside it,
    # but remove it so that the compiled module is the only candidate.
    (dest / "_native.py").unlink(missing_ok=True)
    shutil.copy2(native, dest / native.name)
    return dest


def build_all(force: bool = False) -> None:
    build_c_oracle(force)
    root = reference_root()
    if root is None:
        print("build_oracle: MDSOAP_REFERENCE_ROOT is unset; using the prebuilt oracle/_ref and baseline/_ref")
        return
    build_ref_soap(root, force)
    native = build_ref_native(root, force)
    stage_reference_package(root, native)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print("oracle built")
