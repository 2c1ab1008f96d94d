"""In-tree build of the engine: ``python -m mdescriptor_b200.build``.

* ``lib/libmdsoap.so``  -- the CUDA engine + C ABI, nvcc for sm_100a only
  (``csrc/mdsoap.cu`` and the kernel translation units ``csrc/k_*.cu``,
  compiled in parallel into ``lib/obj/``);
* ``lib/libmdsynth.so`` -- the seeded generator of the large benchmark
  batches (``csrc/synth.c``, gcc + OpenMP; input generation only);
* ``plugin/_cuda<EXT_SUFFIX>`` -- the pybind11 ``mdescriptor._cuda`` drop-in
  (point ``MDESCRIPTOR_CUDA_PLUGIN_DIR`` at ``plugin/``), linked to
  ``libmdsoap.so`` through an $ORIGIN rpath.

Both are written next to the sources so that they travel with the
repository; nothing is installed into site-packages.
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
INCLUDE = PACKAGE.parent / "include"
LIB = PACKAGE / "lib" / "libmdsoap.so"
PLUGIN_DIR = PACKAGE / "plugin"
OBJ_DIR = PACKAGE / "lib" / "obj"
SYNTH = PACKAGE / "lib" / "libmdsynth.so"
PLUGIN = PLUGIN_DIR / f"_cuda{sysconfig.get_config_var('EXT_SUFFIX')}"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(home) / "bin" / "nvcc"
    return str(candidate) if candidate.is_file() else "nvcc"


def _run(cmd: list[str]) -> str:
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{result.stdout}\n{result.stderr}")
    return result.stdout + result.stderr


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(s.stat().st_mtime > mtime for s in sources)


def _compile_object(source: Path, obj: Path, extra: list[str]) -> str:
    obj.parent.mkdir(parents=True, exist_ok=True)
    return _run([_nvcc(), *NVCC_FLAGS, *extra, "-c", str(source), "-o", str(obj)])


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile mdsoap.cu (host runtime, C ABI, non-template kernels) and the
    kernel translation units k_*.cu in parallel, then link libmdsoap.so."""
    from concurrent.futures import ThreadPoolExecutor

    units = [CSRC / "mdsoap.cu", *sorted(CSRC.glob("k_*.cu"))]
    headers = [*sorted(CSRC.glob("*.cuh")), INCLUDE / "mdsoap.h"]
    if force or _stale(LIB, [*units, *headers]):
        LIB.parent.mkdir(parents=True, exist_ok=True)
        extra = ["-Xptxas", "-v"] if verbose else []
        objects = [OBJ_DIR / (u.stem + ".o") for u in units]
        jobs = max(1, min(len(units), os.cpu_count() or 1))
        with ThreadPoolExecutor(jobs) as pool:
            logs = list(pool.map(lambda uo: _compile_object(uo[0], uo[1], extra), zip(units, objects)))
        _run([_nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", *map(str, objects), "-o", str(LIB)])
        if verbose:
            print("\n".join(logs))
    return LIB


def build_plugin(force: bool = False) -> Path:
    import pybind11

    sources = [CSRC / "cuda_plugin.cpp", INCLUDE / "mdsoap.h", LIB]
    if force or _stale(PLUGIN, sources):
        PLUGIN_DIR.mkdir(parents=True, exist_ok=True)
        _run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
              f"-I{pybind11.get_include()}", f"-I{sysconfig.get_paths()['include']}",
              str(CSRC / "cuda_plugin.cpp"), f"-L{LIB.parent}", "-lmdsoap",
              "-Wl,-rpath,$ORIGIN/../lib", "-o", str(PLUGIN)])
    return PLUGIN


def build_synth(force: bool = False) -> Path:
    """The seeded batch generator for the large benchmark configs (host C)."""
    source = CSRC / "synth.c"
    if force or _stale(SYNTH, [source]):
        SYNTH.parent.mkdir(parents=True, exist_ok=True)
        _run(["gcc", "-O2", "-std=c99", "-fopenmp", "-shared", "-fPIC", str(source), "-o", str(SYNTH), "-lm"])
    return SYNTH


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_library(force, verbose)
    build_plugin(force)
    build_synth(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(f"built {LIB} and {PLUGIN}")
