"""ctypes binding of ``libmdsoap.so`` (the C ABI declared in include/mdsoap.h).

The library is built in-tree by ``mdescriptor_b200/build.py`` into
``mdescriptor_b200/lib/``.  There is no fallback: if the library is missing,
importing this module raises ImportError, so nothing can silently run a CPU
path in its place.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

# MDSOAP_LIBRARY may point at another build of the same ABI (e.g. a debug build).
LIB_PATH = Path(os.environ.get("MDSOAP_LIBRARY") or Path(__file__).resolve().parent / "lib" / "libmdsoap.so")

ABI_VERSION = 3  # MDSOAP_ABI_VERSION: layout of Params below

OK = 0
INVALID_ARGUMENT = 1
DEVICE_UNAVAILABLE = 2
OUT_OF_MEMORY = 3
CANCELLED = 4
CAPACITY_OVERFLOW = 5
INTERNAL = 6

NOALLOC_SCRATCH_BYTES = 32 << 20  # MDSOAP_NOALLOC_SCRATCH_BYTES

FLOAT32 = 0
FLOAT64 = 1
AVERAGE = {"off": 0, "inner": 1, "outer": 2}
COMPRESSION = {"off": 0, "mu2": 1, "mu1nu1": 2, "crossover": 3}
WEIGHTING = {None: 0, "poly": 1, "pow": 2, "exp": 3}

_P = ctypes.c_void_p
CancelFn = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p)


class Params(ctypes.Structure):
    _fields_ = [
        ("n_species", ctypes.c_int32),
        ("species", _P),
        ("species_weights", _P),
        ("r_cut", ctypes.c_double),
        ("sigma", ctypes.c_double),
        ("n_max", ctypes.c_int32),
        ("l_max", ctypes.c_int32),
        ("alphas", _P),
        ("betas", _P),
        ("average", ctypes.c_int32),
        ("output_dtype", ctypes.c_int32),
        ("compression", ctypes.c_int32),
        ("weighting_function", ctypes.c_int32),
        ("weighting_has_w0", ctypes.c_int32),
        ("weighting_r0", ctypes.c_double),
        ("weighting_c", ctypes.c_double),
        ("weighting_d", ctypes.c_double),
        ("weighting_m", ctypes.c_double),
        ("weighting_w0", ctypes.c_double),
        ("radial_basis", ctypes.c_int32),
        ("radial_grid_size", ctypes.c_int32),
        ("radial_grid", _P),
        ("radial_weights", _P),
        ("radial_values", _P),
    ]


class LocalParams(ctypes.Structure):
    """``mdsoap_local_params`` (include/mdsoap.h)."""

    _fields_ = [
        ("kind", ctypes.c_int32),
        ("max_radial", ctypes.c_int32),
        ("max_angular", ctypes.c_int32),
        ("n_species", ctypes.c_int32),
        ("species", ctypes.POINTER(ctypes.c_int32)),
        ("cutoff", ctypes.c_double),
        ("density_width", ctypes.c_double),
    ]


class BatchView(ctypes.Structure):
    _fields_ = [
        ("numbers", _P),
        ("positions", _P),
        ("cells", _P),
        ("pbc", _P),
        ("offsets", _P),
        ("structures", ctypes.c_int64),
        ("atoms", ctypes.c_int64),
    ]


def _load() -> ctypes.CDLL:
    if not LIB_PATH.is_file():
        raise ImportError(
            f"mdsoap CUDA library not built ({LIB_PATH}); run `python -m mdescriptor_b200.build`"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.mdsoap_abi_version.restype = ctypes.c_int32
    if lib.mdsoap_abi_version() != ABI_VERSION:
        raise ImportError(f"{LIB_PATH} has C ABI {lib.mdsoap_abi_version()}, this binding needs {ABI_VERSION}; "
                          "rebuild with `python -m mdescriptor_b200.build`")
    lib.mdsoap_last_error.restype = ctypes.c_char_p
    lib.mdsoap_abi_version.restype = ctypes.c_int32
    lib.mdsoap_device_count.restype = ctypes.c_int32
    lib.mdsoap_plan_create.argtypes = [ctypes.POINTER(Params), ctypes.POINTER(_P)]
    lib.mdsoap_plan_create.restype = ctypes.c_int
    lib.mdsoap_plan_destroy.argtypes = [_P]
    lib.mdsoap_plan_destroy.restype = None
    lib.mdsoap_plan_feature_count.argtypes = [_P]
    lib.mdsoap_plan_feature_count.restype = ctypes.c_int64
    lib.mdsoap_plan_rows.argtypes = [_P, ctypes.POINTER(BatchView)]
    lib.mdsoap_plan_rows.restype = ctypes.c_int64
    lib.mdsoap_neighbor_list.argtypes = [ctypes.POINTER(BatchView), ctypes.c_double, ctypes.c_int32, ctypes.c_int32,
                                         ctypes.c_int32, ctypes.POINTER(_P)]
    lib.mdsoap_neighbor_list.restype = ctypes.c_int
    lib.mdsoap_pairs_count.argtypes = [_P]
    lib.mdsoap_pairs_count.restype = ctypes.c_int64
    lib.mdsoap_pairs_copy.argtypes = [_P, _P, _P, _P]
    lib.mdsoap_pairs_copy.restype = ctypes.c_int
    lib.mdsoap_pairs_destroy.argtypes = [_P]
    lib.mdsoap_pairs_destroy.restype = None
    lib.mdsoap_plan_last_timing_split.argtypes = [_P, ctypes.c_int32, _P, _P]
    lib.mdsoap_plan_last_timing_split.restype = ctypes.c_int
    lib.mdsoap_plan_kernel.argtypes = [_P]
    lib.mdsoap_plan_kernel.restype = ctypes.c_char_p
    lib.mdsoap_compute.argtypes = [_P, ctypes.POINTER(BatchView), _P, _P, ctypes.c_int32, _P, _P]
    lib.mdsoap_compute.restype = ctypes.c_int
    lib.mdsoap_compute_device.argtypes = [_P, ctypes.POINTER(BatchView), _P, ctypes.c_int32, _P]
    lib.mdsoap_compute_device.restype = ctypes.c_int
    lib.mdsoap_plan_check.argtypes = [_P, ctypes.c_int32, _P]
    lib.mdsoap_plan_check.restype = ctypes.c_int
    lib.mdsoap_compute_csr.argtypes = [_P, ctypes.POINTER(BatchView), ctypes.c_int32, ctypes.POINTER(_P)]
    lib.mdsoap_compute_csr.restype = ctypes.c_int
    lib.mdsoap_csr_info.argtypes = [_P, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64),
                                    ctypes.POINTER(ctypes.c_int64)]
    lib.mdsoap_csr_info.restype = ctypes.c_int
    lib.mdsoap_csr_copy.argtypes = [_P, _P, _P, _P]
    lib.mdsoap_csr_copy.restype = ctypes.c_int
    lib.mdsoap_csr_destroy.argtypes = [_P]
    lib.mdsoap_csr_destroy.restype = None
    lib.mdsoap_compute_device_noalloc.argtypes = [_P, ctypes.POINTER(BatchView), _P, ctypes.c_int32, _P]
    lib.mdsoap_compute_device_noalloc.restype = ctypes.c_int
    lib.mdsoap_plan_set_timing.argtypes = [_P, ctypes.c_int32]
    lib.mdsoap_plan_set_timing.restype = ctypes.c_int
    lib.mdsoap_plan_last_timing.argtypes = [_P, ctypes.c_int32, _P, _P, _P]
    lib.mdsoap_plan_last_timing.restype = ctypes.c_int
    lib.mdsoap_plan_launch_count.argtypes = [_P, _P]
    lib.mdsoap_plan_launch_count.restype = ctypes.c_int
    lib.mdsoap_probe_exp.argtypes = [ctypes.c_int32, _P, ctypes.c_int64, _P, _P]
    lib.mdsoap_probe_exp.restype = ctypes.c_int
    lib.mdsoap_probe_radial.argtypes = [ctypes.c_int32, ctypes.c_int32, _P, _P, _P, ctypes.c_int64, _P, _P]
    lib.mdsoap_probe_radial.restype = ctypes.c_int
    lib.mdsoap_probe_bounded_wait.argtypes = [ctypes.c_int32, ctypes.c_uint64]
    lib.mdsoap_probe_bounded_wait.restype = ctypes.c_int
    lib.mdsoap_probe_fp64_fma.argtypes = [ctypes.c_int32, _P]
    lib.mdsoap_probe_fp64_fma.restype = ctypes.c_int
    lib.mdsoap_graph_build.argtypes = [ctypes.POINTER(BatchView), ctypes.c_double, ctypes.c_int32, ctypes.POINTER(_P)]
    lib.mdsoap_graph_build.restype = ctypes.c_int
    lib.mdsoap_graph_pairs.argtypes = [_P]
    lib.mdsoap_graph_pairs.restype = ctypes.c_int64
    lib.mdsoap_graph_copy.argtypes = [_P, _P, _P, _P, _P, _P]
    lib.mdsoap_graph_copy.restype = ctypes.c_int
    lib.mdsoap_graph_destroy.argtypes = [_P]
    lib.mdsoap_graph_destroy.restype = None
    lib.mdsoap_local_feature_count.argtypes = [ctypes.POINTER(LocalParams)]
    lib.mdsoap_local_feature_count.restype = ctypes.c_int64
    lib.mdsoap_local_compute.argtypes = [ctypes.POINTER(LocalParams), ctypes.POINTER(BatchView), _P, ctypes.c_int32]
    lib.mdsoap_local_compute.restype = ctypes.c_int
    return lib


lib = _load()

# Every symbol the header declares (checked by the CPU test suite).
EXPORTED = (
    "mdsoap_last_error",
    "mdsoap_abi_version",
    "mdsoap_device_count",
    "mdsoap_plan_create",
    "mdsoap_plan_destroy",
    "mdsoap_plan_feature_count",
    "mdsoap_plan_rows",
    "mdsoap_plan_kernel",
    "mdsoap_plan_last_timing_split",
    "mdsoap_compute",
    "mdsoap_compute_device",
    "mdsoap_plan_check",
    "mdsoap_compute_csr",
    "mdsoap_csr_info",
    "mdsoap_csr_copy",
    "mdsoap_csr_destroy",
    "mdsoap_compute_device_noalloc",
    "mdsoap_host_buffer_acquire",
    "mdsoap_host_buffer_release",
    "mdsoap_plan_set_timing",
    "mdsoap_plan_last_timing",
    "mdsoap_plan_launch_count",
    "mdsoap_probe_exp",
    "mdsoap_probe_radial",
    "mdsoap_probe_fp64_fma",
    "mdsoap_probe_bounded_wait",
    "mdsoap_graph_build",
    "mdsoap_graph_pairs",
    "mdsoap_graph_copy",
    "mdsoap_graph_destroy",
    "mdsoap_neighbor_list",
    "mdsoap_pairs_count",
    "mdsoap_pairs_copy",
    "mdsoap_pairs_destroy",
    "mdsoap_local_feature_count",
    "mdsoap_local_compute",
)


class CudaUnavailable(ImportError):
    """No usable CUDA device or driver (maps to the reference's CudaUnavailable)."""


class CudaOutOfMemory(MemoryError):
    """Device allocation failed (maps to the reference's CudaOutOfMemory)."""


class CudaCancelledError(RuntimeError):
    """The computation was cancelled cooperatively."""


def last_error() -> str:
    return lib.mdsoap_last_error().decode()


def raise_for(status: int) -> None:
    """Map a status onto the reference plugin's exception classes
    (cpp/cuda/src/bindings.cu:18-20, src/mdescriptor/core/errors.py:83-113)."""
    if status == OK:
        return
    message = last_error()
    if status == INVALID_ARGUMENT:
        raise ValueError(message)
    if status == DEVICE_UNAVAILABLE:
        raise CudaUnavailable(message)
    if status == OUT_OF_MEMORY:
        raise CudaOutOfMemory(message)
    if status == CANCELLED:
        raise CudaCancelledError(message)
    raise RuntimeError(message)
