"""Python front-end of the B200 SOAP engine (over the C ABI in include/mdsoap.h).

``Soap`` mirrors the constructor arguments and output layout of MDescriptor's
``SoapKernel`` (src/mdescriptor/descriptors/_kernels/core.py:156-304) for the
GTO / compression-off path: ``compute(batch)`` returns the (rows, F) matrix
that ``SoapKernel.compute(...).values`` holds, in the requested dtype.
"""

from __future__ import annotations

import ctypes
from typing import Any, Callable, Sequence

import numpy as np

from . import _lib
from ._lib import BatchView, CancelFn, LocalParams, Params, last_error, lib, raise_for
from .basis import basis_gto, basis_polynomial, feature_count, graph_cutoff, labels


def _contiguous(batch) -> tuple[np.ndarray, ...]:
    numbers = np.ascontiguousarray(batch.numbers, dtype=np.int32)
    positions = np.ascontiguousarray(batch.positions, dtype=np.float64).reshape(-1, 3)
    cells = np.ascontiguousarray(batch.cells, dtype=np.float64).reshape(-1, 3, 3)
    pbc = np.ascontiguousarray(batch.pbc, dtype=np.int32).reshape(-1, 3)
    offsets = np.ascontiguousarray(batch.offsets, dtype=np.int64)
    return numbers, positions, cells, pbc, offsets


def host_view(arrays: Sequence[np.ndarray]) -> BatchView:
    numbers, positions, cells, pbc, offsets = arrays
    return BatchView(numbers.ctypes.data, positions.ctypes.data, cells.ctypes.data, pbc.ctypes.data,
                     offsets.ctypes.data, int(offsets.shape[0]) - 1, int(numbers.shape[0]))


def device_view(numbers: int, positions: int, cells: int, pbc: int, offsets: int, structures: int,
                atoms: int) -> BatchView:
    """Batch view over device pointers (e.g. ``tensor.data_ptr()``)."""
    return BatchView(numbers, positions, cells, pbc, offsets, structures, atoms)


class Soap:
    """GTO SOAP power spectrum (compression off) computed on B200 GPUs.

    Parameters follow ``SoapKernel``: species (declared order), r_cut, n_max,
    l_max, sigma, average ("off" | "inner" | "outer"), dtype ("float32" |
    "float64"), species_weights (the ``compression["species_weighting"]``
    mapping, optional), compression ("off" | "mu2" | "mu1nu1" | "crossover"),
    weighting (the reference's weighting dict), rbf ("gto" | "polynomial").
    ``alphas``/``betas`` (GTO) and ``radial_grid``/``radial_weights``/
    ``radial_values`` (polynomial) default to the reference basis
    constructions (``basis_gto``, ``basis_polynomial``); the plugin passes the
    adapter's payload.
    """

    def __init__(self, species: Sequence[int], r_cut: float = 6.0, n_max: int = 8, l_max: int = 6,
                 sigma: float = 1.0, average: str = "inner", dtype: str = "float64",
                 species_weights: dict | Sequence[float] | None = None,
                 alphas: np.ndarray | None = None, betas: np.ndarray | None = None,
                 compression: str = "off", weighting: dict | None = None, rbf: str = "gto",
                 radial_grid: np.ndarray | None = None, radial_weights: np.ndarray | None = None,
                 radial_values: np.ndarray | None = None) -> None:
        self.species = tuple(int(z) for z in species)
        self.r_cut = float(r_cut)
        self.n_max = int(n_max)
        self.l_max = int(l_max)
        self.sigma = float(sigma)
        if average not in _lib.AVERAGE:
            raise ValueError("average must be 'off', 'inner', or 'outer'")
        self.average = average
        if dtype not in ("float32", "float64"):
            raise ValueError("dtype must be 'float32' or 'float64'")
        self.dtype = np.dtype(dtype)
        if rbf not in ("gto", "polynomial"):
            raise ValueError("rbf must be 'gto' or 'polynomial'")
        self.rbf = rbf
        if rbf == "gto":
            if alphas is None or betas is None:
                alphas, betas = basis_gto(self.r_cut, self.n_max, self.l_max)
            self._alphas = np.ascontiguousarray(alphas, dtype=np.float64).ravel()
            self._betas = np.ascontiguousarray(betas, dtype=np.float64).ravel()
            self._grid = self._grid_weights = self._grid_values = np.zeros(0)
        else:
            if radial_grid is None or radial_weights is None or radial_values is None:
                radial_grid, radial_weights, radial_values = basis_polynomial(self.r_cut, self.n_max)
            self._grid = np.ascontiguousarray(radial_grid, dtype=np.float64).ravel()
            self._grid_weights = np.ascontiguousarray(radial_weights, dtype=np.float64).ravel()
            self._grid_values = np.ascontiguousarray(radial_values, dtype=np.float64).ravel()
            if self._grid_weights.size != self._grid.size or self._grid_values.size != self.n_max * self._grid.size:
                raise ValueError("invalid SOAP polynomial radial basis size")
            self._alphas = self._betas = np.zeros(0)
        self._species = np.asarray(self.species, dtype=np.int32)
        if species_weights is None:
            self._weights = None
        elif isinstance(species_weights, dict):
            if set(species_weights) != set(self.species):
                raise ValueError("species_weighting must contain exactly the configured species")
            self._weights = np.asarray([float(species_weights[z]) for z in self.species], np.float64)
        else:
            self._weights = np.ascontiguousarray(species_weights, dtype=np.float64)
        if compression not in _lib.COMPRESSION:
            raise ValueError("invalid SOAP compression mode")
        self.compression = compression
        self.weighting = dict(weighting or {})
        function = self.weighting.get("function")
        if function not in _lib.WEIGHTING:
            raise ValueError("SOAP weighting function must be 'poly', 'pow', or 'exp'")
        params = Params(
            len(self.species), self._species.ctypes.data,
            None if self._weights is None else self._weights.ctypes.data,
            self.r_cut, self.sigma, self.n_max, self.l_max, self._alphas.ctypes.data,
            self._betas.ctypes.data, _lib.AVERAGE[average],
            _lib.FLOAT64 if self.dtype == np.float64 else _lib.FLOAT32,
            _lib.COMPRESSION[compression], _lib.WEIGHTING[function], 1 if "w0" in self.weighting else 0,
            float(self.weighting.get("r0", 1.0)), float(self.weighting.get("c", 1.0)),
            float(self.weighting.get("d", 0.0)), float(self.weighting.get("m", 1.0)),
            float(self.weighting.get("w0", 1.0)),
            0 if rbf == "gto" else 1, int(self._grid.size),
            self._grid.ctypes.data if self._grid.size else None,
            self._grid_weights.ctypes.data if self._grid.size else None,
            self._grid_values.ctypes.data if self._grid.size else None)
        handle = ctypes.c_void_p()
        raise_for(lib.mdsoap_plan_create(ctypes.byref(params), ctypes.byref(handle)))
        self._plan = handle
        self.feature_count = int(lib.mdsoap_plan_feature_count(self._plan))
        assert self.feature_count == feature_count(len(self.species), self.n_max, self.l_max, compression)

    @property
    def cutoff(self) -> float:
        return graph_cutoff(self.r_cut, self.sigma)

    def labels(self) -> tuple[str, ...]:
        return labels(self.species, self.n_max, self.l_max, self.compression)

    def rows(self, batch) -> int:
        return int(batch.offsets.shape[0]) - 1 if self.average != "off" else int(batch.offsets[-1])

    def compute(self, batch, devices: Sequence[int] | None = None, out: np.ndarray | None = None,
                cancelled: Callable[[], bool] | None = None) -> np.ndarray:
        """End to end: host batch in, host (rows, F) matrix out (C ABI ``mdsoap_compute``)."""
        arrays = _contiguous(batch)
        view = host_view(arrays)
        rows = self.rows(batch)
        if out is None:
            out = np.empty((rows, self.feature_count), dtype=self.dtype)
        elif out.shape != (rows, self.feature_count) or out.dtype != self.dtype or not out.flags.c_contiguous:
            raise ValueError("out has the wrong shape, dtype or layout")
        ids = None
        count = 0
        if devices:
            ids = np.ascontiguousarray(devices, dtype=np.int32)
            count = len(ids)
        callback = None if cancelled is None else CancelFn(lambda _ctx: 1 if cancelled() else 0)
        status = lib.mdsoap_compute(self._plan, ctypes.byref(view), out.ctypes.data if out.size else None,
                                    None if ids is None else ids.ctypes.data, count,
                                    ctypes.cast(callback, ctypes.c_void_p) if callback else None, None)
        raise_for(status)
        return out

    def compute_csr(self, batch, device: int = 0):
        """Sparse rows (C ABI ``mdsoap_compute_csr``): a ``scipy.sparse.csr_matrix``
        with exact zeros dropped, equal to ``csr_matrix(self.compute(batch))``
        (the ``OutputOptions(sparse=True)`` representation), built on the device
        so that only the nonzeros cross PCIe."""
        import scipy.sparse

        arrays = _contiguous(batch)
        view = host_view(arrays)
        handle = ctypes.c_void_p()
        raise_for(lib.mdsoap_compute_csr(self._plan, ctypes.byref(view), int(device), ctypes.byref(handle)))
        try:
            rows, cols, nnz = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
            raise_for(lib.mdsoap_csr_info(handle, ctypes.byref(rows), ctypes.byref(cols), ctypes.byref(nnz)))
            indptr = np.empty(rows.value + 1, np.int64)
            indices = np.empty(nnz.value, np.int32)
            data = np.empty(nnz.value, self.dtype)
            raise_for(lib.mdsoap_csr_copy(handle, indptr.ctypes.data, indices.ctypes.data, data.ctypes.data))
        finally:
            lib.mdsoap_csr_destroy(handle)
        return scipy.sparse.csr_matrix((data, indices, indptr), shape=(rows.value, cols.value))

    def compute_device(self, view: BatchView, out_ptr: int, device: int = 0, stream: int = 0) -> None:
        """Enqueue the pipeline on device memory (C ABI ``mdsoap_compute_device``)."""
        raise_for(lib.mdsoap_compute_device(self._plan, ctypes.byref(view), out_ptr or None, int(device),
                                            stream or None))

    def set_timing(self, enable: bool) -> None:
        raise_for(lib.mdsoap_plan_set_timing(self._plan, 1 if enable else 0))

    def kernel(self) -> str:
        """Name and template arguments of the centre kernel this plan launches."""
        return lib.mdsoap_plan_kernel(self._plan).decode()

    def launch_count(self) -> int:
        """Kernels this plan has launched so far (all devices, all entry points)."""
        value = ctypes.c_int64()
        raise_for(lib.mdsoap_plan_launch_count(self._plan, ctypes.byref(value)))
        return int(value.value)

    def last_timing(self, device: int = 0) -> tuple[float, float, float]:
        """(bin_ms, center_ms, structure_ms) of the last timed ``compute_device`` call."""
        values = (ctypes.c_double * 3)()
        raise_for(lib.mdsoap_plan_last_timing(self._plan, int(device), ctypes.byref(values, 0),
                                              ctypes.byref(values, 8), ctypes.byref(values, 16)))
        return values[0], values[1], values[2]

    def last_timing_split(self, device: int = 0) -> tuple[float, float]:
        """(expansion_ms, tail_ms) of the last timed call (tail 0 for a fused tail)."""
        values = (ctypes.c_double * 2)()
        raise_for(lib.mdsoap_plan_last_timing_split(self._plan, int(device), ctypes.byref(values, 0),
                                                    ctypes.byref(values, 8)))
        return values[0], values[1]

    def check(self, device: int = 0, stream: int = 0) -> None:
        raise_for(lib.mdsoap_plan_check(self._plan, int(device), stream or None))

    def close(self) -> None:
        if getattr(self, "_plan", None):
            lib.mdsoap_plan_destroy(self._plan)
            self._plan = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


def neighbor_graph(batch, cutoff: float, device: int = 0):
    """GPU neighbour graph (C ABI ``mdsoap_graph_build``):
    (offsets, atoms, shifts, displacements, distance2) like the reference's
    ``build_neighbor_graph`` over the whole batch (cpp/src/common/neighbor.cpp:703-768)."""
    arrays = _contiguous(batch)
    view = host_view(arrays)
    handle = ctypes.c_void_p()
    raise_for(lib.mdsoap_graph_build(ctypes.byref(view), float(cutoff), int(device), ctypes.byref(handle)))
    try:
        pairs = int(lib.mdsoap_graph_pairs(handle))
        atoms_total = int(arrays[4][-1])
        offsets = np.zeros(atoms_total + 1, np.int64)
        atoms = np.zeros(pairs, np.int32)
        shifts = np.zeros((pairs, 3), np.int32)
        displacements = np.zeros((pairs, 3), np.float64)
        distance2 = np.zeros(pairs, np.float64)
        raise_for(lib.mdsoap_graph_copy(handle, offsets.ctypes.data, atoms.ctypes.data, shifts.ctypes.data,
                                        displacements.ctypes.data, distance2.ctypes.data))
    finally:
        lib.mdsoap_graph_destroy(handle)
    return offsets, atoms, shifts, displacements, distance2


def neighbor_list(batch, cutoff: float, full_neighbor_list: bool = True, self_pairs: bool = False,
                  device: int = 0):
    """The NeighborList descriptor on the GPU (C ABI ``mdsoap_neighbor_list``):
    (records (P, 5), values (P, 4), row_offsets (S+1,)) like the reference's
    compute_neighbor_list split into pair records and features
    (cpp/src/standalone/neighbor_list.cpp:15-75, _kernels/local.py:73-112)."""
    arrays = _contiguous(batch)
    view = host_view(arrays)
    handle = ctypes.c_void_p()
    raise_for(lib.mdsoap_neighbor_list(ctypes.byref(view), float(cutoff), 1 if full_neighbor_list else 0,
                                       1 if self_pairs else 0, int(device), ctypes.byref(handle)))
    try:
        pairs = int(lib.mdsoap_pairs_count(handle))
        records = np.zeros((pairs, 5), np.float64)
        values = np.zeros((pairs, 4), np.float64)
        row_offsets = np.zeros(int(arrays[4].shape[0]), np.int64)
        raise_for(lib.mdsoap_pairs_copy(handle, records.ctypes.data, values.ctypes.data, row_offsets.ctypes.data))
    finally:
        lib.mdsoap_pairs_destroy(handle)
    return records, values, row_offsets


LOCAL_KINDS = {"SphericalExpansion": 0, "SoapRadialSpectrum": 2, "SoapPowerSpectrum": 3}


def _local_params(name: str, species: Sequence[int], cutoff: float, density_width: float, max_radial: int,
                  max_angular: int) -> tuple[LocalParams, np.ndarray]:
    if name not in LOCAL_KINDS:
        raise ValueError(f"unknown local spectrum {name!r}; expected one of {sorted(LOCAL_KINDS)}")
    sp = np.ascontiguousarray(np.asarray(tuple(int(z) for z in species), dtype=np.int32))
    params = LocalParams(LOCAL_KINDS[name], int(max_radial), int(max_angular), int(sp.shape[0]),
                         sp.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), float(cutoff), float(density_width))
    return params, sp


def local_feature_count(name: str, species: Sequence[int], max_radial: int = 6, max_angular: int = 4) -> int:
    """Row width of a local spectrum (C ABI ``mdsoap_local_feature_count``;
    cpp/src/common/local_layout.hpp:115-130)."""
    params, _keep = _local_params(name, species, 6.0, 0.3, max_radial, max_angular)
    count = int(lib.mdsoap_local_feature_count(ctypes.byref(params)))
    if count < 0:
        raise ValueError(last_error())
    return count


def local_spectrum(name: str, batch, species: Sequence[int], cutoff: float = 6.0, density_width: float = 0.3,
                   max_radial: int = 6, max_angular: int = 4, device: int = 0) -> np.ndarray:
    """SphericalExpansion, SoapRadialSpectrum or SoapPowerSpectrum rows
    float64[atoms, F] on the GPU (C ABI ``mdsoap_local_compute``), the values
    of the reference's ``compute_spherical_expansion``
    (cpp/src/standalone/spherical_expansion.cpp:124-206) for the same options."""
    params, _keep = _local_params(name, species, cutoff, density_width, max_radial, max_angular)
    count = int(lib.mdsoap_local_feature_count(ctypes.byref(params)))
    if count < 0:
        raise ValueError(last_error())
    arrays = _contiguous(batch)
    view = host_view(arrays)
    out = np.zeros((int(arrays[4][-1]), count), np.float64)
    raise_for(lib.mdsoap_local_compute(ctypes.byref(params), ctypes.byref(view), out.ctypes.data, int(device)))
    return out


def probe_fp64_fma(device: int = 0) -> float:
    """Measured fp64 FMA throughput of one device, TFLOP/s."""
    value = ctypes.c_double()
    raise_for(lib.mdsoap_probe_fp64_fma(int(device), ctypes.byref(value)))
    return float(value.value)


def probe_exp(x, device: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """The engine's exp() and CUDA's exp() of the same arguments on one device."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    ours = np.empty_like(x)
    cuda = np.empty_like(x)
    raise_for(lib.mdsoap_probe_exp(int(device), x.ctypes.data, x.size, ours.ctypes.data, cuda.ctypes.data))
    return ours, cuda


def probe_radial(form: int, u, e, pref, device: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """The kernels' radial factor pref * exp(-e u) in form 0 (float64 rows), 1
    (float32 rows, one-kernel walk) or 2 (float32 rows, expansion-only kernel),
    and pref * CUDA's exp(-e u), on one device."""
    u, e, pref = (np.ascontiguousarray(a, dtype=np.float64) for a in np.broadcast_arrays(u, e, pref))
    ours = np.empty_like(u)
    cuda = np.empty_like(u)
    raise_for(lib.mdsoap_probe_radial(int(device), int(form), u.ctypes.data, e.ctypes.data, pref.ctypes.data, u.size,
                                      ours.ctypes.data, cuda.ctypes.data))
    return ours, cuda


def device_count() -> int:
    return int(lib.mdsoap_device_count())


def options_from_payload(options: dict[str, Any]) -> dict[str, Any]:
    """Decode the adapter's backend options (src/mdescriptor/core/adapter.py:529-603)
    into ``Soap`` keyword arguments; used by tests that mimic the plugin seam."""
    payload = options["_cuda_payload"]["radial_basis"]
    output = options.get("output") or {}
    compression = options.get("compression") or {}
    rbf = options.get("rbf", "gto")
    basis = (dict(alphas=payload["alphas"], betas=payload["betas"]) if rbf == "gto" else
             dict(radial_grid=payload["radial_grid"], radial_weights=payload["radial_weights"],
                  radial_values=payload["radial_values"]))
    return dict(species=options["species"], r_cut=options.get("r_cut", 6.0), n_max=options.get("n_max", 8),
                l_max=options.get("l_max", 6), sigma=options.get("sigma", 1.0),
                average=options.get("average", "inner"), dtype=output.get("dtype", "float64"),
                species_weights=compression.get("species_weighting"),
                compression=compression.get("mode", "off"), weighting=options.get("weighting"),
                rbf=rbf, **basis)
