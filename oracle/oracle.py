"""TEST INFRASTRUCTURE ONLY -- ctypes front-end for the CPU checkers.

``OracleLib`` wraps ``oracle/liboracle_soap.so`` (the plain-C restatement in
``soap_oracle.c``); ``RefLib`` wraps ``oracle/_ref/libref_soap.so`` (the
reference's own ``compute_soap`` / ``build_neighbor_graph`` compiled from its
sources, see ``build_oracle.py``).  Both expose the same two calls:

* ``graph(batch, cutoff)`` -> ``(offsets, atoms, shifts, displacements, distance2)``
  with global atom indices, like ``build_neighbor_graph`` over a whole batch
  (cpp/src/common/neighbor.cpp:703-768);
* ``soap(batch, species, r_cut, n_max, l_max, sigma, alphas, betas, average)``
  -> fp64 ``(rows, F)`` features, like ``compute_soap``
  (cpp/src/standalone/soap.cpp:1149-1246).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this module.  The product package never does.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
_P = ctypes.c_void_p
_AVERAGE = {"off": 0, "inner": 1, "outer": 2}


def _ptr(array: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(array.ctypes.data)


def _batch_arrays(batch):
    numbers = np.ascontiguousarray(batch.numbers, dtype=np.int32)
    positions = np.ascontiguousarray(batch.positions, dtype=np.float64)
    cells = np.ascontiguousarray(batch.cells, dtype=np.float64)
    pbc = np.ascontiguousarray(batch.pbc, dtype=np.int32)
    offsets = np.ascontiguousarray(batch.offsets, dtype=np.int64)
    return numbers, positions, cells, pbc, offsets


_COMPRESSION = {"off": 0, "mu2": 1, "mu1nu1": 2, "crossover": 3}
_WEIGHTING = {None: 0, "poly": 1, "pow": 2, "exp": 3}


def feature_count(n_species: int, n_max: int, l_max: int, compression: str = "off") -> int:
    if compression == "mu2":
        return n_max * (n_max + 1) // 2 * (l_max + 1)
    if compression == "mu1nu1":
        return n_species * n_max * n_max * (l_max + 1)
    if compression == "crossover":
        return n_species * n_max * (n_max + 1) // 2 * (l_max + 1)
    width = n_species * n_max
    return width * (width + 1) // 2 * (l_max + 1)


def _weighting_args(weighting):
    """(function, has_w0, r0, c, d, m, w0) with SoapKernel._ensure_native's
    defaults (_kernels/core.py:247-254)."""
    w = dict(weighting or {})
    return (_WEIGHTING[w.get("function")], 1 if "w0" in w else 0, float(w.get("r0", 1.0)),
            float(w.get("c", 1.0)), float(w.get("d", 0.0)), float(w.get("m", 1.0)), float(w.get("w0", 1.0)))


_EX_TAIL = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int] + [ctypes.c_double] * 5 + [ctypes.c_int, _P]


class _Checker:
    prefix = ""

    def __init__(self, path: Path) -> None:
        if not path.is_file():
            raise FileNotFoundError(f"checker library {path} is not built")
        self.lib = ctypes.CDLL(str(path))
        p = self.prefix
        self._last_error = getattr(self.lib, f"{p}_last_error")
        self._last_error.restype = ctypes.c_char_p
        self._build = getattr(self.lib, f"{p}_graph_build")
        self._pairs = getattr(self.lib, f"{p}_graph_pairs")
        self._pairs.restype = ctypes.c_int64
        self._pairs.argtypes = [_P]
        self._copy = getattr(self.lib, f"{p}_graph_copy")
        self._copy.argtypes = [_P] * 6
        self._free = getattr(self.lib, f"{p}_graph_free")
        self._free.argtypes = [_P]
        self._soap = getattr(self.lib, f"{p}_soap_compute")

    def error(self) -> str:
        return self._last_error().decode()

    def _graph_handle(self, arrays, structures: int, cutoff: float):
        raise NotImplementedError

    def graph(self, batch, cutoff: float):
        arrays = _batch_arrays(batch)
        structures = len(arrays[4]) - 1
        handle = self._graph_handle(arrays, structures, cutoff)
        if not handle:
            raise ValueError(self.error())
        try:
            pairs = self._pairs(handle)
            atoms_total = int(arrays[4][-1])
            offsets = np.zeros(atoms_total + 1, np.int64)
            atoms = np.zeros(pairs, np.int32)
            shifts = np.zeros((pairs, 3), np.int32)
            displacements = np.zeros((pairs, 3), np.float64)
            distance2 = np.zeros(pairs, np.float64)
            self._copy(handle, _ptr(offsets), _ptr(atoms), _ptr(shifts), _ptr(displacements),
                       _ptr(distance2))
        finally:
            self._free(handle)
        return offsets, atoms, shifts, displacements, distance2


_RBF_TAIL = ([ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int] + [ctypes.c_double] * 5
             + [ctypes.c_int, ctypes.c_int, _P, _P, _P, ctypes.c_int, _P])


def _soap_rbf(checker, batch, species, r_cut, n_max, l_max, sigma, radial, average, species_weights,
              num_threads, compression, weighting):
    """<prefix>_soap_compute_rbf: radial = ("gto", alphas, betas) or
    ("polynomial", grid, weights, values)."""
    fn = getattr(checker.lib, f"{checker.prefix}_soap_compute_rbf")
    fn.restype = ctypes.c_int
    fn.argtypes = ([_P] * 5 + [ctypes.c_int64, _P, ctypes.c_int, _P, ctypes.c_double, ctypes.c_int,
                               ctypes.c_int, ctypes.c_double, _P, _P] + _RBF_TAIL)
    arrays = _batch_arrays(batch)
    structures = len(arrays[4]) - 1
    species = np.ascontiguousarray(species, dtype=np.int32)
    rows = structures if average != "off" else int(arrays[4][-1])
    out = np.zeros((rows, feature_count(len(species), n_max, l_max, compression)), np.float64)
    weights = None if species_weights is None else np.ascontiguousarray(species_weights, np.float64)
    kind, *tables = radial
    tables = [np.ascontiguousarray(t, np.float64) for t in tables]
    if kind == "gto":
        alphas, betas = tables
        basis = (_ptr(alphas), _ptr(betas))
        rbf = (0, 0, None, None, None)
    else:
        grid, grid_weights, values = tables
        basis = (None, None)
        rbf = (1, int(grid.size), _ptr(grid), _ptr(grid_weights), _ptr(values))
    status = fn(*map(_ptr, arrays), structures, _ptr(species), len(species),
                None if weights is None else _ptr(weights), float(r_cut), int(n_max), int(l_max), float(sigma),
                *basis, _AVERAGE[average], _COMPRESSION[compression], *_weighting_args(weighting), *rbf,
                int(num_threads), _ptr(out))
    if status:
        raise ValueError(checker.error())
    return out


class OracleLib(_Checker):
    """The plain-C restatement (soap_oracle.c)."""

    prefix = "oracle"

    def __init__(self, path: Path | None = None) -> None:
        super().__init__(path or ORACLE_DIR / "liboracle_soap.so")
        self._build.restype = _P
        self._build.argtypes = [_P] * 5 + [ctypes.c_int64, ctypes.c_double]
        self._soap.restype = ctypes.c_int
        self._soap.argtypes = ([_P] * 5 + [ctypes.c_int64, _P, ctypes.c_int, _P, ctypes.c_double,
                                ctypes.c_int, ctypes.c_int, ctypes.c_double, _P, _P, ctypes.c_int,
                                ctypes.c_int, _P])

        self._soap_ex = self.lib.oracle_soap_compute_ex
        self._soap_ex.restype = ctypes.c_int
        self._soap_ex.argtypes = ([_P] * 5 + [ctypes.c_int64, _P, ctypes.c_int, _P, ctypes.c_double,
                                   ctypes.c_int, ctypes.c_int, ctypes.c_double, _P, _P] + _EX_TAIL)

        self._rows = self.lib.oracle_soap_rows
        self._rows.restype = ctypes.c_int
        self._rows.argtypes = ([_P] * 5 + [ctypes.c_int64, _P, ctypes.c_int, _P, ctypes.c_double,
                                ctypes.c_int, ctypes.c_int, ctypes.c_double, _P, _P, _P, ctypes.c_int64, _P])

    def _graph_handle(self, arrays, structures, cutoff):
        return self._build(*map(_ptr, arrays), structures, cutoff)

    def soap_rows(self, batch, rows, species, r_cut, n_max, l_max, sigma, alphas, betas, species_weights=None):
        """Average-off feature rows of the selected atoms only (global indices)."""
        arrays = _batch_arrays(batch)
        structures = len(arrays[4]) - 1
        species = np.ascontiguousarray(species, dtype=np.int32)
        rows = np.ascontiguousarray(rows, dtype=np.int64)
        out = np.zeros((len(rows), feature_count(len(species), n_max, l_max)), np.float64)
        weights = None if species_weights is None else np.ascontiguousarray(species_weights, np.float64)
        alphas = np.ascontiguousarray(alphas, np.float64)
        betas = np.ascontiguousarray(betas, np.float64)
        status = self._rows(*map(_ptr, arrays), structures, _ptr(species), len(species),
                            None if weights is None else _ptr(weights), float(r_cut), int(n_max), int(l_max),
                            float(sigma), _ptr(alphas), _ptr(betas), _ptr(rows), len(rows), _ptr(out))
        if status:
            raise ValueError(self.error())
        return out

    def soap_poly(self, batch, species, r_cut, n_max, l_max, sigma, grid, grid_weights, values,
                  average="off", species_weights=None, num_threads=0, compression="off", weighting=None):
        """The polynomial radial basis (oracle_soap_compute_rbf)."""
        return _soap_rbf(self, batch, species, r_cut, n_max, l_max, sigma, ("polynomial", grid, grid_weights, values),
                         average, species_weights, num_threads, compression, weighting)

    def soap(self, batch, species, r_cut, n_max, l_max, sigma, alphas, betas, average="off",
             species_weights=None, num_threads=0, compression="off", weighting=None):
        arrays = _batch_arrays(batch)
        structures = len(arrays[4]) - 1
        species = np.ascontiguousarray(species, dtype=np.int32)
        rows = structures if average != "off" else int(arrays[4][-1])
        out = np.zeros((rows, feature_count(len(species), n_max, l_max, compression)), np.float64)
        weights = None if species_weights is None else np.ascontiguousarray(species_weights, np.float64)
        alphas = np.ascontiguousarray(alphas, np.float64)
        betas = np.ascontiguousarray(betas, np.float64)
        status = self._soap_ex(*map(_ptr, arrays), structures, _ptr(species), len(species),
                               None if weights is None else _ptr(weights), float(r_cut), int(n_max),
                               int(l_max), float(sigma), _ptr(alphas), _ptr(betas), _AVERAGE[average],
                               _COMPRESSION[compression], *_weighting_args(weighting), int(num_threads), _ptr(out))
        if status:
            raise ValueError(self.error())
        return out


class ExtendedLib(OracleLib):
    """The same restatement with its SOAP stage in x87 extended precision
    (liboracle_soap_ext.so, built with -DORACLE_EXTENDED): the exact value of
    the reference's algorithm on the same double graph and constants, up to
    ~1e-16 relative.  The float64 parity tests measure every double
    implementation's distance to it."""

    def __init__(self, path: Path | None = None) -> None:
        super().__init__(path or ORACLE_DIR / "liboracle_soap_ext.so")


class RefLib(_Checker):
    """The reference's own CPU path, compiled from its sources into oracle/_ref."""

    prefix = "ref"

    def __init__(self, path: Path | None = None) -> None:
        super().__init__(path or ORACLE_DIR / "_ref" / "libref_soap.so")
        self._build.restype = _P
        self._build.argtypes = [_P] * 5 + [ctypes.c_int64, ctypes.c_double, ctypes.c_int]
        self._soap.restype = ctypes.c_int
        self._soap.argtypes = ([_P] * 5 + [ctypes.c_int64, _P, ctypes.c_int, ctypes.c_double,
                                ctypes.c_int, ctypes.c_int, ctypes.c_double, _P, _P, ctypes.c_int,
                                ctypes.c_int, _P])

    def _graph_handle(self, arrays, structures, cutoff):
        return self._build(*map(_ptr, arrays), structures, cutoff, 1)

    def soap_poly(self, batch, species, r_cut, n_max, l_max, sigma, grid, grid_weights, values,
                  average="off", species_weights=None, num_threads=0, compression="off", weighting=None):
        """compute_soap with the polynomial radial basis (ref_soap_compute_rbf)."""
        return _soap_rbf(self, batch, species, r_cut, n_max, l_max, sigma, ("polynomial", grid, grid_weights, values),
                         average, species_weights, num_threads, compression, weighting)

    def soap_ex(self, batch, species, r_cut, n_max, l_max, sigma, alphas, betas, average="off",
                species_weights=None, num_threads=0, compression="off", weighting=None):
        """compute_soap with species weights, compression and weighting (ref_soap_compute_ex)."""
        fn = self.lib.ref_soap_compute_ex
        fn.restype = ctypes.c_int
        fn.argtypes = ([_P] * 5 + [ctypes.c_int64, _P, ctypes.c_int, _P, ctypes.c_double, ctypes.c_int,
                                   ctypes.c_int, ctypes.c_double, _P, _P] + _EX_TAIL)
        arrays = _batch_arrays(batch)
        structures = len(arrays[4]) - 1
        species = np.ascontiguousarray(species, dtype=np.int32)
        rows = structures if average != "off" else int(arrays[4][-1])
        out = np.zeros((rows, feature_count(len(species), n_max, l_max, compression)), np.float64)
        weights = None if species_weights is None else np.ascontiguousarray(species_weights, np.float64)
        alphas = np.ascontiguousarray(alphas, np.float64)
        betas = np.ascontiguousarray(betas, np.float64)
        status = fn(*map(_ptr, arrays), structures, _ptr(species), len(species),
                    None if weights is None else _ptr(weights), float(r_cut), int(n_max), int(l_max), float(sigma),
                    _ptr(alphas), _ptr(betas), _AVERAGE[average], _COMPRESSION[compression],
                    *_weighting_args(weighting), int(num_threads), _ptr(out))
        if status:
            raise ValueError(self.error())
        return out

    def soap(self, batch, species, r_cut, n_max, l_max, sigma, alphas, betas, average="off",
             species_weights=None, num_threads=0):
        if species_weights is not None:
            raise ValueError("the reference entry layer runs with unit species weights")
        arrays = _batch_arrays(batch)
        structures = len(arrays[4]) - 1
        species = np.ascontiguousarray(species, dtype=np.int32)
        rows = structures if average != "off" else int(arrays[4][-1])
        out = np.zeros((rows, feature_count(len(species), n_max, l_max)), np.float64)
        alphas = np.ascontiguousarray(alphas, np.float64)
        betas = np.ascontiguousarray(betas, np.float64)
        status = self._soap(*map(_ptr, arrays), structures, _ptr(species), len(species),
                            float(r_cut), int(n_max), int(l_max), float(sigma), _ptr(alphas),
                            _ptr(betas), _AVERAGE[average], int(num_threads), _ptr(out))
        if status:
            raise ValueError(self.error())
        return out


def neighbor_list(checker, batch, cutoff: float, full_neighbor_list: bool = True, self_pairs: bool = False):
    """compute_neighbor_list (cpp/src/standalone/neighbor_list.cpp:15-75) over a
    checker's graph (which keeps the reference CPU pair order): drop the exact
    self pair unless self_pairs, keep one orientation unless full
    (keep_half_neighbor, cpp/include/mdescriptor/detail/neighbor_filter.hpp:16-36);
    returns (records (P, 5), values (P, 4), row_offsets (S+1,))."""
    offsets, atoms, shifts, disp, d2 = checker.graph(batch, cutoff)
    n_atoms = len(offsets) - 1
    centre = np.repeat(np.arange(n_atoms, dtype=np.int64), np.diff(offsets))
    atom = atoms.astype(np.int64)
    zero = (shifts == 0).all(axis=1)
    keep = np.ones(len(atom), bool)
    if not self_pairs:
        keep &= ~((atom == centre) & zero)
    if not full_neighbor_list:
        first = np.where(shifts[:, 0] != 0, shifts[:, 0], np.where(shifts[:, 1] != 0, shifts[:, 1], shifts[:, 2]))
        keep &= np.where(atom != centre, atom > centre, np.where(zero, True, first > 0))
    records = np.column_stack([centre, atom, shifts]).astype(np.float64)[keep]
    values = np.column_stack([disp, np.sqrt(np.maximum(0.0, d2))])[keep]
    kept_before = np.concatenate([[0], np.cumsum(keep)])
    pair_offsets_per_atom = kept_before[offsets]
    structure_offsets = np.asarray(batch.offsets, np.int64)
    return records, values, pair_offsets_per_atom[structure_offsets]


def reference_neighbor_list(batch, cutoff: float, full_neighbor_list: bool = True, self_pairs: bool = False):
    """The reference's own compute_neighbor_list (oracle/_ref), split like neighbor_list()."""
    lib = ctypes.CDLL(str(ORACLE_DIR / "_ref" / "libref_soap.so"))
    lib.ref_neighbor_list.restype = _P
    lib.ref_neighbor_list.argtypes = [_P] * 5 + [ctypes.c_int64, ctypes.c_double, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_int]
    lib.ref_neighbor_list_rows.restype = ctypes.c_int64
    lib.ref_neighbor_list_rows.argtypes = [_P]
    lib.ref_neighbor_list_copy.argtypes = [_P, _P, _P]
    lib.ref_neighbor_list_free.argtypes = [_P]
    lib.ref_last_error.restype = ctypes.c_char_p
    arrays = _batch_arrays(batch)
    structures = len(arrays[4]) - 1
    handle = lib.ref_neighbor_list(*map(_ptr, arrays), structures, float(cutoff), int(full_neighbor_list),
                                   int(self_pairs), 1)
    if not handle:
        raise ValueError(lib.ref_last_error().decode())
    try:
        rows = int(lib.ref_neighbor_list_rows(handle))
        table = np.zeros((rows, 9), np.float64)
        offsets = np.zeros(structures + 1, np.int64)
        lib.ref_neighbor_list_copy(handle, _ptr(table), _ptr(offsets))
    finally:
        lib.ref_neighbor_list_free(handle)
    return table[:, :5], table[:, 5:], offsets


def reference_available() -> bool:
    return (ORACLE_DIR / "_ref" / "libref_soap.so").is_file()


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
