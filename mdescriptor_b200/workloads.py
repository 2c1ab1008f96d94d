"""Seeded synthetic structure batches with the shapes of the SOAP benchmark configs.

No public dataset backs the benchmark; these generators stand in for it with
the stated cell shapes, atom counts, species weights and minimum distances.
Configs 1-4 draw from ``numpy.random.default_rng(20261201 + k)`` unless a
seed is given.  Config 5 (16.8 M atoms) uses a per-structure stream of the
C generator in csrc/synth.c instead, so that each rank of a sharded run can
make its own slice of the one batch in well under a second.  Positions are
float64 and never wrapped into the cell.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

SEED_BASE = 20261201


@dataclass
class Batch:
    """Flat structure batch with MDescriptor's ``StructureBatch`` array layout.

    numbers int32[N], positions float64[N,3], cells float64[S,3,3] (lattice
    vectors as rows), pbc int32[S,3], offsets int64[S+1]
    (src/mdescriptor/core/input.py:20-131).
    """

    numbers: np.ndarray
    positions: np.ndarray
    cells: np.ndarray
    pbc: np.ndarray
    offsets: np.ndarray
    ids: tuple = field(default=())

    @property
    def structures(self) -> int:
        return int(self.offsets.shape[0]) - 1

    @property
    def atoms(self) -> int:
        return int(self.offsets[-1])

    def slice(self, start: int, stop: int) -> "Batch":
        a0, a1 = int(self.offsets[start]), int(self.offsets[stop])
        return Batch(self.numbers[a0:a1], self.positions[a0:a1], self.cells[start:stop],
                     self.pbc[start:stop], self.offsets[start:stop + 1] - a0,
                     tuple(self.ids[start:stop]) if self.ids else ())


@dataclass(frozen=True)
class SoapConfig:
    name: str
    species: tuple
    r_cut: float
    n_max: int
    l_max: int
    average: str
    dtype: str
    sigma: float = 1.0


CONFIGS = {
    1: SoapConfig("cfg1-periodic-64x64", (1, 8), 4.5, 4, 3, "off", "float32"),
    2: SoapConfig("cfg2-periodic-1024x128", (1, 6, 7, 8), 5.0, 8, 6, "off", "float32"),
    3: SoapConfig("cfg3-fcc-8x32768", (13, 29), 6.0, 8, 8, "off", "float64"),
    4: SoapConfig("cfg4-clusters-16384", (1, 6, 7, 8, 16), 5.0, 6, 4, "off", "float32"),
    5: SoapConfig("cfg5-periodic-65536x256", (1, 6, 8), 5.5, 8, 6, "off", "float32"),
}


def _periodic_uniform(rng, structures, atoms, side, d_min):
    """Uniform positions in a cubic cell with sequential minimum-image rejection,
    drawn for all structures at once (atom k is redrawn until it keeps d_min to
    atoms 0..k-1 of its own structure)."""
    positions = np.empty((structures, atoms, 3), np.float64)
    d2_min = d_min * d_min
    for k in range(atoms):
        pending = np.arange(structures)
        while pending.size:
            candidate = rng.uniform(0.0, side, size=(pending.size, 3))
            if k == 0:
                positions[pending, 0] = candidate
                break
            delta = positions[pending, :k] - candidate[:, None, :]
            delta -= side * np.round(delta / side)
            ok = np.einsum("sij,sij->si", delta, delta).min(axis=1) >= d2_min
            positions[pending[ok], k] = candidate[ok]
            pending = pending[~ok]
    return positions


def _species(rng, species, weights, count):
    return np.asarray(species, np.int32)[rng.choice(len(species), size=count, p=weights)]


def _cubic_batch(rng, structures, atoms, side, species, weights, d_min):
    positions = _periodic_uniform(rng, structures, atoms, side, d_min).reshape(-1, 3)
    numbers = _species(rng, species, weights, structures * atoms)
    cells = np.broadcast_to(np.eye(3) * side, (structures, 3, 3)).copy()
    pbc = np.ones((structures, 3), np.int32)
    offsets = np.arange(structures + 1, dtype=np.int64) * atoms
    return Batch(numbers, positions, cells, pbc, offsets)


def config1(structures=64, seed=None):
    rng = np.random.default_rng(SEED_BASE + 1 if seed is None else seed)
    return _cubic_batch(rng, structures, 64, 12.0, (1, 8), (2 / 3, 1 / 3), 0.9)


def config2(structures=1024, seed=None):
    rng = np.random.default_rng(SEED_BASE + 2 if seed is None else seed)
    return _cubic_batch(rng, structures, 128, 14.0, (1, 6, 7, 8), (0.4, 0.3, 0.1, 0.2), 0.9)


def config3(structures=8, seed=None, reps=(32, 32, 8)):
    """fcc, a = 4.05 A, 32x32x8 conventional cells (4 atoms each) mapped by a
    volume-preserving affine map onto a cube (fractional coordinates kept),
    then N(0, 0.1 A) jitter; positions are not wrapped."""
    rng = np.random.default_rng(SEED_BASE + 3 if seed is None else seed)
    basis = np.array([[0.0, 0.0, 0.0], [0.0, 0.5, 0.5], [0.5, 0.0, 0.5], [0.5, 0.5, 0.0]])
    reps = np.asarray(reps)
    grid = np.stack(np.meshgrid(*[np.arange(r) for r in reps], indexing="ij"), -1).reshape(-1, 3)
    fractional = ((grid[:, None, :] + basis[None, :, :]) / reps).reshape(-1, 3)
    side = float(np.prod(reps * 4.05) ** (1.0 / 3.0))
    atoms = fractional.shape[0]
    positions = np.empty((structures, atoms, 3))
    for s in range(structures):
        positions[s] = fractional * side + rng.normal(0.0, 0.1, size=(atoms, 3))
    numbers = _species(rng, (13, 29), (0.9, 0.1), structures * atoms)
    cells = np.broadcast_to(np.eye(3) * side, (structures, 3, 3)).copy()
    pbc = np.ones((structures, 3), np.int32)
    offsets = np.arange(structures + 1, dtype=np.int64) * atoms
    return Batch(numbers, positions.reshape(-1, 3), cells, pbc, offsets)


def config4(structures=16384, seed=None):
    """Isolated clusters, N ~ U[20, 60], uniform in a ball of radius
    0.62 N^(1/3) 2.0 A with a 1.0 A minimum distance; zero cell, pbc 0."""
    rng = np.random.default_rng(SEED_BASE + 4 if seed is None else seed)
    counts = rng.integers(20, 61, size=structures)
    chunks = []
    for count in counts:
        radius = 0.62 * count ** (1.0 / 3.0) * 2.0
        accepted = np.empty((count, 3))
        k = 0
        while k < count:
            candidate = rng.uniform(-radius, radius, size=3)
            if candidate @ candidate > radius * radius:
                continue
            if k and (((accepted[:k] - candidate) ** 2).sum(axis=1).min() < 1.0):
                continue
            accepted[k] = candidate
            k += 1
        chunks.append(accepted)
    positions = np.concatenate(chunks)
    numbers = _species(rng, (1, 6, 7, 8, 16), (0.45, 0.3, 0.1, 0.12, 0.03), positions.shape[0])
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    cells = np.zeros((structures, 3, 3))
    pbc = np.zeros((structures, 3), np.int32)
    return Batch(numbers, positions, cells, pbc, offsets)


_SYNTH = None


def _synth_lib():
    global _SYNTH
    if _SYNTH is None:
        import ctypes
        from pathlib import Path

        path = Path(__file__).resolve().parent / "lib" / "libmdsynth.so"
        if not path.is_file():
            raise RuntimeError(f"{path} is missing: run python -m mdescriptor_b200.build")
        lib = ctypes.CDLL(str(path))
        lib.mdsynth_cubic.restype = ctypes.c_int
        lib.mdsynth_cubic.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                      ctypes.c_double, ctypes.c_double, ctypes.c_int32, ctypes.c_void_p,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        _SYNTH = lib
    return _SYNTH


def streamed_cubic_batch(seed, first, structures, atoms, side, species, weights, d_min):
    """Structures [first, first + structures) of a batch of cubic periodic
    cells whose structure s draws only from the stream of (seed, s)
    (csrc/synth.c): any slice equals the same range of the whole batch, so a
    sharded run makes only its own part."""
    species = np.ascontiguousarray(species, np.int32)
    weights = np.ascontiguousarray(weights, np.float64)
    numbers = np.empty(structures * atoms, np.int32)
    positions = np.empty((structures * atoms, 3), np.float64)
    rc = _synth_lib().mdsynth_cubic(seed, first, structures, atoms, side, d_min, len(species),
                                    species.ctypes.data, weights.ctypes.data, numbers.ctypes.data,
                                    positions.ctypes.data, 1 << 20)
    if rc != 0:
        raise RuntimeError("synthetic cell too dense for its minimum distance")
    cells = np.broadcast_to(np.eye(3) * side, (structures, 3, 3)).copy()
    pbc = np.ones((structures, 3), np.int32)
    offsets = np.arange(structures + 1, dtype=np.int64) * atoms
    return Batch(numbers, positions, cells, pbc, offsets)


def config5(structures=65536, seed=None, first=0):
    """Structures [first, first + structures) of the config-5 batch (65 536
    periodic 16 A cells x 256 atoms, species 1/6/8 drawn 0.5/0.3/0.2, 0.9 A
    minimum image distance), per-structure streams (csrc/synth.c)."""
    return streamed_cubic_batch(SEED_BASE + 5 if seed is None else seed, first, structures, 256, 16.0,
                                (1, 6, 8), (0.5, 0.3, 0.2), 0.9)


GENERATORS = {1: config1, 2: config2, 3: config3, 4: config4, 5: config5}


def make(config: int, structures: int | None = None, seed: int | None = None, first: int = 0) -> Batch:
    """Config `config`'s batch (or its first `structures` structures).  For
    config 5, `first` selects structures [first, first + structures) of the
    one seeded batch; the other configs draw a whole batch from one stream
    and take no offset."""
    generator = GENERATORS[config]
    kwargs = {} if structures is None else {"structures": structures}
    if config == 5:
        kwargs["first"] = first
    elif first:
        raise ValueError("only config 5 supports a structure offset")
    return generator(seed=seed, **kwargs)
