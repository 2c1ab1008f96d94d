"""The NeighborList descriptor: the CPU checker (a restatement of
compute_neighbor_list over the checker's graph, which keeps the reference CPU
pair order) against the reference's own compute_neighbor_list (oracle/_ref),
row for row and bit for bit; then the GPU list against the checker, with the
same exactness (records, displacement and distance bits, and order)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from mdescriptor_b200 import workloads

REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libref_soap.so"
MODES = [(True, False), (False, False), (True, True), (False, True)]  # (full list, self pairs)


def varied_batch(seed: int) -> workloads.Batch:
    """Triclinic cells (one small enough for several images per axis), atoms
    outside the cell, an isolated cluster, an empty structure."""
    rng = np.random.default_rng(seed)
    numbers, positions, cells, pbc, offsets = [], [], [], [], [0]
    for s in range(5):
        n = 0 if s == 3 else int(rng.integers(1, 24))
        periodic = s != 2
        scale = 2.2 if s == 4 else rng.uniform(4.0, 8.0)
        cell = np.diag(rng.uniform(0.9, 1.2, 3) * scale) + np.triu(rng.uniform(-0.5, 0.5, (3, 3)), 1)
        frac = rng.uniform(-0.4, 1.4, (n, 3))
        positions.append(frac @ cell if n else np.zeros((0, 3)))
        numbers.append(rng.choice([1, 8], n).astype(np.int32))
        cells.append(cell if periodic else np.zeros((3, 3)))
        pbc.append([1, 1, 1] if periodic else [0, 0, 0])
        offsets.append(offsets[-1] + n)
    return workloads.Batch(np.concatenate(numbers), np.concatenate(positions), np.array(cells),
                           np.array(pbc, np.int32), np.array(offsets, np.int64))


def assert_tables_equal(got, want):
    for a, b, name in zip(got, want, ("records", "values", "row_offsets")):
        assert a.shape == b.shape, (name, a.shape, b.shape)
        np.testing.assert_array_equal(a, b, err_msg=name)


@pytest.mark.skipif(not REF_LIB.is_file(), reason="reference library not built in this tree")
@pytest.mark.parametrize("seed", range(3))
@pytest.mark.parametrize("full,self_pairs", MODES)
def test_checker_matches_reference_neighbor_list(oracle, seed, full, self_pairs):
    from oracle import neighbor_list, reference_neighbor_list

    batch = varied_batch(seed)
    cutoff = 3.1 + seed
    assert_tables_equal(neighbor_list(oracle, batch, cutoff, full, self_pairs),
                        reference_neighbor_list(batch, cutoff, full, self_pairs))


@pytest.mark.gpu
@pytest.mark.parametrize("seed", range(3))
@pytest.mark.parametrize("full,self_pairs", MODES)
def test_gpu_neighbor_list_matches_checker(oracle, cuda_device, seed, full, self_pairs):
    from oracle import neighbor_list as checker_list
    from mdescriptor_b200.soap import neighbor_list

    batch = varied_batch(seed)
    cutoff = 3.1 + seed
    assert_tables_equal(neighbor_list(batch, cutoff, full, self_pairs, cuda_device),
                        checker_list(oracle, batch, cutoff, full, self_pairs))


@pytest.mark.gpu
@pytest.mark.parametrize("config", [1, 2, 4])
def test_gpu_neighbor_list_config_slices(oracle, cuda_device, config):
    from oracle import neighbor_list as checker_list
    from mdescriptor_b200.soap import neighbor_list

    batch = workloads.make(config, {1: 8, 2: 3, 4: 12}[config])
    for full, self_pairs in MODES[:2]:
        assert_tables_equal(neighbor_list(batch, 6.0, full, self_pairs, cuda_device),
                            checker_list(oracle, batch, 6.0, full, self_pairs))


def test_plugin_neighbor_list_backend_contract():
    """create_backend("NeighborList", options) builds without a GPU (the
    reference plugin's option names and defaults, backend.cu:358-362)."""
    from _plugin import load_plugin

    plugin = load_plugin()
    backend = plugin.create_backend("NeighborList", {"cutoff": 3.5, "full_neighbor_list": False})
    assert backend.feature_count == 4
    with pytest.raises(ValueError, match="cutoff"):
        plugin.create_backend("NeighborList", {"cutoff": -1.0})
    backend.close()
    backend.close()


@pytest.mark.gpu
@pytest.mark.parametrize("full,self_pairs", MODES)
def test_plugin_neighbor_list_result(oracle, cuda_device, full, self_pairs):
    """The plugin's pair result dict as the reference plugin builds it
    (cpp/cuda/src/backend.cu:418-470): values (dx, dy, dz, distance),
    pair_records (centre, atom, shift), per-structure row offsets."""
    from _plugin import load_plugin
    from oracle import neighbor_list as checker_list

    batch = varied_batch(7)
    backend = load_plugin().create_backend(
        "NeighborList", {"cutoff": 3.8, "full_neighbor_list": full, "self_pairs": self_pairs})
    result = backend.compute(batch, None)
    records, values, row_offsets = checker_list(oracle, batch, 3.8, full, self_pairs)
    assert result["level"] == "pair" and result["_mdescriptor_owned_values"] is True
    assert list(result["labels"]) == ["dx", "dy", "dz", "distance"]
    np.testing.assert_array_equal(result["values"], values)
    np.testing.assert_array_equal(result["pair_records"], records)
    np.testing.assert_array_equal(result["row_offsets"], row_offsets)
    assert result["metadata"]["descriptor"] == "NeighborList"
    backend.close()
