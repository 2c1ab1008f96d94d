"""Generate the committed golden fixtures in this directory.

Run in the build container (it needs the reference tree and the reference's
``_native`` module built by ``oracle/build_oracle.py``):

    python tests/golden/make_golden.py [--reference-root DIR]

Outputs
* ``reference_goldens.npz`` + ``reference_goldens.json``: the reference's own
  committed SOAP fixtures (tests/golden/soap/{input,expected_output}.npz,
  external_{input,expected_output}.npz: DScribe 2.1.2 static golden) and the
  NeighborList golden (tests/golden/neighborlist), copied verbatim as data
  with their manifests' parameters and tolerances.
* ``adapter_options.json``: the exact options MDescriptor's unchanged adapter
  hands to ``mdescriptor._cuda.create_backend`` (captured by replacing
  ``mdescriptor._runtime.create_cuda_backend`` with a recorder) for two SOAP
  configurations, so the GPU plugin test can replay them where MDescriptor is
  not installed; ``adapter_expected.npz`` holds the batch they run on and the
  reference's CPU result (values, row_offsets) for each.
* ``config_goldens.npz`` + ``config_goldens.json``: for seeded slices of the
  five benchmark configs, the reference's features computed through its
  unchanged public API (``mdescriptor.descriptors.SOAP(..., device="cpu")``),
  the reference ``_basis_gto`` alphas/betas, and a SHA-256 digest of the
  reference neighbour graph in canonical (centre, atom, shift) order.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

from mdescriptor_b200 import workloads  # noqa: E402
from mdescriptor_b200.basis import graph_cutoff  # noqa: E402

# Slices: (config, structures, row stride of the stored rows, averages)
SLICES = {
    "cfg1": dict(config=1, structures=4, stride=1, averages=("off", "inner", "outer")),
    "cfg2": dict(config=2, structures=2, stride=8, averages=("off",)),
    "cfg3": dict(config=3, structures=1, stride=8, averages=("off",), reps=(4, 4, 2)),
    "cfg4": dict(config=4, structures=6, stride=8, averages=("off", "inner")),
    "cfg5": dict(config=5, structures=1, stride=16, averages=("off",)),
}


def canonical_graph_digest(graph) -> tuple[str, int]:
    offsets, atoms, shifts, disp, d2 = graph
    centers = np.repeat(np.arange(len(offsets) - 1, dtype=np.int64), np.diff(offsets))
    order = np.lexsort((shifts[:, 2], shifts[:, 1], shifts[:, 0], atoms, centers))
    h = hashlib.sha256()
    for array in (centers[order], atoms[order].astype(np.int64), shifts[order].astype(np.int64),
                  np.ascontiguousarray(disp[order]), np.ascontiguousarray(d2[order])):
        h.update(np.ascontiguousarray(array).tobytes())
    return h.hexdigest(), int(len(atoms))


def import_reference(root: Path):
    sys.path.insert(0, str(root / "src"))
    import mdescriptor

    mdescriptor.__path__.insert(0, str(ROOT / "oracle" / "_ref" / "pkg"))
    from mdescriptor import ExecutionOptions, OutputOptions, StructureBatch
    from mdescriptor.descriptors import SOAP
    from mdescriptor.descriptors._kernels.core import _basis_gto

    return SOAP, StructureBatch, OutputOptions, ExecutionOptions, _basis_gto


def _jsonable(value):
    if isinstance(value, np.ndarray):
        return {"__ndarray__": value.tolist(), "dtype": str(value.dtype), "shape": list(value.shape)}
    if isinstance(value, dict):
        return {str(k): _jsonable(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [_jsonable(v) for v in value]
    return value


def adapter_batch():
    """Two periodic config-1 boxes and the first box again as an isolated cluster."""
    base = workloads.config1(structures=2)
    first = base.slice(0, 1)
    return workloads.Batch(
        np.concatenate([base.numbers, first.numbers]),
        np.concatenate([base.positions, first.positions]),
        np.concatenate([base.cells, first.cells]),
        np.concatenate([base.pbc, np.zeros_like(first.pbc)]),
        np.concatenate([base.offsets, base.offsets[-1] + first.offsets[1:]]),
    )


ADAPTER_KWARGS = [
    dict(species=[1, 8], r_cut=4.5, n_max=4, l_max=3, average="off"),
    dict(species=[8, 1], r_cut=4.0, n_max=3, l_max=4, sigma=0.8, average="inner",
         compression={"mode": "off", "species_weighting": {1: 0.5, 8: 2.0}}),
    dict(species=[1, 8], r_cut=4.5, n_max=8, l_max=6, average="off",
         compression={"mode": "mu1nu1", "species_weighting": {1: 0.8, 8: 1.25}},
         weighting={"function": "poly", "r0": 6.0, "c": 1.0, "m": 2.0}),
    dict(species=[8, 1], r_cut=4.0, n_max=4, l_max=3, average="outer", compression={"mode": "mu2"},
         weighting={"function": "exp", "r0": 1.5, "c": 2.0, "d": 0.5, "w0": 0.25}),
    dict(species=[1, 8], r_cut=4.0, n_max=4, l_max=3, average="off", rbf="polynomial",
         compression={"mode": "crossover"}),
]


def capture_adapter_options(SOAP, StructureBatch, OutputOptions, ExecutionOptions):
    """Options the adapter passes to the CUDA plugin factory for ADAPTER_KWARGS,
    plus the reference's CPU features for the same options on adapter_batch()."""
    import mdescriptor._runtime as runtime

    captured = []

    class Recorder:
        feature_count = None

        def __init__(self, name, options):
            captured.append({"name": name, "options": options})

        def compute(self, batch, control=None):
            raise ImportError("recorder")

    batch = adapter_batch()
    sb = StructureBatch(batch.numbers, batch.positions, batch.cells, batch.pbc, batch.offsets,
                        tuple(f"s{i}" for i in range(batch.structures)))
    original = runtime.create_cuda_backend
    runtime.create_cuda_backend = lambda name, options: Recorder(name, options)
    cases = []
    try:
        for kw in ADAPTER_KWARGS:
            soap = SOAP(**kw, output=OutputOptions(dtype="float32"), execution=ExecutionOptions(device="cuda"))
            try:
                soap.compute(sb)
            except Exception:  # the recorder stops the computation
                pass
            cases.append({"kwargs": _jsonable(kw), "name": captured[-1]["name"],
                          "options": _jsonable(captured[-1]["options"])})
    finally:
        runtime.create_cuda_backend = original
    arrays = {f"input/{k}": getattr(batch, k) for k in ("numbers", "positions", "cells", "pbc", "offsets")}
    for index, kw in enumerate(ADAPTER_KWARGS):
        result = SOAP(**kw, output=OutputOptions(dtype="float32"), execution=ExecutionOptions(device="cpu")).compute(sb)
        arrays[f"case{index}/values"] = np.asarray(result.values)
        if result.row_offsets is not None:  # structure-level results have none
            arrays[f"case{index}/row_offsets"] = np.asarray(result.row_offsets)
    return cases, arrays


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-root", default=os.environ.get("MDSOAP_REFERENCE_ROOT"),
                        help="reference source tree (default: $MDSOAP_REFERENCE_ROOT)")
    args = parser.parse_args()
    if not args.reference_root:
        parser.error("name the reference source tree with --reference-root or MDSOAP_REFERENCE_ROOT")
    root = Path(args.reference_root)
    SOAP, StructureBatch, OutputOptions, ExecutionOptions, basis_gto = import_reference(root)
    from oracle import RefLib

    ref = RefLib()

    cases, adapter_arrays = capture_adapter_options(SOAP, StructureBatch, OutputOptions, ExecutionOptions)
    (HERE / "adapter_options.json").write_text(json.dumps(cases, indent=1) + "\n")
    np.savez_compressed(HERE / "adapter_expected.npz", **adapter_arrays)

    # 1. Reference goldens, copied as data.
    arrays, meta = {}, {}
    ref_golden = root / "tests" / "golden"
    for name, folder, manifest_name, inp, exp in (
        ("soap", "soap", "manifest.json", "input.npz", "expected_output.npz"),
        ("soap_dscribe", "soap", "external_manifest.json", "external_input.npz", "external_expected_output.npz"),
        ("neighborlist", "neighborlist", "manifest.json", "input.npz", "expected_output.npz"),
    ):
        manifest = json.loads((ref_golden / folder / manifest_name).read_text())
        for key, value in np.load(ref_golden / folder / inp).items():
            arrays[f"{name}/input/{key}"] = value
        for key, value in np.load(ref_golden / folder / exp).items():
            arrays[f"{name}/expected/{key}"] = value
        meta[name] = {
            "source": f"tests/golden/{folder}/{manifest_name}",
            "parameters": manifest["configuration"]["parameters"],
            "tolerance": manifest.get("tolerance"),
            "feature_count": manifest["result"].get("feature_count"),
            "level": manifest["result"].get("level"),
        }
        if name == "neighborlist":
            meta[name]["samples_layout"] = "structure, center, neighbor, shift0, shift1, shift2"
    np.savez_compressed(HERE / "reference_goldens.npz", **arrays)
    (HERE / "reference_goldens.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")

    # 2. Config slices through the reference's public API.
    arrays, meta = {}, {}
    for name, spec in SLICES.items():
        cfg = workloads.CONFIGS[spec["config"]]
        if spec["config"] == 3:
            batch = workloads.config3(structures=spec["structures"], reps=spec["reps"])
        else:
            batch = workloads.make(spec["config"], spec["structures"])
        alphas, betas = basis_gto(cfg.r_cut, cfg.n_max, cfg.l_max)
        for key in ("numbers", "positions", "cells", "pbc", "offsets"):
            arrays[f"{name}/input/{key}"] = getattr(batch, key)
        arrays[f"{name}/alphas"] = alphas
        arrays[f"{name}/betas"] = betas
        sb = StructureBatch(batch.numbers, batch.positions, batch.cells, batch.pbc, batch.offsets,
                            tuple(f"s{i}" for i in range(batch.structures)))
        entry = {"config": spec["config"], "species": list(cfg.species), "r_cut": cfg.r_cut,
                 "n_max": cfg.n_max, "l_max": cfg.l_max, "sigma": cfg.sigma, "dtype": cfg.dtype,
                 "structures": batch.structures, "atoms": batch.atoms, "outputs": {}}
        if spec["config"] == 3:
            entry["reps"] = list(spec["reps"])
        for average in spec["averages"]:
            soap = SOAP(species=list(cfg.species), r_cut=cfg.r_cut, n_max=cfg.n_max, l_max=cfg.l_max,
                        sigma=cfg.sigma, average=average, output=OutputOptions(dtype="float64"),
                        execution=ExecutionOptions(device="cpu"))
            result = soap.compute(sb)
            values = np.asarray(result.values, dtype=np.float64)
            rows = np.arange(0, values.shape[0], spec["stride"] if average == "off" else 1, dtype=np.int64)
            arrays[f"{name}/{average}/rows"] = rows
            arrays[f"{name}/{average}/values"] = values[rows]
            labels = list(result.labels)
            entry["outputs"][average] = {
                "rows_total": int(values.shape[0]), "rows_stored": int(len(rows)), "level": result.level,
                "labels_count": len(labels), "labels_sha256": hashlib.sha256("\n".join(labels).encode()).hexdigest(),
                "labels_first": labels[0], "labels_last": labels[-1]}
        digest, pairs = canonical_graph_digest(ref.graph(batch, graph_cutoff(cfg.r_cut, cfg.sigma)))
        entry["graph_sha256"] = digest
        entry["graph_pairs"] = pairs
        entry["graph_cutoff"] = graph_cutoff(cfg.r_cut, cfg.sigma)
        meta[name] = entry
        print(name, batch.atoms, "atoms", pairs, "pairs")
    np.savez_compressed(HERE / "config_goldens.npz", **arrays)
    (HERE / "config_goldens.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
