"""Load the drop-in ``mdescriptor._cuda`` plugin built in mdescriptor_b200/plugin/,
and rebuild the adapter's captured backend options (tests/golden/adapter_options.json)."""

from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
PLUGIN_DIR = ROOT / "mdescriptor_b200" / "plugin"
GOLDEN = Path(__file__).resolve().parent / "golden"


def plugin_path() -> Path:
    hits = sorted(PLUGIN_DIR.glob("_cuda*.so"))
    if not hits:
        raise FileNotFoundError("plugin not built: python -m mdescriptor_b200.build")
    return hits[0]


def load_plugin():
    """The plugin under its canonical name (one copy per process)."""
    module = sys.modules.get("mdescriptor._cuda")
    if module is not None:
        return module
    spec = importlib.util.spec_from_file_location("mdescriptor._cuda", plugin_path())
    module = importlib.util.module_from_spec(spec)
    sys.modules["mdescriptor._cuda"] = module
    try:
        spec.loader.exec_module(module)
    except BaseException:
        sys.modules.pop("mdescriptor._cuda", None)
        raise
    return module


def _decode(value):
    if isinstance(value, dict):
        if "__ndarray__" in value:
            return np.asarray(value["__ndarray__"], dtype=value["dtype"]).reshape(value["shape"])
        return {k: _decode(v) for k, v in value.items()}
    if isinstance(value, list):
        return [_decode(v) for v in value]
    return value


def adapter_cases():
    """[(name, options, kwargs)] as the adapter built them (label tuples restored;
    species_weighting keys stay strings, as the adapter hands them on)."""
    out = []
    for case in json.loads((GOLDEN / "adapter_options.json").read_text()):
        options = _decode(case["options"])
        options["_cuda_labels"] = tuple(options["_cuda_labels"])
        options["_cuda_payload"]["labels"] = tuple(options["_cuda_payload"]["labels"])
        out.append((case["name"], options, case["kwargs"]))
    return out
