"""The reference's unchanged Python package, as staged by oracle/build_oracle.py
into baseline/_ref/mdescriptor (its Python sources with the ``_native``
extension compiled from the reference's C++ sources beside them).  The staged
copy travels with the repository snapshot, so the same import works in the
build container and on a GPU box.  Test infrastructure only."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
BASELINE_REF = ROOT / "baseline" / "_ref"


def staged() -> bool:
    pkg = BASELINE_REF / "mdescriptor"
    return (pkg / "__init__.py").is_file() and bool(list(pkg.glob("_native*.so")))


def reference_package():
    """``import mdescriptor`` from baseline/_ref, or skip when it is not staged."""
    if not staged():
        pytest.skip("reference package not staged in baseline/_ref (run oracle/build_oracle.py with "
                    "MDSOAP_REFERENCE_ROOT set)")
    if str(BASELINE_REF) not in sys.path:
        sys.path.insert(0, str(BASELINE_REF))
    import mdescriptor  # noqa: PLC0415

    if Path(mdescriptor.__file__).resolve().parent != (BASELINE_REF / "mdescriptor").resolve():
        raise RuntimeError(f"another mdescriptor package shadows the staged reference: {mdescriptor.__file__}")
    return mdescriptor


def reference_native():
    """The reference's compiled ``_native`` module (imported once per process)."""
    reference_package()
    from mdescriptor import _native  # noqa: PLC0415

    return _native
