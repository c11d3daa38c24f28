"""Import shims that let the unmodified reference's CPU PyTorch path run without its optional
third-party dependencies (test infrastructure and CPU-baseline harness only).

Used by ``tests/golden/make_golden.py`` (fixture generation, on a reference source tree) and by
``bench.py``'s reference legs (on the copy installed under ``baseline/_ref``).  Three shims,
nothing else is changed:

1. ``molecular_force_field.models`` becomes a bare package object, so its ``__init__`` (which
   imports e3nn.o3, ``models/__init__.py:3-7``) is skipped; submodules still import from the
   reference sources.
2. ``torch_scatter`` is mapped to the reference's own fallback
   ``molecular_force_field.utils.scatter`` (``utils/scatter.py:63-116``).
3. ``e3nn.math.soft_one_hot_linspace`` is the restatement in ``oracle/radial.py`` (e3nn,
   pinned ``>=0.4.4,<0.6.0`` by the reference, is not installed and not vendored).
"""

from __future__ import annotations

import importlib
import os
import sys
import types

REPO_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def install(root: str) -> None:
    """Make ``molecular_force_field`` importable from ``root`` (a directory that holds the
    package: a source tree or a ``pip install --target`` directory)."""
    if "molecular_force_field.models.pure_cartesian_ictd_layers_full" in sys.modules:
        return
    if not root or not os.path.isdir(os.path.join(root, "molecular_force_field")):
        raise RuntimeError(f"reference package not found under {root!r}")
    if root not in sys.path:
        sys.path.insert(0, root)
    if REPO_ROOT not in sys.path:
        sys.path.insert(0, REPO_ROOT)
    from oracle.radial import soft_one_hot_linspace

    e3nn = types.ModuleType("e3nn")
    e3nn_math = types.ModuleType("e3nn.math")
    e3nn_math.soft_one_hot_linspace = soft_one_hot_linspace
    e3nn.math = e3nn_math
    sys.modules.setdefault("e3nn", e3nn)
    sys.modules.setdefault("e3nn.math", e3nn_math)

    mff = importlib.import_module("molecular_force_field")
    models = types.ModuleType("molecular_force_field.models")
    models.__path__ = [os.path.join(root, "molecular_force_field", "models")]
    sys.modules["molecular_force_field.models"] = models
    mff.models = models

    scatter_mod = importlib.import_module("molecular_force_field.utils.scatter")
    ts = types.ModuleType("torch_scatter")
    ts.scatter = scatter_mod.scatter
    sys.modules["torch_scatter"] = ts
