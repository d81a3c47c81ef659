"""The reference package patched to select the B200 backend (test support).

``patched_reference(tmp)`` copies the reference package installed under
``baseline/_ref`` (the one offline install of the reference) to ``tmp``,
applies ``parrot-h200-worker_b200/integration/reference_model_b200.patch``
with ``patch -p1`` and imports it as ``parrot``.  Returns the module, or None
when the reference package is not installed.
"""
from __future__ import annotations

import importlib
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
REF = ROOT / "baseline" / "_ref"
PATCH = ROOT / "parrot-h200-worker_b200" / "integration" / "reference_model_b200.patch"


def patched_reference(tmp: Path):
    if not (REF / "parrot" / "model.py").exists():
        print("reference package not installed under baseline/_ref: "
              "the integration patch is not exercised")
        return None
    shutil.copytree(REF / "parrot", tmp / "parrot",
                    ignore=shutil.ignore_patterns("__pycache__"))
    subprocess.run(["patch", "-p1", "--quiet", "-i", str(PATCH)], cwd=tmp, check=True)
    for name in [m for m in sys.modules if m == "parrot" or m.startswith("parrot.")]:
        del sys.modules[name]
    sys.path.insert(0, str(tmp))
    try:
        return importlib.import_module("parrot.model")
    finally:
        sys.path.remove(str(tmp))
