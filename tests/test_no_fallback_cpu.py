"""The product path has no CPU fallback and never routes through the oracle:
importing the package without its native extension fails loudly, and no
package module imports the test oracle."""
from __future__ import annotations

import os
import re
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "layerstormexpertkernels_b200")

BLOCKED_IMPORT = """
import importlib.abc, sys
class Block(importlib.abc.MetaPathFinder):
    def find_spec(self, name, path, target=None):
        if name == "layerstormexpertkernels_b200._C":
            raise ImportError("extension hidden for the test")
        return None
sys.meta_path.insert(0, Block())
try:
    import layerstormexpertkernels_b200
except ImportError as exc:
    print("IMPORT-ERROR:", exc)
else:
    print("IMPORTED")
"""


def test_import_fails_loudly_without_the_extension():
    out = subprocess.run([sys.executable, "-c", BLOCKED_IMPORT], cwd=ROOT, capture_output=True,
                         text=True, timeout=600)
    assert "IMPORT-ERROR:" in out.stdout, out.stdout + out.stderr
    assert "native extension is not built" in out.stdout


def test_package_never_imports_the_oracle():
    pattern = re.compile(r"^\s*(from\s+oracle\b|import\s+oracle\b)|\boracle\.", re.M)
    for name in sorted(os.listdir(PKG)):
        if name.endswith(".py"):
            with open(os.path.join(PKG, name)) as f:
                assert not pattern.search(f.read()), f"{name} refers to the test oracle"
