"""Import helper for the hyphenated package.

``conftest.py`` registers the package for the test process; ``load`` also
registers it itself so that spawned worker processes (multi-rank tests) can
import it too.
"""

import importlib
import os
import sys
import types

PACKAGE = "comfyui-int-crush_b200"
_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load(name: str):
    """Import ``comfyui-int-crush_b200.<name>``."""
    if PACKAGE not in sys.modules:
        pkg = types.ModuleType(PACKAGE)
        pkg.__path__ = [os.path.join(_ROOT, PACKAGE)]
        pkg.__package__ = PACKAGE
        sys.modules[PACKAGE] = pkg
    for p in (os.path.join(_ROOT, "oracle"), os.path.join(_ROOT, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    return importlib.import_module(f"{PACKAGE}.{name}")
