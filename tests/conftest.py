"""Pytest configuration.

* Registers the ``gpu`` marker (tests that need a B200; run with ``-m gpu``).
* Registers the hyphenated package directory ``comfyui-int-crush_b200`` as an
  importable package (Python rejects hyphens in ``import`` statements), the
  way the reference's own ``tests/conftest.py`` does for its package.
* Puts ``oracle/`` and ``tests/`` on ``sys.path``.
"""

import os
import sys
import types

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_NAME = "comfyui-int-crush_b200"

for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

if PKG_NAME not in sys.modules:
    pkg = types.ModuleType(PKG_NAME)
    pkg.__path__ = [os.path.join(ROOT, PKG_NAME)]
    pkg.__package__ = PKG_NAME
    sys.modules[PKG_NAME] = pkg


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")
