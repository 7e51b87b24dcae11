"""Import helper for the hyphenated package (registered by conftest.py)."""

import importlib

PACKAGE = "comfyui-int-crush_b200"


def load(name: str):
    """Import ``comfyui-int-crush_b200.<name>``."""
    return importlib.import_module(f"{PACKAGE}.{name}")
