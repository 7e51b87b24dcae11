"""Compatibility name for code that imports the reference's ``_triton_runtime``.

Every flag, toggle and callable read through this module is the B200
implementation in ``_b200_runtime`` (no Triton is involved).  Toggles such as
``USE_CUDA_GRAPHS`` are read by the ops layer from ``_b200_runtime``: set
them there (``_b200_runtime.USE_CUDA_GRAPHS = False``).
"""

from . import _b200_runtime as _rt

__all__ = list(_rt.__all__)


def __getattr__(name):
    return getattr(_rt, name)


def __dir__():
    return sorted(set(__all__) | set(globals()))
