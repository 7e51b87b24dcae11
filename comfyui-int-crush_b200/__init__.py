"""INT-Crush on B200: INT4/INT8 quantised inference for ComfyUI diffusion models.

Drop-in package with the reference's public surface: ``ConvLinear4bit``,
layout registration with ComfyUI's QuantizedTensor dispatch, and the loader
node mappings (reference ``__init__.py:17-32``).  The quantised linears run
on the hand-written sm_100a kernels of ``libintcrush_b200.so``.
"""

import logging

log = logging.getLogger(__name__)

__all__: list[str] = []

try:
    from .convlinear import ConvLinear4bit
    __all__.append("ConvLinear4bit")
except ImportError:
    ConvLinear4bit = None

try:
    from .quant_layout import register_intcrush_layouts
    register_intcrush_layouts()
except Exception:
    log.warning("INT-Crush: layout registration failed", exc_info=True)

try:
    from .comfy_nodes import NODE_CLASS_MAPPINGS, NODE_DISPLAY_NAME_MAPPINGS
    __all__.extend(["NODE_CLASS_MAPPINGS", "NODE_DISPLAY_NAME_MAPPINGS"])
except Exception:
    log.warning("INT-Crush: node import failed", exc_info=True)
