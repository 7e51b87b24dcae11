"""ComfyUI node re-exports (``comfy_nodes.py`` of the reference)."""

from ._loaders import NODE_CLASS_MAPPINGS, NODE_DISPLAY_NAME_MAPPINGS

__all__ = ["NODE_CLASS_MAPPINGS", "NODE_DISPLAY_NAME_MAPPINGS"]
