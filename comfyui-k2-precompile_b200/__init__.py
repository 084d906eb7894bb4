"""ComfyUI-style package directory of the B200 Krea2 W4A4 hot path.

Loaded by path (like a ComfyUI custom node); the importable host package is
the ``k2b`` directory next to this file.
"""
import os
import sys

_here = os.path.dirname(os.path.abspath(__file__))
if _here not in sys.path:
    sys.path.insert(0, _here)

NODE_CLASS_MAPPINGS: dict = {}
NODE_DISPLAY_NAME_MAPPINGS: dict = {}
