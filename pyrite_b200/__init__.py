"""pyrite_b200: B200-native fused GGML dequantize x matvec for Pyrite.

``pyrite_b200.kernels.native`` is the drop-in for the reference's
``pyrite.kernels.native`` (host buffers); ``pyrite_b200.kernels.cuda`` is the
device-resident path.  Both call libpyrite_b200.so (include/pyrite_b200.h).
"""
from . import ggml_types  # noqa: F401

__all__ = ["ggml_types"]
