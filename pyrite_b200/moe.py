"""Qwen3-MoE decode: :class:`pyrite_b200.model.MixedDecoder` on a ``qwen3moe``
checkpoint (routed experts, ``pyrite/executor.py:685-939``)."""
from __future__ import annotations

from .model import MixedDecoder as MoEDecoder

__all__ = ["MoEDecoder"]
