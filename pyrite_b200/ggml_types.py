"""GGML tensor type geometry (ids, block sizes, bytes per block).

The values are the GGML format's own (``enum ggml_type`` and the block structs);
they restate the registry of the reference, ``pyrite/ggml_types.py:34-73``,
which the GGUF byte ranges and the kernel library both depend on.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class GGMLTypeSpec:
    type_id: int
    name: str
    block_size: int
    bytes_per_block: int
    quantized: bool = False

    @property
    def bits_per_weight(self) -> float:
        return self.bytes_per_block * 8 / self.block_size


_ROWS = [
    (0, "F32", 1, 4, False), (1, "F16", 1, 2, False), (2, "Q4_0", 32, 18, True),
    (3, "Q4_1", 32, 20, True), (6, "Q5_0", 32, 22, True), (7, "Q5_1", 32, 24, True),
    (8, "Q8_0", 32, 34, True), (9, "Q8_1", 32, 36, True), (10, "Q2_K", 256, 84, True),
    (11, "Q3_K", 256, 110, True), (12, "Q4_K", 256, 144, True), (13, "Q5_K", 256, 176, True),
    (14, "Q6_K", 256, 210, True), (15, "Q8_K", 256, 292, True), (16, "IQ2_XXS", 256, 66, True),
    (17, "IQ2_XS", 256, 74, True), (18, "IQ3_XXS", 256, 98, True), (19, "IQ1_S", 256, 50, True),
    (20, "IQ4_NL", 32, 18, True), (21, "IQ3_S", 256, 110, True), (22, "IQ2_S", 256, 82, True),
    (23, "IQ4_XS", 256, 136, True), (24, "I8", 1, 1, False), (25, "I16", 1, 2, False),
    (26, "I32", 1, 4, False), (27, "I64", 1, 8, False), (28, "F64", 1, 8, False),
    (29, "IQ1_M", 256, 56, True), (30, "BF16", 1, 2, False), (34, "TQ1_0", 256, 54, True),
    (35, "TQ2_0", 256, 66, True), (39, "MXFP4", 32, 17, True), (40, "NVFP4", 64, 36, True),
    (41, "Q1_0", 128, 18, True), (42, "Q2_0", 64, 18, True),
]
TYPES: dict[int, GGMLTypeSpec] = {r[0]: GGMLTypeSpec(*r) for r in _ROWS}
BY_NAME: dict[str, int] = {s.name: s.type_id for s in TYPES.values()}

#: The 21 types with a fused kernel (the reference's decodable set).
DECODABLE: tuple[int, ...] = (0, 1, 2, 3, 6, 7, 8, 9, 10, 11, 12, 13, 14, 20, 23, 24, 25, 26, 27, 28, 30)


def spec(type_id: int) -> GGMLTypeSpec:
    if not isinstance(type_id, int):
        raise TypeError(f"GGML tensor type must be an integer, got {type_id!r}")
    found = TYPES.get(type_id)
    if found is None:
        raise ValueError(f"unsupported GGML tensor type: {type_id}")
    return found


def type_name(type_id: int) -> str:
    found = TYPES.get(type_id)
    return found.name if found else f"UNKNOWN({type_id})"


def row_size(elements: int, type_id: int) -> int:
    """Bytes of one row of ``elements`` values (must be block aligned)."""
    t = spec(type_id)
    if elements < 0:
        raise ValueError("elements must be non-negative")
    if t.block_size != 1 and elements % t.block_size:
        raise ValueError(f"{t.name} row requires element count divisible by {t.block_size}, got {elements}")
    return elements // t.block_size * t.bytes_per_block
