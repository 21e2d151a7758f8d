"""BF16 rounding and ``.mem`` text helpers (test infrastructure, see package doc).

Restates ``pyfiles/gqa_reference.py``:
  * ``f32_to_bf16``  -> gqa_reference.py:15-19 (double -> FP32 RNE -> BF16 RNE)
  * ``bf16_to_f32``  -> gqa_reference.py:22-23
  * ``pack_bf16`` / ``unpack_bf16`` -> gqa_reference.py:26-36 (element 0 rightmost)
  * ``write_mem`` / ``read_mem``    -> gqa_reference.py:39-46
  * ``ulp_distance`` -> gqa_reference.py:49-53 (monotonic BF16-code distance)
All functions are vectorised over numpy arrays.
"""
from __future__ import annotations

from pathlib import Path
from typing import Iterable

import numpy as np


def f32_to_bf16(values) -> np.ndarray:
    """Round float64 values to BF16 codes (uint16) exactly as gqa_reference.py:15-19.

    The reference packs the double into an IEEE single (round-to-nearest-even),
    then adds ``0x7FFF + lsb`` to the 32-bit pattern and keeps the top half.
    """
    f32 = np.asarray(values, dtype=np.float64).astype(np.float32)
    bits = f32.view(np.uint32).astype(np.uint64)
    lsb = (bits >> np.uint64(16)) & np.uint64(1)
    return (((bits + np.uint64(0x7FFF) + lsb) >> np.uint64(16)) & np.uint64(0xFFFF)).astype(np.uint16)


def bf16_to_f32(codes) -> np.ndarray:
    """BF16 codes -> float64 values (exact), gqa_reference.py:22-23."""
    c = np.asarray(codes).astype(np.uint32) & np.uint32(0xFFFF)
    return (c << np.uint32(16)).view(np.float32).astype(np.float64)


def ulp_distance(a, b) -> np.ndarray:
    """Monotonic BF16-code distance, gqa_reference.py:49-53."""
    def ordered(x):
        x = np.asarray(x).astype(np.int64) & 0xFFFF
        return np.where(x & 0x8000, 0x8000 - (x & 0x7FFF), 0x8000 + x)
    return np.abs(ordered(a) - ordered(b))


def pack_bf16(values: Iterable[int]) -> str:
    """One ``.mem`` line: element 0 is the rightmost 4 hex digits."""
    vals = [int(v) & 0xFFFF for v in values]
    return "".join(f"{v:04x}" for v in reversed(vals))


def unpack_bf16(line: str, elements: int) -> list[int]:
    text = line.strip().replace("_", "")
    if len(text) != elements * 4:
        raise ValueError(f"expected {elements * 4} hex digits, got {len(text)}")
    return [int(text[len(text) - 4 * (i + 1):len(text) - 4 * i], 16) for i in range(elements)]


def write_mem(path: Path, rows) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(mem_text(rows))


def mem_text(rows) -> str:
    """The full text ``write_mem`` writes: one packed row per line, trailing newline."""
    return "\n".join(pack_bf16(row) for row in rows) + "\n"


def read_mem(path: Path, elements: int) -> list[list[int]]:
    return [unpack_bf16(line, elements) for line in Path(path).read_text().splitlines()
            if line.strip() and not line.lstrip().startswith("//")]


def read_mem_array(path: Path, elements: int) -> np.ndarray:
    """``read_mem`` as a uint16 array of shape [rows, elements]."""
    return np.asarray(read_mem(path, elements), dtype=np.uint16).reshape(-1, elements)
