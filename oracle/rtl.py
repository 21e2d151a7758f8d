"""RTL-numerics RoPE (test infrastructure, see package doc).

Restates the RoPE datapath of the reference RTL, ``rope_unit.v``:
  * NCO phase (:159-172): ``phase = (phase_rom[i] * pos) mod 2**32`` for pair
    i, read as an unsigned Q0.32 fraction of a turn;
  * ROM lookup (:166, :221-222): the top ``ROM_ADDR_BITS`` (14) bits of the
    phase address the sincos ROM, ``{cos[31:16], sin[15:0]}`` BF16 codes
    (``tools/gen_rope_rom.py``, restated in ``oracle.rope_rom``);
  * rotation in BF16 units (:124-129): ``x' = bf16_sub(bf16_mul(x, cos),
    bf16_mul(y, sin))``, ``y' = bf16_add(bf16_mul(x, sin), bf16_mul(y, cos))``.
The BF16 units are taken as the reference specifies them for conformance
(``pyfiles/gen_bf16_primitive_vectors.py:31-32``): the float64 result of the
operation on the two BF16 values, rounded by ``f32_to_bf16``.
"""
from __future__ import annotations

import numpy as np

from .bf16 import bf16_to_f32, f32_to_bf16
from .rope_rom import rope_phase_rom, rope_sincos_rom

ROM_ADDR_BITS = 14  # rope_unit.v:46


def rom_factors(positions, head_dim: int = 128, theta: float = 500000.0,
                addr_bits: int = ROM_ADDR_BITS) -> tuple[np.ndarray, np.ndarray]:
    """BF16 codes (cos, sin), each ``[len(positions), head_dim // 2]``."""
    phase = np.asarray(rope_phase_rom(head_dim, theta), dtype=np.uint64)
    table = np.asarray(rope_sincos_rom(addr_bits), dtype=np.uint16)  # [2**bits, 2] (cos, sin)
    pos = np.asarray(positions, dtype=np.uint64)
    ph = (pos[:, None] * phase[None, :]) & np.uint64(0xFFFFFFFF)
    addr = (ph >> np.uint64(32 - addr_bits)).astype(np.int64)
    return table[addr, 0], table[addr, 1]


def _bf16_op(values: np.ndarray) -> np.ndarray:
    return f32_to_bf16(values)


def rope_rtl_rows(rows_bits: np.ndarray, positions, head_dim: int = 128, theta: float = 500000.0,
                  addr_bits: int = ROM_ADDR_BITS) -> np.ndarray:
    """BF16 codes of rope_unit.v's rotated rows: ``rows_bits`` ``[n, head_dim]`` codes,
    row r at ``positions[r]``."""
    rows_bits = np.asarray(rows_bits, dtype=np.uint16)
    half = head_dim // 2
    c_bits, s_bits = rom_factors(positions, head_dim, theta, addr_bits)
    c, s = bf16_to_f32(c_bits), bf16_to_f32(s_bits)
    x, y = bf16_to_f32(rows_bits[:, :half]), bf16_to_f32(rows_bits[:, half:])
    xc, ys = bf16_to_f32(_bf16_op(x * c)), bf16_to_f32(_bf16_op(y * s))
    xs, yc = bf16_to_f32(_bf16_op(x * s)), bf16_to_f32(_bf16_op(y * c))
    return np.concatenate([_bf16_op(xc - ys), _bf16_op(xs + yc)], axis=1)


BF16_SCALE_128 = 0x3DB5  # bf16(1/sqrt(128)), the SCALE_FACTOR register value (gqa_reference.py:56-57)
