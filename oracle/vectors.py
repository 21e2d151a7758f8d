"""Re-generation of the reference's seeded test vectors (test infrastructure, see package doc).

Restates the input side of ``pyfiles/gen_gqa_wrapper_vectors.py``:
  * argument checks and SEQ_LEN derivation     -> :57-78
  * KV_INPUT_LEN padding to whole KV blocks     -> :83
  * smoke inputs (Q=K=0, structured V)          -> :86-94
  * random inputs, ``random.Random(seed)`` draws
    of ``uniform(-0.25, 0.25)`` in q, k, v order,
    no draws for pad rows                       -> :96-103
  * BF16 quantisation                           -> :105-107
  * AXIS beat order of the ``.mem`` files        -> :109-119
  * ``gqa_config.txt`` text                      -> :145-152
The files it writes are byte-identical to the reference's (sha256-pinned in
``tests/golden/manifest.json``).  ``amplitude`` widens the uniform range for the
U[-1, 1) variant named by the benchmark's first configuration.
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass, field

import numpy as np

from .bf16 import f32_to_bf16, mem_text, pack_bf16
from .golden import gqa_golden


@dataclass
class ReferenceCase:
    seq_len: int
    query_position: int
    kv_block_len: int
    mode: str
    seed: int
    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    tile_dim: int = 16
    q_bits: np.ndarray = field(default=None, repr=False)   # [q_heads, D]
    k_bits: np.ndarray = field(default=None, repr=False)   # [kv_heads, KV_INPUT_LEN, D]
    v_bits: np.ndarray = field(default=None, repr=False)

    @property
    def group(self) -> int:
        return self.q_heads // self.kv_heads

    @property
    def kv_input_len(self) -> int:
        return ((self.seq_len + self.kv_block_len - 1) // self.kv_block_len) * self.kv_block_len

    @property
    def n_kv_tiles(self) -> int:
        return self.kv_input_len // self.kv_block_len

    def _beats(self, rows):
        for row in rows:
            for s in range(0, self.head_dim, self.tile_dim):
                yield row[s:s + self.tile_dim]

    def q_mem_text(self) -> str:
        return mem_text(self._beats(self.q_bits.tolist()))

    def kv_mem_text(self, which: str) -> str:
        bits = self.k_bits if which == "k" else self.v_bits
        rows = (bits[h, p].tolist() for h in range(self.kv_heads) for p in range(self.kv_input_len))
        return mem_text(self._beats(rows))

    def golden_bits(self, **kw) -> np.ndarray:
        return gqa_golden(self.q_bits, self.k_bits, self.v_bits, self.seq_len,
                          self.query_position, group=self.group, **kw)

    def golden_mem_text(self, **kw) -> str:
        return "\n".join(pack_bf16(r) for r in self.golden_bits(**kw).tolist()) + "\n"

    def config_text(self) -> str:
        scale = int(f32_to_bf16(1.0 / math.sqrt(self.head_dim)))
        valid = self.q_heads * self.head_dim + 2 * self.kv_heads * self.seq_len * self.head_dim
        transport = self.q_heads * self.head_dim + 2 * self.kv_heads * self.kv_input_len * self.head_dim
        return (f"SEQ_LEN={self.seq_len}\nHEAD_DIM={self.head_dim}\nTILE_DIM={self.tile_dim}\n"
                f"N_Q_HEADS={self.q_heads}\nN_KV_HEADS={self.kv_heads}\nGROUP_SIZE={self.group}\n"
                f"KV_BLOCK_LEN={self.kv_block_len}\n"
                f"QUERY_POSITION={self.query_position}\nKV_INPUT_SEQ_LEN={self.kv_input_len}\n"
                f"SCALE_BF16=0x{scale:04x}\n"
                f"MODE={self.mode}\nSEED={self.seed}\n"
                f"VALID_INPUT_BF16_VECTORS={valid}\n"
                f"TRANSPORT_BF16_VECTORS={transport}\n")


def generate_case(seq_len: int | None = None, *, mode: str = "smoke", seed: int = 20260731,
                  query_position: int | None = None, kv_block_len: int = 16,
                  target_input_vectors: int | None = None, q_heads: int = 32,
                  kv_heads: int = 8, head_dim: int = 128, tile_dim: int = 16,
                  amplitude: float = 0.25) -> ReferenceCase:
    """Build the inputs ``gen_gqa_wrapper_vectors.py`` builds for the same arguments."""
    if q_heads % kv_heads or head_dim % tile_dim:
        raise ValueError("q-heads must be divisible by kv-heads and head-dim by tile-dim")
    if kv_block_len <= 0:
        raise ValueError("kv-block-len must be positive")
    if seq_len is not None and target_input_vectors is not None:
        raise ValueError("--seq-len and --target-input-vectors are mutually exclusive")
    if target_input_vectors is not None:
        remainder = target_input_vectors - q_heads * head_dim
        per_pos = 2 * kv_heads * head_dim
        if remainder <= 0 or remainder % per_pos:
            raise ValueError("target-input-vectors must equal q-heads*head-dim + N*(2*kv-heads*head-dim)")
        seq_len = remainder // per_pos
    if seq_len is None:
        seq_len = 16
    if seq_len <= 0:
        raise ValueError("seq-len must be positive")
    qpos = seq_len - 1 if query_position is None else query_position
    if not 0 <= qpos < seq_len:
        raise ValueError("query-position must be in [0, seq-len)")
    case = ReferenceCase(seq_len, qpos, kv_block_len, mode, seed, q_heads, kv_heads, head_dim, tile_dim)
    L = case.kv_input_len
    if mode == "smoke":
        q = np.zeros((q_heads, head_dim))
        k = np.zeros((kv_heads, L, head_dim))
        v = np.zeros((kv_heads, L, head_dim))
        for h in range(kv_heads):
            for p in range(seq_len):
                for d in range(head_dim):
                    v[h, p, d] = 0.03125 * (1 + h) + 0.0078125 * p + 0.001953125 * (d % 17)
    elif mode == "random":
        rng = random.Random(seed)
        a = amplitude
        q = np.array([[rng.uniform(-a, a) for _ in range(head_dim)] for _ in range(q_heads)])
        k = np.zeros((kv_heads, L, head_dim))
        v = np.zeros((kv_heads, L, head_dim))
        for h in range(kv_heads):
            for p in range(seq_len):
                k[h, p] = [rng.uniform(-a, a) for _ in range(head_dim)]
        for h in range(kv_heads):
            for p in range(seq_len):
                v[h, p] = [rng.uniform(-a, a) for _ in range(head_dim)]
    else:
        raise ValueError(f"unknown mode {mode!r}")
    case.q_bits = f32_to_bf16(q)
    case.k_bits = f32_to_bf16(k)
    case.v_bits = f32_to_bf16(v)
    return case


def rope_kat(rows: int = 512, seed: int = 20260805, exact: bool = True):
    """The RoPE known-answer rows of ``pyfiles/gen_rope_test_vectors.py:10-23``.

    Returns ``(in_bits, golden_bits)``, each ``[rows, 128]`` uint16; row ``r`` is
    rotated at position ``r``.
    """
    from .golden import rope_half_split
    from .bf16 import bf16_to_f32
    rng = random.Random(seed)
    vals = np.array([[rng.uniform(-0.25, 0.25) for _ in range(128)] for _ in range(rows)])
    in_bits = f32_to_bf16(vals)
    rotated = rope_half_split(bf16_to_f32(in_bits), np.arange(rows), exact=exact)
    return in_bits, f32_to_bf16(rotated)


def beats_text(bits: np.ndarray, tile_dim: int = 16) -> str:
    """``.mem`` text of rows split into ``tile_dim``-element beats (gen_rope_test_vectors.py:21-22)."""
    rows = np.asarray(bits).reshape(-1, bits.shape[-1])
    return mem_text(r[s:s + tile_dim] for r in rows.tolist() for s in range(0, rows.shape[1], tile_dim))
