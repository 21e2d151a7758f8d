"""Float64 oracle of chunked multi-query decode (test infrastructure, see package doc).

A chunk is n consecutive query positions t = t0 .. t0+n-1 of one sequence,
each answered exactly as one single-position reference call with
QUERY_POSITION = t and SEQ_LEN = S (gen_gqa_wrapper_vectors.py:121-139): RoPE
of Q at t and of every K row at its position, scores scaled by 1/sqrt(128)
over keys p <= t, softmax, weighted V, BF16 RNE.  This is the same float64
arithmetic as ``gqa_golden_f64(..., exact=False)``, with each sequence's K
rotated once for all of its queries.
"""
from __future__ import annotations

import math

import numpy as np

from .bf16 import bf16_to_f32, f32_to_bf16
from .golden import ROPE_THETA, rope_half_split


def chunked_golden_f64(q_bits: np.ndarray, k_bits: np.ndarray, v_bits: np.ndarray, seq_len: int,
                       first_position: int, *, group: int = 4, theta: float = ROPE_THETA) -> np.ndarray:
    """Float64 outputs ``[B, n, n_q_heads, D]``.

    ``q_bits``: ``[B, n, n_q_heads, D]`` BF16 codes (query i at position
    first_position + i); ``k_bits``/``v_bits``: ``[B, n_kv, >= seq_len, D]``
    head-major BF16 codes.
    """
    b_n, n, n_q, d = q_bits.shape
    if not (0 <= first_position and first_position + n <= seq_len):
        raise ValueError("query positions must lie in [0, seq_len)")
    n_vis = first_position + n                     # keys any query of the chunk can see
    head_of = np.arange(n_q) // group
    scale = 1.0 / math.sqrt(d)
    positions = np.arange(first_position, first_position + n)
    out = np.empty((b_n, n, n_q, d), dtype=np.float64)
    for b in range(b_n):
        k_ref = rope_half_split(bf16_to_f32(k_bits[b, :, :n_vis]), np.arange(n_vis), theta, exact=False)
        v_ref = bf16_to_f32(v_bits[b, :, :n_vis]).astype(np.float64)
        for qh in range(n_q):
            q_rows = bf16_to_f32(q_bits[b, :, qh]).astype(np.float64)               # [n, D]
            q_ref = rope_half_split(q_rows, positions, theta, exact=False)
            g = head_of[qh]
            scores = (q_ref @ k_ref[g].T) * scale                                   # [n, n_vis]
            visible = np.arange(n_vis)[None, :] <= positions[:, None]               # p <= t
            scores = np.where(visible, scores, -np.inf)
            weights = np.exp(scores - scores.max(axis=1, keepdims=True))
            out[b, :, qh] = (weights @ v_ref[g]) / weights.sum(axis=1)[:, None]
    return out


def chunked_golden(q_bits, k_bits, v_bits, seq_len: int, first_position: int, **kw) -> np.ndarray:
    """BF16 codes ``[B, n, n_q_heads, D]`` of the chunked golden."""
    return f32_to_bf16(chunked_golden_f64(q_bits, k_bits, v_bits, seq_len, first_position, **kw))
