"""Float64 partial attention over a key range and its log-sum-exp merge (test infrastructure).

The golden (gen_gqa_wrapper_vectors.py:121-139) takes one softmax over all
visible keys.  Over a key shard [lo, hi) the same quantities split as
  m = max_p s_p,  l = sum_p 2^(s_p - m),  acc = sum_p 2^(s_p - m) v_p
with scores s in log2 units (s_natural * log2(e)); shards merge exactly by
  M = max m_s,  out = sum 2^(m_s - M) acc_s / sum 2^(m_s - M) l_s.
These restatements check the multi-GPU decomposition on CPU.
"""
from __future__ import annotations

import math

import numpy as np

from .bf16 import bf16_to_f32, f32_to_bf16
from .golden import rope_half_split

LOG2E = 1.0 / math.log(2.0)


def partial_f64(q_bits, k_bits, v_bits, query_position: int, lo: int, hi: int, group: int = 4):
    """(acc [n_q, D], m [n_q], l [n_q]) of keys [lo, min(hi, query_position + 1))."""
    n_q, d = q_bits.shape
    hi = min(hi, query_position + 1)
    head_of = np.arange(n_q) // group
    if hi <= lo:
        return np.zeros((n_q, d)), np.full(n_q, -np.inf), np.zeros(n_q)
    q = rope_half_split(bf16_to_f32(q_bits)[None], [query_position], exact=False)[0]
    k = rope_half_split(bf16_to_f32(k_bits[:, lo:hi]), np.arange(lo, hi), exact=False)
    s = np.einsum("hd,hpd->hp", q, k[head_of]) / math.sqrt(d) * LOG2E
    m = s.max(axis=1)
    w = np.exp2(s - m[:, None])
    acc = np.einsum("hp,hpd->hd", w, bf16_to_f32(v_bits[:, lo:hi])[head_of])
    return acc, m, w.sum(axis=1)


def combine_f64(parts) -> np.ndarray:
    """Merge [(acc, m, l), ...] into BF16 output codes [n_q, D]."""
    ms = np.stack([p[1] for p in parts])
    big = ms.max(axis=0)
    f = np.exp2(ms - big[None])
    f[~np.isfinite(ms)] = 0.0
    num = sum(fi[:, None] * p[0] for fi, p in zip(f, parts))
    den = sum(fi * p[2] for fi, p in zip(f, parts))
    return f32_to_bf16(num / den[:, None])


def to_rows(acc, m, l) -> np.ndarray:
    """Pack a partial into the library's gqa_partial_row layout [n_q, 132] (float64)."""
    rows = np.zeros((acc.shape[0], 132))
    rows[:, :128], rows[:, 128], rows[:, 129] = acc, m, l
    return rows


def from_rows(rows):
    rows = np.asarray(rows, dtype=np.float64)
    return rows[:, :128], rows[:, 128], rows[:, 129]
