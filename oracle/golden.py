"""Float64 restatement of the reference GQA golden (test infrastructure, see package doc).

Follows ``pyfiles/gen_gqa_wrapper_vectors.py``:
  * ``rope_half_split``  -> :25-35  (Llama rotate_half, pair (i, i+64),
                                      angle = pos * theta ** (-2.0*i/128))
  * ``gqa_golden``       -> :121-139 (dequantise, RoPE Q at QUERY_POSITION and K
                                      at each key position, scores * 1/sqrt(128)
                                      over keys p <= QUERY_POSITION, exact two-pass
                                      softmax, weighted V / normaliser, BF16 RNE)

``exact=True`` (default) reproduces the reference bit for bit under CPython >= 3.12:
  - the three ``sum()`` calls (:132, :136, :137) are CPython's float ``sum``, which
    since 3.12 is Neumaier's compensated summation (Neumaier 1974, "Rundungs-
    fehleranalyse einiger Verfahren zur Summation endlicher Summen"); it is
    restated here term by term in the same order;
  - ``math.cos``/``math.sin``/``math.exp`` and Python's ``**`` are called (numpy's
    ``exp`` and ``power`` differ from libm in the last ulp on this machine).
``exact=False`` is a BLAS/numpy float64 version of the same math, used as the
timed CPU baseline; its BF16 outputs agree with ``exact=True`` (checked in tests).
"""
from __future__ import annotations

import math

import numpy as np

from .bf16 import bf16_to_f32, f32_to_bf16

HEAD_DIM = 128
ROPE_THETA = 500000.0


def rope_inv_freq(head_dim: int = HEAD_DIM, theta: float = ROPE_THETA) -> np.ndarray:
    """``theta ** (-2.0 * i / head_dim)`` per pair, computed with Python's ``**``."""
    return np.array([theta ** (-2.0 * i / head_dim) for i in range(head_dim // 2)], dtype=np.float64)


def _trig(angle: np.ndarray, exact: bool):
    if exact:
        flat = angle.ravel().tolist()
        c = np.fromiter((math.cos(a) for a in flat), dtype=np.float64, count=len(flat))
        s = np.fromiter((math.sin(a) for a in flat), dtype=np.float64, count=len(flat))
        return c.reshape(angle.shape), s.reshape(angle.shape)
    return np.cos(angle), np.sin(angle)


def rope_half_split(rows: np.ndarray, positions, theta: float = ROPE_THETA,
                    exact: bool = True) -> np.ndarray:
    """Rotate float64 rows ``[..., n, D]`` at integer ``positions`` (shape ``[n]``).

    gen_gqa_wrapper_vectors.py:25-35: out[i] = x*c - y*s, out[i+D/2] = x*s + y*c.
    """
    rows = np.asarray(rows, dtype=np.float64)
    d = rows.shape[-1]
    half = d // 2
    pos = np.asarray(positions, dtype=np.int64).astype(np.float64)
    inv = rope_inv_freq(d, theta)
    angle = pos[:, None] * inv[None, :]                       # [n, half]
    c, s = _trig(angle, exact)
    x, y = rows[..., :half], rows[..., half:]
    out = np.empty_like(rows)
    out[..., :half] = x * c - y * s
    out[..., half:] = x * s + y * c
    return out


def _neumaier_rows(terms: np.ndarray) -> np.ndarray:
    """CPython-3.12 float ``sum()`` over the LAST axis, vectorised over the others.

    The first term becomes the running sum (``0 + x0`` is exact); each later term
    updates the compensation exactly as the Neumaier branch of builtin ``sum``.
    """
    f = terms[..., 0].copy()
    c = np.zeros_like(f)
    for j in range(1, terms.shape[-1]):
        x = terms[..., j]
        t = f + x
        c += np.where(np.abs(f) >= np.abs(x), (f - t) + x, (x - t) + f)
        f = t
    return np.where((c != 0) & np.isfinite(c), f + c, f)


class _Neumaier:
    """Running CPython-style float sum for terms that arrive one slab at a time."""

    def __init__(self, first: np.ndarray):
        self.f = first.astype(np.float64).copy()
        self.c = np.zeros_like(self.f)

    def add(self, x: np.ndarray) -> None:
        f = self.f
        t = f + x
        self.c += np.where(np.abs(f) >= np.abs(x), (f - t) + x, (x - t) + f)
        self.f = t

    def value(self) -> np.ndarray:
        return np.where((self.c != 0) & np.isfinite(self.c), self.f + self.c, self.f)


def gqa_golden_f64(q_bits: np.ndarray, k_bits: np.ndarray, v_bits: np.ndarray,
                   seq_len: int, query_position: int, *, group: int = 4,
                   theta: float = ROPE_THETA, exact: bool = True,
                   pos_chunk: int = 2048, k_rotated: bool = False, q_rotated: bool = False,
                   scale: float | None = None) -> np.ndarray:
    """Float64 attention output ``[n_q_heads, D]`` before the final BF16 rounding.

    ``q_bits``: ``[n_q, D]`` BF16 codes; ``k_bits``/``v_bits``: ``[n_kv, >=seq_len, D]``
    BF16 codes in head-major order (gen_gqa_wrapper_vectors.py:85-107).
    Keys ``p`` in ``[0, query_position]`` contribute (:132-133); rows past that are
    never read, which is the pad/causal mask of :83 and :125-126.
    ``k_rotated``: ``k_bits`` already hold rotated keys (a pre-rotated K cache), so
    the per-key rope_half_split of :122-124 is skipped; ``q_rotated`` likewise for
    Q.  ``scale`` replaces the exact 1/sqrt(D) of :129 (the RTL-numerics mode uses
    the BF16 SCALE_FACTOR register value).
    """
    if not 0 <= query_position < seq_len:
        raise ValueError("query_position must be in [0, seq_len)")
    n_q, d = q_bits.shape
    n_vis = query_position + 1
    head_of = np.arange(n_q) // group                           # gqa_controller.v:159-162
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    q_ref = (bf16_to_f32(q_bits) if q_rotated
             else rope_half_split(bf16_to_f32(q_bits)[None], [query_position], theta, exact)[0])

    # Scores, one slab of key positions at a time (bounded memory at 131072 keys).
    scores = np.empty((n_q, n_vis), dtype=np.float64)
    for p0 in range(0, n_vis, pos_chunk):
        p1 = min(n_vis, p0 + pos_chunk)
        k_ref = (bf16_to_f32(k_bits[:, p0:p1]) if k_rotated
                 else rope_half_split(bf16_to_f32(k_bits[:, p0:p1]), np.arange(p0, p1), theta, exact))
        kq = k_ref[head_of]                                     # [n_q, n, D]
        if exact:
            prods = q_ref[:, None, :] * kq                      # per-element products, :132
            scores[:, p0:p1] = _neumaier_rows(prods) * scale
        else:
            scores[:, p0:p1] = np.einsum("hd,hpd->hp", q_ref, kq) * scale

    max_score = scores.max(axis=1, keepdims=True)
    if exact:
        flat = (scores - max_score).ravel().tolist()
        weights = np.fromiter((math.exp(x) for x in flat), dtype=np.float64,
                              count=len(flat)).reshape(scores.shape)
        normalizer = _neumaier_rows(weights)                    # :136
        acc = None
        for p0 in range(0, n_vis, pos_chunk):                   # :137-138, order p = 0..qpos
            p1 = min(n_vis, p0 + pos_chunk)
            v_ref = bf16_to_f32(v_bits[:, p0:p1])[head_of]      # [n_q, n, D]
            terms = weights[:, p0:p1, None] * v_ref
            for j in range(p1 - p0):
                if acc is None:
                    acc = _Neumaier(terms[:, j])
                else:
                    acc.add(terms[:, j])
        num = acc.value()
    else:
        weights = np.exp(scores - max_score)
        normalizer = weights.sum(axis=1)
        num = np.zeros((n_q, d), dtype=np.float64)
        for p0 in range(0, n_vis, pos_chunk):
            p1 = min(n_vis, p0 + pos_chunk)
            v_ref = bf16_to_f32(v_bits[:, p0:p1])               # [n_kv, n, D]
            for g in range(n_q // group):
                hs = slice(g * group, (g + 1) * group)
                num[hs] += weights[hs, p0:p1] @ v_ref[g]
    return num / normalizer[:, None]


def gqa_golden(q_bits, k_bits, v_bits, seq_len: int, query_position: int, **kw) -> np.ndarray:
    """BF16 codes ``[n_q, D]`` of the golden output (gen_gqa_wrapper_vectors.py:137-139)."""
    return f32_to_bf16(gqa_golden_f64(q_bits, k_bits, v_bits, seq_len, query_position, **kw))
