"""Thread-parallel float64 restatement of the golden, for the timed CPU baseline.

TEST INFRASTRUCTURE / CPU BASELINE ONLY (see package doc).  Same mathematics as
``golden.gqa_golden_f64(exact=False)`` (gen_gqa_wrapper_vectors.py:121-139): RoPE
of Q at QUERY_POSITION and of every key at its position, scores * 1/sqrt(128)
over keys p <= QUERY_POSITION, exact two-pass softmax, weighted V / normaliser,
BF16 rounding.  Key slabs are spread over a thread pool; numpy releases the GIL
inside the slab kernels (elementwise RoPE, BLAS matmul), so the slabs run on
all host cores.
"""
from __future__ import annotations

import math
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .bf16 import bf16_to_f32, f32_to_bf16
from .golden import rope_half_split


def gqa_golden_parallel(q_bits: np.ndarray, k_bits: np.ndarray, v_bits: np.ndarray, seq_len: int,
                        query_position: int, *, group: int = 4, threads: int | None = None,
                        slab: int = 1024, pool: ThreadPoolExecutor | None = None) -> np.ndarray:
    """BF16 codes ``[n_q, D]``; ``k_bits``/``v_bits`` head-major ``[n_kv, >=seq_len, D]``."""
    if not 0 <= query_position < seq_len:
        raise ValueError("query_position must be in [0, seq_len)")
    n_q, d = q_bits.shape
    n_kv = n_q // group
    n_vis = query_position + 1
    scale = 1.0 / math.sqrt(d)
    q_ref = rope_half_split(bf16_to_f32(q_bits)[None], [query_position], exact=False)[0]
    qg = q_ref.reshape(n_kv, group, d)
    slabs = [(p0, min(n_vis, p0 + slab)) for p0 in range(0, n_vis, slab)]

    def scores(rng):
        p0, p1 = rng
        k_ref = rope_half_split(bf16_to_f32(k_bits[:, p0:p1]), np.arange(p0, p1), exact=False)
        return np.matmul(qg, k_ref.transpose(0, 2, 1)) * scale          # [n_kv, group, n]

    own = pool is None
    pool = pool or ThreadPoolExecutor(max_workers=threads or os.cpu_count() or 1)
    try:
        s = np.concatenate(list(pool.map(scores, slabs)), axis=2)           # [n_kv, group, n_vis]
        w = np.exp(s - s.max(axis=2, keepdims=True))
        norm = w.sum(axis=2)

        def weighted(rng):
            p0, p1 = rng
            return np.matmul(w[:, :, p0:p1], bf16_to_f32(v_bits[:, p0:p1]))  # [n_kv, group, D]

        num = sum(pool.map(weighted, slabs))
    finally:
        if own:
            pool.shutdown()
    return f32_to_bf16((num / norm[:, :, None]).reshape(n_q, d))
