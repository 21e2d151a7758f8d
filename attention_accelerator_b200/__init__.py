"""B200-native (sm_100a) GQA decode-attention hot path of the attention_accelerator reference.

Public API (see ``api``): :func:`decode`, :func:`decode_heads`, :func:`plan_batch` + :func:`decode_batch`,
:func:`decode_chunked`, :func:`combine_partials`, :func:`decode_plan`, :func:`rope_rows`, :func:`rope_k_cache`,
:func:`rope_rtl`, :func:`rope_phase_rom`, :func:`rope_sincos_rom`, :func:`validate`,
:func:`read_device_status`; the ``.mem`` codec in ``memfile``; the multi-GPU
long-context exchange in ``distributed``.  All compute runs in
``lib/libgqa_b200.so`` through the C ABI of ``include/gqa_b200.h``.
"""
from .api import (DEFAULT_KV_BLOCK_LEN, GROUP_SIZE, HEAD_DIM, N_KV_HEADS, N_Q_HEADS, ROPE_THETA, TILE_DIM,
                  BatchPlan, GqaConfigError, GqaError, SplitPlan, combine_partials, decode, decode_batch, decode_chunked,
                  decode_heads,
                  decode_plan, make_params, plan_batch, read_device_status, rope_k_cache, rope_phase_rom, rope_rtl,
                  rope_rows, rope_sincos_rom, validate)

__all__ = ["decode", "decode_heads", "decode_batch", "decode_chunked", "plan_batch", "BatchPlan", "decode_plan", "SplitPlan", "combine_partials", "rope_rows",
           "rope_k_cache", "rope_rtl",
           "rope_phase_rom", "rope_sincos_rom", "validate", "make_params", "read_device_status",
           "GqaError", "GqaConfigError", "N_Q_HEADS", "N_KV_HEADS", "HEAD_DIM", "TILE_DIM", "GROUP_SIZE",
           "ROPE_THETA", "DEFAULT_KV_BLOCK_LEN"]
