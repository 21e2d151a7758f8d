"""ctypes binding of ``include/gqa_b200.h`` (the library's C ABI).

Loading fails loudly when ``lib/libgqa_b200.so`` is missing: there is no
fallback implementation of any operation.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libgqa_b200.so"

GQA_OK = 0
GQA_ERR_GEOMETRY = 1
GQA_ERR_SEQ_LEN = 2
GQA_ERR_N_KV_TILES = 3
GQA_ERR_SCALE = 4
GQA_ERR_QUERY_POSITION = 5
GQA_ERR_KV_BLOCK_LEN = 6
GQA_ERR_GROUP_SIZE = 7
GQA_ERR_NULL_POINTER = 8
GQA_ERR_ALIGNMENT = 9
GQA_ERR_WORKSPACE = 10
GQA_ERR_BATCH = 11
GQA_ERR_KV_RANGE = 12
GQA_ERR_CUDA = 13
GQA_ERR_DEVICE_TIMEOUT = 14
GQA_ERR_UNSUPPORTED_DEVICE = 15
GQA_ERR_ROPE_THETA = 16
GQA_ERR_FLAGS = 17
GQA_ERR_MEMORY = 18
GQA_ERR_KV_HEADS = 19

#: codes that describe a bad call configuration (the reference's config_error)
CONFIG_ERRORS = {GQA_ERR_GEOMETRY, GQA_ERR_SEQ_LEN, GQA_ERR_N_KV_TILES, GQA_ERR_SCALE,
                 GQA_ERR_QUERY_POSITION, GQA_ERR_KV_BLOCK_LEN, GQA_ERR_GROUP_SIZE,
                 GQA_ERR_BATCH, GQA_ERR_KV_RANGE, GQA_ERR_ROPE_THETA}

GQA_FLAG_PARTIAL_OUT = 0x1
GQA_FLAG_K_ROTATED = 0x2
GQA_FLAG_Q_ROTATED = 0x4
PARTIAL_FLOATS = 132


class GqaParams(ctypes.Structure):
    """Mirror of ``struct gqa_params``."""
    _fields_ = [
        ("n_q_heads", ctypes.c_uint32), ("n_kv_heads", ctypes.c_uint32),
        ("head_dim", ctypes.c_uint32), ("tile_dim", ctypes.c_uint32),
        ("seq_len", ctypes.c_uint32), ("n_kv_tiles", ctypes.c_uint32),
        ("scale", ctypes.c_float), ("query_position", ctypes.c_uint32),
        ("kv_block_len", ctypes.c_uint32), ("group_size", ctypes.c_uint32),
        ("rope_theta", ctypes.c_float), ("flags", ctypes.c_uint32),
        ("q_batch_stride", ctypes.c_int64), ("q_head_stride", ctypes.c_int64),
        ("k_pos_stride", ctypes.c_int64), ("k_head_stride", ctypes.c_int64),
        ("v_pos_stride", ctypes.c_int64), ("v_head_stride", ctypes.c_int64),
        ("out_batch_stride", ctypes.c_int64), ("out_head_stride", ctypes.c_int64),
        ("mask_out", ctypes.c_void_p), ("mask_stride", ctypes.c_int64),
    ]


class GqaSeqDesc(ctypes.Structure):
    """Mirror of ``struct gqa_seq_desc`` (24 bytes)."""
    _fields_ = [("kv_start", ctypes.c_int64), ("seq_len", ctypes.c_int32),
                ("query_position", ctypes.c_int32), ("pos_begin", ctypes.c_int32),
                ("pos_end", ctypes.c_int32)]


class GqaChunkParams(ctypes.Structure):
    """Mirror of ``struct gqa_chunk_params`` (48 bytes)."""
    _fields_ = [("batch", ctypes.c_uint32), ("n_queries", ctypes.c_uint32),
                ("first_position", ctypes.c_uint32), ("reserved", ctypes.c_uint32),
                ("q_query_stride", ctypes.c_int64), ("out_query_stride", ctypes.c_int64),
                ("k_batch_stride", ctypes.c_int64), ("v_batch_stride", ctypes.c_int64)]


CHUNKED_WORKSPACE_BYTES = 256
PEER_HANDLE_BYTES = 64
CHUNKED_MAX_QUERIES = 128
MEM_MAX_ELEMENTS = 4096

_P = ctypes.c_void_p
_SIGNATURES = {
    "gqa_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "gqa_version": (ctypes.c_int, []),
    "gqa_device_supported": (ctypes.c_int, [ctypes.c_int]),
    "gqa_validate": (ctypes.c_int, [ctypes.POINTER(GqaParams)]),
    "gqa_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(GqaParams), ctypes.POINTER(GqaSeqDesc), ctypes.c_int]),
    "gqa_decode_plan": (ctypes.c_int, [ctypes.POINTER(GqaParams), ctypes.POINTER(GqaSeqDesc), ctypes.c_int,
                                       ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                       ctypes.POINTER(ctypes.c_int)]),
    "gqa_decode_plan_host": (ctypes.c_int, [ctypes.POINTER(GqaParams), ctypes.POINTER(GqaSeqDesc), ctypes.c_int,
                                            ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    "gqa_decode": (ctypes.c_int, [_P, _P, _P, _P, ctypes.POINTER(GqaParams), _P, ctypes.c_size_t, _P]),
    "gqa_decode_noalloc": (ctypes.c_int, [_P, _P, _P, _P, ctypes.POINTER(GqaParams), _P]),
    "gqa_workspace_bytes_heads": (ctypes.c_size_t, [ctypes.POINTER(GqaParams), ctypes.c_int]),
    "gqa_decode_heads": (ctypes.c_int, [_P, _P, _P, _P, ctypes.POINTER(GqaParams), ctypes.c_int, ctypes.c_int, _P,
                                        ctypes.c_size_t, _P]),
    "gqa_decode_batched": (ctypes.c_int, [_P, _P, _P, _P, ctypes.POINTER(GqaParams), ctypes.POINTER(GqaSeqDesc),
                                          _P, ctypes.c_int, _P, ctypes.c_size_t, _P]),
    "gqa_decode_chunked": (ctypes.c_int, [_P, _P, _P, _P, ctypes.POINTER(GqaParams), ctypes.POINTER(GqaChunkParams),
                                          _P, ctypes.c_size_t, _P]),
    "gqa_peer_buffer_bytes": (ctypes.c_size_t, [ctypes.c_int]),
    "gqa_peer_buffer_create": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), _P]),
    "gqa_peer_buffer_open": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "gqa_peer_buffer_close": (ctypes.c_int, [_P]),
    "gqa_peer_buffer_destroy": (ctypes.c_int, [_P]),
    "gqa_combine_peers": (ctypes.c_int, [_P, ctypes.c_int64, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P,
                                         ctypes.c_int64, ctypes.c_int64, _P, _P]),
    "gqa_decode_exchange": (ctypes.c_int, [_P, _P, _P, _P, ctypes.POINTER(GqaParams), ctypes.POINTER(GqaSeqDesc), _P,
                                           ctypes.c_int, ctypes.c_int, _P, ctypes.c_size_t, _P]),
    "gqa_combine_partials": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _P,
                                            ctypes.c_int64, ctypes.c_int64, _P]),
    "gqa_rope_rows": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, ctypes.c_float, _P]),
    "gqa_rope_phase_rom": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int, ctypes.c_double]),
    "gqa_rope_sincos_rom": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]),
    "gqa_read_status": (ctypes.c_int, [_P, _P, ctypes.POINTER(ctypes.c_int)]),
    "gqa_rope_k_cache": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, _P]),
    "gqa_rope_rtl": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, _P, _P,
                                    ctypes.c_int, _P]),
    "gqa_chunked_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(GqaParams), ctypes.POINTER(GqaChunkParams)]),
    "gqa_mem_decode_workspace_bytes": (ctypes.c_size_t, [ctypes.c_size_t]),
    "gqa_mem_decode": (ctypes.c_int, [_P, ctypes.c_size_t, ctypes.c_int, _P, ctypes.c_uint64, _P, _P,
                                      ctypes.c_size_t, _P]),
    "gqa_mem_encode_bytes": (ctypes.c_size_t, [ctypes.c_uint64, ctypes.c_int]),
    "gqa_mem_encode": (ctypes.c_int, [_P, ctypes.c_uint64, ctypes.c_int, _P, _P]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the CUDA library (once); raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.is_file():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m attention_accelerator_b200.build` "
                    "(there is no CPU implementation to fall back to)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def status_string(code: int) -> str:
    return load().gqa_status_string(int(code)).decode()


def exported_symbols() -> list[str]:
    return sorted(_SIGNATURES)
