"""Python host API over the C ABI: the reference's call surface for the GQA hot path.

The reference drives one decode token per START: Q/K/V BF16 rows plus the
QUERY_POSITION, SEQ_LEN, N_KV_TILES/KV_BLOCK_LEN and GROUP_SIZE registers
(axi_lite_regs.v:5-24, tb_gqa_attention_wrapper.sv:323-329), and receives BF16
[32][128] output rows.  ``decode`` keeps those names and meanings; invalid
register programming raises :class:`GqaConfigError` before anything is
launched, as the RTL's ``config_error`` rejects a START
(gqa_attention_wrapper.v:230-237).

Tensors are torch tensors.  CUDA inputs are used in place; ``decode`` also
takes CPU inputs, copies them to the current CUDA device and copies the result
back (the end-to-end path), while the other entry points refuse CPU tensors.
Tensors of one call must share a device, and a caller's ``out`` must hold every
row the kernel writes; both are checked before anything is launched.  Every
operation runs in ``lib/libgqa_b200.so``; there is no CPU implementation.
"""
from __future__ import annotations

import ctypes
import math
import threading
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import GqaParams, GqaSeqDesc, PARTIAL_FLOATS

N_Q_HEADS = 32
N_KV_HEADS = 8
HEAD_DIM = 128
TILE_DIM = 16
GROUP_SIZE = 4
ROPE_THETA = 500000.0
DEFAULT_KV_BLOCK_LEN = 16

LAYOUTS = ("position_major", "head_major")


class GqaError(RuntimeError):
    """A library call returned a non-zero status."""

    def __init__(self, status: int, where: str = ""):
        self.status = int(status)
        msg = _lib.status_string(status)
        super().__init__(f"{where}: {msg} (status {status})" if where else f"{msg} (status {status})")


class GqaConfigError(GqaError, ValueError):
    """Invalid register programming: the call was rejected before launch."""


def _check(status: int, where: str) -> None:
    if status != _lib.GQA_OK:
        cls = GqaConfigError if status in _lib.CONFIG_ERRORS else GqaError
        raise cls(status, where)


def make_params(*, seq_len: int = 0, query_position: int | None = None,
                kv_block_len: int = DEFAULT_KV_BLOCK_LEN, group_size: int = GROUP_SIZE,
                n_kv_tiles: int | None = None, scale: float | None = None,
                n_q_heads: int = N_Q_HEADS, n_kv_heads: int = N_KV_HEADS, head_dim: int = HEAD_DIM,
                tile_dim: int = TILE_DIM, rope_theta: float = ROPE_THETA) -> GqaParams:
    """Fill the register block of ``gqa_params`` (layout fields are set by the callers)."""
    p = GqaParams()
    p.n_q_heads, p.n_kv_heads, p.head_dim, p.tile_dim = n_q_heads, n_kv_heads, head_dim, tile_dim
    p.seq_len = max(0, int(seq_len))
    p.query_position = (p.seq_len - 1 if query_position is None else int(query_position)) & 0xFFFFFFFF
    p.kv_block_len = max(0, int(kv_block_len))
    if n_kv_tiles is None:
        n_kv_tiles = (p.seq_len + p.kv_block_len - 1) // p.kv_block_len if p.kv_block_len else 0
    p.n_kv_tiles = max(0, int(n_kv_tiles))
    p.scale = 1.0 / math.sqrt(head_dim) if scale is None else float(scale)
    p.group_size = group_size
    p.rope_theta = rope_theta
    return p


def validate(**registers) -> None:
    """Host-only configuration check of a single-sequence call (no GPU needed)."""
    p = make_params(**registers)
    _check(_lib.load().gqa_validate(ctypes.byref(p)), "validate")


# ---------------------------------------------------------------------------
# workspace: one zero-initialised buffer per (device, stream); kernels leave it zeroed
# ---------------------------------------------------------------------------
_ws_lock = threading.Lock()
_ws: dict[tuple[int, int], torch.Tensor] = {}
# Buffers replaced by a larger one stay allocated: a CUDA graph captured with an
# earlier call still holds their device address and would otherwise write into
# memory the allocator has handed to another tensor.
_ws_retired: list[torch.Tensor] = []


def _workspace(device: torch.device, stream_ptr: int, nbytes: int) -> torch.Tensor:
    key = (device.index, stream_ptr)
    with _ws_lock:
        buf = _ws.get(key)
        if buf is None or buf.numel() < nbytes:
            if buf is not None:
                _ws_retired.append(buf)
            buf = torch.zeros(max(nbytes, 4096), dtype=torch.uint8, device=device)
            _ws[key] = buf
        return buf


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _kv_strides(t: torch.Tensor, layout: str) -> tuple[int, int, int]:
    """(pos_stride, head_stride, stored rows) of a K or V tensor."""
    if t.dtype != torch.bfloat16 or t.dim() != 3 or t.shape[-1] != HEAD_DIM or t.stride(-1) != 1:
        raise ValueError(f"K/V must be bfloat16 [..., {HEAD_DIM}] with a contiguous last dim, got {tuple(t.shape)}")
    if layout == "position_major":   # [rows][8][128]
        if t.shape[1] != N_KV_HEADS:
            raise ValueError("position_major K/V must be [rows, 8, 128]")
        return t.stride(0), t.stride(1), t.shape[0]
    if layout == "head_major":       # [8][rows][128]
        if t.shape[0] != N_KV_HEADS:
            raise ValueError("head_major K/V must be [8, rows, 128]")
        return t.stride(1), t.stride(0), t.shape[1]
    raise ValueError(f"layout must be one of {LAYOUTS}")


def _to_device(t: torch.Tensor, device: torch.device) -> torch.Tensor:
    return t.to(device, non_blocking=t.is_pinned())


def _check_out(out: torch.Tensor, shape: tuple, dtype: torch.dtype, device: torch.device) -> None:
    """A caller-supplied output must hold every row the kernel writes: the kernels
    write through the pointer and strides they are given, so a smaller tensor would
    be written past its end."""
    if tuple(out.shape) != tuple(shape) or out.dtype != dtype or out.stride(-1) != 1 or out.device != device:
        raise ValueError(f"out must be {dtype} {list(shape)} on {device} with a contiguous last dim, "
                         f"got {out.dtype} {list(out.shape)} on {out.device}")


def _check_cuda(device: torch.device, **tensors: torch.Tensor) -> None:
    for name, t in tensors.items():
        if t.device != device:
            raise ValueError(f"{name} is on {t.device}; every tensor of this call must be on {device}")


def _set_q_out(p: GqaParams, q: torch.Tensor, out: torch.Tensor, partial: bool) -> None:
    p.q_batch_stride = q.stride(0) if q.dim() == 3 else N_Q_HEADS * HEAD_DIM
    p.q_head_stride = q.stride(-2)
    p.out_batch_stride = out.stride(0) if out.dim() == 3 else (N_Q_HEADS * (PARTIAL_FLOATS if partial else HEAD_DIM))
    p.out_head_stride = out.stride(-2)


def decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, seq_len: int | None = None,
           query_position: int | None = None, kv_block_len: int = DEFAULT_KV_BLOCK_LEN,
           group_size: int = GROUP_SIZE, n_kv_tiles: int | None = None, scale: float | None = None,
           layout: str = "position_major", rope_theta: float = ROPE_THETA,
           n_q_heads: int = N_Q_HEADS, n_kv_heads: int = N_KV_HEADS, head_dim: int = HEAD_DIM,
           tile_dim: int = TILE_DIM, out: torch.Tensor | None = None,
           mask_out: torch.Tensor | None = None, k_rotated: bool = False,
           rtl_numerics: bool = False) -> torch.Tensor:
    """Single-token GQA decode of one sequence; returns BF16 ``[32, 128]``.

    ``q``: BF16 ``[32, 128]``.  ``k``/``v``: BF16 ``[rows, 8, 128]`` (``layout=
    "position_major"``, a KV cache) or ``[8, rows, 128]`` (``"head_major"``, the
    reference's transport order, gen_gqa_wrapper_vectors.py:116-119), rows >= SEQ_LEN.
    ``seq_len`` defaults to the stored rows, ``query_position`` to SEQ_LEN-1,
    ``n_kv_tiles`` to ceil(SEQ_LEN/KV_BLOCK_LEN).  ``mask_out`` (uint8, CUDA,
    >= N_KV_TILES*KV_BLOCK_LEN entries) receives the kernel's key_valid() decisions.
    ``k_rotated``: the K rows were rotated when they were stored (:func:`rope_k_cache`);
    only Q is rotated here (``GQA_FLAG_K_ROTATED``).
    ``rtl_numerics``: reproduce the two quantisations the reference RTL applies
    before the attention arithmetic -- Q and K rotated through its ROM NCO and
    BF16 units (:func:`rope_rtl`, rope_unit.v) and the BF16 SCALE_FACTOR register
    value (0x3DB5, gqa_reference.py:56-57) -- for comparison with an RTL dump.
    """
    lib = _lib.load()
    if rtl_numerics:
        if k_rotated:
            raise ValueError("rtl_numerics rotates K itself; pass the unrotated cache")
        if scale is None:
            scale = RTL_SCALE_128
    if seq_len is None:
        seq_len = k.shape[0] if layout == "position_major" else k.shape[1]
    p = make_params(seq_len=seq_len, query_position=query_position, kv_block_len=kv_block_len,
                    group_size=group_size, n_kv_tiles=n_kv_tiles, scale=scale, n_q_heads=n_q_heads,
                    n_kv_heads=n_kv_heads, head_dim=head_dim, tile_dim=tile_dim, rope_theta=rope_theta)
    _check(lib.gqa_validate(ctypes.byref(p)), "decode")
    if k_rotated:
        p.flags |= _lib.GQA_FLAG_K_ROTATED
    host_io = not q.is_cuda
    device = torch.device("cuda", torch.cuda.current_device()) if host_io else q.device
    if host_io:
        q, k, v = (_to_device(t, device) for t in (q, k, v))
    if q.dtype != torch.bfloat16 or tuple(q.shape[-2:]) != (N_Q_HEADS, HEAD_DIM) or q.stride(-1) != 1:
        raise ValueError("q must be bfloat16 [32, 128] with a contiguous last dim")
    if rtl_numerics:
        qpos = p.query_position
        q = rope_rtl(q.reshape(1, N_Q_HEADS, HEAD_DIM), torch.tensor([qpos], dtype=torch.int32),
                     rope_theta=rope_theta).reshape(N_Q_HEADS, HEAD_DIM)
        rows_k = k.shape[0] if layout == "position_major" else k.shape[1]
        k = rope_rtl(k, torch.arange(rows_k, dtype=torch.int32), layout=layout, rope_theta=rope_theta)
        p.flags |= _lib.GQA_FLAG_Q_ROTATED | _lib.GQA_FLAG_K_ROTATED
    p.k_pos_stride, p.k_head_stride, rows = _kv_strides(k, layout)
    p.v_pos_stride, p.v_head_stride, vrows = _kv_strides(v, layout)
    if rows < seq_len or vrows < seq_len:
        raise ValueError(f"K/V hold {min(rows, vrows)} rows, SEQ_LEN is {seq_len}")
    _check_cuda(device, k=k, v=v)
    if out is not None and out.is_cuda:
        _check_out(out, (N_Q_HEADS, HEAD_DIM) if out.dim() == 2 else (1, N_Q_HEADS, HEAD_DIM), torch.bfloat16, device)
    dev_out = out if (out is not None and out.is_cuda) else torch.empty(
        (N_Q_HEADS, HEAD_DIM), dtype=torch.bfloat16, device=device)
    _set_q_out(p, q, dev_out, False)
    if mask_out is not None:
        need = p.n_kv_tiles * p.kv_block_len
        if mask_out.dtype != torch.uint8 or mask_out.device != device or not mask_out.is_contiguous() \
                or mask_out.numel() < need:
            raise ValueError(f"mask_out must be a contiguous uint8 tensor on {device} with >= {need} entries")
        p.mask_out = mask_out.data_ptr()
        p.mask_stride = mask_out.shape[-1]
    stream = _stream_ptr(device)
    nbytes = lib.gqa_workspace_bytes(ctypes.byref(p), None, 1)
    if nbytes == 0:
        raise GqaError(_lib.GQA_ERR_CUDA, "decode: workspace sizing failed (no supported GPU?)")
    ws = _workspace(device, stream, nbytes)
    _check(lib.gqa_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), dev_out.data_ptr(), ctypes.byref(p),
                          ws.data_ptr(), ws.numel(), stream), "decode")
    if host_io or (out is not None and not out.is_cuda):
        host = out if out is not None else torch.empty((N_Q_HEADS, HEAD_DIM), dtype=torch.bfloat16,
                                                        pin_memory=True)
        host.copy_(dev_out, non_blocking=False)
        return host
    return dev_out


def decode_heads(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, kv_heads: tuple[int, int],
                 seq_len: int | None = None, query_position: int | None = None,
                 kv_block_len: int = DEFAULT_KV_BLOCK_LEN, scale: float | None = None,
                 rope_theta: float = ROPE_THETA, out: torch.Tensor | None = None,
                 k_rotated: bool = False) -> torch.Tensor:
    """:func:`decode` of the KV heads ``kv_heads = (begin, count)`` only (C ABI
    ``gqa_decode_heads``): each KV head and its 4 Q heads depend on no other head
    (gqa_controller.v:159-162), so a sequence's heads can be sharded across GPUs
    with no exchange.

    ``q``: BF16 ``[32, 128]`` on this GPU (the Q rows of the range are read).
    ``k``/``v``: BF16 ``[rows, count, 128]``, position-major, the range's heads
    only.  Writes the range's rows of ``out`` (BF16 ``[32, 128]``, zeros
    elsewhere when allocated here) and returns it.
    """
    lib = _lib.load()
    begin, count = (int(x) for x in kv_heads)
    if seq_len is None:
        seq_len = k.shape[0]
    p = make_params(seq_len=seq_len, query_position=query_position, kv_block_len=kv_block_len, scale=scale,
                    rope_theta=rope_theta)
    _check(lib.gqa_validate(ctypes.byref(p)), "decode_heads")
    if k_rotated:
        p.flags |= _lib.GQA_FLAG_K_ROTATED
    if not q.is_cuda:
        raise ValueError("decode_heads takes CUDA tensors")
    device = q.device
    if q.dtype != torch.bfloat16 or tuple(q.shape) != (N_Q_HEADS, HEAD_DIM) or q.stride(-1) != 1:
        raise ValueError("q must be bfloat16 [32, 128] with a contiguous last dim")
    for name, t in (("k", k), ("v", v)):
        if t.dtype != torch.bfloat16 or t.dim() != 3 or tuple(t.shape[1:]) != (count, HEAD_DIM) or t.stride(-1) != 1:
            raise ValueError(f"{name} must be bfloat16 [rows, {count}, {HEAD_DIM}] with a contiguous last dim")
        if t.shape[0] < seq_len:
            raise ValueError(f"{name} holds {t.shape[0]} rows, SEQ_LEN is {seq_len}")
    _check_cuda(device, k=k, v=v)
    p.k_pos_stride, p.k_head_stride = k.stride(0), k.stride(1)
    p.v_pos_stride, p.v_head_stride = v.stride(0), v.stride(1)
    if out is None:
        out = torch.zeros((N_Q_HEADS, HEAD_DIM), dtype=torch.bfloat16, device=device)
    else:
        _check_out(out, (N_Q_HEADS, HEAD_DIM), torch.bfloat16, device)
    _set_q_out(p, q, out, False)
    stream = _stream_ptr(device)
    nbytes = lib.gqa_workspace_bytes_heads(ctypes.byref(p), count)
    if nbytes == 0:
        raise GqaError(_lib.GQA_ERR_KV_HEADS if not 1 <= count <= N_KV_HEADS else _lib.GQA_ERR_CUDA,
                       "decode_heads: workspace sizing failed")
    ws = _workspace(device, stream, nbytes)
    _check(lib.gqa_decode_heads(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), ctypes.byref(p), begin,
                                count, ws.data_ptr(), ws.numel(), stream), "decode_heads")
    return out


def decode_chunked(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, first_position: int,
                   seq_len: int | None = None, kv_block_len: int = DEFAULT_KV_BLOCK_LEN,
                   scale: float | None = None, layout: str = "position_major", rope_theta: float = ROPE_THETA,
                   out: torch.Tensor | None = None, split_last_wave: bool = True) -> torch.Tensor:
    """Chunked multi-query decode on the tensor cores.

    ``q``: BF16 ``[B, n, 32, 128]`` with n <= 128; query i of sequence b sits at
    position ``first_position + i`` and is answered exactly as :func:`decode`
    with that ``query_position`` and ``seq_len`` (keys p < SEQ_LEN, p <= position).
    ``k``/``v``: BF16 ``[B, rows, 8, 128]`` (``"position_major"``) or
    ``[B, 8, rows, 128]`` (``"head_major"``), rows >= SEQ_LEN.  Returns BF16
    ``[B, n, 32, 128]``.
    """
    lib = _lib.load()
    if q.dim() != 4 or tuple(q.shape[-2:]) != (N_Q_HEADS, HEAD_DIM) or q.dtype != torch.bfloat16 or q.stride(-1) != 1:
        raise ValueError("q must be bfloat16 [B, n, 32, 128] with a contiguous last dim")
    batch, n = q.shape[0], q.shape[1]
    if k.dim() != 4 or v.dim() != 4 or k.shape[0] != batch or v.shape[0] != batch:
        raise ValueError("k and v must be [B, rows, 8, 128] or [B, 8, rows, 128]")
    rows_dim = 1 if layout == "position_major" else 2
    if seq_len is None:
        seq_len = k.shape[rows_dim]
    p = make_params(seq_len=seq_len, query_position=first_position + n - 1, kv_block_len=kv_block_len, scale=scale,
                    rope_theta=rope_theta)
    for t in (k, v):
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1 or t.shape[rows_dim] < seq_len:
            raise ValueError(f"K/V must be bfloat16 with >= SEQ_LEN={seq_len} rows and a contiguous last dim")
    head_dim_idx = 2 if layout == "position_major" else 1
    p.k_pos_stride, p.k_head_stride = k.stride(rows_dim), k.stride(head_dim_idx)
    p.v_pos_stride, p.v_head_stride = v.stride(rows_dim), v.stride(head_dim_idx)
    device = q.device
    if device.type != "cuda":
        raise ValueError("decode_chunked takes CUDA tensors")
    _check_cuda(device, k=k, v=v)
    if out is None:
        out = torch.empty((batch, n, N_Q_HEADS, HEAD_DIM), dtype=torch.bfloat16, device=device)
    _check_out(out, (batch, n, N_Q_HEADS, HEAD_DIM), torch.bfloat16, device)
    p.q_batch_stride, p.q_head_stride = q.stride(0), q.stride(2)
    p.out_batch_stride, p.out_head_stride = out.stride(0), out.stride(2)
    c = _lib.GqaChunkParams(batch=batch, n_queries=n, first_position=first_position, reserved=0,
                            q_query_stride=q.stride(1), out_query_stride=out.stride(1),
                            k_batch_stride=k.stride(0), v_batch_stride=v.stride(0))
    stream = _stream_ptr(device)
    # With room for the partial rows the last, partly filled wave of (sequence,
    # Q head) units is split along the keys (split_last_wave=False: every unit whole).
    nbytes = _lib.CHUNKED_WORKSPACE_BYTES
    if split_last_wave:
        nbytes = max(nbytes, lib.gqa_chunked_workspace_bytes(ctypes.byref(p), ctypes.byref(c)))
    ws = _workspace(device, stream, nbytes)
    _check(lib.gqa_decode_chunked(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), ctypes.byref(p),
                                  ctypes.byref(c), ws.data_ptr(), nbytes, stream), "decode_chunked")
    return out


@dataclass(frozen=True)
class SplitPlan:
    """How a call cuts the keys on the current device (diagnostic)."""
    splits: int          # key splits in total (each runs on 8 CTAs, one per KV head)
    keys_per_split: int
    cluster: int         # > 0: one thread-block cluster per KV head merges on chip


def decode_plan(seq_len: int | None = None, *, query_position: int | None = None,
                plan: "BatchPlan | None" = None) -> SplitPlan:
    """The split plan of :func:`decode` (``seq_len``) or :func:`decode_batch` (``plan``)."""
    lib = _lib.load()
    if (seq_len is None) == (plan is None):
        raise ValueError("give exactly one of seq_len or plan")
    splits, keys, cluster = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    if plan is None:
        p = make_params(seq_len=seq_len, query_position=query_position)
        st = lib.gqa_decode_plan(ctypes.byref(p), None, 1, ctypes.byref(splits), ctypes.byref(keys),
                                 ctypes.byref(cluster))
    else:
        p = make_params(seq_len=1)
        st = lib.gqa_decode_plan(ctypes.byref(p), plan.host, plan.batch, ctypes.byref(splits), ctypes.byref(keys),
                                 ctypes.byref(cluster))
    _check(st, "decode_plan")
    return SplitPlan(splits.value, keys.value, cluster.value)


@dataclass
class BatchPlan:
    """Per-sequence register values of a batched call, in host and device memory.

    Build once with :func:`plan_batch` and reuse across calls with the same
    sequence geometry (a serving loop re-plans only when lengths change).
    """
    host: ctypes.Array
    device: torch.Tensor
    batch: int
    partial: bool

    @property
    def dev_ptr(self) -> int:
        return self.device.data_ptr()


def plan_batch(seq_lens, *, query_positions=None, kv_starts=None, pos_begin=None, pos_end=None,
               device: torch.device | None = None, partial: bool = False) -> BatchPlan:
    """Descriptors for :func:`decode_batch`.

    ``kv_starts[b]`` is the stored row of sequence b's first key (default: the
    sequences packed back to back); ``pos_begin``/``pos_end`` restrict each
    sequence to a stored key range (sequence sharding; defaults 0 / SEQ_LEN).
    """
    seq_lens = [int(s) for s in seq_lens]
    n = len(seq_lens)
    qpos = [s - 1 for s in seq_lens] if query_positions is None else [int(x) for x in query_positions]
    if kv_starts is None:
        kv_starts, acc = [], 0
        for s in seq_lens:
            kv_starts.append(acc)
            acc += s
    pb = [0] * n if pos_begin is None else [int(x) for x in pos_begin]
    pe = list(seq_lens) if pos_end is None else [int(x) for x in pos_end]
    host = (GqaSeqDesc * n)()
    for i in range(n):
        host[i].kv_start, host[i].seq_len, host[i].query_position = int(kv_starts[i]), seq_lens[i], qpos[i]
        host[i].pos_begin, host[i].pos_end = pb[i], pe[i]
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    raw = torch.frombuffer(bytearray(bytes(host)), dtype=torch.uint8)
    dev = raw.pin_memory().to(device, non_blocking=True) if device.type == "cuda" else raw
    return BatchPlan(host=host, device=dev, batch=n, partial=partial)


def decode_batch(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, plan: BatchPlan, *,
                 layout: str = "position_major", scale: float | None = None,
                 rope_theta: float = ROPE_THETA, out: torch.Tensor | None = None,
                 k_rotated: bool = False) -> torch.Tensor:
    """Batched ragged decode: ``q`` BF16 ``[B, 32, 128]``; one token per sequence.

    Returns BF16 ``[B, 32, 128]``, or with ``plan.partial`` FP32 ``[B, 32, 132]``
    partial rows (acc[128], m, l, pad) for a later :func:`combine_partials`.
    ``k_rotated`` as for :func:`decode`.
    """
    lib = _lib.load()
    if q.dim() != 3 or q.shape[0] != plan.batch:
        raise ValueError(f"q must be [B={plan.batch}, 32, 128]")
    p = make_params(seq_len=1, scale=scale, rope_theta=rope_theta)
    p.flags = (_lib.GQA_FLAG_PARTIAL_OUT if plan.partial else 0) | (_lib.GQA_FLAG_K_ROTATED if k_rotated else 0)
    device = q.device
    p.k_pos_stride, p.k_head_stride, k_rows = _kv_strides(k, layout)
    p.v_pos_stride, p.v_head_stride, v_rows = _kv_strides(v, layout)
    for i, d in enumerate(plan.host):
        hi = min(d.pos_end, min(d.seq_len, d.query_position + 1))
        if d.kv_start + max(0, hi - d.pos_begin) > min(k_rows, v_rows):
            raise ValueError(f"sequence {i}: its keys end at stored row "
                             f"{d.kv_start + hi - d.pos_begin}, K/V hold {min(k_rows, v_rows)} rows")
    if device.type != "cuda":
        raise ValueError("decode_batch takes CUDA tensors")
    _check_cuda(device, k=k, v=v, plan=plan.device)
    shape = (plan.batch, N_Q_HEADS, PARTIAL_FLOATS if plan.partial else HEAD_DIM)
    dtype = torch.float32 if plan.partial else torch.bfloat16
    if out is None:
        out = torch.empty(shape, dtype=dtype, device=device)
    _check_out(out, shape, dtype, device)
    _set_q_out(p, q, out, plan.partial)
    stream = _stream_ptr(device)
    nbytes = lib.gqa_workspace_bytes(ctypes.byref(p), plan.host, plan.batch)
    if nbytes == 0:
        _check(lib.gqa_decode_batched(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), ctypes.byref(p),
                                      plan.host, plan.dev_ptr, plan.batch, None, 0, stream), "decode_batch")
        raise GqaError(_lib.GQA_ERR_CUDA, "decode_batch: workspace sizing failed")
    ws = _workspace(device, stream, nbytes)
    _check(lib.gqa_decode_batched(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), ctypes.byref(p),
                                  plan.host, plan.dev_ptr, plan.batch, ws.data_ptr(), ws.numel(), stream),
           "decode_batch")
    return out


def combine_partials(parts: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Log-sum-exp merge of FP32 partials ``[n_parts, B, 32, 132]`` into BF16 ``[B, 32, 128]``."""
    lib = _lib.load()
    if parts.dtype != torch.float32 or parts.dim() != 4 or parts.shape[-1] != PARTIAL_FLOATS \
            or parts.shape[-2] != N_Q_HEADS or parts.stride(-1) != 1 or parts.stride(-2) != PARTIAL_FLOATS:
        raise ValueError("parts must be float32 [n_parts, B, 32, 132] with contiguous rows")
    n, b = parts.shape[0], parts.shape[1]
    if parts.device.type != "cuda":
        raise ValueError("combine_partials takes CUDA tensors")
    if out is None:
        out = torch.empty((b, N_Q_HEADS, HEAD_DIM), dtype=torch.bfloat16, device=parts.device)
    _check_out(out, (b, N_Q_HEADS, HEAD_DIM), torch.bfloat16, parts.device)
    _check(lib.gqa_combine_partials(parts.data_ptr(), n, parts.stride(0), parts.stride(1), b, out.data_ptr(),
                                    out.stride(0), out.stride(1), _stream_ptr(parts.device)), "combine_partials")
    return out


def rope_rows(x: torch.Tensor, positions: torch.Tensor, rope_theta: float = ROPE_THETA) -> torch.Tensor:
    """RoPE of BF16 rows ``[rows, 128]`` at int32 ``positions`` -> FP32 rows (device code of the kernels)."""
    lib = _lib.load()
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != HEAD_DIM or not x.is_contiguous() or not x.is_cuda:
        raise ValueError("x must be a contiguous bfloat16 CUDA tensor [rows, 128]")
    positions = positions.to(device=x.device, dtype=torch.int32).contiguous()
    out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    _check(lib.gqa_rope_rows(x.data_ptr(), positions.data_ptr(), out.data_ptr(), x.shape[0], rope_theta,
                             _stream_ptr(x.device)), "rope_rows")
    return out


def rope_k_cache(k: torch.Tensor, positions: torch.Tensor, *, layout: str = "position_major",
                 rope_theta: float = ROPE_THETA, out: torch.Tensor | None = None) -> torch.Tensor:
    """Pre-rotated K cache: RoPE of BF16 K rows ``[n, 8, 128]`` (``position_major``) or
    ``[8, n, 128]`` (``head_major``), position i turned by ``positions[i]``, to BF16 rows
    of the same layout (``out=k`` rotates in place).  Decode the result with
    ``k_rotated=True``.  This is the append-time half of the reference's per-call K
    RoPE (gen_gqa_wrapper_vectors.py:122-124)."""
    lib = _lib.load()
    if k.dtype != torch.bfloat16 or k.dim() != 3 or not k.is_cuda:
        raise ValueError("k must be a bfloat16 CUDA tensor [n, 8, 128] or [8, n, 128]")
    pos_stride, head_stride, n = _kv_strides(k, layout)
    positions = positions.to(device=k.device, dtype=torch.int32).contiguous()
    if positions.numel() != n:
        raise ValueError(f"{positions.numel()} positions for {n} stored rows")
    if out is None:
        out = torch.empty_like(k)
    if out.shape != k.shape or out.stride() != k.stride() or out.dtype != torch.bfloat16 or out.device != k.device:
        raise ValueError("out must match k's shape, strides, dtype and device")
    _check(lib.gqa_rope_k_cache(k.data_ptr(), out.data_ptr(), positions.data_ptr(), n, pos_stride, head_stride,
                                rope_theta, _stream_ptr(k.device)), "rope_k_cache")
    return out


RTL_ROM_ADDR_BITS = 14           # rope_unit.v:46
RTL_SCALE_128 = 0.08837890625    # BF16 0x3DB5 = bf16(1/sqrt(128)), the SCALE_FACTOR register value
_rtl_roms: dict = {}


def _rtl_rom_tables(device: torch.device, rope_theta: float, bits: int):
    """Device copies of the phase and sincos ROMs, built once per (device, theta, bits)."""
    key = (device, float(rope_theta), bits)
    with _ws_lock:
        if key not in _rtl_roms:
            phase = torch.tensor(rope_phase_rom(HEAD_DIM, rope_theta), dtype=torch.int64).to(torch.int32)
            sincos = torch.tensor(rope_sincos_rom(bits), dtype=torch.int64).to(torch.int32)
            _rtl_roms[key] = (phase.to(device), sincos.to(device))
        return _rtl_roms[key]


def rope_rtl(x: torch.Tensor, positions: torch.Tensor, *, layout: str = "position_major",
             rope_theta: float = ROPE_THETA, rom_addr_bits: int = RTL_ROM_ADDR_BITS,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """RoPE as the reference RTL computes it (rope_unit.v): ROM NCO factors and BF16
    multiply/add units.  ``x``: BF16 rows ``[n, H, 128]`` (``position_major``) or
    ``[H, n, 128]`` (``head_major``), position i turned by ``positions[i]``; returns
    BF16 rows of the same layout."""
    lib = _lib.load()
    if x.dtype != torch.bfloat16 or x.dim() != 3 or x.shape[-1] != HEAD_DIM or not x.is_cuda or x.stride(-1) != 1:
        raise ValueError("x must be a bfloat16 CUDA tensor [n, H, 128] or [H, n, 128]")
    if layout == "position_major":
        n, heads, pos_stride, head_stride = x.shape[0], x.shape[1], x.stride(0), x.stride(1)
    elif layout == "head_major":
        n, heads, pos_stride, head_stride = x.shape[1], x.shape[0], x.stride(1), x.stride(0)
    else:
        raise ValueError(f"layout must be one of {LAYOUTS}")
    positions = positions.to(device=x.device, dtype=torch.int32).contiguous()
    if positions.numel() != n:
        raise ValueError(f"{positions.numel()} positions for {n} rows per head")
    phase, sincos = _rtl_rom_tables(x.device, rope_theta, rom_addr_bits)
    if out is None:
        out = torch.empty_like(x)
    if out.shape != x.shape or out.stride() != x.stride() or out.dtype != torch.bfloat16 or out.device != x.device:
        raise ValueError("out must match x's shape, strides, dtype and device")  # written with x's strides
    _check(lib.gqa_rope_rtl(x.data_ptr(), out.data_ptr(), positions.data_ptr(), n, heads, pos_stride, head_stride,
                            phase.data_ptr(), sincos.data_ptr(), rom_addr_bits, _stream_ptr(x.device)), "rope_rtl")
    return out


def rope_phase_rom(head_dim: int = HEAD_DIM, rope_theta: float = ROPE_THETA) -> list[int]:
    """Phase ROM of tools/gen_rope_rom.py (Q0.32 turns per position, one per pair)."""
    buf = (ctypes.c_uint32 * (head_dim // 2))()
    _check(_lib.load().gqa_rope_phase_rom(buf, head_dim, rope_theta), "rope_phase_rom")
    return list(buf)


def rope_sincos_rom(addr_bits: int = 10) -> list[int]:
    """{cos_bf16, sin_bf16} ROM of tools/gen_rope_rom.py, 2**addr_bits 32-bit entries."""
    buf = (ctypes.c_uint32 * (1 << addr_bits))()
    _check(_lib.load().gqa_rope_sincos_rom(buf, addr_bits), "rope_sincos_rom")
    return list(buf)


def read_device_status(device: torch.device | None = None) -> int:
    """Status word the kernels left in this stream's workspace (GQA_OK or GQA_ERR_DEVICE_TIMEOUT)."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    stream = _stream_ptr(device)
    ws = _workspace(device, stream, 4096)
    st = ctypes.c_int(0)
    _check(_lib.load().gqa_read_status(ws.data_ptr(), stream, ctypes.byref(st)), "read_device_status")
    return st.value
