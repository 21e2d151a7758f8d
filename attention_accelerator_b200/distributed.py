"""Multi-GPU plumbing for the decode path: one process per GPU over torch.distributed.

Three schemes:

* **KV-head sharding (no collective).**  One sequence's 8 KV heads are split
  across ranks by :func:`head_range`; each rank holds the K/V rows of its heads
  only and decodes them with ``decode_heads`` (a KV head and its 4 Q heads
  depend on no other head, gqa_controller.v:159-162); the output rows are
  disjoint.
* **Sequence sharding (no collective).**  A batch of decode requests is split
  across ranks by :func:`balance_sequences` (greedy longest-first assignment
  by visible-key count); every rank decodes its own sequences.
* **Long-context split.**  One sequence's keys are cut into contiguous shards,
  :func:`shard_range`; each rank computes FP32 partial rows for its shard
  (``plan_batch(..., pos_begin, pos_end, partial=True)`` + ``decode_batch``).
  :class:`PeerExchange` then exchanges them over NVLink peer memory and merges
  them: :meth:`PeerExchange.decode` does it inside the decode kernel (the CTA
  that merges each KV head's splits publishes the rows, waits for the peers'
  and writes the final output), :meth:`PeerExchange.combine` in a separate
  kernel after ``decode_batch(partial=True)``; :func:`gather_partials` +
  ``combine_partials`` is the same step with an NCCL all-gather.

The reference has a single device and no collective; this is the scaling
scheme of the new build.
"""
from __future__ import annotations

import ctypes
import heapq

import torch
import torch.distributed as dist

from . import _lib


def shard_range(n_keys: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous key range ``[lo, hi)`` of ``rank`` among ``world`` shards (sizes differ by <= 1)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, extra = divmod(n_keys, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def head_range(rank: int, world: int, n_kv_heads: int = 8) -> tuple[int, int]:
    """KV heads ``(begin, count)`` of ``rank`` when a sequence's ``n_kv_heads``
    heads are sharded over ``world`` ranks (counts differ by <= 1; every rank gets
    at least one, so ``world`` <= ``n_kv_heads``)."""
    if not 1 <= world <= n_kv_heads:
        raise ValueError(f"world must be in [1, {n_kv_heads}] to shard {n_kv_heads} KV heads")
    lo, hi = shard_range(n_kv_heads, rank, world)
    return lo, hi - lo


def balance_sequences(visible_keys, world: int) -> list[list[int]]:
    """Assign sequence indices to ``world`` ranks, longest first to the least-loaded rank."""
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for idx in sorted(range(len(visible_keys)), key=lambda i: (-int(visible_keys[i]), i)):
        load, r = heapq.heappop(heap)
        out[r].append(idx)
        heapq.heappush(heap, (load + int(visible_keys[idx]), r))
    return [sorted(x) for x in out]


def gather_partials(local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather one rank's partial rows ``[B, 32, 132]`` into ``[world, B, 32, 132]``."""
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
    if local.is_cuda:
        dist.all_gather_into_tensor(out.view(world, -1), local.contiguous().view(-1), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), local.contiguous(), group=group)
    return out


class PeerExchange:
    """NVLink peer-memory exchange of FP32 partial rows, fused with the LSE combine.

    Collective over ``group``: every rank constructs it with the same ``batch``
    (sequences whose partials it exchanges), then calls :meth:`combine` in the
    same order.  The ranks' exchange buffers are mapped into each other through
    CUDA IPC handles shared over ``torch.distributed``; no collective library
    runs in :meth:`combine`, which is CUDA-graph capturable.
    """

    def __init__(self, batch: int, group=None, device: torch.device | None = None):
        lib = _lib.load()
        self.lib, self.group, self.batch = lib, group, int(batch)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        nbytes = lib.gqa_peer_buffer_bytes(self.batch)
        if nbytes == 0:
            raise ValueError("batch must be >= 1")
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * _lib.PEER_HANDLE_BYTES)()
        st = lib.gqa_peer_buffer_create(nbytes, ctypes.byref(own), handle)
        if st != _lib.GQA_OK:
            raise RuntimeError(f"gqa_peer_buffer_create: {_lib.status_string(st)}")
        self._own = own.value
        self._opened = []
        try:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            ptrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self._own)
                    continue
                p = ctypes.c_void_p()
                hb = (ctypes.c_ubyte * _lib.PEER_HANDLE_BYTES).from_buffer_copy(h)
                st = lib.gqa_peer_buffer_open(hb, ctypes.byref(p))
                if st != _lib.GQA_OK:
                    raise RuntimeError(f"gqa_peer_buffer_open(rank {r}): {_lib.status_string(st)}")
                self._opened.append(p.value)
                ptrs.append(p.value)
            self.bases = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
            self.status = torch.zeros(64, dtype=torch.int32, device=self.device)
            dist.barrier(group)
        except BaseException:
            # A peer's handle did not open or a collective failed (e.g. a rank is
            # gone): release what this rank holds; nothing has been launched yet.
            for p in self._opened:
                lib.gqa_peer_buffer_close(p)
            self._opened = []
            lib.gqa_peer_buffer_destroy(self._own)
            self._own = None
            raise

    def combine(self, partials: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's partials ``[batch, 32, 132]`` (FP32, CUDA) -> merged BF16 ``[batch, 32, 128]``."""
        from . import api
        if partials.shape != (self.batch, 32, _lib.PARTIAL_FLOATS) or partials.dtype != torch.float32 \
                or partials.stride(-1) != 1 or partials.stride(-2) != _lib.PARTIAL_FLOATS or not partials.is_cuda:
            raise ValueError(f"partials must be CUDA float32 [{self.batch}, 32, {_lib.PARTIAL_FLOATS}] "
                             "with contiguous rows")
        if out is None:
            out = torch.empty((self.batch, 32, 128), dtype=torch.bfloat16, device=partials.device)
        api._check_out(out, (self.batch, 32, 128), torch.bfloat16, partials.device)
        stream = torch.cuda.current_stream(partials.device).cuda_stream
        st = self.lib.gqa_combine_peers(partials.data_ptr(), partials.stride(0), self.bases.data_ptr(), self.world,
                                        self.rank, self.batch, out.data_ptr(), out.stride(0), out.stride(1),
                                        self.status.data_ptr(), stream)
        if st != _lib.GQA_OK:
            raise RuntimeError(f"gqa_combine_peers: {_lib.status_string(st)}")
        return out

    def decode(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, plan, *, layout: str = "position_major",
               scale: float | None = None, rope_theta: float | None = None,
               out: torch.Tensor | None = None, k_rotated: bool = False) -> torch.Tensor:
        """Decode this rank's shard of one sequence and exchange inside the same kernel.

        ``plan``: :func:`attention_accelerator_b200.plan_batch` of one sequence with
        this rank's ``pos_begin``/``pos_end`` (``partial=False``); ``q``: BF16
        ``[1, 32, 128]``; ``k``/``v``: this rank's stored rows.  Returns the merged
        BF16 ``[1, 32, 128]`` rows of the whole sequence, identical on every rank.
        Requires ``batch == 1`` for this exchange.
        """
        from . import api
        if self.batch != 1 or plan.batch != 1 or plan.partial:
            raise ValueError("decode() exchanges one sequence: PeerExchange(1) and a plan of one, partial=False")
        if tuple(q.shape) != (1, 32, 128) or q.dtype != torch.bfloat16 or q.stride(-1) != 1 or not q.is_cuda:
            raise ValueError("q must be a CUDA bfloat16 [1, 32, 128] with a contiguous last dim")
        api._check_cuda(q.device, k=k, v=v, plan=plan.device)
        p = api.make_params(seq_len=1, scale=scale, rope_theta=api.ROPE_THETA if rope_theta is None else rope_theta)
        if k_rotated:  # pre-rotated K cache (api.rope_k_cache)
            p.flags |= _lib.GQA_FLAG_K_ROTATED
        p.k_pos_stride, p.k_head_stride, _ = api._kv_strides(k, layout)
        p.v_pos_stride, p.v_head_stride, _ = api._kv_strides(v, layout)
        if out is None:
            out = torch.empty((1, 32, 128), dtype=torch.bfloat16, device=q.device)
        api._check_out(out, (1, 32, 128), torch.bfloat16, q.device)
        api._set_q_out(p, q, out, False)
        stream = torch.cuda.current_stream(q.device).cuda_stream
        nbytes = self.lib.gqa_workspace_bytes(ctypes.byref(p), plan.host, 1)
        ws = api._workspace(q.device, stream, max(nbytes, 256))
        st = self.lib.gqa_decode_exchange(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), ctypes.byref(p),
                                          plan.host, self.bases.data_ptr(), self.world, self.rank, ws.data_ptr(),
                                          ws.numel(), stream)
        if st != _lib.GQA_OK:
            raise RuntimeError(f"gqa_decode_exchange: {_lib.status_string(st)}")
        return out

    def timed_out(self) -> bool:
        """True if a wait for a peer gave up (synchronises the device)."""
        torch.cuda.synchronize(self.device)
        return bool(self.status[0].item() != 0)

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's after every rank is done."""
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        for p in self._opened:
            self.lib.gqa_peer_buffer_close(p)
        self._opened = []
        dist.barrier(self.group)
        if self._own:
            self.lib.gqa_peer_buffer_destroy(self._own)
            self._own = None
