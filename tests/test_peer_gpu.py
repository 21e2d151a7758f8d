"""GPU tests of the NVLink peer-memory exchange of the long-context split:
gqa_combine_peers (exchange fused with the LSE combine) and gqa_decode_exchange
(exchange fused into the decode kernel).

On one GPU a second rank is emulated without any kernel waiting for a later
kernel.  gqa_combine_peers pulls rows from the peers' buffers, so a world-size-1
call on rank 1's buffer publishes its rows before rank 0's world-size-2 call.
gqa_decode_exchange pushes rows into every rank's buffer, so rank 1's call runs
first: it pushes its rows into rank 0's buffer, and its own wait for rank 0
gives up after ~1 s and reports it.  Rank 0's call then finds the rows.  The
timeout tests leave a peer's flag (combine) or words (decode exchange, whose
pushed values carry their epoch) unwritten and check that the bounded wait
gives up and reports it.  The two-process test (2 GPUs) runs the real IPC-mapped
exchange with torch.distributed ranks.
"""
from __future__ import annotations

import ctypes
import os
import socket

import numpy as np
import pytest
import torch

import attention_accelerator_b200 as gqa
from attention_accelerator_b200 import _lib
from conftest import bits_to_torch, torch_to_bits
from oracle import check_rows, gqa_golden

pytestmark = pytest.mark.gpu


def _inputs(seq_len: int, seed: int):
    g = torch.Generator().manual_seed(seed)

    def bits(shape):
        return torch_to_bits(torch.randn(shape, generator=g).to(torch.bfloat16))
    return bits((32, 128)), bits((8, seq_len, 128)), bits((8, seq_len, 128))


def _shard_partial(q, k, v, s, lo, hi, device):
    plan = gqa.plan_batch([s], pos_begin=[lo], pos_end=[hi], kv_starts=[0], partial=True, device=device)
    return gqa.decode_batch(bits_to_torch(q[None], device), bits_to_torch(k[:, lo:hi].transpose(1, 0, 2).copy(), device),
                            bits_to_torch(v[:, lo:hi].transpose(1, 0, 2).copy(), device), plan)


class _Buffer:
    def __init__(self, batch):
        self.lib = _lib.load()
        p = ctypes.c_void_p()
        h = (ctypes.c_ubyte * _lib.PEER_HANDLE_BYTES)()
        assert self.lib.gqa_peer_buffer_create(self.lib.gqa_peer_buffer_bytes(batch), ctypes.byref(p), h) == 0
        self.ptr = p.value

    def free(self):
        self.lib.gqa_peer_buffer_destroy(self.ptr)


def _combine(parts, bases, world, rank, device, status):
    lib = _lib.load()
    out = torch.empty((parts.shape[0], 32, 128), dtype=torch.bfloat16, device=device)
    b = torch.tensor(bases, dtype=torch.int64, device=device)
    st = lib.gqa_combine_peers(parts.data_ptr(), parts.stride(0), b.data_ptr(), world, rank, parts.shape[0],
                               out.data_ptr(), out.stride(0), out.stride(1), status.data_ptr(), None)
    assert st == _lib.GQA_OK
    return out


def test_combine_peers_matches_combine_partials_over_epochs(cuda_device):
    s = 3000
    a, b = _Buffer(1), _Buffer(1)
    status = torch.zeros(64, dtype=torch.int32, device=cuda_device)
    try:
        for epoch in range(3):  # both parities, then reuse of the first
            q, k, v = _inputs(s, seed=40 + epoch)
            p0 = _shard_partial(q, k, v, s, 0, 1400, cuda_device)
            p1 = _shard_partial(q, k, v, s, 1400, s, cuda_device)
            _combine(p1, [b.ptr], 1, 0, cuda_device, status)            # "rank 1" publishes
            got = _combine(p0, [a.ptr, b.ptr], 2, 0, cuda_device, status)  # rank 0 exchanges + merges
            want = gqa.combine_partials(torch.stack([p0, p1]))
            torch.cuda.synchronize()
            assert int(status[0]) == 0
            np.testing.assert_array_equal(torch_to_bits(got), torch_to_bits(want))
            res = check_rows(gqa_golden(q, k, v, s, s - 1, exact=False), torch_to_bits(got)[0], 64)
            assert res.passed and res.worst_ulp <= 2, res.line()
    finally:
        a.free()
        b.free()


def test_combine_peers_wait_times_out_and_reports(cuda_device):
    """A peer that never publishes: the bounded wait (~1 s) gives up and sets the status word."""
    a, b = _Buffer(1), _Buffer(1)
    status = torch.zeros(64, dtype=torch.int32, device=cuda_device)
    try:
        q, k, v = _inputs(256, seed=3)
        p0 = _shard_partial(q, k, v, 256, 0, 256, cuda_device)
        _combine(p0, [a.ptr, b.ptr], 2, 0, cuda_device, status)
        torch.cuda.synchronize()
        assert int(status[0]) == 1  # kDevStatusTimeout
    finally:
        a.free()
        b.free()


def _exchange_decode(q, k, v, s, lo, hi, bases, world, rank, device):
    """gqa_decode_exchange of shard [lo, hi) on this device; returns (out bits, status word)."""
    from attention_accelerator_b200.distributed import PeerExchange
    ex = PeerExchange.__new__(PeerExchange)  # the method only needs these fields
    ex.lib, ex.batch, ex.world, ex.rank = _lib.load(), 1, world, rank
    ex.bases = torch.tensor(bases, dtype=torch.int64, device=device)
    plan = gqa.plan_batch([s], pos_begin=[lo], pos_end=[hi], kv_starts=[0], device=device)
    out = ex.decode(bits_to_torch(q[None], device), bits_to_torch(k[:, lo:hi].transpose(1, 0, 2).copy(), device),
                    bits_to_torch(v[:, lo:hi].transpose(1, 0, 2).copy(), device), plan)
    from attention_accelerator_b200 import api
    torch.cuda.synchronize()
    ws = api._workspace(device, api._stream_ptr(device), 256)
    status = int(ws[:4].view(torch.int32)[0])
    ws[:4].zero_()
    return torch_to_bits(out), status


def test_decode_exchange_matches_combine_partials(cuda_device):
    """Rank 1's decode pushes its rows into rank 0's buffer first (its own wait for rank 0,
    which has not run yet, gives up after ~1 s and reports it); rank 0's decode kernel then
    finds them, merges and writes the whole sequence's rows."""
    s = 6000
    a, b = _Buffer(1), _Buffer(1)
    try:
        for epoch in range(3):
            q, k, v = _inputs(s, seed=60 + epoch)
            p0 = _shard_partial(q, k, v, s, 0, 2500, cuda_device)
            p1 = _shard_partial(q, k, v, s, 2500, s, cuda_device)
            _, st1 = _exchange_decode(q, k, v, s, 2500, s, [a.ptr, b.ptr], 2, 1, cuda_device)
            assert st1 == 1  # rank 1 waited for rank 0 in vain
            got, st = _exchange_decode(q, k, v, s, 0, 2500, [a.ptr, b.ptr], 2, 0, cuda_device)
            assert st == 0
            want = torch_to_bits(gqa.combine_partials(torch.stack([p0, p1])))[0]
            assert check_rows(want, got[0], 2).passed
            res = check_rows(gqa_golden(q, k, v, s, s - 1, exact=False), got[0], 64)
            assert res.passed and res.worst_ulp <= 2, res.line()
    finally:
        a.free()
        b.free()


def test_decode_exchange_wait_times_out_and_reports(cuda_device):
    a, b = _Buffer(1), _Buffer(1)
    try:
        q, k, v = _inputs(1000, seed=8)
        _, st = _exchange_decode(q, k, v, 1000, 0, 500, [a.ptr, b.ptr], 2, 0, cuda_device)
        assert st == 1  # kDevStatusTimeout: the peer never published
    finally:
        a.free()
        b.free()


def _free_port() -> int:
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _two_rank_worker(rank: int, port: int, result_q):
    import torch.distributed as dist
    from attention_accelerator_b200.distributed import PeerExchange, shard_range
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev)
    try:
        s = 5000
        q, k, v = _inputs(s, seed=77)
        lo, hi = shard_range(s, rank, 2)
        ex = PeerExchange(1, device=dev)
        outs = []
        plan = gqa.plan_batch([s], pos_begin=[lo], pos_end=[hi], kv_starts=[0], device=dev)
        kd = bits_to_torch(k[:, lo:hi].transpose(1, 0, 2).copy(), dev)
        vd = bits_to_torch(v[:, lo:hi].transpose(1, 0, 2).copy(), dev)
        for _ in range(3):  # separate combine kernel, then the exchange inside the decode kernel
            part = _shard_partial(q, k, v, s, lo, hi, dev)
            outs.append(torch_to_bits(ex.combine(part)))
            outs.append(torch_to_bits(ex.decode(bits_to_torch(q[None], dev), kd, vd, plan)))
        timed_out = ex.timed_out()
        ex.close()
        result_q.put((rank, outs, timed_out))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_exchange_two_processes():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, port, result_q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (o, t)) for r, o, t in (result_q.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    q, k, v = _inputs(5000, seed=77)
    golden = gqa_golden(q, k, v, 5000, 4999, exact=False)
    for r in range(2):
        outs, timed_out = results[r]
        assert not timed_out
        for o in outs:
            res = check_rows(golden, o[0], 64)
            assert res.passed and res.worst_ulp <= 2, res.line()
        assert all(np.array_equal(outs[0], o) for o in outs[0::2])  # combine path, every epoch
        assert all(np.array_equal(outs[1], o) for o in outs[1::2])  # fused path, every epoch
    np.testing.assert_array_equal(results[0][0][0], results[1][0][0])
