"""Multi-rank host logic on CPU: world-size-2 ``gloo`` process groups.

The GPU kernels are replaced here by the oracle's float64 partials (this is a
test of the decomposition and the collective plumbing, not of the kernels,
which tests/test_decode_gpu.py covers): each rank computes the partial of its
contiguous key shard, ``gather_partials`` all-gathers them over gloo, and the
log-sum-exp merge must reproduce the single-process golden.  Sequence
sharding is checked for coverage and balance.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from attention_accelerator_b200.distributed import balance_sequences, gather_partials, head_range, shard_range


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(seq_len: int, seed: int):
    g = torch.Generator().manual_seed(seed)

    def bits(t):
        return t.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)
    return (bits(torch.randn(32, 128, generator=g)), bits(torch.randn(8, seq_len, 128, generator=g)),
            bits(torch.randn(8, seq_len, 128, generator=g)))


def _worker(rank: int, world: int, port: int, seq_len: int, qpos: int, result_q):
    from oracle.partials import combine_f64, from_rows, partial_f64, to_rows
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v = _inputs(seq_len, seed=7)
        lo, hi = shard_range(seq_len, rank, world)
        local = torch.from_numpy(to_rows(*partial_f64(q, k, v, qpos, lo, hi)).astype(np.float32))[None]
        gathered = gather_partials(local)  # [world, 1, 32, 132]
        parts = [from_rows(gathered[r, 0].numpy()) for r in range(world)]
        result_q.put((rank, combine_f64(parts)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("seq_len,qpos", [(300, 299), (300, 120)])
def test_sequence_split_over_gloo_matches_single_process(seq_len, qpos):
    from oracle import check_rows, gqa_golden
    world = 2
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, seq_len, qpos, result_q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(result_q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, k, v = _inputs(seq_len, seed=7)
    golden = gqa_golden(q, k, v, seq_len, qpos, exact=False)
    for r in range(world):
        res = check_rows(golden, results[r], 64)
        assert res.passed and res.worst_ulp <= 1, res.line()
    np.testing.assert_array_equal(results[0], results[1])


def _head_worker(rank: int, world: int, port: int, seq_len: int, result_q):
    """One rank of a KV-head-sharded decode: the golden of its heads only (K/V of
    those heads, their Q rows), then an all-gather of the output rows."""
    from oracle.golden import gqa_golden_f64
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v = _inputs(seq_len, seed=11)
        begin, count = head_range(rank, world)
        mine = gqa_golden_f64(q[4 * begin:4 * (begin + count)], k[begin:begin + count], v[begin:begin + count],
                              seq_len, seq_len - 1, exact=False)
        rows = torch.zeros((32, 128), dtype=torch.float64)
        rows[4 * begin:4 * (begin + count)] = torch.from_numpy(mine)
        gathered = [torch.zeros_like(rows) for _ in range(world)]
        dist.all_gather(gathered, rows)
        result_q.put((rank, sum(gathered).numpy()))  # disjoint rows: the sum assembles them
    finally:
        dist.destroy_process_group()


def test_head_sharding_over_gloo_matches_single_process():
    """KV heads split over 2 ranks with no exchange of partial results: the
    assembled rows equal the single-process golden bit for bit."""
    from oracle.golden import gqa_golden_f64
    world, seq_len = 2, 200
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_head_worker, args=(r, world, port, seq_len, result_q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(result_q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, k, v = _inputs(seq_len, seed=11)
    golden = gqa_golden_f64(q, k, v, seq_len, seq_len - 1, exact=False)
    for r in range(world):
        np.testing.assert_array_equal(results[r], golden)


def test_head_ranges_partition_the_kv_heads():
    for world in range(1, 9):
        ranges = [head_range(r, world) for r in range(world)]
        heads = [h for b, c in ranges for h in range(b, b + c)]
        assert heads == list(range(8))
        assert min(c for _, c in ranges) >= 1 and max(c for _, c in ranges) - min(c for _, c in ranges) <= 1
    for bad in (0, 9):
        with pytest.raises(ValueError):
            head_range(0, bad)


def test_shard_ranges_cover_exactly():
    for n in (1, 7, 131072, 131071):
        for world in (1, 2, 4, 8):
            ranges = [shard_range(n, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [hi - lo for lo, hi in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_balance_sequences_covers_and_balances():
    rng = np.random.default_rng(0)
    lens = rng.integers(512, 8193, size=64).tolist()
    for world in (1, 2, 4, 8):
        parts = balance_sequences(lens, world)
        assert sorted(i for p in parts for i in p) == list(range(64))
        loads = [sum(lens[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(lens)
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


class _FakePeerLib:
    """Stands in for the library's CUDA IPC buffer calls on CPU: it records what
    PeerExchange creates, opens, closes and destroys; on ``fail_rank`` opening a
    peer's handle fails, as it would for a peer whose process has gone."""

    def __init__(self, rank: int, fail_rank: int):
        self.rank, self.fail_rank, self.log = rank, fail_rank, []

    def gqa_peer_buffer_bytes(self, batch):
        return 4096

    def gqa_peer_buffer_create(self, nbytes, ptr_ref, handle):
        ptr_ref._obj.value = 0x10000 * (self.rank + 1)
        handle[0] = self.rank
        self.log.append(("create", ptr_ref._obj.value))
        return 0

    def gqa_peer_buffer_open(self, handle, ptr_ref):
        if self.rank == self.fail_rank:
            return 13  # GQA_ERR_CUDA
        ptr_ref._obj.value = 0x10000 * (handle[0] + 1) + 0x100
        self.log.append(("open", ptr_ref._obj.value))
        return 0

    def gqa_peer_buffer_close(self, ptr):
        self.log.append(("close", ptr))

    def gqa_peer_buffer_destroy(self, ptr):
        self.log.append(("destroy", ptr))

    def gqa_status_string(self, code):
        return b"CUDA runtime error"


def _peer_failure_worker(rank: int, port: int, result_q):
    from datetime import timedelta

    from attention_accelerator_b200 import _lib, distributed
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=5))
    fake = _FakePeerLib(rank, fail_rank=1)
    _lib.load = lambda: fake
    try:
        distributed.PeerExchange(1, device=torch.device("cpu"))
        result_q.put((rank, "constructed", fake.log))
    except Exception as e:  # rank 1: its open failed; rank 0: its barrier timed out
        result_q.put((rank, type(e).__name__, fake.log))
    finally:
        dist.destroy_process_group()


def test_peer_exchange_releases_its_buffers_when_set_up_fails():
    """Rank 1 cannot open rank 0's handle and raises; rank 0 opened rank 1's and
    then waits at the set-up barrier until the process group's timeout.  Both
    ranks must unmap what they opened and free their own buffer."""
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_failure_worker, args=(r, port, result_q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (what, log)) for r, what, log in (result_q.get(timeout=120) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
    assert results[1][0] == "RuntimeError"
    assert results[1][1] == [("create", 0x20000), ("destroy", 0x20000)]
    assert results[0][0] != "constructed"
    assert results[0][1] == [("create", 0x10000), ("open", 0x20100), ("close", 0x20100), ("destroy", 0x10000)]
