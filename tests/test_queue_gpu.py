"""The batched decode's work queue (decode_queue_kernel).

A batch runs one CTA per SM; each CTA takes (split, KV head) items in plan
order from a counter pair in the workspace header, and the last CTA to leave
clears the pair for the next call.  These tests check that a batch's outputs
do not depend on which CTA took which item (repeated calls agree bit for bit
and match the float64 oracle), that the counters are back at zero after every
call, and that an item without keys (a shard past its query position) still
yields an empty partial.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import attention_accelerator_b200 as gqa
from attention_accelerator_b200 import api
from conftest import assert_parity, bits_to_torch, torch_to_bits
from oracle.golden import gqa_golden
from test_decode_gpu import normal_inputs

pytestmark = pytest.mark.gpu

QUEUE_OFFSET = 128  # bytes: the work-queue counters (next item, CTAs done) in the workspace header


def _packed(seqs, seed):
    parts = [normal_inputs(s, seed=seed + i) for i, s in enumerate(seqs)]
    qs = np.stack([p[0] for p in parts])
    k = np.concatenate([p[1].transpose(1, 0, 2) for p in parts])
    v = np.concatenate([p[2].transpose(1, 0, 2) for p in parts])
    return parts, qs, k, v


def _queue_words(device):
    ws = api._workspace(device, torch.cuda.current_stream(device).cuda_stream, 4096)
    return ws[QUEUE_OFFSET:QUEUE_OFFSET + 8].view(torch.int32).cpu().tolist()


# 40 sequences: more (split, KV head) items than SMs; 2 short ones: fewer.
@pytest.mark.parametrize("seqs", [
    [1 + (977 * i) % 6000 for i in range(40)],
    [5, 70],
], ids=["items_above_sms", "items_below_sms"])
def test_queue_batches_repeat_bit_for_bit_and_clear_the_queue(seqs, cuda_device):
    parts, qs, k, v = _packed(seqs, seed=500 + len(seqs))
    qpos = [s - 1 for s in seqs]
    plan = gqa.plan_batch(seqs, query_positions=qpos, device=cuda_device)
    q_t, k_t, v_t = (bits_to_torch(x, cuda_device) for x in (qs, k, v))
    outs = []
    for _ in range(3):
        outs.append(torch_to_bits(gqa.decode_batch(q_t, k_t, v_t, plan)))
        torch.cuda.synchronize()
        assert _queue_words(cuda_device) == [0, 0]
    for o in outs[1:]:
        np.testing.assert_array_equal(o, outs[0])
    for i, s in enumerate(seqs):
        if s <= 1024 or i % 8 == 0:
            golden = gqa_golden(parts[i][0], parts[i][1], parts[i][2], s, qpos[i], exact=s <= 1024)
            assert_parity(golden, outs[0][i])
    assert gqa.read_device_status(cuda_device) == 0


def test_queue_partial_batch_with_an_empty_shard(cuda_device):
    """Shards of three sequences; the middle one lies past its query position."""
    seqs = [900, 300, 2000]
    qpos = [899, 99, 1999]
    begin, end = [0, 200, 500], [900, 300, 2000]
    parts = [normal_inputs(s, seed=700 + i) for i, s in enumerate(seqs)]
    qs = np.stack([p[0] for p in parts])
    k = np.concatenate([p[1][:, lo:hi].transpose(1, 0, 2) for p, lo, hi in zip(parts, begin, end)])
    v = np.concatenate([p[2][:, lo:hi].transpose(1, 0, 2) for p, lo, hi in zip(parts, begin, end)])
    # kv_starts[b]: the stored row of sequence b's first key in [begin, end)
    starts = np.concatenate([[0], np.cumsum([hi - lo for lo, hi in zip(begin, end)])[:-1]]).astype(int).tolist()
    plan = gqa.plan_batch(seqs, query_positions=qpos, pos_begin=begin, pos_end=end,
                          kv_starts=starts, partial=True, device=cuda_device)
    part = gqa.decode_batch(bits_to_torch(qs, cuda_device), bits_to_torch(k, cuda_device),
                            bits_to_torch(v, cuda_device), plan)
    torch.cuda.synchronize()
    assert _queue_words(cuda_device) == [0, 0]
    p = part.cpu()
    assert torch.isinf(p[1, :, 128]).all() and (p[1, :, 128] < 0).all()
    assert (p[1, :, 129] == 0).all() and (p[1, :, :128] == 0).all()
    # The other two shards cover their sequences' visible keys [begin, end):
    # their combined rows are the oracle's attention over those keys.
    for i in (0, 2):
        got = torch_to_bits(gqa.combine_partials(part[i:i + 1].unsqueeze(0)))[0]
        lo, hi = begin[i], end[i]
        golden = gqa_golden(parts[i][0], parts[i][1][:, lo:hi], parts[i][2][:, lo:hi], hi - lo, qpos[i] - lo,
                            exact=False)
        assert_parity(golden, got)
