"""gqa_decode_noalloc: the decode for callers that may not allocate device memory.

Such callers (a plug-in inside a host program that owns every device
allocation, or a loop that cannot afford cudaMalloc's implicit synchronisation)
pass only inputs and outputs; the scratch lives in a fixed library-owned
device array.  This file is named to be collected last, so that a run stopping
at its first failure has already run every other test; it also passes on its
own in a fresh process (the entry point does its own one-time set-up per
device).

What the scratch array holds on this path: a single sequence of more than one
split writes its FP32 split partials there, and the last split CTA of each KV
head to finish -- elected through a per-head arrival counter in the array's
header -- merges them.  The counters are the one piece of state that must
start at zero; each call's last split sets its head's counter back to zero.
Calls with different split counts in a row (one split, a cluster merge that
keeps its partials on chip, and last-split merges of 17 and 18 splits) must
therefore repeat bit for bit and match the workspace entry point.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import attention_accelerator_b200 as gqa
from attention_accelerator_b200 import _lib
from attention_accelerator_b200.api import make_params
from conftest import assert_parity, torch_to_bits
from oracle.golden import gqa_golden

pytestmark = pytest.mark.gpu

NOALLOC_SCRATCH_BYTES = 1 << 20  # GQA_NOALLOC_SCRATCH_BYTES in include/gqa_b200.h


def _inputs(seq_len: int, seed: int, device):
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn((32, 128), generator=g, device=device).to(torch.bfloat16)
    k = torch.randn((seq_len, 8, 128), generator=g, device=device).to(torch.bfloat16)
    v = torch.randn((seq_len, 8, 128), generator=g, device=device).to(torch.bfloat16)
    return q, k, v


def _noalloc(q, k, v, seq_len: int, out: torch.Tensor) -> int:
    p = make_params(seq_len=seq_len)
    p.q_batch_stride, p.q_head_stride = 32 * 128, q.stride(0)
    p.k_pos_stride, p.k_head_stride = k.stride(0), k.stride(1)
    p.v_pos_stride, p.v_head_stride = v.stride(0), v.stride(1)
    p.out_batch_stride, p.out_head_stride = 32 * 128, out.stride(0)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    return _lib.load().gqa_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                          ctypes.byref(p), stream)


def _oracle(q, k, v, seq_len: int):
    """BF16 codes of the float64 golden of the same inputs (head-major codes for the oracle)."""
    kh, vh = torch_to_bits(k.transpose(0, 1)), torch_to_bits(v.transpose(0, 1))
    return gqa_golden(torch_to_bits(q), kh, vh, seq_len, seq_len - 1, exact=False)


# 30 keys: one split, written directly (no partials); 4096 keys: 17 splits whose
# partials sit in the static scratch, merged by the last split of each KV head.
@pytest.mark.parametrize("seq_len", [30, 4096])
def test_noalloc_matches_workspace_entry_point_and_oracle(seq_len, cuda_device):
    for call in range(2):  # consecutive calls share (and overwrite) the one scratch array
        q, k, v = _inputs(seq_len, seed=1000 * seq_len + call, device=cuda_device)
        want = gqa.decode(q, k, v, seq_len=seq_len)
        got = torch.full_like(want, float("nan"))
        assert _noalloc(q, k, v, seq_len, got) == _lib.GQA_OK
        torch.cuda.synchronize()
        # same kernels and split plan as the workspace entry point: the same bits
        np.testing.assert_array_equal(torch_to_bits(got), torch_to_bits(want))
        # and the reference's rule (64 ULP) plus this build's FP32 bar against the float64 golden
        assert_parity(_oracle(q, k, v, seq_len), torch_to_bits(got))


def test_noalloc_interleaved_split_counts(cuda_device):
    """Calls of 1 split, a cluster merge, and last-split merges of 17 and 18
    splits, interleaved twice on one stream: every call repeats bit for bit and
    equals gqa_decode, so each last-split merge found its head's arrival
    counter at zero."""
    lens = [4096, 30, 600, 131072, 2000, 4096]
    splits = {s: gqa.decode_plan(s) for s in set(lens)}
    assert splits[30].splits == 1
    assert splits[4096].cluster == 0 and splits[4096].splits > 1
    assert splits[131072].cluster == 0 and splits[131072].splits > splits[4096].splits
    inputs = {s: _inputs(s, seed=77 + s, device=cuda_device) for s in set(lens)}
    want = {s: torch_to_bits(gqa.decode(*inputs[s], seq_len=s)) for s in set(lens)}
    for _ in range(2):
        for s in lens:
            out = torch.full((32, 128), float("nan"), dtype=torch.bfloat16, device=cuda_device)
            assert _noalloc(*inputs[s], s, out) == _lib.GQA_OK
            np.testing.assert_array_equal(torch_to_bits(out), want[s])
    assert gqa.read_device_status(cuda_device) == 0


def test_noalloc_scratch_limit_covers_every_single_sequence(cuda_device):
    """A single sequence is cut into at most one wave of splits and at most 32,
    so its scratch is bounded by the SM count, not by SEQ_LEN: even the longest
    sequence fits the fixed array and the GQA_ERR_WORKSPACE refusal is a guard
    that valid calls do not reach."""
    lib = _lib.load()
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    for s in (30, 4096, 131072, 1 << 24):
        p = make_params(seq_len=s)
        need = lib.gqa_workspace_bytes(ctypes.byref(p), None, 1)
        assert 0 < need <= 512 + min(sms // 8, 32) * 16896 <= NOALLOC_SCRATCH_BYTES


def test_noalloc_rejects_bad_configuration_before_launch(cuda_device):
    q, k, v = _inputs(32, seed=7, device=cuda_device)
    out = torch.zeros((32, 128), dtype=torch.bfloat16, device=cuda_device)
    p = make_params(seq_len=32, n_q_heads=31)
    status = _lib.load().gqa_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                            ctypes.byref(p), None)
    assert status == _lib.GQA_ERR_GEOMETRY
    torch.cuda.synchronize()
    assert not torch.any(out.view(torch.int16) != 0)
