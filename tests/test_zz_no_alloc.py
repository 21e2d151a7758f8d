"""gqa_decode_noalloc: the decode for callers that may not allocate device memory.

Such callers (a plug-in inside a host program that owns every device
allocation, or a loop that cannot afford cudaMalloc's implicit synchronisation)
pass only inputs and outputs; the scratch lives in a fixed library-owned device
array.  This file is named to be collected last, so that a run stopping at its
first failure has already run every other test; it also passes on its own in a
fresh process (the entry point does its own one-time set-up per device).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import attention_accelerator_b200 as gqa
from attention_accelerator_b200 import _lib
from attention_accelerator_b200.api import make_params
from conftest import torch_to_bits
from oracle import check_rows

pytestmark = pytest.mark.gpu

MAX_ULP = 64
TIGHT_ULP = 2


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


# 30 keys: one split (no partials); 4096 keys: many splits, partials and split
# table in the static scratch, merged by the split-merge kernel.
@pytest.mark.parametrize("seq_len", [30, 4096])
def test_noalloc_matches_workspace_entry_point(seq_len, cuda_device):
    for call in range(2):  # consecutive calls share (and overwrite) the one scratch array
        q, k, v = _inputs(seq_len, seed=1000 * seq_len + call, device=cuda_device)
        want = gqa.decode(q, k, v, seq_len=seq_len)
        got = torch.full_like(want, float("nan"))
        assert _noalloc(q, k, v, seq_len, got) == _lib.GQA_OK
        torch.cuda.synchronize()
        res = check_rows(torch_to_bits(want), torch_to_bits(got), MAX_ULP)
        assert res.passed and res.worst_ulp <= TIGHT_ULP, res.line()  # same kernels: agree to rounding


def test_noalloc_rejects_bad_configuration_before_launch(cuda_device):
    q, k, v = _inputs(32, seed=7, device=cuda_device)
    out = torch.zeros((32, 128), dtype=torch.bfloat16, device=cuda_device)
    p = make_params(seq_len=32, n_q_heads=31)
    status = _lib.load().gqa_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                            ctypes.byref(p), None)
    assert status == _lib.GQA_ERR_GEOMETRY
    assert not torch.any(out.view(torch.int16) != 0)
