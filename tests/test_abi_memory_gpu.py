"""GPU tests of the C boundary's memory check (GQA_ERR_MEMORY).

A host pointer or another GPU's allocation handed to a kernel or to a TMA tensor
map would fault the GPU; the library asks the CUDA runtime what each pointer is
and refuses those with GQA_ERR_MEMORY before anything is launched.

Every call here that passes a wrong pointer also passes no workspace: the memory
check runs before the workspace check, so the expected status is
GQA_ERR_MEMORY, and a library whose memory check missed the pointer would
return GQA_ERR_WORKSPACE instead -- nothing is launched either way.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import attention_accelerator_b200 as gqa
from attention_accelerator_b200 import _lib
from attention_accelerator_b200.api import make_params

pytestmark = pytest.mark.gpu

S = 64


def _params() -> _lib.GqaParams:
    p = make_params(seq_len=S)
    p.q_batch_stride, p.q_head_stride = 32 * 128, 128
    p.k_pos_stride, p.k_head_stride = 8 * 128, 128
    p.v_pos_stride, p.v_head_stride = 8 * 128, 128
    p.out_batch_stride, p.out_head_stride = 32 * 128, 128
    return p


def _decode_status(q, k, v, out) -> int:
    p = _params()
    return _lib.load().gqa_decode(q, k, v, out, ctypes.byref(p), None, 0, None)


def test_device_pointers_pass_the_check(cuda_device):
    q = torch.zeros((32, 128), dtype=torch.bfloat16, device=cuda_device)
    kv = torch.zeros((S, 8, 128), dtype=torch.bfloat16, device=cuda_device)
    out = torch.zeros_like(q)
    # valid device memory: the call gets as far as the (missing) workspace
    assert _decode_status(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), out.data_ptr()) == _lib.GQA_ERR_WORKSPACE


@pytest.mark.parametrize("which", ["q", "k", "v", "out"])
@pytest.mark.parametrize("kind", ["pageable", "pinned"])
def test_host_memory_is_refused(which, kind, cuda_device):
    dev = {n: torch.zeros(shape, dtype=torch.bfloat16, device=cuda_device)
           for n, shape in (("q", (32, 128)), ("k", (S, 8, 128)), ("v", (S, 8, 128)), ("out", (32, 128)))}
    host = torch.zeros(dev[which].shape, dtype=torch.bfloat16)
    if kind == "pinned":
        host = host.pin_memory()
    assert host.data_ptr() % 16 == 0
    ptrs = {n: t.data_ptr() for n, t in dev.items()}
    ptrs[which] = host.data_ptr()
    st = _decode_status(ptrs["q"], ptrs["k"], ptrs["v"], ptrs["out"])
    assert st == _lib.GQA_ERR_MEMORY, _lib.status_string(st)
    assert "memory of the current GPU" in _lib.status_string(st)


def test_host_memory_refused_by_the_chunked_path(cuda_device):
    p = _params()
    c = _lib.GqaChunkParams(batch=1, n_queries=1, first_position=S - 1, q_query_stride=4096, out_query_stride=4096,
                            k_batch_stride=S * 1024, v_batch_stride=S * 1024)
    host_q = np.zeros(32 * 128 + 8, dtype=np.uint16)
    qptr = host_q.ctypes.data + (-host_q.ctypes.data % 16)  # 16-byte aligned pageable host memory
    kv = torch.zeros((S, 8, 128), dtype=torch.bfloat16, device=cuda_device)
    out = torch.zeros((32, 128), dtype=torch.bfloat16, device=cuda_device)
    st = _lib.load().gqa_decode_chunked(qptr, kv.data_ptr(), kv.data_ptr(), out.data_ptr(), ctypes.byref(p),
                                        ctypes.byref(c), None, 0, None)
    assert st == _lib.GQA_ERR_MEMORY


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_another_gpus_memory_is_refused():
    torch.cuda.set_device(0)
    q = torch.zeros((32, 128), dtype=torch.bfloat16, device="cuda:0")
    kv = torch.zeros((S, 8, 128), dtype=torch.bfloat16, device="cuda:0")
    other = torch.zeros((S, 8, 128), dtype=torch.bfloat16, device="cuda:1")
    out = torch.zeros_like(q)
    assert _decode_status(q.data_ptr(), other.data_ptr(), kv.data_ptr(), out.data_ptr()) == _lib.GQA_ERR_MEMORY


def test_api_checks_outputs_and_devices(cuda_device):
    """The Python layer refuses, before calling the library, an ``out`` too small for
    the rows the kernel writes and K/V on another device than Q."""
    q = torch.zeros((32, 128), dtype=torch.bfloat16, device=cuda_device)
    kv = torch.zeros((S, 8, 128), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError, match="out must be"):
        gqa.decode(q, kv, kv, out=torch.empty((16, 128), dtype=torch.bfloat16, device=cuda_device))
    with pytest.raises(ValueError, match="every tensor"):
        gqa.decode(q, kv.cpu(), kv.cpu())
    plan = gqa.plan_batch([S], device=cuda_device)
    with pytest.raises(ValueError, match="out must be"):
        gqa.decode_batch(q[None], kv, kv, plan, out=torch.empty((1, 32, 64), dtype=torch.bfloat16, device=cuda_device))
    qc = torch.zeros((1, 2, 32, 128), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError, match="out must be"):
        gqa.decode_chunked(qc, kv[None], kv[None], first_position=S - 2,
                           out=torch.empty((1, 1, 32, 128), dtype=torch.bfloat16, device=cuda_device))
    x = torch.zeros((4, 8, 128), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError, match="out must match"):
        gqa.rope_rtl(x, torch.arange(4), out=torch.empty((2, 8, 128), dtype=torch.bfloat16, device=cuda_device))
    # the valid calls still run
    assert gqa.decode(q, kv, kv).shape == (32, 128)
    torch.cuda.synchronize()
