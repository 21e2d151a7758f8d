"""GPU parity of the KV-head-sharded decode (``decode_heads`` / ``gqa_decode_heads``).

A KV head and its 4 Q heads depend on no other head (gqa_controller.v:159-162),
so a sequence's heads can be decoded on different GPUs from K/V tensors that
hold only those heads.  Each range's rows must meet the reference's rule against
the float64 oracle, agree with the whole-sequence decode within the FP32 bar,
and leave the other output rows untouched; ranges that partition the 8 heads
assemble the whole output.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import attention_accelerator_b200 as gqa
from attention_accelerator_b200.distributed import head_range
from conftest import assert_parity, bits_to_torch, torch_to_bits
from oracle import check_rows, gqa_golden

pytestmark = pytest.mark.gpu


def _inputs(seq_len: int, seed: int):
    g = torch.Generator().manual_seed(seed)

    def bits(shape):
        return torch_to_bits(torch.randn(shape, generator=g).to(torch.bfloat16))
    return bits((32, 128)), bits((8, seq_len, 128)), bits((8, seq_len, 128))


@pytest.mark.parametrize("seq_len", [30, 4096, 20000])
@pytest.mark.parametrize("begin,count", [(0, 8), (0, 1), (3, 2), (6, 2), (7, 1), (2, 4)])
def test_head_range_matches_oracle_and_whole_decode(seq_len, begin, count, cuda_device):
    q, k, v = _inputs(seq_len, seed=seq_len + 10 * begin + count)
    qd = bits_to_torch(q, cuda_device)
    kpos = k.transpose(1, 0, 2)  # position-major [S, 8, 128]
    vpos = v.transpose(1, 0, 2)
    kd = bits_to_torch(np.ascontiguousarray(kpos[:, begin:begin + count]), cuda_device)
    vd = bits_to_torch(np.ascontiguousarray(vpos[:, begin:begin + count]), cuda_device)
    sentinel = torch.full((32, 128), 7.0, dtype=torch.bfloat16, device=cuda_device)
    got = torch_to_bits(gqa.decode_heads(qd, kd, vd, kv_heads=(begin, count), out=sentinel))
    torch.cuda.synchronize()
    assert gqa.read_device_status(cuda_device) == 0
    rows = slice(4 * begin, 4 * (begin + count))
    others = np.ones(32, dtype=bool)
    others[rows] = False
    assert (got[others] == torch_to_bits(torch.tensor(7.0, dtype=torch.bfloat16))).all()
    golden = gqa_golden(q, k, v, seq_len, seq_len - 1, exact=seq_len <= 4096)
    assert_parity(golden[rows], got[rows])
    whole = torch_to_bits(gqa.decode(qd, bits_to_torch(kpos.copy(), cuda_device),
                                     bits_to_torch(vpos.copy(), cuda_device)))
    assert check_rows(whole[rows], got[rows], 64).passed


def test_head_partitions_assemble_the_whole_output(cuda_device):
    """The ranges of 2, 4 and 8 ranks (distributed.head_range) decoded one after
    another into one output: every row written once, equal to the whole decode
    within the FP32 bar, and each repeated call is bit-identical."""
    s = 4096
    q, k, v = _inputs(s, seed=99)
    qd = bits_to_torch(q, cuda_device)
    kpos, vpos = k.transpose(1, 0, 2), v.transpose(1, 0, 2)
    whole = torch_to_bits(gqa.decode(qd, bits_to_torch(kpos.copy(), cuda_device), bits_to_torch(vpos.copy(), cuda_device)))
    golden = gqa_golden(q, k, v, s, s - 1, exact=True)
    for world in (2, 4, 8):
        out = torch.zeros((32, 128), dtype=torch.bfloat16, device=cuda_device)
        for r in range(world):
            b, c = head_range(r, world)
            kd = bits_to_torch(np.ascontiguousarray(kpos[:, b:b + c]), cuda_device)
            vd = bits_to_torch(np.ascontiguousarray(vpos[:, b:b + c]), cuda_device)
            gqa.decode_heads(qd, kd, vd, kv_heads=(b, c), out=out)
            again = torch_to_bits(gqa.decode_heads(qd, kd, vd, kv_heads=(b, c)))
            np.testing.assert_array_equal(again[4 * b:4 * (b + c)], torch_to_bits(out)[4 * b:4 * (b + c)])
        got = torch_to_bits(out)
        assert_parity(golden, got)
        assert check_rows(whole, got, 2).passed


def test_head_range_refused(cuda_device):
    q, k, v = _inputs(64, seed=1)
    qd = bits_to_torch(q, cuda_device)
    kd = bits_to_torch(np.ascontiguousarray(k.transpose(1, 0, 2)[:, :2]), cuda_device)
    with pytest.raises(gqa.GqaError):
        gqa.decode_heads(qd, kd, kd, kv_heads=(7, 2))
