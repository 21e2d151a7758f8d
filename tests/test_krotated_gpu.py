"""GPU tests of the pre-rotated K-cache mode (GQA_FLAG_K_ROTATED, gqa_rope_k_cache).

In the reference every call rotates every K row at its position
(gen_gqa_wrapper_vectors.py:122-124, rope_unit.v).  A production KV cache
stores K already rotated: gqa_rope_k_cache rotates rows when they are appended
and the decode kernel then rotates only Q.  Checked here:
  * the append-time rotation against the oracle's float64 rope_half_split,
    rounded to BF16 as the reference rounds (f32_to_bf16);
  * decode of the rotated cache against the oracle with the same (rotated)
    keys, at the decode kernel's usual bar, for every split path (one tile,
    thread-block clusters, last-split merge, long context) and both layouts;
  * how far the convention moves the output from the reference golden
    computed from the unrotated keys: storing rotated K in BF16 rounds every
    key by up to 2^-9 relative, which moves each output by at most 2^-6 of its
    row's RMS (measured about 1.1 %).  Outputs that cancel to near zero can then
    differ by more than 64 BF16 ULP (about 0.3 % of them), so the pre-rotated
    cache is a different numerical contract from the reference's per-call RoPE
    and the 64-ULP rule is reported, not required;
  * batched ragged decode and flag validation.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import attention_accelerator_b200 as gqa
from attention_accelerator_b200 import _lib
from conftest import assert_chunk_parity, bits_to_torch, torch_to_bits
from oracle.bf16 import bf16_to_f32, f32_to_bf16, ulp_distance
from oracle.golden import gqa_golden_f64, rope_half_split

pytestmark = pytest.mark.gpu


def _inputs(seq_len: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(s, generator=g) for s in ((32, 128), (8, seq_len, 128), (8, seq_len, 128)))
    return tuple(torch_to_bits(t.to(torch.bfloat16)) for t in (q, k, v))


def _rotate_on_gpu(k_bits: np.ndarray, device, positions=None) -> np.ndarray:
    """Head-major [8, n, 128] codes -> rotated codes, through a position-major cache."""
    n = k_bits.shape[1]
    kd = bits_to_torch(k_bits.transpose(1, 0, 2).copy(), device)
    pos = torch.arange(n, dtype=torch.int32) if positions is None else torch.as_tensor(positions, dtype=torch.int32)
    return torch_to_bits(gqa.rope_k_cache(kd, pos)).transpose(1, 0, 2).copy()


def test_append_rotation_matches_oracle(cuda_device):
    """BF16(RoPE(k)) per element against the float64 rotation: within BF16 rounding
    (2^-8 relative) plus the FP32 rotation's absolute error, bounded by
    2^-20 (|x| + |y|) of the pair -- which dominates only where x c - y s cancels
    to a value far below its operands.  Almost every code equals the reference's
    f32_to_bf16 rounding of the float64 value."""
    _, k, _ = _inputs(4096, 11)
    positions = np.concatenate([np.arange(2048), np.random.default_rng(3).integers(0, 131072, 2048)])
    got = _rotate_on_gpu(k, cuda_device, positions)
    exact = rope_half_split(bf16_to_f32(k), positions)
    x = bf16_to_f32(k)
    pair_mag = np.abs(x[..., :64]) + np.abs(x[..., 64:])
    floor = 2.0 ** -20 * np.concatenate([pair_mag, pair_mag], axis=-1)
    err = np.abs(bf16_to_f32(got) - exact)
    assert (err <= 2.0 ** -8 * np.abs(exact) + floor).all()
    assert (ulp_distance(got, f32_to_bf16(exact)) == 0).mean() > 0.999


def test_rotation_in_place_and_head_major(cuda_device):
    _, k, _ = _inputs(777, 12)
    pos = torch.arange(777, dtype=torch.int32)
    pm = bits_to_torch(k.transpose(1, 0, 2).copy(), cuda_device)
    out_of_place = gqa.rope_k_cache(pm, pos)
    gqa.rope_k_cache(pm, pos, out=pm)
    assert torch.equal(pm, out_of_place)
    hm = bits_to_torch(k, cuda_device)
    rot_hm = gqa.rope_k_cache(hm, pos, layout="head_major")
    assert torch.equal(rot_hm.transpose(0, 1), out_of_place)


@pytest.mark.parametrize("seq_len", [30, 600, 4096, 5000, 131072])
@pytest.mark.parametrize("layout", ["position_major", "head_major"])
def test_decode_rotated_cache(seq_len, layout, cuda_device):
    if seq_len == 131072 and layout == "head_major":
        pytest.skip("one layout suffices at the longest length")
    q, k, v = _inputs(seq_len, 100 + seq_len % 97)
    k_rot = _rotate_on_gpu(k, cuda_device)
    if layout == "head_major":
        kd, vd = bits_to_torch(k_rot, cuda_device), bits_to_torch(v, cuda_device)
    else:
        kd = bits_to_torch(k_rot.transpose(1, 0, 2).copy(), cuda_device)
        vd = bits_to_torch(v.transpose(1, 0, 2).copy(), cuda_device)
    got = torch_to_bits(gqa.decode(bits_to_torch(q, cuda_device), kd, vd, layout=layout, k_rotated=True))
    chunk = 8192 if seq_len > 8192 else 2048
    # same keys: the decode kernel's usual bar against the float64 oracle
    assert_chunk_parity(gqa_golden_f64(q, k_rot, v, seq_len, seq_len - 1, exact=False, k_rotated=True,
                                       pos_chunk=chunk), got)
    # against the reference golden from the unrotated keys: within the effect of
    # rounding the rotated keys to BF16
    ref = gqa_golden_f64(q, k, v, seq_len, seq_len - 1, exact=False, pos_chunk=chunk)
    rms = np.sqrt((ref ** 2).mean(axis=1, keepdims=True))
    assert (np.abs(bf16_to_f32(got) - ref) <= 2.0 ** -6 * rms).all()


def test_batched_ragged_rotated(cuda_device):
    lens = [1, 17, 300, 2049, 4096]
    seqs = [_inputs(n, 300 + n) for n in lens]
    k_all = np.concatenate([_rotate_on_gpu(k, cuda_device) for _, k, _ in seqs], axis=1)
    v_all = np.concatenate([v for _, _, v in seqs], axis=1)
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]]).tolist()
    plan = gqa.plan_batch(lens, kv_starts=starts, device=cuda_device)
    q = bits_to_torch(np.stack([s[0] for s in seqs]), cuda_device)
    out = torch_to_bits(gqa.decode_batch(q, bits_to_torch(k_all.transpose(1, 0, 2).copy(), cuda_device),
                                         bits_to_torch(v_all.transpose(1, 0, 2).copy(), cuda_device), plan,
                                         k_rotated=True))
    for i, n in enumerate(lens):
        k_rot = k_all[:, starts[i]:starts[i] + n]
        assert_chunk_parity(gqa_golden_f64(seqs[i][0], k_rot, seqs[i][2], n, n - 1, exact=False, k_rotated=True),
                            out[i])


def test_flags_validation(cuda_device):
    lib = _lib.load()
    p = gqa.make_params(seq_len=64)
    p.k_pos_stride, p.k_head_stride = 1024, 128
    p.v_pos_stride, p.v_head_stride = 1024, 128
    p.q_head_stride, p.q_batch_stride = 128, 4096
    p.out_head_stride, p.out_batch_stride = 128, 4096
    buf = torch.zeros(64 * 8 * 128, dtype=torch.bfloat16, device=cuda_device)
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device=cuda_device)
    p.flags = 0x8  # unknown bit
    st = lib.gqa_decode(buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), ctypes.byref(p),
                        ws.data_ptr(), ws.numel(), None)
    assert st == _lib.GQA_ERR_FLAGS
    assert "flags" in _lib.status_string(st)
    # the chunked tensor-core path keeps per-call RoPE and refuses the flag
    c = _lib.GqaChunkParams(batch=1, n_queries=1, first_position=63, q_query_stride=4096, out_query_stride=4096,
                            k_batch_stride=64 * 1024, v_batch_stride=64 * 1024)
    p.flags = _lib.GQA_FLAG_K_ROTATED
    st = lib.gqa_decode_chunked(buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), ctypes.byref(p),
                                ctypes.byref(c), ws.data_ptr(), ws.numel(), None)
    assert st != _lib.GQA_OK
