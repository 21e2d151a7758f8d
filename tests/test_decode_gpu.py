"""GPU parity of the decode kernel against the oracle and the reference's golden files.

Bound: the reference's 64 BF16-ULP rule with its 0x3d exponent exemption
(README.md:91-92, pyfiles/check_gqa_output.py:33,57-69).  The FP32 kernel is
additionally held to TIGHT_ULP, and mask decisions must match bit for bit.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import attention_accelerator_b200 as gqa
from conftest import GOLDEN, assert_parity, bits_to_torch, case_kwargs, torch_to_bits
from oracle import check_rows, generate_case, gqa_golden
from oracle.bf16 import f32_to_bf16, read_mem_array
from oracle.vectors import rope_kat

pytestmark = pytest.mark.gpu

MAX_ULP = 64
TIGHT_ULP = 2


def normal_inputs(seq_len: int, seed: int, k_channel_scale: bool = False):
    """BF16 codes of N(0,1) Q [32,128] and K, V [8, seq_len, 128] (head-major)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((32, 128), generator=g)
    k = torch.randn((8, seq_len, 128), generator=g)
    v = torch.randn((8, seq_len, 128), generator=g)
    if k_channel_scale:
        k = k * torch.exp(torch.randn((8, 1, 128), generator=g))
    return tuple(torch_to_bits(t.to(torch.bfloat16)) for t in (q, k, v))


def run_decode(q_bits, k_bits, v_bits, device, *, layout="position_major", **kw):
    q = bits_to_torch(q_bits, device)
    if layout == "head_major":
        k, v = bits_to_torch(k_bits, device), bits_to_torch(v_bits, device)
    else:
        k = bits_to_torch(k_bits.transpose(1, 0, 2), device)
        v = bits_to_torch(v_bits.transpose(1, 0, 2), device)
    return torch_to_bits(gqa.decode(q, k, v, layout=layout, **kw))


def _case_names():
    import json
    return sorted(json.loads((GOLDEN / "manifest.json").read_text())["cases"])


@pytest.mark.parametrize("layout", ["head_major", "position_major"])
@pytest.mark.parametrize("name", _case_names())
def test_reference_golden_cases(name, layout, manifest, cuda_device):
    case = generate_case(**case_kwargs(manifest["cases"][name]["args"]))
    golden = read_mem_array(GOLDEN / "cases" / name / "gqa_golden.mem", 128)
    got = run_decode(case.q_bits, case.k_bits, case.v_bits, cuda_device, layout=layout,
                     seq_len=case.seq_len, query_position=case.query_position,
                     kv_block_len=case.kv_block_len)
    assert_parity(golden, got)


def test_config1_uniform_pm1(cuda_device):
    """S=30, qpos 29, KVB 16, U[-1,1) from seed 20260805."""
    case = generate_case(30, mode="random", seed=20260805, amplitude=1.0)
    got = run_decode(case.q_bits, case.k_bits, case.v_bits, cuda_device, layout="head_major",
                     seq_len=30, query_position=29, kv_block_len=16)
    assert_parity(case.golden_bits(), got)


@pytest.mark.parametrize("seq_len,qpos", [(1, 0), (2, 1), (63, 62), (64, 63), (65, 64), (129, 5),
                                          (200, 199), (1000, 600), (2048, 2047)])
def test_normal_inputs(seq_len, qpos, cuda_device):
    q, k, v = normal_inputs(seq_len, seed=seq_len * 7 + qpos)
    golden = gqa_golden(q, k, v, seq_len, qpos, exact=seq_len <= 1024)
    got = run_decode(q, k, v, cuda_device, seq_len=seq_len, query_position=qpos)
    assert_parity(golden, got)


def test_config2_s4096(cuda_device):
    q, k, v = normal_inputs(4096, seed=20260805)
    got = run_decode(q, k, v, cuda_device, seq_len=4096, query_position=4095)
    res = assert_parity(gqa_golden(q, k, v, 4096, 4095, exact=False), got)
    assert res.mean_ulp < 0.1


def test_outlier_channels(cuda_device):
    """K with per-channel log-normal scales (BASELINE config 3's outlier channels)."""
    q, k, v = normal_inputs(3000, seed=3, k_channel_scale=True)
    got = run_decode(q, k, v, cuda_device, seq_len=3000, query_position=2999)
    assert_parity(gqa_golden(q, k, v, 3000, 2999, exact=False), got)


@pytest.mark.parametrize("kvb", [4, 16])
@pytest.mark.parametrize("seq_len", [1, 2, 15, 16, 17, 30, 32])
def test_mask_export_bit_exact(seq_len, kvb, cuda_device):
    """The kernel's key_valid() decisions against the RTL rule
    (kv_pos < SEQ_LEN) && (kv_pos <= QUERY_POSITION), gqa_attention_wrapper.v:279,
    over every padded key position of N_KV_TILES*KV_BLOCK_LEN."""
    n_pad = -(-seq_len // kvb) * kvb
    for qpos in sorted({0, seq_len // 2, seq_len - 1}):
        q, k, v = normal_inputs(n_pad, seed=seq_len + qpos)
        mask = torch.full((1, n_pad + 16), 7, dtype=torch.uint8, device=cuda_device)
        gqa.decode(bits_to_torch(q, cuda_device), bits_to_torch(k, cuda_device), bits_to_torch(v, cuda_device),
                   layout="head_major", seq_len=seq_len, query_position=qpos, kv_block_len=kvb, mask_out=mask)
        got = mask[0].cpu().numpy()
        p = np.arange(n_pad)
        want = ((p < seq_len) & (p <= qpos)).astype(np.uint8)
        np.testing.assert_array_equal(got[:n_pad], want)
        assert (got[n_pad:] == 7).all()


def test_score_tile_mask_pattern(cuda_device):
    """tests/tb_score_tile_mask.v:32-39: a 4-key block with keys 0,1 valid -> mask 0b0011."""
    q, k, v = normal_inputs(4, seed=1)
    mask = torch.zeros((1, 4), dtype=torch.uint8, device=cuda_device)
    gqa.decode(bits_to_torch(q, cuda_device), bits_to_torch(k, cuda_device), bits_to_torch(v, cuda_device),
               layout="head_major", seq_len=2, query_position=1, kv_block_len=4, mask_out=mask)
    bits = mask[0].cpu().numpy()
    assert int(sum(int(b) << i for i, b in enumerate(bits))) == 0b0011


def test_one_key_row_masked_lanes_are_zero(cuda_device):
    """tests/tb_flash_softmax_mask.v:26-42: one visible key in a 4-wide block; the masked
    lanes must contribute exactly zero, so the output is V row 0 exactly, even with
    large non-zero K/V in the masked pad rows."""
    q, k, v = normal_inputs(4, seed=2)
    k[:, 1:] = f32_to_bf16(np.full((8, 3, 128), 30.0))
    v[:, 1:] = f32_to_bf16(np.full((8, 3, 128), -1000.0))
    got = run_decode(q, k, v, cuda_device, layout="head_major", seq_len=1, query_position=0, kv_block_len=4)
    want = np.repeat(v[:, 0, :], 4, axis=0)  # Q head h reads KV head h // 4
    np.testing.assert_array_equal(got, want)


def test_causal_mask_inside_sequence(cuda_device):
    """QUERY_POSITION < SEQ_LEN-1: keys after the query are masked even though stored."""
    q, k, v = normal_inputs(300, seed=9)
    got = run_decode(q, k, v, cuda_device, seq_len=300, query_position=100)
    assert_parity(gqa_golden(q, k, v, 300, 100), got)
    # garbage after the query position must not matter
    k2, v2 = k.copy(), v.copy()
    k2[:, 101:] = f32_to_bf16(np.full((8, 199, 128), 50.0))
    v2[:, 101:] = f32_to_bf16(np.full((8, 199, 128), 9999.0))
    got2 = run_decode(q, k2, v2, cuda_device, seq_len=300, query_position=100)
    np.testing.assert_array_equal(got, got2)


def test_rope_known_answer_rows(cuda_device):
    """gen_rope_test_vectors.py:10-23 (512 rows at pos = row) through gqa_rope_rows."""
    x, golden = rope_kat()
    out = gqa.rope_rows(bits_to_torch(x, cuda_device), torch.arange(512, dtype=torch.int32))
    got = f32_to_bf16(out.cpu().numpy().astype(np.float64))
    res = check_rows(golden, got, 64)
    assert res.passed and res.worst_ulp <= 1, res.line()
    assert (got == golden).mean() > 0.99


def test_rope_large_positions(cuda_device):
    """RoPE at positions up to 131071 against the float64 restatement (FP32 tolerance)."""
    from oracle.golden import rope_half_split
    from oracle.bf16 import bf16_to_f32
    g = torch.Generator().manual_seed(5)
    x = torch_to_bits(torch.randn((256, 128), generator=g).to(torch.bfloat16))
    pos = np.concatenate([np.arange(128) * 1021 + 7, 131071 - np.arange(128)]).astype(np.int32)
    out = gqa.rope_rows(bits_to_torch(x, cuda_device), torch.from_numpy(pos)).cpu().numpy()
    ref = rope_half_split(bf16_to_f32(x), pos)
    assert np.abs(out - ref).max() < 2e-5 * max(1.0, np.abs(ref).max())


def test_host_buffers_end_to_end(cuda_device):
    """CPU tensors in, CPU tensor out: same bits as the device-resident call."""
    q, k, v = normal_inputs(777, seed=11)
    dev = run_decode(q, k, v, cuda_device, seq_len=777, query_position=776)
    out = gqa.decode(bits_to_torch(q), bits_to_torch(k.transpose(1, 0, 2).copy()),
                     bits_to_torch(v.transpose(1, 0, 2).copy()), seq_len=777, query_position=776)
    assert out.device.type == "cpu"
    np.testing.assert_array_equal(torch_to_bits(out), dev)


def test_repeat_calls_bitwise_stable(cuda_device):
    """Multi-split calls reuse the workspace: split counters must reset every call."""
    q, k, v = normal_inputs(4096, seed=12)
    outs = [run_decode(q, k, v, cuda_device, seq_len=4096, query_position=4095) for _ in range(4)]
    for o in outs[1:]:
        np.testing.assert_array_equal(o, outs[0])
    assert gqa.read_device_status(cuda_device) == 0


def test_config_errors_rejected_before_launch(cuda_device):
    q, k, v = (bits_to_torch(a, cuda_device) for a in normal_inputs(32, seed=4))
    cases = [dict(n_q_heads=31), dict(n_kv_heads=4), dict(head_dim=64), dict(tile_dim=8),
             dict(n_kv_tiles=3), dict(scale=0.0), dict(query_position=32), dict(kv_block_len=0),
             dict(group_size=2)]
    for kw in cases:
        with pytest.raises(gqa.GqaConfigError):
            gqa.decode(q, k, v, layout="head_major", seq_len=32, **kw)
    with pytest.raises(gqa.GqaConfigError):
        gqa.decode(q, k, v, layout="head_major", seq_len=0)


def _packed_cache(seqs, seed):
    """Position-major packed K/V cache [sum S, 8, 128] and per-sequence head-major views."""
    parts = [normal_inputs(s, seed=seed + i) for i, s in enumerate(seqs)]
    qs = np.stack([p[0] for p in parts])
    k = np.concatenate([p[1].transpose(1, 0, 2) for p in parts])
    v = np.concatenate([p[2].transpose(1, 0, 2) for p in parts])
    return parts, qs, k, v


def test_batched_ragged(cuda_device):
    seqs = [1, 17, 64, 65, 513, 1000, 2500, 4096]
    qpos = [0, 16, 10, 64, 300, 999, 2499, 4000]
    parts, qs, k, v = _packed_cache(seqs, seed=100)
    plan = gqa.plan_batch(seqs, query_positions=qpos, device=cuda_device)
    out = gqa.decode_batch(bits_to_torch(qs, cuda_device), bits_to_torch(k, cuda_device),
                           bits_to_torch(v, cuda_device), plan)
    got = torch_to_bits(out)
    for i, (s, qp) in enumerate(zip(seqs, qpos)):
        golden = gqa_golden(parts[i][0], parts[i][1], parts[i][2], s, qp, exact=s <= 1024)
        assert_parity(golden, got[i])


def test_sequence_split_partials_and_combine(cuda_device):
    """Long-context scheme on one GPU: contiguous key shards -> FP32 partials -> LSE combine."""
    s = 5000
    q, k, v = normal_inputs(s, seed=21)
    bounds = [0, 1200, 1201, 3333, 5000]
    shards = []
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        plan = gqa.plan_batch([s], pos_begin=[lo], pos_end=[hi], kv_starts=[0], partial=True, device=cuda_device)
        kk = bits_to_torch(k[:, lo:hi].transpose(1, 0, 2).copy(), cuda_device)
        vv = bits_to_torch(v[:, lo:hi].transpose(1, 0, 2).copy(), cuda_device)
        shards.append(gqa.decode_batch(bits_to_torch(q[None], cuda_device), kk, vv, plan))
    out = gqa.combine_partials(torch.stack(shards))
    got = torch_to_bits(out)[0]
    assert_parity(gqa_golden(q, k, v, s, s - 1, exact=False), got)
    full = run_decode(q, k, v, cuda_device, seq_len=s, query_position=s - 1)
    assert check_rows(full, got, 2).passed


def test_empty_shard_partial(cuda_device):
    """A shard entirely after QUERY_POSITION contributes m=-inf, l=0."""
    s = 300
    q, k, v = normal_inputs(s, seed=22)
    plan = gqa.plan_batch([s], query_positions=[99], pos_begin=[200], pos_end=[300], kv_starts=[0],
                          partial=True, device=cuda_device)
    part = gqa.decode_batch(bits_to_torch(q[None], cuda_device),
                            bits_to_torch(k[:, 200:].transpose(1, 0, 2).copy(), cuda_device),
                            bits_to_torch(v[:, 200:].transpose(1, 0, 2).copy(), cuda_device), plan).cpu()
    assert torch.isinf(part[0, :, 128]).all() and (part[0, :, 128] < 0).all()
    assert (part[0, :, 129] == 0).all() and (part[0, :, :128] == 0).all()


def test_long_context_131072(cuda_device):
    """BASELINE config 4 geometry: S=131072 against the float64 oracle, and a 4-shard split."""
    s = 131072
    q, k, v = normal_inputs(s, seed=131)
    got = run_decode(q, k, v, cuda_device, seq_len=s, query_position=s - 1)
    assert_parity(gqa_golden(q, k, v, s, s - 1, exact=False, pos_chunk=8192), got)
    step = s // 4
    kd = bits_to_torch(k.transpose(1, 0, 2).copy(), cuda_device)
    vd = bits_to_torch(v.transpose(1, 0, 2).copy(), cuda_device)
    parts = []
    for r in range(4):
        plan = gqa.plan_batch([s], pos_begin=[r * step], pos_end=[(r + 1) * step], kv_starts=[0],
                              partial=True, device=cuda_device)
        parts.append(gqa.decode_batch(bits_to_torch(q[None], cuda_device), kd[r * step:(r + 1) * step],
                                      vd[r * step:(r + 1) * step], plan))
    split = torch_to_bits(gqa.combine_partials(torch.stack(parts)))[0]
    assert check_rows(got, split, 2).passed  # summation order differs; both match the oracle above


def test_split_plans(cuda_device):
    """Short single sequences merge their splits inside clusters (one per KV head);
    longer ones in the last split of each KV head to finish; batches in
    split_merge_kernel."""
    assert gqa.decode_plan(30) == gqa.SplitPlan(1, 88, 0)
    p = gqa.decode_plan(600)
    assert 2 <= p.cluster <= 16 and p.splits == p.cluster and p.splits * p.keys_per_split >= 600
    for s in (4096, 131072):
        p = gqa.decode_plan(s)
        assert p.cluster == 0 and p.splits > 1 and p.splits * p.keys_per_split >= s
    one = gqa.decode_plan(plan=gqa.plan_batch([4096], device=cuda_device))
    assert one == gqa.decode_plan(4096)  # a batch of one takes the single-sequence plan
    two = gqa.decode_plan(plan=gqa.plan_batch([4096, 4096], device=cuda_device))
    assert two.cluster == 0 and two.splits > 2


# (seq_len, qpos): 100 / 600 / 1000 keys take the cluster merge, the rest the
# last-split merge.
@pytest.mark.parametrize("seq_len,qpos", [(100, 99), (600, 599), (1000, 999), (4096, 4095), (4096, 1500),
                                          (20000, 19999), (33000, 32999)])
def test_single_sequence_merges_match_split_merge_kernel(seq_len, qpos, cuda_device):
    """The single-sequence merges (cluster or last split) and split_merge_kernel
    (the same sequence twice in one batch) agree to FP32 rounding, and both meet
    the oracle."""
    assert gqa.decode_plan(seq_len, query_position=qpos).splits > 1
    q, k, v = normal_inputs(seq_len, seed=seq_len + qpos)
    clustered = run_decode(q, k, v, cuda_device, seq_len=seq_len, query_position=qpos)
    plan = gqa.plan_batch([seq_len, seq_len], query_positions=[qpos, qpos], kv_starts=[0, 0], device=cuda_device)
    assert gqa.decode_plan(plan=plan).cluster == 0
    out2 = gqa.decode_batch(bits_to_torch(np.stack([q, q]), cuda_device),
                            bits_to_torch(k.transpose(1, 0, 2).copy(), cuda_device),
                            bits_to_torch(v.transpose(1, 0, 2).copy(), cuda_device), plan)
    merged = torch_to_bits(out2)[0]
    np.testing.assert_array_equal(torch_to_bits(out2)[1], merged)
    assert check_rows(merged, clustered, 2).passed
    golden = gqa_golden(q, k, v, seq_len, qpos, exact=seq_len <= 1024)
    assert_parity(golden, clustered)
    assert_parity(golden, merged)


def test_interleaved_split_counts_share_workspace(cuda_device):
    """Calls with different split counts and merges on one stream (one workspace):
    the per-head arrival counters return to zero after every call, so each
    result repeats bit for bit."""
    lens = [4096, 20000, 600, 2000, 131, 4096]
    inputs = {s: normal_inputs(s, seed=s) for s in set(lens)}
    first = {}
    for rnd in range(3):
        for s in lens:
            got = run_decode(*inputs[s], cuda_device, seq_len=s, query_position=s - 1)
            if s in first:
                np.testing.assert_array_equal(first[s], got)
            else:
                first[s] = got
    from attention_accelerator_b200 import api
    torch.cuda.synchronize()
    ws = api._workspace(cuda_device, api._stream_ptr(cuda_device), 4096)
    assert int(torch.count_nonzero(ws[:256])) == 0  # status word and arrival counters


def test_config3_full_batch(cuda_device):
    """BASELINE config 3 at full size: the bench's 64 sequence lengths
    (U{512..8192}, 301,934 keys, K with per-channel outlier scales) in one
    launch of 1088 (split, KV head) items plus the split merge, each sequence against the float64
    oracle.  Bar: the reference's per-element rule on all 262,144 outputs with
    no exception (``assert_chunk_parity``, measured on B200: 0 beyond 64 ULP,
    worst 43 ULP on a near-zero output), <= 2 ULP on large outputs."""
    from conftest import assert_chunk_parity
    from oracle.golden import gqa_golden_f64
    seqs = [int(x) for x in np.random.default_rng(20260805).integers(512, 8193, size=64)]
    assert sum(seqs) == 301934
    parts = [normal_inputs(s, seed=3000 + i, k_channel_scale=True) for i, s in enumerate(seqs)]
    qs = np.stack([p[0] for p in parts])
    k = np.concatenate([p[1].transpose(1, 0, 2) for p in parts])
    v = np.concatenate([p[2].transpose(1, 0, 2) for p in parts])
    plan = gqa.plan_batch(seqs, device=cuda_device)
    out = gqa.decode_batch(bits_to_torch(qs, cuda_device), bits_to_torch(k, cuda_device),
                           bits_to_torch(v, cuda_device), plan)
    got = torch_to_bits(out)
    golden = np.stack([gqa_golden_f64(parts[i][0], parts[i][1], parts[i][2], s, s - 1, exact=False)
                       for i, s in enumerate(seqs)])
    assert_chunk_parity(golden, got, max_exceptions=0, label="config 3 (64 ragged sequences)")

