"""The oracle pinned against files the reference's own scripts wrote (sha256 + golden rows).

If these pass, every regenerated input, config text, golden output, RoPE
known-answer row and ROM table used by the GPU tests is byte-identical to what
``pyfiles/gen_gqa_wrapper_vectors.py``, ``pyfiles/gen_rope_test_vectors.py`` and
``tools/gen_rope_rom.py`` produce (tests/golden/make_golden.py recorded them).
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

from conftest import GOLDEN, case_kwargs
from oracle import check_rows, generate_case, gqa_golden
from oracle.bf16 import bf16_to_f32, f32_to_bf16, read_mem_array, ulp_distance, unpack_bf16, pack_bf16
from oracle.rope_rom import rom_texts
from oracle.vectors import beats_text, rope_kat


def sha(text: str) -> str:
    return hashlib.sha256(text.encode()).hexdigest()


def test_every_case_regenerates_byte_identical(manifest):
    for name, entry in manifest["cases"].items():
        case = generate_case(**case_kwargs(entry["args"]))
        want = entry["sha256"]
        assert sha(case.q_mem_text()) == want["gqa_q.mem"], name
        assert sha(case.kv_mem_text("k")) == want["gqa_k.mem"], name
        assert sha(case.kv_mem_text("v")) == want["gqa_v.mem"], name
        assert sha(case.config_text()) == want["gqa_config.txt"], name
        golden_file = GOLDEN / "cases" / name / "gqa_golden.mem"
        assert hashlib.sha256(golden_file.read_bytes()).hexdigest() == want["gqa_golden.mem"], name


@pytest.mark.parametrize("name", ["smoke_len1", "random_len15", "random_len17_bp", "random_len30",
                                  "causal_len30_q7", "causal_len64_q0", "block8_len30_q20", "random_len256"])
def test_oracle_golden_is_bit_identical(name, manifest):
    case = generate_case(**case_kwargs(manifest["cases"][name]["args"]))
    assert sha(case.golden_mem_text()) == manifest["cases"][name]["sha256"]["gqa_golden.mem"]


def test_fast_oracle_agrees_with_exact(manifest):
    for name in ("random_len256", "causal_len100_q63", "random_len1024"):
        case = generate_case(**case_kwargs(manifest["cases"][name]["args"]))
        golden = read_mem_array(GOLDEN / "cases" / name / "gqa_golden.mem", 128)
        fast = case.golden_bits(exact=False)
        assert check_rows(golden, fast, 0).worst_ulp <= 1


def test_parallel_port_agrees_with_the_pinned_golden(manifest):
    """The thread-parallel float64 port that bench.py times as the reference's CPU
    path (oracle/parallel.py) gives the reference golden files within 1 ULP,
    including a causal case and slab boundaries (1024 keys per slab)."""
    from oracle.parallel import gqa_golden_parallel
    for name in ("random_len30", "causal_len100_q63", "random_len1024", "random_len256"):
        case = generate_case(**case_kwargs(manifest["cases"][name]["args"]))
        golden = read_mem_array(GOLDEN / "cases" / name / "gqa_golden.mem", 128)
        got = gqa_golden_parallel(case.q_bits, case.k_bits, case.v_bits, case.seq_len, case.query_position,
                                  threads=4, slab=96)
        assert check_rows(golden, got, 0).worst_ulp <= 1, name


@pytest.mark.parametrize("seq_len,first,n", [(300, 280, 20), (300, 100, 16), (64, 0, 64)])
def test_chunked_oracle_is_the_per_query_golden(seq_len, first, n):
    """oracle/chunked.py (the checker of the tensor-core path and config 5's CPU
    baseline) answers query i exactly as the single-position golden with
    QUERY_POSITION = first + i (gen_gqa_wrapper_vectors.py:121-139)."""
    from oracle import chunked_golden_f64
    from oracle.golden import gqa_golden_f64
    rng = np.random.default_rng(seq_len + first)
    q = f32_to_bf16(rng.standard_normal((2, n, 32, 128)).astype(np.float32))
    k = f32_to_bf16(rng.standard_normal((2, 8, seq_len, 128)).astype(np.float32))
    v = f32_to_bf16(rng.standard_normal((2, 8, seq_len, 128)).astype(np.float32))
    got = chunked_golden_f64(q, k, v, seq_len, first)
    for b in range(2):
        for i in range(0, n, 3):
            want = gqa_golden_f64(q[b, i], k[b], v[b], seq_len, first + i, exact=False)
            np.testing.assert_allclose(got[b, i], want, rtol=1e-12, atol=1e-15)


def test_corpus_65536_is_the_len30_case(manifest):
    """README.md:121-138: 65,536 valid elements select SEQ_LEN=30 with two pad rows."""
    c = manifest["cases"]
    assert c["corpus_65536"]["sha256"] == c["random_len30"]["sha256"]
    case = generate_case(**case_kwargs(c["corpus_65536"]["args"]))
    assert case.seq_len == 30 and case.kv_input_len == 32
    assert "VALID_INPUT_BF16_VECTORS=65536" in case.config_text()
    assert "TRANSPORT_BF16_VECTORS=69632" in case.config_text()


def test_rope_known_answer_set(manifest):
    x, golden = rope_kat()
    assert sha(beats_text(x)) == manifest["rope_kat"]["sha256"]["in.mem"]
    assert sha(beats_text(golden)) == manifest["rope_kat"]["sha256"]["golden.mem"]


@pytest.mark.parametrize("bits", [10, 14])
def test_rope_rom_tables(bits, manifest):
    texts = rom_texts(addr_bits=bits)
    want = manifest["rope_rom"][f"tools_bits{bits}"]
    for fname, text in texts.items():
        assert sha(text) == want[fname]
    if bits == 14:
        assert {f: sha(t) for f, t in texts.items()} == manifest["rope_rom"]["pyfiles_bits14"]


def test_bf16_rounding_edges():
    vals = np.array([0.0, -0.0, 1.0, 1.0 + 2**-8, 1.0 + 3 * 2**-8, 1e-40, -3.0e38, np.inf, -np.inf])
    bits = f32_to_bf16(vals)
    assert bits[3] == 0x3F80  # tie to even
    assert bits[4] == 0x3F82
    assert bits[7] == 0x7F80 and bits[8] == 0xFF80
    np.testing.assert_array_equal(f32_to_bf16(bf16_to_f32(bits)), bits)


def test_ulp_and_checker_rule():
    assert ulp_distance(0x3F80, 0x3F81) == 1
    assert ulp_distance(0x0001, 0x8001) == 2
    golden = np.full((2, 128), 0x3F80, dtype=np.uint16)
    actual = golden.copy()
    actual[0, 5] = 0x3F80 + 65
    res = check_rows(golden, actual, 64)
    assert not res.passed and res.failures == 1 and res.worst_ulp == 65
    # exponent fields <= 0x3d on both sides are exempt (check_gqa_output.py:61-64)
    tiny_g = np.full((1, 128), 0x1E00, dtype=np.uint16)
    tiny_a = np.full((1, 128), 0x1E90, dtype=np.uint16)
    assert check_rows(tiny_g, tiny_a, 64).passed


def test_mem_line_order():
    line = pack_bf16(list(range(16)))
    assert line.endswith("0000") and line.startswith("000f")
    assert unpack_bf16(line, 16) == list(range(16))


def test_golden_causal_only_reads_visible_keys():
    """Changing keys after QUERY_POSITION changes nothing (the implicit mask of :132-133)."""
    case = generate_case(40, mode="random", seed=5, query_position=9)
    base = case.golden_bits()
    case.k_bits[:, 10:] ^= 0x1234
    case.v_bits[:, 10:] ^= 0x0F0F
    np.testing.assert_array_equal(case.golden_bits(), base)


def test_generator_argument_checks():
    with pytest.raises(ValueError):
        generate_case(0)
    with pytest.raises(ValueError):
        generate_case(10, query_position=10)
    with pytest.raises(ValueError):
        generate_case(target_input_vectors=65537)
    with pytest.raises(ValueError):
        generate_case(10, kv_block_len=0)


def _primitive_vectors(cases: int = 65536, seed: int = 20260805):
    """The operands of pyfiles/gen_bf16_primitive_vectors.py:26-30 (all a, then all b)."""
    import random
    rng = random.Random(seed)
    a = f32_to_bf16(np.array([rng.uniform(-0.25, 0.25) for _ in range(cases)]))
    b = f32_to_bf16(np.array([rng.uniform(-0.25, 0.25) for _ in range(cases)]))
    return a, b


def test_bf16_unit_semantics_match_reference_conformance_vectors(manifest):
    """The RTL's BF16 adder and multiplier as the reference defines them for
    conformance (gen_bf16_primitive_vectors.py:31-32): float64 result of the two
    BF16 operands, rounded by f32_to_bf16.  The oracle's RTL-numerics RoPE uses
    exactly these operations; here they reproduce the reference's own files."""
    a, b = _primitive_vectors()
    fa, fb = bf16_to_f32(a), bf16_to_f32(b)

    def words(x):
        return ("\n".join(f"{int(w):04x}" for w in x) + "\n").encode()
    want = manifest["bf16_primitives"]["sha256"]
    assert hashlib.sha256(words(a)).hexdigest() == want["a.mem"]
    assert hashlib.sha256(words(b)).hexdigest() == want["b.mem"]
    assert hashlib.sha256(words(f32_to_bf16(fa + fb))).hexdigest() == want["add_golden.mem"]
    assert hashlib.sha256(words(f32_to_bf16(fa * fb))).hexdigest() == want["mul_golden.mem"]


def test_rtl_rope_restatement():
    """oracle.rtl follows rope_unit.v: 32-bit NCO phase, top 14 bits into the BF16
    sincos ROM, rotation through BF16 multiply/subtract/add.  No RTL output dump
    exists to pin it end to end; its parts are pinned (ROMs above, BF16 units
    above), and against the float64 RoPE known-answer rows it stays within the
    BF16 units' error: 2^-7 of the row pair's magnitude."""
    from oracle.rtl import rom_factors, rope_rtl_rows
    inp, gold = rope_kat()
    got = rope_rtl_rows(inp, np.arange(512))
    x = bf16_to_f32(inp)
    mag = np.abs(x[:, :64]) + np.abs(x[:, 64:])
    err = np.abs(bf16_to_f32(got) - bf16_to_f32(gold))
    assert (err <= 2.0 ** -7 * np.concatenate([mag, mag], axis=1) + 2.0 ** -8 * np.abs(bf16_to_f32(gold))).all()
    # the NCO: position 0 is angle 0 (cos 1, sin 0) for every pair
    c, s = rom_factors([0])
    assert (c == 0x3F80).all() and (s == 0).all()
