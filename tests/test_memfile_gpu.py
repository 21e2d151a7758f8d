"""GPU parity tests of the ``.mem`` codec (gqa_mem_decode / gqa_mem_encode)
against the reference's host codec, restated in ``oracle.bf16``
(pyfiles/gqa_reference.py:26-46): the committed golden files (written by the
reference generator), the transport Q/K/V texts, a seeded fuzz of every text
form read_mem accepts (case, '_', blanks, blank and comment lines, CRLF and CR
line ends, no final newline, lines crossing the kernel's 64-byte segments and
16 KB blocks), the malformed forms it rejects, and a size-independent
encode -> decode round trip on a long-context-sized file.
"""
from __future__ import annotations

import random
from pathlib import Path

import numpy as np
import pytest
import torch

from attention_accelerator_b200 import memfile
from oracle.bf16 import mem_text, read_mem_array
from oracle.vectors import generate_case

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).parent / "golden" / "cases"


def _oracle_decode(text: bytes, elements: int, tmp_path: Path) -> np.ndarray:
    f = tmp_path / "x.mem"
    f.write_bytes(text)
    return read_mem_array(f, elements)


def _gpu(text: bytes, elements: int) -> np.ndarray:
    return memfile.decode_mem(text, elements).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("case", sorted(p.name for p in GOLDEN.iterdir()))
def test_golden_files_decode_and_re_encode_byte_exact(case, cuda_device):
    """The committed golden files were written by the reference generator's
    write_mem: decoding matches read_mem, and encoding gives the file back."""
    path = GOLDEN / case / "gqa_golden.mem"
    want = read_mem_array(path, 128)
    got = _gpu(path.read_bytes(), 128)
    np.testing.assert_array_equal(got, want)
    assert memfile.encode_mem(torch.from_numpy(want.view(np.int16)).to(cuda_device)) == path.read_bytes()


@pytest.mark.parametrize("seq_len,mode,seed", [(30, "random", 20260805), (17, "random", 20260817), (1, "smoke", 0)])
def test_transport_files_q_k_v(seq_len, mode, seed, cuda_device, tmp_path):
    """The AXIS-order Q, K and V beats of gen_gqa_wrapper_vectors.py:111-119 (16 elements a line)."""
    case = generate_case(seq_len, mode=mode, seed=seed)
    for text in (case.q_mem_text(), case.kv_mem_text("k"), case.kv_mem_text("v")):
        want = _oracle_decode(text.encode(), 16, tmp_path)
        got = _gpu(text.encode(), 16)
        np.testing.assert_array_equal(got, want)
        assert memfile.encode_mem(torch.from_numpy(want.view(np.int16)).to(cuda_device)) == text.encode()


def _fuzz_text(rng: random.Random, elements: int, n_lines: int) -> bytes:
    out = []
    for _ in range(n_lines):
        kind = rng.random()
        if kind < 0.08:
            out.append(rng.choice(["", " ", "\t", "  \t "]))
        elif kind < 0.14:
            out.append(rng.choice(["", " ", "\t"]) + "//" + rng.choice(["", " comment", " 0123 zz", "//"]))
        else:
            digits = "".join(rng.choice("0123456789abcdefABCDEF") for _ in range(4 * elements))
            if rng.random() < 0.3:  # underscores anywhere among the digits
                chars = list(digits)
                for _ in range(rng.randrange(1, 12)):
                    chars.insert(rng.randrange(len(chars) + 1), "_" * rng.randrange(1, 90))
                digits = "".join(chars)
            lead = rng.choice(["", "", " ", "\t", "  "])
            trail = rng.choice(["", "", " ", "\t "])
            out.append(lead + digits + trail)
    ends = [rng.choice(["\n", "\n", "\n", "\r\n", "\r"]) for _ in out]
    text = "".join(a + b for a, b in zip(out, ends))
    if rng.random() < 0.5:
        text = text.rstrip("\r\n")
    return text.encode()


@pytest.mark.parametrize("seed", range(12))
def test_fuzzed_text_forms(seed, cuda_device, tmp_path):
    rng = random.Random(1000 + seed)
    elements = rng.choice([16, 16, 128, 1, 3, 8])
    text = _fuzz_text(rng, elements, rng.choice([1, 7, 300, 2500]))
    np.testing.assert_array_equal(_gpu(text, elements), _oracle_decode(text, elements, tmp_path))


def test_one_long_line_across_blocks(cuda_device, tmp_path):
    """A data line of 40 KB ('_' padding) spans three 16 KB blocks and many segments."""
    digits = "0123456789abcdef" * 4
    text = ("\n\n" + digits[:20] + "_" * 40000 + digits[20:] + "\n" + digits + "\n").encode()
    np.testing.assert_array_equal(_gpu(text, 16), _oracle_decode(text, 16, tmp_path))


def test_empty_and_blank_only(cuda_device):
    assert _gpu(b"", 16).shape == (0, 16)
    assert _gpu(b"\n\n  \n// x\n", 16).shape == (0, 16)


@pytest.mark.parametrize("bad", [
    "0123",                        # too few digits
    "0123456789abcdef" * 4 + "0",  # too many
    "0123456789abcdeg" + "0" * 48,  # not hex
    "0123456789abcdef" * 2 + " " + "0123456789abcdef" * 2,  # blank between digits
    "/",                           # a lone slash is no comment
    "/x" + "0" * 62,
    "0" * 60 + "é",           # non-ASCII
])
def test_malformed_line_rejected_with_its_line_number(bad, cuda_device, tmp_path):
    good = "0123456789abcdef" * 4
    text = "\n".join([good, "// c", "", good, bad, good]) + "\n"
    with pytest.raises((ValueError, UnicodeDecodeError)):
        _oracle_decode(text.encode(), 16, tmp_path)
    with pytest.raises(ValueError, match=r"^line 5:"):
        memfile.decode_mem(text.encode(), 16)


@pytest.mark.parametrize("end", ["\r", "\r\n", "\n\r"])
def test_malformed_line_number_with_other_line_ends(end, cuda_device, tmp_path):
    """CR and CRLF line ends count one line each (a '\n\r' pair is two)."""
    good = "0123456789abcdef" * 4
    text = end.join([good, "// c", good, "0123", good]) + end
    with pytest.raises(ValueError):
        _oracle_decode(text.encode(), 16, tmp_path)
    want = 4 if end != "\n\r" else 7
    with pytest.raises(ValueError, match=rf"^line {want}:"):
        memfile.decode_mem(text.encode(), 16)


def host_encode(rows: np.ndarray) -> bytes:
    """Vectorised write_mem text for large arrays (the bytes of oracle.bf16.mem_text)."""
    hexd = np.frombuffer(b"0123456789abcdef", dtype=np.uint8)
    r = rows[:, ::-1].astype(np.uint32)
    nib = np.stack([(r >> s) & 0xF for s in (12, 8, 4, 0)], axis=-1).reshape(rows.shape[0], -1)
    lines = np.concatenate([hexd[nib], np.full((rows.shape[0], 1), ord("\n"), np.uint8)], axis=1)
    return lines.tobytes()


def test_round_trip_long_context_k_file(cuda_device):
    """8 KV heads x 8192 positions x 128 dims as 16-element beats (a 34 MB text):
    encode then decode is the identity, and the encoded bytes are write_mem's."""
    g = torch.Generator().manual_seed(5)
    rows = torch.randint(-32768, 32767, (8 * 8192 * 8, 16), generator=g, dtype=torch.int16)
    dev_rows = rows.to(cuda_device)
    text = memfile.encode_mem(dev_rows)
    host = rows.numpy().view(np.uint16)
    assert mem_text(host[:50]).encode() == text[:50 * 65]
    assert text == host_encode(host)
    back = memfile.decode_mem(text, 16)
    assert torch.equal(back, dev_rows)


@pytest.mark.parametrize("variant", ["plain", "upper", "no_final_newline", "comment_same_length", "cr_line_end",
                                     "blank_padded_line", "short_line_long_line"])
def test_fixed_width_shape_and_look_alikes(variant, cuda_device, tmp_path):
    """Texts whose byte count fits R lines of 4*elements digits + '\\n' take the fast
    path; the look-alikes among them (same length, other content) must fall back to
    the general parser and still match read_mem."""
    rng = np.random.default_rng(7)
    rows = rng.integers(0, 65536, size=(40, 16), dtype=np.uint16)
    lines = mem_text(rows).splitlines()
    if variant == "upper":
        lines = [ln.upper() for ln in lines]
    elif variant == "comment_same_length":
        lines[7] = "//" + "x" * 62
    elif variant == "blank_padded_line":
        lines[3] = "  " + lines[3][:62]
        lines[4] = lines[4][:60] + "    "
    elif variant == "short_line_long_line":
        lines[9], lines[10] = lines[9][:60], lines[10] + lines[9][60:]
    text = "\n".join(lines) + ("" if variant == "no_final_newline" else "\n")
    if variant == "cr_line_end":
        text = text.replace("\n", "\r", 1)
    data = text.encode()
    assert len(data) in (40 * 65, 40 * 65 - 1)
    try:
        want = _oracle_decode(data, 16, tmp_path)
    except ValueError:
        with pytest.raises(ValueError):
            memfile.decode_mem(data, 16)
        return
    np.testing.assert_array_equal(_gpu(data, 16), want)


def test_general_parser_at_scale(cuda_device):
    """A 41 MB CRLF file (the fixed-width fast path does not apply) is larger than
    the general parser's grid of 148 x 8 blocks x 16 KB, so every block walks
    several chunks; the decode equals the rows it was written from."""
    g = torch.Generator().manual_seed(9)
    rows = torch.randint(-32768, 32767, (600_000, 16), generator=g, dtype=torch.int16)
    host = rows.numpy().view(np.uint16)
    text = host_encode(host).replace(b"\n", b"\r\n")
    assert len(text) > 148 * 8 * 16384
    back = memfile.decode_mem(text, 16)
    assert torch.equal(back.cpu(), rows)
