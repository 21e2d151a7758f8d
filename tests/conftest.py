"""Shared test setup: the ``gpu`` marker, repo import path and golden-fixture helpers."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def manifest():
    return json.loads((GOLDEN / "manifest.json").read_text())


def case_kwargs(args: list[str]) -> dict:
    """Generator CLI arguments of a manifest case -> oracle.generate_case keywords."""
    kw, it = {}, iter(args)
    for flag in it:
        key = flag[2:].replace("-", "_")
        val = next(it)
        kw[key] = val if key == "mode" else int(val)
    return kw


def bits_to_torch(bits: np.ndarray, device=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).astype(np.int16)).view(torch.bfloat16)
    return t.to(device) if device is not None else t


def torch_to_bits(t) -> np.ndarray:
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().astype(np.uint16)


def assert_parity(golden, got, tight: int = 2, max_ulp: int = 64):
    """The reference's rule (<= 64 ULP with the 0x3d exemption,
    pyfiles/check_gqa_output.py:55-75), then the FP32 bar of this build: <=
    `tight` ULP wherever the golden is at least 2^-10 of its row's largest
    magnitude (outputs that nearly cancel carry FP32 rounding of the large
    terms, a few ULP of a tiny number), and a small mean."""
    from oracle import check_rows
    from oracle.bf16 import bf16_to_f32, ulp_distance
    golden = np.asarray(golden).reshape(-1, 128)
    got = np.asarray(got).reshape(-1, 128)
    res = check_rows(golden, got, max_ulp)
    assert res.passed, res.line()
    mag = np.abs(bf16_to_f32(golden))
    big = mag >= np.ldexp(mag.max(axis=-1, keepdims=True), -10)
    dist = ulp_distance(golden, got)
    assert int(dist[big].max(initial=0)) <= tight, res.line()
    assert res.mean_ulp < 0.1, res.line()
    return res


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import attention_accelerator_b200  # noqa: F401  (loads the library; fails loudly if unbuilt)
    return torch.device("cuda", 0)


RESIDUE_FLOOR = 2.0 ** -18  # |golden| below this fraction of its row's largest: a cancellation residue
RESIDUE_ERR = 2.0 ** -20    # absolute error allowed on an accepted exception, as a fraction of the row max


def parity_exceptions(golden64, got):
    """Elements that fail the reference's rule exactly as pyfiles/check_gqa_output.py:
    57-69 applies it: BF16-code distance above 64 unless BOTH exponent fields are
    <= 0x3d.  Returns (exceptions, ulp distance, golden BF16 codes, row max), each
    exception a dict with its position, golden and output values, ULP and the
    magnitudes relative to its row's largest output."""
    from oracle.bf16 import bf16_to_f32, f32_to_bf16, ulp_distance
    g64 = np.asarray(golden64, dtype=np.float64).reshape(-1, 128)
    golden = f32_to_bf16(g64)
    got = np.asarray(got).reshape(-1, 128)
    dist = ulp_distance(golden, got)
    exempt = ((((golden.astype(np.int64) >> 7) & 0xFF) <= 0x3D) &
              (((got.astype(np.int64) >> 7) & 0xFF) <= 0x3D))
    rowmax = np.abs(g64).max(axis=-1, keepdims=True)
    out = []
    for r, c in zip(*np.nonzero((dist > 64) & ~exempt)):
        a = float(bf16_to_f32(got[r, c]))
        out.append({"row": int(r), "col": int(c), "golden": float(g64[r, c]), "got": a, "ulp": int(dist[r, c]),
                    "golden_of_rowmax": float(abs(g64[r, c]) / rowmax[r, 0]),
                    "err_of_rowmax": float(abs(a - g64[r, c]) / rowmax[r, 0])})
    return out, dist, golden, rowmax


def assert_chunk_parity(golden64, got, tight: int = 2, max_exceptions: int = 0, label: str = ""):
    """Parity against a float64 golden, held to the reference's per-element rule.

    * The reference's rule (pyfiles/check_gqa_output.py:55-75: <= 64 BF16 ULP
      unless both exponents are <= 0x3d) on every element.  At most
      `max_exceptions` elements may miss it, and only as bounded cancellation
      residues: golden below RESIDUE_FLOOR of its row's largest magnitude and
      absolute error at most RESIDUE_ERR of it.  The rule has no relative
      floor, so an output that cancels to ~2^-22 of its row is as strict as
      FP32 arithmetic itself; each caller that allows exceptions states the
      measured count.
    * This build's FP32 bar: <= `tight` ULP wherever the golden is at least
      2^-10 of its row's largest magnitude, mean ULP < 0.1 over the elements
      at least RESIDUE_FLOOR of it.
    Prints the exception count, worst and mean ULP (and each exception), and
    returns the exception list."""
    exc, dist, golden, rowmax = parity_exceptions(golden64, got)
    g64 = np.asarray(golden64, dtype=np.float64).reshape(-1, 128)
    print(f"parity {label}: {dist.size} outputs, {len(exc)} beyond 64 ULP (reference rule), "
          f"worst {int(dist.max(initial=0))} ULP, mean {float(dist.mean()):.5f} ULP")
    for e in exc:
        print(f"  exception {e}")
    assert len(exc) <= max_exceptions, exc
    for e in exc:
        assert e["golden_of_rowmax"] < RESIDUE_FLOOR and e["err_of_rowmax"] <= RESIDUE_ERR, e
    big = np.abs(g64) >= np.ldexp(rowmax, -10)
    assert int(dist[big].max(initial=0)) <= tight, f"worst {int(dist[big].max())} ULP on large outputs"
    strict = np.abs(g64) >= RESIDUE_FLOOR * rowmax
    assert dist[strict].mean() < 0.1, float(dist[strict].mean())
    return exc
