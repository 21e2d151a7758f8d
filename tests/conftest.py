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


CANCEL_FLOOR = 2.0 ** -18   # below this fraction of the row max the 64-ULP rule is not FP32-attainable
ABS_BOUND = 2.0 ** -20      # absolute bound there, as a fraction of the row max


def assert_chunk_parity(golden64, got, tight: int = 2):
    """Parity against a float64 golden where outputs may cancel to a few FP32
    ulps of their row: the reference's 64-ULP rule (pyfiles/check_gqa_output.py:
    55-75) on every element at least CANCEL_FLOOR of its row's largest magnitude,
    an absolute error of at most ABS_BOUND of the row's largest below that (FP32
    arithmetic itself cannot hold 64 ULP there: a float32 restatement of the
    golden misses the strict rule on about 1 element in 262,144), and this
    build's FP32 bar on the rest (<= `tight` ULP where the golden is at least
    2^-10 of its row's largest, mean ULP < 0.1 over the strict elements).
    Returns the count of
    strict-rule exceptions."""
    from oracle import check_rows
    from oracle.bf16 import bf16_to_f32, f32_to_bf16, ulp_distance
    golden = f32_to_bf16(np.asarray(golden64)).reshape(-1, 128)
    g64 = np.asarray(golden64, dtype=np.float64).reshape(-1, 128)
    got = np.asarray(got).reshape(-1, 128)
    res = check_rows(golden, got, 64)
    dist = ulp_distance(golden, got)
    rowmax = np.abs(g64).max(axis=-1, keepdims=True)
    strict = np.abs(g64) >= CANCEL_FLOOR * rowmax
    exempt = ((golden.astype(np.int64) >> 7) & 0xFF) <= 0x3D
    assert not np.any((dist > 64) & strict & ~exempt), res.line()
    err = np.abs(bf16_to_f32(got).astype(np.float64) - g64)
    assert np.all(strict | (err <= ABS_BOUND * rowmax)), float((err / rowmax)[~strict].max())
    big = np.abs(g64) >= np.ldexp(rowmax, -10)
    assert int(dist[big].max(initial=0)) <= tight, res.line()
    assert dist[strict].mean() < 0.1, res.line()  # the mean where the ULP metric means something
    return int(np.sum((dist > 64) & ~exempt))
