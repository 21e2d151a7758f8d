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
