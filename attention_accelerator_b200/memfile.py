"""``.mem`` transport files and ``gqa_config.txt`` of the reference's toolflow.

Format (pyfiles/gqa_reference.py:1-46): one packed AXIS word per line in hex,
element 0 in the rightmost 4 digits.  Q is 32 rows x 8 beats of 16 BF16
elements; K and V are head-major [8][KV_INPUT_LEN] rows of 8 beats each
(gen_gqa_wrapper_vectors.py:109-119); output and golden files hold one
128-element row per line.  The per-element BF16-code ULP rule of
pyfiles/check_gqa_output.py:55-69 is here too, because the ``$VIVADO``
drop-in reports PASS/FAIL the way the reference testbench does.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np


def parse_mem_text(text: str, elements: int) -> np.ndarray:
    """Lines of packed hex -> uint16 array ``[lines, elements]`` (element 0 first)."""
    lines = [ln.strip().replace("_", "") for ln in text.splitlines()]
    lines = [ln for ln in lines if ln and not ln.startswith("//")]
    if not lines:
        return np.zeros((0, elements), dtype=np.uint16)
    for ln in lines:
        if len(ln) != 4 * elements:
            raise ValueError(f"expected {4 * elements} hex digits per line, got {len(ln)}")
    raw = np.frombuffer(bytes.fromhex("".join(lines)), dtype=">u2").reshape(len(lines), elements)
    return raw[:, ::-1].astype(np.uint16)


def format_mem_text(rows: np.ndarray) -> str:
    """uint16 ``[lines, elements]`` -> ``.mem`` text (element 0 rightmost), trailing newline."""
    rows = np.asarray(rows, dtype=np.uint16)
    packed = np.ascontiguousarray(rows[:, ::-1]).astype(">u2")
    return "".join(packed[i].tobytes().hex() + "\n" for i in range(packed.shape[0]))


def read_mem(path: Path, elements: int) -> np.ndarray:
    return parse_mem_text(Path(path).read_text(), elements)


def write_mem(path: Path, rows: np.ndarray) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(format_mem_text(rows))


def rows_from_beats(beats: np.ndarray, head_dim: int = 128) -> np.ndarray:
    """``[n_beats, tile_dim]`` -> ``[n_rows, head_dim]`` (a row is head_dim/tile_dim consecutive beats)."""
    return beats.reshape(-1, head_dim)


def read_config(path: Path) -> dict[str, str]:
    """``KEY=VALUE`` lines of gqa_config.txt (gen_gqa_wrapper_vectors.py:145-152)."""
    cfg = {}
    for line in Path(path).read_text().splitlines():
        if "=" in line:
            key, _, val = line.partition("=")
            cfg[key.strip()] = val.strip()
    return cfg


def ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Monotonic BF16-code distance (gqa_reference.py:49-53)."""
    def ordered(x):
        x = np.asarray(x).astype(np.int64) & 0xFFFF
        return np.where(x & 0x8000, 0x8000 - (x & 0x7FFF), 0x8000 + x)
    return np.abs(ordered(a) - ordered(b))


def compare_rows(golden: np.ndarray, actual: np.ndarray, max_ulp: int = 64) -> dict:
    """check_gqa_output.py:55-69: failures are distances above max_ulp unless both
    exponent fields are <= 0x3d.  Also reports the mean distance."""
    golden = np.asarray(golden, dtype=np.uint16)
    actual = np.asarray(actual, dtype=np.uint16)
    dist = ulp_distance(golden, actual)
    exempt = ((golden.astype(np.int64) >> 7) & 0xFF <= 0x3D) & ((actual.astype(np.int64) >> 7) & 0xFF <= 0x3D)
    fail = (dist > max_ulp) & ~exempt
    flat = int(np.argmax(dist)) if dist.size else 0
    row, col = divmod(flat, golden.shape[-1]) if dist.size else (0, 0)
    return {"failures": int(fail.sum()), "worst": int(dist.max()) if dist.size else 0,
            "worst_row": row, "worst_col": col, "mean": float(dist.mean()) if dist.size else 0.0}
