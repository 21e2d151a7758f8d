"""Restatement of the reference's output checker (test infrastructure, see package doc).

``check_rows`` follows ``pyfiles/check_gqa_output.py:55-75``: per element BF16-code
ULP distance (gqa_reference.py:49-53); a distance above ``max_ulp`` fails unless
both exponent fields are <= 0x3d (true underflow-scale values, :61-64).  It also
returns the mean ULP, which the reference does not print.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .bf16 import ulp_distance


@dataclass
class CheckResult:
    passed: bool
    failures: int
    worst_ulp: int
    worst_row: int
    worst_col: int
    mean_ulp: float

    def line(self, max_ulp: int = 64) -> str:
        if self.passed:
            return (f"PASS: worst ULP={self.worst_ulp} at row={self.worst_row}, "
                    f"col={self.worst_col}; mean ULP={self.mean_ulp:.4f} (limit {max_ulp})")
        return (f"FAIL: {self.failures} elements exceed {max_ulp} ULP; worst={self.worst_ulp} "
                f"at row={self.worst_row}, col={self.worst_col}")


def check_rows(golden, actual, max_ulp: int = 64) -> CheckResult:
    golden = np.asarray(golden, dtype=np.uint16)
    actual = np.asarray(actual, dtype=np.uint16)
    if golden.shape != actual.shape:
        raise ValueError(f"shape mismatch {golden.shape} vs {actual.shape}")
    dist = ulp_distance(golden, actual)
    exempt = (((golden.astype(np.int64) >> 7) & 0xFF) <= 0x3D) & (((actual.astype(np.int64) >> 7) & 0xFF) <= 0x3D)
    fail = (dist > max_ulp) & ~exempt
    flat = int(np.argmax(dist)) if dist.size else 0
    rows = golden.shape[-1] if golden.ndim else 1
    worst_row, worst_col = divmod(flat, rows)
    return CheckResult(passed=not bool(fail.any()), failures=int(fail.sum()),
                       worst_ulp=int(dist.max()) if dist.size else 0,
                       worst_row=worst_row, worst_col=worst_col,
                       mean_ulp=float(dist.mean()) if dist.size else 0.0)
