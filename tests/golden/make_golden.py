#!/usr/bin/env python3
"""Regenerate the golden fixtures in this folder from the reference's own scripts.

Runs, unchanged and with ``python3 -B`` (the reference tree is read-only), the
reference's generators:
  * ``pyfiles/gen_gqa_wrapper_vectors.py`` for every case in ``CASES`` (the six
    ``run_gqa_regression.py:13-20`` cases, the README 65,536-element corpus, the
    default smoke corpus, and extra causal / block-length / longer cases);
  * ``pyfiles/gen_rope_test_vectors.py`` (512-row RoPE known-answer set);
  * ``pyfiles/gen_bf16_primitive_vectors.py`` (65,536 BF16 add/multiply
    conformance cases, the reference's definition of its BF16 units);
  * ``tools/gen_rope_rom.py`` at 10 and 14 address bits, and ``pyfiles/gen_rope_rom.py``.
It records the sha256 of every file they write in ``manifest.json`` and copies
each case's ``gqa_golden.mem`` and ``gqa_config.txt`` under ``cases/<name>/``.
Input ``.mem`` files are not stored: the oracle regenerates them and the tests
compare their sha256 with the manifest.

Usage (build container only; the GPU box has no reference tree):
    python tests/golden/make_golden.py --reference /path/to/reference
"""
from __future__ import annotations

import argparse
import hashlib
import json
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent

# name, generator arguments
CASES = [
    ("smoke_len1", ["--mode", "smoke", "--seq-len", "1"]),
    ("random_len15", ["--mode", "random", "--seq-len", "15", "--seed", "20260815"]),
    ("random_len16", ["--mode", "random", "--seq-len", "16", "--seed", "20260816"]),
    ("random_len17_bp", ["--mode", "random", "--seq-len", "17", "--seed", "20260817"]),
    ("random_len30", ["--mode", "random", "--seq-len", "30", "--seed", "20260805"]),
    ("random_len32_bp", ["--mode", "random", "--seq-len", "32", "--seed", "20260832"]),
    ("corpus_65536", ["--mode", "random", "--seed", "20260805", "--target-input-vectors", "65536"]),
    ("smoke_default", []),
    ("causal_len30_q7", ["--mode", "random", "--seq-len", "30", "--seed", "11", "--query-position", "7"]),
    ("causal_len64_q0", ["--mode", "random", "--seq-len", "64", "--seed", "12", "--query-position", "0"]),
    ("causal_len100_q63", ["--mode", "random", "--seq-len", "100", "--seed", "13", "--query-position", "63"]),
    ("block4_len17", ["--mode", "random", "--seq-len", "17", "--seed", "14", "--kv-block-len", "4"]),
    ("block8_len30_q20", ["--mode", "random", "--seq-len", "30", "--seed", "15", "--kv-block-len", "8",
                          "--query-position", "20"]),
    ("random_len256", ["--mode", "random", "--seq-len", "256", "--seed", "16"]),
    ("random_len1024", ["--mode", "random", "--seq-len", "1024", "--seed", "17"]),
]


def sha256(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def run(cmd, cwd=None, env=None):
    res = subprocess.run(cmd, cwd=cwd, env=env, text=True, capture_output=True)
    if res.returncode:
        raise SystemExit(f"{' '.join(map(str, cmd))} failed:\n{res.stdout}{res.stderr}")
    return res.stdout


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    args = ap.parse_args()
    ref = args.reference.resolve()
    py = [sys.executable, "-B"]
    manifest = {"python": sys.version.split()[0], "cases": {}, "rope_kat": {}, "rope_rom": {},
                "bf16_primitives": {}}
    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        for name, extra in CASES:
            out = tmp / name
            run(py + [str(ref / "pyfiles/gen_gqa_wrapper_vectors.py"), "--out-dir", str(out)] + extra)
            files = {f: sha256(out / f) for f in
                     ("gqa_q.mem", "gqa_k.mem", "gqa_v.mem", "gqa_golden.mem", "gqa_config.txt")}
            manifest["cases"][name] = {"args": extra, "sha256": files}
            dst = HERE / "cases" / name
            dst.mkdir(parents=True, exist_ok=True)
            shutil.copy(out / "gqa_golden.mem", dst / "gqa_golden.mem")
            shutil.copy(out / "gqa_config.txt", dst / "gqa_config.txt")
        out = tmp / "rope"
        run(py + [str(ref / "pyfiles/gen_rope_test_vectors.py"), "--out-dir", str(out)])
        manifest["rope_kat"] = {"rows": 512, "seed": 20260805,
                                "sha256": {f: sha256(out / f) for f in ("in.mem", "golden.mem")}}
        out = tmp / "bf16"
        run(py + [str(ref / "pyfiles/gen_bf16_primitive_vectors.py"), "--out-dir", str(out)])
        manifest["bf16_primitives"] = {"cases": 65536, "seed": 20260805, "sha256": {
            f: sha256(out / f) for f in ("a.mem", "b.mem", "add_golden.mem", "mul_golden.mem")}}
        for bits in (10, 14):
            out = tmp / f"rom{bits}"
            run(py + [str(ref / "tools/gen_rope_rom.py"), "--out-dir", str(out), "--rom-addr-bits", str(bits)])
            manifest["rope_rom"][f"tools_bits{bits}"] = {
                f: sha256(out / f) for f in ("rope_phase_rom.mem", "rope_sincos_rom.mem")}
        cwd = tmp / "pyrom"
        cwd.mkdir()
        run(py + [str(ref / "pyfiles/gen_rope_rom.py")], cwd=cwd,
            env={"PYTHONPATH": str(ref / "pyfiles"), "PATH": "/usr/bin:/bin"})
        manifest["rope_rom"]["pyfiles_bits14"] = {
            f: sha256(cwd / "rope_rom" / f) for f in ("rope_phase_rom.mem", "rope_sincos_rom.mem")}
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(CASES)} cases to {HERE}")


if __name__ == "__main__":
    main()
