"""Stage the reference's own Python harness into ``oracle/_ref/`` (test infrastructure).

The reference's regression flow is three scripts run unchanged:
``pyfiles/run_gqa_regression.py`` (generates each case's vectors with
``pyfiles/gen_gqa_wrapper_vectors.py`` and runs ``$VIVADO -mode batch -source
scripts/run_gqa_wrapper_sim.tcl`` on them, :36-77), and
``pyfiles/check_gqa_output.py`` (the 64-ULP checker, :26-75), both importing
``pyfiles/gqa_reference.py``.  The GPU box has no reference tree, so this
recipe copies those four files, byte for byte, into the git-ignored
``oracle/_ref/pyfiles/`` of the build host's checkout, from where they travel
with the working tree.  ``tests/test_reference_harness_gpu.py`` then runs them
with ``VIVADO`` pointing at this build's drop-in executable.

Nothing here is product code and nothing is committed from the reference: the
copies live only under ``oracle/_ref/`` (listed in ``.gitignore``).

Usage: ``python -m oracle.stage_reference [--reference DIR]``; ``build()`` in
``__graft_entry__`` calls :func:`stage` when the reference tree is present.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
from pathlib import Path

ORACLE = Path(__file__).resolve().parent
REF_OUT = ORACLE / "_ref"
HARNESS = ("pyfiles/run_gqa_regression.py", "pyfiles/gen_gqa_wrapper_vectors.py",
           "pyfiles/gqa_reference.py", "pyfiles/check_gqa_output.py")
DEFAULT_REFERENCE = Path(os.environ.get("GQA_REFERENCE_DIR", "/root/reference"))


def staged() -> bool:
    """True when every harness file is in ``oracle/_ref/``."""
    return all((REF_OUT / rel).is_file() for rel in HARNESS)


def stage(reference: Path = DEFAULT_REFERENCE) -> bool:
    """Copy the harness files from ``reference``; False (nothing copied) when it is absent."""
    reference = Path(reference)
    if not all((reference / rel).is_file() for rel in HARNESS):
        return False
    digests = {}
    for rel in HARNESS:
        dst = REF_OUT / rel
        dst.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(reference / rel, dst)
        digests[rel] = hashlib.sha256(dst.read_bytes()).hexdigest()
    (REF_OUT / "staged.json").write_text(json.dumps(digests, indent=1) + "\n")
    return True


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=DEFAULT_REFERENCE)
    args = ap.parse_args()
    if not stage(args.reference):
        print(f"reference harness not found under {args.reference}")
        return 1
    print(f"staged {len(HARNESS)} files into {REF_OUT}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
