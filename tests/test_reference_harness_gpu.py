"""The reference's own regression harness, run unchanged against the ``$VIVADO`` drop-in.

``pyfiles/run_gqa_regression.py`` generates the vectors of its six cases with
``pyfiles/gen_gqa_wrapper_vectors.py`` and runs ``$VIVADO -mode batch -source
scripts/run_gqa_wrapper_sim.tcl`` on each (:36-77), passing a case on exit 0
plus ``PASS:``, then the invalid-configuration case.  Here ``VIVADO`` is this
build's ``bin/vivado``, so every case runs one decode on the GPU.  Each output
file is then checked again by the reference's ``pyfiles/check_gqa_output.py``
(:26-75).  The scripts are the reference's files, copied byte for byte into
``oracle/_ref/pyfiles/`` by ``oracle/stage_reference.py`` on the build host;
the test is skipped where they were not staged.
"""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

REF = ROOT / "oracle" / "_ref" / "pyfiles"
SHIM = ROOT / "attention_accelerator_b200" / "bin" / "vivado"
CASES = ("smoke_len1", "random_len15", "random_len16", "random_len17_bp", "random_len30", "random_len32_bp")


def _staged() -> bool:
    from oracle.stage_reference import staged
    return staged()


@pytest.fixture(scope="module")
def regression_run(tmp_path_factory, cuda_device):
    if not _staged():
        pytest.skip("reference harness not staged into oracle/_ref (python -m oracle.stage_reference)")
    out = tmp_path_factory.mktemp("gqa_regression")
    env = dict(os.environ, VIVADO=str(SHIM), PYTHONDONTWRITEBYTECODE="1")
    res = subprocess.run([sys.executable, "-B", str(REF / "run_gqa_regression.py"), "--out-dir", str(out)],
                         cwd=out, env=env, text=True, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                         timeout=900)
    return res, out


def test_run_gqa_regression_unchanged_passes_every_case(regression_run):
    res, out = regression_run
    assert res.returncode == 0, res.stdout[-4000:]
    assert "GQA REGRESSION PASSED: 6 datapath cases plus invalid-config rejection" in res.stdout, res.stdout[-4000:]
    for name in CASES + ("invalid_config",):
        assert f"[{name}] PASS" in res.stdout, name
    for name in CASES:
        log = (out / name / "vivado.log").read_text()
        assert "PASS:" in log and "FAIL" not in log, log


@pytest.mark.parametrize("name", CASES)
def test_check_gqa_output_unchanged_passes(name, regression_run):
    res, out = regression_run
    golden = out / name / "vectors" / "gqa_golden.mem"
    actual = out / name / "sim" / "gqa_rtl_out.mem"
    assert actual.is_file(), res.stdout[-2000:]
    chk = subprocess.run([sys.executable, "-B", str(REF / "check_gqa_output.py"), "--golden", str(golden),
                          "--actual", str(actual), "--show-rows", "0"],
                         cwd=REF, text=True, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, timeout=120)
    assert chk.returncode == 0, chk.stdout
    assert "PASS: all 32 output rows (4096 BF16 values) matched golden within 64 ULP" in chk.stdout, chk.stdout
