"""Drop-in for the ``$VIVADO`` executable that ``pyfiles/run_gqa_regression.py`` runs.

The regression driver calls ``$VIVADO -mode batch -source
scripts/run_gqa_wrapper_sim.tcl`` (run_gqa_regression.py:36,57,70) with
``VECTORS_DIR`` and ``SIM_BUILD_DIR`` in the environment, optionally
``OUTPUT_BACKPRESSURE`` or ``INVALID_CONFIG``, and passes a case when the exit
status is 0 and stdout contains ``PASS:`` (:59, :72).  This program keeps that
contract with the B200 library in place of the XSim testbench:

* reads ``gqa_{q,k,v,golden}.mem`` and ``gqa_config.txt`` from VECTORS_DIR
  (run_gqa_wrapper_sim.tcl:13-27), parsing the hex text on the GPU
  (``gqa_mem_decode``);
* programs the registers as the testbench does (tb_gqa_attention_wrapper.sv:323-329),
  taking QUERY_POSITION and KV_BLOCK_LEN from the config, and the exact
  1/sqrt(128) scale of the golden;
* runs one decode through ``gqa_decode`` on the GPU, writes the rows to
  ``SIM_BUILD_DIR/gqa_rtl_out.mem`` (one 128-element row per line, the
  testbench's ``$fdisplay`` format), checks every element against the golden
  with the checker's rule (<= MAX_ULP, default 64, with the 0x3d exponent
  exemption) and prints ``PASS:``/``FAIL:``;
* with INVALID_CONFIG, programs N_Q_HEADS=31 (tb :323) and passes only if the
  library rejects the start (tb :330-336).
OUTPUT_BACKPRESSURE only throttles the RTL's AXIS egress; it has no GPU meaning
and is accepted and ignored.  With GQA_RTL_NUMERICS=1 the decode reproduces the
RTL's RoPE (ROM NCO, BF16 units) and BF16 scale register (``rtl_numerics``), so
``gqa_rtl_out.mem`` approximates what the RTL testbench would write; the check
against the golden then reports those quantisations as the RTL would show them.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np


def _fail(msg: str, code: int = 1) -> int:
    print(f"ERROR: {msg}")
    return code


def main(argv: list[str] | None = None) -> int:
    from . import _lib
    from .api import GqaConfigError, GqaError, make_params
    from .memfile import compare_rows, decode_mem, encode_mem, read_config

    vectors = Path(os.environ.get("VECTORS_DIR") or "tests/data").resolve()
    build = Path(os.environ.get("SIM_BUILD_DIR") or "build/gqa_wrapper_sim").resolve()
    max_ulp = int(os.environ.get("MAX_ULP", "64"))
    for req in ("gqa_q.mem", "gqa_k.mem", "gqa_v.mem", "gqa_golden.mem"):
        if not (vectors / req).is_file():
            return _fail(f"Missing {vectors / req}.")
    if not (vectors / "gqa_config.txt").is_file():
        return _fail(f"Missing {vectors / 'gqa_config.txt'}.")
    cfg = read_config(vectors / "gqa_config.txt")
    if "SEQ_LEN" not in cfg:
        return _fail("SEQ_LEN missing from gqa_config.txt")
    try:
        seq_len = int(cfg["SEQ_LEN"])
        kv_block_len = int(cfg.get("KV_BLOCK_LEN", 16))
        qpos = int(cfg.get("QUERY_POSITION", seq_len - 1))
    except ValueError as exc:
        return _fail(f"gqa_config.txt: {exc}")
    build.mkdir(parents=True, exist_ok=True)
    out_path = build / "gqa_rtl_out.mem"

    if os.environ.get("INVALID_CONFIG"):
        # N_Q_HEADS = 31 with everything else as in the testbench, then START.
        p = make_params(seq_len=seq_len, query_position=qpos, kv_block_len=kv_block_len, n_q_heads=31)
        lib = _lib.load()
        import ctypes
        status = lib.gqa_decode(None, None, None, None, ctypes.byref(p), None, 0, None)
        out_path.write_text("")
        if status in _lib.CONFIG_ERRORS:
            print(f"config_error: {_lib.status_string(status)}")
            print("PASS: invalid configuration rejected")
            return 0
        print(f"FAIL: invalid configuration was not rejected (status {status})")
        return 1

    import torch
    from .api import decode
    if not torch.cuda.is_available():
        return _fail("no CUDA device: the B200 library has no CPU path")
    dev = torch.device("cuda", torch.cuda.current_device())

    def load(name, elements):  # the .mem text is parsed on the GPU
        try:
            return decode_mem((vectors / name).read_bytes(), elements, dev)
        except ValueError as exc:
            raise SystemExit(_fail(f"{vectors / name}: {exc}"))

    q, k, v = (load(f"gqa_{n}.mem", 16).view(torch.bfloat16) for n in "qkv")
    # transport beats of 16 elements: Q is 32 rows of 128, K and V are 8 heads x rows x 128
    if q.numel() != 32 * 128:
        return _fail(f"gqa_q.mem holds {q.numel()} elements, expected {32 * 128}")
    for name, t in (("gqa_k.mem", k), ("gqa_v.mem", v)):
        if t.numel() == 0 or t.numel() % (8 * 128):
            return _fail(f"{name} holds {t.numel()} elements, not a whole number of 8 x 128-element rows")
    q, k, v = q.reshape(32, 128), k.reshape(8, -1, 128), v.reshape(8, -1, 128)
    golden = load("gqa_golden.mem", 128).cpu().numpy().view(np.uint16)
    try:
        out = decode(q, k, v, seq_len=seq_len, query_position=qpos, kv_block_len=kv_block_len, layout="head_major",
                     rtl_numerics=os.environ.get("GQA_RTL_NUMERICS", "0") not in ("", "0"))
    except GqaConfigError as exc:
        print(f"FAIL: configuration rejected: {exc}")
        return 1
    except ValueError as exc:  # e.g. fewer stored K/V rows than SEQ_LEN
        return _fail(str(exc))
    except GqaError as exc:  # the library refused the call for another reason
        return _fail(str(exc))
    out_rows = out.view(torch.int16)
    out_path.write_bytes(encode_mem(out_rows))  # the testbench's row format, encoded on the GPU
    rows = out_rows.cpu().numpy().view(np.uint16)
    if golden.shape != rows.shape:
        print(f"FAIL: golden has {golden.shape[0]} rows, output has {rows.shape[0]}")
        return 1
    res = compare_rows(golden, rows, max_ulp)
    if res["failures"]:
        print(f"FAIL: {res['failures']} elements exceeded {max_ulp} ULP; worst={res['worst']} "
              f"at row={res['worst_row']}, col={res['worst_col']}")
        return 1
    print(f"PASS: {rows.shape[0]} GQA output rows matched golden within {max_ulp} ULP "
          f"(worst ULP={res['worst']} at row={res['worst_row']}, col={res['worst_col']}; "
          f"mean ULP={res['mean']:.4f}); output {out_path}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
