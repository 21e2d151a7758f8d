"""Host-side logic of the C ABI and the Python API; runs without a GPU.

* the library loads and exports every function ``include/gqa_b200.h`` declares;
* ``gqa_validate`` rejects exactly what the RTL's ``config_error``
  (gqa_attention_wrapper.v:230-237) and the generator (gen_gqa_wrapper_vectors.py:57-78) reject;
* the ROM tables computed by the library are byte-identical to ``tools/gen_rope_rom.py``;
* the ``.mem`` codec matches the oracle's restatement of gqa_reference.py;
* the product package never imports the oracle and has no fallback when the library is absent.
"""
from __future__ import annotations

import ctypes
import os
import hashlib
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import attention_accelerator_b200 as gqa
from attention_accelerator_b200 import _lib, memfile
from attention_accelerator_b200.api import make_params
from conftest import GOLDEN, ROOT
from oracle.bf16 import mem_text, read_mem_array

HEADER = ROOT / "include" / "gqa_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gqa_\w+)\s*\(", text)))


def test_header_declarations_match_binding():
    assert declared_functions() == _lib.exported_symbols()


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    nm = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True)
    exported = set(re.findall(r"\bT (gqa_\w+)", nm.stdout))
    assert set(declared_functions()) <= exported


def test_status_codes_match_header():
    """Every GQA_ERR_* value of the header's enum is the binding's, and has its own message."""
    codes = dict((n, int(v)) for n, v in re.findall(r"\b(GQA_ERR_\w+)\s*=\s*(\d+)", HEADER.read_text()))
    assert codes and codes["GQA_ERR_MEMORY"] == 18
    for name, value in codes.items():
        assert getattr(_lib, name) == value, name
    messages = {_lib.status_string(v) for v in codes.values()}
    assert len(messages) == len(codes) and "unknown status" not in messages


def test_api_refuses_host_tensors_and_wrong_outputs_before_any_call():
    """Paths with no host-buffer support refuse CPU tensors, and a caller's ``out``
    must hold every row the kernel writes; both are checked in Python, before the
    library is called."""
    import torch
    from attention_accelerator_b200 import api
    q = torch.zeros((1, 2, 32, 128), dtype=torch.bfloat16)
    kv = torch.zeros((1, 64, 8, 128), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        gqa.decode_chunked(q, kv, kv, first_position=62)
    plan = gqa.plan_batch([64], device=torch.device("cpu"))
    with pytest.raises(ValueError, match="CUDA"):
        gqa.decode_batch(q[:, 0], kv[0], kv[0], plan)
    with pytest.raises(ValueError, match="CUDA"):
        gqa.combine_partials(torch.zeros((2, 1, 32, 132)))
    with pytest.raises(ValueError, match="CUDA"):
        gqa.rope_rows(torch.zeros((4, 128), dtype=torch.bfloat16), torch.arange(4))
    out = torch.empty((32, 128), dtype=torch.bfloat16)
    api._check_out(out, (32, 128), torch.bfloat16, torch.device("cpu"))
    for bad in (torch.empty((16, 128), dtype=torch.bfloat16), torch.empty((32, 128)),
                torch.empty((128, 32), dtype=torch.bfloat16).t()):
        with pytest.raises(ValueError, match="out must be"):
            api._check_out(bad, (32, 128), torch.bfloat16, torch.device("cpu"))


def test_bench_traffic_applies_only_to_the_captured_launch():
    import bench
    assert bench.traffic_for("config4_decode_s131072", 536887296) == 541605632
    assert bench.traffic_for("config4_decode_s131072", 536887296 / 4) is None  # a rank's shard at N=4
    assert bench.traffic_for("config3_ragged_b64", 1237770240) == 1257566976  # decode_queue_kernel
    assert bench.traffic_for("no_such_workload", 1.0) is None


def test_workspace_grows_without_freeing_the_old_buffer():
    """A larger call on the same stream gets a new workspace; the old one stays
    allocated (a captured CUDA graph may still address it) and is not reused."""
    import torch
    from attention_accelerator_b200 import api
    dev, stream = torch.device("cpu"), 0x5eed
    small = api._workspace(dev, stream, 100)
    assert api._workspace(dev, stream, 4096) is small  # fits: same buffer
    big = api._workspace(dev, stream, 1 << 16)
    assert big is not small and big.numel() >= 1 << 16 and int(big.sum()) == 0
    assert any(b is small for b in api._ws_retired)
    assert api._workspace(dev, stream, 100) is big
    del api._ws[(None, stream)]


_NULL_PROBE = r"""
import ctypes
import os
from attention_accelerator_b200 import _lib
lib = _lib.load()
def is_ptr(a):
    return issubclass(a, (ctypes._Pointer, ctypes.c_void_p, ctypes.c_char_p))
for name, (res, argtypes) in sorted(_lib._SIGNATURES.items()):
    if not any(is_ptr(a) for a in argtypes) or res not in (ctypes.c_int, ctypes.c_size_t):
        continue
    args = [None if is_ptr(a) else (1.0 if a in (ctypes.c_float, ctypes.c_double) else 1) for a in argtypes]
    print(name, getattr(lib, name)(*args), flush=True)
"""


def test_every_entry_point_refuses_null_pointers_without_crashing():
    """Each entry point that takes pointers, called with all of them NULL (sizes 1),
    returns an error status (or 0 bytes) before it touches CUDA or dereferences an
    argument -- in a child process, so a crash fails this test alone."""
    import sys
    res = subprocess.run([sys.executable, "-c", _NULL_PROBE], capture_output=True, text=True, cwd=ROOT, timeout=120)
    assert res.returncode == 0, res.stderr[-2000:]
    got = dict((ln.split()[0], int(ln.split()[1])) for ln in res.stdout.splitlines())
    sizes = {n for n, (r, _) in _lib._SIGNATURES.items() if r is ctypes.c_size_t}
    assert len(got) >= 20
    for name, value in got.items():
        if name in sizes:
            assert value == 0, name
        else:
            assert value == _lib.GQA_ERR_NULL_POINTER, (name, value, _lib.status_string(value))


def _host_plan(seq_len=None, seqs=None, sms=148):
    sp, kp = ctypes.c_int(), ctypes.c_int()
    lib = _lib.load()
    if seqs is None:
        p = make_params(seq_len=seq_len)
        st = lib.gqa_decode_plan_host(ctypes.byref(p), None, 1, sms, ctypes.byref(sp), ctypes.byref(kp))
    else:
        p = make_params(seq_len=1)
        arr = (_lib.GqaSeqDesc * len(seqs))()
        start = 0
        for i, n in enumerate(seqs):
            arr[i].kv_start, arr[i].seq_len, arr[i].query_position = start, n, n - 1
            arr[i].pos_begin, arr[i].pos_end = 0, n
            start += n
        st = lib.gqa_decode_plan_host(ctypes.byref(p), arr, len(seqs), sms, ctypes.byref(sp), ctypes.byref(kp))
    assert st == _lib.GQA_OK, _lib.status_string(st)
    return sp.value, kp.value


def test_host_planner_reproduces_the_grids_measured_on_b200():
    """The split planner, run without a GPU for 148 SMs, gives the splits ncu recorded
    on the B200 (8 per split, one per KV head): config 2 136 CTAs, config 4 144, config 3
    1088 (split, KV head) items (a batch runs them from a work queue on one CTA per SM)."""
    assert _host_plan(4096) == (17, 248)       # one head group of SMs left for the next call
    assert _host_plan(131072) == (18, 7288)
    seqs = [int(x) for x in np.random.default_rng(20260805).integers(512, 8193, size=64)]  # bench config 3
    assert sum(seqs) == 301934
    assert _host_plan(seqs=seqs) == (136, 2800)
    assert _host_plan(30) == (1, 88)


@pytest.mark.parametrize("sms", [1, 8, 132, 148, 160])
def test_host_planner_covers_every_key(sms):
    rng = np.random.default_rng(sms)
    for n in (1, 87, 88, 89, 4096, 65535, 131072):
        splits, chunk = _host_plan(n, sms=sms)
        assert chunk % 8 == 0 and 1 <= splits <= 64 and (splits - 1) * chunk < n <= splits * chunk
    seqs = [int(x) for x in rng.integers(1, 20000, size=37)]
    splits, chunk = _host_plan(seqs=seqs, sms=sms)
    assert splits == sum(-(-n // chunk) for n in seqs)


def test_host_planner_rejects_bad_arguments():
    lib = _lib.load()
    p = make_params(seq_len=100)
    sp, kp = ctypes.c_int(), ctypes.c_int()
    assert lib.gqa_decode_plan_host(ctypes.byref(p), None, 1, 0, ctypes.byref(sp), ctypes.byref(kp)) == _lib.GQA_ERR_BATCH
    assert lib.gqa_decode_plan_host(ctypes.byref(p), None, 2, 148, ctypes.byref(sp), ctypes.byref(kp)) == _lib.GQA_ERR_BATCH
    bad = make_params(seq_len=100, n_q_heads=31)
    assert lib.gqa_decode_plan_host(ctypes.byref(bad), None, 1, 148, ctypes.byref(sp), ctypes.byref(kp)) == \
        _lib.GQA_ERR_GEOMETRY


def test_header_compiles_as_plain_c(tmp_path):
    """include/gqa_b200.h is the boundary for C callers: a C99 translation unit that
    includes it and takes the address of every declared function compiles without
    warnings, and its struct sizes are the ones the Python binding uses."""
    import shutil
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    names = declared_functions()
    src = tmp_path / "abi.c"
    src.write_text("#include \"gqa_b200.h\"\n#include <stdio.h>\n"
                   "typedef void (*any_fn)(void);\n"
                   "static const any_fn fns[] = {\n"
                   + "".join(f"    (any_fn)&{n},\n" for n in names) + "};\n"
                   "int main(void) {\n"
                   "    printf(\"%zu %zu %zu %zu\\n\", sizeof(gqa_params), sizeof(gqa_seq_desc),\n"
                   "           sizeof(gqa_partial_row), sizeof(fns) / sizeof(fns[0]));\n"
                   "    return GQA_OK;\n}\n")
    exe = tmp_path / "abi"
    res = subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", str(ROOT / "include"),
                          str(src), "-o", str(exe), "-Wl,--unresolved-symbols=ignore-all"],
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    assert [int(x) for x in out] == [ctypes.sizeof(_lib.GqaParams), ctypes.sizeof(_lib.GqaSeqDesc), 132 * 4,
                                     len(names)]


def test_struct_layouts():
    assert ctypes.sizeof(_lib.GqaSeqDesc) == 24
    assert ctypes.sizeof(_lib.GqaParams) == 12 * 4 + 8 * 8 + 8 + 8


def _validate(**kw) -> int:
    p = make_params(**kw)
    return _lib.load().gqa_validate(ctypes.byref(p))


@pytest.mark.parametrize("kw,status", [
    (dict(seq_len=30), _lib.GQA_OK),
    (dict(seq_len=30, n_q_heads=31), _lib.GQA_ERR_GEOMETRY),      # tb_gqa_attention_wrapper.sv:323
    (dict(seq_len=30, n_kv_heads=7), _lib.GQA_ERR_GEOMETRY),
    (dict(seq_len=30, head_dim=64), _lib.GQA_ERR_GEOMETRY),
    (dict(seq_len=30, tile_dim=8), _lib.GQA_ERR_GEOMETRY),
    (dict(seq_len=0, n_kv_tiles=0), _lib.GQA_ERR_SEQ_LEN),
    (dict(seq_len=30, n_kv_tiles=3), _lib.GQA_ERR_N_KV_TILES),
    (dict(seq_len=30, n_kv_tiles=1), _lib.GQA_ERR_N_KV_TILES),
    (dict(seq_len=32, n_kv_tiles=2), _lib.GQA_OK),
    (dict(seq_len=33, n_kv_tiles=2), _lib.GQA_ERR_N_KV_TILES),
    (dict(seq_len=17, kv_block_len=4, n_kv_tiles=5), _lib.GQA_OK),
    (dict(seq_len=30, scale=0.0), _lib.GQA_ERR_SCALE),
    (dict(seq_len=30, scale=float("nan")), _lib.GQA_ERR_SCALE),
    (dict(seq_len=30, query_position=30), _lib.GQA_ERR_QUERY_POSITION),
    (dict(seq_len=30, query_position=0), _lib.GQA_OK),
    (dict(seq_len=30, kv_block_len=0, n_kv_tiles=0), _lib.GQA_ERR_KV_BLOCK_LEN),
    (dict(seq_len=30, group_size=2), _lib.GQA_ERR_GROUP_SIZE),
    (dict(seq_len=30, rope_theta=0.0), _lib.GQA_ERR_ROPE_THETA),
    (dict(seq_len=131072), _lib.GQA_OK),
])
def test_validate_mirrors_config_error(kw, status):
    assert _validate(**kw) == status


def test_api_raises_config_error_without_gpu():
    with pytest.raises(gqa.GqaConfigError):
        gqa.validate(seq_len=30, n_q_heads=31)
    import torch
    q = torch.zeros((32, 128), dtype=torch.bfloat16)
    k = torch.zeros((30, 8, 128), dtype=torch.bfloat16)
    with pytest.raises(gqa.GqaConfigError):
        gqa.decode(q, k, k, seq_len=30, query_position=30)


def test_decode_rejects_bad_pointers_before_launch():
    lib = _lib.load()
    p = make_params(seq_len=30)
    assert lib.gqa_decode(None, None, None, None, ctypes.byref(p), None, 0, None) == _lib.GQA_ERR_NULL_POINTER
    p.q_head_stride = 128
    p.k_pos_stride = p.v_pos_stride = 1024
    p.k_head_stride = p.v_head_stride = 128
    assert lib.gqa_decode(8, 16, 16, 16, ctypes.byref(p), None, 0, None) == _lib.GQA_ERR_ALIGNMENT
    p.k_pos_stride = 1001
    assert lib.gqa_decode(16, 16, 16, 16, ctypes.byref(p), None, 0, None) == _lib.GQA_ERR_ALIGNMENT


@pytest.mark.parametrize("bits", [10, 14])
def test_library_rom_tables_match_reference(bits, manifest):
    phase = gqa.rope_phase_rom()
    sincos = gqa.rope_sincos_rom(bits)
    phase_text = "".join(f"{p:08x}\n" for p in phase)
    sincos_text = "".join(f"{s:08x}\n" for s in sincos)
    want = manifest["rope_rom"][f"tools_bits{bits}"]
    assert hashlib.sha256(phase_text.encode()).hexdigest() == want["rope_phase_rom.mem"]
    assert hashlib.sha256(sincos_text.encode()).hexdigest() == want["rope_sincos_rom.mem"]


def test_mem_codec_matches_oracle():
    rng = np.random.default_rng(0)
    rows = rng.integers(0, 1 << 16, size=(37, 16), dtype=np.uint16)
    text = memfile.format_mem_text(rows)
    assert text == mem_text(rows.tolist())
    np.testing.assert_array_equal(memfile.parse_mem_text(text, 16), rows)
    golden_path = GOLDEN / "cases" / "random_len30" / "gqa_golden.mem"
    np.testing.assert_array_equal(memfile.read_mem(golden_path, 128), read_mem_array(golden_path, 128))


def test_mem_compare_rule():
    g = np.full((1, 128), 0x3F80, dtype=np.uint16)
    a = g.copy()
    a[0, 0] += 64
    assert memfile.compare_rows(g, a, 64)["failures"] == 0
    a[0, 0] += 1
    assert memfile.compare_rows(g, a, 64)["failures"] == 1


def test_product_never_imports_the_oracle():
    pkg = ROOT / "attention_accelerator_b200"
    for path in list(pkg.rglob("*.py")) + [pkg / "bin" / "vivado"]:
        text = path.read_text()
        assert not re.search(r"^\s*(from|import)\s+oracle\b", text, re.M), path


def test_no_fallback_when_library_missing(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "missing.so")
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(RuntimeError, match="missing"):
        _lib.load()


def test_plan_batch_descriptors_on_host():
    plan = gqa.plan_batch([5, 9, 1], query_positions=[4, 3, 0], device=__import__("torch").device("cpu"))
    assert [d.kv_start for d in plan.host] == [0, 5, 14]
    assert [d.pos_end for d in plan.host] == [5, 9, 1]
    assert plan.device.numel() == 3 * 24


def test_bench_parallel_read_mem_uses_every_core():
    """The reference arm's .mem leg: read_mem on one spawned process per host core."""
    import bench
    value, cores, sample = bench.mem_cpu_run_parallel(0.2, lines_per_proc=512)
    assert value > 0 and cores == min(64, os.cpu_count() or 1) and f"{cores} pieces" in sample


def test_bench_cpu_baseline_reports_all_cores_and_one_core():
    """Our arm's cpu_baseline for a workload without oracle inputs (configs 3 and 4):
    the float64 port on a config-2-sized sample, on all cores and on one."""
    import bench

    class Sampled:
        def oracle_inputs(self):
            return None

    out = bench.cpu_baseline(Sampled(), budget_s=0.3)
    assert out["kind"] == "port" and out["value"] > 0 and out["cores"] == (os.cpu_count() or 1)
    assert out["one_core"]["cores"] == 1 and out["one_core"]["value"] > 0


def test_bench_chunked_cpu_run_is_bounded():
    """config 5's CPU leg: whole sequences of the float64 chunked restatement, at
    least one, stopping at the budget."""
    import bench
    reps, dt = bench.chunked_cpu_run(0.05, n_keys=256)
    assert reps >= 1 and dt > 0


def test_bench_reference_arm_json_line():
    """`bench.py --impl reference` (the reference algorithm on the host cores) prints one
    JSON line with the contract's keys; config 1 keeps it to a few seconds."""
    import json
    import sys
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "config1", "--steps", "2",
                          "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads([ln for ln in res.stdout.splitlines() if ln.startswith("{")][-1])
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["metric"].startswith("decode-attn KV-read HBM GB/s")
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    one = line["cpu_baseline"]["one_core"]  # the single-core figure beside the all-cores one
    assert one["cores"] == 1 and one["value"] > 0
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_bench_output_check_counts_ulps_like_the_reference():
    """bench.compare_outputs: BF16 code distance across zero, the 64-ULP count, the
    bar on large outputs (<= 2 ULP where |x| >= 2^-10 of the row's largest), and
    cancellation residues (below 2^-18 of the row's largest, the two values within
    2^-19 of it) counted apart from failures."""
    import torch
    import bench
    want = torch.zeros((2, 128), dtype=torch.bfloat16)
    want[0, :] = 1.0
    want[1, 0] = 4.0
    want[1, 1] = 2.0 ** -20                      # tiny next to 4.0: not a large output
    got = want.clone()
    res = bench.compare_outputs(got, want, "same")
    assert res["ok"] and res["max_ulp"] == 0 and res["beyond_64_ulp"] == 0
    got[0, 5] = torch.tensor(1.0).to(torch.bfloat16).view(torch.int16).add(2).view(torch.bfloat16)  # +2 ULP
    assert bench.compare_outputs(got, want, "x")["ok"]
    got[0, 6] = torch.tensor(1.0).to(torch.bfloat16).view(torch.int16).add(3).view(torch.bfloat16)  # +3 ULP
    res = bench.compare_outputs(got, want, "x")
    assert not res["ok"] and res["max_ulp_large_outputs"] == 3
    got = want.clone()
    got[1, 1] = -got[1, 1]                        # sign flip of a residue: far beyond 64 codes, 2^-19 apart
    res = bench.compare_outputs(got, want, "x")
    assert res["ok"] and res["beyond_64_ulp"] == 0 and res["residues_beyond_64_ulp"] == 1
    got[1, 1] = 2.0 ** -14                        # a residue, but the values are 2^-16 of the row max apart
    res = bench.compare_outputs(got, want, "x")
    assert not res["ok"] and res["beyond_64_ulp"] == 1 and res["max_ulp_large_outputs"] == 0
    want[1, 2] = 2.0 ** -12                       # not a residue (2^-14 of the row max)
    got = want.clone()
    got[1, 2] = -got[1, 2]
    res = bench.compare_outputs(got, want, "x")
    assert not res["ok"] and res["beyond_64_ulp"] == 1 and res["residues_beyond_64_ulp"] == 0


def test_decode_heads_refuses_bad_head_ranges_before_any_gpu_work():
    """gqa_decode_heads checks the KV-head range on the host (GQA_ERR_KV_HEADS),
    after the register checks and before touching any pointer or device."""
    import ctypes
    from attention_accelerator_b200.api import make_params
    lib = _lib.load()
    p = make_params(seq_len=64)
    for begin, count in ((0, 0), (-1, 2), (7, 2), (0, 9), (8, 1)):
        st = lib.gqa_decode_heads(None, None, None, None, ctypes.byref(p), begin, count, None, 0, None)
        assert st == _lib.GQA_ERR_KV_HEADS, (begin, count, st)
    bad = make_params(seq_len=64, n_q_heads=31)
    assert lib.gqa_decode_heads(None, None, None, None, ctypes.byref(bad), 0, 1, None, 0, None) == _lib.GQA_ERR_GEOMETRY
    assert lib.gqa_workspace_bytes_heads(ctypes.byref(p), 0) == 0
