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


# ---------------------------------------------------------------------------
# The same codec on the GPU (gqa_mem_decode / gqa_mem_encode): the text goes to
# the device once and is parsed there, so large vector files (K and V at long
# SEQ_LEN are hundreds of MB of hex) skip host-side parsing.
# ---------------------------------------------------------------------------

def _device(device):
    import torch
    if device is None:
        if not torch.cuda.is_available():
            raise RuntimeError("the GPU .mem codec needs a CUDA device (there is no CPU path)")
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device(device)


def decode_mem(data, elements: int, device=None):
    """``.mem`` text -> int16 tensor ``[rows, elements]`` of BF16 codes on the GPU.

    ``data`` is ``bytes`` (copied to the device) or a uint8 CUDA tensor.  Lines
    follow ``read_mem`` (gqa_reference.py:44-46 with unpack_bf16, :31-36): blank
    and ``//`` lines are skipped, ``_`` is ignored and every other line must hold
    exactly ``4 * elements`` hex digits, else ``ValueError`` names the line.
    """
    import torch
    from . import _lib
    lib = _lib.load()
    if not 1 <= elements <= _lib.MEM_MAX_ELEMENTS:
        raise ValueError(f"elements must be in [1, {_lib.MEM_MAX_ELEMENTS}]")
    if isinstance(data, torch.Tensor):
        text = data.reshape(-1)
        dev = text.device
        if text.dtype != torch.uint8 or dev.type != "cuda":
            raise TypeError("a tensor argument must be uint8 on a CUDA device")
        if text.data_ptr() % 16:
            text = text.clone()
    else:
        dev = _device(device)
        host = torch.frombuffer(bytearray(data), dtype=torch.uint8) if len(data) else torch.empty(0, dtype=torch.uint8)
        text = host.to(dev)
    n = text.numel()
    max_rows = n // (4 * elements)
    rows = torch.empty((max(max_rows, 1), elements), dtype=torch.int16, device=dev)
    result = torch.empty(2, dtype=torch.int64, device=dev)  # struct gqa_mem_result
    ws_bytes = lib.gqa_mem_decode_workspace_bytes(n)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        st = lib.gqa_mem_decode(text.data_ptr() if n else None, n, elements, rows.data_ptr(), max_rows,
                                result.data_ptr(), ws.data_ptr(), ws_bytes, stream)
    if st != _lib.GQA_OK:
        raise RuntimeError(f"gqa_mem_decode: {_lib.status_string(st)}")
    n_rows, bad = (int(x) for x in result.cpu())
    if bad != -1:  # UINT64_MAX read as int64
        # line ends as the parser reads them: '\n', '\r\n', or a '\r' alone
        head = text[:min(bad + 1, n)].cpu().numpy()
        nxt = np.append(head[1:bad + 1], 0)[:bad]
        line = int(((head[:bad] == 10) | ((head[:bad] == 13) & (nxt != 10))).sum()) + 1
        raise ValueError(f"line {line}: expected {4 * elements} hex digits (and '_'), "
                         f"surrounded by blanks only")
    if n_rows > max_rows:
        raise RuntimeError("gqa_mem_decode found more rows than the text can hold")
    return rows[:n_rows]


def encode_mem(rows, device=None) -> bytes:
    """int16/uint16 codes ``[rows, elements]`` -> the text ``write_mem`` writes, encoded on the GPU."""
    import torch
    from . import _lib
    lib = _lib.load()
    if isinstance(rows, np.ndarray):
        rows = torch.from_numpy(np.ascontiguousarray(rows, dtype=np.uint16).view(np.int16)).to(_device(device))
    if rows.dim() != 2 or rows.dtype not in (torch.int16, torch.bfloat16) or rows.device.type != "cuda":
        raise TypeError("rows must be a 2-D int16 or bfloat16 CUDA tensor")
    rows = rows.contiguous()
    n_rows, elements = rows.shape
    nbytes = lib.gqa_mem_encode_bytes(n_rows, elements)
    if n_rows and nbytes == 0:
        raise ValueError(f"elements must be in [1, {_lib.MEM_MAX_ELEMENTS}]")
    text = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=rows.device)
    with torch.cuda.device(rows.device):
        stream = torch.cuda.current_stream(rows.device).cuda_stream
        st = lib.gqa_mem_encode(rows.data_ptr(), n_rows, elements, text.data_ptr(), stream)
    if st != _lib.GQA_OK:
        raise RuntimeError(f"gqa_mem_encode: {_lib.status_string(st)}")
    return text[:nbytes].cpu().numpy().tobytes()


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
