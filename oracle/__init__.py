"""CPU oracle for the GQA decode-attention hot path.

TEST INFRASTRUCTURE ONLY.  This package is a restatement of the reference's
Python golden model (``pyfiles/gen_gqa_wrapper_vectors.py``,
``pyfiles/gqa_reference.py``, ``pyfiles/check_gqa_output.py``,
``tools/gen_rope_rom.py``) in numpy float64.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg (plus its
``--impl reference`` arm) may import it, and only as the checker or as the
timed CPU baseline.  The product path in ``attention_accelerator_b200`` never
imports it and has no CPU fallback.

Parity pinning: every function here is checked byte-for-byte against files the
reference's own scripts wrote in the build container (sha256 digests and
golden ``.mem`` rows under ``tests/golden/``, produced by
``tests/golden/make_golden.py``).
"""

from .bf16 import (bf16_to_f32, f32_to_bf16, pack_bf16, read_mem, read_mem_array,
                   ulp_distance, unpack_bf16, write_mem)
from .golden import gqa_golden, gqa_golden_f64, rope_half_split, rope_inv_freq
from .chunked import chunked_golden, chunked_golden_f64
from .vectors import ReferenceCase, generate_case
from .checker import check_rows
from .rope_rom import rope_phase_rom, rope_sincos_rom

__all__ = [
    "bf16_to_f32", "f32_to_bf16", "pack_bf16", "unpack_bf16", "read_mem", "read_mem_array",
    "write_mem", "ulp_distance", "gqa_golden", "gqa_golden_f64", "rope_half_split",
    "rope_inv_freq", "ReferenceCase", "generate_case", "check_rows", "rope_phase_rom",
    "rope_sincos_rom", "chunked_golden", "chunked_golden_f64",
]
