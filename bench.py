#!/usr/bin/env python3
"""Benchmark of the GQA decode-attention hot path (BASELINE metric: decode-attn
KV-read HBM GB/s, % of the measured HBM peak, and query-heads/s, at 1/2/4/8 B200).

One step = one pass of the hot path over one batch of synthetic input:
  config4 (default): one single-token decode, SEQ_LEN=131072, QUERY_POSITION=131071,
                     position-major BF16 KV cache [131072, 8, 128] -- the largest
                     single-sequence BASELINE configuration; at N>1 GPUs the
                     sequence is split into contiguous shards whose (m, l, O) rows
                     are exchanged over NVLink peer memory inside the decode kernel
                     and merged by log-sum-exp (strong scaling; --exchange nccl: an
                     NCCL all-gather + combine kernel instead).
  config2:           SEQ_LEN=4096, QUERY_POSITION=4095 (one sequence per GPU).
  config1:           SEQ_LEN=30, QUERY_POSITION=29, KV_BLOCK_LEN=16, U[-1,1) inputs.
  config3:           batch 64, SEQ_LEN ~ U{512..8192}, K with log-normal channel scales.
  config5:           chunked multi-query decode on the tensor cores: batch 16,
                     SEQ_LEN=8192, queries 8064..8191 per sequence (causal); the 16
                     sequences are split across ranks (strong scaling).  Its roofline
                     line is tensor-bound (algorithmic FLOPs / measured BF16 peak).
Configs 1-3 shard by sequence: every rank decodes its own sequences, no
collective (weak scaling).

Timing: K steps replayed from CUDA graphs on one stream between CUDA events,
after W warm-up steps, barrier + synchronize on both sides, max over ranks.
Inputs rotate over buffer sets whose total exceeds twice the L2 size, so every
step reads K/V from HBM.  After timing, every rank checks the output of the last
timed step against an independent decode of the same inputs (``check`` in the
JSON line): another split plan and merge on the same GPU, and for the sequence
split a single-GPU decode of the whole sequence.  ``--impl reference`` times the CPU restatement of the
reference golden (the reference itself is Python that cannot run on the GPU box)
on all host threads.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode-attn KV-read HBM GB/s (% of peak) + query-heads/sec at 1/2/4/8 B200"
UNIT = "GB/s"
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 1024 * 1024
HEAD_BYTES = 32 * 128 * 2


def kv_bytes(n_keys: int) -> int:
    """Algorithmic bytes of one sequence's decode: K+V rows of the visible keys, Q and out."""
    return 2 * n_keys * 8 * 128 * 2 + 2 * HEAD_BYTES


def _ordered(codes):
    """BF16 codes as integers that order like the values (sign-magnitude to two's complement)."""
    import numpy as np
    c = np.asarray(codes).astype(np.int64) & 0xFFFF
    return np.where(c & 0x8000, 0x8000 - c, c)


def compare_outputs(got, want, what: str) -> dict:
    """BF16 outputs of the timed steps (`got`) against an independent decode of the
    same inputs (`want`), rows of 128: per-element code distance, the count beyond
    the reference's 64-ULP limit, and the worst distance where the output is at
    least 2^-10 of its row's largest magnitude.  Two FP32 computations that sum
    in different orders (another split plan) may differ by more than 64 ULP on a
    cancellation residue, an output far below its row's largest: such an output
    (below 2^-18 of the row's largest, the two values within 2^-19 of it, twice
    the per-result error bound the parity tests allow against the float64 oracle)
    is counted as a residue, not a failure.
    ok: none beyond 64 ULP but residues, <= 2 ULP on the large outputs."""
    import numpy as np
    import torch
    g = got.detach().reshape(-1, 128).contiguous().view(torch.int16).cpu().numpy()
    w = want.detach().reshape(-1, 128).contiguous().view(torch.int16).cpu().numpy()
    dist = np.abs(_ordered(g) - _ordered(w))
    wv = want.detach().reshape(-1, 128).float().cpu().numpy()
    gv = got.detach().reshape(-1, 128).float().cpu().numpy()
    mag = np.abs(wv)
    rowmax = mag.max(axis=1, keepdims=True)
    big = mag >= np.ldexp(rowmax, -10)
    over = dist > 64
    residue = over & (mag < np.ldexp(rowmax, -18)) & (np.abs(gv - wv) <= np.ldexp(rowmax, -19))
    beyond = int((over & ~residue).sum())
    large = int(dist[big].max(initial=0))
    worst_rel = float((np.abs(gv - wv)[over] / np.broadcast_to(rowmax, dist.shape)[over]).max(initial=0.0))
    return {"ok": beyond == 0 and large <= 2 and bool(np.isfinite(mag).all()), "against": what,
            "outputs": int(dist.size), "max_ulp": int(dist.max(initial=0)), "max_ulp_large_outputs": large,
            "beyond_64_ulp": beyond, "residues_beyond_64_ulp": int(residue.sum()),
            "worst_abs_diff_beyond_64_of_row_max": worst_rel, "mean_ulp": round(float(dist.mean()), 5)}


def peak_bf16():
    """Dense BF16 tensor peak: the measured burst figure (a kernel timed alone)."""
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["bf16_tflops"]), "measured burst"
    except (OSError, ValueError, KeyError):
        return 1590.0, "fallback"


def peak_hbm():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples taken while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,clocks.mem")

    def __init__(self, gpu_index: int):
        self.rows, self.window = [], None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.monotonic(), [x.strip() for x in line.split(",")]))

    def mark(self, start: float, end: float):
        self.window = (start, end)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = self.rows
        if self.window:
            inside = [r for t, r in rows if self.window[0] - 0.06 <= t <= self.window[1] + 0.06]
            rows = inside if inside else [r for _, r in rows]
        else:
            rows = [r for _, r in rows]
        sm = [float(r[1]) for r in rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows if len(r) > 8 for n, v in zip(names, r[5:9]) if v == "Active"})
        mem = [float(r[9]) for r in rows if len(r) > 9 and r[9].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "mem_mhz": statistics.median(mem) if mem else None, "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
class Workload:
    name = ""
    scaling = "weak"
    k_rotated = False  # --k-rotated: K stored pre-rotated (GQA_FLAG_K_ROTATED), only Q rotated per call
    launches_per_step = 1
    graph_ok = False  # multi-launch steps under torch.distributed: graphs only without collectives

    def close(self):
        pass
    bound = "hbm"
    flops_per_step = 0

    def launch(self, i: int):
        raise NotImplementedError

    @property
    def sets(self) -> int:
        return 1


def split_reference(gqa, torch, q, k, v, seq_len, qpos, layout="position_major", k_rotated=False, shards=2):
    """One sequence decoded as `shards` contiguous key ranges (FP32 partial rows
    of decode_batch) merged by combine_partials: a different split plan and
    merge from a single decode call, for checking its output."""
    dev = q.device
    n = qpos + 1
    bounds = [round(i * n / shards) for i in range(shards + 1)]
    parts = []
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        plan = gqa.plan_batch([seq_len], query_positions=[qpos], pos_begin=[lo], pos_end=[hi], kv_starts=[0],
                              partial=True, device=dev)
        kk = k[lo:hi] if layout == "position_major" else k[:, lo:hi].transpose(0, 1)
        vv = v[lo:hi] if layout == "position_major" else v[:, lo:hi].transpose(0, 1)
        parts.append(gqa.decode_batch(q.reshape(1, 32, 128), kk.contiguous(), vv.contiguous(), plan,
                                      k_rotated=k_rotated))
    return gqa.combine_partials(torch.stack(parts))[0]


class SingleDecode(Workload):
    """One sequence per step per GPU; rotating buffer sets beat the L2."""

    def __init__(self, device, rank, seq_len, qpos, uniform=False, seed=20260805, layout="position_major"):
        import torch
        import attention_accelerator_b200 as gqa
        self.gqa, self.torch = gqa, torch
        self.S, self.qpos = seq_len, qpos
        self.name = f"config1_decode_s{seq_len}" if uniform else f"config2_decode_s{seq_len}"
        self.bytes_per_step = kv_bytes(qpos + 1)
        self.qheads_per_step = 32
        per_set = 2 * seq_len * 8 * 128 * 2
        self.nsets = max(2, math.ceil(2 * L2_BYTES / per_set)) if per_set < 2 * L2_BYTES else 2
        self.nsets = min(self.nsets, 64)
        g = torch.Generator(device=device).manual_seed(seed + 7919 * rank)

        def rnd(shape):
            if uniform:
                return (torch.rand(shape, generator=g, device=device) * 2 - 1).to(torch.bfloat16)
            return torch.randn(shape, generator=g, device=device).to(torch.bfloat16)

        self.layout = layout
        kv_shape = (seq_len, 8, 128) if layout == "position_major" else (8, seq_len, 128)
        self.q = [rnd((32, 128)) for _ in range(self.nsets)]
        self.k = [rnd(kv_shape) for _ in range(self.nsets)]
        self.v = [rnd(kv_shape) for _ in range(self.nsets)]
        self.out = torch.empty((32, 128), dtype=torch.bfloat16, device=device)
        self.l2_note = (f"{self.nsets} rotating buffer sets of {per_set / 2**20:.1f} MiB "
                        f"({self.nsets * per_set / 2**20:.0f} MiB > 2x L2)")

    @property
    def sets(self):
        return self.nsets

    def launch(self, i):
        j = i % self.nsets
        self.gqa.decode(self.q[j], self.k[j], self.v[j], seq_len=self.S, query_position=self.qpos, out=self.out,
                        layout=self.layout, k_rotated=self.k_rotated)

    def config(self):
        lay = "position_major [S,8,128]" if self.layout == "position_major" else "head_major [8,S,128]"
        sp = self.gqa.decode_plan(self.S, query_position=self.qpos)
        merge = (f"in-cluster merge, clusters of {sp.cluster}" if sp.cluster else
                 "last-split merge" if sp.splits > 1 else "none")
        return {"workload": self.name, "batch_per_gpu": 1, "seq_len": self.S, "query_position": self.qpos,
                "kv_block_len": 16, "kv_layout": f"{lay} bf16", "l2": self.l2_note,
                "splits": f"{sp.splits} x {sp.keys_per_split} keys x 8 KV heads ({merge})"}

    def check(self, steps: int) -> dict:
        """The last timed step's output against the same inputs decoded as two
        key shards (FP32 partials of decode_batch) merged by combine_partials."""
        j = (steps - 1) % self.nsets
        return compare_outputs(self.out, split_reference(self.gqa, self.torch, self.q[j], self.k[j], self.v[j],
                                                         self.S, self.qpos, self.layout, self.k_rotated),
                               "2 key shards (decode_batch partials) + combine_partials, same inputs")

    def e2e_inputs(self):
        t = self.torch
        return [x.cpu().pin_memory() for x in (self.q[0], self.k[0], self.v[0])]

    def e2e_step(self, host):
        q, k, v = host
        return self.gqa.decode(q, k, v, seq_len=self.S, query_position=self.qpos, layout=self.layout,
                               k_rotated=self.k_rotated)

    def oracle_inputs(self):
        """Head-major BF16 codes of buffer set 0 for the CPU restatement."""
        import numpy as np
        t = self.torch

        def bits(x):
            return x.contiguous().view(t.int16).cpu().numpy().astype(np.uint16)
        k, v = self.k[0], self.v[0]
        if self.layout == "position_major":
            k, v = k.transpose(0, 1), v.transpose(0, 1)
        return bits(self.q[0]), bits(k), bits(v), self.S, self.qpos

    def gpu_result_set0(self):
        import numpy as np
        if self.k_rotated:  # the oracle port below rotates K per call
            return None
        self.launch(0)
        self.torch.cuda.synchronize()
        return self.out.view(self.torch.int16).cpu().numpy().astype(np.uint16)


class HeadShardDecode(Workload):
    """`--shard heads`: one config-1/2 sequence per step with its 8 KV heads
    sharded over the ranks (distributed.head_range): every rank holds the K/V
    rows of its heads only and decodes them with decode_heads, no collective.
    Strong scaling (one sequence per step for the whole job)."""

    def __init__(self, device, rank, world, seq_len, qpos, seed=20260805):
        import torch
        import attention_accelerator_b200 as gqa
        from attention_accelerator_b200.distributed import head_range
        self.gqa, self.torch = gqa, torch
        self.S, self.qpos = seq_len, qpos
        self.world = world
        self.begin, self.count = head_range(rank, world)
        self.name = f"config2_heads_s{seq_len}"
        self.scaling = "strong"
        self.bytes_per_step = kv_bytes(qpos + 1)  # the whole sequence, all ranks together
        self.qheads_per_step = 32
        per_set = 2 * seq_len * self.count * 128 * 2
        self.nsets = max(2, math.ceil(2 * L2_BYTES / per_set))
        g = torch.Generator(device=device).manual_seed(seed)  # the same sequences on every rank
        self.q, self.kfull, self.vfull, self.k, self.v = [], [], [], [], []
        b, c = self.begin, self.count
        for _ in range(self.nsets):
            self.q.append(torch.randn((32, 128), generator=g, device=device).to(torch.bfloat16))
            kf = torch.randn((seq_len, 8, 128), generator=g, device=device).to(torch.bfloat16)
            vf = torch.randn((seq_len, 8, 128), generator=g, device=device).to(torch.bfloat16)
            self.k.append(kf[:, b:b + c].contiguous())
            self.v.append(vf[:, b:b + c].contiguous())
            self.kfull.append(kf)
            self.vfull.append(vf)
        self.out = torch.zeros((32, 128), dtype=torch.bfloat16, device=device)
        self.graph_ok = True
        # decode_kernel, plus split_merge_kernel when a head's splits exceed the in-kernel merge
        self.launches_per_step = 1
        self.l2_note = (f"{self.nsets} rotating buffer sets of {per_set / 2**20:.1f} MiB per rank "
                        f"({self.nsets * per_set / 2**20:.0f} MiB > 2x L2)")

    @property
    def sets(self):
        return self.nsets

    def launch(self, i):
        j = i % self.nsets
        self.gqa.decode_heads(self.q[j], self.k[j], self.v[j], kv_heads=(self.begin, self.count), seq_len=self.S,
                              query_position=self.qpos, out=self.out, k_rotated=self.k_rotated)

    def check(self, steps: int) -> dict:
        """This rank's rows of the last timed step against a single-GPU decode of
        the whole sequence (all 8 heads) on this rank."""
        j = (steps - 1) % self.nsets
        want = self.gqa.decode(self.q[j], self.kfull[j], self.vfull[j], seq_len=self.S, query_position=self.qpos,
                               k_rotated=self.k_rotated)
        rows = slice(4 * self.begin, 4 * (self.begin + self.count))
        return compare_outputs(self.out[rows], want[rows],
                               "single-GPU decode of the whole sequence (this rank's heads' rows)")

    def config(self):
        return {"workload": self.name, "batch": 1, "seq_len": self.S, "query_position": self.qpos,
                "kv_layout": f"position_major [S,{self.count},128] bf16: KV heads {self.begin}.."
                             f"{self.begin + self.count - 1} on this rank",
                "parallelism": f"KV-head sharding x{self.world} (decode_heads, no collective)",
                "l2": self.l2_note}

    def e2e_inputs(self):
        return [x.cpu().pin_memory() for x in (self.q[0], self.k[0], self.v[0])]

    def e2e_step(self, host):
        dev = self.out.device
        q, k, v = (x.to(dev, non_blocking=True) for x in host)
        return self.gqa.decode_heads(q, k, v, kv_heads=(self.begin, self.count), seq_len=self.S,
                                     query_position=self.qpos, k_rotated=self.k_rotated).cpu()

    def oracle_inputs(self):
        return None

    def gpu_result_set0(self):
        return None


class RaggedBatch(Workload):
    """64 sequences, SEQ_LEN ~ U{512..8192}, K with outlier channels."""

    def __init__(self, device, rank, batch=64, seed=20260805):
        import numpy as np
        import torch
        import attention_accelerator_b200 as gqa
        self.gqa, self.torch = gqa, torch
        rng = np.random.default_rng(seed + rank)
        self.seq = [int(x) for x in rng.integers(512, 8193, size=batch)]
        self.batch = batch
        self.name = "config3_ragged_b64"
        total = sum(self.seq)
        self.bytes_per_step = sum(kv_bytes(s) for s in self.seq)
        self.qheads_per_step = 32 * batch
        per_set = 2 * total * 8 * 128 * 2
        self.nsets = max(2, math.ceil(2 * L2_BYTES / per_set))
        g = torch.Generator(device=device).manual_seed(seed + 7919 * rank)
        scale = torch.exp(torch.randn((1, 8, 128), generator=g, device=device))
        self.q = [torch.randn((batch, 32, 128), generator=g, device=device).to(torch.bfloat16)
                  for _ in range(self.nsets)]
        self.k = [(torch.randn((total, 8, 128), generator=g, device=device) * scale).to(torch.bfloat16)
                  for _ in range(self.nsets)]
        self.v = [torch.randn((total, 8, 128), generator=g, device=device).to(torch.bfloat16)
                  for _ in range(self.nsets)]
        self.plan = gqa.plan_batch(self.seq, device=device)
        # decode_kernel, plus split_merge_kernel when some sequence has several splits
        self.launches_per_step = 2 if gqa.decode_plan(plan=self.plan).splits > batch else 1
        self.graph_ok = True  # no collective inside the step
        self.out = torch.empty((batch, 32, 128), dtype=torch.bfloat16, device=device)
        self.l2_note = f"{self.nsets} rotating buffer sets of {per_set / 2**20:.0f} MiB"

    @property
    def sets(self):
        return self.nsets

    def launch(self, i):
        j = i % self.nsets
        self.gqa.decode_batch(self.q[j], self.k[j], self.v[j], self.plan, out=self.out, k_rotated=self.k_rotated)

    def config(self):
        return {"workload": self.name, "batch_per_gpu": self.batch, "seq_len": "U{512..8192} seeded",
                "total_keys": sum(self.seq), "kv_layout": "packed position_major [sum S,8,128] bf16",
                "k_channel_scale": "exp(N(0,1)) per (kv head, dim)", "l2": self.l2_note}

    def check(self, steps: int) -> dict:
        """The last timed step's 64 outputs against each sequence decoded on its own
        (gqa.decode: a single-sequence split plan and the in-kernel merge)."""
        j = (steps - 1) % self.nsets
        want, start = [], 0
        for b, n in enumerate(self.seq):
            want.append(self.gqa.decode(self.q[j][b], self.k[j][start:start + n], self.v[j][start:start + n],
                                        seq_len=n, k_rotated=self.k_rotated))
            start += n
        return compare_outputs(self.out, self.torch.stack(want), "each sequence decoded alone (gqa.decode)")

    def e2e_inputs(self):
        return [x.cpu().pin_memory() for x in (self.q[0], self.k[0], self.v[0])]

    def e2e_step(self, host):
        t = self.torch
        dev = self.out.device
        q, k, v = (x.to(dev, non_blocking=True) for x in host)
        out = self.gqa.decode_batch(q, k, v, self.plan, k_rotated=self.k_rotated)
        return out.cpu()

    def oracle_inputs(self):
        return None

    def gpu_result_set0(self):
        return None


class LongContext(Workload):
    """SEQ_LEN=131072; contiguous key shards across ranks + NCCL all-gather."""

    def __init__(self, device, rank, world, seq_len=131072, seed=20260805, exchange="fused"):
        import torch
        import attention_accelerator_b200 as gqa
        self.gqa, self.torch = gqa, torch
        self.rank, self.world = rank, world
        self.exchange = exchange
        self.S = seq_len
        self.name = f"config4_decode_s{seq_len}"
        self.scaling = "strong"
        if world == 1:  # what bounds the single-GPU step (ncu; profiles/decode_kernel_config4_s131072.md)
            self.limiter = ("one decode_kernel launch: a latency-bound consumer loop at 12 warps per SM "
                            "(issue ~52 % active, FMA pipe ~51 %, DRAM traffic 1.009x algorithmic)")
        self.bytes_per_step = kv_bytes(seq_len)  # whole job; each rank reads 1/world of the keys
        self.qheads_per_step = 32
        from attention_accelerator_b200.distributed import shard_range
        lo, hi = shard_range(seq_len, rank, world)
        self.lo, self.hi = lo, hi
        per_set = 2 * (hi - lo) * 8 * 128 * 2
        self.nsets = max(2, math.ceil(2 * L2_BYTES / per_set))
        # Every rank generates the same whole sequences (same seed) and decodes
        # its contiguous shard of them (a view); the whole sequence is kept for
        # the output check, a single-GPU decode of it.
        g = torch.Generator(device=device).manual_seed(seed)
        self.q, self.kfull, self.vfull = [], [], []
        for _ in range(self.nsets):
            self.q.append(torch.randn((1, 32, 128), generator=g, device=device).to(torch.bfloat16))
            self.kfull.append(torch.randn((seq_len, 8, 128), generator=g, device=device).to(torch.bfloat16))
            self.vfull.append(torch.randn((seq_len, 8, 128), generator=g, device=device).to(torch.bfloat16))
        self.k = [x[lo:hi] for x in self.kfull]
        self.v = [x[lo:hi] for x in self.vfull]
        self.device = device
        if world == 1:
            self.out = torch.empty((32, 128), dtype=torch.bfloat16, device=device)
        else:
            self.plan = gqa.plan_batch([seq_len], pos_begin=[lo], pos_end=[hi], kv_starts=[0], partial=True,
                                       device=device)
            self.part = torch.empty((1, 32, 132), dtype=torch.float32, device=device)
            self.out = torch.empty((1, 32, 128), dtype=torch.bfloat16, device=device)
            self.launches_per_step = 2
            if exchange in ("fused", "peer"):
                from attention_accelerator_b200.distributed import PeerExchange
                self.peer = PeerExchange(1, device=device)
                self.graph_ok = True  # no collective library inside the step
                if exchange == "fused":
                    self.launches_per_step = 1
                    self.plan = gqa.plan_batch([seq_len], pos_begin=[lo], pos_end=[hi], kv_starts=[0], device=device)
            else:
                self.gathered = torch.empty((world, 1, 32, 132), dtype=torch.float32, device=device)
        self.l2_note = f"{self.nsets} rotating buffer sets of {per_set / 2**20:.0f} MiB per rank"

    @property
    def sets(self):
        return self.nsets

    def launch(self, i):
        j = i % self.nsets
        kr = self.k_rotated
        if self.world == 1:
            self.gqa.decode(self.q[j][0], self.k[j], self.v[j], seq_len=self.S, query_position=self.S - 1,
                            out=self.out, k_rotated=kr)
            return
        import torch.distributed as dist
        if self.exchange == "fused":
            self.peer.decode(self.q[j], self.k[j], self.v[j], self.plan, out=self.out, k_rotated=kr)
            return
        self.gqa.decode_batch(self.q[j], self.k[j], self.v[j], self.plan, out=self.part, k_rotated=kr)
        if self.exchange == "peer":
            self.peer.combine(self.part, out=self.out)  # NVLink peer exchange fused with the LSE combine
            return
        dist.all_gather_into_tensor(self.gathered.view(self.world, -1), self.part.view(-1))
        self.gqa.combine_partials(self.gathered, out=self.out)  # same as distributed.gather_partials + combine

    def config(self):
        xchg = {"fused": "decode kernel publishes each KV head's merged rows to the NVLink peer exchange, waits for "
                         "the peers' and writes the merged output (gqa_decode_exchange, one launch per step)",
                "peer": "NVLink peer-memory exchange of 32x132 FP32 partials fused with the LSE combine "
                        "(gqa_combine_peers)",
                "nccl": "NCCL all-gather of 32x132 FP32 partials + LSE combine kernel"}[self.exchange]
        return {"workload": self.name, "batch": 1, "seq_len": self.S, "query_position": self.S - 1,
                "kv_layout": "position_major shard [S/N,8,128] bf16 per GPU",
                "parallelism": f"sequence split x{self.world}, {xchg}" if self.world > 1 else "single GPU",
                "l2": self.l2_note}

    def check(self, steps: int) -> dict:
        """The last timed step's output (every rank's, at N > 1) against a
        single-GPU decode of the whole sequence (at N = 1: four key shards
        merged by combine_partials)."""
        j = (steps - 1) % self.nsets
        if self.world == 1:
            want = split_reference(self.gqa, self.torch, self.q[j][0], self.kfull[j], self.vfull[j], self.S,
                                   self.S - 1, k_rotated=self.k_rotated, shards=4)
            what = "4 key shards (decode_batch partials) + combine_partials, same inputs"
        else:
            want = self.gqa.decode(self.q[j][0], self.kfull[j], self.vfull[j], seq_len=self.S,
                                   k_rotated=self.k_rotated)
            what = "single-GPU decode of the whole sequence on this rank"
        return compare_outputs(self.out, want, what)

    def breakdown(self, torch, steps, warmup, stream, dist_on) -> dict | None:
        """At N > 1: the shard decode alone (FP32 partial rows, no exchange), timed
        as the step is; the rest of the step is the exchange and the merge."""
        if self.world == 1:
            return None
        gqa = self.gqa
        plan = gqa.plan_batch([self.S], pos_begin=[self.lo], pos_end=[self.hi], kv_starts=[0], partial=True,
                              device=self.device)
        part = torch.empty((1, 32, 132), dtype=torch.float32, device=self.device)
        outer = self

        class ShardOnly(Workload):
            graph_ok = True

            @property
            def sets(self):
                return outer.nsets

            def launch(self, i):
                j = i % outer.nsets
                gqa.decode_batch(outer.q[j], outer.k[j], outer.v[j], plan, out=part, k_rotated=outer.k_rotated)

        ms, _ = timed_graph_run(torch, ShardOnly(), steps, warmup, stream, dist_on)
        t = torch.tensor([ms], dtype=torch.float64, device=self.device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return {"shard_decode_us": round(float(t.item()) / steps * 1e3, 3)}

    def e2e_inputs(self):
        return [x.cpu().pin_memory() for x in (self.q[0], self.k[0], self.v[0])]

    def e2e_step(self, host):
        dev = self.device
        q, k, v = (x.to(dev, non_blocking=True) for x in host)
        kr = self.k_rotated
        if self.world == 1:
            out = self.gqa.decode(q[0], k, v, seq_len=self.S, query_position=self.S - 1, k_rotated=kr)
        elif self.exchange == "fused":
            out = self.peer.decode(q, k, v, self.plan, k_rotated=kr)
        elif self.exchange == "peer":
            out = self.peer.combine(self.gqa.decode_batch(q, k, v, self.plan, k_rotated=kr))
        else:
            from attention_accelerator_b200.distributed import gather_partials
            part = self.gqa.decode_batch(q, k, v, self.plan, k_rotated=kr)
            out = self.gqa.combine_partials(gather_partials(part))
        return out.cpu()

    def close(self):
        if getattr(self, "peer", None) is not None:
            self.peer.close()

    def oracle_inputs(self):
        """Head-major BF16 codes of buffer set 0 (the whole sequence) for the CPU port."""
        import numpy as np
        t = self.torch

        def bits(x):
            return x.contiguous().view(t.int16).cpu().numpy().astype(np.uint16)
        return (bits(self.q[0][0]), bits(self.kfull[0].transpose(0, 1)), bits(self.vfull[0].transpose(0, 1)),
                self.S, self.S - 1)

    def gpu_result_set0(self):
        import numpy as np
        if self.k_rotated or self.world > 1:
            return None
        self.launch(0)
        self.torch.cuda.synchronize()
        return self.out.view(self.torch.int16).cpu().numpy().astype(np.uint16)


class ChunkedDecode(Workload):
    """batch 16, SEQ_LEN=8192, 128 query positions 8064..8191 per
    sequence, on the tensor cores.  Ranks split the batch (strong scaling)."""

    def __init__(self, device, rank, world, batch=16, seq_len=8192, n_queries=128, seed=20260805):
        import torch
        import attention_accelerator_b200 as gqa
        if batch % world:
            raise SystemExit(f"config5: batch {batch} does not split over {world} ranks")
        self.gqa, self.torch = gqa, torch
        self.S, self.n = seq_len, n_queries
        self.first = seq_len - n_queries
        self.local = batch // world
        self.batch = batch
        self.name = f"config5_chunked_b{batch}_s{seq_len}"
        self.scaling = "strong"
        self.bound = "tensor"
        vis = sum(t + 1 for t in range(self.first, self.first + n_queries))  # visible keys summed over queries
        self.bytes_per_step = batch * (2 * seq_len * 8 * 128 * 2 + 2 * n_queries * HEAD_BYTES)
        self.flops_per_step = batch * 4 * 32 * 128 * vis
        self.qheads_per_step = batch * n_queries * 32
        per_set = self.local * 2 * seq_len * 8 * 128 * 2
        self.nsets = max(2, math.ceil(2 * L2_BYTES / per_set))
        g = torch.Generator(device=device).manual_seed(seed + 7919 * rank)
        self.q = [torch.randn((self.local, n_queries, 32, 128), generator=g, device=device).to(torch.bfloat16)
                  for _ in range(self.nsets)]
        self.k = [torch.randn((self.local, seq_len, 8, 128), generator=g, device=device).to(torch.bfloat16)
                  for _ in range(self.nsets)]
        self.v = [torch.randn((self.local, seq_len, 8, 128), generator=g, device=device).to(torch.bfloat16)
                  for _ in range(self.nsets)]
        self.out = torch.empty((self.local, n_queries, 32, 128), dtype=torch.bfloat16, device=device)
        self.l2_note = f"{self.nsets} rotating buffer sets of {per_set / 2**20:.0f} MiB per rank"
        # Two kernels per step when the last wave's units are split along the keys
        # (chunked_kernel + chunk_combine_kernel): the split needs more than the
        # 256-byte minimum workspace.
        import ctypes
        from attention_accelerator_b200 import _lib
        from attention_accelerator_b200.api import make_params
        p = make_params(seq_len=seq_len, query_position=seq_len - 1)
        c = _lib.GqaChunkParams(batch=self.local, n_queries=n_queries, first_position=self.first)
        need = _lib.load().gqa_chunked_workspace_bytes(ctypes.byref(p), ctypes.byref(c))
        self.launches_per_step = 2 if need > _lib.CHUNKED_WORKSPACE_BYTES else 1
        self.graph_ok = True  # no collective inside the step

    @property
    def sets(self):
        return self.nsets

    def launch(self, i):
        j = i % self.nsets
        self.gqa.decode_chunked(self.q[j], self.k[j], self.v[j], first_position=self.first, seq_len=self.S,
                                out=self.out)

    def config(self):
        return {"workload": self.name, "batch": self.batch, "batch_per_gpu": self.local, "seq_len": self.S,
                "queries": f"{self.first}..{self.first + self.n - 1} per sequence (causal)",
                "kv_layout": "position_major [B,S,8,128] bf16", "l2": self.l2_note,
                "precision": "Q, K, P each split into three BF16 parts: 6 Q.K + 3 P.V tensor-core products "
                             "(FP32-equivalent); executed tensor FLOPs = 4.5 x algorithmic"}

    def check(self, steps: int) -> dict:
        """Queries 0, 63 and 127 of every local sequence of the last timed step
        against single-position calls of the decode kernel (gqa.decode at that
        QUERY_POSITION): another kernel, and the BASELINE's stated equivalence."""
        j = (steps - 1) % self.nsets
        got, want = [], []
        for b in range(self.local):
            for i in (0, self.n // 2 - 1, self.n - 1):
                got.append(self.out[b, i])
                want.append(self.gqa.decode(self.q[j][b, i], self.k[j][b], self.v[j][b], seq_len=self.S,
                                            query_position=self.first + i))
        return compare_outputs(self.torch.stack(got), self.torch.stack(want),
                               "queries 0, 63, 127 of each sequence by single-position gqa.decode calls")

    def e2e_inputs(self):
        return [x.cpu().pin_memory() for x in (self.q[0], self.k[0], self.v[0])]

    def e2e_step(self, host):
        dev = self.out.device
        q, k, v = (x.to(dev, non_blocking=True) for x in host)
        return self.gqa.decode_chunked(q, k, v, first_position=self.first, seq_len=self.S).cpu()

    def oracle_inputs(self):
        return None

    def gpu_result_set0(self):
        return None


MEM_METRIC = ".mem transport text decoded on the GPU: GB/s of text read + BF16 codes written"


def mem_k_text_rows(seq_len: int = 131072):
    """Rows of config 4's K transport file: head-major [8][seq_len][128] as 16-element beats."""
    return 8 * seq_len * 128 // 16


class MemCodec(Workload):
    """Section-8(f) row 1: decode of the reference's K vector file (gqa_k.mem,
    gen_gqa_wrapper_vectors.py:111-119) at config 4's length on the GPU: a 545 MB
    hex text in HBM -> 8 x 131072 x 128 BF16 codes.  One step = gqa_mem_decode
    (two memsets and 4 kernels); the text alone exceeds 2x L2."""

    def __init__(self, device, rank, world, seq_len=131072, seed=20260805):
        import torch
        from attention_accelerator_b200 import _lib, memfile
        self.torch, self.lib = torch, _lib.load()
        self.name = f"memcodec_k_s{seq_len}"
        self.metric, self.unit = MEM_METRIC, "GB/s"
        self.dtype = "u8"
        self.launches_per_step = 4  # fast-path kernel + the general path's three (which return at once)
        self.qheads_per_step = 0
        g = torch.Generator(device=device).manual_seed(seed + 7919 * rank)
        n_rows = mem_k_text_rows(seq_len)
        codes = torch.randn((n_rows, 16), generator=g, device=device).to(torch.bfloat16).view(torch.int16)
        text_bytes = self.lib.gqa_mem_encode_bytes(n_rows, 16)
        self.text = torch.empty(text_bytes, dtype=torch.uint8, device=device)
        st = self.lib.gqa_mem_encode(codes.data_ptr(), n_rows, 16, self.text.data_ptr(),
                                     torch.cuda.current_stream(device).cuda_stream)
        assert st == 0, st
        self.want = codes
        self.rows = torch.empty_like(codes)
        self.result = torch.empty(2, dtype=torch.int64, device=device)
        self.ws_bytes = self.lib.gqa_mem_decode_workspace_bytes(text_bytes)
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=device)
        self.n_rows, self.seq_len = n_rows, seq_len
        self.bytes_per_step = text_bytes + n_rows * 16 * 2
        self.memfile = memfile

    def launch(self, i):
        st = self.lib.gqa_mem_decode(self.text.data_ptr(), self.text.numel(), 16, self.rows.data_ptr(), self.n_rows,
                                     self.result.data_ptr(), self.ws.data_ptr(), self.ws_bytes,
                                     self.torch.cuda.current_stream().cuda_stream)
        assert st == 0, st

    def check(self, steps: int) -> dict:
        n, bad = (int(x) for x in self.result.cpu())
        ok = bad == -1 and n == self.n_rows and bool(self.torch.equal(self.rows, self.want))
        return {"ok": ok, "against": "the codes the text was encoded from (byte-exact)", "rows": n}

    def config(self):
        return {"workload": self.name, "file": "gqa_k.mem of config 4 (head-major [8][131072][128], 16 codes a line)",
                "text_bytes": self.text.numel(), "rows": self.n_rows,
                "l2": "text of 545 MB read once per step (more than 2x L2)", "parallelism": "single GPU"}

    def e2e_inputs(self):
        return [self.text.cpu().pin_memory()]

    def e2e_step(self, host):
        """As the vector-file loader uses the codec: the text goes from pinned host
        memory to the device and is parsed there; the decoded rows stay in HBM for
        the decode kernel, and the caller reads back the 16-byte result (row count,
        first bad offset).  The rows are compared with the encoded codes on the
        device every step."""
        dev = self.rows.device
        text = host[0].to(dev, non_blocking=True)
        n = text.numel()
        self.lib.gqa_mem_decode(text.data_ptr(), n, 16, self.rows.data_ptr(), self.n_rows, self.result.data_ptr(),
                                self.ws.data_ptr(), self.ws_bytes, self.torch.cuda.current_stream().cuda_stream)
        res = self.result.cpu()
        assert int(res[1]) == -1 and int(res[0]) == self.n_rows, "memcodec e2e: parse failed"
        assert self.torch.equal(self.rows, self.want), "memcodec e2e decode mismatch"
        return res

    def oracle_inputs(self):
        return None

    def gpu_result_set0(self):
        return None


def _read_mem_rows(path: str) -> int:
    """One worker's share of the parallel read_mem: parse a piece, return its row count."""
    from oracle.bf16 import read_mem
    return len(read_mem(Path(path), 16))


def mem_cpu_run_parallel(budget_s: float, lines_per_proc: int = 16384):
    """read_mem of the reference (restated in oracle/bf16.py) on every host core: the
    sample text is cut at line ends into one piece per core, each parsed by its own
    spawned process (read_mem is pure Python, so threads would share one core),
    at most 64 processes.  Only row counts come back, so the timing holds the
    parsing alone."""
    import multiprocessing as mp
    import tempfile
    from concurrent.futures import ProcessPoolExecutor
    import numpy as np
    from oracle.bf16 import mem_text
    procs = min(64, os.cpu_count() or 1)
    rng = np.random.default_rng(20260805)
    rows = rng.integers(0, 65536, size=(procs * lines_per_proc, 16), dtype=np.uint16)
    text_bytes = 0
    with tempfile.TemporaryDirectory() as d, \
            ProcessPoolExecutor(max_workers=procs, mp_context=mp.get_context("spawn")) as pool:
        paths = []
        for i, part in enumerate(np.array_split(rows, procs)):
            f = Path(d) / f"gqa_k_{i}.mem"
            text = mem_text(part)
            text_bytes += len(text)
            f.write_text(text)
            paths.append(str(f))
        list(pool.map(_read_mem_rows, paths))  # start and warm every worker
        reps, t0 = 0, time.perf_counter()
        while True:
            got = sum(pool.map(_read_mem_rows, paths))
            reps += 1
            dt = time.perf_counter() - t0
            if dt >= budget_s or reps >= 20:
                break
    assert got == len(rows)
    per = text_bytes + len(rows) * 16 * 2
    return (per * reps / dt / 1e9, procs,
            f"{reps} x read_mem of a {text_bytes / 1e6:.1f} MB sample ({len(rows)} lines) cut into {procs} pieces, "
            f"one spawned process each, {dt:.1f} s")


def make_workload(name, device, rank, world, layout="position_major", chunk_batch=16, exchange="fused",
                  shard="sequences"):
    if name == "memcodec":
        return MemCodec(device, rank, world)
    if shard == "heads":
        if name != "config2":
            raise SystemExit("--shard heads applies to config2 (one sequence's KV heads over the GPUs)")
        return HeadShardDecode(device, rank, world, 4096, 4095)
    if name == "config1":
        return SingleDecode(device, rank, 30, 29, uniform=True, layout=layout)
    if name == "config2":
        return SingleDecode(device, rank, 4096, 4095, layout=layout)
    if name == "config3":
        return RaggedBatch(device, rank)
    if name == "config4":
        return LongContext(device, rank, world, exchange=exchange)
    if name == "config5":
        return ChunkedDecode(device, rank, world, batch=chunk_batch)
    raise SystemExit(f"unknown workload {name}")


# ---------------------------------------------------------------------------
def timed_graph_run(torch, wl, steps, warmup, stream, dist_on):
    """Capture the steps as CUDA graphs of up to 64 steps (a whole number of
    passes over the rotating buffer sets, and a remainder) and time K steps.
    Within a graph each kernel's set-up overlaps the previous kernel's tail
    (programmatic dependent launch); a boundary between graph replays does not."""
    with torch.cuda.stream(stream):
        for i in range(max(warmup, 1)):
            wl.launch(i)
    torch.cuda.synchronize()
    graphs = {}
    use_graphs = not (dist_on and wl.launches_per_step > 1) or wl.graph_ok

    def graph_of(n):
        if n not in graphs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(n):
                    wl.launch(i)
            graphs[n] = g
        return graphs[n]

    n = wl.sets * max(1, min(steps, 64) // wl.sets)
    if use_graphs:
        graph_of(n)
        if steps % n:
            graph_of(steps % n)
        with torch.cuda.stream(stream):
            graphs[n].replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    t0 = time.monotonic()
    with torch.cuda.stream(stream):
        start.record(stream)
        if use_graphs:
            for _ in range(steps // n):
                graphs[n].replay()
            if steps % n:
                graphs[steps % n].replay()
        else:
            for i in range(steps):
                wl.launch(i)
        end.record(stream)
    torch.cuda.synchronize()
    t1 = time.monotonic()
    if dist_on:
        torch.distributed.barrier()
    graphs.clear()
    return start.elapsed_time(end), (t0, t1)


def traffic_for(workload: str, bytes_per_launch: float):
    """DRAM bytes per launch from the committed ncu capture of this workload, or
    None.  A capture is of one launch on one GPU; it applies only to a launch
    with the same algorithmic bytes (not to one rank's shard of a split
    sequence at N > 1, whose launch moves 1/N of them)."""
    path = ROOT / "profiles" / f"traffic_{workload}.json"
    if not path.is_file():
        return None
    rec = json.loads(path.read_text())
    alg = float(rec.get("algorithmic_bytes_per_launch", -1))
    if abs(alg - bytes_per_launch) > 1e-3 * bytes_per_launch:
        return None
    return rec.get("dram_bytes_per_launch")


def box_hbm_copy_gbs(torch, device, elems: int = 1 << 28, reps: int = 5) -> float:
    """This box's device-to-device copy rate (read + write bytes, best of `reps`,
    CUDA events), measured the way the driver measures the HBM peak, but on the
    GPU this run got: GPUs of the pool differ, and the kernel's fraction of this
    figure separates the kernel from the box."""
    a = torch.empty(elems, dtype=torch.bfloat16, device=device)
    b = torch.empty_like(a)
    b.copy_(a)
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        b.copy_(a)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e-3)
    del a, b
    return 2 * elems * 2 / best / 1e9


def pinned_h2d_gbs(torch, nbytes: int, device, reps: int = 20) -> float:
    """Plain host-to-device copy rate of one pinned buffer of `nbytes` on this box
    (wall clock around synchronised copies, as e2e is timed): what e2e is bound by."""
    host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
    dev.copy_(host, non_blocking=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(reps):
        dev.copy_(host, non_blocking=True)
    torch.cuda.synchronize()
    return nbytes * reps / (time.perf_counter() - t0) / 1e9


def e2e_run(torch, wl, steps, device):
    host = wl.e2e_inputs()
    wl.e2e_step(host)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        out = wl.e2e_step(host)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    h2d = sum(x.numel() * x.element_size() for x in host)
    d2h = out.numel() * out.element_size()
    return dt, h2d, d2h


def chunked_cpu_sample(n_keys: int, seed: int = 20260805):
    """One sequence of the config-5 chunk (128 queries at the last positions of n_keys
    keys) as BF16 codes for the float64 chunked restatement."""
    import numpy as np
    import torch
    g = torch.Generator().manual_seed(seed)

    def bits(t):
        return t.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)
    return (bits(torch.randn(1, 128, 32, 128, generator=g)), bits(torch.randn(1, 8, n_keys, 128, generator=g)),
            bits(torch.randn(1, 8, n_keys, 128, generator=g)))


def chunked_cpu_run(budget_s: float, n_keys: int = 8192):
    """Time oracle/chunked.py (numpy float64, BLAS threads) on whole config-5 sequences."""
    from oracle.chunked import chunked_golden_f64
    q, k, v = chunked_cpu_sample(n_keys)
    reps, t0 = 0, time.perf_counter()
    while True:
        chunked_golden_f64(q, k, v, n_keys, n_keys - 128)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= budget_s or reps >= 50:
            return reps, dt


def port_one_core(q, k, v, n, qpos, budget_s):
    """The float64 restatement of the golden on one core (one worker, BLAS limited to
    one thread): the single-core figure beside the all-cores one.  At least one call."""
    from concurrent.futures import ThreadPoolExecutor
    from threadpoolctl import threadpool_limits
    from oracle.parallel import gqa_golden_parallel
    with threadpool_limits(limits=1), ThreadPoolExecutor(max_workers=1) as pool:
        reps, t0 = 0, time.perf_counter()
        while True:
            gqa_golden_parallel(q, k, v, n, qpos, pool=pool)
            reps += 1
            dt = time.perf_counter() - t0
            if dt >= budget_s or reps >= 200:
                break
    return {"value": round(kv_bytes(qpos + 1) * reps / dt / 1e9, 4), "cores": 1,
            "sample": f"{reps} x SEQ_LEN={n} on one thread (BLAS limited to one), {dt:.1f} s"}


def cpu_baseline(wl, budget_s=10.0):
    """Thread-parallel float64 restatement of the golden on this host (kind "port")."""
    import numpy as np
    from oracle import check_rows
    from oracle.parallel import gqa_golden_parallel
    if isinstance(wl, MemCodec):
        value, cores, sample = mem_cpu_run_parallel(budget_s)
        return {"value": round(value, 5), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample}
    if isinstance(wl, ChunkedDecode):
        reps, dt = chunked_cpu_run(budget_s, wl.S)
        per_seq = wl.bytes_per_step / wl.batch
        return {"value": round(per_seq * reps / dt / 1e9, 4), "unit": UNIT, "cores": os.cpu_count() or 1,
                "kind": "port",
                "sample": f"{reps} x one config-5 sequence (128 queries, SEQ_LEN={wl.S}) by the numpy float64 "
                          f"chunked restatement (oracle/chunked.py, BLAS on all cores), {dt:.1f} s"}
    inp = wl.oracle_inputs()
    if inp is None:
        # ragged / sharded workloads: time the restatement on a config-2-sized sample
        import torch
        g = torch.Generator().manual_seed(1)
        S = 4096

        def bits(t):
            return t.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)
        inp = (bits(torch.randn(32, 128, generator=g)), bits(torch.randn(8, S, 128, generator=g)),
               bits(torch.randn(8, S, 128, generator=g)), S, S - 1)
        gpu = None
    else:
        gpu = wl.gpu_result_set0()
    q, k, v, s, qpos = inp
    threads = os.cpu_count() or 1
    from concurrent.futures import ThreadPoolExecutor
    pool = ThreadPoolExecutor(max_workers=threads)
    reps, t0 = 0, time.perf_counter()
    while True:
        ref = gqa_golden_parallel(q, k, v, s, qpos, pool=pool)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= budget_s or reps >= 200:
            break
    pool.shutdown()
    out = {"value": round(kv_bytes(qpos + 1) * reps / dt / 1e9, 4), "unit": UNIT, "cores": threads,
           "kind": "port",
           "sample": f"{reps} x SEQ_LEN={s} decode(s) by the numpy float64 restatement (oracle/parallel.py), "
                     f"{dt:.1f} s on {threads} threads",
           "one_core": port_one_core(q, k, v, s, qpos, budget_s / 2)}
    if gpu is not None:
        res = check_rows(ref, gpu, 64)
        out["gpu_vs_port_ulp"] = {"max": res.worst_ulp, "mean": round(res.mean_ulp, 5), "pass_64": res.passed}
    return out


def reference_arm(args, rank, world):
    """`--impl reference`: the reference algorithm on the host cores (rank 0 only)."""
    if rank != 0:
        return
    import numpy as np
    import torch
    from concurrent.futures import ThreadPoolExecutor
    from oracle.parallel import gqa_golden_parallel
    if args.workload == "memcodec":
        value, cores, sample = mem_cpu_run_parallel(150.0 / max(1, args.steps + args.warmup) * args.steps)
        print(json.dumps({
            "metric": MEM_METRIC, "value": round(value, 5), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic .mem text (seeded codes)", "impl": "reference",
            "config": {"workload": "memcodec", "sample": sample},
            "cpu_baseline": {"value": round(value, 5), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 5), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return
    if args.workload == "config5":
        n_keys = 8192
        chunked_cpu_run(0.0, n_keys)  # warm-up of one sequence
        reps, dt = chunked_cpu_run(150.0 / max(1, args.steps + args.warmup) * args.steps, n_keys)
        per_seq = 2 * n_keys * 8 * 128 * 2 + 2 * 128 * HEAD_BYTES
        value = per_seq * reps / dt / 1e9
        sample = (f"{reps} x one config-5 sequence (128 queries 8064..8191, SEQ_LEN=8192) by the numpy float64 "
                  f"chunked restatement of gen_gqa_wrapper_vectors.py:121-139 (oracle/chunked.py), {dt:.1f} s")
        print(json.dumps({
            "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world, "steps": reps,
            "warmup": 1, "ms_per_step": round(dt / reps * 1e3, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic N(0,1) seeded",
            "impl": "reference", "config": {"workload": "config5", "seq_len": n_keys, "sample_sequences": reps},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": os.cpu_count() or 1, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return
    cfg = {"config1": (30, 29), "config2": (4096, 4095), "config3": (4352, 4351), "config4": (131072, 131071)}
    s, qpos = cfg[args.workload]
    g = torch.Generator().manual_seed(20260805)

    def bits(t):
        return t.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)
    threads = os.cpu_count() or 1
    pool = ThreadPoolExecutor(max_workers=threads)
    q = bits(torch.randn(32, 128, generator=g))
    probe_n = min(s, 4096)
    kp, vp = bits(torch.randn(8, probe_n, 128, generator=g)), bits(torch.randn(8, probe_n, 128, generator=g))
    t = time.perf_counter()
    gqa_golden_parallel(q, kp, vp, probe_n, probe_n - 1, pool=pool)
    t_probe = time.perf_counter() - t
    per_key = t_probe / probe_n
    budget = 150.0 / max(1, args.steps + args.warmup)
    n = int(max(64, min(s, budget / per_key)))
    k, v = bits(torch.randn(8, n, 128, generator=g)), bits(torch.randn(8, n, 128, generator=g))
    for _ in range(args.warmup):
        gqa_golden_parallel(q, k, v, n, n - 1, pool=pool)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        gqa_golden_parallel(q, k, v, n, n - 1, pool=pool)
    dt = time.perf_counter() - t0
    pool.shutdown()
    value = kv_bytes(n) * args.steps / dt / 1e9
    sample = (f"each step: the first {n} keys of the SEQ_LEN={s} workload (float64 numpy restatement of "
              f"gen_gqa_wrapper_vectors.py:121-139, {threads} threads)")
    n1 = int(max(64, min(n, 10.0 / (per_key * threads))))  # about 10 s on one core
    one = port_one_core(q, k[:, :n1], v[:, :n1], n1, n1 - 1, 10.0)
    print(json.dumps({
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic N(0,1) seeded",
        "impl": "reference", "config": {"workload": args.workload, "seq_len": s, "sample_keys": n},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample, "one_core": one},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("config1", "config2", "config3", "config4", "config5", "memcodec"),
                    default="config4")
    ap.add_argument("--layout", choices=("position_major", "head_major"), default="position_major")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", choices=("fused", "peer", "nccl"), default="fused",
                    help="config4 at N>1: exchange inside the decode kernel (fused), in a separate combine kernel "
                         "over peer memory (peer), or NCCL all-gather + combine (nccl)")
    ap.add_argument("--k-rotated", action="store_true",
                    help="configs 1-4: K cache stored pre-rotated (GQA_FLAG_K_ROTATED); decode rotates only Q")
    ap.add_argument("--shard", choices=("sequences", "heads"), default="sequences",
                    help="config2 at N>1: every GPU its own sequences (sequences), or one sequence's 8 KV heads "
                         "split over the GPUs (heads)")
    ap.add_argument("--chunk-batch", type=int, default=16,
                    help="config5 sequences (16 is the BASELINE config; smaller only for profiling captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return

    import torch
    from attention_accelerator_b200.build import build_library
    if rank == 0 or world == 1:
        build_library()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist_on = world > 1
    if dist_on:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
        build_library()
    wl = make_workload(args.workload, device, rank, world, args.layout, args.chunk_batch, args.exchange, args.shard)
    if args.k_rotated:
        if args.workload not in ("config1", "config2", "config3", "config4"):
            raise SystemExit("--k-rotated applies to the decode workloads config1-4")
        wl.k_rotated = True
    stream = torch.cuda.Stream(device)
    sampler = ClockSampler(local) if rank == 0 else None
    ms, window = timed_graph_run(torch, wl, args.steps, args.warmup, stream, dist_on)
    if sampler:
        sampler.mark(*window)
    if dist_on:
        t = torch.tensor([ms], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    scale = world if wl.scaling == "weak" else 1
    value = wl.bytes_per_step * scale / (ms_step * 1e-3) / 1e9
    peak, peak_kind = peak_hbm()
    per_gpu_bytes = wl.bytes_per_step if wl.scaling == "weak" else wl.bytes_per_step / world
    achieved = per_gpu_bytes / (ms_step * 1e-3) / 1e9

    check = wl.check(args.steps) if hasattr(wl, "check") else None  # the last timed step's output
    if check is not None and not check["ok"]:
        print(f"bench: output check FAILED on rank {rank}: {check}", file=sys.stderr, flush=True)
    if dist_on:
        t = torch.tensor([1.0 if check is None or check["ok"] else 0.0], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
        if check is not None:
            check["all_ranks_ok"] = bool(t.item() == 1.0)
    breakdown = wl.breakdown(torch, args.steps, args.warmup, stream, dist_on) if hasattr(wl, "breakdown") else None
    if breakdown:
        breakdown["step_us"] = round(ms_step * 1e3, 3)
        breakdown["exchange_and_merge_us"] = round(breakdown["step_us"] - breakdown["shard_decode_us"], 3)
        breakdown["limiter"] = ("the shard decode" if breakdown["exchange_and_merge_us"] < breakdown["shard_decode_us"]
                                else "the exchange and merge") + " (the larger part of the step)"
    elif getattr(wl, "limiter", None):
        breakdown = {"limiter": wl.limiter}
    e2e_dt, h2d, d2h = e2e_run(torch, wl, args.e2e_steps, device)
    copy_gbs = pinned_h2d_gbs(torch, h2d, device)
    if dist_on:
        t = torch.tensor([e2e_dt, -copy_gbs], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_dt, copy_gbs = float(t[0].item()), -float(t[1].item())  # slowest rank's e2e and copy
    e2e_value = wl.bytes_per_step * scale * args.e2e_steps / e2e_dt / 1e9
    e2e_h2d_gbs = h2d * args.e2e_steps / e2e_dt / 1e9  # this rank's host bytes per second of e2e
    clocks = sampler.stop() if sampler else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(wl, args.cpu_budget)

    box_copy = box_hbm_copy_gbs(torch, device)
    traffic = traffic_for(wl.name, per_gpu_bytes)
    if wl.bound == "tensor":
        tpeak, tkind = peak_bf16()
        per_gpu_flops = wl.flops_per_step if wl.scaling == "weak" else wl.flops_per_step / world
        tflops = per_gpu_flops / (ms_step * 1e-3) / 1e12
        roofline = {"bound": "tensor", "achieved": round(tflops, 2), "peak": tpeak, "peak_kind": tkind,
                    "unit": "TFLOP/s", "frac": round(tflops / tpeak, 4), "traffic": traffic,
                    "algorithmic_flops_per_launch": per_gpu_flops,
                    "executed_tensor_tflops": round(4.5 * tflops, 2),
                    "executed_frac": round(4.5 * tflops / tpeak, 4),
                    "hbm_gbs": round(achieved, 2)}
    else:
        roofline = {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "peak_kind": peak_kind,
                    "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                    "algorithmic_bytes_per_launch": per_gpu_bytes,
                    "box_copy_gbs": round(box_copy, 1), "frac_of_box_copy": round(achieved / box_copy, 4)}
    if rank == 0:
        line = {
            "metric": getattr(wl, "metric", METRIC), "value": round(value, 2), "unit": getattr(wl, "unit", UNIT), "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 6), "higher_is_better": True,
            "scaling": wl.scaling, "vs_baseline": None, "dtype": getattr(wl, "dtype", "bf16"),
            "data": "synthetic, seeded torch RNG (N(0,1) unless the workload says otherwise)",
            "config": dict(wl.config(), **({"k_cache": "pre-rotated at append time (GQA_FLAG_K_ROTATED)"}
                                              if wl.k_rotated else {}), parallelism=(f"dp{world} (independent sequences per GPU)"
                                                     if wl.scaling == "weak" else wl.config().get("parallelism"))),
            "pct_of_peak_hbm": round(100 * achieved / peak, 2),
            "query_heads_per_s": (round(wl.qheads_per_step * scale / (ms_step * 1e-3), 1)
                                  if wl.qheads_per_step else None),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 3), "unit": getattr(wl, "unit", UNIT), "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": args.e2e_steps,
                    "pinned_h2d_copy_gbs": round(copy_gbs, 2),
                    "h2d_rate_of_pinned_copy": round(e2e_h2d_gbs / copy_gbs, 4)},
            "check": check,
            "breakdown": breakdown,
            "gpu_launches": args.steps * wl.launches_per_step,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if dist_on:
        torch.distributed.barrier()
        wl.close()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
