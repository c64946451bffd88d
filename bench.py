#!/usr/bin/env python3
"""Benchmark: int8 GEMM TOPS at M=N=K=8192 on B200, M split across GPUs.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl zoxide|reference] [--workload W]

One step = one launch of this library's GEMM over this rank's M-row shard (each rank holds all
of B and writes its own rows of C; no collective on the data path). Timing: W untimed warm-up
steps, then K steps timed with CUDA events on the launching stream, an L2 flush (a 256 MiB
write) between steps outside the timed events, barrier + synchronize around the loop, max over
ranks. `value` = whole-job ops / max-rank device time.

Every timed run is checked, as the reference bench checks every run it times
(src/bench.zig:665-668, :712-740): C is poisoned with 0xff bytes before the last timed step, and
after the loop that step's C is copied to the host and checked (the reference's 256 samples from
xorshift32 state 0xdeadbeef, exact for the integer kernels; Freivalds' identity over the whole
matrix; 256 full rows within 1e-2 relative Frobenius error for bf16): the `parity` field.

`e2e` times the same GEMM from host (pinned) buffers, the copies inside the timed region: on one
GPU through the library's host-buffer entry (zx_gemm_s8_host / zx_gemm_bf16_host, copies
overlapped with the kernels); on N GPUs each rank copies its rows of A and 1/N of B from the
host, NCCL all-gathers B over NVLink, and copies its rows of C back by chunks
(zoxide_b200.shard.gemm_host_sharded).

On one GPU the default run then adds, each checked the same way and timed with fewer steps:
`configs` (3, 3', 4 and 5, the scaled-bf16 epilogue, the reference's NN
layout, and the reference-contract kernels imma_s8 / imma_s4 / imma_sp_s8 at n = 8192),
`sustained` (the headline back to back for >= 1.5 s, under the power cap) and `library_int8`
(cuBLASLt int8 through torch._int_mm at the same shape, for comparison). On N > 1 GPUs it adds
`allgather_c` (NCCL all-gather of the C slices timed on its own, overlapped with the GEMM, and
fused into the GEMM kernel as stores to the peers' C over NVLink)
and config 5 M-sharded over the N GPUs.

--impl reference times the reference's CPU GEMM check loop (src/bench.zig:723-727, restated in
oracle/zxo.c) on the host cores over a bounded row sample of the same workload; under torchrun
only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from zoxide_b200.shard import row_shard  # noqa: E402  (pure Python; loads no library)

# name: (M, N, K, kind, layout); kind in s8 | s8_scaled | w4a8 | bf16 | sp_s8 | ref_s8 | ref_s4 | ref_sp_s8 |
# ref_sp_s4 | nn_sp_s8 | nn_s4s4 | nn_sp_s4
WORKLOADS = {
    "s8_8192": (8192, 8192, 8192, "s8", 0),
    "s8_8192_scaled_bf16": (8192, 8192, 8192, "s8_scaled", 0),
    "s8_8192_nn": (8192, 8192, 8192, "s8", 1),
    "s8_1024": (1024, 1024, 1024, "s8", 0),
    "s8_shard8": (1024, 8192, 8192, "s8", 0),  # one GPU's share of 8192^3 at 8 GPUs
    "s8_shard4": (2048, 8192, 8192, "s8", 0),  # ... at 4 GPUs
    "s8_shard2": (4096, 8192, 8192, "s8", 0),  # ... at 2 GPUs
    "w4a8_4096": (4096, 28672, 8192, "w4a8", 0),
    "w4a8_16": (16, 28672, 8192, "w4a8", 0),
    "bf16_65536": (65536, 8192, 8192, "bf16", 0),
    "bf16_8192": (8192, 8192, 8192, "bf16", 0),  # config-5 kernel on a smaller M (profiling size)
    "sp_s8_8192": (8192, 8192, 8192, "sp_s8", 0),
    # the reference's own kernels and layouts under its launch contract (src/bench.zig:647-741,
    # :767-869, :1014-1150): square n, B row-major K x N
    "ref_imma_s8_8192": (8192, 8192, 8192, "ref_s8", 1),
    "ref_imma_s4_8192": (8192, 8192, 8192, "ref_s4", 1),
    "ref_imma_sp_s8_8192": (8192, 8192, 8192, "ref_sp_s8", 1),
    "ref_imma_sp_s4_8192": (8192, 8192, 8192, "ref_sp_s4", 1),
    # the same layouts through one layout pass into a workspace, then the fast kernels
    # (zx_gemm_sp_s8_nn, zx_gemm_s4s4_nn, zx_gemm_sp_s4_nn); the pass is inside the timed step
    "nn_sp_s8_8192": (8192, 8192, 8192, "nn_sp_s8", 1),
    "nn_s4s4_8192": (8192, 8192, 8192, "nn_s4s4", 1),
    "nn_sp_s4_8192": (8192, 8192, 8192, "nn_sp_s4", 1),
}
# timed after the headline in the default one-GPU run (steps each: a few ms to ~0.1 s of GPU time)
CONFIG_SET = ["s8_1024", "s8_8192_scaled_bf16", "s8_8192_nn", "w4a8_4096", "w4a8_16", "sp_s8_8192",
              "bf16_65536", "ref_imma_s8_8192", "ref_imma_s4_8192", "ref_imma_sp_s8_8192", "ref_imma_sp_s4_8192",
              "nn_sp_s8_8192", "nn_s4s4_8192", "nn_sp_s4_8192"]
METRIC = "int8 GEMM TOPS at 8192³ per B200 and at 1/2/4/8 GPUs; % of dense INT8 peak"
NOMINAL_INT8_TOPS = 4500.0
NOMINAL_BF16_TFLOPS = 2250.0
FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, FALLBACK_BF16_SUSTAINED = 6650.0, 1590.0, 1400.0
# checker kind (zoxide_b200.verify) of each workload kind
CHECK_KIND = {"s8": "s8", "s8_scaled": "s8_scaled", "w4a8": "w4a8", "bf16": "bf16", "sp_s8": "sp_s8",
              "ref_s8": "s8", "ref_s4": "s4s4", "ref_sp_s8": "sp_s8", "nn_sp_s8": "sp_s8", "nn_s4s4": "s4s4",
              "ref_sp_s4": "sp_s4", "nn_sp_s4": "sp_s4"}


def peaks():
    """(bf16 burst TFLOP/s, bf16 sustained TFLOP/s, HBM GB/s, source) for the roofline."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return (d.get("bf16_tflops", FALLBACK_BF16_TFLOPS),
                d.get("bf16_tflops_sustained", FALLBACK_BF16_SUSTAINED),
                d.get("hbm_gbs", FALLBACK_HBM_GBS), "measured")
    return FALLBACK_BF16_TFLOPS, FALLBACK_BF16_SUSTAINED, FALLBACK_HBM_GBS, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def algorithmic_bytes(kind, Mr, N, K):
    """HBM bytes one launch must move at least: inputs once, output once."""
    esz = 2 if kind == "bf16" else 1
    if kind in ("sp_s8", "ref_sp_s8", "nn_sp_s8"):
        a = Mr * K // 2 + Mr * K // 8  # kept values + metadata
    elif kind in ("ref_sp_s4", "nn_sp_s4"):
        a = Mr * K // 4 + Mr * K // 16  # kept s4 bytes + metadata
    elif kind in ("ref_s4", "nn_s4s4"):
        a = Mr * K // 2
    else:
        a = Mr * K * esz
    b = N * K // 2 if kind in ("w4a8", "ref_s4", "nn_s4s4", "ref_sp_s4", "nn_sp_s4") else N * K * esz
    c = Mr * N * (2 if kind == "s8_scaled" else 4)
    extra = (Mr + N) * 4 if kind == "s8_scaled" else 0
    return a + b + c + extra


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled every 50 ms during the timed region."""

    Q = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: str):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def mark(self, which: str):
        setattr(self, which, time.time())

    @staticmethod
    def _ts(s: str):
        from datetime import datetime

        try:
            return datetime.strptime(s, "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        t0 = getattr(self, "t_start", None)
        t1 = getattr(self, "t_end", None)
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            ts = self._ts(parts[0])
            if t0 is not None and t1 is not None and ts is not None and not (t0 - 0.1 <= ts <= t1 + 0.1):
                continue  # only samples taken while the timed loop ran
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


def cpu_reference_sample(M, N, K, layout, target_s=12.0, max_rows=None):
    """Time the restated reference check loop on all host cores over a bounded row sample."""
    import oracle

    oracle.build()
    rng = oracle.Rng.from_seed(0)
    threads = oracle.num_threads(0)
    # only the sampled rows of A are needed; B in full (the loop reads every column)
    B = rng.s8((N, K) if layout == 0 else (K, N))
    # calibrate on a small block, then size the sample for ~target_s of work on all threads
    A = rng.s8((4 * threads, K))
    t0 = time.perf_counter()
    oracle.ref_loop_s8(A, B, N, K, layout, 0, 4 * threads, threads)
    per_row = (time.perf_counter() - t0) / (4 * threads)
    rows = int(target_s / max(per_row, 1e-9)) // threads * threads
    rows = max(threads, min(M, max_rows or M, rows))
    A = rng.s8((rows, K))
    t0 = time.perf_counter()
    oracle.ref_loop_s8(A, B, N, K, layout, 0, rows, threads)
    dt = time.perf_counter() - t0
    ops = 2.0 * rows * N * K
    return {
        "value": ops / dt / 1e12, "unit": "TOPS", "cores": threads, "kind": "port",
        "sample": f"{rows} of {M} rows x all {N} columns x K={K} (i64 accumulate, "
                  f"restated src/bench.zig:723-727), {dt:.2f} s on {threads} threads",
        "extrapolated": rows < M, "sampled_rows": rows, "seconds": dt,
    }


def describe(name):
    M, N, K, kind, layout = WORKLOADS[name]
    op = {"s8": "int8 x int8 -> int32", "s8_scaled": "int8 x int8 -> scaled bf16",
          "w4a8": "int8 x int4 (packed along K) -> int32", "bf16": "bf16 x bf16 -> fp32",
          "sp_s8": "2:4-sparse int8 x int8 -> int32",
          "ref_s8": "reference-contract imma_s8 (int8 -> int32)",
          "ref_s4": "reference-contract imma_s4 (s4 x s4 -> int32, B packed along N)",
          "ref_sp_s8": "reference-contract imma_sp_s8 (2:4-sparse int8 -> int32)",
          "nn_sp_s8": "2:4-sparse int8 -> int32, reference layout via transpose pass (zx_gemm_sp_s8_nn)",
          "nn_s4s4": "s4 x s4 -> int32, reference layouts via unpack/repack pass (zx_gemm_s4s4_nn)",
          "ref_sp_s4": "reference-contract imma_sp_s4 (4:8 pair-clustered s4 x s4 -> int32)",
          "nn_sp_s4": "4:8 pair-clustered s4 x s4 -> int32, reference layouts via a pass onto the 2:4 int8 "
                      "kernels (zx_gemm_sp_s4_nn)"}[kind]
    bl = "column-major (N x K)" if layout == 0 else "row-major K x N"
    return f"{op} GEMM M={M} N={N} K={K} ({name}), A row-major, B {bl}"


def make_config(args, M, N, K, ws, workload=None):
    Mr = row_shard(M, ws, 0)[1]
    return {
        "workload": describe(workload or args.workload),
        "M": M, "N": N, "K": K, "M_per_gpu": Mr, "parallelism": f"M-row shards x{ws}, full B per GPU",
        "l2": "256 MiB write between timed steps (L2 flush); inputs+output > L2 at N=1",
    }


def run_reference(args, M, N, K, layout, ws, rank):
    """The reference arm: each step is the restated reference check loop over a bounded row
    sample (all host threads); value = sampled ops / sampled time, ms_per_step the sample's own
    time. The full-problem time per step is an extrapolation and is labelled so."""
    if rank != 0:
        return 0
    vals, secs = [], []
    last = None
    # each step is a bounded row sample; the whole run stays within ~3 minutes
    per_step = max(0.5, min(args.ref_seconds, 150.0 / max(1, args.warmup + args.steps)))
    for i in range(args.warmup + args.steps):
        r = cpu_reference_sample(M, N, K, layout, target_s=per_step)
        if i >= args.warmup:
            vals.append(r["value"])
            secs.append(r["seconds"])
            last = r
    v = sum(2.0 * last["sampled_rows"] * N * K for _ in vals) / sum(secs) / 1e12
    full_ms = 2.0 * M * N * K / (v * 1e12) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TOPS", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.mean(secs) * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int64",
        "data": "synthetic (seeded xorshift32 int8, uniform [-128,127])",
        "config": make_config(args, M, N, K, ws),
        "step": f"one bounded row sample of the workload ({last['sampled_rows']} of {M} rows, all columns)",
        "cpu_baseline": {k: last[k] for k in ("value", "unit", "cores", "kind", "sample", "extrapolated")},
        "full_problem": {"ms_per_step": full_ms, "extrapolated": last["extrapolated"],
                         "from": f"{last['sampled_rows']}-row samples at the measured rate"},
        "e2e": {"value": v, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    line["cpu_baseline"]["value"] = v
    print(json.dumps(line), flush=True)
    return 0


class Workload:
    """Device inputs, the library call and the result check of one workload on this rank's rows.

    Data: torch's seeded generators on the device (uniform integers over the full int8 / s4 range,
    N(0,1)/sqrt(K) bf16, 2:4 metadata with every kept pair equally likely in the reference's nibble
    format). Every rank holds the same B; A differs per rank."""

    def __init__(self, name, zx, dev, stream, ws=1, rank=0):
        import torch

        self.name, self.zx, self.dev, self.stream = name, zx, dev, stream
        M, N, K, kind, layout = WORKLOADS[name]
        self.M, self.N, self.K, self.kind, self.layout = M, N, K, kind, layout
        self.m0, self.m1 = row_shard(M, ws, rank)
        Mr = self.Mr = self.m1 - self.m0
        gen = torch.Generator(device=dev)
        gen.manual_seed(1234 + rank)
        self.meta = self.rs = self.cs = self.ws_buf = None
        if kind == "bf16":
            self.A = (torch.randn((Mr, K), device=dev, generator=gen) / K ** 0.5).to(torch.bfloat16)
        elif kind in ("sp_s8", "ref_sp_s8", "nn_sp_s8"):
            self.A = torch.randint(-128, 128, (Mr, K // 2), dtype=torch.int8, device=dev, generator=gen)
            # every nibble one of the 6 kept pairs (idx0 | idx1 << 2), 8 nibbles per u32 word
            lut = torch.tensor([4, 8, 12, 9, 13, 14], dtype=torch.int64, device=dev)
            nib = lut[torch.randint(0, 6, (Mr, K // 32, 8), device=dev, generator=gen)]
            shifts = 4 * torch.arange(8, device=dev, dtype=torch.int64)
            E = ((nib << shifts).sum(-1) & 0xFFFFFFFF).to(torch.int64)
            self.meta = torch.where(E >= 2 ** 31, E - 2 ** 32, E).to(torch.int32).contiguous()
        elif kind in ("ref_sp_s4", "nn_sp_s4"):
            self.A = torch.randint(0, 256, (Mr, K // 4), dtype=torch.uint8, device=dev, generator=gen)
            # per 8-wide k chunk one of the 6 kept sub-chunk pairs (p0 | p1 << 2), 8 nibbles per word
            lut = torch.tensor([4, 8, 12, 9, 13, 14], dtype=torch.int64, device=dev)
            nib = lut[torch.randint(0, 6, (Mr, K // 64, 8), device=dev, generator=gen)]
            shifts = 4 * torch.arange(8, device=dev, dtype=torch.int64)
            E = ((nib << shifts).sum(-1) & 0xFFFFFFFF).to(torch.int64)
            self.meta = torch.where(E >= 2 ** 31, E - 2 ** 32, E).to(torch.int32).contiguous()
        elif kind in ("ref_s4", "nn_s4s4"):
            self.A = torch.randint(0, 256, (Mr, K // 2), dtype=torch.uint8, device=dev, generator=gen)
        else:
            self.A = torch.randint(-128, 128, (Mr, K), dtype=torch.int8, device=dev, generator=gen)
        gen.manual_seed(4321)  # every rank holds the same full B
        if kind == "bf16":
            self.B = (torch.randn((N, K), device=dev, generator=gen) / K ** 0.5).to(torch.bfloat16)
        elif kind == "w4a8":
            self.B = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=gen)
        elif kind in ("ref_s4", "nn_s4s4", "ref_sp_s4", "nn_sp_s4"):
            self.B = torch.randint(0, 256, (K, N // 2), dtype=torch.uint8, device=dev, generator=gen)
        else:
            self.B = torch.randint(-128, 128, (N, K) if layout == 0 else (K, N), dtype=torch.int8, device=dev,
                                   generator=gen)
        self.out_dtype = {"s8_scaled": torch.bfloat16, "bf16": torch.float32}.get(kind, torch.int32)
        self.C = torch.empty((Mr, N), dtype=self.out_dtype, device=dev)
        if kind == "s8_scaled":
            self.rs = torch.rand(Mr, device=dev, generator=gen) * 1.5 + 0.5
            self.cs = torch.rand(N, device=dev, generator=gen) * 9e-3 + 1e-3
        if kind == "w4a8":
            # split-K partials go to a workspace (zeroed once, kept zero by the kernel), so C is stored
            # once without a zeroing pass; the large-M kernel ignores it
            self.ws_buf = zx.w4a8_workspace(Mr, N, K, dev)
        if kind in ("nn_sp_s8", "nn_s4s4", "nn_sp_s4"):
            op = {"nn_sp_s8": zx.NN_SP_S8, "nn_s4s4": zx.NN_S4S4, "nn_sp_s4": zx.NN_SP_S4}[kind]
            self.ws_buf = torch.empty(zx.nn_workspace_bytes(op, Mr, N, K), dtype=torch.uint8, device=dev)

    def call(self, A=None, B=None, C=None):
        A = self.A if A is None else A
        B = self.B if B is None else B
        C = self.C if C is None else C
        zx, kind, s = self.zx, self.kind, self.stream
        if kind == "s8":
            zx.gemm_s8(A, B, C, layout=self.layout, stream=s)
        elif kind == "s8_scaled":
            zx.gemm_s8_scaled_bf16(A, B, self.rs, self.cs, C, layout=self.layout, stream=s)
        elif kind == "w4a8":
            zx.gemm_w4a8_ws(A, B, self.ws_buf, C, stream=s)
        elif kind == "sp_s8":
            zx.gemm_sp_s8(A, self.meta, B, C, stream=s)
        elif kind == "bf16":
            zx.gemm_bf16(A, B, C, layout=self.layout, stream=s)
        elif kind == "ref_s8":
            zx.launch_imma_s8_ref(A, B, C, self.N, stream=s)
        elif kind == "ref_s4":
            zx.launch_imma_s4_ref(A, B, C, self.N, stream=s)
        elif kind == "ref_sp_s8":
            zx.launch_imma_sp_s8_ref(A, B, self.meta, C, self.N, stream=s)
        elif kind == "nn_sp_s8":
            zx.gemm_sp_s8_nn(A, self.meta, B, self.ws_buf, C, stream=s)
        elif kind == "nn_s4s4":
            zx.gemm_s4s4_nn(A, B, self.ws_buf, C, stream=s)
        elif kind == "ref_sp_s4":
            zx.launch_imma_sp_s4_ref(A, B, self.meta, C, self.N, stream=s)
        elif kind == "nn_sp_s4":
            zx.gemm_sp_s4_nn(A, self.meta, B, self.ws_buf, C, stream=s)
        else:
            raise ValueError(kind)

    def poison(self):
        """0xff bytes over all of C, as the reference bench does before its run (src/bench.zig:665-668)."""
        import torch

        self.C.view(-1).view(torch.uint8).fill_(0xFF)

    def check(self):
        """The reference bench's check of the last result (zoxide_b200.verify, host tensors)."""
        from zoxide_b200 import verify

        import torch

        torch.cuda.synchronize(self.dev)
        t0 = time.perf_counter()
        h = lambda t: None if t is None else t.cpu()  # noqa: E731
        res = verify.check_result(CHECK_KIND[self.kind], h(self.A), h(self.B), h(self.C), self.layout,
                                  meta=h(self.meta), rs=h(self.rs), cs=h(self.cs))
        res["check_s"] = round(time.perf_counter() - t0, 2)
        res["poisoned_before_last_step"] = True
        return res


def time_steps(wl, steps, warmup, flush, stream, poison=True, start=None):
    """Per-step CUDA-event times (ms) of `steps` calls after `warmup` untimed ones; an L2 flush
    (and, before the last step, the 0xff poison of C) runs between steps outside the events.
    `start()` runs between the warm-up and the timed loop (barrier, clock sampler)."""
    import torch

    for _ in range(warmup):
        flush.fill_(1)
        wl.call()
    torch.cuda.synchronize(wl.dev)
    if start is not None:
        start()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush.fill_(i & 0xFF)
        if poison and i == steps - 1:
            wl.poison()
        starts[i].record(stream)
        wl.call()
        ends[i].record(stream)
    torch.cuda.synchronize(wl.dev)
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def roofline(kind, Mr, N, K, mean_s, sustained, workload=None):
    """Roofline of one launch from its mean CUDA-event time.

    Tensor-bound kernels: achieved = 2*M*N*K / time (dense-equivalent for 2:4 sparse). The int8
    and sparse peaks are the nominal dense INT8 4.5 POPS and 2:4 9 POPS that BASELINE.json quotes:
    MEASURED_PEAKS.json holds HBM and bf16 figures only, and no measured int8 ceiling exists (the
    cuBLASLt int8 GEMM reaches less than this library's kernel). The figure derived from the
    measured cuBLAS bf16 peak (int8 issues at 2x the bf16 rate, sparse int8 at 4x) is kept as
    `frac_of_measured_bf16_x{2,4}`. bf16 is measured against the measured bf16 peak (burst for a
    short loop, sustained when the loop ran under the power cap). HBM-bound launches (the skinny
    W4A8 decode): algorithmic bytes / time against the measured copy bandwidth."""
    bf16_peak, bf16_sus, hbm_peak, src = peaks()
    bf16_den = bf16_sus if sustained else bf16_peak
    ops = 2.0 * Mr * N * K
    alg = algorithmic_bytes(kind, Mr, N, K)
    mult = {"bf16": 1.0, "sp_s8": 4.0, "ref_sp_s8": 4.0, "nn_sp_s8": 4.0, "ref_sp_s4": 4.0, "nn_sp_s4": 4.0}.get(kind, 2.0)
    ridge = mult * bf16_den * 1e12 / (hbm_peak * 1e9)
    if ops / alg < ridge:
        ach = alg / mean_s / 1e9
        r = {"bound": "hbm", "achieved": ach, "peak": hbm_peak, "unit": "GB/s",
             "peak_source": f"HBM copy bandwidth (of {src})", "frac": ach / hbm_peak}
    else:
        ach = ops / mean_s / 1e12
        if kind == "bf16":
            r = {"bound": "tensor", "achieved": ach, "peak": bf16_den, "unit": "TFLOP/s",
                 "peak_source": f"cuBLAS bf16 {'sustained' if sustained else 'burst'} (of {src})",
                 "frac": ach / bf16_den, "frac_of_nominal": ach / NOMINAL_BF16_TFLOPS}
        else:
            nom = 2 * NOMINAL_INT8_TOPS if mult == 4.0 else NOMINAL_INT8_TOPS
            r = {"bound": "tensor", "achieved": ach, "peak": nom, "unit": "TOPS",
                 "peak_source": ("nominal 2:4-sparse INT8 9 POPS (dense-equivalent)" if mult == 4.0 else
                                 "nominal dense INT8 4.5 POPS") + " (BASELINE.json; no measured int8 ceiling)",
                 "frac": ach / nom, "frac_of_nominal": ach / nom,
                 f"frac_of_measured_bf16_x{mult:.0f}": ach / (mult * bf16_den),
                 "measured_bf16_basis": f"{'sustained' if sustained else 'burst'} {bf16_den:.0f} TFLOP/s (of {src})"}
    r.update({"per_launch_ops": ops, "per_launch_algorithmic_bytes": alg})
    return r


def clocks_norm(value, clocks):
    """Throughput per GHz of median SM clock under load (comparable across power-capped runs)."""
    mhz = clocks.get("sm_mhz") if clocks else None
    return value / (mhz / 1000.0) if mhz else None


def pin_to_gpu_numa(dev_index):
    """Run this process on the host CPUs nearest its GPU (NVML's CPU affinity of the device), so
    the pinned host buffers of the host-buffer run are allocated on that NUMA node: with one rank
    per GPU on a multi-socket host, buffers on the far socket cut host copy bandwidth. A process
    setting only (nothing on the GPU changes). Returns the previous CPU set, to be restored."""
    before = os.sched_getaffinity(0)
    try:
        import pynvml
        import torch

        p = torch.cuda.get_device_properties(dev_index)
        bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, ((os.cpu_count() or 64) + 63) // 64)
        cpus = {64 * i + b for i, m in enumerate(words) for b in range(64) if (m >> b) & 1} & before
        if cpus:
            os.sched_setaffinity(0, cpus)
    except Exception:  # no NVML / no affinity information: leave the process where it is
        pass
    return before


def launch_overhead_us(stream, reps=30):
    """Median CUDA-event time of a one-cycle kernel queued behind a busy one (as every timed step
    is queued behind its L2 flush): the GPU-side fixed cost inside each timed step, without the
    host's launch latency."""
    import torch

    out = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(200000)  # keeps the stream busy while the events and the kernel are queued
        a.record(stream)
        torch.cuda._sleep(1)
        b.record(stream)
        b.synchronize()
        out.append(a.elapsed_time(b) * 1e3)
    return statistics.median(out)


def parity_over_ranks(res, dev, ws):
    """The check results of every rank folded into one: bad samples summed, verdicts and-ed."""
    if ws == 1:
        return res
    import torch
    import torch.distributed as dist

    bad = torch.tensor([float(res["bad"])], dtype=torch.float64, device=dev)
    ok = torch.tensor([1.0 if res["ok"] else 0.0, 1.0 if res.get("freivalds", True) else 0.0],
                      dtype=torch.float64, device=dev)
    dist.all_reduce(bad, op=dist.ReduceOp.SUM)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    out = dict(res)
    out.update({"ranks": ws, "samples": res["samples"] * ws, "bad": int(bad.item()), "ok": bool(ok[0].item() == 1.0)})
    if "freivalds" in res:
        out["freivalds"] = bool(ok[1].item() == 1.0)
    return out


def run_e2e(args, wl, zx, dev, stream, ws):
    """The same GEMM from pinned host buffers with every copy inside the timed events."""
    import torch
    import torch.distributed as dist

    from zoxide_b200.shard import gemm_host_sharded, max_over_ranks

    A_h, B_h = wl.A.cpu().pin_memory(), wl.B.cpu().pin_memory()
    C_h = torch.empty(wl.C.shape, dtype=wl.C.dtype).pin_memory()
    A_d, B_d, C_e = torch.empty_like(wl.A), torch.empty_like(wl.B), torch.empty_like(wl.C)
    native = wl.kind in ("s8", "bf16") and wl.layout == 0
    split_b = native and ws > 1 and wl.N % ws == 0
    nbytes = lambda t: t.numel() * t.element_size()  # noqa: E731
    if split_b:
        how = (f"rows of A and 1/{ws} of B's rows from the host per rank, NCCL all-gather of B over NVLink, "
               "GEMM by 4 row chunks with each chunk of C copied back while the next computes "
               "(zoxide_b200.shard.gemm_host_sharded)")
        h2d = nbytes(wl.A) + nbytes(wl.B) // ws
    elif native:
        how = "L-shaped shells of blocks of >= 1024 rows, at most 4 per operand (zx_gemm_s8_host / zx_gemm_bf16_host)"
        h2d = nbytes(wl.A) + nbytes(wl.B)
    else:
        how = "copy in, one call, copy out, in sequence"
        h2d = nbytes(wl.A) + nbytes(wl.B) + sum(nbytes(t) for t in (wl.meta, wl.rs, wl.cs) if t is not None)
    ms = []
    for i in range(args.e2e_steps + 1):
        if ws > 1:
            dist.barrier()
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record(stream)
        if split_b:
            gemm_host_sharded(lambda a, b, c: wl.call(a, b, c), A_h, B_h, C_h, A_d, B_d, C_e, stream=stream)
        elif native:
            zx.gemm_host(A_h, B_h, C_h, A_d, B_d, C_e, stream=stream)
        else:
            A_d.copy_(A_h, non_blocking=True)
            B_d.copy_(B_h, non_blocking=True)
            wl.call(A_d, B_d, C_e)
            C_h.copy_(C_e, non_blocking=True)
        e_ev.record(stream)
        torch.cuda.synchronize(dev)
        if i > 0:  # the first is warm-up
            ms.append(s_ev.elapsed_time(e_ev))
    ref = wl.C.cpu()
    if wl.out_dtype.is_floating_point:  # other tile shapes per block: equal up to fp32 summation order
        diff = float((C_h.float() - ref.float()).abs().max())
        same = diff <= 1e-3
    else:
        diff, same = None, bool(torch.equal(C_h, ref))
    total = max_over_ranks(sum(ms), dev)
    value = 2.0 * wl.M * wl.N * wl.K * len(ms) / (total * 1e-3) / 1e12
    out = {"value": value, "unit": "TFLOP/s" if wl.kind == "bf16" else "TOPS",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": nbytes(wl.C),
           "bytes_per_step_are": "per rank" if ws > 1 else "the job's",
           "ms_per_step": total / len(ms), "overlap": how, "same_result_as_device_run": same}
    if ws > 1:
        out["job_h2d_bytes_per_step"] = h2d * ws
        out["job_d2h_bytes_per_step"] = nbytes(wl.C) * ws
    if diff is not None:
        out["max_abs_diff_vs_device_run"] = diff
    del A_h, B_h, C_h, A_d, B_d, C_e
    return out


def run_allgather(args, wl, zx, dev, stream, ws, flush, gemm_ms):
    """All-gather of the C slices over NVLink: NCCL on its own, NCCL overlapped with the GEMM by
    chunk-interleaved row blocks, and the gather fused into the GEMM kernel (unless
    --no-allgather-fused)."""
    import torch
    import torch.distributed as dist

    from zoxide_b200.shard import gather_rows, max_over_ranks

    C, M = wl.C, wl.M
    for _ in range(4):
        dist.barrier()
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record(stream)
        full = gather_rows(C, M)
        e_ev.record(stream)
        torch.cuda.synchronize(dev)
    ag_ms = max_over_ranks(s_ev.elapsed_time(e_ev), dev)
    out = {"nccl_ms": ag_ms, "bytes_out_per_gpu": full.numel() * full.element_size(),
           "algbw_gbs": full.numel() * full.element_size() / (ag_ms * 1e-3) / 1e9,
           "gemm_then_gather_ms": gemm_ms + ag_ms}
    del full
    P = args.ag_chunks
    if wl.kind in ("s8", "s8_scaled", "bf16") and M % (ws * P) == 0 and wl.Mr == M // ws:
        from zoxide_b200.shard import gemm_allgather_overlapped

        c_full = torch.empty((M, wl.N), dtype=wl.out_dtype, device=dev)
        ov = []
        for it in range(6):
            dist.barrier()
            flush.fill_(it & 0xFF)
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record(stream)
            gemm_allgather_overlapped(lambda a, c: wl.call(a, None, c), wl.A, c_full, P)
            e_ev.record(stream)
            torch.cuda.synchronize(dev)
            if it >= 2:
                ov.append(s_ev.elapsed_time(e_ev))
        ov_ms = max_over_ranks(statistics.median(ov), dev)
        chk = torch.tensor([float(c_full.view(-1).view(torch.int32).to(torch.int64).sum().item())],
                           dtype=torch.float64, device=dev)
        lo, hi = chk.clone(), chk.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        out["overlapped"] = {
            "chunks": P, "ms": ov_ms, "saved_frac": 1.0 - ov_ms / (gemm_ms + ag_ms),
            "same_c_on_all_ranks": bool(lo.item() == hi.item()),
            "layout": "row block j*world + rank of M/(world*chunks) rows belongs to rank"}
        del c_full
    if args.allgather_fused and wl.kind == "s8" and wl.layout == 0 and wl.Mr == M // ws:
        from zoxide_b200.shard import PeerBuffers, gemm_allgather_fused

        c_full = torch.full((M, wl.N), -1, dtype=torch.int32, device=dev)
        # every rank must agree before the fused launches: one that cannot map its peers skips
        # the fused timing on all ranks (recorded), instead of leaving the others at a barrier
        pb, err = None, None
        try:
            pb = PeerBuffers(c_full)
        except Exception as e:  # noqa: BLE001
            err = f"{type(e).__name__}: {e}"
        flag = torch.tensor([0.0 if err is None else 1.0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        if flag.item() != 0.0:
            if pb is not None:
                pb.close()
            out["fused"] = {"skipped": err or "a peer rank could not map the peer buffers"}
            del c_full
            return out
        try:
            fu = []
            for it in range(6):
                dist.barrier()
                flush.fill_(it & 0xFF)
                s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s_ev.record(stream)
                gemm_allgather_fused(wl.A, wl.B, c_full, wl.m0, pb, stream=stream)
                e_ev.record(stream)
                torch.cuda.synchronize(dev)
                if it >= 2:
                    fu.append(s_ev.elapsed_time(e_ev))
            fu_kernel = zx.last_kernel()
            dist.barrier()  # every rank's stores into this rank's c_full have completed
            fu_ms = max_over_ranks(statistics.median(fu), dev)
            own_ok = bool(torch.equal(c_full[wl.m0:wl.m1], C))
            chk = torch.tensor([float(c_full.to(torch.int64).sum().item()), float(own_ok)],
                               dtype=torch.float64, device=dev)
            lo, hi = chk.clone(), chk.clone()
            dist.all_reduce(lo, op=dist.ReduceOp.MIN)
            dist.all_reduce(hi, op=dist.ReduceOp.MAX)
            # fused roofline: the slower of the tensor work at the nominal int8 peak and the peer
            # bytes at the measured 770 GB/s NVLink peer-copy rate
            peer_bytes = (ws - 1) * C.numel() * C.element_size()
            t_mma = 2.0 * wl.Mr * wl.N * wl.K / (NOMINAL_INT8_TOPS * 1e12) * 1e3
            t_link = peer_bytes / 770e9 * 1e3
            out["fused"] = {
                "ms": fu_ms, "saved_frac": 1.0 - fu_ms / (gemm_ms + ag_ms),
                "same_c_on_all_ranks": bool(lo[0].item() == hi[0].item()),
                "own_rows_equal_gemm": bool(lo[1].item() == 1.0), "kernel": fu_kernel,
                "peer_bytes_out_per_gpu": peer_bytes,
                "roofline": {"bound": "nvlink" if t_link > t_mma else "tensor", "target_ms": max(t_link, t_mma),
                             "tensor_ms": t_mma, "nvlink_ms": t_link, "frac": max(t_link, t_mma) / fu_ms,
                             "nvlink_gbs": "770 measured peer copy per direction"}}
        finally:
            torch.cuda.synchronize(dev)
            dist.barrier()
            pb.close()
            dist.barrier()
        del c_full
    return out


def run_sustained(wl, dev, stream, flush, seconds, sampler_index):
    """The headline call back to back (L2 flush between steps) for >= `seconds` of GPU time,
    with its own clock record: the power-capped rate."""
    import torch

    probe = time_steps(wl, 20, 2, flush, stream, poison=False)
    steps = max(20, int(seconds * 1e3 / statistics.mean(probe)) + 1)
    sampler = ClockSampler(sampler_index)

    def start():
        sampler.start()
        time.sleep(0.5)
        sampler.mark("t_start")

    ms = time_steps(wl, steps, 0, flush, stream, poison=True, start=start)
    sampler.mark("t_end")
    clocks = sampler.stop()
    parity = wl.check()
    ops = 2.0 * wl.Mr * wl.N * wl.K
    value = ops * steps / (sum(ms) * 1e-3) / 1e12
    return {"steps": steps, "seconds": sum(ms) * 1e-3, "value": value, "unit": "TOPS",
            "frac_of_nominal": value / NOMINAL_INT8_TOPS, "clocks": clocks,
            "tops_per_ghz": clocks_norm(value, clocks), "parity": parity}


def run_library_int8(wl, dev, stream, flush, steps=20):
    """cuBLASLt's int8 GEMM (torch._int_mm) at the headline shape, timed the same way: a
    library comparison point, not this library's path."""
    import torch

    M, N, K = wl.Mr, wl.N, wl.K
    bt = wl.B.t()  # K x N, column-major: the NT operand as cuBLASLt takes it
    c = torch._int_mm(wl.A, bt)
    for _ in range(3):
        flush.fill_(1)
        torch._int_mm(wl.A, bt, out=c)
    torch.cuda.synchronize(dev)
    ms = []
    for i in range(steps):
        flush.fill_(i & 0xFF)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        torch._int_mm(wl.A, bt, out=c)
        b.record(stream)
        ms.append((a, b))
    torch.cuda.synchronize(dev)
    t = [a.elapsed_time(b) for a, b in ms]
    same = bool(torch.equal(c, wl.C))
    return {"what": "torch._int_mm (cuBLASLt int8 -> int32), same A, B and shape", "steps": steps,
            "value": 2.0 * M * N * K / (statistics.mean(t) * 1e-3) / 1e12, "unit": "TOPS",
            "ms_per_step": statistics.mean(t), "same_result": same}


def run_configs(names, args, zx, dev, stream, flush, ws, rank):
    """Each workload in `names` on this rank's M shard: timed, checked, roofline."""
    import torch

    from zoxide_b200.shard import max_over_ranks

    out = {}
    for name in names:
        M, N, K, kind, layout = WORKLOADS[name]
        if M < ws * 16 or kind.startswith("ref_") and ws > 1:
            continue  # too few rows to shard / square reference kernels run on one GPU
        wl = Workload(name, zx, dev, stream, ws, rank)
        ms = time_steps(wl, args.config_steps, 3, flush, stream, poison=True)
        kernel = zx.last_kernel()
        parity = parity_over_ranks(wl.check(), dev, ws)
        total = max_over_ranks(sum(ms), dev)
        value = 2.0 * M * N * K * len(ms) / (total * 1e-3) / 1e12
        roof = roofline(kind, wl.Mr, N, K, statistics.mean(ms) * 1e-3, sustained=False)
        out[name] = {"workload": describe(name), "steps": len(ms), "value": value,
                     "unit": "TFLOP/s" if kind == "bf16" else "TOPS", "ms_per_step": total / len(ms),
                     "M_per_gpu": wl.Mr, "kernel": kernel, "roofline": roof, "parity": parity}
        del wl
        torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="zoxide", choices=["zoxide", "reference"])
    ap.add_argument("--workload", default="s8_8192", choices=sorted(WORKLOADS))
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-seconds", type=float, default=10.0)
    ap.add_argument("--policy", type=int, default=0, help="0 auto, 1 one-SM tiles, 2 two-SM tiles")
    ap.add_argument("--configs", default="auto",
                    help="comma-separated workloads timed after the headline, 'none', or 'auto' (every "
                         "BASELINE config on one GPU; config 5 M-sharded on N > 1)")
    ap.add_argument("--config-steps", type=int, default=20)
    ap.add_argument("--sustained-seconds", type=float, default=1.5, help="0 skips the sustained loop")
    ap.add_argument("--no-allgather", action="store_true", help="skip the all-gather of C timings (N>1)")
    ap.add_argument("--no-allgather-fused", dest="allgather_fused", action="store_false",
                    help="skip the gather fused into the GEMM kernel (N>1, CUDA IPC peer stores)")
    ap.add_argument("--ag-chunks", type=int, default=4, help="row-block chunks of the overlapped all-gather")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "zoxide" else args.warmup

    M, N, K, kind, layout = WORKLOADS[args.workload]
    ws, rank, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, M, N, K, layout, ws, rank)

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    all_cpus = pin_to_gpu_numa(local)
    host_cpus = sorted(os.sched_getaffinity(0))
    if ws > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        torch.set_num_threads(max(1, (os.cpu_count() or ws) // ws))  # host checks run on every rank

    import zoxide_b200 as zx
    from zoxide_b200.shard import max_over_ranks

    zx.lib()
    zx.set_kernel_policy(args.policy)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    wl = Workload(args.workload, zx, dev, stream, ws, rank)
    Mr = wl.Mr
    launch_us = launch_overhead_us(stream)

    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    smi_index = cvd.split(",")[local].strip() if cvd else str(local)
    sampler = ClockSampler(smi_index)

    def start():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        sampler.start()
        time.sleep(0.5)  # nvidia-smi start-up
        sampler.mark("t_start")

    kern_ms = time_steps(wl, args.steps, args.warmup, flush, stream, poison=True, start=start)
    timed_kernel = zx.last_kernel()  # what the library launched for the timed call
    sampler.mark("t_end")
    if ws > 1:
        dist.barrier()
    clocks = sampler.stop()
    total_ms = sum(kern_ms)
    max_total_ms = max_over_ranks(total_ms, dev)
    mean_ms = statistics.mean(kern_ms)
    per_rank_us = [mean_ms * 1e3]
    if ws > 1:
        t = torch.zeros(ws, dtype=torch.float64, device=dev)
        t[rank] = mean_ms * 1e3
        dist.all_reduce(t)
        per_rank_us = [round(float(x), 2) for x in t.cpu()]
    ops_per_step = 2.0 * M * N * K
    value = ops_per_step * args.steps / (max_total_ms * 1e-3) / 1e12
    status = zx.device_status()
    parity = parity_over_ranks(wl.check(), dev, ws)

    e2e = run_e2e(args, wl, zx, dev, stream, ws)
    allgather = None
    if ws > 1 and not args.no_allgather:
        allgather = run_allgather(args, wl, zx, dev, stream, ws, flush, max_total_ms / args.steps)

    sustained = lib_int8 = None
    if ws == 1 and args.sustained_seconds > 0 and kind in ("s8", "s8_scaled") and M >= 4096:
        sustained = run_sustained(wl, dev, stream, flush, args.sustained_seconds, smi_index)
    if ws == 1 and kind == "s8" and layout == 0 and M >= 4096:
        lib_int8 = run_library_int8(wl, dev, stream, flush)

    roof = roofline(kind, Mr, N, K, mean_ms * 1e-3,
                    sustained=total_ms > 1000.0 or "sw_power_cap" in (clocks.get("reasons") or []))
    tf = ROOT / "profiles" / "ncu_traffic.json"
    roof["traffic"] = json.loads(tf.read_text()).get(f"{args.workload}_M{Mr}") if tf.exists() else None
    roof["traffic_source"] = "profiles/ncu_traffic.json (dram bytes read + write of one ncu-captured launch)"
    roof["kernel"] = "zx::" + timed_kernel
    del wl
    torch.cuda.empty_cache()

    names = []
    if args.configs == "auto":
        names = CONFIG_SET if ws == 1 else ["bf16_65536"]
    elif args.configs != "none":
        names = [x for x in args.configs.split(",") if x]
    names = [x for x in names if x != args.workload]
    configs = run_configs(names, args, zx, dev, stream, flush, ws, rank) if names else None

    os.sched_setaffinity(0, all_cpus)  # the CPU baseline runs on every host core
    if rank == 0:
        cpu = None
        if ws == 1 and not args.no_cpu_baseline and kind in ("s8", "s8_scaled"):
            cpu = cpu_reference_sample(M, N, K, layout, target_s=args.ref_seconds)
            cpu.pop("seconds", None)
        unit = "TFLOP/s" if kind == "bf16" else "TOPS"
        nominal = NOMINAL_BF16_TFLOPS if kind == "bf16" else 2 * NOMINAL_INT8_TOPS if "sp" in kind else NOMINAL_INT8_TOPS
        line = {
            "metric": METRIC if args.workload == "s8_8192" else f"{describe(args.workload)}: {unit}",
            "value": value, "unit": unit, "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": max_total_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": {"s8": "int8", "s8_scaled": "int8", "w4a8": "int8 x int4", "bf16": "bf16",
                      "sp_s8": "int8 (2:4 sparse A)"}.get(kind, "int8"),
            "data": "synthetic (torch seeded uniform integers / normal bf16); no reference dataset",
            "config": {**make_config(args, M, N, K, ws),
                       "host_cpus": f"{len(host_cpus)} CPUs near GPU {local} ({host_cpus[0]}-{host_cpus[-1]})"},
            "pct_of_nominal_peak": 100.0 * value / (nominal * ws),
            "parity": parity,
            "roofline": roof,
            "per_rank_kernel_us": per_rank_us,
            "launch_overhead_us": launch_us,
            "launch_overhead_what": "median CUDA-event time of a one-cycle kernel queued behind a busy kernel "
                                    "on the same stream (GPU-side cost per timed step)",
            "value_per_ghz": clocks_norm(value, clocks),
            "cpu_baseline": cpu,
            "e2e": e2e,
            "sustained": sustained,
            "library_int8": lib_int8,
            "allgather_c": allgather,
            "configs": configs,
            "gpu_launches": args.steps,
            "clocks": clocks,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
