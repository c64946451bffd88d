#!/usr/bin/env python3
"""Benchmark: int8 GEMM TOPS at M=N=K=8192 on B200, M split across GPUs.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl zoxide|reference] [--workload W]

One step = one launch of this library's GEMM over this rank's M-row shard (each rank holds all
of B and writes its own rows of C; no collective on the data path). Timing: W untimed warm-up
steps, then K steps timed with CUDA events on the launching stream, an L2 flush (a 256 MiB
write) between steps outside the timed events, barrier + synchronize around the loop, max over
ranks. `value` = whole-job ops / max-rank device time. `e2e` times the same call with host
(pinned) buffers: H2D of the shard's inputs, the kernel, D2H of the shard's C (for int8 and bf16
NT through the library's host-buffer entry, zx_gemm_s8_host / zx_gemm_bf16_host, which overlaps
the copies with the kernels).

The default workload is the headline (config 2, int8 NT, int32 out). The others are the
remaining BASELINE configs, measured the same way: s8_8192_scaled_bf16 (config 2 epilogue),
s8_8192_nn (the reference's B layout), s8_1024 (config 1), w4a8_4096 / w4a8_16 (config 3 / 3'),
sp_s8_8192 (config 4, 2:4 sparse; ops counted dense-equivalent 2*M*N*K), bf16_65536 (config 5).

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

# name: (M, N, K, kind, layout); kind in s8 | s8_scaled | w4a8 | bf16 | sp_s8
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
}
METRIC = "int8 GEMM TOPS at 8192³ per B200 and at 1/2/4/8 GPUs; % of dense INT8 peak"
NOMINAL_INT8_TOPS = 4500.0
NOMINAL_BF16_TFLOPS = 2250.0
FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, FALLBACK_BF16_SUSTAINED = 6650.0, 1590.0, 1400.0


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
    a = Mr * K * esz if kind != "sp_s8" else Mr * K // 2 + Mr * K // 8  # A_c + metadata
    b = N * K // 2 if kind == "w4a8" else N * K * esz
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
        "seconds": dt,
    }


def describe(name):
    M, N, K, kind, layout = WORKLOADS[name]
    op = {"s8": "int8 x int8 -> int32", "s8_scaled": "int8 x int8 -> scaled bf16",
          "w4a8": "int8 x int4 (packed along K) -> int32", "bf16": "bf16 x bf16 -> fp32",
          "sp_s8": "2:4-sparse int8 x int8 -> int32"}[kind]
    bl = "column-major (N x K)" if layout == 0 else "row-major K x N"
    return f"{op} GEMM M={M} N={N} K={K} ({name}), A row-major, B {bl}"


def make_config(args, M, N, K, ws):
    Mr = row_shard(M, ws, 0)[1]
    return {
        "workload": describe(args.workload),
        "M": M, "N": N, "K": K, "M_per_gpu": Mr, "parallelism": f"M-row shards x{ws}, full B per GPU",
        "l2": "256 MiB write between timed steps (L2 flush); inputs+output > L2 at N=1",
    }


def run_reference(args, M, N, K, layout, ws, rank):
    if rank != 0:
        return 0
    vals = []
    last = None
    # each step is a bounded row sample; the whole run stays within ~3 minutes
    per_step = max(0.5, min(args.ref_seconds, 150.0 / max(1, args.warmup + args.steps)))
    for i in range(args.warmup + args.steps):
        r = cpu_reference_sample(M, N, K, layout, target_s=per_step)
        if i >= args.warmup:
            vals.append(r["value"])
            last = r
    v = statistics.mean(vals)
    total_s = sum(2.0 * M * N * K / (x * 1e12) for x in vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TOPS", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_s / len(vals) * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int64",
        "data": "synthetic (seeded xorshift32 int8, uniform [-128,127])",
        "config": make_config(args, M, N, K, ws),
        "cpu_baseline": {k: last[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": v, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    line["cpu_baseline"]["value"] = v
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="zoxide", choices=["zoxide", "reference"])
    ap.add_argument("--workload", default="s8_8192", choices=sorted(WORKLOADS))
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-seconds", type=float, default=10.0)
    ap.add_argument("--policy", type=int, default=0, help="0 auto, 1 one-SM tiles, 2 two-SM tiles")
    ap.add_argument("--allgather", action="store_true", help="also time an NCCL all-gather of C (N>1)")
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
    if ws > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    import zoxide_b200 as zx
    from zoxide_b200.shard import gather_rows, max_over_ranks

    zx.lib()
    zx.set_kernel_policy(args.policy)
    # this rank's contiguous M-row shard
    m0, m1 = row_shard(M, ws, rank)
    Mr = m1 - m0
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    E = None
    if kind == "bf16":
        A = (torch.randn((Mr, K), device=dev, generator=gen) / K ** 0.5).to(torch.bfloat16)
    elif kind == "sp_s8":
        A = torch.randint(-128, 128, (Mr, K // 2), dtype=torch.int8, device=dev, generator=gen)
        # metadata: every nibble one of the 6 kept pairs (idx0 | idx1 << 2), 8 nibbles per word
        lut = torch.tensor([4, 8, 12, 9, 13, 14], dtype=torch.int64, device=dev)
        nib = lut[torch.randint(0, 6, (Mr, K // 32, 8), device=dev, generator=gen)]
        shifts = (4 * torch.arange(8, device=dev, dtype=torch.int64))
        E = ((nib << shifts).sum(-1) & 0xFFFFFFFF).to(torch.int64)
        E = torch.where(E >= 2 ** 31, E - 2 ** 32, E).to(torch.int32).contiguous()
    else:
        A = torch.randint(-128, 128, (Mr, K), dtype=torch.int8, device=dev, generator=gen)
    gen.manual_seed(4321)  # every rank holds the same full B
    if kind == "bf16":
        B = (torch.randn((N, K), device=dev, generator=gen) / K ** 0.5).to(torch.bfloat16)
    elif kind == "w4a8":
        B = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=gen)
    else:
        B = torch.randint(-128, 128, (N, K) if layout == 0 else (K, N), dtype=torch.int8, device=dev,
                          generator=gen)
    out_dtype = {"s8": torch.int32, "w4a8": torch.int32, "s8_scaled": torch.bfloat16,
                 "bf16": torch.float32, "sp_s8": torch.int32}[kind]
    C = torch.empty((Mr, N), dtype=out_dtype, device=dev)
    rs = cs = None
    if kind == "s8_scaled":
        rs = torch.rand(Mr, device=dev, generator=gen) * 1.5 + 0.5
        cs = torch.rand(N, device=dev, generator=gen) * 9e-3 + 1e-3
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    # W4A8: split-K partials go to a workspace (zeroed once, kept zero by the kernel), so C is
    # stored once without a zeroing pass; the large-M kernel ignores it
    w4_ws = zx.w4a8_workspace(Mr, N, K, dev) if kind == "w4a8" else None

    def call(a, b, out):
        if kind == "s8":
            zx.gemm_s8(a, b, out, layout=layout, stream=stream)
        elif kind == "s8_scaled":
            zx.gemm_s8_scaled_bf16(a, b, rs, cs, out, layout=layout, stream=stream)
        elif kind == "w4a8":
            zx.gemm_w4a8_ws(a, b, w4_ws, out, stream=stream)
        elif kind == "sp_s8":
            zx.gemm_sp_s8(a, E, b, out, stream=stream)
        else:
            zx.gemm_bf16(a, b, out, layout=layout, stream=stream)

    for _ in range(args.warmup):
        flush.fill_(1)
        call(A, B, C)
    torch.cuda.synchronize(dev)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    sampler = ClockSampler(cvd.split(",")[local].strip() if cvd else str(local))
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    time.sleep(0.5)  # nvidia-smi start-up
    sampler.mark("t_start")
    for i in range(args.steps):
        flush.fill_(i & 0xFF)  # L2 flush, outside the timed events
        starts[i].record(stream)
        call(A, B, C)
        ends[i].record(stream)
    torch.cuda.synchronize(dev)
    timed_kernel = zx.last_kernel()  # what the library launched for the timed call
    sampler.mark("t_end")
    if ws > 1:
        dist.barrier()
    clocks = sampler.stop()
    kern_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(kern_ms)
    max_total_ms = max_over_ranks(total_ms, dev)
    ops_per_step = 2.0 * M * N * K
    value = ops_per_step * args.steps / (max_total_ms * 1e-3) / 1e12
    status = zx.device_status()

    # ---- e2e: same call with host buffers, copies inside the timed region ----
    A_h = A.cpu().pin_memory()
    B_h = B.cpu().pin_memory()
    C_h = torch.empty(C.shape, dtype=C.dtype).pin_memory()
    A_d, B_d = torch.empty_like(A), torch.empty_like(B)
    # int8 / bf16 NT go through the library's host-buffer entry (zx_gemm_s8_host / zx_gemm_bf16_host):
    # A and B stream in by ~1024-row blocks, and each L-shaped part of C that the blocks so far
    # complete is computed and streamed back at once. The others (per-row scales, sparse metadata,
    # packed s4, the NN layout) copy in, run one call and copy out in sequence.
    e2e_native = kind in ("s8", "bf16") and layout == 0
    e2e_chunks = "L-shaped shells of ~1024-row blocks (zx_gemm_*_host)" if e2e_native else "none"
    C_e2e = torch.empty_like(C)
    e2e_ms = []
    for i in range(args.e2e_steps + 1):
        if ws > 1:
            dist.barrier()
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record(stream)
        if e2e_native:
            zx.gemm_host(A_h, B_h, C_h, A_d, B_d, C_e2e, stream=stream)
        else:
            A_d.copy_(A_h, non_blocking=True)
            B_d.copy_(B_h, non_blocking=True)
            call(A_d, B_d, C_e2e)
            C_h.copy_(C_e2e, non_blocking=True)
        e_ev.record(stream)
        torch.cuda.synchronize(dev)
        if i > 0:  # first is warm-up
            e2e_ms.append(s_ev.elapsed_time(e_ev))
    # the host result equals the device-resident run's (float C: the blocks may run on other tile
    # shapes, so equal up to the fp32 accumulation order)
    e2e_diff = float((C_h.float() - C.cpu().float()).abs().max()) if out_dtype.is_floating_point else 0.0
    e2e_same = bool(torch.equal(C_h, C.cpu())) if not out_dtype.is_floating_point else e2e_diff <= 1e-3
    e2e_total_ms = max_over_ranks(sum(e2e_ms), dev) if e2e_ms else None
    e2e_value = ops_per_step * len(e2e_ms) / (e2e_total_ms * 1e-3) / 1e12 if e2e_ms else None

    # ---- optional: all-gather of the C slices over NVLink (NCCL), timed on its own ----
    allgather = None
    if args.allgather and ws > 1:
        for _ in range(4):
            dist.barrier()
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record(stream)
            full = gather_rows(C, M)
            e_ev.record(stream)
            torch.cuda.synchronize(dev)
        ag_ms = max_over_ranks(s_ev.elapsed_time(e_ev), dev)
        allgather = {"ms": ag_ms, "bytes_out_per_gpu": full.numel() * full.element_size(),
                     "algbw_gbs": full.numel() * full.element_size() / (ag_ms * 1e-3) / 1e9}
        del full
        # the same gather overlapped with the GEMM: chunk-interleaved row blocks, each block's
        # in-place all-gather issued as soon as it is computed (zoxide_b200.shard)
        P = args.ag_chunks
        if kind in ("s8", "s8_scaled", "bf16") and M % (ws * P) == 0 and Mr == M // ws:
            from zoxide_b200.shard import gemm_allgather_overlapped

            c_full = torch.empty((M, N), dtype=out_dtype, device=dev)

            def gemm_rows(a_rows, c_rows):
                call(a_rows, B, c_rows)

            ov = []
            for it in range(6):
                dist.barrier()
                flush.fill_(it & 0xFF)
                s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s_ev.record(stream)
                gemm_allgather_overlapped(gemm_rows, A, c_full, P)
                e_ev.record(stream)
                torch.cuda.synchronize(dev)
                if it >= 2:
                    ov.append(s_ev.elapsed_time(e_ev))
            ov_ms = max_over_ranks(statistics.median(ov), dev)
            # every rank must end with the same full C
            chk = torch.tensor([float(c_full.view(torch.int32).to(torch.int64).sum().item())], dtype=torch.float64,
                               device=dev)
            lo, hi = chk.clone(), chk.clone()
            dist.all_reduce(lo, op=dist.ReduceOp.MIN)
            dist.all_reduce(hi, op=dist.ReduceOp.MAX)
            gemm_ms = max_total_ms / args.steps
            allgather["overlapped"] = {
                "chunks": P, "ms": ov_ms, "gemm_then_gather_ms": gemm_ms + ag_ms,
                "saved_frac": 1.0 - ov_ms / (gemm_ms + ag_ms), "same_c_on_all_ranks": bool(lo.item() == hi.item()),
                "layout": "row block j*world + rank of M/(world*chunks) rows belongs to rank",
            }
            del c_full
        # the gather fused into the GEMM: each rank's kernel stores its tiles into every rank's
        # full C over NVLink (CUDA IPC peer mappings), no collective on the data path
        if kind == "s8" and layout == 0 and Mr == M // ws:
            from zoxide_b200.shard import PeerBuffers, gemm_allgather_fused

            c_full = torch.full((M, N), -1, dtype=torch.int32, device=dev)
            pb = PeerBuffers(c_full)
            try:
                fu = []
                for it in range(6):
                    dist.barrier()
                    flush.fill_(it & 0xFF)
                    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s_ev.record(stream)
                    gemm_allgather_fused(A, B, c_full, m0, pb, stream=stream)
                    e_ev.record(stream)
                    torch.cuda.synchronize(dev)
                    if it >= 2:
                        fu.append(s_ev.elapsed_time(e_ev))
                fu_kernel = zx.last_kernel()
                dist.barrier()  # every rank's stores into this rank's c_full have completed
                fu_ms = max_over_ranks(statistics.median(fu), dev)
                own_ok = bool(torch.equal(c_full[m0:m1], C))
                chk = torch.tensor([float(c_full.to(torch.int64).sum().item()), float(own_ok)],
                                   dtype=torch.float64, device=dev)
                lo, hi = chk.clone(), chk.clone()
                dist.all_reduce(lo, op=dist.ReduceOp.MIN)
                dist.all_reduce(hi, op=dist.ReduceOp.MAX)
                gemm_ms = max_total_ms / args.steps
                # fused roofline: the slower of the tensor work at the int8 peak (2x the measured
                # bf16 burst) and the peer bytes at the measured 770 GB/s NVLink peer-copy rate
                peer_bytes = (ws - 1) * C.numel() * C.element_size()
                t_mma = 2.0 * Mr * N * K / (2.0 * peaks()[0] * 1e12) * 1e3  # this rank's shard
                t_link = peer_bytes / 770e9 * 1e3
                allgather["fused"] = {
                    "ms": fu_ms, "gemm_then_gather_ms": gemm_ms + ag_ms,
                    "saved_frac": 1.0 - fu_ms / (gemm_ms + ag_ms),
                    "same_c_on_all_ranks": bool(lo[0].item() == hi[0].item()),
                    "own_rows_equal_gemm": bool(lo[1].item() == 1.0), "kernel": fu_kernel,
                    "peer_bytes_out_per_gpu": peer_bytes,
                    "roofline": {"bound": "nvlink" if t_link > t_mma else "tensor", "target_ms": max(t_link, t_mma),
                                 "tensor_ms": t_mma, "nvlink_ms": t_link, "frac": max(t_link, t_mma) / fu_ms,
                                 "nvlink_gbs": "770 measured peer copy per direction"},
                }
            finally:
                torch.cuda.synchronize(dev)
                dist.barrier()
                pb.close()
                dist.barrier()
            del c_full
    h2d = A.numel() * A.element_size() + B.numel() * B.element_size()
    d2h = C.numel() * C.element_size()

    bf16_peak, bf16_sus, hbm_peak, peak_src = peaks()
    # A kernel timed in a long back-to-back loop runs under the 1 kW power cap: compare it with
    # the sustained GEMM peak; a short burst with the burst peak. int8 tcgen05 issues at twice
    # the bf16 rate, so the int8 denominators are 2x the measured cuBLAS bf16 figures.
    sustained = total_ms > 1000.0 or "sw_power_cap" in (clocks.get("reasons") or [])
    bf16_den = bf16_sus if sustained else bf16_peak
    mean_s = statistics.mean(kern_ms) * 1e-3
    rank_ops = 2.0 * Mr * N * K
    alg_bytes = algorithmic_bytes(kind, Mr, N, K)
    kernel_name = "zx::" + timed_kernel
    traffic = None
    tf = ROOT / "profiles" / "ncu_traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(f"{args.workload}_M{Mr}")
    # tensor peak relative to bf16: int8 issues at 2x, 2:4-sparse int8 at 4x (dense-equivalent ops)
    mult = {"bf16": 1.0, "sp_s8": 4.0}.get(kind, 2.0)
    ridge = mult * bf16_den * 1e12 / (hbm_peak * 1e9)  # ops per byte where the roofs meet
    if rank_ops / alg_bytes < ridge:
        roof = {"bound": "hbm", "achieved": alg_bytes / mean_s / 1e9, "peak": hbm_peak, "unit": "GB/s",
                "peak_source": f"HBM copy bandwidth (of {peak_src})"}
    else:
        ach = rank_ops / mean_s / 1e12
        roof = {"bound": "tensor", "achieved": ach, "peak": mult * bf16_den,
                "unit": "TFLOP/s" if kind == "bf16" else "TOPS",
                "peak_source": f"{'' if kind == 'bf16' else f'{mult:.0f} x '}cuBLAS bf16 "
                               f"{'sustained' if sustained else 'burst'} {bf16_den:.0f} TFLOP/s (of {peak_src})",
                "frac_of_nominal": ach / (NOMINAL_BF16_TFLOPS if kind == "bf16" else
                                          2 * NOMINAL_INT8_TOPS if kind == "sp_s8" else NOMINAL_INT8_TOPS)}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof.update({"traffic": traffic, "kernel": kernel_name, "per_launch_ops": rank_ops,
                 "per_launch_algorithmic_bytes": alg_bytes})

    if rank == 0:
        cpu = None
        if ws == 1 and not args.no_cpu_baseline and kind in ("s8", "s8_scaled"):
            cpu = cpu_reference_sample(M, N, K, layout, target_s=args.ref_seconds)
            cpu.pop("seconds", None)
        unit = "TFLOP/s" if kind == "bf16" else "TOPS"
        line = {
            "metric": METRIC if args.workload == "s8_8192" else f"{describe(args.workload)}: {unit}",
            "value": value, "unit": unit, "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": max_total_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": {"s8": "int8", "s8_scaled": "int8", "w4a8": "int8 x int4", "bf16": "bf16",
                      "sp_s8": "int8 (2:4 sparse A)"}[kind],
            "data": "synthetic (torch seeded uniform integers / normal bf16); no reference dataset",
            "config": make_config(args, M, N, K, ws),
            "pct_of_nominal_peak": 100.0 * value / ((NOMINAL_BF16_TFLOPS if kind == "bf16" else NOMINAL_INT8_TOPS) * ws),
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_total_ms / len(e2e_ms) if e2e_ms else None,
                    "overlap": e2e_chunks, "same_result_as_device_run": e2e_same,
                    **({"max_abs_diff_vs_device_run": e2e_diff} if out_dtype.is_floating_point else {})},
            "allgather_c": allgather,
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
