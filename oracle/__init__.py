"""CPU oracle for the quantised-GEMM path — TEST INFRASTRUCTURE ONLY.

A restatement of the reference's host-side generators and exact CPU GEMM check
(zig-ecosystem/zoxide src/bench.zig, src/examples_abi.zig) in plain C (zxo.c), loaded here
through ctypes. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm use it, and only as the checker or the timed CPU baseline; the product library never
calls into it.

Pinning: the reference is Zig 0.16 and cannot be built or run here, so parity is pinned by
Marsaglia's published xorshift32 output, hand-computed known answers, and golden fixtures
written by an independent pure-Python restatement (tests/golden/make_golden.py).
"""
from .zxo import *  # noqa: F401,F403
