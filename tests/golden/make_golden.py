#!/usr/bin/env python3
"""Write tests/golden/golden.json from an independent pure-Python restatement.

The reference (zig-ecosystem/zoxide) is Zig 0.16 and cannot be compiled or run here, so the
C oracle (oracle/zxo.c) is pinned against values computed by this script, which shares no code
with it: plain Python integers, `fractions` for exact rounding, numpy float32 for IEEE single
multiplies. Each block names the reference lines it restates. Run from the repo root:

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
from fractions import Fraction
from pathlib import Path

import numpy as np

OUT = Path(__file__).with_name("golden.json")
M32 = 0xFFFFFFFF


def xorshift(state: int) -> tuple[int, int]:
    """src/bench.zig:26-33 (x ^= x << 13; x ^= x >> 17; x ^= x << 5)."""
    x = state
    x ^= (x << 13) & M32
    x ^= x >> 17
    x ^= (x << 5) & M32
    return x, x


def draws(state: int, n: int) -> list[int]:
    out = []
    for _ in range(n):
        v, state = xorshift(state)
        out.append(v)
    return out


def s8(u: int) -> int:
    b = u & 0xFF
    return b - 256 if b >= 128 else b


def s4(u: int) -> int:
    nib = u & 0xF
    return nib - 16 if nib >= 8 else nib


def pack_s4(even: int, odd: int) -> int:
    """src/examples_abi.zig:54-56."""
    return (even & 0xF) | ((odd & 0xF) << 4)


def s4_at(buf: list[int], idx: int) -> int:
    """src/bench.zig:753-759."""
    byte = buf[idx // 2]
    nib = byte & 0xF if idx % 2 == 0 else byte >> 4
    return nib - 16 if nib >= 8 else nib


def prune24(rows: int, k: int, state: int):
    """src/bench.zig:1027-1058."""
    combos = [(0, 1), (0, 2), (0, 3), (1, 2), (1, 3), (2, 3)]
    dense = [[0] * k for _ in range(rows)]
    comp = [[0] * (k // 2) for _ in range(rows)]
    meta = [[0] * (k // 32) for _ in range(rows)]
    for r in range(rows):
        for kb in range(k // 32):
            word = 0
            for j in range(8):
                v, state = xorshift(state)
                c = combos[v % 6]
                for e in range(2):
                    v, state = xorshift(state)
                    val = s8(v)
                    dense[r][kb * 32 + 4 * j + c[e]] = val
                    comp[r][kb * 16 + 2 * j + e] = val
                word |= (c[0] | (c[1] << 2)) << (4 * j)
            meta[r][kb] = word
    return dense, comp, meta, state


def prune48(rows: int, k: int, state: int):
    """src/bench.zig:1178-1213: 4:8 pair-clustered s4 prune, one packS4 byte per surviving pair."""
    combos = [(0, 1), (0, 2), (0, 3), (1, 2), (1, 3), (2, 3)]
    dense = [[0] * k for _ in range(rows)]
    comp = [[0] * (k // 4) for _ in range(rows)]
    meta = [[0] * (k // 64) for _ in range(rows)]
    for r in range(rows):
        for kb in range(k // 64):
            word = 0
            for j in range(8):
                v, state = xorshift(state)
                c = combos[v % 6]
                pairs = []
                for _ in range(4):
                    v0, state = xorshift(state)
                    v1, state = xorshift(state)
                    pairs.append((s4(v0), s4(v1)))
                for e in range(2):
                    lo, hi = pairs[c[e]]
                    comp[r][kb * 16 + 2 * j + e] = pack_s4(lo, hi)
                for q in c:
                    dense[r][kb * 64 + 8 * j + 2 * q] = pairs[q][0]
                    dense[r][kb * 64 + 8 * j + 2 * q + 1] = pairs[q][1]
                word |= (c[0] | (c[1] << 2)) << (4 * j)
            meta[r][kb] = word
    return dense, comp, meta, state


def bf16_rne(x: float) -> int:
    """Exact round-to-nearest-even of a finite float32 value to bf16, via rationals."""
    f32 = np.float32(x)
    if f32 == 0:
        return int(np.array([f32]).view(np.uint32)[0] >> 16)
    bits = int(np.array([f32]).view(np.uint32)[0])
    sign = bits >> 31
    val = abs(Fraction(float(f32)))
    # bf16 has 8 significant bits: find exponent e with 2^e <= val < 2^(e+1)
    e = val.numerator.bit_length() - val.denominator.bit_length()
    if Fraction(2) ** e > val:
        e -= 1
    e = max(e, -126)  # subnormal range shares the minimum exponent
    ulp = Fraction(2) ** (e - 7)
    q, rem = divmod(val, ulp)
    q = int(q)
    if rem > ulp / 2 or (rem == ulp / 2 and q % 2 == 1):
        q += 1
    rounded = float(q * ulp)
    rb = int(np.array([np.float32(rounded)]).view(np.uint32)[0]) >> 16
    return rb | (sign << 15)


def main() -> None:
    g: dict = {}
    # Marsaglia (2003), "Xorshift RNGs", J. Stat. Softw. 8(14): xor32 from y=2463534242 prints
    # 723471715 first. Published known answer for the 13/17/5 triple.
    g["marsaglia_first"] = {"state": 2463534242, "first": draws(2463534242, 1)[0]}
    states = {"s8": 0x13579BDF, "s4": 0x0FDB9753, "sp_s8": 0xC0FFEE11, "bf16": 0x2468ACE0,
              "verify": 0xDEADBEEF, "marsaglia": 2463534242, "sp_s4": 0x5CA1AB1E}
    g["xorshift"] = {k: {"state": s, "draws": draws(s, 16)} for k, s in states.items()}

    # runImmaS8 data stream (src/bench.zig:653-655): low byte of each draw, A then B
    g["s8_first64"] = [s8(v) for v in draws(0x13579BDF, 64)]

    # runImmaS4 data stream (src/bench.zig:774-786): per byte a low then a high nibble draw
    d = draws(0x0FDB9753, 64)
    g["s4_packed_first32"] = [pack_s4(s4(d[2 * i]), s4(d[2 * i + 1])) for i in range(32)]
    g["pack_s4_table"] = [[pack_s4(e, o) for o in range(-8, 8)] for e in range(-8, 8)]
    g["s4_at_table"] = [s4_at([b], 0) for b in range(256)] + [s4_at([b], 1) for b in range(256)]

    dense, comp, meta, _ = prune24(2, 64, 0xC0FFEE11)
    g["prune24"] = {"state": 0xC0FFEE11, "rows": 2, "k": 64, "dense": dense, "comp": comp, "meta": meta}

    # runImmaSpS4 (src/bench.zig:1178-1226): pruned packed A, then dense B packed along N from
    # the same stream; C = pruned dense A (logical s4) x B (K x N logical s4)
    M, N, K = 2, 8, 128
    dense, comp, meta, st = prune48(M, K, 0x5CA1AB1E)
    bd = draws(st, K * N)
    Bp = [[pack_s4(s4(bd[2 * (k * N // 2 + i)]), s4(bd[2 * (k * N // 2 + i) + 1])) for i in range(N // 2)]
          for k in range(K)]
    Bl = [[s4_at(Bp[k], n) for n in range(N)] for k in range(K)]
    g["sp_s4_small"] = {"state": 0x5CA1AB1E, "M": M, "N": N, "K": K, "dense": dense, "comp": comp,
                        "meta": meta, "B_packed": Bp,
                        "C": [[sum(dense[m][k] * Bl[k][n] for k in range(K)) for n in range(N)]
                              for m in range(M)]}

    # runImmaS4 (src/bench.zig:767-786, check 840-856): A packed along K, B (K x N) packed
    # along N, one stream, A bytes first
    M = N = K = 16
    d = draws(0x0FDB9753, M * K + K * N)
    Ap = [[pack_s4(s4(d[m * K + 2 * i]), s4(d[m * K + 2 * i + 1])) for i in range(K // 2)] for m in range(M)]
    o = M * K
    Bp = [[pack_s4(s4(d[o + k * N + 2 * i]), s4(d[o + k * N + 2 * i + 1])) for i in range(N // 2)]
          for k in range(K)]
    g["s4s4_small"] = {"state": 0x0FDB9753, "n": M, "A_packed": Ap, "B_packed": Bp,
                       "C": [[sum(s4_at(Ap[m], k) * s4_at(Bp[k], n) for k in range(K)) for n in range(N)]
                             for m in range(M)]}

    # small exact GEMMs (NT and NN) from one stream: A (M x K) then B in storage order
    M, N, K = 8, 12, 64
    v = [s8(x) for x in draws(0x13579BDF, M * K + N * K)]
    A = [v[i * K:(i + 1) * K] for i in range(M)]
    Bnt = [v[M * K + n * K: M * K + (n + 1) * K] for n in range(N)]  # N x K
    Cnt = [[sum(A[m][k] * Bnt[n][k] for k in range(K)) for n in range(N)] for m in range(M)]
    Bnn = [v[M * K + k * N: M * K + (k + 1) * N] for k in range(K)]  # K x N
    Cnn = [[sum(A[m][k] * Bnn[k][n] for k in range(K)) for n in range(N)] for m in range(M)]
    g["gemm_small"] = {"M": M, "N": N, "K": K, "state": 0x13579BDF, "C_nt": Cnt, "C_nn": Cnn}

    # W4A8: A int8 (M x K), W s4 N x K packed along K low nibble first
    M, N, K = 4, 6, 32
    d = draws(0x0FDB9753, M * K + N * K)
    A = [[s8(d[m * K + k]) for k in range(K)] for m in range(M)]
    W = [[s4(d[M * K + n * K + k]) for k in range(K)] for n in range(N)]
    Wp = [[pack_s4(W[n][2 * i], W[n][2 * i + 1]) for i in range(K // 2)] for n in range(N)]
    g["w4a8_small"] = {"M": M, "N": N, "K": K, "A": A, "W_packed": Wp,
                       "C": [[sum(A[m][k] * W[n][k] for k in range(K)) for n in range(N)] for m in range(M)]}

    # the reference's 256-sample check draws (src/bench.zig:717-720) for n = 1024
    vs = draws(0xDEADBEEF, 8)
    g["verify_samples_n1024"] = [[x % (1024 * 1024) // 1024, x % (1024 * 1024) % 1024] for x in vs]

    # bf16 RNE on exact rationals, including ties
    vals = [0.0, 1.0, -1.0, 1.00390625, 1.005859375, 1.0078125, 3.14159265, -2.718281828,
            65504.0, 1e-3, 1e-30, 3.0e38, 1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -9, 0.1]
    g["bf16_rne"] = [[float(np.float32(x)), bf16_rne(x)] for x in vals]

    # scaled epilogue: bf16(((float)acc * rs) * cs), every step an IEEE float32 RNE op
    cases = [(0, 1.0, 1e-3), (1, 0.5, 1e-2), (-1, 1.9999, 0.0099), (134217728, 1.25, 0.00123),
             (-134217727, 0.75, 0.009), (16777217, 1.0, 1.0), (123456789, 1.5, 0.005),
             (-2 ** 31, 0.5, 0.001), (2 ** 31 - 1, 1.999, 0.00999)]
    out = []
    for acc, rs, cs in cases:
        f = np.float32(acc)
        t = np.float32(f * np.float32(rs))
        u = np.float32(t * np.float32(cs))
        out.append([acc, float(np.float32(rs)), float(np.float32(cs)), bf16_rne(float(u))])
    g["scaled_bf16"] = out

    OUT.write_text(json.dumps(g, separators=(",", ":")) + "\n")
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
