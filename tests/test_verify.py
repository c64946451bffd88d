"""The bench's result checker (zoxide_b200.verify) against the oracle, on CPU.

verify.py re-states the reference's 256-sample check (src/bench.zig:712-740, :384-413) with torch
on the host so that bench.py can check the C of every timed run; here it is pinned to the oracle's
own restatement (oracle/zxo.c) and shown to catch planted mistakes.
"""
import numpy as np
import pytest
import torch

from zoxide_b200 import verify as v


def test_sample_positions_match_oracle(zxo):
    # the oracle's check counts mismatches at the reference's positions: plant one at each
    M, N, K = 96, 80, 32
    rng = zxo.Rng.from_seed(3)
    A = rng.s8((M, K))
    B = rng.s8((N, K))
    C = zxo.gemm_s8(A, B, M, N, K, zxo.NT)
    for r, c in v.sample_positions(M, N, 256)[:8]:
        bad = C.copy()
        bad[r, c] += 1
        assert zxo.check_samples_s8(A, B, bad, M, N, K, zxo.NT)[0] >= 1
    assert v.xorshift32(2463534242)[0] == 723471715  # Marsaglia's published value


@pytest.mark.parametrize("layout", [0, 1])
def test_s8_checks(zxo, layout):
    M, N, K = 200, 144, 96
    rng = zxo.Rng.from_seed(5)
    A = rng.s8((M, K))
    B = rng.s8((N, K) if layout == 0 else (K, N))
    C = zxo.gemm_s8(A, B, M, N, K, layout)
    At, Bt, Ct = torch.from_numpy(A), torch.from_numpy(B), torch.from_numpy(C)
    res = v.check_result("s8", At, Bt, Ct, layout)
    assert res["ok"] and res["bad"] == 0 and res["freivalds"]
    bad = Ct.clone()
    bad[M - 1, 3] -= 7  # one element off, usually outside the 256 samples: Freivalds catches it
    assert not v.freivalds("s8", At, Bt, bad, layout, rounds=4)
    poisoned = torch.full_like(Ct, -1)
    assert v.check_samples("s8", At, Bt, poisoned, layout)["bad"] > 200


def test_w4a8_checks(zxo):
    M, N, K = 64, 96, 128
    rng = zxo.Rng.from_seed(7)
    A = rng.s8((M, K))
    W = rng.s4_packed((N, K // 2))
    C = zxo.gemm_w4a8(A, W, M, N, K)
    Wt = torch.from_numpy(W)
    assert np.array_equal(v.unpack_s4_rows(Wt, slice(0, N)).numpy(), zxo.unpack_s4(W, (N, K)))
    res = v.check_result("w4a8", torch.from_numpy(A), Wt, torch.from_numpy(C))
    assert res["ok"]
    bad = torch.from_numpy(C).clone()
    bad[10, 10] += 1
    assert not v.freivalds("w4a8", torch.from_numpy(A), Wt, bad, rounds=4)


def test_sparse_checks(zxo):
    M, N, K = 128, 64, 256
    rng = zxo.Rng.from_seed(9)
    dense, comp, meta = rng.prune24_s8(M, K)
    B = rng.s8((N, K))
    C = zxo.gemm_sp_s8(comp, meta, B, M, N, K, zxo.NT)
    ct, mt = torch.from_numpy(comp), torch.from_numpy(meta.view(np.int32))
    got = v.decompress24_rows(ct, mt, list(range(M)), K).numpy()
    assert np.array_equal(got, dense.astype(np.int16))
    res = v.check_result("sp_s8", ct, torch.from_numpy(B), torch.from_numpy(C), 0, meta=mt)
    assert res["ok"]


def test_scaled_bf16_checks(zxo):
    M, N, K = 64, 48, 64
    rng = zxo.Rng.from_seed(11)
    A = rng.s8((M, K))
    B = rng.s8((N, K))
    rs = rng.uniform_f32(M, 0.5, 2.0)
    cs = rng.uniform_f32(N, 1e-3, 1e-2)
    C = zxo.gemm_s8_scaled_bf16(A, B, rs, cs, N, K, zxo.NT, 0, M)  # uint16 bf16 bits
    Ct = torch.from_numpy(C.view(np.int16)).view(torch.bfloat16)
    res = v.check_result("s8_scaled", torch.from_numpy(A), torch.from_numpy(B), Ct, 0,
                         rs=torch.from_numpy(rs), cs=torch.from_numpy(cs))
    assert res["ok"] and res["full_rows_exact"]
    bad = Ct.clone()
    bad[M - 1] = 0
    assert not v.check_result("s8_scaled", torch.from_numpy(A), torch.from_numpy(B), bad, 0,
                              rs=torch.from_numpy(rs), cs=torch.from_numpy(cs))["ok"]


def test_bf16_checks(zxo):
    M, N, K = 300, 64, 128
    g = torch.Generator().manual_seed(0)
    A = (torch.randn((M, K), generator=g) / K ** 0.5).to(torch.bfloat16)
    B = (torch.randn((N, K), generator=g) / K ** 0.5).to(torch.bfloat16)
    C = (A.double() @ B.double().t()).float()
    res = v.check_result("bf16", A, B, C)
    assert res["ok"] and res["rel_frobenius_256_rows"] < 1e-6
    assert not v.check_result("bf16", A, B, torch.full_like(C, float("nan")))["ok"]


def test_s4s4_checks(zxo):
    # imma_s4's operands: A n x n s4 packed along K, B K x N s4 packed along N
    n = 64
    rng = zxo.Rng.from_seed(13)
    A = rng.s4_packed((n, n // 2))
    B = rng.s4_packed((n, n // 2))
    a = zxo.unpack_s4(A, (n, n)).astype(np.int64)
    b = zxo.unpack_s4(B, (n, n)).astype(np.int64)  # row k holds op(B)[k, 0..n)
    C = torch.from_numpy((a @ b).astype(np.int32))
    res = v.check_result("s4s4", torch.from_numpy(A), torch.from_numpy(B), C, 1)
    assert res["ok"]
    bad = C.clone()
    bad[n - 1, n - 2] += 3
    assert not v.freivalds("s4s4", torch.from_numpy(A), torch.from_numpy(B), bad, 1, rounds=4)


def test_sp_s4_checks(zxo):
    # imma_sp_s4's operands: 4:8 pair-clustered s4 A + metadata, B K x N s4 packed along N
    M, N, K = 64, 48, 128
    rng = zxo.Rng.from_seed(17)
    dense, comp, meta = rng.prune48_s4(M, K)
    Bp = rng.s4_packed((K, N // 2))
    ct, mt = torch.from_numpy(comp), torch.from_numpy(meta.view(np.int32))
    got = v.decompress48_rows(ct, mt, list(range(M)), K).numpy()
    assert np.array_equal(got, dense.astype(np.int16))
    assert np.array_equal(got, zxo.decompress48_s4(comp, meta, M, K).astype(np.int16))
    C = torch.from_numpy(zxo.gemm_s8(dense, zxo.unpack_s4(Bp, (K, N)), M, N, K, zxo.NN))
    res = v.check_result("sp_s4", ct, torch.from_numpy(Bp), C, 1, meta=mt)
    assert res["ok"] and res["freivalds"]
    bad = C.clone()
    bad[M - 1, 0] -= 1
    assert not v.check_result("sp_s4", ct, torch.from_numpy(Bp), bad, 1, meta=mt, freivalds_rounds=4)["ok"]
