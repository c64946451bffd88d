"""The CPU oracle against the golden fixtures and hand-computed known answers (no GPU).

The reference cannot run here (Zig toolchain absent), so the oracle is pinned by: Marsaglia's
published xorshift32 output, fixtures from the independent pure-Python restatement in
tests/golden/make_golden.py, and closed-form known answers. Planted mistakes are planted on the
CPU, in copies of oracle outputs, to show the checks catch them.
"""
import json
from pathlib import Path

import numpy as np
import pytest

G = json.loads((Path(__file__).parent / "golden" / "golden.json").read_text())


def test_marsaglia_published_value(zxo):
    v, _ = zxo.xorshift32(G["marsaglia_first"]["state"])
    assert v == 723471715 == G["marsaglia_first"]["first"]


@pytest.mark.parametrize("name", ["s8", "s4", "sp_s8", "bf16", "verify", "marsaglia", "sp_s4"])
def test_xorshift_streams(zxo, name):
    ent = G["xorshift"][name]
    r = zxo.Rng(ent["state"])
    assert [r.next() for _ in range(16)] == ent["draws"]


def test_state_zero_rejected(zxo):
    with pytest.raises(ValueError):
        zxo.Rng(0)
    assert zxo.state_from_seed(0) != 0


def test_s8_stream(zxo):
    a, _ = zxo.fill_s8(64, zxo.REF_STATE_S8)
    assert a.tolist() == G["s8_first64"]


def test_s4_stream_and_tables(zxo):
    a, _ = zxo.fill_s4_packed(32, zxo.REF_STATE_S4)
    assert a.tolist() == G["s4_packed_first32"]
    for i, e in enumerate(range(-8, 8)):
        for j, o in enumerate(range(-8, 8)):
            assert zxo.pack_s4(e, o) == G["pack_s4_table"][i][j]
    for b in range(256):
        buf = np.array([b], dtype=np.uint8)
        assert zxo.s4_at(buf, 0) == G["s4_at_table"][b]
        assert zxo.s4_at(buf, 1) == G["s4_at_table"][256 + b]
    # closed form: every nibble value round-trips through pack / unpack with sign extension
    for e in range(-8, 8):
        buf = np.array([zxo.pack_s4(e, -e - 1)], dtype=np.uint8)
        assert zxo.s4_at(buf, 0) == e and zxo.s4_at(buf, 1) == -e - 1


def test_prune24_matches_golden(zxo):
    p = G["prune24"]
    d, c, m, _ = zxo.prune24_s8(p["rows"], p["k"], p["state"])
    assert d.tolist() == p["dense"]
    assert c.tolist() == p["comp"]
    assert m.tolist() == p["meta"]


def test_prune24_structure_and_roundtrip(zxo):
    rows, k = 64, 256
    d, c, m, _ = zxo.prune24_s8(rows, k, 0xC0FFEE11)
    g = d.reshape(rows, k // 4, 4)
    # at most 2 non-zeros per group of 4 (a kept value may itself be 0)
    assert ((g != 0).sum(axis=2) <= 2).all()
    # every metadata nibble names two distinct indices in increasing order
    for w in m.ravel():
        for j in range(8):
            nib = (int(w) >> (4 * j)) & 0xF
            assert (nib & 3) < (nib >> 2)
    assert np.array_equal(zxo.decompress24_s8(c, m, rows, k), d)


def test_prune48_s4_matches_golden(zxo):
    """runImmaSpS4's pruned A, the dense packed B drawn after it, and their exact product."""
    p = G["sp_s4_small"]
    M, N, K = p["M"], p["N"], p["K"]
    d, c, m, st = zxo.prune48_s4(M, K, p["state"])
    assert d.tolist() == p["dense"]
    assert c.tolist() == p["comp"]
    assert m.tolist() == p["meta"]
    Bp = zxo.Rng(st).s4_packed((K, N // 2))
    assert Bp.tolist() == p["B_packed"]
    Bl = zxo.unpack_s4(Bp, (K, N))
    assert np.array_equal(zxo.decompress48_s4(c, m, M, K), d)
    assert zxo.gemm_s8(d, Bl, M, N, K, zxo.NN).tolist() == p["C"]


def test_prune48_s4_structure(zxo):
    rows, k = 32, 512
    d, c, m, _ = zxo.prune48_s4(rows, k, zxo.REF_STATE_SP_S4)
    pairs = d.reshape(rows, k // 8, 4, 2)
    # within each 8-wide chunk at most two 2-wide sub-chunks are non-zero
    assert ((np.abs(pairs).sum(axis=3) != 0).sum(axis=2) <= 2).all()
    for w in m.ravel()[:64]:
        for j in range(8):
            nib = (int(w) >> (4 * j)) & 0xF
            assert (nib & 3) < (nib >> 2)
    assert np.array_equal(zxo.decompress48_s4(c, m, rows, k), d)
    # a planted mistake: swapping the two kept bytes of one chunk changes the decompressed row
    bad = c.copy()
    bad[0, 0], bad[0, 1] = c[0, 1], c[0, 0]
    if c[0, 0] != c[0, 1]:
        assert not np.array_equal(zxo.decompress48_s4(bad, m, rows, k), d)


def test_s4s4_gemm_golden(zxo):
    """runImmaS4's stream: A packed along K, then B (K x N) packed along N; exact product."""
    p = G["s4s4_small"]
    n = p["n"]
    r = zxo.Rng(p["state"])
    Ap = r.s4_packed((n, n // 2))
    Bp = r.s4_packed((n, n // 2))
    assert Ap.tolist() == p["A_packed"] and Bp.tolist() == p["B_packed"]
    A = zxo.unpack_s4(Ap, (n, n))
    B = zxo.unpack_s4(Bp, (n, n))
    assert zxo.gemm_s8(A, B, n, n, n, zxo.NN).tolist() == p["C"]
    assert all(A[0, i] == zxo.s4_at(Ap, i) for i in range(n))


def test_small_gemm_golden(zxo):
    s = G["gemm_small"]
    M, N, K = s["M"], s["N"], s["K"]
    r = zxo.Rng(s["state"])
    A = r.s8((M, K))
    Bnt = r.s8((N, K))
    assert zxo.gemm_s8(A, Bnt, M, N, K, zxo.NT).tolist() == s["C_nt"]
    r = zxo.Rng(s["state"])
    A = r.s8((M, K))
    Bnn = r.s8((K, N))
    assert zxo.gemm_s8(A, Bnn, M, N, K, zxo.NN).tolist() == s["C_nn"]
    for row in range(M):
        for col in range(N):
            assert zxo.dot_s8(A, Bnn, N, K, zxo.NN, row, col) == s["C_nn"][row][col]


def test_w4a8_golden(zxo):
    s = G["w4a8_small"]
    A = np.array(s["A"], dtype=np.int8)
    W = np.array(s["W_packed"], dtype=np.uint8)
    assert zxo.gemm_w4a8(A, W, s["M"], s["N"], s["K"]).tolist() == s["C"]


def test_verify_sample_indices(zxo):
    r = zxo.Rng(zxo.REF_VERIFY_STATE)
    n = 1024
    got = []
    for _ in range(8):
        idx = r.next() % (n * n)
        got.append([idx // n, idx % n])
    assert got == G["verify_samples_n1024"]


def test_bf16_rne(zxo):
    for x, want in G["bf16_rne"]:
        assert zxo.f32_to_bf16(x) == want, x


def test_scaled_epilogue_golden(zxo):
    for acc, rs, cs, want in G["scaled_bf16"]:
        assert zxo.scale_to_bf16(acc, rs, cs) == want, (acc, rs, cs)


def test_known_answers(zxo):
    n = 128
    A = np.eye(n, dtype=np.int8)
    B = ((np.arange(n * n) % 255) - 127).astype(np.int8).reshape(n, n)
    assert np.array_equal(zxo.gemm_s8(A, B, n, n, n, zxo.NN), B.astype(np.int32))
    A = np.full((n, n), -128, dtype=np.int8)
    assert (zxo.gemm_s8(A, A, n, n, n, zxo.NT) == n * 16384).all()


def test_fast_gemm_equals_reference_loop(zxo):
    M, N, K = 96, 80, 4096
    r = zxo.Rng.from_seed(3)
    A = r.s8((M, K))
    B = r.s8((K, N))
    C = zxo.gemm_s8(A, B, M, N, K, zxo.NN)
    assert np.array_equal(zxo.ref_loop_s8(A, B, N, K, zxo.NN, 0, M).astype(np.int32), C)
    assert np.array_equal(C.astype(np.int64), A.astype(np.int64) @ B.astype(np.int64))


def test_sparse_and_w4a8_oracles_agree_with_dense(zxo):
    M, N, K = 64, 48, 256
    d, c, m, st = zxo.prune24_s8(M, K, 0xC0FFEE11)
    B = zxo.Rng(st).s8((N, K))
    assert np.array_equal(zxo.gemm_sp_s8(c, m, B, M, N, K, zxo.NT), zxo.gemm_s8(d, B, M, N, K, zxo.NT))
    r = zxo.Rng(zxo.REF_STATE_S4)
    A = r.s8((M, K))
    W = r.s4_packed((N, K // 2))
    W8 = np.array([[zxo.s4_at(W[n], k) for k in range(K)] for n in range(N)], dtype=np.int8)
    assert np.array_equal(zxo.gemm_w4a8(A, W, M, N, K), zxo.gemm_s8(A, W8, M, N, K, zxo.NT))


def test_checks_catch_planted_mistakes(zxo):
    """Mistakes planted on the CPU in a copy of the oracle's own output must be caught."""
    M = N = K = 256
    r = zxo.Rng.from_seed(11)
    A = r.s8((M, K))
    B = r.s8((N, K))
    C = zxo.gemm_s8(A, B, M, N, K, zxo.NT)
    assert zxo.check_samples_s8(A, B, C, M, N, K, zxo.NT)[0] == 0
    assert zxo.freivalds_s8(A, B, C, M, N, K, zxo.NT)
    bad = C.copy()
    bad[17, 201] += 1
    assert not zxo.freivalds_s8(A, B, bad, M, N, K, zxo.NT)
    bad = C.copy()
    bad[:] = -1  # the 0xff poison: "wrote nothing" must fail
    assert zxo.check_samples_s8(A, B, bad, M, N, K, zxo.NT)[0] == 256
    assert not zxo.freivalds_s8(A, B, bad, M, N, K, zxo.NT)


def test_uniform_and_normal_generators(zxo):
    r = zxo.Rng.from_seed(0)
    rs = r.uniform_f32(100000, 0.5, 2.0)
    assert rs.min() >= 0.5 and rs.max() < 2.0
    cs = r.uniform_f32(100000, 1e-3, 1e-2)
    assert cs.min() >= np.float32(1e-3) and cs.max() < np.float32(1e-2)
    b = r.normal_bf16(200000, 1.0 / np.sqrt(8192))
    f = (b.astype(np.uint32) << 16).view(np.float32)
    assert abs(f.mean()) < 1e-3 and abs(f.std() * np.sqrt(8192) - 1.0) < 0.02
