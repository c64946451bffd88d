"""int8 x int8 -> int32 GEMM on the B200 through the C ABI, bit-exact against the oracle.

Mirrors the reference's own check (src/bench.zig:647-741): seeded xorshift data over the full
int8 range, C poisoned with 0xff before the launch, exact integer comparison (no tolerance).
Small and ragged cases compare every element against the oracle's exact GEMM; full-size cases
use the reference's 256-sample check plus an exact Freivalds identity C x == A (op(B) x).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(zx, A, B, M, N, K, layout):
    dA = torch.from_numpy(A).cuda()
    dB = torch.from_numpy(B).cuda()
    dC = torch.full((M, N), -1, dtype=torch.int32, device="cuda")  # 0xff poison
    zx.gemm_s8(dA, dB, dC, layout=layout)
    torch.cuda.synchronize()
    assert zx.device_status() == 0
    return dC.cpu().numpy()


def _data(zxo, M, N, K, layout, state):
    r = zxo.Rng(state)
    A = r.s8((M, K))
    B = r.s8((N, K) if layout == zxo.NT else (K, N))
    return A, B


@pytest.mark.parametrize("layout", [0, 1], ids=["NT", "NN"])
@pytest.mark.parametrize(
    "M,N,K",
    [
        (128, 256, 128),     # one tile, one k-block
        (128, 256, 1024),    # one tile, deep K
        (256, 512, 512),     # 2 x 2 tiles
        (1024, 1024, 1024),
        (384, 768, 2048),
        (1024, 8192, 512),   # an 8-GPU shard of 8192^3: 224-wide pair tiles
        (2048, 3008, 256),   # 224-wide tiles with a ragged last column tile
    ],
)
def test_exact_vs_oracle(zx, zxo, policy, M, N, K, layout):
    A, B = _data(zxo, M, N, K, layout, zxo.state_from_seed(M * 7 + N * 3 + K + layout))
    got = _run(zx, A, B, M, N, K, layout)
    want = zxo.gemm_s8(A, B, M, N, K, layout)
    if not np.array_equal(got, want):
        bad = np.argwhere(got != want)
        r, c = bad[0]
        pytest.fail(f"{len(bad)} mismatches; first at ({r},{c}) want {want[r, c]} got {got[r, c]}")


@pytest.mark.parametrize("layout", [0, 1], ids=["NT", "NN"])
@pytest.mark.parametrize(
    "M,N,K",
    [
        (1, 16, 16),        # smallest legal problem
        (100, 260, 144),    # ragged M, N and K tails
        (129, 4, 32),       # one row past a tile, narrowest C
        (16, 28672 // 8, 8192 // 4),  # skinny decode-like M
        (777, 1000, 208),
    ],
)
def test_ragged_exact(zx, zxo, policy, M, N, K, layout):
    if layout == 1 and N % 16:
        pytest.skip("NN needs N % 16 == 0")
    A, B = _data(zxo, M, N, K, layout, zxo.state_from_seed(M + N + K))
    got = _run(zx, A, B, M, N, K, layout)
    want = zxo.gemm_s8(A, B, M, N, K, layout)
    assert np.array_equal(got, want)


def test_extreme_values(zx, zxo, policy):
    """All -128 x all -128: every output is K * 16384 (max-magnitude products, sign handling)."""
    M, N, K = 256, 256, 4096
    A = np.full((M, K), -128, dtype=np.int8)
    B = np.full((N, K), -128, dtype=np.int8)
    got = _run(zx, A, B, M, N, K, 0)
    assert (got == K * 16384).all()
    B[:, ::2] = 127  # mix signs: half the products are -16256
    got = _run(zx, A, B, M, N, K, 0)
    assert (got == (K // 2) * 16384 + (K // 2) * (-128 * 127)).all()


def test_identity_ramp(zx, zxo, policy):
    """A = I, B = ramp: C must reproduce op(B) exactly (catches transposed / swizzled operands)."""
    n = 256
    A = np.eye(n, dtype=np.int8)
    Bnn = ((np.arange(n * n) % 255) - 127).astype(np.int8).reshape(n, n)  # K x N
    got = _run(zx, A, Bnn, n, n, n, 1)
    assert np.array_equal(got, Bnn.astype(np.int32))
    Bnt = np.ascontiguousarray(Bnn.T)  # N x K, op(B) = Bnt^T = Bnn
    got = _run(zx, A, Bnt, n, n, n, 0)
    assert np.array_equal(got, Bnn.astype(np.int32))


def test_reference_replay_square(zx, zxo):
    """The reference's exact data stream (state 0x13579bdf, A then B, NN) and 256-sample check."""
    n = 1024
    r = zxo.Rng(zxo.REF_STATE_S8)
    A = r.s8((n, n))
    B = r.s8((n, n))
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dC = torch.full((n, n), -1, dtype=torch.int32, device="cuda")
    zx.imma_s8(dA, dB, dC, n)
    torch.cuda.synchronize()
    got = dC.cpu().numpy()
    bad, first = zxo.check_samples_s8(A, B, got, n, n, n, zxo.NN)
    assert bad == 0, f"reference check: {bad}/256 wrong, first {first}"
    assert np.array_equal(got, zxo.gemm_s8(A, B, n, n, n, zxo.NN))


@pytest.mark.slow
@pytest.mark.parametrize("layout", [0, 1], ids=["NT", "NN"])
def test_full_size_8192(zx, zxo, policy, layout):
    """BASELINE config 2 shape: 256 reference samples + exact Freivalds identity."""
    M = N = K = 8192
    A, B = _data(zxo, M, N, K, layout, zxo.state_from_seed(0))
    got = _run(zx, A, B, M, N, K, layout)
    bad, first = zxo.check_samples_s8(A, B, got, M, N, K, layout)
    assert bad == 0, f"{bad}/256 samples wrong, first {first}"
    assert zxo.freivalds_s8(A, B, got, M, N, K, layout)
    # rows at tile and raster-group boundaries, in full
    rows = [0, 127, 128, 2047, 2048, 4095, 8191]
    for r0 in rows:
        ref = zxo.ref_loop_s8(A, B, N, K, layout, r0, r0 + 1)
        assert np.array_equal(got[r0].astype(np.int64), ref[0]), f"row {r0}"


@pytest.mark.parametrize("K", [128, 384, 1152])
def test_many_tiles_short_k(zx, zxo, policy, K):
    """More tiles than CTA pairs (several tiles per pair) with K shorter than, near and beyond the
    operand ring: accumulator hand-over between consecutive tiles of one pair, including tiles
    whose whole K loop is shorter than the ring."""
    M, N = 2560, 4096
    A, B = _data(zxo, M, N, K, 0, zxo.state_from_seed(K + 5))
    got = _run(zx, A, B, M, N, K, 0)
    want = zxo.gemm_s8(A, B, M, N, K, 0)
    assert np.array_equal(got, want)


def test_back_to_back_launches(zx, zxo, policy):
    """Two launches on one stream reuse TMEM / barriers correctly and both results are exact."""
    M, N, K = 512, 512, 512
    A, B = _data(zxo, M, N, K, 0, 99)
    want = zxo.gemm_s8(A, B, M, N, K, 0)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    outs = [torch.full((M, N), -1, dtype=torch.int32, device="cuda") for _ in range(3)]
    for o in outs:
        zx.gemm_s8(dA, dB, o)
    torch.cuda.synchronize()
    for o in outs:
        assert np.array_equal(o.cpu().numpy(), want)


@pytest.mark.parametrize("chunks", [1, 3, 8])
def test_pipelined_host_gemm(zx, zxo, chunks):
    """zoxide_b200.host: pinned host A, B -> device in row chunks, each chunk's GEMM as its rows
    arrive, C rows back as they are computed; exact against the oracle for any chunking."""
    from zoxide_b200.host import pipelined_host_gemm

    M, N, K = 1000, 768, 512
    A, B = _data(zxo, M, N, K, 0, zxo.state_from_seed(chunks + 77))
    a_h, b_h = torch.from_numpy(A).pin_memory(), torch.from_numpy(B).pin_memory()
    c_h = torch.full((M, N), -1, dtype=torch.int32).pin_memory()
    a_d, b_d = torch.empty((M, K), dtype=torch.int8, device="cuda"), torch.empty((N, K), dtype=torch.int8, device="cuda")
    c_d = torch.empty((M, N), dtype=torch.int32, device="cuda")
    pipelined_host_gemm(lambda a, b, c: zx.gemm_s8(a, b, c), a_h, b_h, c_h, a_d, b_d, c_d, chunks=chunks)
    torch.cuda.synchronize()
    assert np.array_equal(c_h.numpy(), zxo.gemm_s8(A, B, M, N, K, 0))


def test_concurrent_threads_and_streams(zx, zxo):
    """Four host threads, each with its own CUDA stream, call the C ABI at once (the per-device
    caches are mutex-guarded, errors are per thread): every result exact, status clean."""
    import threading

    M, N, K = 1024, 1280, 768
    cases = [_data(zxo, M, N, K, 0, 4242 + i) for i in range(4)]
    results, errors = [None] * 4, []

    def worker(i):
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                A, B = cases[i]
                dA, dB = torch.from_numpy(A).cuda(non_blocking=False), torch.from_numpy(B).cuda()
                for _ in range(3):
                    C = zx.gemm_s8(dA, dB, stream=s)
                s.synchronize()
                results[i] = C.cpu().numpy()
        except Exception as e:  # surfaced below
            errors.append(repr(e))

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not errors, errors
    for i, (A, B) in enumerate(cases):
        assert np.array_equal(results[i], zxo.gemm_s8(A, B, M, N, K, 0)), f"thread {i}"
    assert zx.device_status() == 0


@pytest.mark.slow
@pytest.mark.parametrize("M", [1024, 2048], ids=["shard8", "shard4"])
def test_shard_shapes_exact(zx, zxo, M):
    """One GPU's rows of 8192^3 at 8 and 4 GPUs on the automatic tile choice (256 x 464 pair
    tiles: 17 full tiles and one 304-column tile per row block): 256 reference samples, Freivalds,
    and the first row block's 256 rows in full (every tile seam and every 16-column tail piece)."""
    N = K = 8192
    A, B = _data(zxo, M, N, K, 0, zxo.state_from_seed(M))
    got = _run(zx, A, B, M, N, K, 0)
    kernel = zx.last_kernel()
    assert "256x464 tiles" in kernel, kernel
    bad, first = zxo.check_samples_s8(A, B, got, M, N, K, 0)
    assert bad == 0, f"{bad}/256 samples wrong, first {first} ({kernel})"
    assert zxo.freivalds_s8(A, B, got, M, N, K, 0), kernel
    rows = np.ascontiguousarray(A[:256])
    ref = zxo.gemm_s8(rows, B, 256, N, K, 0)
    assert np.array_equal(got[:256], ref), kernel


@pytest.mark.parametrize("M,N,K", [(256, 464, 128), (512, 928, 256), (300, 920, 160), (1000, 1396, 384),
                                   (256, 452, 64), (40, 2000, 96)])
def test_464_tiles_tail_piece(zx, zxo, M, N, K):
    """256 x 464 pair tiles: the hi half's last 16 columns of each tile go out with plain stores
    (a 32-column TMA box would overwrite the next tile). Tiles that end exactly on N, tails cut by
    N inside the piece (920 = 464 + 456, 1396 = 3 x 464 + 4, 452), ragged M, every element."""
    zx.set_kernel_policy(6)
    try:
        A, B = _data(zxo, M, N, K, 0, zxo.state_from_seed(M * 7 + N + K))
        got = _run(zx, A, B, M, N, K, 0)
        kernel = zx.last_kernel()
        assert "256x464 tiles" in kernel, kernel
        assert np.array_equal(got, zxo.gemm_s8(A, B, M, N, K, 0)), kernel
    finally:
        zx.set_kernel_policy(0)


@pytest.mark.parametrize("M,N,K,bn", [(1024, 1024, 1024, 64), (2048, 1024, 512, 128), (300, 200, 256, 64),
                                      (128, 28672, 512, 256)])
def test_one_sm_tile_widths(zx, zxo, M, N, K, bn):
    """The one-SM kernel's width choice (64 / 128 / 256 columns by operand bytes per wave), every
    element exact, int32 and the scaled-bf16 epilogue."""
    zx.set_kernel_policy(1)
    try:
        A, B = _data(zxo, M, N, K, 0, zxo.state_from_seed(M + N + bn))
        got = _run(zx, A, B, M, N, K, 0)
        kernel = zx.last_kernel()
        assert np.array_equal(got, zxo.gemm_s8(A, B, M, N, K, 0)), kernel
        assert f"128x{bn} tiles" in kernel, kernel
        r = zxo.Rng.from_seed(bn)
        rs, cs = r.uniform_f32(M, 0.5, 2.0), r.uniform_f32(N, 1e-3, 1e-2)
        dO = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        zx.gemm_s8_scaled_bf16(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), torch.from_numpy(rs).cuda(),
                               torch.from_numpy(cs).cuda(), dO)
        torch.cuda.synchronize()
        want = zxo.gemm_s8_scaled_bf16(A, B, rs, cs, N, K, 0, 0, M)
        assert np.array_equal(dO.view(torch.int16).cpu().numpy().view(np.uint16), want), zx.last_kernel()
    finally:
        zx.set_kernel_policy(0)
