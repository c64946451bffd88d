"""W4A8: int8 activations x signed int4 weights packed along K, exact int32.

The weights use the reference's packS4 nibble order (src/examples_abi.zig:54-56) along K and are
unpacked to int8 in shared memory on the GPU; the oracle unpacks with the reference's s4At
(src/bench.zig:753-759). Full int4 range [-8, 7] and full int8 range, exact comparison.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(zxo, M, N, K, seed):
    r = zxo.Rng.from_seed(seed)
    A = r.s8((M, K))
    W = r.s4_packed((N, K // 2))
    return A, W


def _run(zx, A, W, M, N):
    dC = torch.full((M, N), -1, dtype=torch.int32, device="cuda")
    zx.gemm_w4a8(torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda(), dC)
    torch.cuda.synchronize()
    assert zx.device_status() == 0
    return dC.cpu().numpy()


@pytest.mark.parametrize(
    "M,N,K",
    [(256, 256, 128), (256, 256, 1024), (512, 768, 512), (1024, 1024, 1024), (300, 260, 96),
     (16, 1024, 2048), (1, 4, 32), (777, 1000, 224)],
)
def test_w4a8_exact(zx, zxo, M, N, K):
    A, W = _case(zxo, M, N, K, M + N + K)
    got = _run(zx, A, W, M, N)
    want = zxo.gemm_w4a8(A, W, M, N, K)
    if not np.array_equal(got, want):
        bad = np.argwhere(got != want)
        r, c = bad[0]
        pytest.fail(f"{len(bad)} mismatches; first ({r},{c}) want {want[r, c]} got {got[r, c]}")


@pytest.mark.parametrize("M,N,K", [(16, 256, 512), (1, 128, 1024), (16, 1000, 4096), (7, 28672 // 4, 8192),
                                   (32, 640, 2048), (33, 384, 1024), (64, 512, 512), (16, 128, 128)])
def test_w4a8_skinny_exact(zx, zxo, M, N, K):
    """M <= 64: weights unpacked into tensor memory, K split across SMs with exact int32 adds."""
    A, W = _case(zxo, M, N, K, 7 * M + N + K)
    got = _run(zx, A, W, M, N)
    assert np.array_equal(got, zxo.gemm_w4a8(A, W, M, N, K))


@pytest.mark.parametrize("M,N,K,path", [(16, 512, 1024, "gemm_w4s_kernel"), (64, 384, 512, "gemm_w4s_kernel"),
                                        (16, 512, 384, "gemm_tc2_kernel"), (65, 256, 512, "gemm_w4t_kernel"),
                                        (300, 256, 384, "gemm_tc2_kernel"), (4096, 512, 1024, "gemm_w4t_kernel")])
def test_w4a8_path_choice(zx, zxo, M, N, K, path):
    """K % 256 == 0: the weights-in-TMEM decode kernel for M <= 64, the weights-in-TMEM pair
    kernel above; other K: the pair kernel that unpacks into shared memory. All exact."""
    A, W = _case(zxo, M, N, K, 3 * M + K)
    got = _run(zx, A, W, M, N)
    assert zx.last_kernel().startswith(path), zx.last_kernel()
    assert np.array_equal(got, zxo.gemm_w4a8(A, W, M, N, K))


@pytest.fixture(params=[0, 2, 4], ids=["auto", "smem_pair", "tmem_pair"])
def w4policy(request, zx):
    """Automatic choice, the pair kernel that unpacks into shared memory (policy 2), and the
    weights-in-TMEM pair kernel at any M (policy 4)."""
    zx.set_kernel_policy(request.param)
    yield request.param
    zx.set_kernel_policy(0)


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (512, 768, 1024), (300, 1000, 512), (1, 260, 256),
                                   (777, 1000, 768), (2048, 4096, 2048), (129, 132, 512)])
def test_w4a8_large_m_paths_exact(zx, zxo, w4policy, M, N, K):
    """Every large-M path against the oracle, exact: full and partial weight tiles (N = 1000,
    132: half a CTA's rows out of range) and activation tiles (M = 300, 129: the second CTA of a
    pair without rows), several tiles per CTA pair (2048 x 4096), K of one to eight stages."""
    A, W = _case(zxo, M, N, K, 13 * M + N + K + w4policy)
    got = _run(zx, A, W, M, N)
    want = zxo.gemm_w4a8(A, W, M, N, K)
    if not np.array_equal(got, want):
        bad = np.argwhere(got != want)
        r, c = bad[0]
        pytest.fail(f"{zx.last_kernel()}: {len(bad)} mismatches; first ({r},{c}) want {want[r, c]} got {got[r, c]}")


def test_w4a8_skinny_back_to_back(zx, zxo):
    """Split-K accumulates into C: a second launch must start from zero again."""
    M, N, K = 16, 2048, 4096
    A, W = _case(zxo, M, N, K, 99)
    dA, dW = torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda()
    dC = torch.full((M, N), 12345, dtype=torch.int32, device="cuda")
    for _ in range(3):
        zx.gemm_w4a8(dA, dW, dC)
    torch.cuda.synchronize()
    assert np.array_equal(dC.cpu().numpy(), zxo.gemm_w4a8(A, W, M, N, K))


def test_w4a8_nibble_extremes(zx, zxo):
    """Every (even, odd) nibble pair, -8 and 7 in both positions: sign extension and order."""
    M, N, K = 256, 256, 512
    A = np.zeros((M, K), dtype=np.int8)
    A[np.arange(M), np.arange(M) % K] = 1  # row m picks weight column k = m
    A[:, 1] = -128                          # and every row also multiplies k = 1 by -128
    vals = np.array([[zxo.pack_s4(e, o) for o in range(-8, 8)] for e in range(-8, 8)], dtype=np.uint8).ravel()
    W = np.resize(vals, (N, K // 2)).astype(np.uint8)
    got = _run(zx, A, W, M, N)
    assert np.array_equal(got, zxo.gemm_w4a8(A, W, M, N, K))


def test_w4a8_reference_stream(zx, zxo):
    """Activations and weights from the reference's s4 state (0x0fdb9753) draw order."""
    M, N, K = 512, 512, 1024
    r = zxo.Rng(zxo.REF_STATE_S4)
    A = r.s8((M, K))
    W = r.s4_packed((N, K // 2))
    got = _run(zx, A, W, M, N)
    assert np.array_equal(got, zxo.gemm_w4a8(A, W, M, N, K))


@pytest.mark.parametrize("M,N,K", [(16, 128, 8192), (16, 256, 512), (7, 28672 // 4, 8192), (32, 1000, 2048),
                                   (17, 640, 4096), (1, 384, 1024), (16, 28672, 8192)])
def test_w4a8_workspace_exact(zx, zxo, M, N, K):
    """Workspace split-K (partials + last-arriver sum): exact against the oracle, C poisoned,
    three calls in a row on one workspace (the counters must come back to zero), including a
    tile shared by 32 CTAs (N = 128, K = 8192) and the M = 16 decode shape."""
    A, W = _case(zxo, M, N, K, 11 * M + N + K)
    want = zxo.gemm_w4a8(A, W, M, N, K)
    dA, dW = torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda()
    ws = zx.w4a8_workspace(M, N, K)
    assert zx.w4a8_workspace_bytes(M, N, K) > 0
    for _ in range(3):
        dC = torch.full((M, N), -1, dtype=torch.int32, device="cuda")
        zx.gemm_w4a8_ws(dA, dW, ws, dC)
        torch.cuda.synchronize()
        assert zx.device_status() == 0
        assert zx.last_kernel().startswith("gemm_w4s_kernel")
        assert np.array_equal(dC.cpu().numpy(), want)
    # layout: 2 x CTAs partial slots of NX x 128 int32, then one counter per 128-column tile
    nx = 16 if M <= 16 else 32
    tiles = (N + 127) // 128
    ctas = min(tiles * (K // 256), zx.sm_count())
    counters = ws[2 * ctas * nx * 128 * 4:].view(torch.int32)[:tiles]
    assert int(counters.abs().sum()) == 0  # every counter is back at zero


def test_w4a8_workspace_rules(zx, zxo):
    """M > 32 needs no workspace (zero-and-add or pair kernel); a too-small one is rejected."""
    assert zx.w4a8_workspace_bytes(64, 256, 512) == 0
    M, N, K = 128, 256, 512
    assert zx.w4a8_workspace_bytes(M, N, K) == 0
    A, W = _case(zxo, M, N, K, 5)
    dA, dW = torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda()
    got = zx.gemm_w4a8_ws(dA, dW, torch.zeros(16, dtype=torch.uint8, device="cuda"))
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), zxo.gemm_w4a8(A, W, M, N, K))
    M64 = 64  # runs as zx_gemm_w4a8 (zero C, add into it) and ignores the workspace
    A, W = _case(zxo, M64, N, 4096, 8)
    got = zx.gemm_w4a8_ws(torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda(),
                          torch.zeros(16, dtype=torch.uint8, device="cuda"))
    torch.cuda.synchronize()
    assert zx.last_kernel().startswith("gemm_w4s_kernel")
    assert np.array_equal(got.cpu().numpy(), zxo.gemm_w4a8(A, W, M64, N, 4096))
    M = 16
    A, W = _case(zxo, M, N, K, 6)
    dA, dW = torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda()
    small = torch.zeros(zx.w4a8_workspace_bytes(M, N, K) - 16, dtype=torch.uint8, device="cuda")
    with pytest.raises(zx.ZxError, match="workspace"):
        zx.gemm_w4a8_ws(dA, dW, small)


@pytest.mark.slow
@pytest.mark.parametrize("M", [4096, 16])
def test_w4a8_config3_full_size(zx, zxo, M):
    """BASELINE config 3 shape (N=28672, K=8192) at M=4096 and the M=16 decode shape."""
    N, K = 28672, 8192
    A, W = _case(zxo, M, N, K, 3)
    got = _run(zx, A, W, M, N)
    rows = sorted(r for r in {0, 1, 127, 128, 255, M // 2, M - 1} if r < M)
    for r0 in rows:
        want = zxo.gemm_w4a8(np.ascontiguousarray(A[r0:r0 + 1]), W, 1, N, K)
        assert np.array_equal(got[r0], want[0]), f"row {r0}"
    # a column block through every row (exercises every M tile)
    cols = slice(28416, 28672)
    want = zxo.gemm_w4a8(A, np.ascontiguousarray(W[cols]), M, 256, K)
    assert np.array_equal(got[:, cols], want)
