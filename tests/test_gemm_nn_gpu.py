"""The reference's own operand layouts on the fast kernels (zx_gemm_sp_s8_nn, zx_gemm_s4s4_nn,
zx_gemm_sp_s4_nn):
a layout pass into a caller workspace, then the K-major tcgen05 kernels. Data are the reference
bench's own streams (runImmaSpS8, src/bench.zig:1027-1063; runImmaS4, src/bench.zig:767-786;
runImmaSpS4, src/bench.zig:1178-1226) and
the results are compared with the oracle element for element (exact int32)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _diff(got, want):
    if np.array_equal(got, want):
        return ""
    bad = np.argwhere(got != want)
    r, c = bad[0]
    return f"{len(bad)} mismatches; first at ({r},{c}) want {want[r, c]} got {got[r, c]}"


def _ws(zx, op, M, N, K, fill=0x5A):
    # filled with a pattern: the pass must overwrite every byte it uses
    return torch.full((zx.nn_workspace_bytes(op, M, N, K),), fill, dtype=torch.uint8, device="cuda")


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (512, 512, 512), (768, 768, 768), (256, 1040, 512),
                                   (2560, 4096, 512)])
def test_sp_s8_nn_exact(zx, zxo, M, N, K):
    r = zxo.Rng(zxo.REF_STATE_SP_S8)
    dense, comp, meta = r.prune24_s8(M, K)
    B = r.s8((K, N))  # row-major K x N, the reference layout
    want = zxo.gemm_s8(dense, B, M, N, K, zxo.NN)
    dC = torch.full((M, N), -1, dtype=torch.int32, device="cuda")
    zx.gemm_sp_s8_nn(_dev(comp), _dev(meta.view(np.int32)), _dev(B), _ws(zx, zx.NN_SP_S8, M, N, K), dC)
    torch.cuda.synchronize()
    assert zx.device_status() == 0
    got = dC.cpu().numpy()
    assert not _diff(got, want), _diff(got, want)


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (256, 256, 256), (640, 640, 640), (16, 512, 1024),
                                   (300, 208, 192), (1024, 2048, 4096)])
def test_s4s4_nn_exact(zx, zxo, M, N, K):
    r = zxo.Rng(zxo.REF_STATE_S4)
    Ap = r.s4_packed((M, K // 2))   # along K
    Bp = r.s4_packed((K, N // 2))   # K x N along N
    want = zxo.gemm_s8(zxo.unpack_s4(Ap, (M, K)), zxo.unpack_s4(Bp, (K, N)), M, N, K, zxo.NN)
    dC = torch.full((M, N), -1, dtype=torch.int32, device="cuda")
    zx.gemm_s4s4_nn(_dev(Ap), _dev(Bp), _ws(zx, zx.NN_S4S4, M, N, K), dC)
    torch.cuda.synchronize()
    assert zx.device_status() == 0
    got = dC.cpu().numpy()
    assert not _diff(got, want), _diff(got, want)


def test_s4s4_nn_nibble_extremes(zx, zxo):
    """Every (a, b) nibble pair -8..7 x -8..7 appears; results exact."""
    M, N, K = 256, 256, 256
    vals = np.arange(256, dtype=np.int64)
    a = ((vals[:, None] + np.arange(K)[None, :]) % 16 - 8).astype(np.int8)        # M x K in -8..7
    b = ((vals[:, None] * 7 + np.arange(N)[None, :] * 3) % 16 - 8).astype(np.int8)  # K x N
    pack = lambda x: ((x[:, 0::2] & 0xF) | ((x[:, 1::2] & 0xF) << 4)).astype(np.uint8)  # noqa: E731
    want = (a.astype(np.int64) @ b.astype(np.int64)).astype(np.int32)
    dC = torch.full((M, N), -1, dtype=torch.int32, device="cuda")
    zx.gemm_s4s4_nn(_dev(pack(a)), _dev(pack(b)), _ws(zx, zx.NN_S4S4, M, N, K), dC)
    torch.cuda.synchronize()
    assert not _diff(dC.cpu().numpy(), want)


@pytest.mark.slow
def test_sp_s8_nn_reference_size(zx, zxo):
    """n = 8192 on the reference's own data stream: 256 reference samples + Freivalds."""
    n = 8192
    r = zxo.Rng(zxo.REF_STATE_SP_S8)
    dense, comp, meta = r.prune24_s8(n, n)
    B = r.s8((n, n))
    dC = torch.full((n, n), -1, dtype=torch.int32, device="cuda")
    zx.gemm_sp_s8_nn(_dev(comp), _dev(meta.view(np.int32)), _dev(B), _ws(zx, zx.NN_SP_S8, n, n, n), dC)
    torch.cuda.synchronize()
    got = dC.cpu().numpy()
    bad, first = zxo.check_samples_s8(dense, B, got, n, n, n, zxo.NN)
    assert bad == 0, f"{bad}/256 wrong, first {first}"
    assert zxo.freivalds_s8(dense, B, got, n, n, n, zxo.NN)


def _sp_s4_case(zxo, M, N, K, state):
    """runImmaSpS4 (src/bench.zig:1178-1226): 4:8 pair-clustered packed A + metadata, then B
    K x N s4 packed along N."""
    r = zxo.Rng(state)
    dense, comp, meta = r.prune48_s4(M, K)
    Bp = r.s4_packed((K, N // 2))
    return comp, meta, Bp, zxo.gemm_s8(dense, zxo.unpack_s4(Bp, (K, N)), M, N, K, zxo.NN)


@pytest.mark.parametrize("policy_id", [0, 2, 6], ids=["auto", "sp224", "sp512x224"])
@pytest.mark.parametrize("M,N,K", [(128, 128, 256), (256, 224, 512), (512, 1040, 768), (384, 304, 256),
                                   (2560, 4096, 512)])
def test_sp_s4_nn_exact(zx, zxo, M, N, K, policy_id):
    """imma_sp_s4's operands through the layout pass (s4 -> int8, k reordered in every 8-wide
    chunk, metadata nibbles doubled) on each 2:4 sparse kernel; every element exact."""
    comp, meta, Bp, want = _sp_s4_case(zxo, M, N, K, zxo.REF_STATE_SP_S4 ^ (M + N + K))
    dC = torch.full((M, N), -1, dtype=torch.int32, device="cuda")
    zx.set_kernel_policy(policy_id)
    try:
        zx.gemm_sp_s4_nn(_dev(comp), _dev(meta.view(np.int32)), _dev(Bp), _ws(zx, zx.NN_SP_S4, M, N, K), dC)
        torch.cuda.synchronize()
    finally:
        zx.set_kernel_policy(0)
    assert zx.device_status() == 0
    got = dC.cpu().numpy()
    assert not _diff(got, want), _diff(got, want)


def test_sp_s4_nn_every_pair_extremes(zx, zxo):
    """Every kept pair pattern with -8 / 7 nibbles against B of -8 and 7: the largest products
    through the reorder, each of the 6 sub-chunk pairs in every chunk position."""
    M, N, K = 256, 256, 512
    _, comp, meta = zxo.Rng(0x7777).prune48_s4(M, K, want_dense=False)
    combos = [(0, 1), (0, 2), (0, 3), (1, 2), (1, 3), (2, 3)]
    rows = np.arange(M)[:, None]
    words = np.zeros((M, K // 64), dtype=np.uint32)
    for j in range(8):
        c = np.array([combos[(r + j + w) % 6] for r in range(M) for w in range(K // 64)]).reshape(M, K // 64, 2)
        words |= ((c[..., 0] | (c[..., 1] << 2)).astype(np.uint32) << np.uint32(4 * j))
    meta = words
    comp[:, 0::2] = np.where(rows % 2 == 0, 0x87, 0x78).astype(np.uint8)
    comp[:, 1::2] = 0x8F
    dense = zxo.decompress48_s4(comp, meta, M, K)
    b = np.where((np.arange(K)[:, None] + np.arange(N)[None, :]) % 3 == 0, -8, 7).astype(np.int8)
    Bp = ((b[:, 0::2] & 0xF) | ((b[:, 1::2] & 0xF) << 4)).astype(np.uint8)
    want = (dense.astype(np.int64) @ b.astype(np.int64)).astype(np.int32)
    dC = torch.full((M, N), -1, dtype=torch.int32, device="cuda")
    zx.gemm_sp_s4_nn(_dev(comp), _dev(meta.view(np.int32)), _dev(Bp), _ws(zx, zx.NN_SP_S4, M, N, K), dC)
    torch.cuda.synchronize()
    assert not _diff(dC.cpu().numpy(), want), _diff(dC.cpu().numpy(), want)


@pytest.mark.slow
def test_sp_s4_nn_reference_size(zx, zxo):
    """n = 8192 on the reference's own imma_sp_s4 data stream: 256 reference samples + Freivalds,
    and the result equals the reference-contract kernel's."""
    n = 8192
    r = zxo.Rng(zxo.REF_STATE_SP_S4)
    dense, comp, meta = r.prune48_s4(n, n)
    Bp = r.s4_packed((n, n // 2))
    B = zxo.unpack_s4(Bp, (n, n))
    dA, dM, dB = _dev(comp), _dev(meta.view(np.int32)), _dev(Bp)
    dC = torch.full((n, n), -1, dtype=torch.int32, device="cuda")
    zx.gemm_sp_s4_nn(dA, dM, dB, _ws(zx, zx.NN_SP_S4, n, n, n), dC)
    torch.cuda.synchronize()
    got = dC.cpu().numpy()
    bad, first = zxo.check_samples_s8(dense, B, got, n, n, n, zxo.NN)
    assert bad == 0, f"{bad}/256 wrong, first {first}"
    assert zxo.freivalds_s8(dense, B, got, n, n, n, zxo.NN)
    dR = torch.full((n, n), -1, dtype=torch.int32, device="cuda")
    zx.check(zx.lib().zx_launch_imma_sp_s4_ref(dA.data_ptr(), dB.data_ptr(), dM.data_ptr(), dR.data_ptr(), n, None))
    torch.cuda.synchronize()
    assert torch.equal(dC, dR)
