"""The reference's own operand layouts on the fast kernels (zx_gemm_sp_s8_nn, zx_gemm_s4s4_nn):
a layout pass into a caller workspace, then the K-major tcgen05 kernels. Data are the reference
bench's own streams (runImmaSpS8, src/bench.zig:1027-1063; runImmaS4, src/bench.zig:767-786) and
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
