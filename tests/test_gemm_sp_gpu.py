"""2:4 structured-sparse int8 GEMM on tcgen05.mma.sp, exact int32.

A is pruned 2:4 along K exactly as the reference's runImmaSpS8 does (src/bench.zig:1027-1058:
combos[xorshift % 6], two value draws per group, nibble metadata idx0 | idx1 << 2, one u32 per
row per 32 dense k) and passed compressed with its metadata unchanged. The oracle multiplies the
pruned dense A (the reference's own check, src/bench.zig:1121-1149).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[0, 2, 5, 6], ids=["auto", "sp224", "sp480", "sp512x224"])
def sp_policy(request, zx):
    """Automatic choice, the 256 x 224 two-accumulator kernel, the 256 x 480 lo/hi kernel and the
    512 x 224 kernel (two 256-row blocks of A sharing B)."""
    zx.set_kernel_policy(request.param)
    yield request.param
    zx.set_kernel_policy(0)


def _case(zxo, M, N, K, state):
    d, comp, meta, st = zxo.prune24_s8(M, K, state)
    B = zxo.Rng(st).s8((N, K))
    return d, comp, meta, B


def _run(zx, comp, meta, B, M, N):
    dC = torch.full((M, N), -1, dtype=torch.int32, device="cuda")
    zx.gemm_sp_s8(torch.from_numpy(comp).cuda(), torch.from_numpy(meta.view(np.int32)).cuda(),
                  torch.from_numpy(B).cuda(), dC)
    torch.cuda.synchronize()
    assert zx.device_status() == 0
    return dC.cpu().numpy()


@pytest.mark.parametrize("M,N,K", [(256, 224, 256), (256, 224, 2048), (512, 448, 1024),
                                   (1024, 1024, 1024), (384, 300, 512), (128, 64, 256),
                                   (512, 1000, 512), (2560, 4096, 512), (2560, 4096, 256),
                                   (4096, 4480, 1024)])  # 2+ tiles per pair on every kernel
def test_sparse_exact(zx, zxo, sp_policy, M, N, K):
    d, comp, meta, B = _case(zxo, M, N, K, 0xC0FFEE11 ^ (M + N + K))
    got = _run(zx, comp, meta, B, M, N)
    want = zxo.gemm_s8(d, B, M, N, K, zxo.NT)
    if not np.array_equal(got, want):
        bad = np.argwhere(got != want)
        r, c = bad[0]
        pytest.fail(f"{len(bad)}/{got.size} mismatches; first ({r},{c}) want {want[r, c]} got {got[r, c]}")


def test_sparse_every_combo(zx, zxo, sp_policy):
    """Each of the 6 kept-pair patterns in isolation, with +-128 / 127 extremes."""
    M, N, K = 256, 224, 256
    combos = [(0, 1), (0, 2), (0, 3), (1, 2), (1, 3), (2, 3)]
    for ci, (i0, i1) in enumerate(combos):
        meta_word = 0
        for j in range(8):
            meta_word |= (i0 | (i1 << 2)) << (4 * j)
        meta = np.full((M, K // 32), meta_word, dtype=np.uint32)
        comp = np.empty((M, K // 2), dtype=np.int8)
        comp[:, 0::2] = -128
        comp[:, 1::2] = 127
        dense = zxo.decompress24_s8(comp, meta, M, K)
        B = zxo.Rng.from_seed(ci).s8((N, K))
        got = _run(zx, comp, meta, B, M, N)
        assert np.array_equal(got, zxo.gemm_s8(dense, B, M, N, K, zxo.NT)), f"combo {(i0, i1)}"


@pytest.mark.slow
def test_sparse_config4_full_size(zx, zxo, sp_policy):
    M = N = K = 8192
    d, comp, meta, B = _case(zxo, M, N, K, zxo.REF_STATE_SP_S8)
    got = _run(zx, comp, meta, B, M, N)
    bad, first = zxo.check_samples_s8(d, B, got, M, N, K, zxo.NT)
    assert bad == 0, f"{bad}/256 reference samples wrong, first {first}"
    assert zxo.freivalds_s8(d, B, got, M, N, K, zxo.NT)


@pytest.mark.parametrize("M,N,K,kernel", [(4096, 8192, 256, "gemm_sp4_kernel"), (256, 2048, 256, "gemm_sp2_kernel")])
def test_sparse_auto_choice(zx, zxo, M, N, K, kernel):
    """The automatic policy picks the 512 x 224 kernel when it needs fewer waves x blocks (4 waves
    against 8 here) and the 256 x 224 kernel for 256 rows (a 512-row tile would compute an empty
    block); either way every element is exact."""
    zx.set_kernel_policy(0)
    d, comp, meta, B = _case(zxo, M, N, K, 0xA5A5 ^ (M + N))
    got = _run(zx, comp, meta, B, M, N)
    assert zx.last_kernel().startswith(kernel), zx.last_kernel()
    assert np.array_equal(got, zxo.gemm_s8(d, B, M, N, K, zxo.NT))
