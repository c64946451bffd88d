"""GEMM on host buffers with the copies overlapped (zx_gemm_s8_host / zx_gemm_bf16_host).

The reference's bench flow copies A and B to the device, launches and copies C back
(src/bench.zig:647-741); the library does the same in 2-D blocks on two copy streams. The
int8 result must equal the oracle's (src/host.zig:302-317 restated) exactly, on shapes that
give one block, ragged blocks and the full 4 x 4 grid; bf16 must match torch's fp32 product."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _pinned(x):
    return x.contiguous().pin_memory()


@pytest.mark.parametrize("M,N,K", [(300, 520, 256), (3000, 3000, 512), (2048, 4096, 256), (1100, 8200, 128)])
def test_s8_host_equals_oracle(zx, zxo, M, N, K, policy):
    """Every tile path (policy fixture) writes its parts of C with row pitch N into C_dev."""
    r = zxo.Rng.from_seed(M + 3 * N)
    A, B = r.s8((M, K)), r.s8((N, K))
    A_h, B_h = _pinned(torch.from_numpy(A)), _pinned(torch.from_numpy(B))
    C_h = torch.full((M, N), -1, dtype=torch.int32).pin_memory()
    A_d, B_d = torch.empty((M, K), dtype=torch.int8, device="cuda"), torch.empty((N, K), dtype=torch.int8, device="cuda")
    C_d = torch.empty((M, N), dtype=torch.int32, device="cuda")
    zx.gemm_host(A_h, B_h, C_h, A_d, B_d, C_d)
    torch.cuda.synchronize()
    assert "zx_gemm_s8_host" in zx.last_kernel()
    want = zxo.gemm_s8(A, B, M, N, K, zxo.NT)
    assert np.array_equal(C_h.numpy(), want)
    assert np.array_equal(C_d.cpu().numpy(), want)  # the device copy is row-major C too
    assert zx.device_status() == 0


def test_s8_host_full_grid_and_repeat(zx):
    """8192 x 8192 (4 x 4 blocks of 2048), called twice on the same buffers with new inputs: the second
    call's copies wait for the first call's work; checked against the device-resident GEMM."""
    M = N = 8192
    K = 512
    g = torch.Generator().manual_seed(5)
    C_d = torch.empty((M, N), dtype=torch.int32, device="cuda")
    A_d, B_d = torch.empty((M, K), dtype=torch.int8, device="cuda"), torch.empty((N, K), dtype=torch.int8, device="cuda")
    C_h = torch.empty((M, N), dtype=torch.int32).pin_memory()
    outs = []
    for it in range(2):
        A_h = _pinned(torch.randint(-128, 128, (M, K), dtype=torch.int8, generator=g))
        B_h = _pinned(torch.randint(-128, 128, (N, K), dtype=torch.int8, generator=g))
        zx.gemm_host(A_h, B_h, C_h, A_d, B_d, C_d)
        torch.cuda.synchronize()
        assert "4 x 4 blocks in 4 shells" in zx.last_kernel(), zx.last_kernel()
        want = zx.gemm_s8(A_h.cuda(), B_h.cuda()).cpu()
        assert torch.equal(C_h, want), it
        outs.append(C_h.clone())
    assert not torch.equal(outs[0], outs[1])


def test_bf16_host_matches_fp32(zx):
    M, N, K = 2500, 3000, 512
    g = torch.Generator().manual_seed(9)
    A = (torch.randn((M, K), generator=g) / K ** 0.5).to(torch.bfloat16)
    B = (torch.randn((N, K), generator=g) / K ** 0.5).to(torch.bfloat16)
    C_h = torch.empty((M, N), dtype=torch.float32).pin_memory()
    zx.gemm_host(_pinned(A), _pinned(B), C_h, torch.empty_like(A, device="cuda"), torch.empty_like(B, device="cuda"),
                 torch.empty((M, N), dtype=torch.float32, device="cuda"))
    torch.cuda.synchronize()
    ref = A.float() @ B.float().T
    err = (C_h - ref).norm() / ref.norm()
    assert err < 1e-5, float(err)


def test_host_arguments(zx):
    lib = zx.lib()
    x = torch.zeros(16, dtype=torch.int8, device="cuda")
    h = torch.zeros(16, dtype=torch.int8)
    assert lib.zx_gemm_s8_host(None, h.data_ptr(), h.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                               16, 16, 16, None) == zx.abi.ZX_ERR_NULL
    assert lib.zx_gemm_s8_host(h.data_ptr(), h.data_ptr(), h.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                               16, 18, 16, None) == zx.abi.ZX_ERR_SHAPE
