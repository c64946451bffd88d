"""zx_gemm_w4a8_noalloc: the W4A8 decode GEMM for callers that cannot allocate device memory.

Some hosts own all device memory through their own allocator or budget (a framework's caching
allocator, an embedding runtime that binds this library over its C ABI), and some decode loops
cannot afford an allocation that might synchronize the device. zx_gemm_w4a8_ws needs a
workspace for its split-K partial sums; zx_gemm_w4a8_noalloc keeps that scratch in an array
built into the library instead, so the caller passes only A, W and C.

The GPU test calls the entry point through the C ABI and checks that its output equals the
existing zx_gemm_w4a8's exactly (integer results, no tolerance), on two calls in a row, because
the built-in array keeps the previous call's contents. The CPU test checks the size limits.
This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch


def _case(zxo, M, N, K, seed):
    r = zxo.Rng.from_seed(seed)
    return r.s8((M, K)), r.s4_packed((N, K // 2))


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(16, 28672, 8192), (7, 1024, 2048), (32, 640, 4096), (1, 128, 8192)])
def test_noalloc_matches_existing_entry_point(zx, zxo, M, N, K):
    """Two calls in a row through the C ABI, each equal to zx_gemm_w4a8's result; (1, 128, 8192)
    has one tile of C shared by 32 CTAs, (16, 28672, 8192) is the decode configuration."""
    A, W = _case(zxo, M, N, K, 5 * M + N + K)
    dA, dW = torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda()
    ref = torch.full((M, N), -1, dtype=torch.int32, device="cuda")
    zx.gemm_w4a8(dA, dW, ref)  # the existing entry point
    torch.cuda.synchronize()
    want = ref.cpu().numpy()
    lib = zx.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream or None)
    for call in range(2):
        dC = torch.full((M, N), 0x5A5A5A5A, dtype=torch.int32, device="cuda")
        rc = lib.zx_gemm_w4a8_noalloc(dA.data_ptr(), dW.data_ptr(), dC.data_ptr(), M, N, K, stream)
        assert rc == 0, zx.abi.last_error()
        torch.cuda.synchronize()
        assert zx.device_status() == 0
        assert zx.last_kernel().startswith("gemm_w4s_kernel")
        got = dC.cpu().numpy()
        if not np.array_equal(got, want):
            bad = np.argwhere(got != want)
            r, c = bad[0]
            pytest.fail(f"call {call}: {len(bad)} mismatches; first ({r},{c}) want {want[r, c]} got {got[r, c]}")


def test_noalloc_rejects_shapes_beyond_its_scratch(zx):
    """M, N and K beyond what the built-in scratch covers fail before any CUDA call."""
    lib = zx.lib()
    good = (0x10000, 0x20000, 0x30000)
    for (M, N, K), needle in [((33, 256, 512), "M=33"), ((16, 65540, 512), "N=65540"),
                              ((16, 256, 384), "multiple of 256")]:
        assert lib.zx_gemm_w4a8_noalloc(*good, M, N, K, None) == 1002
        assert needle in zx.abi.last_error()
    assert lib.zx_gemm_w4a8_noalloc(0, good[1], good[2], 16, 256, 512, None) == 1001
