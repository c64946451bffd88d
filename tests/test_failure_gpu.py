"""Failure detection without a GPU fault: a bounded wait that runs out, read back on the host.

Every mbarrier wait in the kernels is bounded (a wall-clock limit via %globaltimer); a wait that
gives up records `0x100 | site` in the device status word and raises the CTA's abort flag, and
the kernel returns. zx_selftest_bounded_wait runs that same wait code in a one-CTA kernel with a
short limit on a barrier nothing arrives on (cf. the reference's bounded tryWaitFor,
src/tma.zig:142-153, and hgemm_tma's give-up path, src/examples/hgemm_tma.zig:141-156). The test
checks the status code, that the second warp left through the abort flag rather than its own
(longer) limit, and that the context stays usable: a GEMM afterwards is exact.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_survives(zx, zxo):
    lib = zx.lib()
    zx.device_status_clear()
    limit_us = 20000
    out = torch.full((3,), -1, dtype=torch.int32, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        e0.record()
        assert lib.zx_selftest_bounded_wait(out.data_ptr(), limit_us, None) == 0, zx.abi.last_error()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        # thread 0 gave up after ~20 ms; warp 1 (limit 80 ms) left as soon as the abort flag rose
        assert 0.8 * limit_us / 1000 <= ms < 3 * limit_us / 1000, ms
        assert out.tolist() == [0, 0, 1]  # timed out, aborted, completed barrier succeeded
        code = ctypes.c_uint32(0)
        assert lib.zx_device_status(ctypes.byref(code)) == zx.abi.ZX_ERR_TIMEOUT
        assert code.value == 0x1F1
        assert "status code 0x1f1" in zx.abi.last_error()
    finally:
        zx.device_status_clear()  # later tests expect a clean status word
    assert zx.device_status() == 0
    # the context is intact: a GEMM right after is exact and leaves the status clean
    r = zxo.Rng.from_seed(3)
    A, B = r.s8((256, 512)), r.s8((384, 512))
    got = zx.gemm_s8(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), zxo.gemm_s8(A, B, 256, 384, 512, zxo.NT))
    assert zx.device_status() == 0

