"""Reference-contract kernels: the reference's own entry names, arguments and launch shapes.

1. Through the C ABI (zx_launch_*_ref), which launches exactly as the reference bench does.
2. Through the CUDA driver API the way the reference's host layer does (src/cuda_driver.zig:
   cuModuleLoadData, cuModuleGetFunction by the mangled name `<stem>_$_<decl>`, cuLaunchKernel
   with a kernelParams array; src/bench.zig:671-682 grid/block), loading the shipped cubin.
   Also the properties the reference bench reports and its CI pins: no local-memory spill,
   static shared memory only (<= 48 KB), 128-thread launch bound.
Data and checks are the reference's: xorshift streams from its states, exact integer equality,
small-integer bf16 data for the bf16 kernel.
"""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

BUILD = Path(__file__).resolve().parents[1] / "zoxide_b200" / "_build"


@pytest.mark.parametrize("n", [128, 256, 1024])
def test_imma_s8_reference_launch(zx, zxo, n):
    r = zxo.Rng(zxo.REF_STATE_S8)
    A, B = r.s8((n, n)), r.s8((n, n))
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()  # keep both alive
    dC = torch.full((n, n), -1, dtype=torch.int32, device="cuda")
    zx.check(zx.lib().zx_launch_imma_s8_ref(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), n, None))
    torch.cuda.synchronize()
    got = dC.cpu().numpy()
    assert zxo.check_samples_s8(A, B, got, n, n, n, zxo.NN)[0] == 0
    assert np.array_equal(got, zxo.gemm_s8(A, B, n, n, n, zxo.NN))


def _bf16_small_ints(zxo, n):
    r = zxo.Rng(zxo.REF_STATE_BF16)
    vals = np.array([r.next() % 5 for _ in range(2 * n * n)], dtype=np.int64) - 2
    return vals[: n * n].astype(np.float32).reshape(n, n), vals[n * n:].astype(np.float32).reshape(n, n)


@pytest.mark.parametrize("n", [128, 512])
def test_hgemm_bf16_reference_launch(zx, zxo, n):
    a, b = _bf16_small_ints(zxo, n)
    tb = lambda x: torch.from_numpy(x).cuda().to(torch.bfloat16).contiguous()
    dA, dB = tb(a), tb(b)
    dC = torch.full((n, n), float("nan"), dtype=torch.float32, device="cuda")
    zx.check(zx.lib().zx_launch_hgemm_bf16_ref(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), n, None))
    torch.cuda.synchronize()
    assert np.array_equal(dC.cpu().numpy().astype(np.float64), a.astype(np.float64) @ b.astype(np.float64))


class _Driver:
    """Minimal libcuda binding for the reference's module/launch flow."""

    def __init__(self):
        self.cu = C.CDLL("libcuda.so.1")
        for name in ("cuInit", "cuCtxGetCurrent", "cuModuleLoadData", "cuModuleGetFunction",
                     "cuLaunchKernel", "cuCtxSynchronize", "cuFuncGetAttribute", "cuModuleUnload"):
            getattr(self.cu, name).restype = C.c_int
        self.ok(self.cu.cuInit(0))

    @staticmethod
    def ok(rc):
        assert rc == 0, f"CUresult {rc}"

    def module(self, image: bytes):
        mod = C.c_void_p()
        self._image = C.create_string_buffer(image, len(image))
        self.ok(self.cu.cuModuleLoadData(C.byref(mod), self._image))
        return mod

    def function(self, mod, name: str):
        f = C.c_void_p()
        self.ok(self.cu.cuModuleGetFunction(C.byref(f), mod, name.encode()))
        return f

    def attr(self, f, which: int) -> int:
        v = C.c_int()
        self.ok(self.cu.cuFuncGetAttribute(C.byref(v), which, f))
        return v.value

    def launch(self, f, grid, block, args):
        holders = [C.c_uint64(a) if i < 3 else C.c_uint32(a) for i, a in enumerate(args)]
        params = (C.c_void_p * len(holders))(*[C.cast(C.byref(h), C.c_void_p) for h in holders])
        self.ok(self.cu.cuLaunchKernel(f, grid[0], grid[1], 1, block, 1, 1, 0, None, params, None))
        self.ok(self.cu.cuCtxSynchronize())


# CUfunction_attribute values (cuda.h): MAX_THREADS_PER_BLOCK 0, SHARED_SIZE_BYTES 1,
# LOCAL_SIZE_BYTES 3, NUM_REGS 4.
def test_imma_s8_cubin_in_reference_flow(zx, zxo):
    torch.cuda.init()
    torch.empty(1, device="cuda")  # primary context current on this thread
    d = _Driver()
    mod = d.module((BUILD / "imma_s8.cubin").read_bytes())
    f = d.function(mod, "imma_s8_$_immaS8")
    assert d.attr(f, 0) >= 128
    assert d.attr(f, 1) <= 48 * 1024  # static shared memory only, within the default limit
    assert d.attr(f, 3) == 0, "local-memory spill"
    n = 512
    r = zxo.Rng(zxo.REF_STATE_S8)
    A, B = r.s8((n, n)), r.s8((n, n))
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dC = torch.full((n, n), -1, dtype=torch.int32, device="cuda")  # 0xff poison, src/bench.zig:665-668
    d.launch(f, (n // 128, n // 128), 128, [dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), n])
    got = dC.cpu().numpy()
    bad, first = zxo.check_samples_s8(A, B, got, n, n, n, zxo.NN)
    assert bad == 0, first
    assert np.array_equal(got, zxo.gemm_s8(A, B, n, n, n, zxo.NN))
    d.cu.cuModuleUnload(mod)


def test_hgemm_bf16_cubin_in_reference_flow(zx, zxo):
    torch.empty(1, device="cuda")
    d = _Driver()
    mod = d.module((BUILD / "hgemm_wgmma_bf16.cubin").read_bytes())
    f = d.function(mod, "hgemm_wgmma_bf16_$_hgemmWgmmaBf16")
    assert d.attr(f, 3) == 0 and d.attr(f, 1) <= 48 * 1024
    n = 256
    a, b = _bf16_small_ints(zxo, n)
    tb = lambda x: torch.from_numpy(x).cuda().to(torch.bfloat16).contiguous()
    dA, dB = tb(a), tb(b)
    dC = torch.full((n, n), float("nan"), dtype=torch.float32, device="cuda")
    d.launch(f, (n // 128, n // 64), 128, [dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), n])
    assert np.array_equal(dC.cpu().numpy().astype(np.float64), a.astype(np.float64) @ b.astype(np.float64))
    d.cu.cuModuleUnload(mod)
