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

    def launch(self, f, grid, block, args, types=None):
        """kernelParams as the reference passes them (src/cuda_driver.zig:804-845): an array of
        pointers to each argument's value; pointers are u64, `n` u32 unless `types` says."""
        if types is None:
            types = [C.c_uint64] * 3 + [C.c_uint32] * (len(args) - 3)
        holders = [t(a) for t, a in zip(types, args)]
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


# ---------------------------------------------------------------------------------------------
# The other reference kernels: imma_s4, imma_sp_s8, imma_sp_s4, hgemm_bf16 (128 x 128 tile),
# hgemm_tma. Each case builds the reference bench's data stream from its own xorshift state and
# compares every element against the oracle (exact for the integer kernels; the bf16 / f16 data
# are the reference's small integers, so the f32 results are exact too).

def _s4_data(zxo, n):
    """runImmaS4 (src/bench.zig:767-786): packed A (along K) then packed B (K x N, along N)."""
    r = zxo.Rng(zxo.REF_STATE_S4)
    Ap, Bp = r.s4_packed((n, n // 2)), r.s4_packed((n, n // 2))
    want = zxo.gemm_s8(zxo.unpack_s4(Ap, (n, n)), zxo.unpack_s4(Bp, (n, n)), n, n, n, zxo.NN)
    return Ap, Bp, want


def _sp_s8_data(zxo, n):
    """runImmaSpS8 (src/bench.zig:1027-1063): pruned A + metadata, then dense B, one stream."""
    r = zxo.Rng(zxo.REF_STATE_SP_S8)
    dense, comp, meta = r.prune24_s8(n, n)
    B = r.s8((n, n))
    return comp, meta, B, zxo.gemm_s8(dense, B, n, n, n, zxo.NN)


def _sp_s4_data(zxo, n):
    """runImmaSpS4 (src/bench.zig:1178-1226): 4:8 pair-clustered packed A + metadata, then
    dense B packed along N, one stream."""
    r = zxo.Rng(zxo.REF_STATE_SP_S4)
    dense, comp, meta = r.prune48_s4(n, n)
    Bp = r.s4_packed((n, n // 2))
    return comp, meta, Bp, zxo.gemm_s8(dense, zxo.unpack_s4(Bp, (n, n)), n, n, n, zxo.NN)


def _f16_small_ints(zxo, n):
    """runHgemmTma (src/bench.zig:1450-1461): values (xorshift % 5) - 2, A then B."""
    r = zxo.Rng(0x2468ACE0)
    vals = np.array([r.next() % 5 for _ in range(2 * n * n)], dtype=np.int64) - 2
    return vals[: n * n].astype(np.float32).reshape(n, n), vals[n * n:].astype(np.float32).reshape(n, n)


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _diff(got, want):
    if np.array_equal(got, want):
        return ""
    bad = np.argwhere(got != want)
    r, c = bad[0]
    return f"{len(bad)} mismatches; first at ({r},{c}) want {want[r, c]} got {got[r, c]}"


@pytest.mark.parametrize("n", [128, 256, 640])
def test_imma_s4_reference_launch(zx, zxo, n):
    Ap, Bp, want = _s4_data(zxo, n)
    dA, dB = _dev(Ap), _dev(Bp)
    dC = torch.full((n, n), -1, dtype=torch.int32, device="cuda")
    zx.check(zx.lib().zx_launch_imma_s4_ref(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), n, None))
    torch.cuda.synchronize()
    assert zx.device_status() == 0
    assert not _diff(dC.cpu().numpy(), want), _diff(dC.cpu().numpy(), want)


@pytest.mark.parametrize("n", [128, 256, 640])
def test_imma_sp_s8_reference_launch(zx, zxo, n):
    comp, meta, B, want = _sp_s8_data(zxo, n)
    dA, dM, dB = _dev(comp), _dev(meta.view(np.int32)), _dev(B)
    dC = torch.full((n, n), -1, dtype=torch.int32, device="cuda")
    zx.check(zx.lib().zx_launch_imma_sp_s8_ref(dA.data_ptr(), dB.data_ptr(), dM.data_ptr(), dC.data_ptr(), n, None))
    torch.cuda.synchronize()
    assert zx.device_status() == 0
    assert not _diff(dC.cpu().numpy(), want), _diff(dC.cpu().numpy(), want)


@pytest.mark.parametrize("n", [128, 256, 640])
def test_imma_sp_s4_reference_launch(zx, zxo, n):
    comp, meta, Bp, want = _sp_s4_data(zxo, n)
    dA, dM, dB = _dev(comp), _dev(meta.view(np.int32)), _dev(Bp)
    dC = torch.full((n, n), -1, dtype=torch.int32, device="cuda")
    zx.check(zx.lib().zx_launch_imma_sp_s4_ref(dA.data_ptr(), dB.data_ptr(), dM.data_ptr(), dC.data_ptr(), n, None))
    torch.cuda.synchronize()
    assert zx.device_status() == 0
    assert not _diff(dC.cpu().numpy(), want), _diff(dC.cpu().numpy(), want)


def test_imma_sp_s4_extremes(zx, zxo):
    """Every kept pair -8 / 7 against B of -8: max-magnitude products through the k reorder."""
    n = 128
    _, comp, meta = zxo.Rng(0x1234567).prune48_s4(n, n, want_dense=False)
    comp[:, 0::2] = 0x88  # (-8, -8)
    comp[:, 1::2] = 0x77  # (7, 7)
    dense = zxo.decompress48_s4(comp, meta, n, n)
    Bp = np.full((n, n // 2), 0x88, dtype=np.uint8)
    want = zxo.gemm_s8(dense, zxo.unpack_s4(Bp, (n, n)), n, n, n, zxo.NN)
    dA, dM, dB = _dev(comp), _dev(meta.view(np.int32)), _dev(Bp)
    dC = torch.full((n, n), -1, dtype=torch.int32, device="cuda")
    zx.check(zx.lib().zx_launch_imma_sp_s4_ref(dA.data_ptr(), dB.data_ptr(), dM.data_ptr(), dC.data_ptr(), n, None))
    torch.cuda.synchronize()
    assert np.array_equal(dC.cpu().numpy(), want)


@pytest.mark.parametrize("n", [128, 384])
def test_hgemm_bf16_mma_reference_launch(zx, zxo, n):
    a, b = _bf16_small_ints(zxo, n)
    tb = lambda x: torch.from_numpy(x).cuda().to(torch.bfloat16).contiguous()
    dA, dB = tb(a), tb(b)
    dC = torch.full((n, n), float("nan"), dtype=torch.float32, device="cuda")
    zx.check(zx.lib().zx_launch_hgemm_bf16_mma_ref(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), n, None))
    torch.cuda.synchronize()
    assert np.array_equal(dC.cpu().numpy().astype(np.float64), a.astype(np.float64) @ b.astype(np.float64))


@pytest.mark.parametrize("n", [128, 384])
def test_hgemm_tma_reference_launch(zx, zxo, n):
    a, b = _f16_small_ints(zxo, n)
    th = lambda x: torch.from_numpy(x).cuda().to(torch.float16).contiguous()
    dA, dB = th(a), th(b)
    dC = torch.full((n, n), float("nan"), dtype=torch.float32, device="cuda")
    zx.check(zx.lib().zx_launch_hgemm_tma_ref(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), n, 0, 0, None))
    torch.cuda.synchronize()
    assert np.array_equal(dC.cpu().numpy().astype(np.float64), a.astype(np.float64) @ b.astype(np.float64))


@pytest.mark.parametrize("n", [128, 384, 1024])
def test_hgemm_tma_fast_signature(zx, zxo, n):
    """zx_hgemm_tma keeps hgemm_tma's argument list (f16 A, B row-major, fp32 C, two descriptor
    words) and runs the fast f16 kernels: exact on runHgemmTma's small-integer data and equal to the
    reference-contract kernel's result."""
    a, b = _f16_small_ints(zxo, n)
    th = lambda x: torch.from_numpy(x).cuda().to(torch.float16).contiguous()  # noqa: E731
    dA, dB = th(a), th(b)
    dC = torch.full((n, n), float("nan"), dtype=torch.float32, device="cuda")
    zx.hgemm_tma(dA, dB, dC, n, 0x1000, 0x2000)
    dR = torch.full((n, n), float("nan"), dtype=torch.float32, device="cuda")
    zx.check(zx.lib().zx_launch_hgemm_tma_ref(dA.data_ptr(), dB.data_ptr(), dR.data_ptr(), n, 0, 0, None))
    torch.cuda.synchronize()
    assert zx.device_status() == 0
    assert np.array_equal(dC.cpu().numpy().astype(np.float64), a.astype(np.float64) @ b.astype(np.float64))
    assert torch.equal(dC, dR)


def test_reference_gate_messages(zx):
    """n % 128 != 0 is refused before any launch, with the reference bench's wording."""
    lib = zx.lib()
    P = (0x10000, 0x20000, 0x30000)
    assert lib.zx_launch_imma_s4_ref(*P, 200, None) == zx.abi.ZX_ERR_SHAPE
    assert "imma_s4 requires n % 128 == 0 (got 200)" in zx.abi.last_error()
    assert lib.zx_launch_imma_sp_s4_ref(*P, 0x40000, 96, None) == zx.abi.ZX_ERR_SHAPE
    assert "imma_sp_s4 requires n % 128 == 0" in zx.abi.last_error()


@pytest.mark.parametrize("stem,entry,kind", [
    ("imma_s4", "imma_s4_$_immaS4", "s4"),
    ("imma_sp_s8", "imma_sp_s8_$_immaSpS8", "sp_s8"),
    ("imma_sp_s4", "imma_sp_s4_$_immaSpS4", "sp_s4"),
    ("hgemm_bf16", "hgemm_bf16_$_hgemmBf16", "bf16"),
    ("hgemm_tma", "hgemm_tma_$_hgemmTma", "tma"),
])
def test_cubins_in_reference_flow(zx, zxo, stem, entry, kind):
    """Each <stem>.cubin through cuModuleLoadData / cuModuleGetFunction(<entry>) /
    cuLaunchKernel with the reference's grid, block and kernelParams."""
    torch.empty(1, device="cuda")
    d = _Driver()
    mod = d.module((BUILD / f"{stem}.cubin").read_bytes())
    f = d.function(mod, entry)
    assert d.attr(f, 0) >= 128
    assert d.attr(f, 1) <= 48 * 1024
    assert d.attr(f, 3) == 0, "local-memory spill"
    n = 256
    U64, U32 = C.c_uint64, C.c_uint32
    if kind == "s4":
        Ap, Bp, want = _s4_data(zxo, n)
        keep = [_dev(Ap), _dev(Bp), torch.full((n, n), -1, dtype=torch.int32, device="cuda")]
        args, types, grid = [t.data_ptr() for t in keep] + [n], [U64] * 3 + [U32], (n // 128, n // 128)
    elif kind in ("sp_s8", "sp_s4"):
        comp, meta, B, want = (_sp_s8_data if kind == "sp_s8" else _sp_s4_data)(zxo, n)
        keep = [_dev(comp), _dev(B), _dev(meta.view(np.int32)), torch.full((n, n), -1, dtype=torch.int32, device="cuda")]
        args, types, grid = [t.data_ptr() for t in keep] + [n], [U64] * 4 + [U32], (n // 128, n // 128)
    else:
        a, b = (_bf16_small_ints if kind == "bf16" else _f16_small_ints)(zxo, n)
        dt = torch.bfloat16 if kind == "bf16" else torch.float16
        keep = [torch.from_numpy(a).cuda().to(dt), torch.from_numpy(b).cuda().to(dt),
                torch.full((n, n), float("nan"), dtype=torch.float32, device="cuda")]
        want = a.astype(np.float64) @ b.astype(np.float64)
        args, types = [t.data_ptr() for t in keep] + [n], [U64] * 3 + [U32]
        grid = (n // 128, n // 128) if kind == "bf16" else (n // 128, n // 64)
        if kind == "tma":
            args, types = args + [0, 0], types + [U64, U64]
    d.launch(f, grid, 128, args, types)
    got = keep[-1].cpu().numpy()
    if kind in ("bf16", "tma"):
        got = got.astype(np.float64)
    assert not _diff(got, want), _diff(got, want)
    d.cu.cuModuleUnload(mod)
