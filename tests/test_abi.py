"""The C-ABI library without a GPU: it loads, exports every declared symbol, and rejects bad
arguments before touching CUDA (mirrors the reference's pre-launch validation,
src/host.zig:437-494). On a machine with no GPU a valid call fails loudly — there is no CPU
fallback anywhere in the product path."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "zoxide_gemm.h"


def declared_symbols():
    text = HEADER.read_text()
    return re.findall(r"^ZX_API\s+[\w\s\*]+?\b(zx_\w+)\s*\(", text, flags=re.M)


def test_header_declares_expected_entry_points():
    syms = declared_symbols()
    for s in ("zx_gemm_s8", "zx_gemm_s8_scaled_bf16", "zx_gemm_bf16", "zx_imma_s8",
              "zx_hgemm_bf16", "zx_last_error", "zx_device_status"):
        assert s in syms


def test_library_exports_every_declared_symbol(zx):
    lib = zx.lib()
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} declared in {HEADER.name} but not exported"
    assert set(declared_symbols()) <= set(zx.abi.SIGNATURES)


def test_version(zx):
    assert zx.lib().zx_version() >= 100


def _err(zx, rc):
    return rc, zx.abi.last_error()


GOOD = (0x10000, 0x20000, 0x30000)


@pytest.mark.parametrize(
    "args,code,needle",
    [
        ((0, GOOD[1], GOOD[2], 128, 128, 128, 0), 1001, "null"),
        ((*GOOD, 128, 128, 128, 7), 1004, "layout"),
        ((*GOOD, 0, 128, 128, 0), 1002, "empty"),
        ((*GOOD, 128, 128, 100, 0), 1002, "K=100"),
        ((*GOOD, 128, 130, 128, 0), 1002, "N=130"),
        ((*GOOD, 128, 20, 128, 1), 1002, "NN layout"),
        ((GOOD[0] + 8, GOOD[1], GOOD[2], 128, 128, 128, 0), 1003, "aligned"),
    ],
)
def test_gemm_s8_rejects_bad_arguments(zx, args, code, needle):
    rc, msg = _err(zx, zx.lib().zx_gemm_s8(*args, None))
    assert rc == code, msg
    assert needle in msg


def test_scaled_rejects_bad_arguments(zx):
    lib = zx.lib()
    rc, msg = _err(zx, lib.zx_gemm_s8_scaled_bf16(*GOOD[:2], 0, 0x40000, GOOD[2], 128, 128, 128, 0, None))
    assert rc == 1001 and "scale" in msg
    rc, msg = _err(zx, lib.zx_gemm_s8_scaled_bf16(*GOOD[:2], 0x40002, 0x40000, GOOD[2], 128, 128, 128, 0, None))
    assert rc == 1003
    rc, msg = _err(zx, lib.zx_gemm_s8_scaled_bf16(*GOOD[:2], 0x40000, 0x50000, GOOD[2], 128, 132, 128, 0, None))
    assert rc == 1002 and "N=132" in msg


def test_bf16_rejects_bad_arguments(zx):
    rc, msg = _err(zx, zx.lib().zx_gemm_bf16(*GOOD, 128, 128, 12, 0, None))
    assert rc == 1002 and "K=12" in msg


def test_reference_signature_shape_gate(zx):
    """The reference bench's gate: imma_s8 requires n % 128 == 0 (src/bench.zig:96-99)."""
    rc, msg = _err(zx, zx.lib().zx_imma_s8(*GOOD, 200, None))
    assert rc == 1002 and "n % 128 == 0" in msg
    rc, msg = _err(zx, zx.lib().zx_hgemm_bf16(*GOOD, 100, None))
    assert rc == 1002


def test_w4a8_workspace_arguments(zx):
    import ctypes

    lib = zx.lib()
    out = ctypes.c_uint64(7)
    assert lib.zx_gemm_w4a8_workspace_bytes(128, 256, 512, ctypes.byref(out)) == 0 and out.value == 0
    assert lib.zx_gemm_w4a8_workspace_bytes(16, 256, 512, None) == 1001
    assert lib.zx_gemm_w4a8_workspace_bytes(16, 256, 100, ctypes.byref(out)) == 1002
    rc, msg = _err(zx, lib.zx_gemm_w4a8_ws(*GOOD, 16, 256, 512, 0, 0, None))
    assert rc == 1001 and "workspace" in msg
    rc, msg = _err(zx, lib.zx_gemm_w4a8_ws(*GOOD, 16, 256, 512, 0x1008, 4096, None))
    assert rc == 1003 and "workspace" in msg


def test_replicated_arguments(zx):
    """zx_gemm_s8_replicated: int32 NT checks first, then the peer list (before any CUDA call)."""
    lib = zx.lib()
    arr = (ctypes.c_uint64 * 8)(*([0x40000] * 8))
    rc, msg = _err(zx, lib.zx_gemm_s8_replicated(*GOOD, 128, 130, 128, arr, 1, None))
    assert rc == 1002 and "N=130" in msg
    rc, msg = _err(zx, lib.zx_gemm_s8_replicated(*GOOD, 128, 128, 128, arr, 8, None))
    assert rc == 1002 and "at most 7" in msg
    rc, msg = _err(zx, lib.zx_gemm_s8_replicated(*GOOD, 128, 128, 128, None, 2, None))
    assert rc == 1001 and "peer buffer list" in msg
    bad = (ctypes.c_uint64 * 2)(0x40000, 0)
    rc, msg = _err(zx, lib.zx_gemm_s8_replicated(*GOOD, 128, 128, 128, bad, 2, None))
    assert rc == 1001 and "peer buffer 1" in msg
    bad = (ctypes.c_uint64 * 2)(0x40000, 0x50004)
    rc, msg = _err(zx, lib.zx_gemm_s8_replicated(*GOOD, 128, 128, 128, bad, 2, None))
    assert rc == 1003 and "peer buffer 1" in msg


def test_host_pipeline_arguments(zx):
    lib = zx.lib()
    h = ctypes.create_string_buffer(64)
    rc, msg = _err(zx, lib.zx_gemm_s8_host(None, h, h, *GOOD, 128, 128, 128, None))
    assert rc == 1001 and "host" in msg
    rc, msg = _err(zx, lib.zx_gemm_s8_host(h, h, h, *GOOD, 128, 130, 128, None))
    assert rc == 1002 and "N=130" in msg
    rc, msg = _err(zx, lib.zx_gemm_bf16_host(h, h, h, *GOOD, 128, 128, 12, None))
    assert rc == 1002 and "K=12" in msg


def test_ipc_arguments(zx):
    lib = zx.lib()
    h = ctypes.create_string_buffer(64)
    off = ctypes.c_uint64(0)
    assert lib.zx_ipc_export(0, h, ctypes.byref(off)) == 1001
    assert lib.zx_ipc_export(0x10000, None, ctypes.byref(off)) == 1001
    assert lib.zx_ipc_import(None, ctypes.byref(off)) == 1001
    assert lib.zx_ipc_import(bytes(64), None) == 1001
    assert lib.zx_ipc_close(0) == 1001


def test_selftest_arguments(zx):
    lib = zx.lib()
    assert lib.zx_selftest_bounded_wait(0, 1000, None) == 1001
    assert lib.zx_selftest_bounded_wait(0x1002, 1000, None) == 1003
    assert lib.zx_selftest_bounded_wait(0x1000, 0, None) == 1002
    assert lib.zx_selftest_bounded_wait(0x1000, 2000000, None) == 1002


def test_policy_validation(zx):
    lib = zx.lib()
    assert lib.zx_set_kernel_policy(7) == 1002
    assert lib.zx_set_kernel_policy(-1) == 1002
    for p in (1, 2, 3, 4, 5, 6, 0):
        assert lib.zx_set_kernel_policy(p) == 0


def test_valid_call_without_gpu_fails_loudly(zx):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    rc, msg = _err(zx, zx.lib().zx_gemm_s8(*GOOD, 128, 256, 128, 0, None))
    assert rc != 0 and msg, "a valid call on a machine without a GPU must return an error"


def test_errors_are_per_thread(zx):
    """zx_last_error is thread-local (the reference's single err_buf is not thread-safe)."""
    import threading

    lib = zx.lib()
    seen = {}

    def worker(name, args):
        lib.zx_gemm_s8(*args, None)
        seen[name] = zx.abi.last_error()

    t1 = threading.Thread(target=worker, args=("a", (0, 1, 2, 128, 128, 128, 0)))
    t1.start()
    t1.join()
    lib.zx_gemm_s8(*GOOD, 128, 128, 100, 0, None)
    assert "null" in seen["a"] and "K=100" in zx.abi.last_error()


def test_nn_layout_paths_arguments(zx):
    """The reference-layout entry points validate shape, workspace and alignment before any
    CUDA call (ZX_ERR_NULL 1001, ZX_ERR_SHAPE 1002, ZX_ERR_ALIGN 1003)."""
    lib = zx.lib()
    out = ctypes.c_uint64(0)
    assert lib.zx_gemm_nn_workspace_bytes(0, 256, 512, 1024, ctypes.byref(out)) == 0 and out.value == 512 * 1024
    assert lib.zx_gemm_nn_workspace_bytes(1, 100, 512, 1024, ctypes.byref(out)) == 0
    assert out.value == ((100 * 1024 + 255) // 256) * 256 + 512 * 512
    assert lib.zx_gemm_nn_workspace_bytes(2, 256, 512, 1024, ctypes.byref(out)) == 0
    assert out.value == 256 * 512 + 256 * 32 * 4 + 512 * 1024  # int8 A_c | int8 metadata | int8 B
    assert lib.zx_gemm_nn_workspace_bytes(3, 256, 512, 1024, ctypes.byref(out)) == 1002
    meta = 0x2000
    rc, msg = _err(zx, lib.zx_gemm_sp_s8_nn(GOOD[0], meta, GOOD[1], GOOD[2], 256, 512, 1024, 0, 0, None))
    assert rc == 1001 and "workspace" in msg
    rc, msg = _err(zx, lib.zx_gemm_sp_s8_nn(GOOD[0], meta, GOOD[1], GOOD[2], 256, 512, 1024, 0x4000, 4096, None))
    assert rc == 1002 and "workspace" in msg
    rc, msg = _err(zx, lib.zx_gemm_sp_s8_nn(GOOD[0], meta, GOOD[1], GOOD[2], 200, 512, 1024, 0x4000, 1 << 30, None))
    assert rc == 1002 and "M=200" in msg
    rc, msg = _err(zx, lib.zx_gemm_s4s4_nn(*GOOD, 256, 512, 96, 0x4000, 1 << 30, None))
    assert rc == 1002 and "K=96" in msg
    rc, msg = _err(zx, lib.zx_gemm_s4s4_nn(*GOOD, 256, 512, 1024, 0x4008, 1 << 30, None))
    assert rc == 1003 and "workspace" in msg
    rc, msg = _err(zx, lib.zx_gemm_sp_s4_nn(GOOD[0], meta, GOOD[1], GOOD[2], 256, 512, 1024, 0x4000, 4096, None))
    assert rc == 1002 and "workspace" in msg
    rc, msg = _err(zx, lib.zx_gemm_sp_s4_nn(GOOD[0], meta, GOOD[1], GOOD[2], 256, 512, 640, 0x4000, 1 << 30, None))
    assert rc == 1002 and "K=640" in msg
    rc, msg = _err(zx, lib.zx_gemm_sp_s4_nn(GOOD[0], 0, GOOD[1], GOOD[2], 256, 512, 1024, 0x4000, 1 << 30, None))
    assert rc == 1001 and "metadata" in msg


def test_mgpu_arguments(zx):
    """zx_gemm_s8_mgpu validates the shard list before any CUDA launch."""
    lib = zx.lib()
    arr = lambda *v: (ctypes.c_uint64 * len(v))(*v)  # noqa: E731
    devs = (ctypes.c_int * 2)(0, 0)
    rc, msg = _err(zx, lib.zx_gemm_s8_mgpu(0, devs, arr(1, 2), arr(1, 2), arr(1, 2), 256, 256, 256, 0, None))
    assert rc == 1002 and "ngpus=0" in msg
    rc, msg = _err(zx, lib.zx_gemm_s8_mgpu(2, None, arr(1, 2), arr(1, 2), arr(1, 2), 256, 256, 256, 0, None))
    assert rc == 1001
    rc, msg = _err(zx, lib.zx_gemm_s8_mgpu(2, devs, arr(0x10000, 0x20000), arr(0x30000, 0x40000),
                                          arr(0x50000, 0x60000), 1, 256, 256, 0, None))
    assert rc == 1002 and "fewer rows" in msg


def test_zig_bindings_cover_every_declared_symbol():
    """INTEGRATION.md's extern declarations (the binding a Zig caller pastes) name every entry point
    of include/zoxide_gemm.h, and nothing else."""
    import re
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    decl = set(re.findall(r"ZX_API\s+[\w\s\*]+?\b(zx_\w+)\s*\(", (root / "include" / "zoxide_gemm.h").read_text()))
    ext = set(re.findall(r"fn (zx_\w+)\(", (root / "INTEGRATION.md").read_text()))
    assert decl == ext, (sorted(decl - ext), sorted(ext - decl))
