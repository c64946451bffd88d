"""ctypes view of libzoxide_b200.so — the C ABI declared in include/zoxide_gemm.h.

Python is only a caller here: every entry point runs the C++/CUDA library. If the library is
missing the import fails loudly; there is no Python or CPU fallback for any operation.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_build" / "libzoxide_b200.so"

NT, NN = 0, 1

ERRORS = {
    1001: "ZX_ERR_NULL",
    1002: "ZX_ERR_SHAPE",
    1003: "ZX_ERR_ALIGN",
    1004: "ZX_ERR_LAYOUT",
    1005: "ZX_ERR_ARCH",
    1006: "ZX_ERR_DRIVER",
    1007: "ZX_ERR_TIMEOUT",
    1008: "ZX_ERR_NO_DEVICE",
}
ZX_ERR_NULL, ZX_ERR_SHAPE, ZX_ERR_ALIGN, ZX_ERR_LAYOUT = 1001, 1002, 1003, 1004
ZX_ERR_ARCH, ZX_ERR_DRIVER, ZX_ERR_TIMEOUT, ZX_ERR_NO_DEVICE = 1005, 1006, 1007, 1008

# name -> (restype, argtypes); mirrors include/zoxide_gemm.h one to one.
_P, _U32, _I = C.c_uint64, C.c_uint32, C.c_int
_S = C.c_void_p
SIGNATURES = {
    "zx_version": (_I, []),
    "zx_last_error": (C.c_char_p, []),
    "zx_last_kernel": (C.c_char_p, []),
    "zx_set_kernel_policy": (_I, [_I]),
    "zx_gemm_s8": (_I, [_P, _P, _P, _U32, _U32, _U32, _I, _S]),
    "zx_gemm_s8_scaled_bf16": (_I, [_P, _P, _P, _P, _P, _U32, _U32, _U32, _I, _S]),
    "zx_gemm_s8_host": (_I, [_S, _S, _S, _P, _P, _P, _U32, _U32, _U32, _S]),
    "zx_gemm_bf16_host": (_I, [_S, _S, _S, _P, _P, _P, _U32, _U32, _U32, _S]),
    "zx_gemm_s8_mgpu": (_I, [_I, C.POINTER(C.c_int), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                            C.POINTER(C.c_uint64), _U32, _U32, _U32, _I, C.POINTER(C.c_void_p)]),
    "zx_gemm_s8_replicated": (_I, [_P, _P, _P, _U32, _U32, _U32, C.POINTER(C.c_uint64), _U32, _S]),
    "zx_ipc_export": (_I, [_P, C.c_char_p, C.POINTER(C.c_uint64)]),
    "zx_ipc_import": (_I, [C.c_char_p, C.POINTER(C.c_uint64)]),
    "zx_ipc_close": (_I, [_P]),
    "zx_gemm_bf16": (_I, [_P, _P, _P, _U32, _U32, _U32, _I, _S]),
    "zx_gemm_f16": (_I, [_P, _P, _P, _U32, _U32, _U32, _I, _S]),
    "zx_gemm_w4a8": (_I, [_P, _P, _P, _U32, _U32, _U32, _S]),
    "zx_gemm_w4a8_ws": (_I, [_P, _P, _P, _U32, _U32, _U32, _P, C.c_uint64, _S]),
    "zx_gemm_w4a8_workspace_bytes": (_I, [_U32, _U32, _U32, C.POINTER(C.c_uint64)]),
    "zx_gemm_w4a8_noalloc": (_I, [_P, _P, _P, _U32, _U32, _U32, _S]),
    "zx_gemm_sp_s8": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _S]),
    "zx_gemm_nn_workspace_bytes": (_I, [_I, _U32, _U32, _U32, C.POINTER(C.c_uint64)]),
    "zx_gemm_sp_s8_nn": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _P, C.c_uint64, _S]),
    "zx_gemm_s4s4_nn": (_I, [_P, _P, _P, _U32, _U32, _U32, _P, C.c_uint64, _S]),
    "zx_gemm_sp_s4_nn": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _P, C.c_uint64, _S]),
    "zx_imma_s8": (_I, [_P, _P, _P, _U32, _S]),
    "zx_hgemm_bf16": (_I, [_P, _P, _P, _U32, _S]),
    "zx_hgemm_tma": (_I, [_P, _P, _P, _U32, C.c_uint64, C.c_uint64, _S]),
    "zx_launch_imma_s8_ref": (_I, [_P, _P, _P, _U32, _S]),
    "zx_launch_hgemm_bf16_ref": (_I, [_P, _P, _P, _U32, _S]),
    "zx_launch_imma_s4_ref": (_I, [_P, _P, _P, _U32, _S]),
    "zx_launch_imma_sp_s8_ref": (_I, [_P, _P, _P, _P, _U32, _S]),
    "zx_launch_imma_sp_s4_ref": (_I, [_P, _P, _P, _P, _U32, _S]),
    "zx_launch_hgemm_bf16_mma_ref": (_I, [_P, _P, _P, _U32, _S]),
    "zx_launch_hgemm_tma_ref": (_I, [_P, _P, _P, _U32, C.c_uint64, C.c_uint64, _S]),
    "zx_device_status": (_I, [C.POINTER(C.c_uint32)]),
    "zx_device_status_clear": (_I, []),
    "zx_selftest_bounded_wait": (_I, [_P, _U32, _S]),
    "zx_device_sm_count": (_I, []),
}


class ZxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        self.code = code
        name = ERRORS.get(code, f"cudaError {code}")
        super().__init__(f"{name}: {msg}")


_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load the in-tree library (built by zoxide_b200.build / __graft_entry__.build)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m zoxide_b200.build` "
                "(there is no fallback implementation)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != 0:
        raise ZxError(rc, lib().zx_last_error().decode(errors="replace"))


def last_error() -> str:
    return lib().zx_last_error().decode(errors="replace")


def last_kernel() -> str:
    """Kernel launched by this thread's last successful GEMM call."""
    return lib().zx_last_kernel().decode(errors="replace")
