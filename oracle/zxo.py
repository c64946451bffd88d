"""ctypes bindings to oracle/_build/libzxo.so (see zxo.h for the contracts and citations)."""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libzxo.so"

NT, NN = 0, 1
REF_STATE_S8 = 0x13579BDF     # src/bench.zig:653
REF_STATE_S4 = 0x0FDB9753     # src/bench.zig:774
REF_STATE_SP_S8 = 0xC0FFEE11  # src/bench.zig:1029
REF_STATE_BF16 = 0x2468ACE0   # src/bench.zig:559
REF_STATE_SP_S4 = 0x5CA1AB1E  # src/bench.zig:1178
REF_VERIFY_STATE = 0xDEADBEEF  # src/bench.zig:717

__all__ = [
    "NT", "NN", "REF_STATE_S8", "REF_STATE_S4", "REF_STATE_SP_S8", "REF_STATE_BF16", "REF_STATE_SP_S4",
    "prune48_s4", "decompress48_s4", "unpack_s4",
    "REF_VERIFY_STATE", "build", "lib", "xorshift32", "state_from_seed", "fill_s8", "pack_s4",
    "s4_at", "fill_s4_packed", "prune24_s8", "fill_uniform_f32", "fill_normal_bf16",
    "f32_to_bf16", "bf16_to_f32", "dot_s8", "check_samples_s8", "ref_loop_s8", "gemm_s8",
    "gemm_s8_scaled_bf16", "scale_to_bf16", "gemm_w4a8", "gemm_sp_s8", "decompress24_s8",
    "gemm_bf16_f64", "matvec_s32", "gemv_chain_s8", "freivalds_s8", "num_threads",
    "Rng",
]


def build(force: bool = False) -> Path:
    src = [HERE / "zxo.c", HERE / "zxo.h", HERE / "Makefile"]
    if force or not LIB_PATH.exists() or any(s.stat().st_mtime > LIB_PATH.stat().st_mtime for s in src):
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        P, S, I, U32, I64, U64 = C.c_void_p, C.c_size_t, C.c_int, C.c_uint32, C.c_int64, C.c_uint64
        PU32 = C.POINTER(C.c_uint32)
        sig = {
            "zxo_xorshift32": (U32, [PU32]),
            "zxo_state_from_seed": (U32, [U64]),
            "zxo_fill_s8": (None, [P, S, PU32]),
            "zxo_pack_s4": (C.c_uint8, [C.c_int8, C.c_int8]),
            "zxo_s4_at": (C.c_int8, [P, S]),
            "zxo_fill_s4_packed": (None, [P, S, PU32]),
            "zxo_prune24_s8": (None, [S, S, PU32, P, P, P]),
            "zxo_fill_uniform_f32": (None, [P, S, C.c_float, C.c_float, PU32]),
            "zxo_fill_normal_bf16": (None, [P, S, C.c_double, PU32]),
            "zxo_f32_to_bf16_rne": (C.c_uint16, [C.c_float]),
            "zxo_bf16_to_f32": (C.c_float, [C.c_uint16]),
            "zxo_dot_s8": (I64, [P, P, S, S, I, S, S]),
            "zxo_check_samples_s8": (S, [P, P, P, S, S, S, I, S, U32, C.POINTER(S), C.POINTER(I64), C.POINTER(C.c_int32)]),
            "zxo_ref_loop_s8": (None, [P, P, P, S, S, I, S, S, I]),
            "zxo_gemm_s8": (None, [P, P, P, S, S, S, I, I]),
            "zxo_gemm_s8_scaled_bf16": (None, [P, P, P, P, P, S, S, I, S, S, I]),
            "zxo_scale_to_bf16": (C.c_uint16, [C.c_int32, C.c_float, C.c_float]),
            "zxo_gemm_w4a8": (None, [P, P, P, S, S, S, I]),
            "zxo_gemm_sp_s8": (None, [P, P, P, P, S, S, S, I, I]),
            "zxo_decompress24_s8": (None, [P, P, P, S, S]),
            "zxo_prune48_s4": (None, [S, S, PU32, P, P, P]),
            "zxo_decompress48_s4": (None, [P, P, P, S, S]),
            "zxo_unpack_s4": (None, [P, P, S]),
            "zxo_gemm_bf16_f64": (None, [P, P, P, S, S, I, S, S, I]),
            "zxo_matvec_s32": (None, [P, P, P, S, S, I]),
            "zxo_gemv_chain_s8": (None, [P, P, P, P, S, S, S, I, I]),
            "zxo_num_threads": (I, [I]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags.c_contiguous, "oracle buffers must be C-contiguous"
    return a.ctypes.data


class Rng:
    """A xorshift32 stream (src/bench.zig:26-33) held as a mutable state word."""

    def __init__(self, state: int):
        if state == 0:
            raise ValueError("xorshift32 state 0 is a fixed point")
        self.state = C.c_uint32(state & 0xFFFFFFFF)

    @classmethod
    def from_seed(cls, seed: int) -> "Rng":
        return cls(state_from_seed(seed))

    def next(self) -> int:
        return lib().zxo_xorshift32(C.byref(self.state))

    def s8(self, shape) -> np.ndarray:
        a = np.empty(shape, dtype=np.int8)
        lib().zxo_fill_s8(_p(a), a.size, C.byref(self.state))
        return a

    def s4_packed(self, shape_bytes) -> np.ndarray:
        a = np.empty(shape_bytes, dtype=np.uint8)
        lib().zxo_fill_s4_packed(_p(a), a.size, C.byref(self.state))
        return a

    def uniform_f32(self, n: int, lo: float, hi: float) -> np.ndarray:
        a = np.empty(n, dtype=np.float32)
        lib().zxo_fill_uniform_f32(_p(a), n, lo, hi, C.byref(self.state))
        return a

    def normal_bf16(self, shape, scale: float) -> np.ndarray:
        a = np.empty(shape, dtype=np.uint16)
        lib().zxo_fill_normal_bf16(_p(a), a.size, scale, C.byref(self.state))
        return a

    def prune24_s8(self, rows: int, k: int, want_dense: bool = True):
        comp = np.empty((rows, k // 2), dtype=np.int8)
        meta = np.empty((rows, k // 32), dtype=np.uint32)
        dense = np.empty((rows, k), dtype=np.int8) if want_dense else None
        lib().zxo_prune24_s8(rows, k, C.byref(self.state), _p(dense) if dense is not None else None,
                             _p(comp), _p(meta))
        return dense, comp, meta

    def prune48_s4(self, rows: int, k: int, want_dense: bool = True):
        """4:8 pair-clustered s4 A of runImmaSpS4: (dense int8 logical or None, comp bytes
        rows x k/4, meta rows x k/64)."""
        comp = np.empty((rows, k // 4), dtype=np.uint8)
        meta = np.empty((rows, k // 64), dtype=np.uint32)
        dense = np.empty((rows, k), dtype=np.int8) if want_dense else None
        lib().zxo_prune48_s4(rows, k, C.byref(self.state), _p(dense) if dense is not None else None,
                             _p(comp), _p(meta))
        return dense, comp, meta


def xorshift32(state: int) -> tuple[int, int]:
    s = C.c_uint32(state)
    v = lib().zxo_xorshift32(C.byref(s))
    return v, s.value


def state_from_seed(seed: int) -> int:
    return lib().zxo_state_from_seed(seed)


def fill_s8(n: int, state: int) -> tuple[np.ndarray, int]:
    r = Rng(state)
    return r.s8(n), r.state.value


def pack_s4(even: int, odd: int) -> int:
    return lib().zxo_pack_s4(even, odd)


def s4_at(packed: np.ndarray, idx: int) -> int:
    return lib().zxo_s4_at(_p(packed), idx)


def fill_s4_packed(nbytes: int, state: int) -> tuple[np.ndarray, int]:
    r = Rng(state)
    return r.s4_packed(nbytes), r.state.value


def prune24_s8(rows: int, k: int, state: int):
    r = Rng(state)
    d, c, m = r.prune24_s8(rows, k)
    return d, c, m, r.state.value


def fill_uniform_f32(n: int, lo: float, hi: float, state: int):
    r = Rng(state)
    return r.uniform_f32(n, lo, hi), r.state.value


def fill_normal_bf16(n: int, scale: float, state: int):
    r = Rng(state)
    return r.normal_bf16(n, scale), r.state.value


def f32_to_bf16(x: float) -> int:
    return lib().zxo_f32_to_bf16_rne(x)


def bf16_to_f32(b: int) -> float:
    return lib().zxo_bf16_to_f32(b)


def dot_s8(A, B, N, K, layout, row, col) -> int:
    return lib().zxo_dot_s8(_p(A), _p(B), N, K, layout, row, col)


def check_samples_s8(A, B, Cm, M, N, K, layout, samples=256, vstate=REF_VERIFY_STATE):
    fb, w, g = C.c_size_t(0), C.c_int64(0), C.c_int32(0)
    bad = lib().zxo_check_samples_s8(_p(A), _p(B), _p(Cm), M, N, K, layout, samples, vstate,
                                     C.byref(fb), C.byref(w), C.byref(g))
    return bad, (fb.value, w.value, g.value)


def ref_loop_s8(A, B, N, K, layout, r0, r1, threads=0) -> np.ndarray:
    out = np.empty((r1 - r0, N), dtype=np.int64)
    lib().zxo_ref_loop_s8(_p(A), _p(B), _p(out), N, K, layout, r0, r1, threads)
    return out


def gemm_s8(A, B, M, N, K, layout, threads=0) -> np.ndarray:
    Cm = np.empty((M, N), dtype=np.int32)
    lib().zxo_gemm_s8(_p(A), _p(B), _p(Cm), M, N, K, layout, threads)
    return Cm


def gemm_s8_scaled_bf16(A, B, rs, cs, N, K, layout, r0, r1, threads=0) -> np.ndarray:
    out = np.empty((r1 - r0, N), dtype=np.uint16)
    lib().zxo_gemm_s8_scaled_bf16(_p(A), _p(B), _p(rs), _p(cs), _p(out), N, K, layout, r0, r1, threads)
    return out


def scale_to_bf16(acc: int, rs: float, cs: float) -> int:
    return lib().zxo_scale_to_bf16(acc, rs, cs)


def gemm_w4a8(A, W, M, N, K, threads=0) -> np.ndarray:
    Cm = np.empty((M, N), dtype=np.int32)
    lib().zxo_gemm_w4a8(_p(A), _p(W), _p(Cm), M, N, K, threads)
    return Cm


def gemm_sp_s8(comp, meta, B, M, N, K, layout, threads=0) -> np.ndarray:
    Cm = np.empty((M, N), dtype=np.int32)
    lib().zxo_gemm_sp_s8(_p(comp), _p(meta), _p(B), _p(Cm), M, N, K, layout, threads)
    return Cm


def prune48_s4(rows: int, k: int, state: int):
    r = Rng(state)
    d, c, m = r.prune48_s4(rows, k)
    return d, c, m, r.state.value


def decompress48_s4(comp, meta, M, K) -> np.ndarray:
    d = np.empty((M, K), dtype=np.int8)
    lib().zxo_decompress48_s4(_p(comp), _p(meta), _p(d), M, K)
    return d


def unpack_s4(packed: np.ndarray, shape) -> np.ndarray:
    """Packed s4 (two per byte along the last axis, low nibble first) -> int8 of `shape`."""
    out = np.empty(shape, dtype=np.int8)
    assert out.size == 2 * packed.size
    lib().zxo_unpack_s4(_p(np.ascontiguousarray(packed)), _p(out), out.size)
    return out


def decompress24_s8(comp, meta, M, K) -> np.ndarray:
    d = np.empty((M, K), dtype=np.int8)
    lib().zxo_decompress24_s8(_p(comp), _p(meta), _p(d), M, K)
    return d


def gemm_bf16_f64(A, B, N, K, layout, r0, r1, threads=0) -> np.ndarray:
    out = np.empty((r1 - r0, N), dtype=np.float64)
    lib().zxo_gemm_bf16_f64(_p(A), _p(B), _p(out), N, K, layout, r0, r1, threads)
    return out


def matvec_s32(Cm, x, M, N, threads=0) -> np.ndarray:
    y = np.empty(M, dtype=np.int64)
    lib().zxo_matvec_s32(_p(Cm), _p(x), _p(y), M, N, threads)
    return y


def gemv_chain_s8(A, B, x, M, N, K, layout, threads=0) -> np.ndarray:
    y = np.empty(M, dtype=np.int64)
    lib().zxo_gemv_chain_s8(_p(A), _p(B), _p(x), _p(y), M, N, K, layout, threads)
    return y


def freivalds_s8(A, B, Cm, M, N, K, layout, rounds=3, seed=1234) -> bool:
    """Exact size-independent check of C == A op(B): C x == A (op(B) x) for random int x."""
    rng = np.random.default_rng(seed)
    for _ in range(rounds):
        x = rng.integers(-1000, 1000, size=N, dtype=np.int64)
        if not np.array_equal(matvec_s32(Cm, x, M, N), gemv_chain_s8(A, B, x, M, N, K, layout)):
            return False
    return True


def num_threads(requested: int = 0) -> int:
    return lib().zxo_num_threads(requested)
