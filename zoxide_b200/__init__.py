"""zoxide_b200 — B200-native (sm_100a) quantised GEMM path behind zoxide's kernel ABI.

The product is libzoxide_b200.so (C ABI: include/zoxide_gemm.h): hand-written tcgen05 / TMA
kernels plus the host launcher. This package is a thin Python caller over that ABI for tests
and benchmarks. The functions below take torch CUDA tensors (torch supplies device memory and
streams) and call the C entry points; shapes and layouts follow the reference kernel ABI
(zig-ecosystem/zoxide src/examples_abi.zig).
"""
from __future__ import annotations

from . import abi
from .abi import NN, NT, ZxError, check, last_kernel, lib

__all__ = [
    "NN", "NT", "ZxError", "lib", "check", "last_kernel", "gemm_s8", "gemm_s8_mgpu", "gemm_s8_replicated", "gemm_host", "gemm_s8_scaled_bf16", "gemm_bf16", "gemm_f16", "hgemm_tma", "gemm_w4a8", "gemm_w4a8_ws", "w4a8_workspace", "w4a8_workspace_bytes", "gemm_w4a8_noalloc",
    "gemm_sp_s8", "gemm_sp_s8_nn", "gemm_s4s4_nn", "gemm_sp_s4_nn", "nn_workspace_bytes", "NN_SP_S8", "NN_S4S4",
    "NN_SP_S4",
    "imma_s8", "hgemm_bf16", "launch_imma_s8_ref", "launch_imma_s4_ref", "launch_imma_sp_s8_ref",
    "launch_imma_sp_s4_ref",
    "set_kernel_policy", "device_status", "device_status_clear", "sm_count",
]


def _stream(stream) -> int | None:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream or None


def _ptr(t) -> int:
    if not t.is_cuda:
        raise ValueError("zoxide_b200 operates on CUDA tensors only (no CPU path)")
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return t.data_ptr()


def gemm_s8(A, B, C=None, layout: int = NT, stream=None):
    """C (int32 M x N) = A (int8 M x K) * op(B); op(B) = B^T for NT (B is N x K), B for NN."""
    import torch

    M, K = A.shape
    N = B.shape[0] if layout == NT else B.shape[1]
    if C is None:
        C = torch.empty((M, N), dtype=torch.int32, device=A.device)
    check(lib().zx_gemm_s8(_ptr(A), _ptr(B), _ptr(C), M, N, K, layout, _stream(stream)))
    return C


def gemm_s8_mgpu(A_shards, B_copies, C_shards, M: int, layout: int = NT, streams=None):
    """zx_gemm_s8_mgpu: shard i = rows [i*M/n, (i+1)*M/n) on A_shards[i].device; B_copies[i] is a full
    B on the same device, C_shards[i] that device's rows of C. Enqueues on `streams` (one per
    shard; default: each device's current stream) and returns C_shards."""
    import ctypes

    import torch

    n = len(A_shards)
    if not (len(B_copies) == len(C_shards) == n):
        raise ValueError("one A shard, one B copy and one C shard per GPU")
    K = A_shards[0].shape[1]
    N = B_copies[0].shape[0] if layout == NT else B_copies[0].shape[1]
    devs = (ctypes.c_int * n)(*[t.device.index for t in A_shards])
    arr = lambda ts: (ctypes.c_uint64 * n)(*[_ptr(t) for t in ts])  # noqa: E731
    if streams is None:
        streams = [torch.cuda.current_stream(t.device) for t in A_shards]
    ss = (ctypes.c_void_p * n)(*[s.cuda_stream or None for s in streams])
    check(lib().zx_gemm_s8_mgpu(n, devs, arr(A_shards), arr(B_copies), arr(C_shards), M, N, K, layout, ss))
    return C_shards


def gemm_s8_replicated(A, B, C, peers, stream=None):
    """gemm_s8 (NT) that also stores C into each device address in `peers` (up to 7 buffers of
    at least M x N int32 from that address, e.g. the same rows of C on the other GPUs, mapped
    with shard.PeerBuffers). The peer copies are complete when the kernel is."""
    import ctypes

    M, K = A.shape
    N = B.shape[0]
    arr = (ctypes.c_uint64 * max(1, len(peers)))(*[int(x) for x in peers])
    check(lib().zx_gemm_s8_replicated(_ptr(A), _ptr(B), _ptr(C), M, N, K, arr, len(peers), _stream(stream)))
    return C


def gemm_host(A_host, B_host, C_host, A_dev, B_dev, C_dev, stream=None):
    """C_host = A_host * B_host^T (int8 -> int32 or bf16 -> fp32, NT) with the PCIe copies overlapped
    with the kernels (zx_gemm_s8_host / zx_gemm_bf16_host). Host tensors: CPU, contiguous, pinned
    for the overlap; device tensors: scratch of the same shapes. Enqueued on `stream`."""
    import torch

    for t in (A_host, B_host, C_host):
        if t.is_cuda or not t.is_contiguous():
            raise ValueError("host operands must be contiguous CPU tensors")
    M, K = A_host.shape
    N = B_host.shape[0]
    if A_host.dtype == torch.int8:
        fn = lib().zx_gemm_s8_host
    elif A_host.dtype == torch.bfloat16:
        fn = lib().zx_gemm_bf16_host
    else:
        raise ValueError(f"unsupported dtype {A_host.dtype}")
    check(fn(A_host.data_ptr(), B_host.data_ptr(), C_host.data_ptr(), _ptr(A_dev), _ptr(B_dev), _ptr(C_dev),
             M, N, K, _stream(stream)))
    return C_host


def gemm_s8_scaled_bf16(A, B, row_scale, col_scale, C=None, layout: int = NT, stream=None):
    """C (bf16 M x N) = bf16(((float)(A op(B)) * row_scale[m]) * col_scale[n])."""
    import torch

    M, K = A.shape
    N = B.shape[0] if layout == NT else B.shape[1]
    if C is None:
        C = torch.empty((M, N), dtype=torch.bfloat16, device=A.device)
    check(lib().zx_gemm_s8_scaled_bf16(_ptr(A), _ptr(B), _ptr(row_scale), _ptr(col_scale),
                                       _ptr(C), M, N, K, layout, _stream(stream)))
    return C


def gemm_bf16(A, B, C=None, layout: int = NT, stream=None):
    """C (fp32 M x N) = A (bf16 M x K) * op(B) on tcgen05 kind::f16."""
    import torch

    M, K = A.shape
    N = B.shape[0] if layout == NT else B.shape[1]
    if C is None:
        C = torch.empty((M, N), dtype=torch.float32, device=A.device)
    check(lib().zx_gemm_bf16(_ptr(A), _ptr(B), _ptr(C), M, N, K, layout, _stream(stream)))
    return C


def gemm_f16(A, B, C=None, layout: int = NT, stream=None):
    """C (fp32 M x N) = A (f16 M x K) * op(B) on tcgen05 kind::f16 (the hgemm_tma operand type)."""
    import torch

    M, K = A.shape
    N = B.shape[0] if layout == NT else B.shape[1]
    if C is None:
        C = torch.empty((M, N), dtype=torch.float32, device=A.device)
    check(lib().zx_gemm_f16(_ptr(A), _ptr(B), _ptr(C), M, N, K, layout, _stream(stream)))
    return C


def gemm_w4a8(A, W, C=None, stream=None):
    """C (int32 M x N) = A (int8 M x K) * W^T, W = N x K/2 bytes of packed s4 (low nibble = even k)."""
    import torch

    M, K = A.shape
    N = W.shape[0]
    if W.shape[1] * 2 != K:
        raise ValueError(f"W has {W.shape[1]} bytes per row, expected K/2 = {K // 2}")
    if C is None:
        C = torch.empty((M, N), dtype=torch.int32, device=A.device)
    check(lib().zx_gemm_w4a8(_ptr(A), _ptr(W), _ptr(C), M, N, K, _stream(stream)))
    return C


def w4a8_workspace_bytes(M: int, N: int, K: int) -> int:
    """Bytes of workspace gemm_w4a8_ws needs for this shape on the current device (0: none)."""
    import ctypes

    out = ctypes.c_uint64(0)
    check(lib().zx_gemm_w4a8_workspace_bytes(M, N, K, ctypes.byref(out)))
    return out.value


def w4a8_workspace(M: int, N: int, K: int, device=None):
    """A zero-filled workspace tensor for gemm_w4a8_ws (kept zero by every call)."""
    import torch

    return torch.zeros(max(16, w4a8_workspace_bytes(M, N, K)), dtype=torch.uint8, device=device or "cuda")


def gemm_w4a8_ws(A, W, workspace, C=None, stream=None):
    """gemm_w4a8 with a caller workspace: C is stored once, without a zeroing pass and atomics."""
    import torch

    M, K = A.shape
    N = W.shape[0]
    if W.shape[1] * 2 != K:
        raise ValueError(f"W has {W.shape[1]} bytes per row, expected K/2 = {K // 2}")
    if C is None:
        C = torch.empty((M, N), dtype=torch.int32, device=A.device)
    check(lib().zx_gemm_w4a8_ws(_ptr(A), _ptr(W), _ptr(C), M, N, K, _ptr(workspace),
                                workspace.numel() * workspace.element_size(), _stream(stream)))
    return C


def gemm_w4a8_noalloc(A, W, C=None, stream=None):
    """gemm_w4a8 for M <= 32 whose library call allocates nothing: its split-K scratch is an array
    built into the library (shared by every call on a device; calls must not overlap on the GPU).
    Pass C to allocate nothing here either: C=None makes this wrapper allocate the output with
    torch."""
    import torch

    M, K = A.shape
    N = W.shape[0]
    if W.shape[1] * 2 != K:
        raise ValueError(f"W has {W.shape[1]} bytes per row, expected K/2 = {K // 2}")
    if C is None:
        C = torch.empty((M, N), dtype=torch.int32, device=A.device)
    check(lib().zx_gemm_w4a8_noalloc(_ptr(A), _ptr(W), _ptr(C), M, N, K, _stream(stream)))
    return C


def gemm_sp_s8(A_c, meta, B, C=None, stream=None):
    """C (int32 M x N) = decompress(A_c, meta) * B^T; A_c M x K/2 int8, meta M x K/32 uint32
    (reference nibble format), B N x K int8."""
    import torch

    M, Kh = A_c.shape
    K = 2 * Kh
    N = B.shape[0]
    if meta.shape != (M, K // 32) or B.shape[1] != K:
        raise ValueError(f"shape mismatch: A_c {tuple(A_c.shape)} meta {tuple(meta.shape)} B {tuple(B.shape)}")
    if C is None:
        C = torch.empty((M, N), dtype=torch.int32, device=A_c.device)
    check(lib().zx_gemm_sp_s8(_ptr(A_c), _ptr(meta), _ptr(B), _ptr(C), M, N, K, _stream(stream)))
    return C


NN_SP_S8, NN_S4S4, NN_SP_S4 = 0, 1, 2


def nn_workspace_bytes(op: int, M: int, N: int, K: int) -> int:
    """Workspace bytes of gemm_sp_s8_nn (op NN_SP_S8), gemm_s4s4_nn (op NN_S4S4) or gemm_sp_s4_nn
    (op NN_SP_S4)."""
    import ctypes

    out = ctypes.c_uint64(0)
    check(lib().zx_gemm_nn_workspace_bytes(op, M, N, K, ctypes.byref(out)))
    return out.value


def gemm_sp_s8_nn(A_c, meta, B_kn, workspace, C=None, stream=None):
    """gemm_sp_s8 with B in the reference's row-major K x N layout (imma_sp_s8), transposed into
    `workspace` (>= N * K bytes) first."""
    import torch

    M, Kh = A_c.shape
    K, N = B_kn.shape
    if 2 * Kh != K or meta.shape != (M, K // 32):
        raise ValueError(f"shape mismatch: A_c {tuple(A_c.shape)} meta {tuple(meta.shape)} B {tuple(B_kn.shape)}")
    if C is None:
        C = torch.empty((M, N), dtype=torch.int32, device=A_c.device)
    check(lib().zx_gemm_sp_s8_nn(_ptr(A_c), _ptr(meta), _ptr(B_kn), _ptr(C), M, N, K, _ptr(workspace),
                                 workspace.numel() * workspace.element_size(), _stream(stream)))
    return C


def gemm_s4s4_nn(A_s4, B_s4_kn, workspace, C=None, stream=None):
    """imma_s4's operands: A M x K/2 bytes (s4 along K), B K x N/2 bytes (s4 along N); the
    workspace (nn_workspace_bytes(NN_S4S4, ...)) receives A as int8 and B repacked along K."""
    import torch

    M, Kh = A_s4.shape
    K, Nh = B_s4_kn.shape
    if 2 * Kh != K:
        raise ValueError(f"A has {Kh} bytes per row, B has {K} rows: expected K/2 bytes per A row")
    N = 2 * Nh
    if C is None:
        C = torch.empty((M, N), dtype=torch.int32, device=A_s4.device)
    check(lib().zx_gemm_s4s4_nn(_ptr(A_s4), _ptr(B_s4_kn), _ptr(C), M, N, K, _ptr(workspace),
                                workspace.numel() * workspace.element_size(), _stream(stream)))
    return C


def gemm_sp_s4_nn(A_c4, meta4, B_s4_kn, workspace, C=None, stream=None):
    """imma_sp_s4's operands: A_c4 M x K/4 bytes of 4:8 pair-clustered s4, meta4 M x K/64 words,
    B K x N/2 bytes (s4 along N); the workspace (nn_workspace_bytes(NN_SP_S4, ...)) receives the
    int8 2:4 operands, then the 2:4 sparse kernels run."""
    import torch

    M, Kq = A_c4.shape
    K, Nh = B_s4_kn.shape
    if 4 * Kq != K or meta4.shape != (M, K // 64):
        raise ValueError(f"shape mismatch: A_c {tuple(A_c4.shape)} meta {tuple(meta4.shape)} B {tuple(B_s4_kn.shape)}")
    N = 2 * Nh
    if C is None:
        C = torch.empty((M, N), dtype=torch.int32, device=A_c4.device)
    check(lib().zx_gemm_sp_s4_nn(_ptr(A_c4), _ptr(meta4), _ptr(B_s4_kn), _ptr(C), M, N, K, _ptr(workspace),
                                 workspace.numel() * workspace.element_size(), _stream(stream)))
    return C


def imma_s8(a, b, c, n: int, stream=None) -> None:
    """Reference signature imma_s8(a, b, c, n) (src/examples_abi.zig:42): square, B is K x N."""
    check(lib().zx_imma_s8(_ptr(a), _ptr(b), _ptr(c), n, _stream(stream)))


def hgemm_bf16(a, b, c, n: int, stream=None) -> None:
    """Reference signature hgemm_bf16(a, b, c, n) (src/examples_abi.zig:33-36)."""
    check(lib().zx_hgemm_bf16(_ptr(a), _ptr(b), _ptr(c), n, _stream(stream)))


def hgemm_tma(a, b, c, n: int, desc_a: int = 0, desc_b: int = 0, stream=None) -> None:
    """Reference signature hgemm_tma(a, b, c, n, desc_a, desc_b) (src/examples_abi.zig:168-190): f16
    A, B row-major n x n (B is K x N), fp32 C; the descriptors are accepted and not read."""
    check(lib().zx_hgemm_tma(_ptr(a), _ptr(b), _ptr(c), n, desc_a, desc_b, _stream(stream)))


def launch_imma_s8_ref(a, b, c, n: int, stream=None) -> None:
    """The reference's own imma_s8_$_immaS8 launch (block 128, grid n/128 x n/128, no dynamic
    shared memory, no cluster): A n x n int8, B n x n int8 row-major K x N, C n x n int32."""
    check(lib().zx_launch_imma_s8_ref(_ptr(a), _ptr(b), _ptr(c), n, _stream(stream)))


def launch_imma_s4_ref(a, b, c, n: int, stream=None) -> None:
    """imma_s4_$_immaS4 under the reference launch contract: A n x n s4 packed along K (n x n/2
    bytes), B K x N s4 packed along N (n x n/2 bytes), C n x n int32."""
    check(lib().zx_launch_imma_s4_ref(_ptr(a), _ptr(b), _ptr(c), n, _stream(stream)))


def launch_imma_sp_s8_ref(a_c, b, meta, c, n: int, stream=None) -> None:
    """imma_sp_s8_$_immaSpS8 under the reference launch contract: A_c n x n/2 int8 kept values,
    B n x n int8 row-major K x N, meta n x n/32 u32 (reference nibble format), C n x n int32."""
    check(lib().zx_launch_imma_sp_s8_ref(_ptr(a_c), _ptr(b), _ptr(meta), _ptr(c), n, _stream(stream)))


def launch_imma_sp_s4_ref(a_c, b, meta, c, n: int, stream=None) -> None:
    """imma_sp_s4_$_immaSpS4 under the reference launch contract: A n x n/4 bytes of 4:8
    pair-clustered s4, B n x n/2 bytes (K x N s4 packed along N), meta n x n/64 u32, C n x n int32."""
    check(lib().zx_launch_imma_sp_s4_ref(_ptr(a_c), _ptr(b), _ptr(meta), _ptr(c), n, _stream(stream)))


def set_kernel_policy(policy: int) -> None:
    """0 automatic, 1 one-SM 128x256 tiles, 2 two-SM pair tiles (256 or 224 wide), 3 two-SM 256-wide,
    4 two-SM 256x512 tiles, 5 two-SM 256x480 tiles, 6 two-SM 256x464 tiles (4-6: K-major B). For the
    2:4 sparse GEMMs: 1-3 the 256 x 224 kernel, 4-5 the 256 x 480 one, 6 the 512 x 224 one."""
    check(lib().zx_set_kernel_policy(policy))


def device_status() -> int:
    import ctypes

    v = ctypes.c_uint32(0)
    rc = lib().zx_device_status(ctypes.byref(v))
    if rc not in (0, abi.ZX_ERR_TIMEOUT):
        check(rc)
    return v.value


def device_status_clear() -> None:
    check(lib().zx_device_status_clear())


def sm_count() -> int:
    return lib().zx_device_sm_count()
