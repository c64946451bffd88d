/* zoxide_gemm.h — C ABI of the B200 (sm_100a) quantised-GEMM path.
 *
 * Plain C types only: device buffers are 64-bit device addresses (CUdeviceptr / the value of a
 * cudaMalloc'd pointer), streams are opaque handles (cudaStream_t / CUstream; 0 = legacy default
 * stream). Every buffer is owned by the caller; no entry point allocates device memory or keeps
 * state between calls beyond per-device attribute caches. Calls are asynchronous on `stream`.
 *
 * Layout names follow BLAS "op" letters for C = A * op(B), A always row-major M x K:
 *   ZX_LAYOUT_NT  B stored N x K with K contiguous ("B column-major")
 *   ZX_LAYOUT_NN  B stored K x N with N contiguous (the reference's own layout:
 *                 src/examples/imma_s8.zig:75 loads b[(k0+k)*n + col]; src/bench.zig:726)
 *
 * Return codes: 0 on success; 1..999 are cudaError_t values passed through; ZX_ERR_* below are
 * this library's own. Argument checks run before any CUDA call, mirroring the reference's
 * pre-launch geometry validation (src/host.zig:437-494) and tensor-map validation
 * (src/cuda_driver.zig:414-451). zx_last_error() returns a per-thread message for the last
 * failure on that thread (the reference keeps one shared buffer, src/cuda_driver.zig:104-108).
 */
#ifndef ZOXIDE_GEMM_H
#define ZOXIDE_GEMM_H

#include <stdint.h>

#if defined(__GNUC__)
#define ZX_API __attribute__((visibility("default")))
#else
#define ZX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef uint64_t zx_devptr;
typedef void* zx_stream;

enum zx_layout { ZX_LAYOUT_NT = 0, ZX_LAYOUT_NN = 1 };
/* Operations of zx_gemm_nn_workspace_bytes. */
enum zx_nn_op { ZX_NN_SP_S8 = 0, ZX_NN_S4S4 = 1, ZX_NN_SP_S4 = 2 };

enum zx_error {
  ZX_OK = 0,
  ZX_ERR_NULL = 1001,      /* a required pointer is 0 */
  ZX_ERR_SHAPE = 1002,     /* M/N/K out of range or not a supported multiple */
  ZX_ERR_ALIGN = 1003,     /* a buffer is not 16-byte aligned */
  ZX_ERR_LAYOUT = 1004,    /* unknown zx_layout value */
  ZX_ERR_ARCH = 1005,      /* current device is not sm_100 (B200) */
  ZX_ERR_DRIVER = 1006,    /* driver entry point missing or cuTensorMapEncodeTiled failed */
  ZX_ERR_TIMEOUT = 1007,   /* a kernel's bounded device wait gave up (see zx_device_status) */
  ZX_ERR_NO_DEVICE = 1008  /* no CUDA device visible */
};

/* Library version as 10000*major + 100*minor + patch. */
ZX_API int zx_version(void);

/* Tile policy for the dense GEMM entry points (process-wide): 0 = automatic (picks from the
 * number of full-machine waves of each tile shape: one-SM tiles for M <= 128 or when they fit
 * one wave, 256 x 512 two-SM tiles for short int8 launches and bf16, else 256 x 256 / 256 x 224
 * two-SM tiles), 1 = always one-SM 128 x 256 tiles, 2 = always two-SM tiles (256 x 256, or
 * 256 x 224 where that evens out the waves of tiles over the 74 SM pairs), 3 = always two-SM
 * 256 x 256 tiles, 4 = two-SM 256 x 512 tiles (B K-major; the NN layout uses policy 3),
 * 5 = two-SM 256 x 480 tiles (hi half 224 wide; 256 x 512 for the scaled-bf16 epilogue; B K-major),
 * 6 = two-SM 256 x 464 tiles (hi half 208 wide; otherwise as 5); the automatic choice also weighs
 * the 480- and 464-wide tiles (e.g. the 4- and 8-GPU M shards of 8192^3 run on 464).
 * zx_gemm_sp_s8: 0 = automatic (512 x 224 tiles of two 256-row blocks when they need no more work
 * per wave than 256 x 224 tiles, e.g. 8192^3; else 256 x 224), 1-3 = 256 x 224, 4-5 = 256 x 480,
 * 6 = 512 x 224.
 * A tuning and testing knob; results are identical. No reference counterpart (the reference
 * picks one tile per kernel file). */
ZX_API int zx_set_kernel_policy(int policy);

/* Message for the last non-zero return on the calling thread ("" if none). */
ZX_API const char* zx_last_error(void);

/* Name and launch shape of the kernel that the calling thread's last successful GEMM call
 * launched ("" if none), e.g. "gemm_tc2w_kernel 2-SM 256x512 tiles, 64 CTA pairs". For logs and
 * benchmarks; no reference counterpart. */
ZX_API const char* zx_last_kernel(void);

/* ---------------------------------------------------------------------------------------
 * int8 x int8 -> int32 GEMM, C[M x N] (int32, row-major) = A * op(B), exact int32 accumulate.
 * Replaces: examples_abi.imma_s8 (src/examples_abi.zig:42) launched by runImmaS8
 * (src/bench.zig:647-741) as kernel imma_s8_$_immaS8 (src/examples/imma_s8.zig:130-173),
 * generalised from square n (n % 128 == 0) to M, N, K.
 * Requirements: M, N, K >= 1, K % 16 == 0, N % 4 == 0 (NN: N % 16 == 0), buffers 16-B aligned.
 * Ragged M / N / K tails are handled (TMA zero-fill on loads, clipped stores).
 * ------------------------------------------------------------------------------------- */
ZX_API int zx_gemm_s8(zx_devptr A, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
               int layout, zx_stream stream);

/* GEMM on host buffers (the reference's bench flow: copy A and B in, launch, copy C out;
 * src/bench.zig:647-741), with the copies overlapped with the kernels: A and B move in blocks of
 * at least 1024 rows (at most 4 per operand) on one copy stream, each block of C is computed as soon as its rows of A and B
 * have arrived and copied back on two more (alternating). A_host M x K, B_host N x K (NT), C_host M x N row-major;
 * pinned host memory for the overlap. With pageable host memory the result is the same but the
 * copies do not overlap, and the host buffers are read when the call is made: A_host and B_host
 * must then already hold their final contents (no earlier work queued on `stream` may still write
 * them), which pinned memory does not require.
 * C is produced in growing L-shaped shells (the part of C that the blocks of A and B copied so far
 * complete), two GEMMs and two 2-D copies back per shell.
 * A_dev, B_dev, C_dev: device buffers of the same sizes (C_dev also ends up holding C, row-major).
 * Enqueued on `stream`: C_host is complete when work queued after the call on `stream` runs.
 * One call at a time per device enqueues (an internal lock); the buffers of a call must not be
 * reused before it completes. zx_gemm_s8_host: int8 -> int32; zx_gemm_bf16_host: bf16 -> fp32. */
ZX_API int zx_gemm_s8_host(const void* A_host, const void* B_host, void* C_host, zx_devptr A_dev, zx_devptr B_dev,
                           zx_devptr C_dev, uint32_t M, uint32_t N, uint32_t K, zx_stream stream);
ZX_API int zx_gemm_bf16_host(const void* A_host, const void* B_host, void* C_host, zx_devptr A_dev,
                             zx_devptr B_dev, zx_devptr C_dev, uint32_t M, uint32_t N, uint32_t K,
                             zx_stream stream);

/* int8 GEMM over several GPUs of this process, M split in contiguous row blocks (no collective):
 * shard i is rows [i*M/ngpus, (i+1)*M/ngpus) of A and C and runs on device devices[i]. A[i] and
 * C[i] are that device's rows of A (row-major, K contiguous) and of C (row pitch N), B[i] a full
 * copy of B on that device (layout as zx_gemm_s8), streams[i] a stream of that device (streams
 * may be null: each device's legacy default stream). Every shard is validated before any is
 * launched; the call enqueues one GEMM per shard and returns (the caller synchronizes the
 * streams), restoring the caller's current device. A device may appear more than once.
 * For a single host process driving the GPUs of a node over the C ABI (e.g. a Zig or C caller
 * without torch.distributed); one process per GPU uses zx_gemm_s8 on its own shard instead.
 * No reference counterpart (the reference is single-device, src/cuda_driver.zig:284-288). */
ZX_API int zx_gemm_s8_mgpu(int ngpus, const int* devices, const zx_devptr* A, const zx_devptr* B, const zx_devptr* C,
                           uint32_t M, uint32_t N, uint32_t K, int layout, const zx_stream* streams);

/* zx_gemm_s8 (NT) that also writes C into up to 7 other buffers, typically the same rows of C on
 * the other GPUs of the node (their memory mapped into this process, e.g. through CUDA IPC
 * handles, with peer access): the GEMM and the all-gather of C in one kernel. Every tile of C is
 * stored to C, then copied by two extra warps per CTA from C to each peer_c[i] (same row pitch
 * N * 4 bytes) with 16-byte stores, so the NVLink traffic overlaps the tensor-core work.
 * Stores only: nothing waits on another GPU. The peer writes are complete when the kernel has
 * completed; a reader on another GPU must order its reads after that (e.g. a stream
 * synchronisation and a host barrier, or an event). Runs on the 256 x 512 pair kernel.
 * peer_c: host array of npeers (<= 7) device addresses, each 16-byte aligned.
 * No reference counterpart (the reference is single-device, src/cuda_driver.zig:284-288). */
ZX_API int zx_gemm_s8_replicated(zx_devptr A, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                                 const zx_devptr* peer_c, uint32_t npeers, zx_stream stream);

/* CUDA IPC for the peer buffers of zx_gemm_s8_replicated, one process per GPU.
 * zx_ipc_export: a 64-byte handle for the allocation holding `ptr`, and ptr's offset in it; send
 * both to the other processes. zx_ipc_import (in another process, its own device current): maps
 * that allocation, peer access enabled, and returns its base here; base + offset is the peer's
 * ptr. zx_ipc_close unmaps it (after the last kernel that writes to it has completed). */
ZX_API int zx_ipc_export(zx_devptr ptr, unsigned char handle_out[64], uint64_t* offset_out);
ZX_API int zx_ipc_import(const unsigned char handle[64], zx_devptr* base_out);
ZX_API int zx_ipc_close(zx_devptr base);

/* int8 GEMM with the fp32-scaled bf16 epilogue of BASELINE config 2 (no reference kernel; the
 * reference GEMMs store raw accumulators, src/examples/imma_s8.zig:161-172):
 *   C[m,n] = bf16_rne( ((float)acc[m,n] * row_scale[m]) * col_scale[n] )
 * float conversion and both multiplies round-to-nearest-even, in this order, no FMA.
 * C is bf16 (uint16 storage) row-major M x N. Requirements as zx_gemm_s8 plus N % 8 == 0. */
ZX_API int zx_gemm_s8_scaled_bf16(zx_devptr A, zx_devptr B, zx_devptr row_scale, zx_devptr col_scale,
                           zx_devptr C, uint32_t M, uint32_t N, uint32_t K, int layout,
                           zx_stream stream);

/* bf16 x bf16 -> fp32 GEMM (tcgen05 kind::f16, TMA-fed). A, B are bf16 bit patterns (uint16).
 * Replaces: examples_abi.hgemm_bf16 (src/examples_abi.zig:33-36) as launched for
 * hgemm_wgmma_bf16 (src/bench.zig:549-631; src/examples/hgemm_wgmma_bf16.zig:105-169) and the
 * TMA-fed hgemm_tma flow (src/bench.zig:1438-1553).
 * Requirements: K % 8 == 0, N % 4 == 0 (NN: N % 8 == 0), buffers 16-B aligned. */
ZX_API int zx_gemm_bf16(zx_devptr A, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                 int layout, zx_stream stream);
/* f16 x f16 -> fp32 GEMM on the same kernels (the instruction descriptor's A/B format f16).
 * Replaces: the hgemm_tma kernel's f16 operands (src/examples_abi.zig:168-190,
 * src/examples/hgemm_tma.zig:109-192, launched by runHgemmTma, src/bench.zig:1438-1553).
 * Requirements as zx_gemm_bf16. */
ZX_API int zx_gemm_f16(zx_devptr A, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                int layout, zx_stream stream);

/* W4A8 GEMM: C[M x N] int32 = A[M x K] int8 * W^T, W = N x K signed int4
 * packed two per byte along K (row pitch K/2 bytes), low nibble = even k: the reference's
 * packS4 convention (src/examples_abi.zig:54-56, read back by s4At, src/bench.zig:753-759)
 * applied along K. Replaces: examples_abi.imma_s4 (src/examples_abi.zig:44-56) launched by
 * runImmaS4 (src/bench.zig:767-869) as imma_s4_$_immaS4 (src/examples/imma_s4.zig:130-173);
 * the weights are unpacked to int8 in shared memory and multiplied on tcgen05 kind::i8.
 * Requirements: K % 32 == 0, N % 4 == 0, buffers 16-byte aligned. Exact int32 accumulation. */
ZX_API int zx_gemm_w4a8(zx_devptr A, zx_devptr W, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                        zx_stream stream);

/* zx_gemm_w4a8 with a caller-owned workspace, for the decode-like shapes (M <= 32, K % 256 == 0)
 * that split the weight stream across all SMs: the CTAs that share a 128-column tile of C leave
 * their partial sums in the workspace and the last of them adds them up and stores the tile, so
 * C is written once with plain stores and no zeroing pass over C runs first (zx_gemm_w4a8
 * zeroes C and adds into it with atomics). Same result, bit for bit.
 * The workspace must be zero-filled before its first use (e.g. one cudaMemset after allocation);
 * every call leaves it zero again. Calls that overlap on the GPU must not share a workspace.
 * After a call that ends with ZX_ERR_TIMEOUT (zx_device_status), zero it again.
 * Size: zx_gemm_w4a8_workspace_bytes (0 for shapes that use none: M > 32 or K % 256 != 0, which
 * run exactly as zx_gemm_w4a8 and ignore the workspace). Requirements as zx_gemm_w4a8 plus a
 * 16-byte aligned workspace.
 * No reference counterpart (the reference's int4 kernel has one tile per CTA, no split-K). */
ZX_API int zx_gemm_w4a8_ws(zx_devptr A, zx_devptr W, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                           zx_devptr workspace, uint64_t workspace_bytes, zx_stream stream);

/* Workspace bytes zx_gemm_w4a8_ws needs for this shape on the current device (written to *bytes;
 * 0 when the shape does not use one). */
ZX_API int zx_gemm_w4a8_workspace_bytes(uint32_t M, uint32_t N, uint32_t K, uint64_t* bytes);

/* zx_gemm_w4a8_ws for callers that cannot allocate device memory: it takes no workspace and
 * calls no allocating routine (no cudaMalloc / cudaFree, no allocating library routine; the
 * first call in a context is the exception described below).
 * For a host that owns every byte of device memory through its own allocator or budget (a
 * framework's caching allocator, an embedding runtime calling this library over its C ABI) and
 * for decode loops where an allocation could synchronize the device, but that still want the
 * split-K decode kernel. The caller passes A, W and C as for zx_gemm_w4a8; the scratch lives in
 * one array of 5 MiB + 2 KiB built into the library, which every GPU that loads the library holds
 * until the process exits.
 * Limits (anything beyond returns ZX_ERR_SHAPE with a message): M <= 32, N <= 65536,
 * K % 256 == 0, and at most 160 SMs on the device; other requirements as zx_gemm_w4a8.
 * The first call in a CUDA context (per device, per context) may load this library's module into
 * that context, which is when the array is placed, and looks up the array's address there: make
 * that first call once, outside any decode loop and before any stream capture; later calls in the
 * same context allocate nothing. Every call on a device shares the one array, and it keeps the last call's
 * contents: each call clears the counters it needs before the kernel runs, and calls that overlap
 * on the GPU (other streams, other host threads) race on the array and must not be issued.
 * Results are identical to zx_gemm_w4a8's. No counterpart in the reference. */
ZX_API int zx_gemm_w4a8_noalloc(zx_devptr A, zx_devptr W, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                                zx_stream stream);

/* 2:4 structured-sparse int8 GEMM: C[M x N] int32 = A * B^T with A given
 * compressed. A_c is M x K/2 int8 (the two kept values of every group of 4 dense k, in k order);
 * meta is M x K/32 uint32 in the reference's format (src/examples_abi.zig:71-81): in the word for
 * dense k 32w..32w+31, nibble j describes the group at 4j..4j+3, low 2 bits = index of the first
 * kept element, high 2 bits = the second (idx0 < idx1). B is N x K int8 (K contiguous).
 * Replaces: examples_abi.imma_sp_s8 (src/examples_abi.zig:71-81) launched by runImmaSpS8
 * (src/bench.zig:1014-1150) as imma_sp_s8_$_immaSpS8 (src/examples/imma_sp_s8.zig:144-187); runs
 * on tcgen05.mma.sp kind::i8 with the metadata copied to tensor memory unchanged.
 * Requirements: M % 128 == 0, K % 256 == 0, N % 4 == 0, buffers 16-byte aligned. Exact int32
 * accumulation. */
ZX_API int zx_gemm_sp_s8(zx_devptr A_c, zx_devptr meta, zx_devptr B, zx_devptr C, uint32_t M,
                         uint32_t N, uint32_t K, zx_stream stream);

/* The reference's own operand layouts on the fast kernels, through one layout pass into a caller
 * workspace (no reference counterpart for the pass; the reference kernels read these layouts
 * directly at a legacy rate).
 * zx_gemm_sp_s8_nn: zx_gemm_sp_s8 with B row-major K x N (imma_sp_s8's layout,
 *   src/examples/imma_sp_s8.zig:144-187; examples_abi.zig:71-81): B is transposed into the
 *   workspace (N x K), then the 2:4 sparse kernel runs. Requirements as zx_gemm_sp_s8 plus
 *   N % 16 == 0; workspace >= N * K bytes.
 * zx_gemm_s4s4_nn: imma_s4's operands (src/examples/imma_s4.zig:89-101, examples_abi.zig:44-56):
 *   A M x K signed int4 packed two per byte along K (low nibble = even k), B K x N signed int4
 *   packed along N (low nibble = even n), C M x N int32 exact. A is unpacked to int8 and B
 *   repacked along K in the workspace, then the W4A8 kernels run. K % 64 == 0, N % 16 == 0;
 *   workspace >= round_up(M * K, 256) + N * K / 2 bytes.
 * zx_gemm_sp_s4_nn: imma_sp_s4's operands (src/examples/imma_sp_s4.zig:153-196,
 *   examples_abi.zig:83-96): A M x K/4 bytes of 4:8 pair-clustered s4 (per 8-wide k chunk the two
 *   kept 2-wide sub-chunks, one packS4 byte each), meta M x K/64 words (nibble j = p0 | p1 << 2),
 *   B K x N signed int4 packed along N, C M x N int32 exact. In the workspace A becomes int8 2:4
 *   operands and B int8 N x K, both with k reordered inside every 8-wide chunk (element e of
 *   sub-chunk p at position 4e + p; a GEMM's sum over k is unchanged), then the 2:4 sparse kernels
 *   run. M % 128 == 0, K % 256 == 0, N % 16 == 0; workspace >= round_up(M * K / 2, 256) +
 *   round_up(M * K / 8, 256) + N * K bytes.
 * zx_gemm_nn_workspace_bytes: the workspace size of any of them (op = ZX_NN_SP_S8 / ZX_NN_S4S4 /
 *   ZX_NN_SP_S4).
 * The workspace is scratch: its contents are overwritten, and it must not be reused before the
 * call's work on `stream` completes. */
ZX_API int zx_gemm_nn_workspace_bytes(int op, uint32_t M, uint32_t N, uint32_t K, uint64_t* bytes);
ZX_API int zx_gemm_sp_s8_nn(zx_devptr A_c, zx_devptr meta, zx_devptr B_kn, zx_devptr C, uint32_t M, uint32_t N,
                            uint32_t K, zx_devptr workspace, uint64_t workspace_bytes, zx_stream stream);
ZX_API int zx_gemm_s4s4_nn(zx_devptr A, zx_devptr B_kn, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                           zx_devptr workspace, uint64_t workspace_bytes, zx_stream stream);
ZX_API int zx_gemm_sp_s4_nn(zx_devptr A_c, zx_devptr meta, zx_devptr B_kn, zx_devptr C, uint32_t M, uint32_t N,
                            uint32_t K, zx_devptr workspace, uint64_t workspace_bytes, zx_stream stream);

/* ---------------------------------------------------------------------------------------
 * Reference-signature entry points: same argument list and meaning as the reference kernel
 * ABI (square n, B row-major K x N, C row-major), so a caller of examples_abi can switch by
 * replacing the launch with this call. n % 128 == 0 as the reference's shape gate
 * (src/bench.zig:96-124).
 * ------------------------------------------------------------------------------------- */
/* src/examples_abi.zig:42  imma_s8(a: [*]const i8, b: [*]const i8, c: [*]i32, n: u32) */
ZX_API int zx_imma_s8(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, zx_stream stream);
/* src/examples_abi.zig:33-36  hgemm_bf16.signature (a: [*]const u16, b: [*]const u16, c: [*]f32, n) */
ZX_API int zx_hgemm_bf16(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, zx_stream stream);
/* src/examples_abi.zig:168-190  hgemm_tma.signature (a: [*]const f16, b: [*]const f16, c: [*]f32,
 * n, desc_a: u64, desc_b: u64): the descriptors (the caller's tensor maps of A and B) are accepted
 * and not read; the tiles are read through a and b, which the reference binds to the same
 * buffers (src/bench.zig:1475-1512). */
ZX_API int zx_hgemm_tma(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, uint64_t desc_a, uint64_t desc_b,
                        zx_stream stream);

/* The reference's kernels themselves, under the reference's launch contract: these launch the
 * entry points imma_s8_$_immaS8 / hgemm_wgmma_bf16_$_hgemmWgmmaBf16 (same names, parameter
 * lists and grid/block shapes as src/bench.zig:671-682 and :589-600: block 128, grid
 * (n/128, n/128) resp. (n/128, n/64), no dynamic shared memory, no cluster). The same kernels
 * are shipped as zoxide_b200/_build/imma_s8.cubin and hgemm_wgmma_bf16.cubin for the
 * reference's own cubin loader (`zoxide bench <file>.cubin`). Slower than zx_imma_s8 /
 * zx_hgemm_bf16, which keep the reference's argument list but choose their own launch. */
ZX_API int zx_launch_imma_s8_ref(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, zx_stream stream);
ZX_API int zx_launch_hgemm_bf16_ref(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n,
                                    zx_stream stream);

/* The remaining reference kernels under the same contract (block 128, no dynamic shared memory,
 * no cluster), each also shipped as zoxide_b200/_build/<stem>.cubin:
 *   imma_s4_$_immaS4 (src/examples_abi.zig:44-56): A n x n s4 packed along K, B (K x N) s4
 *     packed along N, two per byte, low nibble = even index; grid (n/128, n/128)
 *     (src/bench.zig:800-811).
 *   imma_sp_s8_$_immaSpS8 (src/examples_abi.zig:71-81): A 2:4-compressed n x n/2, meta
 *     n x n/32 words, B dense K x N int8; grid (n/128, n/128) (src/bench.zig:1081-1092).
 *   imma_sp_s4_$_immaSpS4 (src/examples_abi.zig:83-96): A 4:8 pair-clustered n x n/4 bytes,
 *     meta n x n/64 words, B dense K x N s4 packed along N; grid (n/128, n/128)
 *     (src/bench.zig:1240-1251). Runs on the int8 2:4 sparse MMA after a k reorder inside each
 *     8-wide chunk (element e of sub-chunk p at position 4e + p), applied to A and B alike.
 *   hgemm_bf16_$_hgemmBf16 (src/examples_abi.zig:33-36): the hgemm_bf16 stem's 128 x 128 tile,
 *     grid (n/128, n/128) (src/bench.zig:77-78).
 *   hgemm_tma_$_hgemmTma (src/examples_abi.zig:168-190): f16 A, B n x n row-major, f32 C,
 *     grid (n/128, n/64) (src/bench.zig:1511-1522); desc_a / desc_b (device addresses of the
 *     caller's tensor maps of A and B) are accepted and not read.
 * All require n % 128 == 0 (the reference's gate for these stems; its guarded hgemm_bf16 kernel
 * also takes n % 16 == 0, this one does not). Exact int32 for the integer kernels. */
ZX_API int zx_launch_imma_s4_ref(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, zx_stream stream);
ZX_API int zx_launch_imma_sp_s8_ref(zx_devptr a, zx_devptr b, zx_devptr meta, zx_devptr c, uint32_t n,
                                    zx_stream stream);
ZX_API int zx_launch_imma_sp_s4_ref(zx_devptr a, zx_devptr b, zx_devptr meta, zx_devptr c, uint32_t n,
                                    zx_stream stream);
ZX_API int zx_launch_hgemm_bf16_mma_ref(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n,
                                        zx_stream stream);
ZX_API int zx_launch_hgemm_tma_ref(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, uint64_t desc_a,
                                   uint64_t desc_b, zx_stream stream);

/* ---------------------------------------------------------------------------------------
 * Device status. Kernels never trap; a bounded mbarrier wait that expires writes a non-zero
 * code (0x100 | site) into a per-device status word and the kernel exits early. Reading the
 * word synchronises the current device. Returns ZX_ERR_TIMEOUT if the word is non-zero.
 * ------------------------------------------------------------------------------------- */
ZX_API int zx_device_status(uint32_t* code_out);
ZX_API int zx_device_status_clear(void);

/* Self-test of that failure path, without any GPU fault: a one-CTA kernel waits, with the same
 * bounded-wait code the GEMM kernels use and a limit of `limit_us` microseconds (1 .. 10^6), on an
 * mbarrier that nothing arrives on; the wait gives up and records status code 0x1F1, a second
 * warp leaves its own never-completed wait through the kernel's abort flag, and a wait on a
 * barrier the kernel completes itself succeeds. Writes the three outcomes (1 = wait succeeded) to
 * out[0..2] (int32, device memory) on `stream`. The device status word is left set; clear it with
 * zx_device_status_clear. No reference counterpart (cf. the reference's bounded tryWaitFor,
 * src/tma.zig:142-153). */
ZX_API int zx_selftest_bounded_wait(zx_devptr out, uint32_t limit_us, zx_stream stream);

/* Number of streaming multiprocessors on the current device (0 on error). */
ZX_API int zx_device_sm_count(void);

#ifdef __cplusplus
}
#endif

#endif /* ZOXIDE_GEMM_H */
