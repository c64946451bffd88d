// zx_api.cu — C-ABI entry points of libzoxide_b200 (declared in include/zoxide_gemm.h).
//
// Host side of the drop-in boundary. It plays the role of the reference's typed host API and
// driver layer for this path (src/host.zig:359-567 Kernel.launchOn / checkGeometry,
// src/cuda_driver.zig:396-486 encodeTensorMap, :820-845 cuLaunchKernel): validate arguments,
// build TMA descriptors, pick the persistent grid, launch. Arguments are checked before any
// CUDA call, so the validation paths run (and are tested) on machines without a GPU.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/zoxide_gemm.h"
#include "zx_gemm_tc.cuh"
#include "zx_gemm_tc2.cuh"
#include "zx_gemm_tc2w.cuh"
#include "zx_gemm_sp2.cuh"
#include "zx_gemm_sp2w.cuh"
#include "zx_gemm_sp4.cuh"
#include "zx_layout.cuh"
#include "zx_compat.cuh"
#include "zx_gemm_w4s.cuh"
#include "zx_gemm_w4t.cuh"
#include <atomic>
#include <initializer_list>

namespace {

thread_local char t_err[512] = "";
thread_local char t_kernel[160] = "";  // kernel launched by this thread's last successful call
// Set by the f16 entry points for the duration of one call: the 16-bit float kernels then read
// f16 operands (TMA maps typed FLOAT16, instruction descriptor A/B formats f16 instead of bf16).
thread_local bool t_f16 = false;
constexpr uint32_t kF16Xor = (1u << 7) | (1u << 10);  // A and B format fields: bf16 (1) -> f16 (0)
struct F16Call {
  F16Call() { t_f16 = true; }
  ~F16Call() { t_f16 = false; }
};

void note_kernel(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_kernel, sizeof(t_kernel), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  t_kernel[0] = 0;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(static_cast<int>(e), "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// ----------------------------------- per-device cache -----------------------------------
constexpr int kMaxDevices = 64;
struct DeviceInfo {
  bool ready = false;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
};
std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::atomic<int> g_policy{0};  // 0 auto, 1 one-SM, 2 two-SM, 3 two-SM 256-wide, 4/5/6 two-SM 512/480/464-wide

int current_device(int* dev, DeviceInfo** info) {
  int d = 0;
  cudaError_t e = cudaGetDevice(&d);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (d < 0 || d >= kMaxDevices) return fail(ZX_ERR_NO_DEVICE, "device ordinal %d out of range", d);
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& di = g_dev[d];
  if (!di.ready) {
    if ((e = cudaDeviceGetAttribute(&di.sm_count, cudaDevAttrMultiProcessorCount, d)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    if ((e = cudaDeviceGetAttribute(&di.cc_major, cudaDevAttrComputeCapabilityMajor, d)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute(cc major)");
    if ((e = cudaDeviceGetAttribute(&di.cc_minor, cudaDevAttrComputeCapabilityMinor, d)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute(cc minor)");
    di.ready = true;
  }
  if (di.cc_major != 10 || di.cc_minor != 0)
    return fail(ZX_ERR_ARCH, "device %d is sm_%d%d; this library is built for sm_100a (B200) only",
                d, di.cc_major, di.cc_minor);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return fail(ZX_ERR_DRIVER, "driver entry point cuTensorMapEncodeTiled unavailable");
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  *dev = d;
  *info = &di;
  return 0;
}

// Base and size of the allocation that holds device address `ptr` (driver cuMemGetAddressRange,
// fetched once through the runtime's entry-point query; works for IPC-imported mappings too).
using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
int address_range(uint64_t ptr, uint64_t* base, uint64_t* size, const char* fn) {
  static AddressRangeFn range = nullptr;
  if (!range) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !f)
      return fail(ZX_ERR_DRIVER, "%s: driver entry point cuMemGetAddressRange unavailable", fn);
    range = reinterpret_cast<AddressRangeFn>(f);
  }
  CUdeviceptr b = 0;
  size_t n = 0;
  CUresult r = range(&b, &n, static_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS)
    return fail(ZX_ERR_NULL, "%s: %#llx is not device memory mapped in this process (CUresult %d)", fn,
                (unsigned long long)ptr, static_cast<int>(r));
  *base = b;
  *size = n;
  return 0;
}

// Device memory at `ptr` that kernels on the current device can store to: memory of this device,
// or of a device it can reach peer to peer (the IPC mapping enables the access itself).
int check_reachable(uint64_t ptr, const char* fn) {
  int cur = 0;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  cudaPointerAttributes at{};
  e = cudaPointerGetAttributes(&at, reinterpret_cast<const void*>(ptr));
  if (e != cudaSuccess) return cuda_fail(e, "cudaPointerGetAttributes");
  if (at.type != cudaMemoryTypeDevice)
    return fail(ZX_ERR_NULL, "%s: %#llx is not device memory", fn, (unsigned long long)ptr);
  if (at.device != cur) {
    int ok = 0;
    e = cudaDeviceCanAccessPeer(&ok, cur, at.device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceCanAccessPeer");
    if (!ok)
      return fail(ZX_ERR_DRIVER, "%s: device %d cannot reach device %d peer to peer", fn, cur, at.device);
  }
  return 0;
}

// 2-D tensor map: dims {inner, outer} elements, row pitch in bytes, box {bx, by}, 128B swizzle.
int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
              uint64_t outer, uint64_t pitch_bytes, uint32_t bx, uint32_t by,
              CUtensorMapL2promotion l2, const char* what,
              CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {pitch_bytes};
  const cuuint32_t box[2] = {bx, by};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, l2,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(ZX_ERR_DRIVER,
                "cuTensorMapEncodeTiled(%s) failed with CUresult %d (dims %llu x %llu, pitch %llu, box %u x %u)",
                what, static_cast<int>(r), (unsigned long long)inner, (unsigned long long)outer,
                (unsigned long long)pitch_bytes, bx, by);
  return 0;
}

// 2-CTA clusters of `kern` that can be resident at once on device `dev`, cached per kernel (the
// caller's `cache`) and device: sets the dynamic shared memory limit and asks the occupancy API
// for a 2 x 1 x 1 cluster launch of `threads` threads and `smem` bytes.
template <class Kern>
int pair_capacity(Kern kern, int threads, int smem, int dev, const DeviceInfo* di, int (&cache)[kMaxDevices],
                  const char* fn) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (cache[dev] != 0) return 0;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * (di->sm_count / 2), 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
  if (n <= 0) return fail(ZX_ERR_ARCH, "%s: no 2-CTA cluster fits on device %d", fn, dev);
  cache[dev] = n;
  return 0;
}

// --------------------------------------- validation ---------------------------------------
bool aligned16(zx_devptr p) { return (p & 15u) == 0; }

int check_common(zx_devptr A, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                 int layout, uint32_t k_mult, uint32_t n_mult_c, uint32_t n_mult_b_nn,
                 const char* fn) {
  if (!A || !B || !C) return fail(ZX_ERR_NULL, "%s: null buffer (A=%#llx B=%#llx C=%#llx)", fn,
                                  (unsigned long long)A, (unsigned long long)B, (unsigned long long)C);
  if (layout != ZX_LAYOUT_NT && layout != ZX_LAYOUT_NN)
    return fail(ZX_ERR_LAYOUT, "%s: unknown layout %d (0 = NT, 1 = NN)", fn, layout);
  if (M == 0 || N == 0 || K == 0)
    return fail(ZX_ERR_SHAPE, "%s: empty problem M=%u N=%u K=%u", fn, M, N, K);
  if (M > (1u << 31) || N > (1u << 31) || K > (1u << 31))
    return fail(ZX_ERR_SHAPE, "%s: dimension above 2^31 (M=%u N=%u K=%u)", fn, M, N, K);
  if (K % k_mult != 0)
    return fail(ZX_ERR_SHAPE, "%s: K=%u must be a multiple of %u (16-byte TMA row pitch)", fn, K, k_mult);
  if (N % n_mult_c != 0)
    return fail(ZX_ERR_SHAPE, "%s: N=%u must be a multiple of %u (16-byte C row pitch)", fn, N, n_mult_c);
  if (layout == ZX_LAYOUT_NN && N % n_mult_b_nn != 0)
    return fail(ZX_ERR_SHAPE, "%s: NN layout needs N=%u to be a multiple of %u (16-byte B row pitch)",
                fn, N, n_mult_b_nn);
  if (!aligned16(A) || !aligned16(B) || !aligned16(C))
    return fail(ZX_ERR_ALIGN, "%s: buffers must be 16-byte aligned (A=%#llx B=%#llx C=%#llx)", fn,
                (unsigned long long)A, (unsigned long long)B, (unsigned long long)C);
  return 0;
}

// ------------------------------------------ launch ------------------------------------------
template <zx::Kind kKind, bool kMN, zx::Out kOut, int kBN, int kStages>
int launch_gemm(zx_devptr A, zx_devptr B, zx_devptr C, const float* rs, const float* cs,
                uint32_t M, uint32_t N, uint32_t K, cudaStream_t stream, const char* fn, uint32_t ldc = 0) {
  using Cfg = zx::GemmCfg<kKind, kMN, kOut, kBN, kStages>;
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;

  zx::GemmParams p;
  memset(&p, 0, sizeof(p));
  const CUtensorMapDataType in_t = kKind != zx::Kind::BF16 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : t_f16                  ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  p.idesc_xor = (kKind == zx::Kind::BF16 && t_f16) ? kF16Xor : 0u;
  const CUtensorMapDataType out_t = kOut == zx::Out::S32     ? CU_TENSOR_MAP_DATA_TYPE_INT32
                                    : kOut == zx::Out::F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                             : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t esz = Cfg::ESZ;
  int rc = encode_2d(&p.tmA, in_t, reinterpret_cast<void*>(A), K, M, K * esz, Cfg::BK, Cfg::BM,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "A");
  if (rc) return rc;
  if constexpr (!kMN)
    rc = encode_2d(&p.tmB, in_t, reinterpret_cast<void*>(B), K, N, K * esz, Cfg::BK, Cfg::BN,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "B (N x K)");
  else
    rc = encode_2d(&p.tmB, in_t, reinterpret_cast<void*>(B), N, K, N * esz, 128 / Cfg::ESZ, Cfg::BK,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "B (K x N)");
  if (rc) return rc;
  rc = encode_2d(&p.tmC, out_t, reinterpret_cast<void*>(C), N, M, uint64_t(ldc ? ldc : N) * Cfg::OUT_ESZ,
                 Cfg::CHUNK_COLS, 32, CU_TENSOR_MAP_L2_PROMOTION_NONE, "C");
  if (rc) return rc;
  p.row_scale = rs;
  p.col_scale = cs;
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_m_blk = (M + Cfg::BM - 1) / Cfg::BM;
  p.num_n_blk = (N + Cfg::BN - 1) / Cfg::BN;
  p.num_k_blk = (K + Cfg::BK - 1) / Cfg::BK;
  p.group_m = 16;

  auto kern = zx::gemm_tc_kernel<kKind, kMN, kOut, kBN, kStages>;
  static bool attr_done[kMaxDevices] = {};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           Cfg::SMEM_BYTES);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
      attr_done[dev] = true;
    }
  }
  const uint32_t tiles = p.num_m_blk * p.num_n_blk;
  const uint32_t grid = tiles < static_cast<uint32_t>(di->sm_count) ? tiles : di->sm_count;
  kern<<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(p);
  note_kernel("gemm_tc_kernel 1-SM %dx%d tiles, grid %u", Cfg::BM, Cfg::BN, grid);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return 0;
}


template <zx::Kind kKind, bool kMN, zx::Out kOut, int kStages, int kBN = 256>
int launch_gemm2(zx_devptr A, zx_devptr B, zx_devptr C, const float* rs, const float* cs,
                 uint32_t M, uint32_t N, uint32_t K, cudaStream_t stream, const char* fn, uint32_t ldc = 0) {
  using Cfg = zx::Gemm2Cfg<kKind, kMN, kOut, kStages, kBN>;
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;

  zx::GemmParams p;
  memset(&p, 0, sizeof(p));
  const CUtensorMapDataType in_t = kKind != zx::Kind::BF16 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : t_f16                  ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  p.idesc_xor = (kKind == zx::Kind::BF16 && t_f16) ? kF16Xor : 0u;
  const CUtensorMapDataType out_t = kOut == zx::Out::S32     ? CU_TENSOR_MAP_DATA_TYPE_INT32
                                    : kOut == zx::Out::F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                             : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t esz = Cfg::ESZ;
  int rc = encode_2d(&p.tmA, in_t, reinterpret_cast<void*>(A), K, M, K * esz, Cfg::ROWB / Cfg::ESZ,
                     Cfg::BM_CTA, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "A");
  if (rc) return rc;
  if constexpr (kKind == zx::Kind::W4)
    rc = encode_2d(&p.tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, reinterpret_cast<void*>(B), K / 2, N, K / 2,
                   Cfg::BK / 2, Cfg::BN_CTA, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "W (N x K/2 packed s4)",
                   CU_TENSOR_MAP_SWIZZLE_NONE);
  else if constexpr (!kMN)
    rc = encode_2d(&p.tmB, in_t, reinterpret_cast<void*>(B), K, N, K * esz, Cfg::ROWB / Cfg::ESZ,
                   Cfg::BN_CTA, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "B (N x K)");
  else
    rc = encode_2d(&p.tmB, in_t, reinterpret_cast<void*>(B), N, K, N * esz, 128 / Cfg::ESZ, Cfg::BK,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "B (K x N)");
  if (rc) return rc;
  rc = encode_2d(&p.tmC, out_t, reinterpret_cast<void*>(C), N, M, uint64_t(ldc ? ldc : N) * Cfg::OUT_ESZ,
                 Cfg::CHUNK_COLS, 32, CU_TENSOR_MAP_L2_PROMOTION_NONE, "C");
  if (rc) return rc;
  p.row_scale = rs;
  p.col_scale = cs;
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_m_blk = (M + Cfg::BM - 1) / Cfg::BM;
  p.num_n_blk = (N + Cfg::BN - 1) / Cfg::BN;
  p.num_k_blk = (K + Cfg::BK - 1) / Cfg::BK;
#ifndef ZX_GROUP_M2
#define ZX_GROUP_M2 16
#endif
  p.group_m = ZX_GROUP_M2;

  auto kern = zx::gemm_tc2_kernel<kKind, kMN, kOut, kStages, kBN>;
  static int max_clusters[kMaxDevices] = {};
  if (int rc = pair_capacity(kern, Cfg::THREADS, Cfg::SMEM_BYTES, dev, di, max_clusters, fn)) return rc;
  const uint32_t tiles = p.num_m_blk * p.num_n_blk;
  const uint32_t pairs = tiles < static_cast<uint32_t>(max_clusters[dev]) ? tiles : max_clusters[dev];
  kern<<<2 * pairs, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(p);
  note_kernel("gemm_tc2_kernel 2-SM %dx%d tiles, %u CTA pairs", Cfg::BM, Cfg::BN, pairs);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return 0;
}

// 256 x 512 pair tiles (zx_gemm_tc2w.cuh): K-major A and B.
template <zx::Kind kKind, zx::Out kOut, int kHi = 256>
int launch_gemm2w(zx_devptr A, zx_devptr B, zx_devptr C, const float* rs, const float* cs,
                  uint32_t M, uint32_t N, uint32_t K, cudaStream_t stream, const char* fn,
                  const zx_devptr* peers = nullptr, uint32_t npeers = 0, uint32_t ldc = 0) {
  using Cfg = zx::Gemm2wCfg<kKind, kOut, 4, kHi>;
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  zx::GemmParams p;
  memset(&p, 0, sizeof(p));
  const CUtensorMapDataType in_t = kKind != zx::Kind::BF16 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : t_f16                  ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  p.idesc_xor = (kKind == zx::Kind::BF16 && t_f16) ? kF16Xor : 0u;
  const uint64_t esz = Cfg::ESZ;
  int rc = encode_2d(&p.tmA, in_t, reinterpret_cast<void*>(A), K, M, K * esz, Cfg::ROWB / Cfg::ESZ,
                     Cfg::BM_CTA, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "A");
  if (rc) return rc;
  rc = encode_2d(&p.tmB, in_t, reinterpret_cast<void*>(B), K, N, K * esz, Cfg::ROWB / Cfg::ESZ, 128,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "B (N x K)");
  if (rc) return rc;
  if (kHi != 256) {
    rc = encode_2d(&p.tmB2, in_t, reinterpret_cast<void*>(B), K, N, K * esz, Cfg::ROWB / Cfg::ESZ, Cfg::BNH_HI / 2,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "B (N x K, hi-half box)");
    if (rc) return rc;
  }
  const CUtensorMapDataType out_t = kOut == zx::Out::S32     ? CU_TENSOR_MAP_DATA_TYPE_INT32
                                    : kOut == zx::Out::F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                             : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  rc = encode_2d(&p.tmC, out_t, reinterpret_cast<void*>(C), N, M, uint64_t(ldc ? ldc : N) * Cfg::OUT_ESZ,
                 Cfg::CHUNK_COLS, 32, CU_TENSOR_MAP_L2_PROMOTION_NONE, "C");
  if (rc) return rc;
  p.row_scale = rs;
  p.col_scale = cs;
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_m_blk = (M + Cfg::BM - 1) / Cfg::BM;
  p.num_n_blk = (N + Cfg::BN - 1) / Cfg::BN;
  p.num_k_blk = (K + Cfg::BK - 1) / Cfg::BK;
  p.group_m = ZX_GROUP_M2;
  for (uint32_t i = 0; i < npeers; ++i) p.peer_c[i] = peers[i];
  p.npeers = npeers;
  p.ldc = ldc ? ldc : N;
  p.c_base = reinterpret_cast<const uint32_t*>(C);
  auto kern = zx::gemm_tc2w_kernel<kKind, kOut, 4, kHi>;
  static int max_clusters[kMaxDevices] = {};
  if (int rc = pair_capacity(kern, Cfg::THREADS, Cfg::SMEM_BYTES, dev, di, max_clusters, fn)) return rc;
  const uint32_t tiles = p.num_m_blk * p.num_n_blk;
  const uint32_t pairs = tiles < static_cast<uint32_t>(max_clusters[dev]) ? tiles : max_clusters[dev];
  kern<<<2 * pairs, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(p);
  note_kernel("gemm_tc2w_kernel 2-SM %dx%d tiles, %u CTA pairs", Cfg::BM, Cfg::BN, pairs);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return 0;
}

constexpr int kPairStages = 6 / ZX_PAIR_KATOMS;

// N width of the pair tile: 256, or 224 when that needs fewer full-machine waves of tile work
// (time ~ waves x tile width). 74 pairs run at once on a 148-SM B200. Example: M = 1024,
// N = 8192 (one eighth of 8192^3) gives 128 tiles of 256 (2 waves, the second 73 % full) but
// 148 tiles of 224 (2 full waves).
int pair_tile_n(uint32_t M, uint32_t N) {
  const uint64_t pairs = 74, mt = (M + 255) / 256;
  auto cost = [&](uint64_t bn) { return ((mt * ((N + bn - 1) / bn) + pairs - 1) / pairs) * bn; };
  return cost(224) < cost(256) ? 224 : 256;
}

// N width of the one-SM tile (K-major B): 256, 128 or 64. A one-SM tile's loop is bound by the
// operand bytes it takes in, (128 + BN) per byte of K, so the cost of a width is full-machine waves
// x (128 + BN); narrower tiles win when they put idle SMs to work (1024^3: 32 tiles of 256 on 148
// SMs against 128 tiles of 64, 384 against 192).
uint32_t small_tile_n(uint32_t M, uint32_t N, uint32_t sms) {
  const uint64_t mt = (M + 127) / 128;
  uint32_t best = 256;
  uint64_t best_cost = ~0ull;
  for (uint32_t bn : {256u, 128u, 64u}) {
    const uint64_t waves = (mt * ((N + bn - 1) / bn) + sms - 1) / sms;
    const uint64_t cost = waves * (128 + bn);
    if (cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

// Tile path for the automatic policy, from the number of full-machine waves each tile shape
// needs (time ~ waves x tile work; measured on B200):
//   - one-SM 128 x 256 tiles when M <= 128 (a pair would leave half its MMA rows empty) or when
//     they fit one wave (e.g. 1024^3: 32 tiles; the pair's set-up costs more than it saves);
//   - 256 x 512 pair tiles (K-major B, int32 / fp32 out) when their waves x 2 x t_w beat the
//     256-wide pair tiles' waves; t_w = 0.93 (their lower operand intake per multiply-add shows
//     as ~7 % shorter time per unit of work) for bf16 and for launches of at most two waves, and
//     1.01 for longer int8 launches, which run at the 1 kW power limit where intake does not bind;
//   - 256 x 480 or 256 x 464 pair tiles (hi half 224 or 208 wide) instead of 256 x 512 when they
//     need fewer waves x width, e.g. M = 1024 or 2048 with N = 8192 (the 8- and 4-GPU shards of
//     8192^3: 72 or 144 tiles of 464 against 64 or 128 of 512);
//   - otherwise 256 x 256 pair tiles, or 256 x 224 where that needs fewer waves.
// zx_set_kernel_policy() forces any one path.
template <zx::Kind kKind, bool kMN, zx::Out kOut>
int dispatch_gemm(zx_devptr A, zx_devptr B, zx_devptr C, const float* rs, const float* cs,
                  uint32_t M, uint32_t N, uint32_t K, cudaStream_t stream, const char* fn, uint32_t ldc = 0) {
  int pol = g_policy.load(std::memory_order_relaxed);
  if (pol == 0) {
    int dev = 0;
    DeviceInfo* di = nullptr;
    if (int rc = current_device(&dev, &di)) return rc;
    const uint64_t sms = static_cast<uint64_t>(di->sm_count), pairs = sms / 2;
    auto cdiv = [](uint64_t a, uint64_t b) { return (a + b - 1) / b; };
    const uint64_t t1 = cdiv(M, 128) * cdiv(N, 256);
    if (M <= 128 || t1 <= sms) {
      pol = 1;
    } else {
      pol = 2;
      if constexpr (!kMN && kOut != zx::Out::BF16_SCALED) {
        // cost of a shape = full-machine waves x tile width (MMA time is proportional to N)
        const uint64_t mt = cdiv(M, 256);
        auto waves = [&](uint64_t bn) { return cdiv(mt * cdiv(N, bn), pairs); };
        const uint64_t c256 = 256 * waves(256), c224 = 224 * waves(224);
        const double pair_cost = static_cast<double>(c224 < c256 ? c224 : c256);
        const double tw = (kKind == zx::Kind::BF16 || waves(512) <= 2) ? 0.93 : 1.01;
        const double w512 = tw * 512.0 * static_cast<double>(waves(512));
        const double w480 = tw * 480.0 * static_cast<double>(waves(480));
        const double w464 = tw * 464.0 * static_cast<double>(waves(464));
        const double wide = w464 < w480 ? (w464 < w512 ? w464 : w512) : (w480 < w512 ? w480 : w512);
        if (wide < pair_cost) pol = wide == w464 ? 6 : wide == w480 ? 5 : 4;
      }
    }
  }
  if constexpr (!kMN) {
    if (pol == 4) return launch_gemm2w<kKind, kOut>(A, B, C, rs, cs, M, N, K, stream, fn, nullptr, 0, ldc);
    if (pol == 5 || pol == 6) {
      constexpr bool kNarrow = kOut != zx::Out::BF16_SCALED;  // the scaled-bf16 epilogue keeps 512
      if (pol == 6 && kNarrow)
        return launch_gemm2w<kKind, kOut, kNarrow ? 208 : 256>(A, B, C, rs, cs, M, N, K, stream, fn, nullptr, 0, ldc);
      return launch_gemm2w<kKind, kOut, kNarrow ? 224 : 256>(A, B, C, rs, cs, M, N, K, stream, fn, nullptr, 0, ldc);
    }
  }
  if (pol == 1) {
    if constexpr (!kMN) {  // narrower one-SM tiles when they put more SMs to work (see small_tile_n)
      int dev = 0;
      DeviceInfo* di = nullptr;
      if (int rc = current_device(&dev, &di)) return rc;
      const uint32_t bn = small_tile_n(M, N, static_cast<uint32_t>(di->sm_count));
      if (bn == 64) return launch_gemm<kKind, kMN, kOut, 64, 8>(A, B, C, rs, cs, M, N, K, stream, fn, ldc);
      if (bn == 128) return launch_gemm<kKind, kMN, kOut, 128, 6>(A, B, C, rs, cs, M, N, K, stream, fn, ldc);
    }
    return launch_gemm<kKind, kMN, kOut, 256, 4>(A, B, C, rs, cs, M, N, K, stream, fn, ldc);
  }
  if constexpr (!kMN && kOut != zx::Out::BF16_SCALED) {
    if (pol == 2 && pair_tile_n(M, N) == 224)
      return launch_gemm2<kKind, kMN, kOut, kPairStages, 224>(A, B, C, rs, cs, M, N, K, stream, fn, ldc);
  }
  return launch_gemm2<kKind, kMN, kOut, kPairStages>(A, B, C, rs, cs, M, N, K, stream, fn, ldc);
}
int launch_sp2(zx_devptr Ac, zx_devptr E, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N,
               uint32_t K, cudaStream_t stream, const char* fn) {
  using Cfg = zx::Sp2Cfg;
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  zx::SpParams sp;
  memset(&sp, 0, sizeof(sp));
  zx::GemmParams& p = sp.g;
  int rc = encode_2d(&p.tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, reinterpret_cast<void*>(Ac), K / 2, M, K / 2,
                     128, Cfg::BM_CTA, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "A_c (M x K/2 kept values)");
  if (rc) return rc;
  rc = encode_2d(&sp.tmE, CU_TENSOR_MAP_DATA_TYPE_UINT32, reinterpret_cast<void*>(E), K / 32, M, K / 8, 4,
                 Cfg::BM_CTA, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "meta (M x K/32 u32)",
                 CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  rc = encode_2d(&p.tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, reinterpret_cast<void*>(B), K, N, K, 128, Cfg::BN_CTA,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "B (N x K)");
  if (rc) return rc;
  rc = encode_2d(&p.tmC, CU_TENSOR_MAP_DATA_TYPE_INT32, reinterpret_cast<void*>(C), N, M, uint64_t(N) * 4,
                 Cfg::CHUNK_COLS, 32, CU_TENSOR_MAP_L2_PROMOTION_NONE, "C");
  if (rc) return rc;
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_m_blk = (M + Cfg::BM - 1) / Cfg::BM;
  p.num_n_blk = (N + Cfg::BN - 1) / Cfg::BN;
  p.num_k_blk = K / Cfg::KD;
  p.group_m = ZX_GROUP_M2;
  auto kern = zx::gemm_sp2_kernel;
  static int max_clusters[kMaxDevices] = {};
  if (int rc = pair_capacity(kern, Cfg::THREADS, Cfg::SMEM_BYTES, dev, di, max_clusters, fn)) return rc;
  const uint32_t tiles = p.num_m_blk * p.num_n_blk;
  const uint32_t pairs = tiles < static_cast<uint32_t>(max_clusters[dev]) ? tiles : max_clusters[dev];
  kern<<<2 * pairs, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(sp);
  note_kernel("gemm_sp2_kernel 2-SM %dx%d sparse tiles, %u CTA pairs", Cfg::BM, Cfg::BN, pairs);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return 0;
}

// 2:4 sparse on 512 x 224 pair tiles (zx_gemm_sp4.cuh): two 256-row blocks of A share each B
// block, 29 % fewer operand bytes per multiply-add than the 256 x 224 tiles.
int launch_sp4(zx_devptr Ac, zx_devptr E, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N,
               uint32_t K, cudaStream_t stream, const char* fn) {
  using Cfg = zx::Sp4Cfg;
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  zx::SpParams sp;
  memset(&sp, 0, sizeof(sp));
  zx::GemmParams& p = sp.g;
  int rc = encode_2d(&p.tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, reinterpret_cast<void*>(Ac), K / 2, M, K / 2,
                     128, Cfg::BM_CTA, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "A_c (M x K/2 kept values)");
  if (rc) return rc;
  rc = encode_2d(&sp.tmE, CU_TENSOR_MAP_DATA_TYPE_UINT32, reinterpret_cast<void*>(E), K / 32, M, K / 8, 4,
                 Cfg::BM_CTA, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "meta (M x K/32 u32)",
                 CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  rc = encode_2d(&p.tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, reinterpret_cast<void*>(B), K, N, K, 128, Cfg::BN_CTA,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "B (N x K)");
  if (rc) return rc;
  rc = encode_2d(&p.tmC, CU_TENSOR_MAP_DATA_TYPE_INT32, reinterpret_cast<void*>(C), N, M, uint64_t(N) * 4,
                 Cfg::CHUNK_COLS, Cfg::EPI_ROWS, CU_TENSOR_MAP_L2_PROMOTION_NONE, "C");
  if (rc) return rc;
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_m_blk = (M + Cfg::BM - 1) / Cfg::BM;
  p.num_n_blk = (N + Cfg::BN - 1) / Cfg::BN;
  p.num_k_blk = K / Cfg::KD;
  p.group_m = ZX_GROUP_M2 / 2;  // the same rows of A per raster group as the 256-row tiles
  auto kern = zx::gemm_sp4_kernel;
  static int max_clusters[kMaxDevices] = {};
  if (int rc = pair_capacity(kern, Cfg::THREADS, Cfg::SMEM_BYTES, dev, di, max_clusters, fn)) return rc;
  const uint32_t tiles = p.num_m_blk * p.num_n_blk;
  const uint32_t pairs = tiles < static_cast<uint32_t>(max_clusters[dev]) ? tiles : max_clusters[dev];
  kern<<<2 * pairs, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(sp);
  note_kernel("gemm_sp4_kernel 2-SM %dx%d sparse tiles, %u CTA pairs", Cfg::BM, Cfg::BN, pairs);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return 0;
}

// 2:4 sparse on 256 x 480 pair tiles (zx_gemm_sp2w.cuh): 25 % fewer operand bytes per
// multiply-add than the 256 x 224 tiles, whose loop is bound by each SM's operand intake.
int launch_sp2w(zx_devptr Ac, zx_devptr E, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N,
                uint32_t K, cudaStream_t stream, const char* fn) {
  using Cfg = zx::Sp2wCfg;
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  zx::SpParams sp;
  memset(&sp, 0, sizeof(sp));
  zx::GemmParams& p = sp.g;
  int rc = encode_2d(&p.tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, reinterpret_cast<void*>(Ac), K / 2, M, K / 2,
                     64, Cfg::BM_CTA, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "A_c (M x K/2 kept values)",
                     CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  rc = encode_2d(&sp.tmE, CU_TENSOR_MAP_DATA_TYPE_UINT32, reinterpret_cast<void*>(E), K / 32, M, K / 8, 4,
                 Cfg::BM_CTA, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "meta (M x K/32 u32)",
                 CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  rc = encode_2d(&p.tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, reinterpret_cast<void*>(B), K, N, K, 128, Cfg::BN_LO / 2,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "B (N x K, lo half)");
  if (rc) return rc;
  rc = encode_2d(&p.tmB2, CU_TENSOR_MAP_DATA_TYPE_UINT8, reinterpret_cast<void*>(B), K, N, K, 128, Cfg::BN_HI / 2,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "B (N x K, hi half)");
  if (rc) return rc;
  rc = encode_2d(&p.tmC, CU_TENSOR_MAP_DATA_TYPE_INT32, reinterpret_cast<void*>(C), N, M, uint64_t(N) * 4,
                 Cfg::CHUNK_COLS, Cfg::EPI_ROWS, CU_TENSOR_MAP_L2_PROMOTION_NONE, "C");
  if (rc) return rc;
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_m_blk = (M + Cfg::BM - 1) / Cfg::BM;
  p.num_n_blk = (N + Cfg::BN - 1) / Cfg::BN;
  p.num_k_blk = K / Cfg::KD;
  p.group_m = ZX_GROUP_M2;
  auto kern = zx::gemm_sp2w_kernel;
  static int max_clusters[kMaxDevices] = {};
  if (int rc = pair_capacity(kern, Cfg::THREADS, Cfg::SMEM_BYTES, dev, di, max_clusters, fn)) return rc;
  const uint32_t tiles = p.num_m_blk * p.num_n_blk;
  const uint32_t pairs = tiles < static_cast<uint32_t>(max_clusters[dev]) ? tiles : max_clusters[dev];
  kern<<<2 * pairs, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(sp);
  note_kernel("gemm_sp2w_kernel 2-SM %dx%d sparse tiles, %u CTA pairs", Cfg::BM, Cfg::BN, pairs);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return 0;
}

// Sparse tile choice. Measured on B200 at 8192^3: 512 x 224 tiles 247 us, 256 x 224 tiles 264 us,
// 256 x 480 tiles 275-281 us (the 256-row kernels keep the tensor pipe about half busy, bound by
// operand delivery; the 512 x 224 tile takes in 29 % fewer bytes per multiply-add). Automatic
// policy: cost = full-machine waves x 256-row blocks per tile, the 512-row tiles weighted 0.94 per
// block for their faster blocks; a 512-row tile over M <= 256 rows would compute an empty block.
// Policies 1-3 force the 256 x 224 kernel, 4 and 5 the 256 x 480 one, 6 the 512 x 224 one.
int dispatch_sp(zx_devptr Ac, zx_devptr E, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                cudaStream_t stream, const char* fn) {
  const int pol = g_policy.load(std::memory_order_relaxed);
  if (pol == 6) return launch_sp4(Ac, E, B, C, M, N, K, stream, fn);
  if (pol == 4 || pol == 5) return launch_sp2w(Ac, E, B, C, M, N, K, stream, fn);
  if (pol == 0) {
    int dev = 0;
    DeviceInfo* di = nullptr;
    if (int rc = current_device(&dev, &di)) return rc;
    const uint64_t pairs = static_cast<uint64_t>(di->sm_count) / 2;
    auto cdiv = [](uint64_t a, uint64_t b) { return (a + b - 1) / b; };
    const uint64_t nt = cdiv(N, zx::Sp2Cfg::BN);
    const double w2 = static_cast<double>(cdiv(cdiv(M, 256) * nt, pairs));
    const double w4 = static_cast<double>(cdiv(cdiv(M, 512) * nt, pairs));
    if (2.0 * 0.94 * w4 < w2) return launch_sp4(Ac, E, B, C, M, N, K, stream, fn);
  }
  return launch_sp2(Ac, E, B, C, M, N, K, stream, fn);
}

// W4A8 for large M with the unpacked weights in tensor memory (zx_gemm_w4t.cuh); K % 256 == 0.
int launch_w4t(zx_devptr A, zx_devptr W, zx_devptr C, uint32_t M, uint32_t N, uint32_t K, cudaStream_t stream,
               const char* fn) {
  using Cfg = zx::W4tCfg;
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  zx::GemmParams p;
  memset(&p, 0, sizeof(p));
  int rc = encode_2d(&p.tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, reinterpret_cast<void*>(A), K, M, K, 128, Cfg::BX_CTA,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "A (M x K activations)");
  if (rc) return rc;
  rc = encode_2d(&p.tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, reinterpret_cast<void*>(W), K / 2, N, K / 2, 128, Cfg::BW_CTA,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "W (N x K/2 packed s4)");
  if (rc) return rc;
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_m_blk = (M + Cfg::BX - 1) / Cfg::BX;
  p.num_n_blk = (N + Cfg::BW - 1) / Cfg::BW;
  p.num_k_blk = K / Cfg::KSTEP;
  p.group_m = p.num_m_blk;  // all activation blocks of a weight block back to back: W read once
  auto kern = zx::gemm_w4t_kernel;
  static int max_clusters[kMaxDevices] = {};
  if (int rc = pair_capacity(kern, Cfg::THREADS, Cfg::SMEM_BYTES, dev, di, max_clusters, fn)) return rc;
  const uint32_t tiles = p.num_m_blk * p.num_n_blk;
  const uint32_t pairs = tiles < static_cast<uint32_t>(max_clusters[dev]) ? tiles : max_clusters[dev];
  kern<<<2 * pairs, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(p, reinterpret_cast<int32_t*>(C));
  note_kernel("gemm_w4t_kernel 2-SM 256x256 tiles, weights in TMEM, %u CTA pairs", pairs);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : cuda_fail(e, fn);
}

// W4A8 shapes that do not take the weights-in-TMEM decode kernel: the weights-in-TMEM pair kernel
// when K % 256 == 0 (policies 0, 1, 4 and 5), else (or under policies 2 and 3) the pair kernel that
// unpacks the weights into shared memory.
int w4a8_large(zx_devptr A, zx_devptr W, zx_devptr C, uint32_t M, uint32_t N, uint32_t K, cudaStream_t s,
               const char* fn) {
  const int pol = g_policy.load(std::memory_order_relaxed);
  if (K % 256 == 0 && (pol <= 1 || pol >= 4)) return launch_w4t(A, W, C, M, N, K, s, fn);
  return launch_gemm2<zx::Kind::W4, false, zx::Out::S32, 5>(A, W, C, nullptr, nullptr, M, N, K, s, fn);
}

// Split-tile workspace of the weights-in-TMEM W4A8 kernel: partial-sum slots, then one counter per
// 128-row weight tile; `ctas` = the launch's grid.
struct W4sWorkspace {
  uint64_t part_bytes, cnt_bytes, ctas;
};
W4sWorkspace w4s_workspace(uint32_t nx, uint32_t N, uint32_t K, uint32_t sms) {
  const uint64_t n_tiles = (N + 127) / 128, steps = n_tiles * (K / 256);
  const uint64_t ctas = steps < sms ? steps : sms;
  return {zx::w4s_ws_part_bytes(nx, static_cast<uint32_t>(ctas)), ((n_tiles * 4 + 255) / 256) * 256, ctas};
}
uint32_t w4s_nx(uint32_t M) { return M <= 16 ? 16u : (M <= 32 ? 32u : 64u); }
// The weights-in-TMEM kernel runs for M <= 64 with K % 256 == 0 unless a policy forces pairs.
bool w4s_path(uint32_t M, uint32_t K) { return M <= 64 && K % 256 == 0 && g_policy.load(std::memory_order_relaxed) <= 1; }
// zx_gemm_w4a8_ws uses its workspace for M <= 32: there the partial-sum hand-over measured faster
// than zeroing C and adding into it (M = 16: 41.0 vs 41.7 us, M = 32: 43.0 vs 44.0 us); at
// M = 64 the 32 KB partial per CTA costs more (55.3 vs 53.1 us) and C is zeroed and added into.
bool w4s_ws_used(uint32_t M, uint32_t K) { return w4s_path(M, K) && M <= 32; }

template <int NX>
int launch_w4s(zx_devptr A, zx_devptr W, zx_devptr C, uint32_t M, uint32_t N, uint32_t K, zx_devptr ws,
               uint64_t ws_bytes, cudaStream_t stream, const char* fn) {
  using Cfg = zx::W4sCfg<NX>;
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  zx::W4sParams p;
  memset(&p, 0, sizeof(p));
  int rc = encode_2d(&p.tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, reinterpret_cast<void*>(W), K / 2, N, K / 2, 128,
                     128, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "W (N x K/2 packed s4)");
  if (rc) return rc;
  rc = encode_2d(&p.tmX, CU_TENSOR_MAP_DATA_TYPE_UINT8, reinterpret_cast<void*>(A), K, M, K, 128, NX,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "A (M x K)");
  if (rc) return rc;
  p.C = reinterpret_cast<int32_t*>(C);
  p.M = M;
  p.N = N;
  p.K = K;
  p.n_tiles = (N + 127) / 128;
  p.nk = K / Cfg::KSTEP;
  const uint32_t sms = static_cast<uint32_t>(di->sm_count);
  if (ws) {
    const W4sWorkspace w = w4s_workspace(NX, N, K, sms);
    if (ws_bytes < w.part_bytes + w.cnt_bytes)
      return fail(ZX_ERR_SHAPE, "%s: workspace of %llu bytes, this shape needs %llu", fn,
                  (unsigned long long)ws_bytes, (unsigned long long)(w.part_bytes + w.cnt_bytes));
    p.ws_part = reinterpret_cast<int32_t*>(ws);
    p.ws_cnt = reinterpret_cast<uint32_t*>(ws + w.part_bytes);
  } else {
    // every CTA adds its partial sums into C
    cudaError_t ez = cudaMemsetAsync(reinterpret_cast<void*>(C), 0, size_t(M) * N * 4, stream);
    if (ez != cudaSuccess) return cuda_fail(ez, "cudaMemsetAsync(C)");
  }
  auto kern = zx::gemm_w4s_kernel<NX>;
  static bool attr_done[kMaxDevices] = {};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
      attr_done[dev] = true;
    }
  }
  const uint64_t steps = uint64_t(p.n_tiles) * p.nk;
  kern<<<steps < sms ? static_cast<uint32_t>(steps) : sms, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(p);
  note_kernel("gemm_w4s_kernel weights-in-TMEM W4A8, %d activation rows, grid %u", NX,
              steps < sms ? static_cast<uint32_t>(steps) : sms);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : cuda_fail(e, fn);
}

}  // namespace

// ------------------------- W4A8 decode without any device allocation -------------------------
// Scratch of zx_gemm_w4a8_noalloc: the split-tile partial sums and tile counters that
// zx_gemm_w4a8_ws keeps in a caller workspace, here in one file-scope device array that every
// GPU loading this library holds until the process exits. Sized for M <= 32 (32 partial rows per
// slot), up to 160 CTAs (two slots each) and N <= 65536 (512 tile counters): 5 MiB + 2 KiB.
constexpr uint32_t kNoAllocMaxM = 32;
constexpr uint32_t kNoAllocMaxN = 65536;
constexpr uint32_t kNoAllocMaxCtas = 160;
constexpr uint64_t kNoAllocBytes = zx::w4s_ws_part_bytes(kNoAllocMaxM, kNoAllocMaxCtas) + (kNoAllocMaxN / 128) * 4;
static __device__ __align__(256) unsigned char g_w4a8_scratch[kNoAllocBytes];

namespace {
// Host code cannot use g_w4a8_scratch's name as a device address (it names a host-side shadow),
// so each device's address of the array is looked up once, with that device current.
// The address is per CUDA context (each context loads its own copy of the module), so it is cached
// per (device, current context): a caller that makes its own driver context current gets that
// context's copy, not the primary context's.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
constexpr int kScratchCtxs = 8;
struct ScratchAddr {
  CUcontext ctx;
  zx_devptr addr;
};
ScratchAddr g_w4a8_scratch_addr[kMaxDevices][kScratchCtxs] = {};

int w4a8_scratch_addr(int dev, zx_devptr* out) {
  static CtxGetCurrentFn get_ctx = nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!get_ctx) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !f)
      return fail(ZX_ERR_DRIVER, "driver entry point cuCtxGetCurrent unavailable");
    get_ctx = reinterpret_cast<CtxGetCurrentFn>(f);
  }
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS || !ctx)
    return fail(ZX_ERR_DRIVER, "zx_gemm_w4a8_noalloc: no current CUDA context on device %d", dev);
  ScratchAddr* row = g_w4a8_scratch_addr[dev];
  for (int i = 0; i < kScratchCtxs; ++i)
    if (row[i].ctx == ctx) {
      *out = row[i].addr;
      return 0;
    }
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_w4a8_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(W4A8 scratch)");
  if (!ptr) return fail(ZX_ERR_DRIVER, "cudaGetSymbolAddress(W4A8 scratch) returned a null address");
  for (int i = 0; i < kScratchCtxs; ++i)
    if (!row[i].ctx) {
      row[i] = {ctx, reinterpret_cast<zx_devptr>(ptr)};
      break;
    }  // with every slot taken the address is simply looked up on each call
  *out = reinterpret_cast<zx_devptr>(ptr);
  return 0;
}

// ------------------------- GEMM on host buffers, copies overlapped -------------------------
// The reference's bench flow copies A and B to the device, launches, and copies C back, one step
// after the other (src/bench.zig:647-741). Here A and B travel in blocks of rows (A: ci blocks,
// B: cj blocks = column blocks of C) on one copy stream, in the order B0 A0 B1 A1 ..., and C is
// produced in growing shells: shell t is the L-shaped region of C that A_0..A_t and B_0..B_t
// complete, computed as two GEMMs (its column part, rows of A_0..A_{t-1} against B_t, as soon as
// B_t has arrived; its row part, A_t against B_0..B_t, as soon as A_t has) and copied back as two
// 2-D copies on a second copy stream as soon as each is computed. The first bytes of C then leave
// after two input blocks instead of all of B, and the copy back (the larger transfer) runs nearly
// the whole time; C on the device is row-major, each GEMM writing its part with row pitch N.
#ifndef ZX_PIPE_ROWS
#define ZX_PIPE_ROWS 1024
#endif
#ifndef ZX_PIPE_MAX
#define ZX_PIPE_MAX 4
#endif
constexpr int kPipeMaxChunks = ZX_PIPE_MAX;
constexpr int kPipeEvents = 2 + 4 * kPipeMaxChunks;
struct HostPipe {
  bool ready = false;
  cudaStream_t h2d = nullptr, d2h[2] = {nullptr, nullptr};  // copies back alternate between two streams
  cudaEvent_t ev[kPipeEvents] = {};
  std::mutex mu;  // one enqueue at a time per device: the events are reused by the next call
};
HostPipe g_pipe[kMaxDevices];

int host_pipe(int dev, HostPipe** out) {
  HostPipe& hp = g_pipe[dev];
  if (!hp.ready) {
    cudaError_t e;
    if ((e = cudaStreamCreateWithFlags(&hp.h2d, cudaStreamNonBlocking)) != cudaSuccess)
      return cuda_fail(e, "cudaStreamCreateWithFlags(host-to-device copies)");
    for (auto& d : hp.d2h)
      if ((e = cudaStreamCreateWithFlags(&d, cudaStreamNonBlocking)) != cudaSuccess)
        return cuda_fail(e, "cudaStreamCreateWithFlags(device-to-host copies)");
    for (auto& ev : hp.ev)
      if ((e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming)) != cudaSuccess)
        return cuda_fail(e, "cudaEventCreateWithFlags(pipeline)");
    hp.ready = true;
  }
  *out = &hp;
  return 0;
}

// Blocks of at least 1024 rows / columns, at most kPipeMaxChunks (4) per side: at 8192^3, 4 blocks
// of 2048 measured 5.94 ms per call against 5.97-6.02 ms for 8 of 1024 and 6.43-6.50 ms for 2 of
// 4096 (fewer, larger copies against an earlier first shell). Column bounds are
// multiples of 4 so every part of int32 / fp32 C starts on a 16-byte boundary.
inline uint32_t pipe_chunks(uint32_t n) {
  const uint32_t c = n / ZX_PIPE_ROWS;
  return c < 1 ? 1 : (c > kPipeMaxChunks ? kPipeMaxChunks : c);
}

template <zx::Kind kKind, zx::Out kOut>
int gemm_host_pipeline(const void* A_h, const void* B_h, void* C_h, zx_devptr A_d, zx_devptr B_d,
                       zx_devptr C_d, uint32_t M, uint32_t N, uint32_t K, uint32_t esz, cudaStream_t s,
                       const char* fn) {
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  std::lock_guard<std::mutex> lk(g_pipe[dev].mu);
  HostPipe* hp = nullptr;
  {
    std::lock_guard<std::mutex> lk2(g_mu);
    if (int rc = host_pipe(dev, &hp)) return rc;
  }
  const uint32_t ci = pipe_chunks(M), cj = pipe_chunks(N), shells = ci > cj ? ci : cj;
  uint32_t rb[kPipeMaxChunks + 1], cb[kPipeMaxChunks + 1];
  for (uint32_t i = 0; i <= ci; ++i) rb[i] = static_cast<uint32_t>(uint64_t(M) * i / ci);
  for (uint32_t j = 0; j <= cj; ++j) cb[j] = static_cast<uint32_t>(uint64_t(N / 4u) * j / cj) * 4u;
  cudaEvent_t start = hp->ev[0], done = hp->ev[1];
  cudaEvent_t* a_in = hp->ev + 2;
  cudaEvent_t* b_in = a_in + kPipeMaxChunks;
  cudaEvent_t* computed = b_in + kPipeMaxChunks;  // 2 per shell: column part, row part
  const auto* a_host = static_cast<const unsigned char*>(A_h);
  const auto* b_host = static_cast<const unsigned char*>(B_h);
  auto* c_host = static_cast<unsigned char*>(C_h);
  const uint64_t arow = uint64_t(K) * esz, crow = uint64_t(N) * 4u;  // bytes per row of A / B, of C
  cudaError_t e;
#define ZX_PIPE(call, what) \
  if ((e = (call)) != cudaSuccess) return cuda_fail(e, what)
  // the copies start after the caller's earlier work on `s` (which may still use the buffers)
  ZX_PIPE(cudaEventRecord(start, s), "cudaEventRecord");
  ZX_PIPE(cudaStreamWaitEvent(hp->h2d, start, 0), "cudaStreamWaitEvent");
  for (cudaStream_t d : hp->d2h) ZX_PIPE(cudaStreamWaitEvent(d, start, 0), "cudaStreamWaitEvent");
  uint32_t part_no = 0;
  for (uint32_t t = 0; t < shells; ++t) {
    if (t < cj) {
      ZX_PIPE(cudaMemcpyAsync(reinterpret_cast<void*>(B_d + cb[t] * arow), b_host + cb[t] * arow,
                              (cb[t + 1] - cb[t]) * arow, cudaMemcpyHostToDevice, hp->h2d), "cudaMemcpyAsync(B block)");
      ZX_PIPE(cudaEventRecord(b_in[t], hp->h2d), "cudaEventRecord");
    }
    if (t < ci) {
      ZX_PIPE(cudaMemcpyAsync(reinterpret_cast<void*>(A_d + rb[t] * arow), a_host + rb[t] * arow,
                              (rb[t + 1] - rb[t]) * arow, cudaMemcpyHostToDevice, hp->h2d), "cudaMemcpyAsync(A block)");
      ZX_PIPE(cudaEventRecord(a_in[t], hp->h2d), "cudaEventRecord");
    }
  }
  // rows [r0, r1) x columns [c0, c1) of C, once `ready` has completed: GEMM, then the copy back
  auto part = [&](uint32_t r0, uint32_t r1, uint32_t c0, uint32_t c1, cudaEvent_t ready, cudaEvent_t ev) -> int {
    ZX_PIPE(cudaStreamWaitEvent(s, ready, 0), "cudaStreamWaitEvent");
    const uint64_t off = uint64_t(r0) * crow + uint64_t(c0) * 4u;
    if (int rc = dispatch_gemm<kKind, false, kOut>(A_d + r0 * arow, B_d + c0 * arow, C_d + off, nullptr, nullptr,
                                                   r1 - r0, c1 - c0, K, s, fn, N))
      return rc;
    ZX_PIPE(cudaEventRecord(ev, s), "cudaEventRecord");
    // consecutive parts go back on alternate copy streams (measured ~2 % shorter at 8192^3 than one)
    cudaStream_t back = hp->d2h[part_no++ & 1u];
    ZX_PIPE(cudaStreamWaitEvent(back, ev, 0), "cudaStreamWaitEvent");
    ZX_PIPE(cudaMemcpy2DAsync(c_host + off, crow, reinterpret_cast<const void*>(C_d + off), crow,
                              uint64_t(c1 - c0) * 4u, r1 - r0, cudaMemcpyDeviceToHost, back),
            "cudaMemcpy2DAsync(C part)");
    return 0;
  };
  for (uint32_t t = 0; t < shells; ++t) {
    const uint32_t rows_before = rb[t < ci ? t : ci];
    if (t < cj && rows_before > 0)  // column part: A_0..A_{t-1} against B_t
      if (int rc = part(0, rows_before, cb[t], cb[t + 1], b_in[t], computed[2 * t])) return rc;
    if (t < ci)  // row part: A_t against B_0..B_t
      if (int rc = part(rb[t], rb[t + 1], 0, cb[t + 1 < cj ? t + 1 : cj], a_in[t], computed[2 * t + 1])) return rc;
  }
  for (cudaStream_t d : hp->d2h) {  // the caller's stream waits for both copy-back streams
    ZX_PIPE(cudaEventRecord(done, d), "cudaEventRecord");
    ZX_PIPE(cudaStreamWaitEvent(s, done, 0), "cudaStreamWaitEvent");
  }
#undef ZX_PIPE
  char last[sizeof(t_kernel)];
  std::memcpy(last, t_kernel, sizeof(last));
  note_kernel("%s: %u x %u blocks in %u shells, copies overlapped; last part on %s", fn, ci, cj, shells, last);
  return 0;
}

}  // namespace

extern "C" {

int zx_gemm_w4a8_noalloc(zx_devptr A, zx_devptr W, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                         zx_stream stream) {
  t_err[0] = 0;
  const char* fn = "zx_gemm_w4a8_noalloc";
  if (int rc = check_common(A, W, C, M, N, K, ZX_LAYOUT_NT, 32, 4, 16, fn)) return rc;
  if (M > kNoAllocMaxM)
    return fail(ZX_ERR_SHAPE, "%s: M=%u is above the maximum of %u that its built-in scratch holds "
                "(zx_gemm_w4a8 takes any M)", fn, M, kNoAllocMaxM);
  if (N > kNoAllocMaxN)
    return fail(ZX_ERR_SHAPE, "%s: N=%u is above the maximum of %u that its built-in scratch holds "
                "(zx_gemm_w4a8 takes any N)", fn, N, kNoAllocMaxN);
  if (K % 256 != 0) return fail(ZX_ERR_SHAPE, "%s: K=%u must be a multiple of 256", fn, K);
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  if (static_cast<uint32_t>(di->sm_count) > kNoAllocMaxCtas)
    return fail(ZX_ERR_SHAPE, "%s: device %d has %d SMs; the built-in scratch holds %u CTAs", fn, dev,
                di->sm_count, kNoAllocMaxCtas);
  zx_devptr scratch = 0;
  if (int rc = w4a8_scratch_addr(dev, &scratch)) return rc;
  const uint32_t nx = M <= 16 ? 16u : 32u;
  const W4sWorkspace w = w4s_workspace(nx, N, K, static_cast<uint32_t>(di->sm_count));
  if (w.part_bytes + w.cnt_bytes > kNoAllocBytes)
    return fail(ZX_ERR_SHAPE, "%s: this shape needs %llu bytes of scratch, the built-in array has %llu", fn,
                (unsigned long long)(w.part_bytes + w.cnt_bytes), (unsigned long long)kNoAllocBytes);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  // the tile counters must start at zero (a completed call leaves them so; a call that gave up on
  // a device wait may not)
  cudaError_t e = cudaMemsetAsync(reinterpret_cast<void*>(scratch + w.part_bytes), 0, w.cnt_bytes, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(W4A8 scratch counters)");
  if (nx == 16) return launch_w4s<16>(A, W, C, M, N, K, scratch, kNoAllocBytes, s, fn);
  return launch_w4s<32>(A, W, C, M, N, K, scratch, kNoAllocBytes, s, fn);
}


int zx_gemm_sp_s8(zx_devptr A_c, zx_devptr meta, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N,
                  uint32_t K, zx_stream stream) {
  t_err[0] = 0;
  if (int rc = check_common(A_c, B, C, M, N, K, ZX_LAYOUT_NT, 256, 4, 16, "zx_gemm_sp_s8")) return rc;
  if (M % 128 != 0) return fail(ZX_ERR_SHAPE, "zx_gemm_sp_s8: M=%u must be a multiple of 128", M);
  if (!meta) return fail(ZX_ERR_NULL, "zx_gemm_sp_s8: null metadata buffer");
  if (!aligned16(meta)) return fail(ZX_ERR_ALIGN, "zx_gemm_sp_s8: metadata must be 16-byte aligned");
  return dispatch_sp(A_c, meta, B, C, M, N, K, reinterpret_cast<cudaStream_t>(stream), "zx_gemm_sp_s8");
}

// ------------------------- the reference's NN operand layouts, fast path -------------------------
// One layout pass into the caller's workspace (HBM-bound, zx_layout.cuh), then the K-major kernels.
namespace {
constexpr uint64_t round256(uint64_t x) { return (x + 255u) & ~uint64_t(255u); }
uint64_t nn_workspace_bytes(int op, uint32_t M, uint32_t N, uint32_t K) {
  if (op == ZX_NN_SP_S4)  // int8 2:4 A_c | int8 metadata | int8 B (N x K)
    return round256(uint64_t(M) * (K / 2u)) + round256(uint64_t(M) * (K / 32u) * 4u) + uint64_t(N) * K;
  return op == ZX_NN_SP_S8 ? uint64_t(N) * K : round256(uint64_t(M) * K) + uint64_t(N) * (K / 2u);
}
int check_workspace(zx_devptr ws, uint64_t have, uint64_t need, const char* fn) {
  if (!ws) return fail(ZX_ERR_NULL, "%s: null workspace", fn);
  if (!aligned16(ws)) return fail(ZX_ERR_ALIGN, "%s: workspace must be 16-byte aligned", fn);
  if (have < need)
    return fail(ZX_ERR_SHAPE, "%s: workspace of %llu bytes, this shape needs %llu", fn, (unsigned long long)have,
                (unsigned long long)need);
  return 0;
}
}  // namespace

int zx_gemm_nn_workspace_bytes(int op, uint32_t M, uint32_t N, uint32_t K, uint64_t* bytes) {
  t_err[0] = 0;
  if (!bytes) return fail(ZX_ERR_NULL, "zx_gemm_nn_workspace_bytes: null output pointer");
  if (op != ZX_NN_SP_S8 && op != ZX_NN_S4S4 && op != ZX_NN_SP_S4)
    return fail(ZX_ERR_SHAPE, "zx_gemm_nn_workspace_bytes: unknown op %d (%d sparse int8, %d s4 x s4, %d sparse s4)",
                op, ZX_NN_SP_S8, ZX_NN_S4S4, ZX_NN_SP_S4);
  *bytes = nn_workspace_bytes(op, M, N, K);
  return 0;
}

int zx_gemm_sp_s8_nn(zx_devptr A_c, zx_devptr meta, zx_devptr B_kn, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                     zx_devptr workspace, uint64_t workspace_bytes, zx_stream stream) {
  t_err[0] = 0;
  const char* fn = "zx_gemm_sp_s8_nn";
  if (int rc = check_common(A_c, B_kn, C, M, N, K, ZX_LAYOUT_NN, 256, 16, 16, fn)) return rc;
  if (M % 128 != 0) return fail(ZX_ERR_SHAPE, "%s: M=%u must be a multiple of 128", fn, M);
  if (!meta) return fail(ZX_ERR_NULL, "%s: null metadata buffer", fn);
  if (!aligned16(meta)) return fail(ZX_ERR_ALIGN, "%s: metadata must be 16-byte aligned", fn);
  if (int rc = check_workspace(workspace, workspace_bytes, nn_workspace_bytes(ZX_NN_SP_S8, M, N, K), fn)) return rc;
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  zx::transpose_u8_kernel<<<dim3((N + 63) / 64, (K + 63) / 64), 256, 0, s>>>(
      reinterpret_cast<const uint8_t*>(B_kn), reinterpret_cast<uint8_t*>(workspace), K, N);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return dispatch_sp(A_c, meta, workspace, C, M, N, K, s, fn);
}

int zx_gemm_sp_s4_nn(zx_devptr A_c, zx_devptr meta, zx_devptr B_kn, zx_devptr C, uint32_t M, uint32_t N,
                     uint32_t K, zx_devptr workspace, uint64_t workspace_bytes, zx_stream stream) {
  t_err[0] = 0;
  const char* fn = "zx_gemm_sp_s4_nn";
  if (int rc = check_common(A_c, B_kn, C, M, N, K, ZX_LAYOUT_NN, 256, 16, 16, fn)) return rc;
  if (M % 128 != 0) return fail(ZX_ERR_SHAPE, "%s: M=%u must be a multiple of 128", fn, M);
  if (!meta) return fail(ZX_ERR_NULL, "%s: null metadata buffer", fn);
  if (!aligned16(meta)) return fail(ZX_ERR_ALIGN, "%s: metadata must be 16-byte aligned", fn);
  if (int rc = check_workspace(workspace, workspace_bytes, nn_workspace_bytes(ZX_NN_SP_S4, M, N, K), fn)) return rc;
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  const zx_devptr A8 = workspace, E8 = A8 + round256(uint64_t(M) * (K / 2u));
  const zx_devptr B8 = E8 + round256(uint64_t(M) * (K / 32u) * 4u);
  const uint64_t units = uint64_t(M) * (K / 64u);
  const uint64_t blocks = (units + 255u) / 256u, cap = uint64_t(di->sm_count) * 16u;
  zx::sp48_a_kernel<<<static_cast<unsigned>(blocks < cap ? blocks : cap), 256, 0, s>>>(
      reinterpret_cast<const uint8_t*>(A_c), reinterpret_cast<const uint32_t*>(meta), reinterpret_cast<int8_t*>(A8),
      reinterpret_cast<uint32_t*>(E8), units);
  zx::sp48_b_kernel<<<dim3((N + 63) / 64, (K + 63) / 64), 256, 0, s>>>(reinterpret_cast<const uint8_t*>(B_kn),
                                                                       reinterpret_cast<int8_t*>(B8), K, N);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return dispatch_sp(A8, E8, B8, C, M, N, K, s, fn);
}

int zx_gemm_s4s4_nn(zx_devptr A, zx_devptr B_kn, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                    zx_devptr workspace, uint64_t workspace_bytes, zx_stream stream) {
  t_err[0] = 0;
  const char* fn = "zx_gemm_s4s4_nn";
  if (int rc = check_common(A, B_kn, C, M, N, K, ZX_LAYOUT_NN, 64, 16, 16, fn)) return rc;
  if (int rc = check_workspace(workspace, workspace_bytes, nn_workspace_bytes(ZX_NN_S4S4, M, N, K), fn)) return rc;
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  const zx_devptr A8 = workspace, W = workspace + round256(uint64_t(M) * K);
  const uint64_t groups = uint64_t(M) * K / 16u;
  const uint64_t blocks = (groups + 255u) / 256u, cap = uint64_t(di->sm_count) * 16u;
  zx::unpack_s4_kernel<<<static_cast<unsigned>(blocks < cap ? blocks : cap), 256, 0, s>>>(
      reinterpret_cast<const uint8_t*>(A), reinterpret_cast<int8_t*>(A8), groups);
  zx::s4_repack_kernel<<<dim3((N + 63) / 64, (K + 63) / 64), 256, 0, s>>>(
      reinterpret_cast<const uint8_t*>(B_kn), reinterpret_cast<uint8_t*>(W), K, N);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, fn);
  if (w4s_path(M, K)) {
    if (M <= 16) return launch_w4s<16>(A8, W, C, M, N, K, 0, 0, s, fn);
    if (M <= 32) return launch_w4s<32>(A8, W, C, M, N, K, 0, 0, s, fn);
    return launch_w4s<64>(A8, W, C, M, N, K, 0, 0, s, fn);
  }
  return w4a8_large(A8, W, C, M, N, K, s, fn);
}


int zx_gemm_w4a8(zx_devptr A, zx_devptr W, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                 zx_stream stream) {
  t_err[0] = 0;
  if (int rc = check_common(A, W, C, M, N, K, ZX_LAYOUT_NT, 32, 4, 16, "zx_gemm_w4a8")) return rc;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (w4s_path(M, K)) {  // few activation rows: weights in TMEM, HBM-bound
    if (M <= 16) return launch_w4s<16>(A, W, C, M, N, K, 0, 0, s, "zx_gemm_w4a8");
    if (M <= 32) return launch_w4s<32>(A, W, C, M, N, K, 0, 0, s, "zx_gemm_w4a8");
    return launch_w4s<64>(A, W, C, M, N, K, 0, 0, s, "zx_gemm_w4a8");
  }
  return w4a8_large(A, W, C, M, N, K, s, "zx_gemm_w4a8");
}


int zx_gemm_w4a8_workspace_bytes(uint32_t M, uint32_t N, uint32_t K, uint64_t* bytes) {
  t_err[0] = 0;
  if (!bytes) return fail(ZX_ERR_NULL, "zx_gemm_w4a8_workspace_bytes: null output pointer");
  if (M == 0 || N == 0 || K == 0 || K % 32 != 0)
    return fail(ZX_ERR_SHAPE, "zx_gemm_w4a8_workspace_bytes: bad shape M=%u N=%u K=%u", M, N, K);
  *bytes = 0;
  if (!w4s_ws_used(M, K)) return 0;
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  const W4sWorkspace w = w4s_workspace(w4s_nx(M), N, K, static_cast<uint32_t>(di->sm_count));
  *bytes = w.part_bytes + w.cnt_bytes;
  return 0;
}

int zx_gemm_w4a8_ws(zx_devptr A, zx_devptr W, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                    zx_devptr workspace, uint64_t workspace_bytes, zx_stream stream) {
  t_err[0] = 0;
  if (int rc = check_common(A, W, C, M, N, K, ZX_LAYOUT_NT, 32, 4, 16, "zx_gemm_w4a8_ws")) return rc;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (!w4s_path(M, K)) return w4a8_large(A, W, C, M, N, K, s, "zx_gemm_w4a8_ws");  // no workspace needed
  if (!w4s_ws_used(M, K)) return launch_w4s<64>(A, W, C, M, N, K, 0, 0, s, "zx_gemm_w4a8_ws");
  if (!workspace) return fail(ZX_ERR_NULL, "zx_gemm_w4a8_ws: null workspace");
  if (!aligned16(workspace)) return fail(ZX_ERR_ALIGN, "zx_gemm_w4a8_ws: workspace must be 16-byte aligned");
  if (M <= 16) return launch_w4s<16>(A, W, C, M, N, K, workspace, workspace_bytes, s, "zx_gemm_w4a8_ws");
  return launch_w4s<32>(A, W, C, M, N, K, workspace, workspace_bytes, s, "zx_gemm_w4a8_ws");
}

int zx_version(void) { return 100; }

int zx_set_kernel_policy(int policy) {
  t_err[0] = 0;
  if (policy < 0 || policy > 6)
    return fail(ZX_ERR_SHAPE, "zx_set_kernel_policy: policy %d not in {0, 1, 2, 3, 4, 5, 6}", policy);
  g_policy.store(policy);
  return 0;
}

const char* zx_last_error(void) { return t_err; }

const char* zx_last_kernel(void) { return t_kernel; }

int zx_gemm_s8(zx_devptr A, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
               int layout, zx_stream stream) {
  t_err[0] = 0;
  if (int rc = check_common(A, B, C, M, N, K, layout, 16, 4, 16, "zx_gemm_s8")) return rc;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (layout == ZX_LAYOUT_NT)
    return dispatch_gemm<zx::Kind::I8, false, zx::Out::S32>(A, B, C, nullptr, nullptr, M, N, K, s, "zx_gemm_s8");
  return dispatch_gemm<zx::Kind::I8, true, zx::Out::S32>(A, B, C, nullptr, nullptr, M, N, K, s, "zx_gemm_s8");
}

int zx_gemm_s8_mgpu(int ngpus, const int* devices, const zx_devptr* A, const zx_devptr* B, const zx_devptr* C,
                    uint32_t M, uint32_t N, uint32_t K, int layout, const zx_stream* streams) {
  t_err[0] = 0;
  const char* fn = "zx_gemm_s8_mgpu";
  if (ngpus < 1 || ngpus > kMaxDevices) return fail(ZX_ERR_SHAPE, "%s: ngpus=%d not in [1, %d]", fn, ngpus, kMaxDevices);
  if (!devices || !A || !B || !C) return fail(ZX_ERR_NULL, "%s: null device or buffer array", fn);
  if (M < static_cast<uint32_t>(ngpus))
    return fail(ZX_ERR_SHAPE, "%s: M=%u has fewer rows than the %d shards", fn, M, ngpus);
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  // validate every shard before launching any
  for (int i = 0; i < ngpus; ++i) {
    if (devices[i] < 0 || devices[i] >= count || devices[i] >= kMaxDevices)
      return fail(ZX_ERR_NO_DEVICE, "%s: shard %d names device %d (this process sees %d)", fn, i, devices[i], count);
    const uint32_t rows = static_cast<uint32_t>(uint64_t(M) * (i + 1) / ngpus - uint64_t(M) * i / ngpus);
    if (int rc = check_common(A[i], B[i], C[i], rows, N, K, layout, 16, 4, 16, fn)) return rc;
  }
  int prev = 0;
  if ((e = cudaGetDevice(&prev)) != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int rc = 0;
  for (int i = 0; i < ngpus && rc == 0; ++i) {
    if ((e = cudaSetDevice(devices[i])) != cudaSuccess) {
      rc = cuda_fail(e, "cudaSetDevice");
      break;
    }
    const uint32_t rows = static_cast<uint32_t>(uint64_t(M) * (i + 1) / ngpus - uint64_t(M) * i / ngpus);
    auto s = streams ? reinterpret_cast<cudaStream_t>(streams[i]) : nullptr;
    rc = layout == ZX_LAYOUT_NT
             ? dispatch_gemm<zx::Kind::I8, false, zx::Out::S32>(A[i], B[i], C[i], nullptr, nullptr, rows, N, K, s, fn)
             : dispatch_gemm<zx::Kind::I8, true, zx::Out::S32>(A[i], B[i], C[i], nullptr, nullptr, rows, N, K, s, fn);
  }
  if ((e = cudaSetDevice(prev)) != cudaSuccess && rc == 0) rc = cuda_fail(e, "cudaSetDevice(restore)");
  return rc;
}

int zx_gemm_s8_replicated(zx_devptr A, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                          const zx_devptr* peer_c, uint32_t npeers, zx_stream stream) {
  t_err[0] = 0;
  const char* fn = "zx_gemm_s8_replicated";
  if (int rc = check_common(A, B, C, M, N, K, ZX_LAYOUT_NT, 16, 4, 16, fn)) return rc;
  if (npeers > 7) return fail(ZX_ERR_SHAPE, "%s: %u peer buffers, at most 7", fn, npeers);
  if (npeers && !peer_c) return fail(ZX_ERR_NULL, "%s: null peer buffer list", fn);
  for (uint32_t i = 0; i < npeers; ++i) {
    if (!peer_c[i]) return fail(ZX_ERR_NULL, "%s: peer buffer %u is null", fn, i);
    if (!aligned16(peer_c[i])) return fail(ZX_ERR_ALIGN, "%s: peer buffer %u must be 16-byte aligned", fn, i);
  }
  // Every peer buffer must be mapped here and hold all M x N int32 outputs: a store past its end
  // would land in another allocation on another GPU.
  for (uint32_t i = 0; i < npeers; ++i) {
    uint64_t base = 0, size = 0;
    if (int rc = address_range(peer_c[i], &base, &size, fn)) return rc;
    if (int rc = check_reachable(peer_c[i], fn)) return rc;
    const uint64_t need = uint64_t(M) * N * 4u;
    if (peer_c[i] + need > base + size)
      return fail(ZX_ERR_SHAPE, "%s: peer buffer %u holds %llu bytes from its address, the output needs %llu", fn, i,
                  (unsigned long long)(base + size - peer_c[i]), (unsigned long long)need);
  }
  return launch_gemm2w<zx::Kind::I8, zx::Out::S32>(A, B, C, nullptr, nullptr, M, N, K,
                                                   reinterpret_cast<cudaStream_t>(stream), fn, peer_c, npeers);
}

int zx_gemm_s8_scaled_bf16(zx_devptr A, zx_devptr B, zx_devptr row_scale, zx_devptr col_scale,
                           zx_devptr C, uint32_t M, uint32_t N, uint32_t K, int layout,
                           zx_stream stream) {
  t_err[0] = 0;
  if (int rc = check_common(A, B, C, M, N, K, layout, 16, 8, 16, "zx_gemm_s8_scaled_bf16")) return rc;
  if (!row_scale || !col_scale)
    return fail(ZX_ERR_NULL, "zx_gemm_s8_scaled_bf16: null scale vector");
  if ((row_scale & 3u) || (col_scale & 3u))
    return fail(ZX_ERR_ALIGN, "zx_gemm_s8_scaled_bf16: scale vectors must be 4-byte aligned");
  auto s = reinterpret_cast<cudaStream_t>(stream);
  auto rs = reinterpret_cast<const float*>(row_scale);
  auto cs = reinterpret_cast<const float*>(col_scale);
  if (layout == ZX_LAYOUT_NT)
    return dispatch_gemm<zx::Kind::I8, false, zx::Out::BF16_SCALED>(A, B, C, rs, cs, M, N, K, s, "zx_gemm_s8_scaled_bf16");
  return dispatch_gemm<zx::Kind::I8, true, zx::Out::BF16_SCALED>(A, B, C, rs, cs, M, N, K, s, "zx_gemm_s8_scaled_bf16");
}

int zx_gemm_bf16(zx_devptr A, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                 int layout, zx_stream stream) {
  t_err[0] = 0;
  if (int rc = check_common(A, B, C, M, N, K, layout, 8, 4, 8, "zx_gemm_bf16")) return rc;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (layout == ZX_LAYOUT_NT)
    return dispatch_gemm<zx::Kind::BF16, false, zx::Out::F32>(A, B, C, nullptr, nullptr, M, N, K, s, "zx_gemm_bf16");
  return dispatch_gemm<zx::Kind::BF16, true, zx::Out::F32>(A, B, C, nullptr, nullptr, M, N, K, s, "zx_gemm_bf16");
}

int zx_gemm_f16(zx_devptr A, zx_devptr B, zx_devptr C, uint32_t M, uint32_t N, uint32_t K,
                int layout, zx_stream stream) {
  t_err[0] = 0;
  if (int rc = check_common(A, B, C, M, N, K, layout, 8, 4, 8, "zx_gemm_f16")) return rc;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  F16Call f16;
  if (layout == ZX_LAYOUT_NT)
    return dispatch_gemm<zx::Kind::BF16, false, zx::Out::F32>(A, B, C, nullptr, nullptr, M, N, K, s, "zx_gemm_f16");
  return dispatch_gemm<zx::Kind::BF16, true, zx::Out::F32>(A, B, C, nullptr, nullptr, M, N, K, s, "zx_gemm_f16");
}

int zx_gemm_s8_host(const void* A_host, const void* B_host, void* C_host, zx_devptr A_dev, zx_devptr B_dev,
                    zx_devptr C_dev, uint32_t M, uint32_t N, uint32_t K, zx_stream stream) {
  t_err[0] = 0;
  const char* fn = "zx_gemm_s8_host";
  if (!A_host || !B_host || !C_host) return fail(ZX_ERR_NULL, "%s: null host buffer", fn);
  if (int rc = check_common(A_dev, B_dev, C_dev, M, N, K, ZX_LAYOUT_NT, 16, 4, 16, fn)) return rc;
  return gemm_host_pipeline<zx::Kind::I8, zx::Out::S32>(A_host, B_host, C_host, A_dev, B_dev, C_dev, M, N, K, 1,
                                                        reinterpret_cast<cudaStream_t>(stream), fn);
}

int zx_gemm_bf16_host(const void* A_host, const void* B_host, void* C_host, zx_devptr A_dev, zx_devptr B_dev,
                      zx_devptr C_dev, uint32_t M, uint32_t N, uint32_t K, zx_stream stream) {
  t_err[0] = 0;
  const char* fn = "zx_gemm_bf16_host";
  if (!A_host || !B_host || !C_host) return fail(ZX_ERR_NULL, "%s: null host buffer", fn);
  if (int rc = check_common(A_dev, B_dev, C_dev, M, N, K, ZX_LAYOUT_NT, 8, 4, 8, fn)) return rc;
  return gemm_host_pipeline<zx::Kind::BF16, zx::Out::F32>(A_host, B_host, C_host, A_dev, B_dev, C_dev, M, N, K, 2,
                                                          reinterpret_cast<cudaStream_t>(stream), fn);
}

int zx_launch_imma_s8_ref(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, zx_stream stream) {
  t_err[0] = 0;
  if (!a || !b || !c) return fail(ZX_ERR_NULL, "zx_launch_imma_s8_ref: null buffer");
  if (n == 0 || n % 128 != 0) return fail(ZX_ERR_SHAPE, "error: imma_s8 requires n %% 128 == 0 (got %u)", n);
  if (!aligned16(a) || !aligned16(b) || !aligned16(c))
    return fail(ZX_ERR_ALIGN, "zx_launch_imma_s8_ref: buffers must be 16-byte aligned");
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  // the reference launch: grid (n/128, n/128), block 128, no dynamic smem (src/bench.zig:671-682)
  imma_s8_$_immaS8<<<dim3(n / 128, n / 128), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const int8_t*>(a), reinterpret_cast<const int8_t*>(b), reinterpret_cast<int32_t*>(c), n);
  note_kernel("imma_s8_$_immaS8 (reference launch contract)");
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : cuda_fail(e, "imma_s8_$_immaS8");
}

int zx_launch_hgemm_bf16_ref(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, zx_stream stream) {
  t_err[0] = 0;
  if (!a || !b || !c) return fail(ZX_ERR_NULL, "zx_launch_hgemm_bf16_ref: null buffer");
  if (n == 0 || n % 128 != 0) return fail(ZX_ERR_SHAPE, "error: hgemm_wgmma* requires n %% 128 == 0 (got %u)", n);
  if (!aligned16(a) || !aligned16(b) || !aligned16(c))
    return fail(ZX_ERR_ALIGN, "zx_launch_hgemm_bf16_ref: buffers must be 16-byte aligned");
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  // the reference launch: grid (n/128, n/64), block 128 (src/bench.zig:589-600)
  hgemm_wgmma_bf16_$_hgemmWgmmaBf16<<<dim3(n / 128, n / 64), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint16_t*>(a), reinterpret_cast<const uint16_t*>(b), reinterpret_cast<float*>(c), n);
  note_kernel("hgemm_wgmma_bf16_$_hgemmWgmmaBf16 (reference launch contract)");
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : cuda_fail(e, "hgemm_wgmma_bf16_$_hgemmWgmmaBf16");
}

namespace {
// Common checks of the reference-contract launchers: the reference bench's own n % 128 gate and
// message (src/bench.zig:96-124), null and alignment checks, a current B200.
int ref_launch_checks(std::initializer_list<zx_devptr> bufs, uint32_t n, const char* gate, const char* fn) {
  for (zx_devptr p : bufs)
    if (!p) return fail(ZX_ERR_NULL, "%s: null buffer", fn);
  if (n == 0 || n % 128 != 0) return fail(ZX_ERR_SHAPE, "error: %s requires n %% 128 == 0 (got %u)", gate, n);
  for (zx_devptr p : bufs)
    if (!aligned16(p)) return fail(ZX_ERR_ALIGN, "%s: buffers must be 16-byte aligned", fn);
  int dev = 0;
  DeviceInfo* di = nullptr;
  return current_device(&dev, &di);
}
int launched(const char* entry) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : cuda_fail(e, entry);
}
}  // namespace

// grid (n/128, n/128), block 128 (src/bench.zig:77, :800-811)
int zx_launch_imma_s4_ref(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, zx_stream stream) {
  t_err[0] = 0;
  if (int rc = ref_launch_checks({a, b, c}, n, "imma_s4", "zx_launch_imma_s4_ref")) return rc;
  imma_s4_$_immaS4<<<dim3(n / 128, n / 128), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint8_t*>(a), reinterpret_cast<const uint8_t*>(b), reinterpret_cast<int32_t*>(c), n);
  note_kernel("imma_s4_$_immaS4 (reference launch contract)");
  return launched("imma_s4_$_immaS4");
}

// grid (n/128, n/128), block 128 (src/bench.zig:1081-1092)
int zx_launch_imma_sp_s8_ref(zx_devptr a, zx_devptr b, zx_devptr meta, zx_devptr c, uint32_t n,
                             zx_stream stream) {
  t_err[0] = 0;
  if (int rc = ref_launch_checks({a, b, meta, c}, n, "imma_sp_s8", "zx_launch_imma_sp_s8_ref")) return rc;
  imma_sp_s8_$_immaSpS8<<<dim3(n / 128, n / 128), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const int8_t*>(a), reinterpret_cast<const int8_t*>(b),
      reinterpret_cast<const uint32_t*>(meta), reinterpret_cast<int32_t*>(c), n);
  note_kernel("imma_sp_s8_$_immaSpS8 (reference launch contract)");
  return launched("imma_sp_s8_$_immaSpS8");
}

// grid (n/128, n/128), block 128 (src/bench.zig:1237-1251)
int zx_launch_imma_sp_s4_ref(zx_devptr a, zx_devptr b, zx_devptr meta, zx_devptr c, uint32_t n,
                             zx_stream stream) {
  t_err[0] = 0;
  if (int rc = ref_launch_checks({a, b, meta, c}, n, "imma_sp_s4", "zx_launch_imma_sp_s4_ref")) return rc;
  imma_sp_s4_$_immaSpS4<<<dim3(n / 128, n / 128), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint8_t*>(a), reinterpret_cast<const uint8_t*>(b),
      reinterpret_cast<const uint32_t*>(meta), reinterpret_cast<int32_t*>(c), n);
  note_kernel("imma_sp_s4_$_immaSpS4 (reference launch contract)");
  return launched("imma_sp_s4_$_immaSpS4");
}

// hgemm_bf16 stem: 128 x 128 tiles, grid (n/128, n/128), block 128 (src/bench.zig:77-78)
int zx_launch_hgemm_bf16_mma_ref(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, zx_stream stream) {
  t_err[0] = 0;
  if (int rc = ref_launch_checks({a, b, c}, n, "hgemm_bf16", "zx_launch_hgemm_bf16_mma_ref")) return rc;
  hgemm_bf16_$_hgemmBf16<<<dim3(n / 128, n / 128), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint16_t*>(a), reinterpret_cast<const uint16_t*>(b), reinterpret_cast<float*>(c), n);
  note_kernel("hgemm_bf16_$_hgemmBf16 (reference launch contract)");
  return launched("hgemm_bf16_$_hgemmBf16");
}

// 64 x 128 tiles, grid (n/128, n/64), block 128 (src/bench.zig:1511-1522); the two descriptor
// addresses are passed through untouched
int zx_launch_hgemm_tma_ref(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, uint64_t desc_a,
                            uint64_t desc_b, zx_stream stream) {
  t_err[0] = 0;
  if (int rc = ref_launch_checks({a, b, c}, n, "hgemm_wgmma*", "zx_launch_hgemm_tma_ref")) return rc;
  hgemm_tma_$_hgemmTma<<<dim3(n / 128, n / 64), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint16_t*>(a), reinterpret_cast<const uint16_t*>(b), reinterpret_cast<float*>(c), n,
      desc_a, desc_b);
  note_kernel("hgemm_tma_$_hgemmTma (reference launch contract)");
  return launched("hgemm_tma_$_hgemmTma");
}

int zx_imma_s8(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, zx_stream stream) {
  t_err[0] = 0;
  if (n % 128 != 0) return fail(ZX_ERR_SHAPE, "error: imma_s8 requires n %% 128 == 0 (got %u)", n);
  return zx_gemm_s8(a, b, c, n, n, n, ZX_LAYOUT_NN, stream);
}

int zx_hgemm_bf16(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, zx_stream stream) {
  t_err[0] = 0;
  if (n % 128 != 0) return fail(ZX_ERR_SHAPE, "error: hgemm_wgmma* requires n %% 128 == 0 (got %u)", n);
  return zx_gemm_bf16(a, b, c, n, n, n, ZX_LAYOUT_NN, stream);
}

int zx_hgemm_tma(zx_devptr a, zx_devptr b, zx_devptr c, uint32_t n, uint64_t desc_a, uint64_t desc_b,
                 zx_stream stream) {
  t_err[0] = 0;
  (void)desc_a;
  (void)desc_b;
  if (n % 128 != 0) return fail(ZX_ERR_SHAPE, "error: hgemm_tma requires n %% 128 == 0 (got %u)", n);
  return zx_gemm_f16(a, b, c, n, n, n, ZX_LAYOUT_NN, stream);
}

int zx_device_status(uint32_t* code_out) {
  t_err[0] = 0;
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, zx::g_status, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "zx_device_status");
  if (code_out) *code_out = v;
  if (v != 0) return fail(ZX_ERR_TIMEOUT, "device wait gave up: status code %#x", v);
  return 0;
}

int zx_device_status_clear(void) {
  t_err[0] = 0;
  const unsigned int z = 0;
  cudaError_t e = cudaMemcpyToSymbol(zx::g_status, &z, sizeof(z));
  if (e != cudaSuccess) return cuda_fail(e, "zx_device_status_clear");
  return 0;
}

int zx_selftest_bounded_wait(zx_devptr out, uint32_t limit_us, zx_stream stream) {
  t_err[0] = 0;
  if (!out) return fail(ZX_ERR_NULL, "zx_selftest_bounded_wait: null output buffer");
  if (out & 3u) return fail(ZX_ERR_ALIGN, "zx_selftest_bounded_wait: output must be 4-byte aligned");
  if (limit_us == 0 || limit_us > 1000000u)
    return fail(ZX_ERR_SHAPE, "zx_selftest_bounded_wait: limit %u us not in [1, 1000000]", limit_us);
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (int rc = current_device(&dev, &di)) return rc;
  zx::selftest_wait_kernel<<<1, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<int32_t*>(out), uint64_t(limit_us) * 1000u);
  note_kernel("selftest_wait_kernel (bounded-wait self-test)");
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : cuda_fail(e, "zx_selftest_bounded_wait");
}

int zx_ipc_export(zx_devptr ptr, unsigned char handle_out[64], uint64_t* offset_out) {
  t_err[0] = 0;
  if (!ptr || !handle_out || !offset_out) return fail(ZX_ERR_NULL, "zx_ipc_export: null argument");
  uint64_t base = 0, size = 0;
  if (int rc = address_range(ptr, &base, &size, "zx_ipc_export")) return rc;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "zx_ipc_export: cudaIpcGetMemHandle");
  static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = ptr - base;
  return 0;
}

int zx_ipc_import(const unsigned char handle[64], zx_devptr* base_out) {
  t_err[0] = 0;
  if (!handle || !base_out) return fail(ZX_ERR_NULL, "zx_ipc_import: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "zx_ipc_import: cudaIpcOpenMemHandle");
  if (int rc = check_reachable(reinterpret_cast<uint64_t>(p), "zx_ipc_import")) {
    cudaIpcCloseMemHandle(p);
    return rc;
  }
  *base_out = reinterpret_cast<zx_devptr>(p);
  return 0;
}

int zx_ipc_close(zx_devptr base) {
  t_err[0] = 0;
  if (!base) return fail(ZX_ERR_NULL, "zx_ipc_close: null address");
  cudaError_t e = cudaIpcCloseMemHandle(reinterpret_cast<void*>(base));
  return e == cudaSuccess ? 0 : cuda_fail(e, "zx_ipc_close: cudaIpcCloseMemHandle");
}

int zx_device_sm_count(void) {
  int dev = 0;
  DeviceInfo* di = nullptr;
  if (current_device(&dev, &di)) return 0;
  return di->sm_count;
}

}  // extern "C"
