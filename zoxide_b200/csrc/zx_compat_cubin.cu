// zx_compat_cubin.cu — standalone module holding the reference-contract kernels
// (imma_s8_$_immaS8, hgemm_wgmma_bf16_$_hgemmWgmmaBf16), built with `nvcc -cubin` into
// zoxide_b200/_build/imma_s8.cubin and hgemm_wgmma_bf16.cubin: files the reference's
// `zoxide bench <path>` loads through cuModuleLoadData (its stem selects the harness,
// src/bench.zig:51-72) and launches by the mangled entry name (src/bench.zig:159-190).
#include "zx_compat.cuh"
