// zx_compat_cubin.cu — standalone module holding the reference-contract kernels of
// zx_compat.cuh (imma_s8_$_immaS8, imma_s4_$_immaS4, imma_sp_s8_$_immaSpS8, imma_sp_s4_$_immaSpS4,
// hgemm_bf16_$_hgemmBf16, hgemm_wgmma_bf16_$_hgemmWgmmaBf16, hgemm_tma_$_hgemmTma), built with
// `nvcc -cubin` into zoxide_b200/_build/<stem>.cubin: files the reference's `zoxide bench <path>`
// loads through cuModuleLoadData (its stem selects the harness, src/bench.zig:51-72) and
// launches by the mangled entry name (src/bench.zig:159-190).
#include "zx_compat.cuh"
