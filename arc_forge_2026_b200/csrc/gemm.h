// Host-side declarations of the GEMM launchers (raw pointers + stream; no torch headers).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace afb {

struct GemmEpilogue {
  void* out = nullptr;             // [M, ldo] bf16 or fp32
  int ldo = 0;
  int out_fp32 = 0;
  const void* residual = nullptr;  // optional bf16 [M, ldr] added after alpha
  int ldr = 0;
  float alpha = 1.f;
  void* partial = nullptr;         // split-K scratch: fp32 [splits, M, N]
};

struct GemmPlan {
  int bn = 128;
  int splits = 1;
};

GemmPlan plan_gemm(int M, int N, int K, int num_sms);
int gemm_bf16_tn(const void* A, int lda, const void* B, int ldb, int M, int N, int K, const GemmEpilogue& epi, int bn,
                 int splits, uint32_t* status, cudaStream_t stream);
int make_tmap_2d(CUtensorMap* map, const void* base, int dtype_bytes, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, int swizzle128);

}  // namespace afb
