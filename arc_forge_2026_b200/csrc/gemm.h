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
  const void* bias = nullptr;      // optional bf16 [N], added after alpha (before the activation and the residual)
  int act = 0;                     // 0 none, 1 tanh-GELU, 2 erf-GELU (applied to alpha * acc + bias)
  void* partial = nullptr;         // split-K scratch: fp32 [splits, M, N]
};

// Grouped GEMMs (the experts of a MoE layer), two forms:
//  ROWS (mode 1):   C[r, :] = A[r, :] @ B_e^T for the rows r of group e: rows [seg[e], seg[e+1]) of A, B_e = rows
//                   [e * group_rows, (e + 1) * group_rows) of B. tiles[e] = sum over groups before e of
//                   ceil(rows / 128) (prefix over E + 1 entries); the grid covers an upper bound, surplus CTAs exit.
//  REDUCE (mode 2): C_e = A[:, seg[e]:seg[e+1]] @ B[:, seg[e]:seg[e+1]]^T, written at C + e * group_out_stride;
//                   seg entries are multiples of 64 (the K block), so no block mixes two groups.
struct GemmGroups {
  int mode = 0;
  const int* seg = nullptr;     // [E + 1]
  const int* tiles = nullptr;   // [E + 1] (ROWS)
  int E = 0;
  int group_rows = 0;           // ROWS: rows of B per group; REDUCE: rows of A (= rows of each C_e)
  int64_t group_out_stride = 0; // REDUCE: elements between consecutive C_e
};

struct GemmPlan {
  int bn = 128;
  int splits = 1;
};

GemmPlan plan_gemm(int M, int N, int K, int num_sms);
int gemm_bf16_tn(const void* A, int lda, const void* B, int ldb, int M, int N, int K, const GemmEpilogue& epi, int bn,
                 int splits, uint32_t* status, cudaStream_t stream);
int gemm_bf16_grouped(const void* A, int lda, int rows_a, const void* B, int ldb, int rows_b, int N, int K,
                      const GemmEpilogue& epi, const GemmGroups& g, int max_tiles, uint32_t* status,
                      cudaStream_t stream);
int make_tmap_2d(CUtensorMap* map, const void* base, int dtype_bytes, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, int swizzle128);
// bf16, 128-byte swizzle: dims / box innermost first, strides of dims 1 and 2 in bytes
int make_tmap_3d_bf16(CUtensorMap* map, const void* base, const uint64_t dims[3], const uint64_t strides_bytes[2],
                      const uint32_t box[3]);

}  // namespace afb
