// Host-callable launchers of the non-GEMM kernels (raw device pointers + stream; no torch headers).
// Every launcher returns 0 on success, 3 for an unsupported shape, or a cudaError_t code.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace afb {

// elementwise.cu
int rmsnorm(const void* x, void* residual, const void* w, void* y, int rows, int H, float eps, int zero_centered,
            cudaStream_t st);
int qk_norm_rope_store(const void* qkv, int T, int Hq, int Hkv, int D, int rot, const void* qw, const void* kw,
                       const int* positions, const int* slots, const float* cos_t, const float* sin_t, float eps,
                       void* q_out, void* kcache, void* vcache, int page_size, cudaStream_t st);
int router_topk(const float* logits, int ld, int T, int E, int k, int renorm, int* ids, float* weights,
                cudaStream_t st);
int expert_sort(const int* ids, int n, int E, const int* expert_map, int* offsets, int* row_token, int* row_entry,
                int* entry_row, int k, cudaStream_t st);
int quant_rows_e4m3(const void* x, int ldx, const int* row_token, const int* nrows_dev, int nrows, int K, void* q,
                    float* scales, cudaStream_t st);
int moe_combine(const void* y, const int* entry_row, int k, const void* shared, const float* router_logits,
                int ld_logits, int sg_col, const void* resid, void* out, int T, int H, cudaStream_t st);
int swiglu(const void* x, void* y, int T, int I, cudaStream_t st);
int embedding(const int* ids, const void* table, void* out, int T, int H, int V, uint32_t* status, cudaStream_t st);

}  // namespace afb
