// Elementwise kernels of the vision tower (a Qwen3-VL-style ViT: patch embedding, learned position table resampled to
// the image grid, 2-D rotary attention blocks, 2x2 patch mergers). The tower's projections run on the tcgen05 GEMM
// with bias, GELU and the residual add in its epilogue, and its attention on the tcgen05 training-attention forward
// (bidirectional mode, heads padded to 128); these kernels do the rest, each in one pass over the rows:
//   vit_patch_pos   h = bf16(bf16(acc + b) + pos), acc the fp32 patch-embedding GEMM, pos the four-tap bilinear
//                   resample of the position table with bf16 products and bf16 running sums (the deployed
//                   interpolation's rounding)
//   vit_qkv_rope    q / k / v split per head from the bf16 QKV projection, 2-D rotary on q and k in fp32, written
//                   head-padded (zeros past the head dim)
//   vit_layernorm   y = LayerNorm(x) with fp32 statistics, rows of any width up to 5,120 (the post-shuffle norm of
//                   the deepstack mergers normalises four patches' rows as one)
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"

namespace afb {

namespace {
AFB_DEV float bf(float x) { return __bfloat162float(__float2bfloat16(x)); }

AFB_DEV float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

constexpr int LN_THREADS = 256, LN_PER = 20;  // rows up to 5,120 wide
}  // namespace

__global__ void vit_patch_pos_kernel(const float* __restrict__ acc, const __nv_bfloat16* __restrict__ bias,
                                     const __nv_bfloat16* __restrict__ table, const int* __restrict__ idx,
                                     const __nv_bfloat16* __restrict__ wts, __nv_bfloat16* __restrict__ h, int P,
                                     int C) {
  const int p = blockIdx.x;
  if (p >= P) return;
  const int i0 = idx[4 * p], i1 = idx[4 * p + 1], i2 = idx[4 * p + 2], i3 = idx[4 * p + 3];
  const float w0 = __bfloat162float(wts[4 * p]), w1 = __bfloat162float(wts[4 * p + 1]);
  const float w2 = __bfloat162float(wts[4 * p + 2]), w3 = __bfloat162float(wts[4 * p + 3]);
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float t0 = bf(__bfloat162float(table[(size_t)i0 * C + c]) * w0);
    const float t1 = bf(__bfloat162float(table[(size_t)i1 * C + c]) * w1);
    const float t2 = bf(__bfloat162float(table[(size_t)i2 * C + c]) * w2);
    const float t3 = bf(__bfloat162float(table[(size_t)i3 * C + c]) * w3);
    const float pos = bf(bf(bf(t0 + t1) + t2) + t3);
    const float x = bf(acc[(size_t)p * C + c] + __bfloat162float(bias[c]));
    h[(size_t)p * C + c] = __float2bfloat16(x + pos);
  }
}

// one block per patch; rotary pair (j, j + Dh / 2) of each head
__global__ void vit_qkv_rope_kernel(const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ cosv,
                                    const float* __restrict__ sinv, int P, int H, int Dh, int Dp,
                                    __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k,
                                    __nv_bfloat16* __restrict__ v) {
  const int p = blockIdx.x;
  if (p >= P) return;
  const int half = Dh / 2, W = H * Dh;
  const __nv_bfloat16* a = qkv + (size_t)p * 3 * W;
  for (int e = threadIdx.x; e < H * Dp; e += blockDim.x) {  // v, and the zero padding of all three
    const int hd = e / Dp, d = e - hd * Dp;
    const size_t o = (size_t)p * H * Dp + e;
    if (d >= Dh) {
      q[o] = k[o] = v[o] = __float2bfloat16(0.f);
    } else {
      v[o] = a[2 * W + hd * Dh + d];
    }
  }
  for (int e = threadIdx.x; e < H * half; e += blockDim.x) {
    const int hd = e / half, j = e - hd * half;
    const float c = cosv[(size_t)p * half + j], s = sinv[(size_t)p * half + j];
    const size_t o = (size_t)p * H * Dp + (size_t)hd * Dp;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      const int base = which * W + hd * Dh;
      const float x0 = __bfloat162float(a[base + j]), x1 = __bfloat162float(a[base + j + half]);
      __nv_bfloat16* dst = which ? k : q;
      dst[o + j] = __float2bfloat16(x0 * c - x1 * s);
      dst[o + j + half] = __float2bfloat16(x1 * c + x0 * s);
    }
  }
}

__global__ void __launch_bounds__(LN_THREADS) vit_layernorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                                   const __nv_bfloat16* __restrict__ w,
                                                                   const __nv_bfloat16* __restrict__ b, float eps,
                                                                   __nv_bfloat16* __restrict__ y, int C) {
  __shared__ float red[LN_THREADS / 32];
  const size_t r = blockIdx.x;
  float v[LN_PER];
  const int per = (C + LN_THREADS - 1) / LN_THREADS;
  float s = 0.f;
  for (int i = 0; i < per; ++i) {
    const int c = threadIdx.x + i * LN_THREADS;
    v[i] = c < C ? __bfloat162float(x[r * C + c]) : 0.f;
    s += v[i];
  }
  const float mean = block_sum(s, red) / (float)C;
  float q = 0.f;
  for (int i = 0; i < per; ++i) {
    const int c = threadIdx.x + i * LN_THREADS;
    if (c < C) q += (v[i] - mean) * (v[i] - mean);
  }
  const float rstd = rsqrtf(block_sum(q, red) / (float)C + eps);
  for (int i = 0; i < per; ++i) {
    const int c = threadIdx.x + i * LN_THREADS;
    if (c < C)
      y[r * C + c] = __float2bfloat16((v[i] - mean) * rstd * __bfloat162float(w[c]) + __bfloat162float(b[c]));
  }
}

int vit_patch_pos(const float* acc, const void* bias, const void* table, const int* idx, const void* wts, void* h,
                  int P, int C, cudaStream_t st) {
  if (P <= 0) return 0;
  vit_patch_pos_kernel<<<P, 256, 0, st>>>(acc, (const __nv_bfloat16*)bias, (const __nv_bfloat16*)table, idx,
                                          (const __nv_bfloat16*)wts, (__nv_bfloat16*)h, P, C);
  return (int)cudaGetLastError();
}

int vit_qkv_rope(const void* qkv, const float* cosv, const float* sinv, int P, int H, int Dh, int Dp, void* q,
                 void* k, void* v, cudaStream_t st) {
  if (Dh % 2 || Dh > Dp) return 3;
  if (P <= 0) return 0;
  vit_qkv_rope_kernel<<<P, 256, 0, st>>>((const __nv_bfloat16*)qkv, cosv, sinv, P, H, Dh, Dp, (__nv_bfloat16*)q,
                                         (__nv_bfloat16*)k, (__nv_bfloat16*)v);
  return (int)cudaGetLastError();
}

int vit_layernorm(const void* x, const void* w, const void* b, float eps, void* y, int rows, int C, cudaStream_t st) {
  if (C > LN_THREADS * LN_PER || C < 1) return 3;
  if (rows <= 0) return 0;
  vit_layernorm_kernel<<<rows, LN_THREADS, 0, st>>>((const __nv_bfloat16*)x, (const __nv_bfloat16*)w,
                                                    (const __nv_bfloat16*)b, eps, (__nv_bfloat16*)y, C);
  return (int)cudaGetLastError();
}

}  // namespace afb
