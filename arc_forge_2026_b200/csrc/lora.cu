// LoRA adapter products on the tensor cores without fp32 copies of the activations (the reference's fused LoRA
// gradients, training/work/qwen38fn_lora/lora_grad.py:1-14).
//
//   rows_times(P, W)  out[t, j] = sum_k P[t, k] W[j, k]      P bf16 [T, K] (big), W fp32 [R, K] (small)
//   tgrad(P, Q)       out[m, j] = sum_t P[t, m] Q[t, j]      P bf16 [T, M] (big), Q fp32 [T, R] (small)
//
// The adapter's forward is s = x A^T (rows_times) and its backward dB = dY^T s, dA = (dY B)^T x (tgrad), ds = dY B
// (rows_times). The big operand is read once in bf16; the small fp32 operand is split per element into bf16
// hi = bf16(v) and lo = bf16(v - hi) (hi + lo = v to ~2^-16), so one bf16 MMA over [hi | lo] with fp32
// accumulation keeps fp32-level accuracy: out = acc_hi + acc_lo. m16n8k16 tiles (mma.sync) from padded shared
// memory: both products are read-bound (R <= 64 columns per byte of P), so the legacy tensor path is not the limit.
// tgrad splits T over CTAs and sums the split partials in split order (bitwise reproducible).
#include "common.cuh"
#include "kernels.h"

namespace afb {
namespace lorad {
using bf16 = __nv_bfloat16;
constexpr int BT = 128, BK = 64;  // rows_times: 128 rows x 64-wide K blocks
constexpr int PK = BK + 8;         // padded pitch (elements) of [*, 64] tiles
constexpr int PM = 128 + 8;        // padded pitch of the [64, 128] tgrad tile

AFB_DEV void split_hi_lo(float v, bf16& hi, bf16& lo) {
  hi = __float2bfloat16_rn(v);
  lo = __float2bfloat16_rn(v - __bfloat162float(hi));
}

template <int R>
__global__ void __launch_bounds__(256) rows_times_kernel(const bf16* __restrict__ P, int64_t ldp,
                                                          const float* __restrict__ W, int T, int K,
                                                          float* __restrict__ out) {
  __shared__ __align__(16) bf16 Ps[BT * PK];
  __shared__ __align__(16) bf16 Ws[2 * R * PK];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * BT;
  constexpr int NT = 2 * R / 8;  // n-tiles over [hi | lo]
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  for (int k0 = 0; k0 < K; k0 += BK) {
    __syncthreads();
    for (int c = threadIdx.x; c < BT * (BK / 8); c += blockDim.x) {  // P tile: 16-byte chunks
      const int r = c / (BK / 8), cc = c % (BK / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (t0 + r < T && k0 + cc * 8 < K) v = *reinterpret_cast<const uint4*>(P + (size_t)(t0 + r) * ldp + k0 + cc * 8);
      *reinterpret_cast<uint4*>(Ps + r * PK + cc * 8) = v;
    }
    for (int i = threadIdx.x; i < R * BK; i += blockDim.x) {  // W block -> hi / lo rows
      const int j = i / BK, kk = i % BK;
      const float v = k0 + kk < K ? W[(size_t)j * K + k0 + kk] : 0.f;
      bf16 hi, lo;
      split_hi_lo(v, hi, lo);
      Ws[j * PK + kk] = hi;
      Ws[(R + j) * PK + kk] = lo;
    }
    __syncthreads();
    const uint32_t pbase = smem_u32(Ps), wbase = smem_u32(Ws);
#pragma unroll
    for (int ks = 0; ks < BK / 16; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(pbase + ((warp * 16 + (lane & 15)) * PK + ks * 16 + (lane >> 4) * 8) * 2, a0, a1, a2, a3);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t b0, b1, b2, b3;
        const int n = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        ldsm_x4(wbase + (n * PK + ks * 16 + ((lane >> 3) & 1) * 8) * 2, b0, b1, b2, b3);
        mma_bf16(acc[2 * np], a0, a1, a2, a3, b0, b1);
        mma_bf16(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }
  const int r0 = t0 + warp * 16 + (lane >> 2);
#pragma unroll
  for (int j = 0; j < R / 8; ++j) {
    const int col = j * 8 + (lane & 3) * 2;
    if (r0 < T) {
      out[(size_t)r0 * R + col] = acc[j][0] + acc[j + R / 8][0];
      out[(size_t)r0 * R + col + 1] = acc[j][1] + acc[j + R / 8][1];
    }
    if (r0 + 8 < T) {
      out[(size_t)(r0 + 8) * R + col] = acc[j][2] + acc[j + R / 8][2];
      out[(size_t)(r0 + 8) * R + col + 1] = acc[j][3] + acc[j + R / 8][3];
    }
  }
}

template <int R>
__global__ void __launch_bounds__(256) tgrad_kernel(const bf16* __restrict__ P, int64_t ldp,
                                                     const float* __restrict__ Q, int T, int M, int rows_per_split,
                                                     float* __restrict__ part) {
  __shared__ __align__(16) bf16 Ps[BK * PM];     // [64 t][128 m]
  __shared__ __align__(16) bf16 Qs[2 * R * PK];  // [hi | lo][64 t]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * 128;
  const int tb = blockIdx.y * rows_per_split, te = min(T, tb + rows_per_split);
  constexpr int NT = 2 * R / 8;
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  for (int t0 = tb; t0 < te; t0 += BK) {
    __syncthreads();
    for (int c = threadIdx.x; c < BK * 16; c += blockDim.x) {  // P tile: 64 t x 128 m
      const int r = c / 16, cc = c % 16;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (t0 + r < te && m0 + cc * 8 < M) v = *reinterpret_cast<const uint4*>(P + (size_t)(t0 + r) * ldp + m0 + cc * 8);
      *reinterpret_cast<uint4*>(Ps + r * PM + cc * 8) = v;
    }
    for (int i = threadIdx.x; i < BK * R; i += blockDim.x) {  // Q block (t-major) -> transposed hi / lo rows
      const int tt = i / R, j = i % R;
      const float v = t0 + tt < te ? Q[(size_t)(t0 + tt) * R + j] : 0.f;
      bf16 hi, lo;
      split_hi_lo(v, hi, lo);
      Qs[j * PK + tt] = hi;
      Qs[(R + j) * PK + tt] = lo;
    }
    __syncthreads();
    const uint32_t pbase = smem_u32(Ps), qbase = smem_u32(Qs);
#pragma unroll
    for (int ks = 0; ks < BK / 16; ++ks) {
      uint32_t a0, a1, a2, a3;  // A[m][t] from the [t][m] tile: transposed 8x8 loads
      const int k = ks * 16 + (lane & 7) + ((lane >> 4) << 3);
      const int m = warp * 16 + ((lane >> 3) & 1) * 8;
      ldsm_x4_t(pbase + (k * PM + m) * 2, a0, a1, a2, a3);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t b0, b1, b2, b3;
        const int n = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        ldsm_x4(qbase + (n * PK + ks * 16 + ((lane >> 3) & 1) * 8) * 2, b0, b1, b2, b3);
        mma_bf16(acc[2 * np], a0, a1, a2, a3, b0, b1);
        mma_bf16(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }
  const int r0 = m0 + warp * 16 + (lane >> 2);
  float* dst = part + (size_t)blockIdx.y * M * R;
#pragma unroll
  for (int j = 0; j < R / 8; ++j) {
    const int col = j * 8 + (lane & 3) * 2;
    if (r0 < M) {
      dst[(size_t)r0 * R + col] = acc[j][0] + acc[j + R / 8][0];
      dst[(size_t)r0 * R + col + 1] = acc[j][1] + acc[j + R / 8][1];
    }
    if (r0 + 8 < M) {
      dst[(size_t)(r0 + 8) * R + col] = acc[j][2] + acc[j + R / 8][2];
      dst[(size_t)(r0 + 8) * R + col + 1] = acc[j][3] + acc[j + R / 8][3];
    }
  }
}

__global__ void sum_splits_kernel(const float* __restrict__ part, int splits, int64_t n, float* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < splits; ++k) s += part[(size_t)k * n + i];  // split order: reproducible
    out[i] = s;
  }
}
}  // namespace lorad

int lora_rows_times(const void* P, int64_t ldp, const float* W, int T, int K, int R, float* out, cudaStream_t st) {
  if (T <= 0) return 0;
  if (K % 8 || ldp % 8) return 3;
  const unsigned grid = (T + lorad::BT - 1) / lorad::BT;
  const auto* p = reinterpret_cast<const __nv_bfloat16*>(P);
  switch (R) {
    case 8: lorad::rows_times_kernel<8><<<grid, 256, 0, st>>>(p, ldp, W, T, K, out); break;
    case 16: lorad::rows_times_kernel<16><<<grid, 256, 0, st>>>(p, ldp, W, T, K, out); break;
    case 32: lorad::rows_times_kernel<32><<<grid, 256, 0, st>>>(p, ldp, W, T, K, out); break;
    case 64: lorad::rows_times_kernel<64><<<grid, 256, 0, st>>>(p, ldp, W, T, K, out); break;
    default: return 3;
  }
  return (int)cudaGetLastError();
}

int lora_tgrad(const void* P, int64_t ldp, const float* Q, int T, int M, int R, int splits, float* part, float* out,
               cudaStream_t st) {
  if (M % 8 || ldp % 8 || splits < 1) return 3;
  const int rps = ((T + splits - 1) / splits + lorad::BK - 1) / lorad::BK * lorad::BK;
  dim3 grid((M + 127) / 128, splits);
  const auto* p = reinterpret_cast<const __nv_bfloat16*>(P);
  switch (R) {
    case 8: lorad::tgrad_kernel<8><<<grid, 256, 0, st>>>(p, ldp, Q, T, M, rps, part); break;
    case 16: lorad::tgrad_kernel<16><<<grid, 256, 0, st>>>(p, ldp, Q, T, M, rps, part); break;
    case 32: lorad::tgrad_kernel<32><<<grid, 256, 0, st>>>(p, ldp, Q, T, M, rps, part); break;
    case 64: lorad::tgrad_kernel<64><<<grid, 256, 0, st>>>(p, ldp, Q, T, M, rps, part); break;
    default: return 3;
  }
  int rc = (int)cudaGetLastError();
  if (rc) return rc;
  const int64_t n = (int64_t)M * R;
  const int64_t blocks = (n + 255) / 256;
  lorad::sum_splits_kernel<<<(unsigned)(blocks < 148 * 8 ? blocks : 148 * 8), 256, 0, st>>>(part, splits, n, out);
  return (int)cudaGetLastError();
}
}  // namespace afb
