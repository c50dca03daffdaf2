// Fused element-wise / row-wise training ops of the QAD student, forward and backward, each one pass over its
// tensors (the reference's fused Triton training kernels: trainer_kernels.py GatedRMSNormFLA, int3_moe.py
// _swiglu_bf16 / token aggregation, fp8_moe.py _swiglu_backward / _routing_backward; here CUDA, bf16 I/O with fp32
// math, every reduction in a fixed order so gradients are bitwise reproducible).
//
//   conv_silu     y = silu(sum_k w[c][k] x[t-3+k][c])         causal depthwise conv (kernel 4) + SiLU; the input
//                                                             may be a strided view (the conv channels of in_proj)
//   rmsnorm       y = x * rstd * (1 + w)                      zero-centred RMSNorm (frozen w), rstd saved
//   gated_rmsnorm y = x * rstd * w * silu(z)                  GDN output norm (frozen w)
//   swiglu        h = silu(g) * u over [rows, 2I] = [g | u]
//   moe_combine   out[t] = sum_k w[t,k] y[inv[t*K+k]]         routed rows back to tokens, weighted (no permuted copy)
//   dispatch_bwd  dx[t] = sum_k dxs[inv[t*K+k]]               gradient of the token -> routed-row gather
#include "common.cuh"
#include "kernels.h"

namespace afb {
namespace tfu {
using bf16 = __nv_bfloat16;
AFB_DEV void unpack8(const uint4& v, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(h[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}
AFB_DEV uint4 pack8(const float* f) {
  uint4 o;
  o.x = pack_bf16x2(f[0], f[1]);
  o.y = pack_bf16x2(f[2], f[3]);
  o.z = pack_bf16x2(f[4], f[5]);
  o.w = pack_bf16x2(f[6], f[7]);
  return o;
}
AFB_DEV float sigmoidf(float x) { return 1.f / (1.f + __expf(-x)); }
constexpr int RUN = 64;  // tokens per thread in the conv kernels
}  // namespace tfu
using namespace tfu;

// ------------------------------------------------------------------------------------------------ conv + SiLU
// thread: 8 channels x RUN tokens of one sequence, sliding window over the 3 previous inputs
// pos (optional, [B * T]): position of each token inside its packed sequence; taps before the sequence start read 0
__global__ void __launch_bounds__(256) conv_silu_fwd_kernel(const bf16* __restrict__ x, int64_t ldx,
                                                            const float* __restrict__ w, bf16* __restrict__ y, int B,
                                                            int T, int Cc, const int* __restrict__ pos) {
  const int groups = Cc / 8, tiles = (T + RUN - 1) / RUN;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)B * tiles * groups) return;
  const int cg = (int)(idx % groups), tile = (int)(idx / groups % tiles), b = (int)(idx / groups / tiles);
  const int c0 = cg * 8, t0 = tile * RUN;
  float wk[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 v = reinterpret_cast<const float4*>(w)[c0 + i];
    wk[i][0] = v.x;
    wk[i][1] = v.y;
    wk[i][2] = v.z;
    wk[i][3] = v.w;
  }
  float win[3][8];  // x[t-3], x[t-2], x[t-1]
#pragma unroll
  for (int s = 0; s < 3; ++s) {
    const int t = t0 - 3 + s;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t >= 0) v = *reinterpret_cast<const uint4*>(x + ((int64_t)b * T + t) * ldx + c0);
    unpack8(v, win[s]);
  }
  const int t1 = min(T, t0 + RUN);
  for (int t = t0; t < t1; ++t) {
    float cur[8], out[8];
    unpack8(*reinterpret_cast<const uint4*>(x + ((int64_t)b * T + t) * ldx + c0), cur);
    const int ps = pos ? pos[(int64_t)b * T + t] : 3;
    const float m0 = ps >= 3 ? 1.f : 0.f, m1 = ps >= 2 ? 1.f : 0.f, m2 = ps >= 1 ? 1.f : 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float p = m0 * wk[i][0] * win[0][i] + m1 * wk[i][1] * win[1][i] + m2 * wk[i][2] * win[2][i] +
                      wk[i][3] * cur[i];
      out[i] = p * sigmoidf(p);
      win[0][i] = win[1][i];
      win[1][i] = win[2][i];
      win[2][i] = cur[i];
    }
    *reinterpret_cast<uint4*>(y + ((int64_t)b * T + t) * Cc + c0) = pack8(out);
  }
}

// dx[t] = sum_k w[k] dpre[t+3-k],  dpre = dy * silu'(pre): the thread recomputes pre for its tokens and the 3 after
__global__ void __launch_bounds__(256) conv_silu_bwd_kernel(const bf16* __restrict__ x, int64_t ldx,
                                                            const float* __restrict__ w, const bf16* __restrict__ dy,
                                                            bf16* __restrict__ dx, int B, int T, int Cc,
                                                            const int* __restrict__ pos) {
  const int groups = Cc / 8, tiles = (T + RUN - 1) / RUN;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)B * tiles * groups) return;
  const int cg = (int)(idx % groups), tile = (int)(idx / groups % tiles), b = (int)(idx / groups / tiles);
  const int c0 = cg * 8, t0 = tile * RUN;
  float wk[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 v = reinterpret_cast<const float4*>(w)[c0 + i];
    wk[i][0] = v.x;
    wk[i][1] = v.y;
    wk[i][2] = v.z;
    wk[i][3] = v.w;
  }
  float win[3][8], dp[3][8];  // x[s-3..s-1]; dpre[s-3..s-1]
  int pw[3] = {3, 3, 3};      // positions of s-3..s-1 (with pos: the taps of those outputs that are live)
#pragma unroll
  for (int s = 0; s < 3; ++s) {
    const int t = t0 - 3 + s;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t >= 0) v = *reinterpret_cast<const uint4*>(x + ((int64_t)b * T + t) * ldx + c0);
    unpack8(v, win[s]);
#pragma unroll
    for (int i = 0; i < 8; ++i) dp[s][i] = 0.f;
  }
  const int s1 = min(T, t0 + RUN) + 3;  // dpre needed up to t1 + 2
  for (int s = t0; s < s1; ++s) {
    float cur[8], g[8], dcur[8];
    uint4 xv = make_uint4(0, 0, 0, 0), gv = make_uint4(0, 0, 0, 0);
    if (s < T) {
      xv = *reinterpret_cast<const uint4*>(x + ((int64_t)b * T + s) * ldx + c0);
      gv = *reinterpret_cast<const uint4*>(dy + ((int64_t)b * T + s) * Cc + c0);
    }
    unpack8(xv, cur);
    unpack8(gv, g);
    const int ps = (pos && s < T) ? pos[(int64_t)b * T + s] : 3;
    const float m0 = ps >= 3 ? 1.f : 0.f, m1 = ps >= 2 ? 1.f : 0.f, m2 = ps >= 1 ? 1.f : 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float p = m0 * wk[i][0] * win[0][i] + m1 * wk[i][1] * win[1][i] + m2 * wk[i][2] * win[2][i] +
                      wk[i][3] * cur[i];
      const float sg = sigmoidf(p);
      dcur[i] = g[i] * sg * (1.f + p * (1.f - sg));
    }
    if (s >= t0 + 3) {  // dx[s-3] complete: output s-3+j used x[s-3] through tap 3-j when its position >= j
      const float a1 = pw[1] >= 1 ? 1.f : 0.f, a2 = pw[2] >= 2 ? 1.f : 0.f;
      float out[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        out[i] = wk[i][3] * dp[0][i] + a1 * wk[i][2] * dp[1][i] + a2 * wk[i][1] * dp[2][i] + m0 * wk[i][0] * dcur[i];
      *reinterpret_cast<uint4*>(dx + ((int64_t)b * T + s - 3) * Cc + c0) = pack8(out);
    }
    pw[0] = pw[1];
    pw[1] = pw[2];
    pw[2] = ps;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      win[0][i] = win[1][i];
      win[1][i] = win[2][i];
      win[2][i] = cur[i];
      dp[0][i] = dp[1][i];
      dp[1][i] = dp[2][i];
      dp[2][i] = dcur[i];
    }
  }
}

int conv_silu_fwd(const void* x, int64_t ldx, const float* w, void* y, int B, int T, int Cc, const int* pos,
                  cudaStream_t st) {
  if (Cc % 8 || ldx % 8 || B < 1 || T < 1) return 3;
  const int64_t n = (int64_t)B * ((T + RUN - 1) / RUN) * (Cc / 8);
  conv_silu_fwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((const bf16*)x, ldx, w, (bf16*)y, B, T, Cc, pos);
  return (int)cudaGetLastError();
}
int conv_silu_bwd(const void* x, int64_t ldx, const float* w, const void* dy, void* dx, int B, int T, int Cc,
                  const int* pos, cudaStream_t st) {
  if (Cc % 8 || ldx % 8 || B < 1 || T < 1) return 3;
  const int64_t n = (int64_t)B * ((T + RUN - 1) / RUN) * (Cc / 8);
  conv_silu_bwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((const bf16*)x, ldx, w, (const bf16*)dy,
                                                                    (bf16*)dx, B, T, Cc, pos);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ RMSNorms
// one warp per row of H; lane slice p of a row: 8 interleaved elements (H >= 256) or 4 contiguous (H = 128)
template <int H>
struct Lanes {
  static constexpr int E = H / 32, W = E >= 8 ? 8 : E, NV = E / W;
  AFB_DEV static int col(int p, int lane) { return E >= 8 ? (p * 32 + lane) * 8 : lane * E; }
};
template <int W>
AFB_DEV void ld_chunk(const bf16* p, float* f) {
  if constexpr (W == 8) {
    unpack8(*reinterpret_cast<const uint4*>(p), f);
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
  }
}
template <int W>
AFB_DEV void st_chunk(bf16* p, const float* f) {
  if constexpr (W == 8) {
    *reinterpret_cast<uint4*>(p) = pack8(f);
  } else {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]));
  }
}
AFB_DEV int64_t row_off(const RowMap& m, int64_t r) { return (r / m.inner) * m.ld_outer + (r % m.inner) * m.ld_inner; }

template <int H>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const bf16* __restrict__ x, RowMap mx,
                                                          const bf16* __restrict__ z, RowMap mz,
                                                          const float* __restrict__ w, float eps,
                                                          bf16* __restrict__ y, float* __restrict__ rstd, int64_t rows) {
  using L = Lanes<H>;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const bool gated = z != nullptr;
  const bf16* xr = x + row_off(mx, row);
  float v[L::NV][L::W];
  float ss = 0.f;
#pragma unroll
  for (int p = 0; p < L::NV; ++p) {
    ld_chunk<L::W>(xr + L::col(p, lane), v[p]);
#pragma unroll
    for (int i = 0; i < L::W; ++i) ss += v[p][i] * v[p][i];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / H + eps);
  if (lane == 0) rstd[row] = r;
#pragma unroll
  for (int p = 0; p < L::NV; ++p) {
    const int c = L::col(p, lane);
    float zf[L::W], o[L::W];
    if (gated) ld_chunk<L::W>(z + row_off(mz, row) + c, zf);
#pragma unroll
    for (int i = 0; i < L::W; ++i) {
      const float wi = w[c + i];
      o[i] = gated ? v[p][i] * r * wi * (zf[i] * sigmoidf(zf[i])) : v[p][i] * r * (1.f + wi);
    }
    st_chunk<L::W>(y + row * H + c, o);
  }
}

// dx = rstd (u - xh mean(u xh)), u = m dy with m = (1 + w) or w silu(z); gated: dz = dy xh w silu'(z)
template <int H>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const bf16* __restrict__ x, RowMap mx,
                                                          const bf16* __restrict__ z, RowMap mz,
                                                          const float* __restrict__ w, const float* __restrict__ rstd,
                                                          const bf16* __restrict__ dy, bf16* __restrict__ dx,
                                                          bf16* __restrict__ dz, int64_t rows) {
  using L = Lanes<H>;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const bool gated = z != nullptr;
  const float r = rstd[row];
  const bf16* xr = x + row_off(mx, row);
  float xh[L::NV][L::W], u[L::NV][L::W];
  float dot = 0.f;
#pragma unroll
  for (int p = 0; p < L::NV; ++p) {
    const int c = L::col(p, lane);
    float g[L::W], zf[L::W], dzv[L::W];
    ld_chunk<L::W>(xr + c, xh[p]);
    ld_chunk<L::W>(dy + row * H + c, g);
    if (gated) ld_chunk<L::W>(z + row_off(mz, row) + c, zf);
#pragma unroll
    for (int i = 0; i < L::W; ++i) {
      const float wi = w[c + i];
      xh[p][i] *= r;
      if (gated) {
        const float sg = sigmoidf(zf[i]);
        u[p][i] = g[i] * wi * zf[i] * sg;
        dzv[i] = g[i] * xh[p][i] * wi * sg * (1.f + zf[i] * (1.f - sg));
      } else {
        u[p][i] = g[i] * (1.f + wi);
      }
      dot += u[p][i] * xh[p][i];
    }
    if (gated) st_chunk<L::W>(dz + row * H + c, dzv);
  }
  dot = warp_sum(dot) / H;
#pragma unroll
  for (int p = 0; p < L::NV; ++p) {
    float o[L::W];
#pragma unroll
    for (int i = 0; i < L::W; ++i) o[i] = r * (u[p][i] - xh[p][i] * dot);
    st_chunk<L::W>(dx + row * H + L::col(p, lane), o);
  }
}

#define AFB_RMS_H(X) X(128) X(256) X(512) X(1024) X(2048)

int rmsnorm_train_fwd(const void* x, RowMap mx, const void* z, RowMap mz, const float* w, float eps, void* y,
                      float* rstd, int64_t rows, int H, cudaStream_t st) {
  if (rows < 1) return 0;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  switch (H) {
#define X(h)                                                                                                   \
  case h:                                                                                                      \
    rmsnorm_fwd_kernel<h><<<grid, 256, 0, st>>>((const bf16*)x, mx, (const bf16*)z, mz, w, eps, (bf16*)y, rstd, \
                                                rows);                                                         \
    break;
    AFB_RMS_H(X)
#undef X
    default:
      return 3;
  }
  return (int)cudaGetLastError();
}
int rmsnorm_train_bwd(const void* x, RowMap mx, const void* z, RowMap mz, const float* w, const float* rstd,
                      const void* dy, void* dx, void* dz, int64_t rows, int H, cudaStream_t st) {
  if (rows < 1) return 0;
  if (z && !dz) return 3;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  switch (H) {
#define X(h)                                                                                                     \
  case h:                                                                                                        \
    rmsnorm_bwd_kernel<h><<<grid, 256, 0, st>>>((const bf16*)x, mx, (const bf16*)z, mz, w, rstd, (const bf16*)dy, \
                                                (bf16*)dx, (bf16*)dz, rows);                                     \
    break;
    AFB_RMS_H(X)
#undef X
    default:
      return 3;
  }
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ SwiGLU
__global__ void __launch_bounds__(256) swiglu_fwd_kernel(const bf16* __restrict__ gu, bf16* __restrict__ h,
                                                         int64_t rows, int I) {
  const int v8 = I / 8;
  const int64_t n = rows * v8;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = q / v8;
    const int c = (int)(q % v8) * 8;
    float g[8], u[8], o[8];
    unpack8(*reinterpret_cast<const uint4*>(gu + r * 2 * I + c), g);
    unpack8(*reinterpret_cast<const uint4*>(gu + r * 2 * I + I + c), u);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = g[i] * sigmoidf(g[i]) * u[i];
    *reinterpret_cast<uint4*>(h + r * I + c) = pack8(o);
  }
}
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const bf16* __restrict__ gu, const bf16* __restrict__ dh,
                                                         bf16* __restrict__ dgu, int64_t rows, int I) {
  const int v8 = I / 8;
  const int64_t n = rows * v8;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = q / v8;
    const int c = (int)(q % v8) * 8;
    float g[8], u[8], d[8], dg[8], du[8];
    unpack8(*reinterpret_cast<const uint4*>(gu + r * 2 * I + c), g);
    unpack8(*reinterpret_cast<const uint4*>(gu + r * 2 * I + I + c), u);
    unpack8(*reinterpret_cast<const uint4*>(dh + r * I + c), d);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float sg = sigmoidf(g[i]);
      du[i] = d[i] * g[i] * sg;
      dg[i] = d[i] * u[i] * sg * (1.f + g[i] * (1.f - sg));
    }
    *reinterpret_cast<uint4*>(dgu + r * 2 * I + c) = pack8(dg);
    *reinterpret_cast<uint4*>(dgu + r * 2 * I + I + c) = pack8(du);
  }
}
static unsigned grid_for(int64_t n) { return (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16); }
int swiglu_train_fwd(const void* gu, void* h, int64_t rows, int I, cudaStream_t st) {
  if (I % 8 || rows < 1) return rows == 0 ? 0 : 3;
  swiglu_fwd_kernel<<<grid_for(rows * (I / 8)), 256, 0, st>>>((const bf16*)gu, (bf16*)h, rows, I);
  return (int)cudaGetLastError();
}
int swiglu_train_bwd(const void* gu, const void* dh, void* dgu, int64_t rows, int I, cudaStream_t st) {
  if (I % 8 || rows < 1) return rows == 0 ? 0 : 3;
  swiglu_bwd_kernel<<<grid_for(rows * (I / 8)), 256, 0, st>>>((const bf16*)gu, (const bf16*)dh, (bf16*)dgu, rows, I);
  return (int)cudaGetLastError();
}

#define AFB_RMS_V(X) X(1) X(2) X(4) X(8)

// ------------------------------------------------------------------------------------------------ MoE combine
// one warp per token; H = 256 * V
template <int V>
__global__ void __launch_bounds__(256) combine_fwd_kernel(const bf16* __restrict__ y, const int64_t* __restrict__ inv,
                                                          const float* __restrict__ wt, int K, bf16* __restrict__ out,
                                                          int64_t T) {
  constexpr int H = 256 * V;
  const int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float acc[V][8] = {};
  for (int k = 0; k < K; ++k) {
    const float wk = wt[t * K + k];
    const bf16* row = y + inv[t * K + k] * H;
#pragma unroll
    for (int p = 0; p < V; ++p) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(row + (p * 32 + lane) * 8), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[p][i] = fmaf(wk, f[i], acc[p][i]);
    }
  }
#pragma unroll
  for (int p = 0; p < V; ++p) *reinterpret_cast<uint4*>(out + t * H + (p * 32 + lane) * 8) = pack8(acc[p]);
}
// dy[inv[t*K+k]] = w[t,k] dout[t];  dw[t,k] = dout[t] . y[inv[t*K+k]]
template <int V>
__global__ void __launch_bounds__(256) combine_bwd_kernel(const bf16* __restrict__ y, const int64_t* __restrict__ inv,
                                                          const float* __restrict__ wt, int K,
                                                          const bf16* __restrict__ dout, bf16* __restrict__ dy,
                                                          float* __restrict__ dw, int64_t T) {
  constexpr int H = 256 * V;
  const int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float d[V][8];
#pragma unroll
  for (int p = 0; p < V; ++p) unpack8(*reinterpret_cast<const uint4*>(dout + t * H + (p * 32 + lane) * 8), d[p]);
  for (int k = 0; k < K; ++k) {
    const float wk = wt[t * K + k];
    const int64_t r = inv[t * K + k];
    float dot = 0.f;
#pragma unroll
    for (int p = 0; p < V; ++p) {
      const int c = (p * 32 + lane) * 8;
      float f[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(y + r * H + c), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dot = fmaf(d[p][i], f[i], dot);
        o[i] = wk * d[p][i];
      }
      *reinterpret_cast<uint4*>(dy + r * H + c) = pack8(o);
    }
    dot = warp_sum(dot);
    if (lane == 0) dw[t * K + k] = dot;
  }
}
// dx[t] = sum_k g[inv[t*K+k]] (k order)
template <int V>
__global__ void __launch_bounds__(256) dispatch_bwd_kernel(const bf16* __restrict__ g, const int64_t* __restrict__ inv,
                                                           int K, bf16* __restrict__ dx, int64_t T) {
  constexpr int H = 256 * V;
  const int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float acc[V][8] = {};
  for (int k = 0; k < K; ++k) {
    const bf16* row = g + inv[t * K + k] * H;
#pragma unroll
    for (int p = 0; p < V; ++p) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(row + (p * 32 + lane) * 8), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[p][i] += f[i];
    }
  }
#pragma unroll
  for (int p = 0; p < V; ++p) *reinterpret_cast<uint4*>(dx + t * H + (p * 32 + lane) * 8) = pack8(acc[p]);
}

int moe_combine_train_fwd(const void* y, const int64_t* inv, const float* w, int K, void* out, int64_t T, int H,
                          cudaStream_t st) {
  if (T < 1) return 0;
  const unsigned grid = (unsigned)((T + 7) / 8);
  switch (H) {
#define X(v)                                                                                                     \
  case 256 * v:                                                                                                  \
    combine_fwd_kernel<v><<<grid, 256, 0, st>>>((const bf16*)y, inv, w, K, (bf16*)out, T);                       \
    break;
    AFB_RMS_V(X)
#undef X
    default:
      return 3;
  }
  return (int)cudaGetLastError();
}
int moe_combine_train_bwd(const void* y, const int64_t* inv, const float* w, int K, const void* dout, void* dy,
                          float* dw, int64_t T, int H, cudaStream_t st) {
  if (T < 1) return 0;
  const unsigned grid = (unsigned)((T + 7) / 8);
  switch (H) {
#define X(v)                                                                                                     \
  case 256 * v:                                                                                                  \
    combine_bwd_kernel<v><<<grid, 256, 0, st>>>((const bf16*)y, inv, w, K, (const bf16*)dout, (bf16*)dy, dw, T); \
    break;
    AFB_RMS_V(X)
#undef X
    default:
      return 3;
  }
  return (int)cudaGetLastError();
}
int moe_dispatch_train_bwd(const void* g, const int64_t* inv, int K, void* dx, int64_t T, int H, cudaStream_t st) {
  if (T < 1) return 0;
  const unsigned grid = (unsigned)((T + 7) / 8);
  switch (H) {
#define X(v)                                                                                    \
  case 256 * v:                                                                                 \
    dispatch_bwd_kernel<v><<<grid, 256, 0, st>>>((const bf16*)g, inv, K, (bf16*)dx, T);         \
    break;
    AFB_RMS_V(X)
#undef X
    default:
      return 3;
  }
  return (int)cudaGetLastError();
}

}  // namespace afb
