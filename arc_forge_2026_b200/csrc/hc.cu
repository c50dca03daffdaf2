// Hyper-connection kernels (residual stream of G branches [rows, G, H], bf16 in / out, fp32 math; the reference's
// hc_mix.py _norm_fwd / _mix / _norm_bwd / _inject kernels and the hc_gate epilogue, patch 0006 hc_gate.cuh:436):
//
//   hc_norm_fwd    zb[r, g, :] = h[r, g, :] * rstd[r, g] * (1 + w[g, :])        one warp per (row, branch)
//   hc_mix_fwd     x[r, :]    = mean_g sigmoid(pre[r, g, :]) * zb[r, g, :]      (pre = silu(du / 4) @ W_up^T)
//   hc_inject_fwd  out[r, g, :] = h[r, g, :] + y[r, :] * gate[r, g]             the write-back of a sub-layer
//   hc_inject_bwd  dy[r, :] = sum_g dout[r, g, :] gate[r, g];  dgate[r, g] = dout[r, g, :] . y[r, :]
//   hc_mix_bwd     dpre = dx / G * zb * s'(pre) (s = sigmoid), dzb = dx / G * s(pre)
//   hc_norm_bwd    dh = rstd (u - xh mean(u xh)), u = (1 + w) dzb, xh = h rstd   (two passes, no per-lane arrays)
//
// The two projections (du = zb @ [W_down; W_inject]^T, pre = s @ W_up^T) are plain GEMMs around these kernels.
// Weights are frozen (the backward is dX only, as in the reference). Every reduction is in a fixed order.
#include "common.cuh"
#include "kernels.h"

namespace afb {
namespace hcd {
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
AFB_DEV float sig(float x) { return 1.f / (1.f + __expf(-x)); }
constexpr int MAXG = 8;
}  // namespace hcd
using namespace hcd;

// ------------------------------------------------------------------------------------------------ grouped norm
template <int H>
__global__ void __launch_bounds__(256) hc_norm_fwd_kernel(const bf16* __restrict__ h, const float* __restrict__ w,
                                                          bf16* __restrict__ zb, float* __restrict__ rstd, int64_t rg,
                                                          int G, float eps) {
  constexpr int NV = H / 256;  // 8-element chunks per lane
  const int64_t item = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);  // (row, branch)
  const int lane = threadIdx.x & 31;
  if (item >= rg) return;
  const int g = (int)(item % G);
  const bf16* src = h + item * H;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int p = 0; p < NV; ++p) {
    unpack8(*reinterpret_cast<const uint4*>(src + (p * 32 + lane) * 8), v[p]);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[p][i] * v[p][i];
  }
  const float r = rsqrtf(warp_sum(ss) / H + eps);
  if (lane == 0) rstd[item] = r;
  const float* wg = w + (size_t)g * H;
#pragma unroll
  for (int p = 0; p < NV; ++p) {
    const int c = (p * 32 + lane) * 8;
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = v[p][i] * r * (1.f + wg[c + i]);
    *reinterpret_cast<uint4*>(zb + item * H + c) = pack8(o);
  }
}

template <int H>
__global__ void __launch_bounds__(256) hc_norm_bwd_kernel(const bf16* __restrict__ h, const float* __restrict__ w,
                                                          const float* __restrict__ rstd, const float* __restrict__ dzb,
                                                          bf16* __restrict__ dh, int64_t rg, int G) {
  constexpr int NV = H / 256;
  const int64_t item = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= rg) return;
  const int g = (int)(item % G);
  const float r = rstd[item];
  const float* wg = w + (size_t)g * H;
  float dot = 0.f;
  for (int p = 0; p < NV; ++p) {  // pass 1: mean(u xh)
    const int c = (p * 32 + lane) * 8;
    float x[8];
    unpack8(*reinterpret_cast<const uint4*>(h + item * H + c), x);
    const float4 d0 = *reinterpret_cast<const float4*>(dzb + item * H + c);
    const float4 d1 = *reinterpret_cast<const float4*>(dzb + item * H + c + 4);
    const float d[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) dot += (1.f + wg[c + i]) * d[i] * x[i] * r;
  }
  dot = warp_sum(dot) / H;
  for (int p = 0; p < NV; ++p) {  // pass 2: dh
    const int c = (p * 32 + lane) * 8;
    float x[8], o[8];
    unpack8(*reinterpret_cast<const uint4*>(h + item * H + c), x);
    const float4 d0 = *reinterpret_cast<const float4*>(dzb + item * H + c);
    const float4 d1 = *reinterpret_cast<const float4*>(dzb + item * H + c + 4);
    const float d[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = r * ((1.f + wg[c + i]) * d[i] - x[i] * r * dot);
    *reinterpret_cast<uint4*>(dh + item * H + c) = pack8(o);
  }
}

// ------------------------------------------------------------------------------------------------ mix
// thread per (row, 8 columns)
__global__ void __launch_bounds__(256) hc_mix_fwd_kernel(const bf16* __restrict__ pre, const bf16* __restrict__ zb,
                                                         bf16* __restrict__ x, int64_t rows, int G, int H) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int c8 = H / 8;
  const float inv = 1.f / G;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < rows * c8; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = q / c8;
    const int c = (int)(q % c8) * 8;
    float acc[8] = {};
    for (int g = 0; g < G; ++g) {  // branch order fixed
      float p[8], z[8];
      unpack8(*reinterpret_cast<const uint4*>(pre + (r * G + g) * H + c), p);
      unpack8(*reinterpret_cast<const uint4*>(zb + (r * G + g) * H + c), z);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(sig(p[i]), z[i], acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= inv;
    *reinterpret_cast<uint4*>(x + r * H + c) = pack8(acc);
  }
}

__global__ void __launch_bounds__(256) hc_mix_bwd_kernel(const bf16* __restrict__ pre, const bf16* __restrict__ zb,
                                                         const bf16* __restrict__ dx, bf16* __restrict__ dpre,
                                                         float* __restrict__ dzb, int64_t rows, int G, int H) {
  const int c8 = H / 8;
  const float inv = 1.f / G;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < rows * c8; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = q / c8;
    const int c = (int)(q % c8) * 8;
    float d[8];
    unpack8(*reinterpret_cast<const uint4*>(dx + r * H + c), d);
    for (int g = 0; g < G; ++g) {
      float p[8], z[8], dp[8], dz[8];
      const int64_t off = (r * G + g) * H + c;
      unpack8(*reinterpret_cast<const uint4*>(pre + off), p);
      unpack8(*reinterpret_cast<const uint4*>(zb + off), z);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float s = sig(p[i]);
        dz[i] = d[i] * inv * s;
        dp[i] = d[i] * inv * z[i] * s * (1.f - s);
      }
      *reinterpret_cast<uint4*>(dpre + off) = pack8(dp);
      *reinterpret_cast<float4*>(dzb + off) = make_float4(dz[0], dz[1], dz[2], dz[3]);
      *reinterpret_cast<float4*>(dzb + off + 4) = make_float4(dz[4], dz[5], dz[6], dz[7]);
    }
  }
}

// ------------------------------------------------------------------------------------------------ write-back
__global__ void __launch_bounds__(256) hc_inject_fwd_kernel(const bf16* __restrict__ h, const bf16* __restrict__ y,
                                                            const bf16* __restrict__ gate, bf16* __restrict__ out,
                                                            int64_t rows, int G, int H) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int c8 = H / 8;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < rows * c8; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = q / c8;
    const int c = (int)(q % c8) * 8;
    float yv[8];
    unpack8(*reinterpret_cast<const uint4*>(y + r * H + c), yv);
    for (int g = 0; g < G; ++g) {
      const float gt = __bfloat162float(gate[r * G + g]);
      float hv[8];
      const int64_t off = (r * G + g) * H + c;
      unpack8(*reinterpret_cast<const uint4*>(h + off), hv);
#pragma unroll
      for (int i = 0; i < 8; ++i) hv[i] = fmaf(yv[i], gt, hv[i]);
      *reinterpret_cast<uint4*>(out + off) = pack8(hv);
    }
  }
}

// warp per row: dy chunks, and the branch gates' gradients reduced over the row in lane order
__global__ void __launch_bounds__(256) hc_inject_bwd_kernel(const bf16* __restrict__ y, const bf16* __restrict__ gate,
                                                            const bf16* __restrict__ dout, bf16* __restrict__ dy,
                                                            float* __restrict__ dgate, int64_t rows, int G, int H) {
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float gt[MAXG], pg[MAXG];
  for (int g = 0; g < G; ++g) {
    gt[g] = __bfloat162float(gate[r * G + g]);
    pg[g] = 0.f;
  }
  for (int c = lane * 8; c < H; c += 256) {
    float yv[8], acc[8] = {};
    unpack8(*reinterpret_cast<const uint4*>(y + r * H + c), yv);
    for (int g = 0; g < G; ++g) {
      float d[8];
      unpack8(*reinterpret_cast<const uint4*>(dout + (r * G + g) * H + c), d);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        acc[i] = fmaf(d[i], gt[g], acc[i]);
        pg[g] = fmaf(d[i], yv[i], pg[g]);
      }
    }
    *reinterpret_cast<uint4*>(dy + r * H + c) = pack8(acc);
  }
  for (int g = 0; g < G; ++g) {
    const float t = warp_sum(pg[g]);
    if (lane == 0) dgate[r * G + g] = t;
  }
}

// ------------------------------------------------------------------------------------------------ launchers
#define AFB_HC_H(X) X(256) X(512) X(1024) X(2048) X(2560)

static unsigned grid8(int64_t n) { return (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16); }

int hc_norm_fwd(const void* h, const float* w, void* zb, float* rstd, int64_t rows, int G, int H, float eps,
                cudaStream_t st) {
  if (rows < 1) return 0;
  if (G < 1 || G > MAXG) return 3;
  const int64_t rg = rows * G;
  const unsigned grid = (unsigned)((rg + 7) / 8);
  switch (H) {
#define X(hh)                                                                                                    \
  case hh:                                                                                                       \
    hc_norm_fwd_kernel<hh><<<grid, 256, 0, st>>>((const bf16*)h, w, (bf16*)zb, rstd, rg, G, eps);              \
    break;
    AFB_HC_H(X)
#undef X
    default:
      return 3;
  }
  return (int)cudaGetLastError();
}
int hc_norm_bwd(const void* h, const float* w, const float* rstd, const float* dzb, void* dh, int64_t rows, int G,
                int H, cudaStream_t st) {
  if (rows < 1) return 0;
  if (G < 1 || G > MAXG) return 3;
  const int64_t rg = rows * G;
  const unsigned grid = (unsigned)((rg + 7) / 8);
  switch (H) {
#define X(hh)                                                                                                    \
  case hh:                                                                                                       \
    hc_norm_bwd_kernel<hh><<<grid, 256, 0, st>>>((const bf16*)h, w, rstd, dzb, (bf16*)dh, rg, G);              \
    break;
    AFB_HC_H(X)
#undef X
    default:
      return 3;
  }
  return (int)cudaGetLastError();
}
// Serving read-side activations of the down / inject projection du [rows, ld] (bf16): s = silu(du[:, :R] / 4) and
// gate = 2 sigmoid(du[:, R:R+G] / 4), both bf16 (one launch instead of the elementwise chain).
__global__ void __launch_bounds__(256) hc_act_kernel(const bf16* __restrict__ du, int ld, int64_t rows, int R, int G,
                                                     bf16* __restrict__ s, bf16* __restrict__ gate) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int per = R + (gate ? G : 0);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * per) return;
  const int64_t r = i / per;
  const int c = (int)(i % per);
  const float z = __bfloat162float(du[r * ld + c]) * 0.25f;
  if (c < R) s[r * R + c] = __float2bfloat16(z / (1.f + __expf(-z)));
  else gate[r * G + (c - R)] = __float2bfloat16(2.f / (1.f + __expf(-z)));
}
int hc_act_fwd(const void* du, int ld, int64_t rows, int R, int G, void* s, void* gate, cudaStream_t st) {
  if (rows < 1) return 0;
  if (R < 1 || G < 0 || ld < R + (gate ? G : 0)) return 3;
  const int64_t n = rows * (R + (gate ? G : 0));
  if (const int pdl_rc = launch_pdl(hc_act_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st,
      (const bf16*)du, ld, rows, R, G, (bf16*)s, (bf16*)gate)) return pdl_rc;
  return (int)cudaGetLastError();
}

int hc_mix_fwd(const void* pre, const void* zb, void* x, int64_t rows, int G, int H, cudaStream_t st) {
  if (rows < 1) return 0;
  if (H % 8 || G < 1 || G > MAXG) return 3;
  if (const int pdl_rc = launch_pdl(hc_mix_fwd_kernel, dim3(grid8(rows * (H / 8))), dim3(256), 0, st,
      (const bf16*)pre, (const bf16*)zb, (bf16*)x, rows, G, H)) return pdl_rc;
  return (int)cudaGetLastError();
}
int hc_mix_bwd(const void* pre, const void* zb, const void* dx, void* dpre, float* dzb, int64_t rows, int G, int H,
               cudaStream_t st) {
  if (rows < 1) return 0;
  if (H % 8 || G < 1 || G > MAXG) return 3;
  hc_mix_bwd_kernel<<<grid8(rows * (H / 8)), 256, 0, st>>>((const bf16*)pre, (const bf16*)zb, (const bf16*)dx,
                                                           (bf16*)dpre, dzb, rows, G, H);
  return (int)cudaGetLastError();
}
int hc_inject_fwd(const void* h, const void* y, const void* gate, void* out, int64_t rows, int G, int H,
                  cudaStream_t st) {
  if (rows < 1) return 0;
  if (H % 8 || G < 1 || G > MAXG) return 3;
  if (const int pdl_rc = launch_pdl(hc_inject_fwd_kernel, dim3(grid8(rows * (H / 8))), dim3(256), 0, st,
      (const bf16*)h, (const bf16*)y, (const bf16*)gate,
                                                              (bf16*)out, rows, G, H)) return pdl_rc;
  return (int)cudaGetLastError();
}
int hc_inject_bwd(const void* y, const void* gate, const void* dout, void* dy, float* dgate, int64_t rows, int G,
                  int H, cudaStream_t st) {
  if (rows < 1) return 0;
  if (H % 256 || G < 1 || G > MAXG) return 3;
  hc_inject_bwd_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>((const bf16*)y, (const bf16*)gate,
                                                                   (const bf16*)dout, (bf16*)dy, dgate, rows, G, H);
  return (int)cudaGetLastError();
}

}  // namespace afb
