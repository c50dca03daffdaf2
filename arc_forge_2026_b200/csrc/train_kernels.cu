// Training-side kernels of quantisation-aware distillation (QAD).
//
// * int3_dequant: W[e, n, k] = bf16((c - 4) * bf16(s[e, n, k/128])) from the INT3 tile layout and fp32 master
//   scales -- the STE forward of trainable group scales (codes frozen), the same product the serving pack holds.
// * int3_scale_grad: dS[e, n, g] = sum_{k in g} (c - 4) * dW[e, n, k] (one half-warp per (e, n, g)), the gradient of the
//   scales given dW; fixed-order reduction, bitwise reproducible.
// * fp8_block_fakequant: W -> dequant(quant_e4m3(W)) with one scale per 128x128 block (scale = amax / 448), the
//   STE forward of the dense block-FP8 projections (one CTA per block).
// * topk_tail_kl: per row of fp32 logits z (one CTA per row): log-sum-exp over the vocabulary and over the
//   non-top-k tail, the loss of the (k + 1)-class coarsening (forward or reverse KL), and dL/dz written as bf16.
// * adamw: fused AdamW on fp32 masters with bf16 moment states; writes the bf16 compute copy of the weights.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace afb {

// -------------------------------------------------------------------------------------------- INT3 STE forward
// codes: tile layout [E, R/128, K/128, 128, 12]; scales fp32 [E, R, K/128]; out bf16 [E, R, K]
// One thread per 32 codes (3 words -> 64 bytes of bf16, four 16-byte stores); consecutive threads walk along K so
// a warp writes 2 KB of one row contiguously.
AFB_DEV int code_at(uint32_t L0, uint32_t L1, uint32_t H, int n) {
  const int m = n & 7;
  switch (n >> 3) {
    case 0: return (int)((L0 >> (4 * m)) & 3) | (int)(((H >> (4 * m + 2)) & 1) << 2);
    case 1: return (int)((L0 >> (4 * m + 2)) & 3) | (int)(((H >> (4 * m + 3)) & 1) << 2);
    case 2: return (int)((L1 >> (4 * m)) & 3) | (int)(((H >> (4 * m)) & 1) << 2);
    default: return (int)((L1 >> (4 * m + 2)) & 3) | (int)(((H >> (4 * m + 1)) & 1) << 2);
  }
}

__global__ void int3_dequant_kernel(const uint32_t* __restrict__ codes, const float* __restrict__ scales, int E, int R,
                                    int K, __nv_bfloat16* __restrict__ out) {
  const int KG = K / 128;
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (tid >= (size_t)E * R * KG * 4) return;
  const int q = (int)(tid & 3);
  const size_t rest = tid >> 2;
  const int g = (int)(rest % KG);
  const size_t er = rest / KG;  // e * R + row
  const int e = (int)(er / R), row = (int)(er % R);
  const uint32_t* w = codes + ((((size_t)e * (R / 128) + row / 128) * KG + g) * 128 + (row & 127)) * 12 + 3 * q;
  const uint32_t L0 = __ldg(w), L1 = __ldg(w + 1), H = __ldg(w + 2);
  const float s = __bfloat162float(__float2bfloat16(scales[er * KG + g]));
  uint4* o = reinterpret_cast<uint4*>(out + er * K + g * 128 + q * 32);
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    uint32_t p[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int n = v * 8 + h * 2;
      p[h] = pack_bf16x2((float)(code_at(L0, L1, H, n) - 4) * s, (float)(code_at(L0, L1, H, n + 1) - 4) * s);
    }
    o[v] = make_uint4(p[0], p[1], p[2], p[3]);
  }
}

int int3_dequant(const void* codes, const float* scales, int E, int R, int K, void* out, cudaStream_t st) {
  if (R % 128 || K % 128) return 3;
  const size_t threads = (size_t)E * R * (K / 128) * 4;
  int3_dequant_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>((const uint32_t*)codes, scales, E, R, K,
                                                                         (__nv_bfloat16*)out);
  return (int)cudaGetLastError();
}

// dS[e, n, g] = sum_k (c - 4) * dW[e, n, g*128 + k]; dW bf16 [E, R, K]; codes as above; dS fp32 [E, R, K/128]
// dS[e, r, g] = sum_{k in group g} (code[e, r, k] - 4) * dW[e, r, k]. A half-warp owns one (row, group) pair: lane
// l of the half takes the 8 codes 8l..8l+7 (quad q = l / 4, sub-block j = l % 4 of the 12-word tile row) and one
// 16-byte vector of dW; every thread has 4 pairs' loads in flight before it reduces (persistent grid).
AFB_DEV int code8_word_lo(int j) { return j < 2 ? 0 : 1; }
__global__ void __launch_bounds__(256) int3_scale_grad_kernel(const uint32_t* __restrict__ codes,
                                                              const __nv_bfloat16* __restrict__ dW, int E, int R,
                                                              int K, float* __restrict__ dS) {
  constexpr int U = 4;
  const int KG = K / 128;
  const int64_t pairs = (int64_t)E * R * KG;
  const int hl = threadIdx.x & 15;                 // lane within the half-warp
  const int q = hl >> 2, j = hl & 3;               // quad and 8-code sub-block
  const int64_t half = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
  const int64_t halves = ((int64_t)gridDim.x * blockDim.x) >> 4;
  for (int64_t p0 = half; p0 < pairs; p0 += halves * U) {
    uint4 dv[U];
    uint32_t lw[U], hw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t p = p0 + u * halves;
      dv[u] = make_uint4(0, 0, 0, 0);
      lw[u] = hw[u] = 0;
      if (p < pairs) {
        const int64_t er = p / KG;                 // e * R + row
        const int g = (int)(p % KG), row = (int)(er % R);
        const int64_t e = er / R;
        const uint32_t* w = codes + (((e * (R / 128) + row / 128) * KG + g) * 128 + (row & 127)) * 12;
        lw[u] = w[3 * q + code8_word_lo(j)];
        hw[u] = w[3 * q + 2];
        dv[u] = *reinterpret_cast<const uint4*>(dW + er * K + g * 128 + hl * 8);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const __nv_bfloat16* dh = reinterpret_cast<const __nv_bfloat16*>(&dv[u]);
      float acc = 0.f;
#pragma unroll
      for (int t = 0; t < 8; ++t) {  // code c = 8j + t within the quad (bit layout of quant/int3_tiles.py)
        int code;
        if (j == 0)
          code = (int)((lw[u] >> (4 * t)) & 3) | (int)(((hw[u] >> (4 * t + 2)) & 1) << 2);
        else if (j == 1)
          code = (int)((lw[u] >> (4 * t + 2)) & 3) | (int)(((hw[u] >> (4 * t + 3)) & 1) << 2);
        else if (j == 2)
          code = (int)((lw[u] >> (4 * t)) & 3) | (int)(((hw[u] >> (4 * t)) & 1) << 2);
        else
          code = (int)((lw[u] >> (4 * t + 2)) & 3) | (int)(((hw[u] >> (4 * t + 1)) & 1) << 2);
        acc = fmaf((float)(code - 4), __bfloat162float(dh[t]), acc);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);  // within the half-warp
      const int64_t p = p0 + u * halves;
      if (hl == 0 && p < pairs) dS[p] = acc;
    }
  }
}

int int3_scale_grad(const void* codes, const void* dW, int E, int R, int K, float* dS, cudaStream_t st) {
  if (R % 128 || K % 128) return 3;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t halves = (int64_t)E * R * (K / 128);
  const int64_t blocks = std::min<int64_t>((halves * 16 + 255) / 256, (int64_t)sms * 8);
  int3_scale_grad_kernel<<<(unsigned)blocks, 256, 0, st>>>((const uint32_t*)codes, (const __nv_bfloat16*)dW, E, R, K,
                                                           dS);
  return (int)cudaGetLastError();
}

// -------------------------------------------------------------------------------------------- block FP8 fake quant
// one CTA (256 threads) per 128x128 block of an [N, K] matrix (fp32 master in, bf16 dequantised out)
__global__ void fp8_block_fakequant_kernel(const float* __restrict__ w, int N, int K, __nv_bfloat16* __restrict__ out,
                                           float* __restrict__ scale_inv) {
  const int bn = blockIdx.y, bk = blockIdx.x;
  __shared__ float red[8];
  float amax = 0.f;
  for (int i = threadIdx.x; i < 128 * 128; i += blockDim.x) {
    const int r = bn * 128 + i / 128, c = bk * 128 + i % 128;
    if (r < N && c < K) amax = fmaxf(amax, fabsf(__bfloat162float(__float2bfloat16(w[(size_t)r * K + c]))));
  }
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float m = 0.f;
  for (int i = 0; i < 8; ++i) m = fmaxf(m, red[i]);
  const float s = m > 0.f ? m / 448.f : 1.f;
  if (threadIdx.x == 0 && scale_inv) scale_inv[bn * gridDim.x + bk] = s;
  for (int i = threadIdx.x; i < 128 * 128; i += blockDim.x) {
    const int r = bn * 128 + i / 128, c = bk * 128 + i % 128;
    if (r < N && c < K) {
      const float x = __bfloat162float(__float2bfloat16(w[(size_t)r * K + c]));  // the bf16 cast, then FP8
      const __nv_fp8_e4m3 q(fminf(fmaxf(x / s, -448.f), 448.f));
      out[(size_t)r * K + c] = __float2bfloat16(float(q) * s);
    }
  }
}

int fp8_block_fakequant(const float* w, int N, int K, void* out, float* scale_inv, cudaStream_t st) {
  dim3 grid((K + 127) / 128, (N + 127) / 128);
  fp8_block_fakequant_kernel<<<grid, 256, 0, st>>>(w, N, K, (__nv_bfloat16*)out, scale_inv);
  return (int)cudaGetLastError();
}

// -------------------------------------------------------------------------------------------- top-k tail KL
// z fp32 [rows, V] logits; ids int64 [rows, k]; t_lp fp32 [rows, k]; t_tail fp32 [rows];
// loss fp32 [rows]; dz bf16 [rows, V] (scaled by grad_scale). One CTA of 256 threads per row; k <= 256.
__global__ void __launch_bounds__(256) topk_tail_kl_kernel(const float* __restrict__ z, int ldz, int V,
                                                           const long long* __restrict__ ids, int k,
                                                           const float* __restrict__ t_lp, const float* __restrict__ t_tail,
                                                           int reverse, float grad_scale, float* __restrict__ loss,
                                                           __nv_bfloat16* __restrict__ dz, int ldd) {
  const int row = blockIdx.x;
  const float* zr = z + (size_t)row * ldz;
  __shared__ float red[8];
  __shared__ float sh_q[256], sh_lp[256];
  __shared__ int sh_id[256];
  __shared__ float s_lse, s_tail, s_loss, s_extra;
  // pass 1: max and sum-exp over V
  float mx = -INFINITY;
  for (int c = threadIdx.x; c < V; c += blockDim.x) mx = fmaxf(mx, zr[c]);
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  float M = red[0];
  for (int i = 1; i < 8; ++i) M = fmaxf(M, red[i]);
  __syncthreads();
  float se = 0.f;
  for (int c = threadIdx.x; c < V; c += blockDim.x) se += __expf(zr[c] - M);
  se = warp_sum(se);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = se;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < 8; ++i) t += red[i];
    s_lse = M + __logf(t);
  }
  if (threadIdx.x < k) {
    const long long id = ids[(size_t)row * k + threadIdx.x];
    sh_id[threadIdx.x] = (int)id;
    sh_lp[threadIdx.x] = t_lp[(size_t)row * k + threadIdx.x];
  }
  __shared__ int sorted_id[256];
  if (threadIdx.x < k) sorted_id[threadIdx.x] = sh_id[threadIdx.x];
  __syncthreads();
  if (threadIdx.x == 0) {  // insertion sort of the (<= 256) class ids for the membership test below
    for (int i = 1; i < k; ++i) {
      const int x = sorted_id[i];
      int j = i - 1;
      while (j >= 0 && sorted_id[j] > x) {
        sorted_id[j + 1] = sorted_id[j];
        --j;
      }
      sorted_id[j + 1] = x;
    }
  }
  __syncthreads();
  const float lse = s_lse;
  // per top-k class: log q_i; tail mass summed directly over the non-top-k columns (no 1 - sum cancellation)
  if (threadIdx.x < k) sh_q[threadIdx.x] = zr[sh_id[threadIdx.x]] - lse;
  float te = 0.f;
  for (int c = threadIdx.x; c < V; c += blockDim.x) {
    int lo = 0, hi = k - 1;
    bool in = false;
    while (lo <= hi) {
      const int mid = (lo + hi) >> 1;
      const int x = sorted_id[mid];
      if (x == c) {
        in = true;
        break;
      }
      if (x < c) lo = mid + 1; else hi = mid - 1;
    }
    if (!in) te += __expf(zr[c] - M);
  }
  te = warp_sum(te);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = te;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tsum = 0.f;
    for (int i = 0; i < 8; ++i) tsum += red[i];
    const float lq_r = tsum > 0.f ? __logf(tsum) + M - lse : -INFINITY;
    const float qr = __expf(lq_r);
    const float p_r = __expf(t_tail[row]);
    float L = 0.f;
    if (!reverse) {
      for (int i = 0; i < k; ++i) L += __expf(sh_lp[i]) * (sh_lp[i] - sh_q[i]);
      if (p_r > 0.f) L += p_r * (t_tail[row] - lq_r);
      s_extra = qr > 0.f ? 1.f - p_r / qr : 1.f;  // factor for tail columns
    } else {
      for (int i = 0; i < k; ++i) {
        const float qi = __expf(sh_q[i]);
        if (qi > 0.f) L += qi * (sh_q[i] - sh_lp[i]);
      }
      const float gr = lq_r - t_tail[row];
      if (qr > 0.f) L += qr * gr;
      s_extra = qr > 0.f ? gr : 0.f;  // g_R
    }
    s_loss = L;
    s_tail = lq_r;
    loss[row] = L;
  }
  __syncthreads();
  const float L = s_loss, ex = s_extra;
  // pass 2: gradient of every column; tail columns first, then overwrite the top-k columns
  __nv_bfloat16* dr = dz + (size_t)row * ldd;
  for (int c = threadIdx.x; c < V; c += blockDim.x) {
    const float q = __expf(zr[c] - lse);
    const float g = reverse ? q * (ex - L) : q * ex;
    dr[c] = __float2bfloat16(g * grad_scale);
  }
  __syncthreads();
  if (threadIdx.x < k) {
    const float qi = __expf(sh_q[threadIdx.x]);
    float g;
    if (!reverse)
      g = qi - __expf(sh_lp[threadIdx.x]);
    else
      g = qi > 0.f ? qi * ((sh_q[threadIdx.x] - sh_lp[threadIdx.x]) - L) : 0.f;
    dr[sh_id[threadIdx.x]] = __float2bfloat16(g * grad_scale);
  }
}

int topk_tail_kl(const float* z, int ldz, int rows, int V, const long long* ids, int k, const float* t_lp,
                 const float* t_tail, int reverse, float grad_scale, float* loss, void* dz, int ldd, cudaStream_t st) {
  if (k > 256) return 3;
  if (!rows) return 0;
  topk_tail_kl_kernel<<<rows, 256, 0, st>>>(z, ldz, V, ids, k, t_lp, t_tail, reverse, grad_scale, loss,
                                            (__nv_bfloat16*)dz, ldd);
  return (int)cudaGetLastError();
}

// -------------------------------------------------------------------------------------------- AdamW
// p fp32 master, g fp32 grad, m/v bf16 moments; bf16 copy of the updated weights into w (optional).
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, __nv_bfloat16* __restrict__ m,
                             __nv_bfloat16* __restrict__ v, __nv_bfloat16* __restrict__ w, size_t n, float lr, float b1,
                             float b2, float eps, float wd, float bc1, float bc2) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float gi = g[i];
  const float mi = b1 * __bfloat162float(m[i]) + (1.f - b1) * gi;
  const float vi = b2 * __bfloat162float(v[i]) + (1.f - b2) * gi * gi;
  m[i] = __float2bfloat16(mi);
  v[i] = __float2bfloat16(vi);
  float pi = p[i];
  pi -= lr * (wd * pi + (mi / bc1) / (sqrtf(vi / bc2) + eps));
  p[i] = pi;
  if (w) w[i] = __float2bfloat16(pi);
}

int adamw(float* p, const float* g, void* m, void* v, void* w, size_t n, float lr, float b1, float b2, float eps,
          float wd, int step, cudaStream_t st) {
  if (!n) return 0;
  const float bc1 = 1.f - powf(b1, (float)step), bc2 = 1.f - powf(b2, (float)step);
  adamw_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(p, g, (__nv_bfloat16*)m, (__nv_bfloat16*)v,
                                                           (__nv_bfloat16*)w, n, lr, b1, b2, eps, wd, bc1, bc2);
  return (int)cudaGetLastError();
}

}  // namespace afb

namespace afb {
// ------------------------------------------------------------------------------------------ tiled transpose
// out[b][col_map(c)... ] : out[b][c][dst(r)] = src[b][r][c] for a batch of [R, C] bf16 matrices, through 64 x 64
// shared-memory tiles (reads and writes coalesced). dst (optional, [R]) remaps rows of src to columns of out: the
// grouped expert GEMM's dW operands are the activations transposed into 64-row-aligned expert segments.
namespace tpd {
constexpr int TILE = 64;
}
__global__ void __launch_bounds__(256) transpose_bf16_kernel(const __nv_bfloat16* __restrict__ src, int64_t R,
                                                             int64_t C, int64_t lds, int64_t src_batch,
                                                             const int64_t* __restrict__ dst,
                                                             __nv_bfloat16* __restrict__ out, int64_t ldo,
                                                             int64_t out_batch) {
  __shared__ __nv_bfloat16 t[tpd::TILE][tpd::TILE + 2];
  const int64_t r0 = (int64_t)blockIdx.y * tpd::TILE, c0 = (int64_t)blockIdx.x * tpd::TILE;
  const __nv_bfloat16* s = src + (int64_t)blockIdx.z * src_batch;
  __nv_bfloat16* o = out + (int64_t)blockIdx.z * out_batch;
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;  // 64 x 4 threads
  for (int i = ty; i < tpd::TILE; i += 4) {
    const int64_t r = r0 + i, c = c0 + tx;
    t[i][tx] = (r < R && c < C) ? s[r * lds + c] : __float2bfloat16(0.f);
  }
  __syncthreads();
  const int64_t r = r0 + tx;
  if (r >= R) return;
  const int64_t col = dst ? dst[r] : r;
  for (int i = ty; i < tpd::TILE; i += 4) {
    const int64_t c = c0 + i;
    if (c < C) o[c * ldo + col] = t[tx][i];
  }
}

int transpose_bf16(const void* src, int64_t R, int64_t C, int64_t lds, int64_t batch, int64_t src_batch,
                   const int64_t* dst, void* out, int64_t ldo, int64_t out_batch, cudaStream_t st) {
  if (R <= 0 || C <= 0 || batch <= 0) return 0;
  dim3 grid((unsigned)((C + tpd::TILE - 1) / tpd::TILE), (unsigned)((R + tpd::TILE - 1) / tpd::TILE), (unsigned)batch);
  transpose_bf16_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(src), R, C, lds, src_batch, dst,
                                              reinterpret_cast<__nv_bfloat16*>(out), ldo, out_batch);
  return (int)cudaGetLastError();
}
}  // namespace afb
