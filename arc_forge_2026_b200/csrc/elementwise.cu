// Memory-bound fused kernels of the decode/verify step: RMSNorm (+residual), per-head q/k norm + partial
// RoPE + paged KV store, router softmax/top-k, deterministic expert sort, fp8 group quantisation for the
// expert GEMMs, SwiGLU, the top-k combine with the shared expert, and the embedding gather.
// Each is one pass over HBM with vectorised 16-byte accesses; reductions are per warp in a fixed order,
// so results are bitwise reproducible run to run.
#include <cuda_fp4.h>

#include "common.cuh"
#include "kernels.h"

namespace afb {

// ------------------------------------------------------------------------------------------ RMSNorm
// y = x/rms(x) * (1 + w) (zero-centred) or * w; with `residual`: h = x + residual, residual <- h (bf16),
// y = norm(h). One warp per row; pass 2 re-reads the row (L1/L2 hit) instead of holding it in registers.
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ residual,
                               const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y, int rows, int H,
                               float eps, int zero_centered) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + (size_t)row * H;
  __nv_bfloat16* rr = residual ? residual + (size_t)row * H : nullptr;
  float ss = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    uint4 q = *reinterpret_cast<const uint4*>(xr + c);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&q);
    float f[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) f[t] = __bfloat162float(h[t]);
    if (rr) {
      uint4 r = *reinterpret_cast<const uint4*>(rr + c);
      const __nv_bfloat16* hr = reinterpret_cast<const __nv_bfloat16*>(&r);
#pragma unroll
      for (int t = 0; t < 8; ++t) f[t] += __bfloat162float(hr[t]);
      uint4 o = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                           pack_bf16x2(f[6], f[7]));
      *reinterpret_cast<uint4*>(rr + c) = o;
      const __nv_bfloat16* ho = reinterpret_cast<const __nv_bfloat16*>(&o);
#pragma unroll
      for (int t = 0; t < 8; ++t) f[t] = __bfloat162float(ho[t]);  // normalise the stored bf16 stream
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) ss += f[t] * f[t];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / H + eps);
  const __nv_bfloat16* src = rr ? rr : xr;
  for (int c = lane * 8; c < H; c += 256) {
    uint4 q = *reinterpret_cast<const uint4*>(src + c);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&q);
    uint4 wq = *reinterpret_cast<const uint4*>(w + c);
    const __nv_bfloat16* wh = reinterpret_cast<const __nv_bfloat16*>(&wq);
    float o[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float ww = __bfloat162float(wh[t]);
      o[t] = __bfloat162float(h[t]) * inv * (zero_centered ? 1.f + ww : ww);
    }
    *reinterpret_cast<uint4*>(y + (size_t)row * H + c) =
        make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
  }
}

int rmsnorm(const void* x, void* residual, const void* w, void* y, int rows, int H, float eps, int zero_centered,
            cudaStream_t st) {
  if (H % 8) return 3;
  if (!rows) return 0;
  const int warps = 4;
  {
    const int pdl_rc = launch_pdl(rmsnorm_kernel, dim3((rows + warps - 1) / warps), dim3(warps * 32), 0, st,
      (const __nv_bfloat16*)x, (__nv_bfloat16*)residual, (const __nv_bfloat16*)w, (__nv_bfloat16*)y, rows, H, eps,
      zero_centered);
    if (pdl_rc) return pdl_rc;
  }
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------ q/k norm + RoPE + KV store
// qkv: [T, Hq*2D + 2*Hkv*D] bf16 GEMM output, per token [q_h | gate_h] x Hq, then k x Hkv, v x Hkv.
// Writes q_out [T, Hq, D] (RMS-normed with (1+w), NeoX RoPE on the first `rot` channels) and k (same) / v into
// the paged cache at slots[t] (page = slot / page_size): cache layout [num_pages, Hkv, page_size, D].
// cos/sin come from a table [max_pos, rot/2] built in fp64 on the host. One warp per (token, head);
// the head vector is staged in shared memory so each lane can read its rotation partner.
// NVFP4 cache (kscale / vscale given): k and v rows are stored as e2m1 pairs [.., D/2] with one e4m3 scale per 16
// elements [.., D/16]: scale = e4m3(amax / 6), codes = e2m1(x / scale) rounded to nearest, saturating at +-6.
AFB_DEV void store_nvfp4_row(const float* x, int D, int lane, uint8_t* packed, uint8_t* scales) {
  if (lane < D / 16) {
    const float* blk = x + lane * 16;
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(blk[i]));
    const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(amax / 6.f, __NV_SATFINITE, __NV_E4M3);
    const float sd = __half2float(__half(__nv_cvt_fp8_to_halfraw(s8, __NV_E4M3)));
    const float inv = sd > 0.f ? 1.f / sd : 0.f;
    uint8_t b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      b[i] = __nv_cvt_float2_to_fp4x2(make_float2(blk[2 * i] * inv, blk[2 * i + 1] * inv), __NV_E2M1,
                                      cudaRoundNearest);
    *reinterpret_cast<uint2*>(packed + lane * 8) = *reinterpret_cast<const uint2*>(b);
    scales[lane] = s8;
  }
}

__global__ void qk_norm_rope_store_kernel(const __nv_bfloat16* __restrict__ qkv, int ld, int T, int Hq, int Hkv, int D,
                                          int rot, const __nv_bfloat16* __restrict__ qw,
                                          const __nv_bfloat16* __restrict__ kw, const int* __restrict__ positions,
                                          const int* __restrict__ slots, const float* __restrict__ cos_t,
                                          const float* __restrict__ sin_t, float eps, __nv_bfloat16* __restrict__ q_out,
                                          __nv_bfloat16* __restrict__ kcache, __nv_bfloat16* __restrict__ vcache,
                                          int page_size, uint8_t* __restrict__ kscale, uint8_t* __restrict__ vscale) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  __shared__ float buf[8][256];
  __shared__ float obuf[8][256];
  const int wi = threadIdx.x >> 5;
  const int gw = blockIdx.x * (blockDim.x >> 5) + wi;
  const int lane = threadIdx.x & 31;
  const int heads = Hq + 2 * Hkv;
  if (gw >= T * heads) return;
  const int t = gw / heads, h = gw % heads;
  const int row_len = ld;  // row stride of the projection output (>= Hq*2D + 2*Hkv*D)
  const __nv_bfloat16* src;
  int kind;  // 0 q, 1 k, 2 v
  if (h < Hq) {
    src = qkv + (size_t)t * row_len + h * 2 * D;
    kind = 0;
  } else if (h < Hq + Hkv) {
    src = qkv + (size_t)t * row_len + Hq * 2 * D + (h - Hq) * D;
    kind = 1;
  } else {
    src = qkv + (size_t)t * row_len + Hq * 2 * D + Hkv * D + (h - Hq - Hkv) * D;
    kind = 2;
  }
  const int slot = slots[t];
  const int page = slot / page_size, tok = slot % page_size;
  const bool fp4 = kscale != nullptr;
  float* b = buf[wi];
  if (kind == 2) {
    const size_t row = ((size_t)page * Hkv + (h - Hq - Hkv)) * page_size + tok;
    if (fp4) {
      for (int j = lane; j < D; j += 32) b[j] = __bfloat162float(src[j]);
      __syncwarp();
      store_nvfp4_row(b, D, lane, reinterpret_cast<uint8_t*>(vcache) + row * (D / 2), vscale + row * (D / 16));
      return;
    }
    __nv_bfloat16* dst = vcache + row * D;
    for (int j = lane; j < D; j += 32) dst[j] = src[j];
    return;
  }
  float ss = 0.f;
  for (int j = lane; j < D; j += 32) {
    const float f = __bfloat162float(src[j]);
    b[j] = f;
    ss += f * f;
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / D + eps);
  const __nv_bfloat16* nw = kind == 0 ? qw : kw;
  for (int j = lane; j < D; j += 32) b[j] = b[j] * inv * (1.f + __bfloat162float(nw[j]));
  __syncwarp();
  const int half = rot / 2;
  const int p = positions[t];
  const size_t krow = ((size_t)page * Hkv + (h - Hq)) * page_size + tok;
  const bool k_fp4 = fp4 && kind == 1;
  __nv_bfloat16* dst = kind == 0 ? q_out + ((size_t)t * Hq + h) * D : kcache + krow * D;
  float* ob = obuf[wi];
  for (int j = lane; j < D; j += 32) {
    float o = b[j];
    if (j < rot) {
      const int fi = j < half ? j : j - half;
      const float cs = cos_t[(size_t)p * half + fi], sn = sin_t[(size_t)p * half + fi];
      o = j < half ? b[j] * cs - b[j + half] * sn : b[j] * cs + b[j - half] * sn;
    }
    if (k_fp4)
      ob[j] = o;
    else
      dst[j] = __float2bfloat16(o);
  }
  if (k_fp4) {
    __syncwarp();
    store_nvfp4_row(ob, D, lane, reinterpret_cast<uint8_t*>(kcache) + krow * (D / 2), kscale + krow * (D / 16));
  }
}

int qk_norm_rope_store(const void* qkv, int ld, int T, int Hq, int Hkv, int D, int rot, const void* qw, const void* kw,
                       const int* positions, const int* slots, const float* cos_t, const float* sin_t, float eps,
                       void* q_out, void* kcache, void* vcache, int page_size, cudaStream_t st, uint8_t* kscale,
                       uint8_t* vscale) {
  if (D > 256 || rot > D || rot % 2 || (kscale && D % 32)) return 3;
  if (!T) return 0;
  const int warps = 8;
  const int total = T * (Hq + 2 * Hkv);
  {
    const int pdl_rc = launch_pdl(qk_norm_rope_store_kernel, dim3((total + warps - 1) / warps), dim3(warps * 32), 0, st,
      (const __nv_bfloat16*)qkv, ld, T, Hq, Hkv, D, rot, (const __nv_bfloat16*)qw, (const __nv_bfloat16*)kw, positions,
      slots, cos_t, sin_t, eps, (__nv_bfloat16*)q_out, (__nv_bfloat16*)kcache, (__nv_bfloat16*)vcache, page_size,
      kscale, vscale);
    if (pdl_rc) return pdl_rc;
  }
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------ router
// logits [T, ld] fp32 (first E columns are experts). softmax -> top-k (ties: lower id) -> renorm.
// One warp per token; lane i owns experts i, i+32, ... (E <= 1024).
// With `cnt` / `list` given (cnt zeroed before the launch) every (token, slot) entry e = t * k + j is also appended
// to its expert's list: list[expert * cap + pos] = e, pos from an atomic counter cnt[expert] (the order inside a list
// is arbitrary; the expert kernels' results do not depend on it). cap >= T: a token picks an expert once.
__global__ void router_topk_kernel(const float* __restrict__ logits, int ld, int T, int E, int k, int renorm,
                                   int* __restrict__ ids, float* __restrict__ weights, int* __restrict__ cnt,
                                   int* __restrict__ list, int cap) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const float* l = logits + (size_t)t * ld;
  float v[32];
  const int per = (E + 31) / 32;
  float mx = -INFINITY;
  for (int i = 0; i < per; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < E ? l[e] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
  for (int i = 0; i < per; ++i) {
    v[i] = (i * 32 + lane) < E ? __expf(v[i] - mx) : 0.f;
    sum += v[i];
  }
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
  float picked_sum = 0.f;
  float wsel = 0.f;
  int isel = 0;
  for (int j = 0; j < k; ++j) {
    // local best (value desc, id asc)
    float bv = -1.f;
    int be = 0x7fffffff;
    for (int i = 0; i < per; ++i) {
      const int e = i * 32 + lane;
      if (e < E && (v[i] > bv || (v[i] == bv && e < be))) {
        bv = v[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    if ((be & 31) == lane) v[be >> 5] = -2.f;  // remove
    const float p = bv * inv;
    picked_sum += p;
    if (lane == j) {
      wsel = p;
      isel = be;
    }
  }
  if (lane < k) {
    ids[(size_t)t * k + lane] = isel;
    weights[(size_t)t * k + lane] = renorm ? wsel / picked_sum : wsel;
    if (cnt) {
      const int pos = atomicAdd(&cnt[isel], 1);
      list[(size_t)isel * cap + pos] = t * k + lane;
    }
  }
}

int router_topk(const float* logits, int ld, int T, int E, int k, int renorm, int* ids, float* weights,
                cudaStream_t st, int* cnt, int* list, int cap) {
  if (E > 1024 || k > 32) return 3;
  if (cnt && (!list || cap < T)) return 3;
  const int warps = 4;
  if (cnt) {
    const cudaError_t e = cudaMemsetAsync(cnt, 0, (size_t)E * sizeof(int), st);
    if (e != cudaSuccess) return (int)e;
  }
  if (T <= 0) return 0;
  {
    const int pdl_rc = launch_pdl(router_topk_kernel, dim3((T + warps - 1) / warps), dim3(warps * 32), 0, st, logits,
        ld, T, E, k, renorm, ids, weights, cnt,
                                                                      list, cap);
    if (pdl_rc) return pdl_rc;
  }
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------ expert sort
// Stable counting sort of the T*k (token, slot) entries by expert, in one CTA of 1024 threads:
// entry i -> position offsets[e] + (# entries i' < i with the same expert). Each expert's segment starts on a
// multiple of `pad` rows (the expert GEMM moves per-segment scale vectors with 16-byte bulk copies); pad rows
// get row_token 0 and row_entry -1. Outputs:
//   offsets [E+1] (segment starts; offsets[E] = rows used), row_token [rows] (token of each sorted row),
//   row_entry [rows] (entry index t*k+j), entry_row [T*k] (inverse; -1 if the expert is not local).
// `expert_map` (optional) maps global expert ids to local ones (-1 = not on this rank) for EP.
__global__ void __launch_bounds__(1024) expert_sort_kernel(const int* __restrict__ ids, int n, int E,
                                                           const int* __restrict__ expert_map, int* __restrict__ offsets,
                                                           int* __restrict__ row_token, int* __restrict__ row_entry,
                                                           int* __restrict__ entry_row, int k, int pad) {
  extern __shared__ int sm[];
  int* cnt = sm;             // [E] running base per expert
  int* hist = sm + E;        // [32 warps][E] per-warp counts of the current chunk
  int* ccount = sm + 33 * E; // [E] counts
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < E; e += blockDim.x) ccount[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int e = ids[i];  // < 0: empty slot (expert-parallel receive regions)
    if (e >= 0 && expert_map) e = expert_map[e];
    if (e >= 0) atomicAdd(&ccount[e], 1);
  }
  __syncthreads();
  {  // segment starts: block-wide exclusive scan of the padded counts (each thread owns `per` experts)
    int* wsum = sm + 34 * E;  // [32]
    const int per = (E + blockDim.x - 1) / blockDim.x, e0 = threadIdx.x * per;
    int local = 0;
    for (int i = 0; i < per; ++i)
      if (e0 + i < E) local += (ccount[e0 + i] + pad - 1) / pad * pad;
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int nw = blockDim.x >> 5;
      int v = lane < nw ? wsum[lane] : 0, x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += u;
      }
      if (lane < nw) wsum[lane] = x - v;
    }
    __syncthreads();
    int base = wsum[warp] + incl - local;
    for (int i = 0; i < per; ++i)
      if (e0 + i < E) {
        offsets[e0 + i] = base;
        cnt[e0 + i] = base;
        base += (ccount[e0 + i] + pad - 1) / pad * pad;
      }
    if (threadIdx.x == blockDim.x - 1) offsets[E] = base;
  }
  __syncthreads();
  // pad rows
  for (int e = warp; e < E; e += 32) {
    const int start = offsets[e] + ccount[e], end = offsets[e + 1];
    for (int r = start + lane; r < end; r += 32) {
      row_token[r] = 0;
      row_entry[r] = -1;
    }
  }
  // stable positions, chunk of 1024 entries at a time
  for (int base = 0; base < n; base += blockDim.x) {
    for (int x = threadIdx.x; x < 32 * E; x += blockDim.x) hist[x] = 0;
    __syncthreads();
    const int i = base + threadIdx.x;
    int e = -1;
    if (i < n) {
      e = ids[i];
      if (e >= 0 && expert_map) e = expert_map[e];
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_in_warp = __popc(peers & ((1u << lane) - 1));
    if (e >= 0 && rank_in_warp == 0) hist[warp * E + e] = __popc(peers);
    __syncthreads();
    for (int x = threadIdx.x; x < E; x += blockDim.x) {
      int acc = cnt[x];
      for (int w = 0; w < 32; ++w) {
        const int c = hist[w * E + x];
        hist[w * E + x] = acc;
        acc += c;
      }
      cnt[x] = acc;
    }
    __syncthreads();
    if (e >= 0) {
      const int pos = hist[warp * E + e] + rank_in_warp;
      row_token[pos] = i / k;
      row_entry[pos] = i;
      entry_row[i] = pos;
    } else if (i < n) {
      entry_row[i] = -1;
    }
    __syncthreads();
  }
}

int expert_sort(const int* ids, int n, int E, const int* expert_map, int* offsets, int* row_token, int* row_entry,
                int* entry_row, int k, int pad, cudaStream_t st) {
  const size_t smem = (size_t)(34 * E + 32) * sizeof(int);
  if (smem > 200 * 1024) return 3;
  static std::atomic<uint64_t> attr_devs{0};
  if (const int e = smem_attr_once(attr_devs, (const void*)expert_sort_kernel, 200 * 1024)) return e;
  expert_sort_kernel<<<1, 1024, smem, st>>>(ids, n, E, expert_map, offsets, row_token, row_entry, entry_row, k,
                                              pad < 1 ? 1 : pad);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------ fp8 group quant + gather
// out_q[r, :] = e4m3(x[src(r), :] / s), s = amax/448 per 128-column group (1 if the group is all zero);
// src(r) = row_token[r] when given, else r. Scales are row-major [rows, K/128], or group-major
// [K/128, ld_s] when ld_s > 0 (the layout the expert GEMM reads). One warp per (row, group): lane owns 4 consecutive values.
__global__ void quant_rows_e4m3_kernel(const __nv_bfloat16* __restrict__ x, int ldx, const int* __restrict__ row_token,
                                       const int* __restrict__ nrows_dev, int nrows, int K,
                                       __nv_fp8_e4m3* __restrict__ q, float* __restrict__ scales, int ld_s) {
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int groups = K / 128;
  const int n = nrows_dev ? *nrows_dev : nrows;
  const int r = gw / groups, g = gw % groups;
  if (r >= n) return;
  const int src = row_token ? row_token[r] : r;
  const __nv_bfloat16* p = x + (size_t)src * ldx + g * 128 + lane * 4;
  uint2 raw = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
  float f[4];
  float a = 0.f;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    f[t] = __bfloat162float(h[t]);
    a = fmaxf(a, fabsf(f[t]));
  }
  a = warp_max(a);
  const float s = a > 0.f ? a / 448.f : 1.f;
  const float inv = 1.f / s;
  __nv_fp8x4_e4m3 o(make_float4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv));
  *reinterpret_cast<__nv_fp8x4_e4m3*>(q + (size_t)r * K + g * 128 + lane * 4) = o;
  if (lane == 0) scales[ld_s > 0 ? (size_t)g * ld_s + r : (size_t)r * groups + g] = s;
}

int quant_rows_e4m3(const void* x, int ldx, const int* row_token, const int* nrows_dev, int nrows, int K, void* q,
                    float* scales, int ld_s, cudaStream_t st) {
  if (K % 128) return 3;
  const int warps = 8;
  const long total = (long)nrows * (K / 128);
  if (total == 0) return 0;
  quant_rows_e4m3_kernel<<<(unsigned)((total + warps - 1) / warps), warps * 32, 0, st>>>(
      (const __nv_bfloat16*)x, ldx, row_token, nrows_dev, nrows, K, (__nv_fp8_e4m3*)q, scales, ld_s);
  return (int)cudaGetLastError();
}

// out_q[r, :] = e4m3(x[src(r), :] * (1 / s)) with ONE scale per row, s = max(amax of the row, 1e-30) / 448: the
// reference's W3A8 activation rule (training/work/qwen38fn_lora/int3_moe.py:108-118, Humming's per-row input
// quantisation). One warp per row; the second pass over the row re-reads it from L1/L2.
__global__ void quant_rows_e4m3_row_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                           const int* __restrict__ row_token, const int* __restrict__ nrows_dev,
                                           int nrows, int K, uint8_t* __restrict__ q, float* __restrict__ scales) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int n = nrows_dev ? min(*nrows_dev, nrows) : nrows;
  if (r >= n) return;
  const int src = row_token ? row_token[r] : r;
  const uint4* p = reinterpret_cast<const uint4*>(x + (size_t)src * ldx);
  const int nv = K / 8;
  float a = 0.f;
  for (int v = lane; v < nv; v += 32) {
    const uint4 raw = p[v];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      a = fmaxf(a, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
  a = warp_max(a);
  const float s = fmaxf(a, 1e-30f) / 448.f;
  const float inv = 1.f / s;
  uint2* out = reinterpret_cast<uint2*>(q + (size_t)r * K);
  for (int v = lane; v < nv; v += 32) {
    const uint4 raw = p[v];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x * inv;
      f[2 * i + 1] = t.y * inv;
    }
    const __nv_fp8x4_e4m3 lo(make_float4(f[0], f[1], f[2], f[3])), hi(make_float4(f[4], f[5], f[6], f[7]));
    out[v] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
  }
  if (lane == 0) scales[r] = s;
}

int quant_rows_e4m3_row(const void* x, int ldx, const int* row_token, const int* nrows_dev, int nrows, int K, void* q,
                        float* scales, cudaStream_t st) {
  if (K % 8 || ldx % 8) return 3;
  if (nrows <= 0) return 0;
  const int warps = 8;
  {
    const int pdl_rc = launch_pdl(quant_rows_e4m3_row_kernel, dim3((nrows + warps - 1) / warps), dim3(warps * 32), 0,
        st,
      (const __nv_bfloat16*)x, ldx, row_token, nrows_dev, nrows, K, (uint8_t*)q, scales);
    if (pdl_rc) return pdl_rc;
  }
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------ MoE combine
// out[t] = x_res[t] + sigmoid(sg[t]) * shared[t] + sum_j y[entry_row[t*k+j]]   (y already carries the route weight)
// sg is read from column `sg_col` of the router logits (the shared-expert gate rides along the router GEMM).
// entry_row null: y rows are the entries themselves (row t*k + j). Rows of y absent on this rank (entry_row < 0) are
// skipped. With `ew` (expert parallelism) every CTA first waits, bounded, until every rank has published this
// exchange's combine rows into this rank's region, and the last CTA counts the exchange consumed.
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ entry_row, int k,
                                   const __nv_bfloat16* __restrict__ shared, const float* __restrict__ router_logits,
                                   int ld_logits, int sg_col, const __nv_bfloat16* __restrict__ resid,
                                   __nv_bfloat16* __restrict__ out, int T, int H, EpArgs ew, uint32_t* status) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  // one CTA per token, one thread per 8 columns; all k row loads of a thread are issued before the sums
  const int t = blockIdx.x;
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  const bool waiting = ew.world > 0;
  if (waiting) {
    if (threadIdx.x == 0) {
      const uint64_t want = ew.expected[1] + 1;
      const uint64_t tw0 = globaltimer_ns();
      for (int p = 0; p < ew.world; ++p) {
        const uint64_t* f = reinterpret_cast<const uint64_t*>(ew.peer[ew.rank] + ew.off_flags) + EP_MAX_RANKS + p;
        const uint64_t t0 = globaltimer_ns();
        uint32_t polls = 0;
        while (ld_acquire_sys_u64(f) < want) {
          if ((++polls & 63) == 0 && globaltimer_ns() - t0 > AFB_WAIT_NS) {
            flag_error(status, AFB_ERR_PEER_TIMEOUT);
            break;
          }
          __nanosleep(64);
        }
      }
      if (ew.wait_ns && blockIdx.x == 0 && blockIdx.y == 0)
        atomicAdd(ew.wait_ns + 1, (unsigned long long)(globaltimer_ns() - tw0));
    }
    __syncthreads();
  }
  if (t < T && c < H) {
    float sg = 1.f;
    if (router_logits) sg = 1.f / (1.f + __expf(-router_logits[(size_t)t * ld_logits + sg_col]));
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    constexpr int KB = 4;  // rows in flight per batch
    for (int j0 = 0; j0 < k; j0 += KB) {
      uint4 q[KB];
#pragma unroll
      for (int u = 0; u < KB; ++u) {
        const int r = j0 + u < k ? (entry_row ? entry_row[t * k + j0 + u] : t * k + j0 + u) : -1;
        q[u] = r >= 0 ? *reinterpret_cast<const uint4*>(y + (size_t)r * H + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < KB; ++u) {  // slot order is kept: the sum is the same on every run and every rank count
        const __nv_bfloat16* hq = reinterpret_cast<const __nv_bfloat16*>(&q[u]);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += __bfloat162float(hq[i]);
      }
    }
    if (shared) {
      uint4 q = *reinterpret_cast<const uint4*>(shared + (size_t)t * H + c);
      const __nv_bfloat16* hq = reinterpret_cast<const __nv_bfloat16*>(&q);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += sg * __bfloat162float(hq[i]);
    }
    if (resid) {
      uint4 q = *reinterpret_cast<const uint4*>(resid + (size_t)t * H + c);
      const __nv_bfloat16* hq = reinterpret_cast<const __nv_bfloat16*>(&q);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += __bfloat162float(hq[i]);
    }
    *reinterpret_cast<uint4*>(out + (size_t)t * H + c) = make_uint4(
        pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
  }
  if (waiting && threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&ew.wait_done[1], 1u) == gridDim.x * gridDim.y - 1) {
      ew.wait_done[1] = 0;
      ew.expected[1] += 1;
    }
  }
}

int moe_combine(const void* y, const int* entry_row, int k, const void* shared, const float* router_logits,
                int ld_logits, int sg_col, const void* resid, void* out, int T, int H, cudaStream_t st,
                const EpArgs* wait_combine, uint32_t* status) {
  if (H % 8 || k > 64) return 3;
  EpArgs ew;
  if (wait_combine) ew = *wait_combine;
  else ew.world = 0;
  // a rank with no tokens still joins the exchange: one CTA waits and counts it consumed
  const int rows = T > 0 ? T : (wait_combine ? 1 : 0);
  if (rows <= 0) return 0;
  const int threads = 256;
  dim3 grid(rows, (H / 8 + threads - 1) / threads);
  {
    const int pdl_rc = launch_pdl(moe_combine_kernel, dim3(grid), dim3(threads), 0, st, (const __nv_bfloat16*)y,
        entry_row, k, (const __nv_bfloat16*)shared,
                                               router_logits, ld_logits, sg_col, (const __nv_bfloat16*)resid,
                                               (__nv_bfloat16*)out, T, H, ew, status);
    if (pdl_rc) return pdl_rc;
  }
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------ SwiGLU (dense)
// x [T, 2I] = [gate | up] -> y [T, I] = silu(gate) * up
__global__ void swiglu_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int T, int I) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const size_t i8 = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i8 >= (size_t)T * I) return;
  const size_t t = i8 / I, c = i8 % I;
  uint4 g = *reinterpret_cast<const uint4*>(x + t * 2 * I + c);
  uint4 u = *reinterpret_cast<const uint4*>(x + t * 2 * I + I + c);
  const __nv_bfloat16* gh = reinterpret_cast<const __nv_bfloat16*>(&g);
  const __nv_bfloat16* uh = reinterpret_cast<const __nv_bfloat16*>(&u);
  float o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = silu(__bfloat162float(gh[j])) * __bfloat162float(uh[j]);
  *reinterpret_cast<uint4*>(y + t * I + c) =
      make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
}

int swiglu(const void* x, void* y, int T, int I, cudaStream_t st) {
  if (I % 8) return 3;
  const size_t n = (size_t)T * I / 8;
  if (!n) return 0;
  {
    const int pdl_rc = launch_pdl(swiglu_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st,
        (const __nv_bfloat16*)x, (__nv_bfloat16*)y, T, I);
    if (pdl_rc) return pdl_rc;
  }
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------ embedding
__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* __restrict__ out, int T, int H, int V, uint32_t* status) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= V) {
    flag_error(status, AFB_ERR_BOUNDS);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)id * H);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

int embedding(const int* ids, const void* table, void* out, int T, int H, int V, uint32_t* status, cudaStream_t st) {
  if (H % 8) return 3;
  if (!T) return 0;
  if (const int pdl_rc = launch_pdl(embedding_kernel, dim3(T), dim3(128), 0, st, ids, (const __nv_bfloat16*)table,
      (__nv_bfloat16*)out, T, H, V, status)) return pdl_rc;
  return (int)cudaGetLastError();
}

}  // namespace afb
