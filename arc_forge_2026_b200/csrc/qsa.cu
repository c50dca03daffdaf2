// QSA block-sparse attention for speculative verify: indexer, block selection and the per-session page union.
//
// Semantics (the reference's QSA, training/work/qwen38fn_lora/sparse_qsa.py:83-153, with the block equal to one
// 64-token KV page so a selected block is exactly one page to fetch):
//   index query  q[t, h]  = RoPE_t(RMSNorm_q(x_t W_iq,h))                         (Hi heads of Di dims)
//   index key    k[b]     = RoPE_{64 b}(RMSNorm_k(mean_{j<64} x_{64b+j} W_ik))     (one key per finalised page,
//                                                                             stored by (session row, page index))
//   score[t, b] = sum_h relu(q[t,h] . k[b]) / sqrt(Di)
//   a verify row attends to the top-K finalised pages by score (all of them when there are <= K) plus the
//   "local" pages from the first non-finalised page through its own position (causal inside).
// A page is finalised (its pooled key written) once all its 64 tokens are committed; pages completed inside the
// current verify window are local, so rejected draft tokens never reach a pooled key.
//
// Kernels:
//   qsa_prep     -- per token: index query (norm + RoPE) into idx_q, raw index key into the per-token raw cache
//   qsa_finalize -- per (session, layer): pooled keys of pages that became complete since the last call
//   qsa_select   -- per session: scores of its W rows over its finalised pages, top-K per row by a radix
//                   threshold (ties to the lower page index), then the union of the rows' pages (ascending) +
//                   local pages, each with a bitmask of the rows that see it. paged_attn_kernel's sparse mode walks
//                   this union once for all W rows of the session.
#include "common.cuh"
#include "kernels.h"

namespace afb {

namespace qsa {
constexpr int DI = 128;  // index head dim
constexpr int MAXW = 8;  // verify rows per session
constexpr int MAXH = 4;  // index heads
constexpr int THREADS = 256;
}  // namespace qsa

// ------------------------------------------------------------------------------------------------ prep
// one warp per (token, j): j < Hi -> index query head j, j == Hi -> raw index key
__global__ void qsa_prep_kernel(QsaArgs a, const __nv_bfloat16* __restrict__ proj, int ld, int T,
                                const int* __restrict__ positions, const int* __restrict__ slots) {
  __shared__ float buf[8][qsa::DI];
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int per = a.Hi + 1;
  if (gw >= T * per) return;
  const int t = gw / per, j = gw % per;
  const __nv_bfloat16* src = proj + (size_t)t * ld + j * qsa::DI;  // [q heads | raw key] columns
  float v[4];
  {
    const uint2 raw = *reinterpret_cast<const uint2*>(src + lane * 4);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 x0 = __bfloat1622float2(h[0]), x1 = __bfloat1622float2(h[1]);
    v[0] = x0.x;
    v[1] = x0.y;
    v[2] = x1.x;
    v[3] = x1.y;
  }
  if (j == a.Hi) {  // raw key: stored as is (pooled and normalised at finalisation)
    *reinterpret_cast<uint2*>(a.idx_raw + (size_t)slots[t] * qsa::DI + lane * 4) =
        make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
    return;
  }
  const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
  const float inv = rsqrtf(ss / qsa::DI + a.eps);
  float* b = buf[threadIdx.x >> 5];
#pragma unroll
  for (int i = 0; i < 4; ++i) b[lane * 4 + i] = v[i] * inv * (1.f + __bfloat162float(a.q_norm[lane * 4 + i]));
  __syncwarp();
  const int half = a.rot / 2, p = positions[t];
  float o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = lane * 4 + i;
    o[i] = b[d];
    if (d < a.rot) {
      const int fi = d < half ? d : d - half;
      const float cs = a.cos_t[(size_t)p * half + fi], sn = a.sin_t[(size_t)p * half + fi];
      o[i] = d < half ? b[d] * cs - b[d + half] * sn : b[d] * cs + b[d - half] * sn;
    }
  }
  *reinterpret_cast<uint2*>(a.idx_q + ((size_t)t * a.Hi + j) * qsa::DI + lane * 4) =
      make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
}

int qsa_prep(const QsaArgs& a, const void* proj, int ld, int T, const int* positions, const int* slots,
             cudaStream_t st) {
  if (a.Di != qsa::DI || a.Hi < 1 || a.Hi > qsa::MAXH || a.rot > qsa::DI || a.rot % 2 || ld % 4) return 3;
  if (T <= 0) return 0;
  const int warps = 8, total = T * (a.Hi + 1);
  qsa_prep_kernel<<<(total + warps - 1) / warps, warps * 32, 0, st>>>(a, (const __nv_bfloat16*)proj, ld, T,
                                                                      positions, slots);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ finalize
// grid (sessions, layers); 128 threads = one per index dim. Pages [fin[s], ctx[s]/64) of session s get pooled keys.
__global__ void qsa_finalize_kernel(QsaFinalizeArgs f) {
  __shared__ float red[4];
  __shared__ float buf[qsa::DI];
  const int s = blockIdx.x, l = blockIdx.y, d = threadIdx.x;
  const int lo = f.fin[s], hi = min(f.ctx[s] / 64, f.max_pages);
  const __nv_bfloat16* raw = f.idx_raw[l];
  __nv_bfloat16* key = f.idx_key[l];
  for (int p = lo; p < hi; ++p) {
    const int page = f.block_table[(size_t)s * f.max_pages + p];
    float acc = 0.f;
    for (int j = 0; j < 64; ++j) acc += __bfloat162float(raw[((size_t)page * 64 + j) * qsa::DI + d]);
    const float m = __bfloat162float(__float2bfloat16(acc / 64.f));  // the pooled key is a bf16 value
    float ss = warp_sum(m * m);
    if ((d & 31) == 0) red[d >> 5] = ss;
    __syncthreads();
    ss = red[0] + red[1] + red[2] + red[3];
    const float x = m * rsqrtf(ss / qsa::DI + f.eps) * (1.f + __bfloat162float(f.k_norm[l][d]));
    buf[d] = x;
    __syncthreads();
    const int half = f.rot / 2, pos = p * 64;
    float o = x;
    if (d < f.rot) {
      const int fi = d < half ? d : d - half;
      const float cs = f.cos_t[(size_t)pos * half + fi], sn = f.sin_t[(size_t)pos * half + fi];
      o = d < half ? x * cs - buf[d + half] * sn : x * cs + buf[d - half] * sn;
    }
    key[((size_t)s * f.max_pages + p) * qsa::DI + d] = __float2bfloat16(o);
    __syncthreads();  // red / buf are reused by the next page
  }
}

__global__ void qsa_fin_update_kernel(int* fin, const int* ctx, int S, int max_pages) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s < S) fin[s] = min(ctx[s] / 64, max_pages);
}

int qsa_finalize(const QsaFinalizeArgs& f, int S, int layers, cudaStream_t st) {
  if (layers < 1 || layers > QSA_MAX_LAYERS || f.rot > qsa::DI || f.rot % 2) return 3;
  if (S <= 0) return 0;
  qsa_finalize_kernel<<<dim3(S, layers), qsa::DI, 0, st>>>(f);
  qsa_fin_update_kernel<<<(S + 127) / 128, 128, 0, st>>>(f.fin, f.ctx, S, f.max_pages);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ select
AFB_DEV uint32_t order_key(float x) {  // monotone map float -> uint32 (NaN-free inputs)
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

AFB_DEV int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(qsa::THREADS) qsa_select_kernel(QsaArgs a, QsaSelectArgs sa, uint32_t* status) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int s = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int W = sa.W, K = sa.K, Hi = a.Hi;
  const int F = min(sa.fin[s], sa.max_blocks);  // finalised pages (scored)
  if (tid == 0 && sa.fin[s] > sa.max_blocks) flag_error(status, AFB_ERR_BOUNDS);
  const int seq_len = sa.seq_lens[s];
  const int last_page = min((seq_len - 1) / 64, sa.max_pages - 1);
  float* qs = reinterpret_cast<float*>(smem_raw);                                        // [W*Hi][DI]
  float* score = qs + qsa::MAXW * qsa::MAXH * qsa::DI;                                   // [W][max_blocks]
  uint32_t* mask = reinterpret_cast<uint32_t*>(score + (size_t)qsa::MAXW * sa.max_blocks);  // [max_blocks]
  const int* bt = sa.block_table + (size_t)s * sa.max_pages;

  for (int b = tid; b < F; b += blockDim.x) mask[b] = F <= K ? (1u << W) - 1 : 0u;
  if (F > K) {
    for (int i = tid; i < W * Hi * qsa::DI; i += blockDim.x)
      qs[i] = __bfloat162float(a.idx_q[(size_t)s * W * Hi * qsa::DI + i]);
    __syncthreads();
    const float rs = rsqrtf((float)qsa::DI);
    for (int b = tid; b < F; b += blockDim.x) {
      const uint4* kr = reinterpret_cast<const uint4*>(a.idx_key + ((size_t)s * sa.max_pages + b) * qsa::DI);
      float acc[qsa::MAXW * qsa::MAXH];
#pragma unroll
      for (int i = 0; i < qsa::MAXW * qsa::MAXH; ++i) acc[i] = 0.f;
      for (int c = 0; c < qsa::DI / 8; ++c) {
        const uint4 u = kr[c];
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
        float kf[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 x = __bfloat1622float2(h2[i]);
          kf[2 * i] = x.x;
          kf[2 * i + 1] = x.y;
        }
#pragma unroll
        for (int r = 0; r < qsa::MAXW; ++r) {
#pragma unroll
          for (int h = 0; h < qsa::MAXH; ++h) {
            if (r < W && h < Hi) {  // accumulator slots at compile-time indices (r, h); q rows at r * Hi + h
              const float* qr = qs + (r * Hi + h) * qsa::DI + c * 8;
              const float4 q0 = *reinterpret_cast<const float4*>(qr);
              const float4 q1 = *reinterpret_cast<const float4*>(qr + 4);
              acc[r * qsa::MAXH + h] += q0.x * kf[0] + q0.y * kf[1] + q0.z * kf[2] + q0.w * kf[3] + q1.x * kf[4] +
                                        q1.y * kf[5] + q1.z * kf[6] + q1.w * kf[7];
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < qsa::MAXW; ++r) {
        if (r < W) {
          float sc = 0.f;
#pragma unroll
          for (int h = 0; h < qsa::MAXH; ++h)
            if (h < Hi) sc += fmaxf(acc[r * qsa::MAXH + h], 0.f);
          score[(size_t)r * sa.max_blocks + b] = sc * rs;
        }
      }
    }
    __syncthreads();
    // top-K per row: warp r finds the K-th largest order key bit by bit (MSB first), then marks the pages above
    // it and, in page order, as many equal to it as K still needs
    for (int r = warp; r < W; r += blockDim.x / 32) {
      const float* sr = score + (size_t)r * sa.max_blocks;
      uint32_t prefix = 0;
      for (int bit = 31; bit >= 0; --bit) {
        const uint32_t cand = prefix | (1u << bit);
        int c = 0;
        for (int b = lane; b < F; b += 32) c += order_key(sr[b]) >= cand;
        if (warp_sum_i(c) >= K) prefix = cand;
      }
      int above = 0;
      for (int b = lane; b < F; b += 32) above += order_key(sr[b]) > prefix;
      int need_eq = K - warp_sum_i(above);
      for (int base = 0; base < F; base += 32) {
        const int b = base + lane;
        const uint32_t k = b < F ? order_key(sr[b]) : 0u;
        if (b < F && k > prefix) atomicOr(&mask[b], 1u << r);
        const unsigned eq = __ballot_sync(0xffffffffu, b < F && k == prefix);
        if (need_eq > 0 && (eq >> lane & 1u) && __popc(eq & ((1u << lane) - 1)) < need_eq)
          atomicOr(&mask[b], 1u << r);
        need_eq -= __popc(eq);
      }
    }
  }
  __syncthreads();
  // union (ascending page index) + local pages, written by warp 0
  if (warp == 0) {
    int n = 0;
    int* up = sa.u_page + (size_t)s * sa.ucap;
    int* ul = sa.u_lpage + (size_t)s * sa.ucap;
    uint8_t* um = sa.u_mask + (size_t)s * sa.ucap;
    for (int base = 0; base < F; base += 32) {
      const int b = base + lane;
      const uint32_t m = b < F ? mask[b] : 0u;
      const unsigned on = __ballot_sync(0xffffffffu, m != 0);
      const int at = n + __popc(on & ((1u << lane) - 1));
      if (m && at < sa.ucap) {
        up[at] = bt[b];
        ul[at] = b;
        um[at] = (uint8_t)m;
      }
      n += __popc(on);
    }
    for (int p = F + lane; p <= last_page; p += 32) {  // local pages: row r sees page p if its position reaches it
      const int at = n + (p - F);
      uint32_t m = 0;
      for (int r = 0; r < W; ++r)
        if (seq_len - W + r >= p * 64) m |= 1u << r;
      if (at < sa.ucap) {
        up[at] = bt[p];
        ul[at] = p;
        um[at] = (uint8_t)m;
      }
    }
    n += max(0, last_page - F + 1);
    if (lane == 0) {
      if (n > sa.ucap) flag_error(status, AFB_ERR_BOUNDS);
      sa.u_count[s] = min(n, sa.ucap);
    }
  }
}

int qsa_select(const QsaArgs& a, const QsaSelectArgs& sa, int S, uint32_t* status, cudaStream_t st) {
  if (a.Di != qsa::DI || a.Hi < 1 || a.Hi > qsa::MAXH || sa.W < 1 || sa.W > qsa::MAXW || sa.K < 1 ||
      sa.max_blocks < 1 || sa.ucap < 1)
    return 3;
  if (S <= 0) return 0;
  const size_t smem = (size_t)qsa::MAXW * qsa::MAXH * qsa::DI * 4 + (size_t)qsa::MAXW * sa.max_blocks * 4 +
                      (size_t)sa.max_blocks * 4;
  if (smem > 220 * 1024) return 3;
  static std::atomic<uint64_t> attr_devs{0};
  if (const int e = smem_attr_once(attr_devs, (const void*)qsa_select_kernel, 220 * 1024)) return e;
  qsa_select_kernel<<<S, qsa::THREADS, smem, st>>>(a, sa, status);
  return (int)cudaGetLastError();
}

}  // namespace afb
