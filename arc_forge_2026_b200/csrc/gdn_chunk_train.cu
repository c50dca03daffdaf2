// Per-chunk work of the chunked gated delta rule for training (Dk = Dv = 128, chunks of 64 tokens), forward and
// backward, on tensor cores (mma.sync m16n8k16, bf16 operands, fp32 accumulation), around the inter-chunk scan of
// gdn_chunk.cu. One CTA per (sequence-head, chunk), 8 warps; warp w owns output rows 16*(w&3).. and the column
// half w>>2 of every per-chunk product. Operands sit in shared memory as padded bf16 tiles (pitch 136 / 72
// elements: conflict-free ldmatrix rows).
//
// Math of one chunk (C = 64 rows i, j; gc = within-chunk cumsum of the log decay g; Gam[i][j] = e^{gc_i - gc_j}):
//   forward  a = -strict_lower(beta k k^T * Gam)     A = (I - a)^-1 (forward substitution, fp32)
//            w = A (beta e^{gc} k)   u = A (beta v)   kd = e^{last - gc} k                 [fwd_prep]
//            scan: X = u - w S,  S <- e^{last} S + kd^T X                                   [gdn_chunk.cu]
//            o = e^{gc} (q S) + (q k^T * Gam_incl) X                                        [fwd_out]
//   backward P = attn^T dO, Qm = (e^{gc} q)^T dO                                            [bwd_prep]
//            reverse scan -> dS after each chunk (dnext) and du = dL/du                    [gdn_chunk.cu]
//            dq, dk (attention and decayed-key parts), dw = -du S^T, dL/dgc of these terms  [bwd_inter]
//            through w = A Kbg, u = A Vb, A = (I - a)^-1, a(k, beta, gc): dk, dv, dbeta, dgc;
//            dg = reverse cumsum of dgc within the chunk                                    [bwd_wy]
// This is the work the reference runs in FlashQLA's chunk kernels (train/preflight.py:280-365); here it is one
// kernel per stage with every reduction in a fixed order (the gradients are bitwise reproducible).
#include "common.cuh"
#include "kernels.h"

namespace afb {
namespace gtr {
constexpr int C = 64, D = 128, PW = 136, PN = 72, THREADS = 256;
using bf16 = __nv_bfloat16;

template <typename T>
AFB_DEV T& smem_as(uint8_t* raw) {
  return *reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(raw) + 127) & ~uintptr_t(127));
}

// acc[16 x 8*NT] += A[16 x K] B[K x 8*NT] for the warp's tile (rows m0.., cols n0..), operands in shared memory:
// A stored [m][k] (AT = false) or [k][m] (AT = true, A = X^T); B stored [k][n] (BT = false) or [n][k] (BT = true).
template <int NT, bool AT, bool BT>
AFB_DEV void mma_tile(float (&acc)[NT][4], uint32_t a_base, int pa, int m0, uint32_t b_base, int pb, int n0, int K) {
  const int lane = threadIdx.x & 31, lj = lane >> 3, li = lane & 7;
#pragma unroll 2
  for (int k0 = 0; k0 < K; k0 += 16) {
    uint32_t a0, a1, a2, a3;
    if (!AT)
      ldsm_x4(a_base + 2u * (uint32_t)((m0 + li + ((lj & 1) << 3)) * pa + k0 + ((lj >> 1) << 3)), a0, a1, a2, a3);
    else
      ldsm_x4_t(a_base + 2u * (uint32_t)((k0 + li + ((lj >> 1) << 3)) * pa + m0 + ((lj & 1) << 3)), a0, a1, a2, a3);
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      const int n = n0 + 8 * j;
      uint32_t b0, b1, b2, b3;
      if (!BT)
        ldsm_x4_t(b_base + 2u * (uint32_t)((k0 + li + ((lj & 1) << 3)) * pb + n + ((lj >> 1) << 3)), b0, b1, b2, b3);
      else
        ldsm_x4(b_base + 2u * (uint32_t)((n + li + ((lj >> 1) << 3)) * pb + k0 + ((lj & 1) << 3)), b0, b1, b2, b3);
      mma_bf16(acc[j], a0, a1, a2, a3, b0, b1);
      mma_bf16(acc[j + 1], a0, a1, a2, a3, b2, b3);
    }
  }
}

template <int NT>
AFB_DEV void zero(float (&acc)[NT][4]) {
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;
}

AFB_DEV void unpack8(const uint4& v, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(h[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}
AFB_DEV uint4 pack8(const float* f, float s) {
  uint4 o;
  o.x = pack_bf16x2(f[0] * s, f[1] * s);
  o.y = pack_bf16x2(f[2] * s, f[3] * s);
  o.z = pack_bf16x2(f[4] * s, f[5] * s);
  o.w = pack_bf16x2(f[6] * s, f[7] * s);
  return o;
}

// 64 rows (tokens t0..) of head h of a [B, T, H, 128] bf16 tensor -> padded tile; rows past T are zero. Every
// thread issues all of its loads before its first shared-memory store (memory-level parallelism).
constexpr int RV = C * 16 / THREADS;  // 16-byte row vectors per thread
AFB_DEV void load_rows(bf16* dst, const bf16* src, int b, int t0, int T, int H, int h) {
  uint4 v[RV];
#pragma unroll
  for (int u = 0; u < RV; ++u) {
    const int q = threadIdx.x + u * THREADS, r = q >> 4, cc = q & 15, t = t0 + r;
    v[u] = make_uint4(0, 0, 0, 0);
    if (t < T) v[u] = *reinterpret_cast<const uint4*>(src + (((size_t)b * T + t) * H + h) * D + cc * 8);
  }
#pragma unroll
  for (int u = 0; u < RV; ++u) {
    const int q = threadIdx.x + u * THREADS;
    *reinterpret_cast<uint4*>(dst + (q >> 4) * PW + (q & 15) * 8) = v[u];
  }
}
// contiguous fp32 [ROWS x 128] -> padded bf16 tile, 8 loads in flight per thread
template <int ROWS>
AFB_DEV void load_f32(bf16* dst, const float* src) {
  constexpr int N = ROWS * 32 / THREADS;
#pragma unroll
  for (int b0 = 0; b0 < N; b0 += 8) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int q = threadIdx.x + (b0 + u) * THREADS;
      v[u] = reinterpret_cast<const float4*>(src + (size_t)(q >> 5) * D)[q & 31];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int q = threadIdx.x + (b0 + u) * THREADS;
      uint2 o;
      o.x = pack_bf16x2(v[u].x, v[u].y);
      o.y = pack_bf16x2(v[u].z, v[u].w);
      *reinterpret_cast<uint2*>(dst + (q >> 5) * PW + (q & 31) * 4) = o;
    }
  }
}

// sum over the 4 lanes of a quad (the lanes holding one accumulator row)
AFB_DEV float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}

// byte offset of element (row, col) inside a swizzled [64 x 128] bf16 scan tile (see gdn_pack_tiles)
AFB_DEV uint32_t tile_byte(int row, int col) {
  return (uint32_t)(row * 256 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2);
}

struct Coord {
  int chunk, bh, b, h, hk, t0;
  size_t ci;
};
AFB_DEV Coord coord(const GdnTrainArgs& a) {
  Coord c;
  c.chunk = blockIdx.x;
  c.bh = blockIdx.y;
  c.b = c.bh / a.Hv;
  c.h = c.bh % a.Hv;
  c.hk = c.h / (a.Hv / a.Hk);
  c.t0 = c.chunk * C;
  c.ci = (size_t)c.bh * a.n + c.chunk;
  return c;
}
AFB_DEV size_t tok(const GdnTrainArgs& a, const Coord& c, int r) { return ((size_t)c.b * a.T + c.t0 + r) * a.Hv + c.h; }

// attn (or any 64x64 product with the decay): rows 16*(w&3).., cols 32*(w>>2)..; Gam[i][j] = e^{gc_i - gc_j}
AFB_DEV float gam(const float* gc, int i, int j, bool incl) {
  return (incl ? j <= i : j < i) ? __expf(gc[i] - gc[j]) : 0.f;
}

}  // namespace gtr

using namespace gtr;

// ------------------------------------------------------------------------------------------------ forward prep
struct PrepSmem {
  bf16 kr[C * PW], kb[C * PW], kbg[C * PW], vb[C * PW];
  bf16 As[C * PN];
  float am[C * C];
  float gc[C], beta[C], egc[C];
};

__global__ void __launch_bounds__(THREADS) gdn_train_fwd_prep_kernel(GdnTrainArgs a) {
  extern __shared__ uint8_t smem_raw[];
  PrepSmem& sm = smem_as<PrepSmem>(smem_raw);
  const Coord c = coord(a);
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
  if (w == 0) {  // within-chunk inclusive cumsum of g
    float gv[2], bv[2];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int r = lane + 32 * s;
      const bool ok = c.t0 + r < a.T;
      gv[s] = ok ? a.g[tok(a, c, r)] : 0.f;
      bv[s] = ok ? a.beta[tok(a, c, r)] : 0.f;
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1)
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const float y = __shfl_up_sync(0xffffffffu, gv[s], o);
        if (lane >= o) gv[s] += y;
      }
    gv[1] += __shfl_sync(0xffffffffu, gv[0], 31);
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      sm.gc[lane + 32 * s] = gv[s];
      sm.beta[lane + 32 * s] = bv[s];
      sm.egc[lane + 32 * s] = __expf(gv[s]);
    }
  }
  __syncthreads();
  const float last = sm.gc[C - 1];
  uint8_t* kd_tile = reinterpret_cast<uint8_t*>(a.kd_tiles + c.ci * C * D);
  {
    uint4 kv[RV], vv[RV];
#pragma unroll
    for (int u = 0; u < RV; ++u) {
      const int q = tid + u * THREADS, r = q >> 4, cc = q & 15, t = c.t0 + r;
      kv[u] = vv[u] = make_uint4(0, 0, 0, 0);
      if (t < a.T) {
        kv[u] = *reinterpret_cast<const uint4*>(a.k + (((size_t)c.b * a.T + t) * a.Hk + c.hk) * D + cc * 8);
        vv[u] = *reinterpret_cast<const uint4*>(a.v + (((size_t)c.b * a.T + t) * a.Hv + c.h) * D + cc * 8);
      }
    }
#pragma unroll
    for (int u = 0; u < RV; ++u) {
      const int q = tid + u * THREADS, r = q >> 4, cc = q & 15;
      float kf[8], vf[8];
      unpack8(kv[u], kf);
      unpack8(vv[u], vf);
      const float be = sm.beta[r];
      *reinterpret_cast<uint4*>(&sm.kr[r * PW + cc * 8]) = kv[u];
      *reinterpret_cast<uint4*>(&sm.kb[r * PW + cc * 8]) = pack8(kf, be);
      *reinterpret_cast<uint4*>(&sm.kbg[r * PW + cc * 8]) = pack8(kf, be * sm.egc[r]);
      *reinterpret_cast<uint4*>(&sm.vb[r * PW + cc * 8]) = pack8(vf, be);
      *reinterpret_cast<uint4*>(kd_tile + tile_byte(r, cc * 8)) = pack8(kf, __expf(last - sm.gc[r]));
    }
  }
  __syncthreads();
  const int mt = w & 3, nh = w >> 2;
  {  // a = -strict_lower((beta k) k^T * Gam)
    float acc[4][4];
    zero(acc);
    mma_tile<4, false, true>(acc, smem_u32(sm.kb), PW, 16 * mt, smem_u32(sm.kr), PW, 32 * nh, D);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 16 * mt + g8 + 8 * (e >> 1), jj = 32 * nh + 8 * j + 2 * t4 + (e & 1);
        sm.am[i * C + jj] = -acc[j][e] * gam(sm.gc, i, jj, false);
      }
  }
  __syncthreads();
  if (tid < C) {  // A = (I - a)^-1, one column per thread: x_i = delta_ic + sum_{j<i} a_ij x_j
    const int col = tid;
    float x[C];
#pragma unroll
    for (int i = 0; i < C; ++i) x[i] = 0.f;
#pragma unroll
    for (int i = 0; i < C; ++i) {
      float s = (i == col) ? 1.f : 0.f;
#pragma unroll
      for (int j4 = 0; j4 < (i + 3) / 4; ++j4) {  // a_ij = 0 and x_j = 0 for j >= i
        const float4 a4 = *reinterpret_cast<const float4*>(&sm.am[i * C + 4 * j4]);
        s = fmaf(a4.x, x[4 * j4], s);
        s = fmaf(a4.y, x[4 * j4 + 1], s);
        s = fmaf(a4.z, x[4 * j4 + 2], s);
        s = fmaf(a4.w, x[4 * j4 + 3], s);
      }
      x[i] = s;
    }
#pragma unroll
    for (int i = 0; i < C; ++i) {
      sm.As[i * PN + col] = __float2bfloat16(x[i]);
      a.A[(c.ci * C + i) * C + col] = x[i];
    }
  }
  __syncthreads();
  {  // w = A Kbg (swizzled bf16 scan tile), u = A Vb (fp32)
    float acc[8][4];
    zero(acc);
    mma_tile<8, false, false>(acc, smem_u32(sm.As), PN, 16 * mt, smem_u32(sm.kbg), PW, 64 * nh, C);
    uint8_t* w_tile = reinterpret_cast<uint8_t*>(a.w_tiles + c.ci * C * D);
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int row = 16 * mt + g8 + 8 * hh, col = 64 * nh + 8 * j + 2 * t4;
        *reinterpret_cast<uint32_t*>(w_tile + tile_byte(row, col)) = pack_bf16x2(acc[j][2 * hh], acc[j][2 * hh + 1]);
      }
    zero(acc);
    mma_tile<8, false, false>(acc, smem_u32(sm.As), PN, 16 * mt, smem_u32(sm.vb), PW, 64 * nh, C);
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int row = 16 * mt + g8 + 8 * hh, col = 64 * nh + 8 * j + 2 * t4;
        *reinterpret_cast<float2*>(a.u + (c.ci * C + row) * D + col) = make_float2(acc[j][2 * hh], acc[j][2 * hh + 1]);
      }
  }
  if (tid < C) a.gc[c.ci * C + tid] = sm.gc[tid];
  if (tid == 0) a.last[c.ci] = last;
}

// ------------------------------------------------------------------------------------------------ forward output
struct OutSmem {
  bf16 qs[C * PW], ks[C * PW], xs[C * PW];
  bf16 ss[D * PW];
  bf16 at[C * PN];
  float gc[C];
};

// attn = (q k^T) * Gam_incl of the warp's 16 x 32 tile -> bf16 tile `dst`
AFB_DEV void attn_tile(bf16* dst, uint32_t qs, uint32_t ks, const float* gc) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, g8 = lane >> 2, t4 = lane & 3, mt = w & 3, nh = w >> 2;
  float acc[4][4];
  zero(acc);
  mma_tile<4, false, true>(acc, qs, PW, 16 * mt, ks, PW, 32 * nh, D);
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int i = 16 * mt + g8 + 8 * hh, jj = 32 * nh + 8 * j + 2 * t4;
      *reinterpret_cast<uint32_t*>(&dst[i * PN + jj]) = pack_bf16x2(acc[j][2 * hh] * gam(gc, i, jj, true),
                                                                    acc[j][2 * hh + 1] * gam(gc, i, jj + 1, true));
    }
}

__global__ void __launch_bounds__(THREADS) gdn_train_fwd_out_kernel(GdnTrainArgs a) {
  extern __shared__ uint8_t smem_raw[];
  OutSmem& sm = smem_as<OutSmem>(smem_raw);
  const Coord c = coord(a);
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
  load_rows(sm.qs, a.q, c.b, c.t0, a.T, a.Hk, c.hk);
  load_rows(sm.ks, a.k, c.b, c.t0, a.T, a.Hk, c.hk);
  load_f32<C>(sm.xs, a.vnew + c.ci * C * D);
  load_f32<D>(sm.ss, a.states + c.ci * D * D);
  if (tid < C) sm.gc[tid] = a.gc[c.ci * C + tid];
  __syncthreads();
  attn_tile(sm.at, smem_u32(sm.qs), smem_u32(sm.ks), sm.gc);
  __syncthreads();
  const int mt = w & 3, nh = w >> 2;
  float acc[8][4];
  zero(acc);
  mma_tile<8, false, false>(acc, smem_u32(sm.qs), PW, 16 * mt, smem_u32(sm.ss), PW, 64 * nh, D);
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const float e = __expf(sm.gc[16 * mt + g8 + 8 * hh]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      acc[j][2 * hh] *= e;
      acc[j][2 * hh + 1] *= e;
    }
  }
  mma_tile<8, false, false>(acc, smem_u32(sm.at), PN, 16 * mt, smem_u32(sm.xs), PW, 64 * nh, C);
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int r = 16 * mt + g8 + 8 * hh;
    if (c.t0 + r >= a.T) continue;
    bf16* orow = a.o + tok(a, c, r) * D;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint32_t*>(orow + 64 * nh + 8 * j + 2 * t4) = pack_bf16x2(acc[j][2 * hh], acc[j][2 * hh + 1]);
  }
}

// ------------------------------------------------------------------------------------------------ backward prep
struct BPrepSmem {
  bf16 qs[C * PW], ks[C * PW], qd[C * PW], dos[C * PW];
  bf16 at[C * PN];
  float gc[C];
};

__global__ void __launch_bounds__(THREADS) gdn_train_bwd_prep_kernel(GdnTrainArgs a) {
  extern __shared__ uint8_t smem_raw[];
  BPrepSmem& sm = smem_as<BPrepSmem>(smem_raw);
  const Coord c = coord(a);
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
  if (tid < C) sm.gc[tid] = a.gc[c.ci * C + tid];
  load_rows(sm.ks, a.k, c.b, c.t0, a.T, a.Hk, c.hk);
  load_rows(sm.dos, a.dout, c.b, c.t0, a.T, a.Hv, c.h);
  __syncthreads();
  load_rows(sm.qs, a.q, c.b, c.t0, a.T, a.Hk, c.hk);
  __syncthreads();
  for (int q = tid; q < C * 16; q += THREADS) {  // q e^{gc}
    const int r = q >> 4, cc = q & 15;
    float f[8];
    unpack8(*reinterpret_cast<const uint4*>(&sm.qs[r * PW + cc * 8]), f);
    *reinterpret_cast<uint4*>(&sm.qd[r * PW + cc * 8]) = pack8(f, __expf(sm.gc[r]));
  }
  __syncthreads();
  attn_tile(sm.at, smem_u32(sm.qs), smem_u32(sm.ks), sm.gc);
  __syncthreads();
  const int mt = w & 3, nh = w >> 2;
  {  // P = attn^T dO
    float acc[8][4];
    zero(acc);
    mma_tile<8, true, false>(acc, smem_u32(sm.at), PN, 16 * mt, smem_u32(sm.dos), PW, 64 * nh, C);
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int row = 16 * mt + g8 + 8 * hh, col = 64 * nh + 8 * j + 2 * t4;
        *reinterpret_cast<float2*>(a.P + (c.ci * C + row) * D + col) = make_float2(acc[j][2 * hh], acc[j][2 * hh + 1]);
      }
  }
  {  // Qm = (q e^{gc})^T dO: warp w owns rows 16w.. of the 128 x 128 product
    float acc[16][4];
    zero(acc);
    mma_tile<16, true, false>(acc, smem_u32(sm.qd), PW, 16 * w, smem_u32(sm.dos), PW, 0, C);
#pragma unroll
    for (int j = 0; j < 16; ++j)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int row = 16 * w + g8 + 8 * hh, col = 8 * j + 2 * t4;
        *reinterpret_cast<float2*>(a.Qm + (c.ci * D + row) * D + col) = make_float2(acc[j][2 * hh], acc[j][2 * hh + 1]);
      }
  }
}

// ------------------------------------------------------------------------------------------------ backward: inter
struct BInterSmem {
  bf16 qs[C * PW], ks[C * PW], dos[C * PW], xs[C * PW], dus[C * PW];
  bf16 ss[D * PW], dns[D * PW];
  bf16 dag[C * PN];
  float G[C * (C + 1)];
  float gc[C], rowv[C], colv[C];
  float part[2][C];  // per column-half partial row sums
  float part2[2][C];
  float red[8];
};

__global__ void __launch_bounds__(THREADS) gdn_train_bwd_inter_kernel(GdnTrainArgs a) {
  extern __shared__ uint8_t smem_raw[];
  BInterSmem& sm = smem_as<BInterSmem>(smem_raw);
  const Coord c = coord(a);
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
  const int mt = w & 3, nh = w >> 2;
  load_rows(sm.qs, a.q, c.b, c.t0, a.T, a.Hk, c.hk);
  load_rows(sm.ks, a.k, c.b, c.t0, a.T, a.Hk, c.hk);
  load_rows(sm.dos, a.dout, c.b, c.t0, a.T, a.Hv, c.h);
  load_f32<C>(sm.xs, a.vnew + c.ci * C * D);
  load_f32<C>(sm.dus, a.du + c.ci * C * D);
  float sdot = 0.f;  // sum(dnext * S)
  {
    const float* S = a.states + c.ci * D * D;
    const float* N = a.dnext + c.ci * D * D;
    constexpr int NQ = D * 32 / THREADS;
#pragma unroll
    for (int b0 = 0; b0 < NQ; b0 += 4) {
      float4 s4[4], n4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int q = tid + (b0 + u) * THREADS;
        s4[u] = reinterpret_cast<const float4*>(S + (size_t)(q >> 5) * D)[q & 31];
        n4[u] = reinterpret_cast<const float4*>(N + (size_t)(q >> 5) * D)[q & 31];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int q = tid + (b0 + u) * THREADS, r = q >> 5, c4 = q & 31;
        sdot += s4[u].x * n4[u].x + s4[u].y * n4[u].y + s4[u].z * n4[u].z + s4[u].w * n4[u].w;
        uint2 o;
        o.x = pack_bf16x2(s4[u].x, s4[u].y);
        o.y = pack_bf16x2(s4[u].z, s4[u].w);
        *reinterpret_cast<uint2*>(&sm.ss[r * PW + c4 * 4]) = o;
        o.x = pack_bf16x2(n4[u].x, n4[u].y);
        o.y = pack_bf16x2(n4[u].z, n4[u].w);
        *reinterpret_cast<uint2*>(&sm.dns[r * PW + c4 * 4]) = o;
      }
    }
  }
  sdot = warp_sum(sdot);
  if (lane == 0) sm.red[w] = sdot;
  if (tid < C) sm.gc[tid] = a.gc[c.ci * C + tid];
  __syncthreads();
  const float last = sm.gc[C - 1];
  {  // attn (recomputed), dattn = dO X^T; G = dattn * attn; dag = dattn * Gam_incl
    float qa[4][4], da[4][4];
    zero(qa);
    zero(da);
    mma_tile<4, false, true>(qa, smem_u32(sm.qs), PW, 16 * mt, smem_u32(sm.ks), PW, 32 * nh, D);
    mma_tile<4, false, true>(da, smem_u32(sm.dos), PW, 16 * mt, smem_u32(sm.xs), PW, 32 * nh, D);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = 16 * mt + g8 + 8 * hh, jj = 32 * nh + 8 * j + 2 * t4;
        const float ga = gam(sm.gc, i, jj, true), gb = gam(sm.gc, i, jj + 1, true);
        sm.G[i * (C + 1) + jj] = da[j][2 * hh] * qa[j][2 * hh] * ga;
        sm.G[i * (C + 1) + jj + 1] = da[j][2 * hh + 1] * qa[j][2 * hh + 1] * gb;
        *reinterpret_cast<uint32_t*>(&sm.dag[i * PN + jj]) = pack_bf16x2(da[j][2 * hh] * ga, da[j][2 * hh + 1] * gb);
      }
  }
  __syncthreads();
  if (tid < C) {  // fixed-order row and column sums of G
    float rs = 0.f, cs = 0.f;
    for (int j = 0; j < C; ++j) {
      rs += sm.G[tid * (C + 1) + j];
      cs += sm.G[j * (C + 1) + tid];
    }
    sm.rowv[tid] = rs;
    sm.colv[tid] = cs;
  }
  {  // dq = e^{gc} (dO S^T) + dag k;  dgc += e^{gc} rowsum(dO S^T * q)
    float acc[8][4];
    zero(acc);
    mma_tile<8, false, true>(acc, smem_u32(sm.dos), PW, 16 * mt, smem_u32(sm.ss), PW, 64 * nh, D);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = 16 * mt + g8 + 8 * hh;
      const float e = __expf(sm.gc[r]);
      float p = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = 64 * nh + 8 * j + 2 * t4;
        const float2 qv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sm.qs[r * PW + col]));
        p += acc[j][2 * hh] * qv.x + acc[j][2 * hh + 1] * qv.y;
        acc[j][2 * hh] *= e;
        acc[j][2 * hh + 1] *= e;
      }
      p = quad_sum(p) * e;
      if (t4 == 0) sm.part[nh][r] = p;
    }
    mma_tile<8, false, false>(acc, smem_u32(sm.dag), PN, 16 * mt, smem_u32(sm.ks), PW, 64 * nh, C);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = 16 * mt + g8 + 8 * hh;
      if (c.t0 + r >= a.T) continue;
      float* dq = a.dq + tok(a, c, r) * D;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float2*>(dq + 64 * nh + 8 * j + 2 * t4) = make_float2(acc[j][2 * hh], acc[j][2 * hh + 1]);
    }
  }
  {  // dk = dag^T q + e^{last - gc} (X dnext^T);  E = rowsum(e^{last-gc} (X dnext^T) * k)
    float acc[8][4], kd[8][4];
    zero(acc);
    zero(kd);
    mma_tile<8, true, false>(acc, smem_u32(sm.dag), PN, 16 * mt, smem_u32(sm.qs), PW, 64 * nh, C);
    mma_tile<8, false, true>(kd, smem_u32(sm.xs), PW, 16 * mt, smem_u32(sm.dns), PW, 64 * nh, D);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = 16 * mt + g8 + 8 * hh;
      const float e = __expf(last - sm.gc[r]);
      float p = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = 64 * nh + 8 * j + 2 * t4;
        const float2 kv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sm.ks[r * PW + col]));
        p += kd[j][2 * hh] * kv.x + kd[j][2 * hh + 1] * kv.y;
        acc[j][2 * hh] += e * kd[j][2 * hh];
        acc[j][2 * hh + 1] += e * kd[j][2 * hh + 1];
      }
      p = quad_sum(p) * e;
      if (t4 == 0) sm.part2[nh][r] = p;
      if (c.t0 + r >= a.T) continue;
      float* dk = a.dk + tok(a, c, r) * D;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float2*>(dk + 64 * nh + 8 * j + 2 * t4) = make_float2(acc[j][2 * hh], acc[j][2 * hh + 1]);
    }
  }
  {  // dw = -du S^T
    float acc[8][4];
    zero(acc);
    mma_tile<8, false, true>(acc, smem_u32(sm.dus), PW, 16 * mt, smem_u32(sm.ss), PW, 64 * nh, D);
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int row = 16 * mt + g8 + 8 * hh, col = 64 * nh + 8 * j + 2 * t4;
        *reinterpret_cast<float2*>(a.dw + (c.ci * C + row) * D + col) =
            make_float2(-acc[j][2 * hh], -acc[j][2 * hh + 1]);
      }
  }
  __syncthreads();
  if (w == 0) {  // dgc of this part; dlast = sum(E) + e^{last} sum(dnext * S) goes to the last row
    float tot = 0.f;
    for (int i = 0; i < 8; ++i) tot += sm.red[i];
    float e0 = sm.part2[0][lane] + sm.part2[1][lane], e1 = sm.part2[0][lane + 32] + sm.part2[1][lane + 32];
    float es = warp_sum(e0 + e1);
    for (int s = 0; s < 2; ++s) {
      const int r = lane + 32 * s;
      float d = sm.part[0][r] + sm.part[1][r] + sm.rowv[r] - sm.colv[r] - (s ? e1 : e0);
      if (r == C - 1) d += es + __expf(last) * tot;
      a.dgc[c.ci * C + r] = d;
    }
  }
}

// ------------------------------------------------------------------------------------------------ backward: WY
struct BWySmem {
  bf16 ks[C * PW], kb[C * PW], kbg[C * PW], vs[C * PW], vb[C * PW], dus[C * PW], dws[C * PW];
  bf16 As[C * PN], dAs[C * PN], T1[C * PN], dmg[C * PN];
  float G[C * (C + 1)];
  float gc[C], beta[C], egc[C], rowv[C], colv[C];
  float pb[2][C], pg[2][C];  // per column-half partials: dbeta, dgc
};

__global__ void __launch_bounds__(THREADS) gdn_train_bwd_wy_kernel(GdnTrainArgs a) {
  extern __shared__ uint8_t smem_raw[];
  BWySmem& sm = smem_as<BWySmem>(smem_raw);
  const Coord c = coord(a);
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
  const int mt = w & 3, nh = w >> 2;
  if (tid < C) {
    const bool ok = c.t0 + tid < a.T;
    sm.gc[tid] = a.gc[c.ci * C + tid];
    sm.beta[tid] = ok ? a.beta[tok(a, c, tid)] : 0.f;
    sm.egc[tid] = __expf(sm.gc[tid]);
  }
  load_f32<C>(sm.dus, a.du + c.ci * C * D);
  load_f32<C>(sm.dws, a.dw + c.ci * C * D);
  {  // A -> bf16
    float4 v[C * C / 4 / THREADS];
#pragma unroll
    for (int u = 0; u < C * C / 4 / THREADS; ++u) {
      const int q = tid + u * THREADS;
      v[u] = reinterpret_cast<const float4*>(a.A + (c.ci * C + (q >> 4)) * C)[q & 15];
    }
#pragma unroll
    for (int u = 0; u < C * C / 4 / THREADS; ++u) {
      const int q = tid + u * THREADS;
      uint2 o;
      o.x = pack_bf16x2(v[u].x, v[u].y);
      o.y = pack_bf16x2(v[u].z, v[u].w);
      *reinterpret_cast<uint2*>(&sm.As[(q >> 4) * PN + (q & 15) * 4]) = o;
    }
  }
  __syncthreads();
  {
    uint4 kv[RV], vv[RV];
#pragma unroll
    for (int u = 0; u < RV; ++u) {
      const int q = tid + u * THREADS, r = q >> 4, cc = q & 15, t = c.t0 + r;
      kv[u] = vv[u] = make_uint4(0, 0, 0, 0);
      if (t < a.T) {
        kv[u] = *reinterpret_cast<const uint4*>(a.k + (((size_t)c.b * a.T + t) * a.Hk + c.hk) * D + cc * 8);
        vv[u] = *reinterpret_cast<const uint4*>(a.v + (((size_t)c.b * a.T + t) * a.Hv + c.h) * D + cc * 8);
      }
    }
#pragma unroll
    for (int u = 0; u < RV; ++u) {
      const int q = tid + u * THREADS, r = q >> 4, cc = q & 15;
      float kf[8], vf[8];
      unpack8(kv[u], kf);
      unpack8(vv[u], vf);
      const float be = sm.beta[r];
      *reinterpret_cast<uint4*>(&sm.ks[r * PW + cc * 8]) = kv[u];
      *reinterpret_cast<uint4*>(&sm.vs[r * PW + cc * 8]) = vv[u];
      *reinterpret_cast<uint4*>(&sm.kb[r * PW + cc * 8]) = pack8(kf, be);
      *reinterpret_cast<uint4*>(&sm.kbg[r * PW + cc * 8]) = pack8(kf, be * sm.egc[r]);
      *reinterpret_cast<uint4*>(&sm.vb[r * PW + cc * 8]) = pack8(vf, be);
    }
  }
  __syncthreads();
  {  // dA = du Vb^T + dw Kbg^T
    float acc[4][4];
    zero(acc);
    mma_tile<4, false, true>(acc, smem_u32(sm.dus), PW, 16 * mt, smem_u32(sm.vb), PW, 32 * nh, D);
    mma_tile<4, false, true>(acc, smem_u32(sm.dws), PW, 16 * mt, smem_u32(sm.kbg), PW, 32 * nh, D);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = 16 * mt + g8 + 8 * hh, jj = 32 * nh + 8 * j + 2 * t4;
        *reinterpret_cast<uint32_t*>(&sm.dAs[i * PN + jj]) = pack_bf16x2(acc[j][2 * hh], acc[j][2 * hh + 1]);
      }
  }
  float dk[8][4];  // this CTA's dk rows (column half nh), accumulated over the WY terms
  float pbeta[2] = {0.f, 0.f}, pgc[2] = {0.f, 0.f};
  {  // dVb = A^T du -> dv = beta dVb, dbeta += v . dVb;  dKbg = A^T dw -> dk, dbeta, dgc
    float acc[8][4];
    zero(acc);
    mma_tile<8, true, false>(acc, smem_u32(sm.As), PN, 16 * mt, smem_u32(sm.dus), PW, 64 * nh, C);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = 16 * mt + g8 + 8 * hh;
      const float be = sm.beta[r];
      float p = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = 64 * nh + 8 * j + 2 * t4;
        const float2 vv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sm.vs[r * PW + col]));
        p += acc[j][2 * hh] * vv.x + acc[j][2 * hh + 1] * vv.y;
      }
      pbeta[hh] += quad_sum(p);
      if (c.t0 + r < a.T) {
        float* dv = a.dv + tok(a, c, r) * D;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float2*>(dv + 64 * nh + 8 * j + 2 * t4) =
              make_float2(be * acc[j][2 * hh], be * acc[j][2 * hh + 1]);
      }
    }
    zero(acc);
    mma_tile<8, true, false>(acc, smem_u32(sm.As), PN, 16 * mt, smem_u32(sm.dws), PW, 64 * nh, C);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = 16 * mt + g8 + 8 * hh;
      const float be = sm.beta[r], eg = sm.egc[r];
      float p = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = 64 * nh + 8 * j + 2 * t4;
        const float2 kv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sm.ks[r * PW + col]));
        p += acc[j][2 * hh] * kv.x + acc[j][2 * hh + 1] * kv.y;
        dk[j][2 * hh] = be * eg * acc[j][2 * hh];
        dk[j][2 * hh + 1] = be * eg * acc[j][2 * hh + 1];
      }
      p = quad_sum(p);
      pbeta[hh] += eg * p;
      pgc[hh] += be * eg * p;
    }
  }
  __syncthreads();  // dA complete
  {  // T1 = A^T dA
    float acc[4][4];
    zero(acc);
    mma_tile<4, true, false>(acc, smem_u32(sm.As), PN, 16 * mt, smem_u32(sm.dAs), PN, 32 * nh, C);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = 16 * mt + g8 + 8 * hh, jj = 32 * nh + 8 * j + 2 * t4;
        *reinterpret_cast<uint32_t*>(&sm.T1[i * PN + jj]) = pack_bf16x2(acc[j][2 * hh], acc[j][2 * hh + 1]);
      }
  }
  __syncthreads();
  {  // da = strict_lower(T1 A^T), dM = -da; M = (beta k) k^T * Gam; G = dM * M; dmg = dM * Gam
    float t2[4][4], mm[4][4];
    zero(t2);
    zero(mm);
    mma_tile<4, false, true>(t2, smem_u32(sm.T1), PN, 16 * mt, smem_u32(sm.As), PN, 32 * nh, C);
    mma_tile<4, false, true>(mm, smem_u32(sm.kb), PW, 16 * mt, smem_u32(sm.ks), PW, 32 * nh, D);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = 16 * mt + g8 + 8 * hh, jj = 32 * nh + 8 * j + 2 * t4;
        float dmg2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float ga = gam(sm.gc, i, jj + e, false);
          const float dm = (jj + e < i) ? -t2[j][2 * hh + e] : 0.f;
          sm.G[i * (C + 1) + jj + e] = dm * mm[j][2 * hh + e] * ga;
          dmg2[e] = dm * ga;
        }
        *reinterpret_cast<uint32_t*>(&sm.dmg[i * PN + jj]) = pack_bf16x2(dmg2[0], dmg2[1]);
      }
  }
  __syncthreads();
  if (tid < C) {
    float rs = 0.f, cs = 0.f;
    for (int j = 0; j < C; ++j) {
      rs += sm.G[tid * (C + 1) + j];
      cs += sm.G[j * (C + 1) + tid];
    }
    sm.rowv[tid] = rs;
    sm.colv[tid] = cs;
  }
  {  // dkb = dmg k -> dk += beta dkb, dbeta += k . dkb;  dk += dmg^T (beta k)
    float acc[8][4];
    zero(acc);
    mma_tile<8, false, false>(acc, smem_u32(sm.dmg), PN, 16 * mt, smem_u32(sm.ks), PW, 64 * nh, C);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = 16 * mt + g8 + 8 * hh;
      const float be = sm.beta[r];
      float p = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = 64 * nh + 8 * j + 2 * t4;
        const float2 kv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sm.ks[r * PW + col]));
        p += acc[j][2 * hh] * kv.x + acc[j][2 * hh + 1] * kv.y;
        dk[j][2 * hh] += be * acc[j][2 * hh];
        dk[j][2 * hh + 1] += be * acc[j][2 * hh + 1];
      }
      pbeta[hh] += quad_sum(p);
    }
    mma_tile<8, true, false>(dk, smem_u32(sm.dmg), PN, 16 * mt, smem_u32(sm.kb), PW, 64 * nh, C);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = 16 * mt + g8 + 8 * hh;
      if (t4 == 0) {
        sm.pb[nh][r] = pbeta[hh];
        sm.pg[nh][r] = pgc[hh];
      }
      if (c.t0 + r >= a.T) continue;
      float* dkr = a.dk + tok(a, c, r) * D;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float2* p = reinterpret_cast<float2*>(dkr + 64 * nh + 8 * j + 2 * t4);
        const float2 prev = *p;  // the inter-chunk part written by gdn_train_bwd_inter
        *p = make_float2(prev.x + dk[j][2 * hh], prev.y + dk[j][2 * hh + 1]);
      }
    }
  }
  __syncthreads();
  if (w == 0) {  // total dgc, then dg = reverse cumsum within the chunk; dbeta
    float d[2];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int r = lane + 32 * s;
      d[s] = a.dgc[c.ci * C + r] + sm.pg[0][r] + sm.pg[1][r] + sm.rowv[r] - sm.colv[r];
    }
    // suffix sums: dg_i = sum_{i' >= i} dgc_i'
#pragma unroll
    for (int o = 1; o < 32; o <<= 1)
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const float y = __shfl_down_sync(0xffffffffu, d[s], o);
        if (lane + o < 32) d[s] += y;
      }
    d[0] += __shfl_sync(0xffffffffu, d[1], 0);
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int r = lane + 32 * s;
      if (c.t0 + r < a.T) {
        a.dg[tok(a, c, r)] = d[s];
        a.dbeta[tok(a, c, r)] = sm.pb[0][r] + sm.pb[1][r];
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------ launchers
template <typename SM, typename K>
static int launch(K kernel, const GdnTrainArgs& a, cudaStream_t st) {
  if (a.Hk < 1 || a.Hv % a.Hk || a.n < 1 || a.B < 1) return 3;
  const size_t smem = sizeof(SM) + 128;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kernel<<<dim3(a.n, a.B * a.Hv), THREADS, smem, st>>>(a);
  return (int)cudaGetLastError();
}

int gdn_train_fwd_prep(const GdnTrainArgs& a, cudaStream_t st) {
  return launch<PrepSmem>(gdn_train_fwd_prep_kernel, a, st);
}
int gdn_train_fwd_out(const GdnTrainArgs& a, cudaStream_t st) { return launch<OutSmem>(gdn_train_fwd_out_kernel, a, st); }
int gdn_train_bwd_prep(const GdnTrainArgs& a, cudaStream_t st) {
  return launch<BPrepSmem>(gdn_train_bwd_prep_kernel, a, st);
}
int gdn_train_bwd_inter(const GdnTrainArgs& a, cudaStream_t st) {
  return launch<BInterSmem>(gdn_train_bwd_inter_kernel, a, st);
}
int gdn_train_bwd_wy(const GdnTrainArgs& a, cudaStream_t st) { return launch<BWySmem>(gdn_train_bwd_wy_kernel, a, st); }

}  // namespace afb
