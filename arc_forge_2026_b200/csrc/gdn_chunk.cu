// Sequential inter-chunk state scan of the chunked gated delta rule (training forward and backward).
//
// Chunked form (WY representation of DeltaNet with the Gated-DeltaNet decay; the reference trains through
// FlashQLA's chunk scan, train/preflight.py:280-365): inside chunk i every quantity is a batched product, and only
// the [Dk, Dv] state S carries from chunk to chunk:
//   forward   X_i = U_i - W_i S_i                  S_{i+1} = e^{last_i} S_i + Kd_i^T X_i
//   backward  X_i = P_i + Kd_i dS_{i+1}           dS_i    = e^{last_i} dS_{i+1} + Qm_i - W_i^T X_i
// Both are one recurrence  X = Y + s1 * M1 St ;  St <- e^{last} St (+ Qm) + s2 * M2^T X  run forward (M1 = W,
// M2 = Kd, s1 = -1, s2 = +1) or in reverse (M1 = Kd, M2 = W, s1 = +1, s2 = -1). The kernel writes the state
// before every step and every X, which are all the backward needs.
//
// Columns of the state are independent (column c of X and of St only ever meets column c), so a CTA owns one
// 32-column slice of one (sequence, head): grid (B*H, Dv/32), 256 threads, the slice lives in registers
// (thread (rg, c) holds rows rg*DK/8 .. rg*DK/8 + DK/8 - 1 of column c; DK = 64 or 128) and in shared memory for
// the broadcast reads.
// fp32 throughout (the gradients of the decay are differences of large terms).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace afb {

namespace gck {
constexpr int C = 64, SL = 32, THREADS = 256;
template <int DK>
struct Smem {
  float m1[2][C][DK];  // double buffer: chunk i+1 lands by bulk copy while chunk i is computed
  float m2[2][C][DK];
  float st[DK][SL];
  float x[C][SL];
  uint64_t full[2];
  int ok;
};
}  // namespace gck

template <bool REV, int DK>
__global__ void __launch_bounds__(gck::THREADS) gdn_chunk_scan_kernel(GdnScanArgs a) {
  using namespace gck;
  constexpr int RPT = DK / 8;  // state rows per thread
  extern __shared__ uint8_t smem_raw[];
  Smem<DK>& sm = *reinterpret_cast<Smem<DK>*>((reinterpret_cast<uintptr_t>(smem_raw) + 15) & ~uintptr_t(15));
  const int bh = blockIdx.x, c0 = blockIdx.y * SL;
  const int t = threadIdx.x, c = t & 31, rg = t >> 5;
  const int n = a.n_chunks, Dv = a.Dv;
  const float s1 = REV ? 1.f : -1.f, s2 = REV ? -1.f : 1.f;

  float S[RPT];
#pragma unroll
  for (int j = 0; j < RPT; ++j)
    S[j] = a.init ? a.init[((size_t)bh * DK + rg * RPT + j) * Dv + c0 + c] : 0.f;
#pragma unroll
  for (int j = 0; j < RPT; ++j) sm.st[rg * RPT + j][c] = S[j];

  if (t == 0) {
    mbar_init(&sm.full[0], 1);
    mbar_init(&sm.full[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int step, int b) {  // thread 0: chunk of this step -> buffer b
    const int i = REV ? n - 1 - step : step;
    const size_t ci = (size_t)bh * n + i;
    mbar_arrive_expect_tx(&sm.full[b], 2u * C * DK * 4);
    bulk_load_1d(&sm.m1[b][0][0], a.m1 + ci * C * DK, C * DK * 4, &sm.full[b]);
    bulk_load_1d(&sm.m2[b][0][0], a.m2 + ci * C * DK, C * DK * 4, &sm.full[b]);
  };
  int issued = 0;
  if (t == 0) {
    issue(0, 0);
    issued = 1;
  }
  int step = 0;
  for (; step < n; ++step) {
    const int i = REV ? n - 1 - step : step;
    const size_t ci = (size_t)bh * n + i;
    const int b = step & 1;
    if (a.reset && (REV ? (i + 1 < n && a.reset[i + 1]) : a.reset[i])) {  // a new sequence starts here
#pragma unroll
      for (int j = 0; j < RPT; ++j) {
        S[j] = 0.f;
        sm.st[rg * RPT + j][c] = 0.f;
      }
    }
    // the other buffer was last read by the previous step, which every thread has finished
    if (t == 0 && step + 1 < n) {
      issue(step + 1, b ^ 1);
      ++issued;
    }
#pragma unroll
    for (int r = rg; r < C; r += 8) sm.x[r][c] = a.y[(ci * C + r) * Dv + c0 + c];
    // the state before this step (forward: S_i, reverse: dS_{i+1})
#pragma unroll
    for (int j = 0; j < RPT; ++j) a.states[(ci * DK + rg * RPT + j) * Dv + c0 + c] = S[j];
    if (t == 0) sm.ok = mbar_wait(&sm.full[b], (step >> 1) & 1, a.status) ? 1 : 0;
    __syncthreads();
    if (!sm.ok) break;
    const float(*m1)[DK] = sm.m1[b];
    const float(*m2)[DK] = sm.m2[b];
    // ---- X[r][c] = Y + s1 * sum_k M1[r][k] St[k][c], rows r = rg + 8 * j
    {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll 4
      for (int k = 0; k < DK; k += 4) {
        const float s0 = sm.st[k][c], sa = sm.st[k + 1][c], sb = sm.st[k + 2][c], sc = sm.st[k + 3][c];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 m = *reinterpret_cast<const float4*>(&m1[rg + 8 * j][k]);
          acc[j] = fmaf(m.x, s0, fmaf(m.y, sa, fmaf(m.z, sb, fmaf(m.w, sc, acc[j]))));
        }
      }
      __syncthreads();  // every thread has read St and the Y values it replaces below
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = rg + 8 * j;
        const float xv = sm.x[r][c] + s1 * acc[j];
        sm.x[r][c] = xv;
        a.x[(ci * C + r) * Dv + c0 + c] = xv;
      }
    }
    __syncthreads();
    // ---- St[k][c] = e^{last} St + Qm + s2 * sum_r M2[r][k] X[r][c], rows k = rg*RPT + j
    {
      const float dec = __expf(a.last[ci]);
      float acc[RPT];
#pragma unroll
      for (int j = 0; j < RPT; ++j) acc[j] = 0.f;
#pragma unroll 2
      for (int r = 0; r < C; ++r) {
        const float xv = sm.x[r][c];
        const float4* mr = reinterpret_cast<const float4*>(&m2[r][rg * RPT]);
#pragma unroll
        for (int q = 0; q < RPT / 4; ++q) {
          const float4 m = mr[q];
          acc[4 * q + 0] = fmaf(m.x, xv, acc[4 * q + 0]);
          acc[4 * q + 1] = fmaf(m.y, xv, acc[4 * q + 1]);
          acc[4 * q + 2] = fmaf(m.z, xv, acc[4 * q + 2]);
          acc[4 * q + 3] = fmaf(m.w, xv, acc[4 * q + 3]);
        }
      }
#pragma unroll
      for (int j = 0; j < RPT; ++j) {
        const float qm = REV && a.qm ? a.qm[(ci * DK + rg * RPT + j) * Dv + c0 + c] : 0.f;
        S[j] = dec * S[j] + qm + s2 * acc[j];
        sm.st[rg * RPT + j][c] = S[j];
      }
    }
    __syncthreads();
  }
  if (step < n && t == 0)  // a wait gave up: let the copies still in flight land before the CTA exits (bounded)
    for (int j = step + 1; j < issued; ++j) mbar_wait(&sm.full[j & 1], (j >> 1) & 1, a.status);
  if (a.final_state)
#pragma unroll
    for (int j = 0; j < RPT; ++j)
      a.final_state[((size_t)bh * DK + rg * RPT + j) * Dv + c0 + c] = (REV && a.reset && a.reset[0]) ? 0.f : S[j];
}

template <bool REV, int DK>
static int launch_scan(const GdnScanArgs& a, cudaStream_t st) {
  const size_t smem = sizeof(gck::Smem<DK>) + 16;
  static std::atomic<uint64_t> attr_devs{0};
  if (const int e = smem_attr_once(attr_devs, (const void*)gdn_chunk_scan_kernel<REV, DK>, (int)smem)) return e;
  gdn_chunk_scan_kernel<REV, DK><<<dim3(a.BH, a.Dv / gck::SL), gck::THREADS, smem, st>>>(a);
  return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------------------
// Tensor-core scan (Dk = 128): the same recurrence with bf16 operands and fp32 accumulation (the precision class of
// the chunk kernels the reference trains with: bf16 W / Kd / state operands, fp32 accumulators), the state slice
// carried in fp32 MMA accumulator registers from chunk to chunk.
//
// CTA = one (sequence-head, 32-column slice), 8 warps. Per step:
//   product 1  X = Y + s1 * M1 S      [64 x 32] = [64 x 128] [128 x 32]: warp w owns rows 16*(w/2).., columns
//                                     16*(w%2).. (two m16n8 tiles); A = M1 by ldmatrix from the swizzled tile,
//                                     B = the bf16 state copy by ldmatrix.trans
//   product 2  S = e^{last} S (+ Qm) + s2 * M2^T X   [128 x 32] = [128 x 64] [64 x 32]: warp w owns state rows
//                                     16w.. (four m16n8 tiles, the persistent accumulators); A = M2^T by
//                                     ldmatrix.trans of the same swizzled layout, B = bf16 (s2 * X)
// M1 / M2 tiles of the next step land by bulk copy while this step computes; Y / Qm / last of the next step are
// loaded into registers one step ahead.
namespace gct {
constexpr int C = 64, DK = 128, SL = 32, THREADS = 256, SP = 40;  // SP: bf16 pitch of the state / X copies
struct Smem {
  __nv_bfloat16 m1[2][C * DK];  // swizzled tiles, 16 KB each, double-buffered
  __nv_bfloat16 m2[2][C * DK];
  __nv_bfloat16 s[DK * SP];     // bf16 state slice [128][32] (pitch 40: conflict-free ldmatrix rows)
  __nv_bfloat16 x[C * SP];      // bf16 s2 * X [64][32]
  uint64_t full[2];
  int ok;
};
// byte offset of element (row, col) of a swizzled [64 x 128] bf16 tile, col a multiple of 8
AFB_DEV uint32_t tile_off(int row, int col) { return (uint32_t)(row * 256 + ((((col >> 3) ^ (row & 7))) << 4)); }
}  // namespace gct

__global__ void __launch_bounds__(256) gdn_pack_tiles_kernel(const float* __restrict__ src,
                                                             __nv_bfloat16* __restrict__ dst, int64_t tiles) {
  const int64_t chunks = tiles * gct::C * (gct::DK / 8);  // 16-byte output chunks
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < chunks; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tile = q / (gct::C * 16);
    const int r = (int)(q / 16 % gct::C), cc = (int)(q % 16);
    const float4* s4 = reinterpret_cast<const float4*>(src + (tile * gct::C + r) * gct::DK + cc * 8);
    const float4 a = s4[0], b = s4[1];
    uint4 o;
    o.x = pack_bf16x2(a.x, a.y);
    o.y = pack_bf16x2(a.z, a.w);
    o.z = pack_bf16x2(b.x, b.y);
    o.w = pack_bf16x2(b.z, b.w);
    *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(dst) + tile * gct::C * gct::DK * 2 + gct::tile_off(r, cc * 8)) =
        o;
  }
}

int gdn_pack_tiles(const float* src, __nv_bfloat16* dst, int64_t tiles, cudaStream_t st) {
  if (tiles < 1) return 0;
  const int64_t chunks = tiles * gct::C * (gct::DK / 8);
  const int blocks = (int)std::min<int64_t>((chunks + 255) / 256, 148 * 16);
  gdn_pack_tiles_kernel<<<blocks, 256, 0, st>>>(src, dst, tiles);
  return (int)cudaGetLastError();
}

template <bool REV>
__global__ void __launch_bounds__(gct::THREADS) gdn_chunk_scan_tc_kernel(GdnScanArgs a) {
  using namespace gct;
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int bh = blockIdx.x, c0 = blockIdx.y * SL;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
  const int n = a.n_chunks, Dv = a.Dv;
  const float s1 = REV ? 1.f : -1.f, s2 = REV ? -1.f : 1.f;
  // product-1 ownership: rows p1r .. p1r+15, columns p1c .. p1c+15 of the slice
  const int p1r = 16 * (w >> 1), p1c = 16 * (w & 1);
  // product-2 ownership: state rows 16w .. 16w+15, all 32 columns
  const int p2r = 16 * w;

  float S[4][4];  // tile j: (row p2r+g, cols 8j+2t, +1), (row p2r+g+8, same cols)
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = p2r + g + 8 * h, col = c0 + 8 * j + 2 * t;
      float2 v = make_float2(0.f, 0.f);
      if (a.init) v = *reinterpret_cast<const float2*>(a.init + ((size_t)bh * DK + row) * Dv + col);
      S[j][2 * h] = v.x;
      S[j][2 * h + 1] = v.y;
    }
  auto store_state_bf16 = [&]() {
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        *reinterpret_cast<uint32_t*>(&sm.s[(p2r + g + 8 * h) * SP + 8 * j + 2 * t]) =
            pack_bf16x2(S[j][2 * h], S[j][2 * h + 1]);
  };
  store_state_bf16();

  if (tid == 0) {
    mbar_init(&sm.full[0], 1);
    mbar_init(&sm.full[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto chunk_of = [&](int step) { return (size_t)bh * n + (REV ? n - 1 - step : step); };
  auto issue = [&](int step, int b) {  // thread 0: the M1 / M2 tiles of `step` -> buffer b
    const size_t ci = chunk_of(step);
    mbar_arrive_expect_tx(&sm.full[b], 2u * C * DK * 2);
    bulk_load_1d(sm.m1[b], a.m1h + ci * C * DK, C * DK * 2, &sm.full[b]);
    bulk_load_1d(sm.m2[b], a.m2h + ci * C * DK, C * DK * 2, &sm.full[b]);
  };
  // register prefetch of Y (product-1 positions), Qm (product-2 positions) and last
  float yn[2][4], qn[4][4], lastn = 0.f;
  auto load_next = [&](int step) {
    const size_t ci = chunk_of(step);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float2 v = *reinterpret_cast<const float2*>(a.y + (ci * C + p1r + g + 8 * h) * Dv + c0 + p1c + 8 * j + 2 * t);
        yn[j][2 * h] = v.x;
        yn[j][2 * h + 1] = v.y;
      }
    if (REV && a.qm) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float2 v =
              *reinterpret_cast<const float2*>(a.qm + (ci * DK + p2r + g + 8 * h) * Dv + c0 + 8 * j + 2 * t);
          qn[j][2 * h] = v.x;
          qn[j][2 * h + 1] = v.y;
        }
    }
    lastn = a.last[ci];
  };
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) qn[j][e] = 0.f;
  int issued = 0;
  if (tid == 0) {
    issue(0, 0);
    issued = 1;
  }
  load_next(0);
  const uint32_t m1_base[2] = {smem_u32(sm.m1[0]), smem_u32(sm.m1[1])};
  const uint32_t m2_base[2] = {smem_u32(sm.m2[0]), smem_u32(sm.m2[1])};
  const uint32_t s_base = smem_u32(sm.s), x_base = smem_u32(sm.x);
  const int lj = lane >> 3, li = lane & 7;  // ldmatrix: matrix index and row within it

  int step = 0;
  for (; step < n; ++step) {
    const size_t ci = chunk_of(step);
    const int b = step & 1;
    const int ic = REV ? n - 1 - step : step;
    if (a.reset && (REV ? (ic + 1 < n && a.reset[ic + 1]) : a.reset[ic])) {  // a new sequence starts here
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[j][e] = 0.f;
      store_state_bf16();  // read by product 1 only after the barrier below
    }
    float y[2][4], qm[4][4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) y[j][e] = yn[j][e];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) qm[j][e] = qn[j][e];
    const float dec = __expf(lastn);
    if (step + 1 < n) {
      if (tid == 0) {  // the other buffer was last read in the previous step, which every thread has finished
        issue(step + 1, b ^ 1);
        ++issued;
      }
      load_next(step + 1);
    }
    // the state before this step (forward: S_i, reverse: dS_{i+1})
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        *reinterpret_cast<float2*>(a.states + (ci * DK + p2r + g + 8 * h) * Dv + c0 + 8 * j + 2 * t) =
            make_float2(S[j][2 * h], S[j][2 * h + 1]);
    if (tid == 0) sm.ok = mbar_wait(&sm.full[b], (step >> 1) & 1, a.status) ? 1 : 0;
    __syncthreads();
    if (!sm.ok) break;
    // ---- product 1: X = Y + s1 * M1 S
    float acc[2][4] = {};
#pragma unroll
    for (int ks = 0; ks < DK / 16; ++ks) {
      uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
      const int ar = p1r + li + ((lj & 1) << 3), ac = 16 * ks + ((lj >> 1) << 3);
      ldsm_x4(m1_base[b] + tile_off(ar, ac), a0, a1, a2, a3);
      const int br = 16 * ks + li + ((lj & 1) << 3), bc = p1c + ((lj >> 1) << 3);
      ldsm_x4_t(s_base + (uint32_t)(br * SP + bc) * 2u, b0, b1, b2, b3);
      mma_bf16(acc[0], a0, a1, a2, a3, b0, b1);
      mma_bf16(acc[1], a0, a1, a2, a3, b2, b3);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = p1r + g + 8 * h, col = p1c + 8 * j + 2 * t;
        const float x0 = y[j][2 * h] + s1 * acc[j][2 * h], x1 = y[j][2 * h + 1] + s1 * acc[j][2 * h + 1];
        *reinterpret_cast<float2*>(a.x + (ci * C + row) * Dv + c0 + col) = make_float2(x0, x1);
        *reinterpret_cast<uint32_t*>(&sm.x[row * SP + col]) = pack_bf16x2(s2 * x0, s2 * x1);
      }
    __syncthreads();  // X complete; every read of the bf16 state copy done
    // ---- product 2: S = e^{last} S (+ Qm) + s2 * M2^T X
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) S[j][e] = dec * S[j][e] + qm[j][e];
#pragma unroll
    for (int ks = 0; ks < C / 16; ++ks) {
      uint32_t a0, a1, a2, a3, b0, b1, b2, b3, b4, b5, b6, b7;
      // A = M2^T: element (r, k) = M2[k][r]; stored rows are tokens k
      const int tr = 16 * ks + li + ((lj >> 1) << 3), tc = p2r + ((lj & 1) << 3);
      ldsm_x4_t(m2_base[b] + tile_off(tr, tc), a0, a1, a2, a3);
      const int br = 16 * ks + li + ((lj & 1) << 3);
      ldsm_x4_t(x_base + (uint32_t)(br * SP + ((lj >> 1) << 3)) * 2u, b0, b1, b2, b3);
      ldsm_x4_t(x_base + (uint32_t)(br * SP + 16 + ((lj >> 1) << 3)) * 2u, b4, b5, b6, b7);
      mma_bf16(S[0], a0, a1, a2, a3, b0, b1);
      mma_bf16(S[1], a0, a1, a2, a3, b2, b3);
      mma_bf16(S[2], a0, a1, a2, a3, b4, b5);
      mma_bf16(S[3], a0, a1, a2, a3, b6, b7);
    }
    store_state_bf16();
    __syncthreads();  // the bf16 state is complete for the next product 1; X reads done
  }
  if (step < n && tid == 0)  // a wait gave up: let the copies still in flight land before the CTA exits (bounded)
    for (int j = step + 1; j < issued; ++j) mbar_wait(&sm.full[j & 1], (j >> 1) & 1, a.status);
  if (a.final_state) {
    const float keep = (REV && a.reset && a.reset[0]) ? 0.f : 1.f;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        *reinterpret_cast<float2*>(a.final_state + ((size_t)bh * DK + p2r + g + 8 * h) * Dv + c0 + 8 * j + 2 * t) =
            make_float2(keep * S[j][2 * h], keep * S[j][2 * h + 1]);
  }
}

template <bool REV>
static int launch_scan_tc(const GdnScanArgs& a, cudaStream_t st) {
  const size_t smem = sizeof(gct::Smem) + 128;
  static std::atomic<uint64_t> attr_devs{0};
  if (const int e = smem_attr_once(attr_devs, (const void*)gdn_chunk_scan_tc_kernel<REV>, (int)smem)) return e;
  gdn_chunk_scan_tc_kernel<REV><<<dim3(a.BH, a.Dv / gct::SL), gct::THREADS, smem, st>>>(a);
  return (int)cudaGetLastError();
}

int gdn_chunk_scan(const GdnScanArgs& a, bool reverse, cudaStream_t st) {
  if (a.C != gck::C || (a.Dk != 64 && a.Dk != 128) || a.Dv % gck::SL || a.n_chunks < 1 || a.BH < 1) return 3;
  if (a.m1h || a.m2h) {
    if (!a.m1h || !a.m2h || a.Dk != gct::DK || a.Dv % gct::SL || a.Dv % 2) return 3;
    return reverse ? launch_scan_tc<true>(a, st) : launch_scan_tc<false>(a, st);
  }
  if (a.Dk == 128) return reverse ? launch_scan<true, 128>(a, st) : launch_scan<false, 128>(a, st);
  return reverse ? launch_scan<true, 64>(a, st) : launch_scan<false, 64>(a, st);
}

}  // namespace afb
