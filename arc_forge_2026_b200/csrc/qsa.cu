// QSA block-sparse attention for speculative verify: indexer, block selection and the per-session block union.
//
// Semantics (the reference's QSA, training/work/qwen38fn_lora/sparse_qsa.py:83-153; block = `block` tokens, a divisor
// of the 64-token KV page -- 4 for the reference's own model, 64 for BASELINE config 5):
//   index query  q[t, h]  = RoPE_t(RMSNorm_q(x_t W_iq,h))                            (Hi heads of Di dims)
//   index key    k[b]     = RoPE_{B b}(RMSNorm_k(bf16(mean_{j<B} x_{B b+j} W_ik)))    (one key per block)
//   score[t, b] = sum_h relu(q[t,h] . k[b]) / sqrt(Di)
//   a query at position p sees its complete blocks b < (p + 1) / B: all of them when there are <= K, else the top-K
//   by score (ties to the lower block index); plus the tokens of its own incomplete block up to p. A block that
//   completed inside the verify window is scored like the others: its pooled key comes from the raw keys of the
//   window's tokens (committed or drafted), pooled on the fly; pooled keys are stored only once a block is committed.
//
// Kernels:
//   qsa_prep     -- per token: index query (norm + RoPE) into idx_q, raw index key into the per-token raw cache
//   qsa_finalize -- per (session, layer): pooled keys of blocks that became committed since the last call, one warp
//                   per block
//   qsa_scores_tc-- per (row set, chunk of 128-block tiles): the committed blocks' scores of all W rows at once on
//                   the tensor cores (A = 128 pooled keys, B = the W x Hi index-query rows, N = 32; relu and the head
//                   sum in the epilogue), each key read from HBM once per row set
//   qsa_score    -- per (row set, row): the row's scores over its complete blocks (from the tensor-core scores,
//                   plus blocks completed inside the window pooled on the fly), top-K by an 8-bit-digit radix select
//                   over order-preserving keys, the chosen blocks (and the row's own incomplete block) OR-ed into a
//                   per-set row bitmask
//   qsa_union    -- per row set: the marked blocks in ascending order with their row bitmasks (the union the
//                   attention walks once for all W rows), clearing the marks for the next call
// A row set is a session's W verify rows, or (prefill, bt_row set) W consecutive prompt positions of the session
// bt_row[set]: keys, finalised count and block table are the session's, selections and unions the set's.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemm.h"
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
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
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
  if (const int pdl_rc = launch_pdl(qsa_prep_kernel, dim3((total + warps - 1) / warps), dim3(warps * 32), 0, st, a,
      (const __nv_bfloat16*)proj, ld, T,
                                                                      positions, slots)) return pdl_rc;
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ pooled keys
// One warp: the pooled, normalised, rotated index key of block b (positions [B b, B b + B)); lane l returns dims
// 4 l .. 4 l + 3. RoPE pairs dim d with d +- rot / 2, which lives rot / 8 lanes away.
AFB_DEV void qsa_pooled_key(const __nv_bfloat16* raw, const int* bt, int B, int b, const __nv_bfloat16* k_norm,
                            const float* cos_t, const float* sin_t, int rot, float eps, float o[4]) {
  const int lane = threadIdx.x & 31;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < B; ++j) {
    const int pos = b * B + j;
    const size_t slot = (size_t)bt[pos >> 6] * 64 + (pos & 63);
    const uint2 u = *reinterpret_cast<const uint2*>(raw + slot * qsa::DI + lane * 4);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 x0 = __bfloat1622float2(h[0]), x1 = __bfloat1622float2(h[1]);
    acc[0] += x0.x;
    acc[1] += x0.y;
    acc[2] += x1.x;
    acc[3] += x1.y;
  }
  float x[4], ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[i] = __bfloat162float(__float2bfloat16(acc[i] / (float)B));  // the pooled key is a bf16 value
    ss += x[i] * x[i];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / qsa::DI + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = x[i] * inv * (1.f + __bfloat162float(k_norm[lane * 4 + i]));
  const int half = rot / 2, pos0 = b * B, dl = half / 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = lane * 4 + i;
    const int src = d < rot ? (d < half ? lane + dl : lane - dl) : lane;
    const float px = __shfl_sync(0xffffffffu, x[i], src & 31);
    if (d < rot) {
      const int fi = d < half ? d : d - half;
      const float cs = cos_t[(size_t)pos0 * half + fi], sn = sin_t[(size_t)pos0 * half + fi];
      o[i] = d < half ? x[i] * cs - px * sn : x[i] * cs + px * sn;
    } else {
      o[i] = x[i];
    }
    o[i] = __bfloat162float(__float2bfloat16(o[i]));  // keys are bf16 values, stored or pooled on the fly
  }
}

// ------------------------------------------------------------------------------------------------ finalize
// grid (sessions, layers), 8 warps: blocks [fin[s], ctx[s] / B) of session s get pooled keys, one warp per block.
__global__ void qsa_finalize_kernel(QsaFinalizeArgs f) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int s = blockIdx.x, l = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lo = f.fin[s], hi = min(f.ctx[s] / f.block, f.max_blocks);
  const int* bt = f.block_table + (size_t)s * f.max_pages;
  __nv_bfloat16* key = f.idx_key[l];
  for (int b = lo + warp; b < hi; b += blockDim.x >> 5) {
    float o[4];
    qsa_pooled_key(f.idx_raw[l], bt, f.block, b, f.k_norm[l], f.cos_t, f.sin_t, f.rot, f.eps, o);
    *reinterpret_cast<uint2*>(key + ((size_t)s * f.max_blocks + b) * qsa::DI + lane * 4) =
        make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
  }
}

__global__ void qsa_fin_update_kernel(int* fin, const int* ctx, int S, int block, int max_blocks) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s < S) fin[s] = min(ctx[s] / block, max_blocks);
}

int qsa_finalize(const QsaFinalizeArgs& f, int S, int layers, cudaStream_t st) {
  if (layers < 1 || layers > QSA_MAX_LAYERS || f.rot > qsa::DI || f.rot % 8 || f.block < 1 || 64 % f.block ||
      f.max_blocks != f.max_pages * (64 / f.block))
    return 3;
  if (S <= 0) return 0;
  if (const int pdl_rc = launch_pdl(qsa_finalize_kernel, dim3(dim3(S, layers)), dim3(256), 0, st, f)) return pdl_rc;
  if (const int pdl_rc = launch_pdl(qsa_fin_update_kernel, dim3((S + 127) / 128), dim3(128), 0, st, f.fin, f.ctx, S,
      f.block, f.max_blocks)) return pdl_rc;
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ select
AFB_DEV uint32_t order_key(float x) {  // monotone map float -> uint32 (NaN-free inputs)
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

AFB_DEV int block_count(int c, int* red) {  // block-wide sum of one int per thread (256 threads)
  c = __reduce_add_sync(0xffffffffu, c);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = c;
  __syncthreads();
  int t = 0;
#pragma unroll
  for (int w = 0; w < qsa::THREADS / 32; ++w) t += red[w];
  return t;
}

// ------------------------------------------------------------------------------------------------ tc scores
namespace qsa_tc {
constexpr int TM = 128;                 // blocks per tile (MMA M)
constexpr int NQ = 32;                  // index-query rows of a row set, W x Hi padded (MMA N)
constexpr int NS = 3;                   // key stages (two CTAs per SM)
constexpr int TPC = 16;                 // tiles per CTA
constexpr int THREADS = 192;            // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue (TMEM lane quadrants 2,3,0,1)
constexpr uint32_t KSUB = TM * 128;     // one 128-row x 64-column swizzled sub-tile
constexpr uint32_t KTILE = 2 * KSUB;
constexpr uint32_t QSUB = NQ * 128;
constexpr uint32_t K_OFF = 2 * QSUB;
constexpr uint32_t BAR_OFF = K_OFF + NS * KTILE;
constexpr uint32_t TOTAL = BAR_OFF + (2 * NS + 5) * 8 + 16 + 1024;
}  // namespace qsa_tc

// one block's scores for the W rows of its set from the accumulator columns r * HI + h
template <int HI>
AFB_DEV void row_scores(const float* v, int W, float rs, float* dst, int ld) {
#pragma unroll
  for (int r = 0; r < qsa_tc::NQ / HI; ++r) {
    if (r >= W) break;
    float sc = 0.f;
#pragma unroll
    for (int h = 0; h < HI; ++h) sc += fmaxf(v[r * HI + h], 0.f);
    dst[(size_t)r * ld] = sc * rs;
  }
}

__global__ void __launch_bounds__(qsa_tc::THREADS, 1)
    qsa_scores_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                         QsaArgs a, QsaSelectArgs sa, uint32_t* status) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  using namespace qsa_tc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* empty = full + NS;
  uint64_t* acc_full = empty + NS;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* q_ready = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_ready + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = blockIdx.x, W = sa.W, Hi = a.Hi;
  const int sr = sa.bt_row ? sa.bt_row[s] : s;
  // committed blocks that some row of the set scores (the last row sees the most)
  const int F = min(min(sa.fin[sr], sa.seq_lens[s] / sa.block), sa.max_blocks);
  const int t0 = blockIdx.y * TPC;
  const int nt = min(TPC, (F + TM - 1) / TM - t0);
  if (nt <= 0) return;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(q_ready, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 64);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmK);
      mbar_arrive_expect_tx(q_ready, 2 * QSUB);
      tma_load_2d(smem, &tmQ, q_ready, 0, s * W * Hi);
      tma_load_2d(smem + QSUB, &tmQ, q_ready, 64, s * W * Hi);
      for (int i = 0; i < nt; ++i) {
        const int st = i % NS;
        if (i >= NS && !mbar_wait(&empty[st], ((i / NS) & 1) ^ 1, status)) break;
        uint8_t* dst = smem + K_OFF + st * KTILE;
        const int row = sr * sa.max_blocks + (t0 + i) * TM;
        mbar_arrive_expect_tx(&full[st], KTILE);
        tma_load_2d(dst, &tmK, &full[st], 0, row);
        tma_load_2d(dst + KSUB, &tmK, &full[st], 64, row);
      }
      // nothing may still land after exit: wait (bounded) for the last fills
      mbar_wait(q_ready, 0, status);
      for (int i = max(0, nt - NS); i < nt; ++i) mbar_wait(&full[i % NS], (i / NS) & 1, status);
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = idesc_f16(TM, NQ, 1);
    bool ok = __all_sync(0xffffffffu, mbar_wait(q_ready, 0, status));
    tc_fence_after();
    const uint32_t q_base = smem_u32(smem);
    for (int i = 0; i < nt && ok; ++i) {
      const int st = i % NS, ab = i & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&full[st], (i / NS) & 1, status)) ||
          (i >= 2 && !__all_sync(0xffffffffu, mbar_wait(&acc_empty[ab], ((i >> 1) & 1) ^ 1, status)))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t k_base = smem_u32(smem + K_OFF + st * KTILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16(tmem + ab * NQ, sw128_desc(k_base + (kk >> 2) * KSUB + (kk & 3) * 32),
                   sw128_desc(q_base + (kk >> 2) * QSUB + (kk & 3) * 32), idesc, kk > 0 ? 1u : 0u);
        umma_commit(&empty[st]);
        umma_commit(&acc_full[ab]);
      }
      __syncwarp();
    }
    // every MMA has completed before TMEM is released: the last tile's accumulator barrier (or the epilogue's
    // bounded wait on it) covers them all
    if (nt > 0) mbar_wait(&acc_full[(nt - 1) & 1], ((nt - 1) >> 1) & 1, status);
  } else {
    const int quad = warp & 3;
    const float rs = rsqrtf((float)qsa::DI);
    for (int i = 0; i < nt; ++i) {
      const int ab = i & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[ab], (i >> 1) & 1, status))) break;
      tc_fence_after();
      float v[32];
      tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + ab * NQ, v);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
      const int b = (t0 + i) * TM + quad * 32 + lane;
      if (b < F) {
        float* dst = sa.scores + (size_t)s * W * sa.scores_ld + b;
        switch (Hi) {  // register-resident column indices per head count
          case 1: row_scores<1>(v, W, rs, dst, sa.scores_ld); break;
          case 2: row_scores<2>(v, W, rs, dst, sa.scores_ld); break;
          case 3: row_scores<3>(v, W, rs, dst, sa.scores_ld); break;
          default: row_scores<4>(v, W, rs, dst, sa.scores_ld); break;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

// block-wide exclusive prefix sum of one int per thread in thread order (256 threads); *total gets the sum
AFB_DEV int block_excl_scan(int c, int* wtot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) wtot[warp] = incl;
  __syncthreads();
  int before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < qsa::THREADS / 32; ++w) {
    before += w < warp ? wtot[w] : 0;
    all += wtot[w];
  }
  if (total) *total = all;
  return before + incl - c;
}

// grid (sessions, W rows), 256 threads; dynamic shared memory: the row's scores [max_blocks] + its index query
__global__ void __launch_bounds__(qsa::THREADS) qsa_score_kernel(QsaArgs a, QsaSelectArgs sa, uint32_t* status) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ int red[qsa::THREADS / 32];
  const int s = blockIdx.x, r = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int B = sa.block, K = sa.K, Hi = a.Hi, W = sa.W;
  const int p = sa.seq_lens[s] - W + r;  // this row's position
  if (p < 0) return;
  const int sr = sa.bt_row ? sa.bt_row[s] : s;    // the session (block table, pooled keys) of this row set
  const int C = min((p + 1) / B, sa.max_blocks);  // complete blocks this row may see
  const int F = min(sa.fin[sr], C);               // of them, committed ones with a stored pooled key
  uint32_t* sel = sa.sel + (size_t)s * (sa.max_blocks + 1);
  const uint32_t bit = 1u << r;
  if ((p + 1) % B && C < sa.max_blocks + 1 && tid == 0) atomicOr(&sel[C], bit);  // own incomplete block
  if (C <= K) {
    for (int b = tid; b < C; b += blockDim.x) atomicOr(&sel[b], bit);
    return;
  }
  float* score = reinterpret_cast<float*>(smem_raw);                       // [max_blocks]
  float* qs = score + ((sa.max_blocks + 3) & ~3);                          // [Hi][DI]
  for (int i = tid; i < Hi * qsa::DI; i += blockDim.x)
    qs[i] = __bfloat162float(a.idx_q[(size_t)(s * W + r) * Hi * qsa::DI + i]);
  __syncthreads();
  const float rs = rsqrtf((float)qsa::DI);
  // committed blocks: the tensor-core scores, or one thread per block with keys from the pooled cache
  if (sa.scores) {  // 8 independent loads in flight per thread (a load-then-store loop would wait on each)
    const float* src = sa.scores + ((size_t)s * W + r) * sa.scores_ld;
    for (int base = 0; base < F; base += 8 * qsa::THREADS) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int b = base + u * qsa::THREADS + tid;
        v[u] = b < F ? __ldg(src + b) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int b = base + u * qsa::THREADS + tid;
        if (b < F) score[b] = v[u];
      }
    }
  }
  for (int b = sa.scores ? F : tid; b < F; b += blockDim.x) {
    const uint4* kr = reinterpret_cast<const uint4*>(a.idx_key + ((size_t)sr * sa.max_blocks + b) * qsa::DI);
    float acc[qsa::MAXH] = {0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < qsa::DI / 8; ++c) {
      const uint4 u = kr[c];
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 x = __bfloat1622float2(h2[i]);
#pragma unroll
        for (int h = 0; h < qsa::MAXH; ++h)
          if (h < Hi) acc[h] += qs[h * qsa::DI + c * 8 + 2 * i] * x.x + qs[h * qsa::DI + c * 8 + 2 * i + 1] * x.y;
      }
    }
    float sc = 0.f;
#pragma unroll
    for (int h = 0; h < qsa::MAXH; ++h)
      if (h < Hi) sc += fmaxf(acc[h], 0.f);
    score[b] = sc * rs;
  }
  // blocks completed inside the verify window: pooled on the fly, one warp per block
  for (int b = F + warp; b < C; b += blockDim.x >> 5) {
    float o[4];
    qsa_pooled_key(a.idx_raw, sa.block_table + (size_t)sr * sa.max_pages, B, b, sa.k_norm, a.cos_t, a.sin_t, a.rot,
                   a.eps, o);
    float sc = 0.f;
    for (int h = 0; h < Hi; ++h) {
      const float* q = qs + h * qsa::DI + lane * 4;
      sc += fmaxf(warp_sum(q[0] * o[0] + q[1] * o[1] + q[2] * o[2] + q[3] * o[3]), 0.f);
    }
    if (lane == 0) score[b] = sc * rs;
  }
  __syncthreads();
  // the K-th largest order key in three radix passes (bits 31..20, 19..8, 7..0: the first two 4,096-bin passes
  // spread the exponent and leading mantissa bits, so few keys collide on a bin): per pass a histogram of the keys
  // that match the digits found so far, then the bin where the count from the top reaches the rank still sought
  uint32_t* hist = reinterpret_cast<uint32_t*>(qs);  // the index query is no longer needed
  __shared__ int wtot[qsa::THREADS / 32];
  uint32_t prefix = 0, pmask = 0;
  int kk = K;  // rank still to find among the matching keys
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass == 0 ? 20 : pass == 1 ? 8 : 0;
    const int nb = pass == 2 ? 256 : 4096, per = nb / qsa::THREADS;
    __syncthreads();
    for (int i = tid; i < nb; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int b = tid; b < C; b += blockDim.x) {
      const uint32_t key = order_key(score[b]);
      if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & (nb - 1)], 1u);
    }
    __syncthreads();
    int tot = 0;  // thread t owns bins nb - 1 - t * per down to nb - (t + 1) * per
    for (int j = 0; j < per; ++j) tot += (int)hist[nb - 1 - tid * per - j];
    const int excl = block_excl_scan(tot, wtot, nullptr);
    if (excl < kk && excl + tot >= kk) {
      int acc = excl, j = 0;
      while (acc + (int)hist[nb - 1 - tid * per - j] < kk) acc += (int)hist[nb - 1 - tid * per - j++];
      red[0] = nb - 1 - tid * per - j;  // the digit
      red[1] = acc;                     // matching keys above it
    }
    __syncthreads();
    prefix |= (uint32_t)red[0] << shift;
    pmask |= (uint32_t)(nb - 1) << shift;
    kk -= red[1];
  }
  int above = 0, equal = 0;
  for (int b = tid; b < C; b += blockDim.x) {
    const uint32_t key = order_key(score[b]);
    above += key > prefix;
    equal += key == prefix;
    if (key > prefix) atomicOr(&sel[b], bit);
  }
  const int need = K - block_count(above, red);
  const int n_equal = block_count(equal, red);
  if (n_equal <= need) {  // every key at the threshold is taken: no ordering needed
    for (int b = tid; b < C; b += blockDim.x)
      if (order_key(score[b]) == prefix) atomicOr(&sel[b], bit);
  } else if (warp == 0) {  // more ties than places: the lowest block indices first
    int need_eq = need;
    for (int base = 0; base < C && need_eq > 0; base += 32) {
      const int b = base + lane;
      const bool eq = b < C && order_key(score[b]) == prefix;
      const unsigned m = __ballot_sync(0xffffffffu, eq);
      if (eq && __popc(m & ((1u << lane) - 1)) < need_eq) atomicOr(&sel[b], bit);
      need_eq -= __popc(m);
    }
  }
  if (tid == 0 && need < 0) flag_error(status, AFB_ERR_BOUNDS);
}

// grid sessions, 256 threads: compact the marked blocks (ascending) into the union, clear the marks. The marks are
// staged in shared memory by independent coalesced loads, then each thread compacts a contiguous run of them at the
// offset a block scan of the per-thread counts gives (no per-chunk barrier round trips through global memory).
__global__ void __launch_bounds__(qsa::THREADS) qsa_union_kernel(QsaSelectArgs sa, uint32_t* status) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  extern __shared__ uint32_t marks[];
  __shared__ int wtot[qsa::THREADS / 32];
  __shared__ int total;
  const int s = blockIdx.x, tid = threadIdx.x;
  const int seq_len = sa.seq_lens[s];
  const int n_scan = min(seq_len / sa.block + 1, sa.max_blocks + 1);
  uint32_t* sel = sa.sel + (size_t)s * (sa.max_blocks + 1);
  const int* bt = sa.block_table + (size_t)(sa.bt_row ? sa.bt_row[s] : s) * sa.max_pages;
  for (int base = 0; base < n_scan; base += 8 * qsa::THREADS) {  // 8 independent loads in flight per thread
    uint32_t v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = base + u * qsa::THREADS + tid;
      v[u] = e < n_scan ? sel[e] : 0u;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = base + u * qsa::THREADS + tid;
      if (e < n_scan) marks[e] = v[u];
    }
  }
  __syncthreads();
  for (int e = tid; e < n_scan; e += blockDim.x)
    if (marks[e]) sel[e] = 0u;
  const int chunk = (n_scan + qsa::THREADS - 1) / qsa::THREADS;
  const int lo = min(n_scan, tid * chunk), hi = min(n_scan, lo + chunk);
  int c = 0;
  for (int e = lo; e < hi; ++e) c += marks[e] != 0u;
  int at = block_excl_scan(c, wtot, &total);
  for (int e = lo; e < hi; ++e) {
    const uint32_t m = marks[e];
    if (!m) continue;
    if (at < sa.ucap) {
      sa.u_lpage[(size_t)s * sa.ucap + at] = e;
      sa.u_mask[(size_t)s * sa.ucap + at] = (uint8_t)m;
      if (sa.u_page)
        sa.u_page[(size_t)s * sa.ucap + at] = sa.block == 64 ? bt[e] : bt[(e * sa.block) >> 6] * 64 + ((e * sa.block) & 63);
    }
    ++at;
  }
  if (tid == 0) {
    if (total > sa.ucap) flag_error(status, AFB_ERR_BOUNDS);
    sa.u_count[s] = min(total, sa.ucap);
  }
}

int qsa_select(const QsaArgs& a, const QsaSelectArgs& sa, int S, uint32_t* status, cudaStream_t st) {
  if (a.Di != qsa::DI || a.Hi < 1 || a.Hi > qsa::MAXH || sa.W < 1 || sa.W > qsa::MAXW || sa.K < 1 ||
      sa.block < 1 || 64 % sa.block || sa.max_blocks != sa.max_pages * (64 / sa.block) || sa.ucap < 1 || !sa.sel ||
      !a.idx_raw || !sa.k_norm || a.rot % 8)
    return 3;
  if (S <= 0) return 0;
  // scores [max_blocks] + the index query, whose space the 4,096-bin radix histogram reuses
  const size_t smem = (size_t)((sa.max_blocks + 3) & ~3) * 4 + (size_t)4096 * 4;
  static_assert(qsa::MAXH * qsa::DI <= 4096, "histogram space");
  if (smem > 220 * 1024) return 3;
  static std::atomic<uint64_t> attr_devs{0};
  if (const int e = smem_attr_once(attr_devs, (const void*)qsa_score_kernel, 220 * 1024)) return e;
  QsaSelectArgs sb = sa;
  if (sa.scores && sa.W * a.Hi <= qsa_tc::NQ && sa.key_rows > 0 && sa.q_rows > 0) {
    CUtensorMap tk{}, tq{};
    if (const int rc = make_tmap_2d(&tk, a.idx_key, 2, qsa::DI, sa.key_rows, qsa::DI * 2, 64, qsa_tc::TM, 1))
      return 1000 + rc;
    if (const int rc = make_tmap_2d(&tq, a.idx_q, 2, qsa::DI, sa.q_rows, qsa::DI * 2, 64, qsa_tc::NQ, 1))
      return 1000 + rc;
    static std::atomic<uint64_t> tc_devs{0};
    if (const int e = smem_attr_once(tc_devs, (const void*)qsa_scores_tc_kernel, qsa_tc::TOTAL)) return e;
    const int tiles = (sa.max_blocks + qsa_tc::TM - 1) / qsa_tc::TM;
    if (const int pdl_rc = launch_pdl(qsa_scores_tc_kernel, dim3(dim3(S, (tiles + qsa_tc::TPC - 1) / qsa_tc::TPC)),
        dim3(qsa_tc::THREADS), qsa_tc::TOTAL, st,
        tk, tq, a, sa, status)) return pdl_rc;
  } else {
    sb.scores = nullptr;  // the per-row kernel scores every block itself
  }
  if (const int pdl_rc = launch_pdl(qsa_score_kernel, dim3(dim3(S, sa.W)), dim3(qsa::THREADS), smem, st, a, sb,
      status)) return pdl_rc;
  static std::atomic<uint64_t> union_devs{0};
  const size_t usmem = (size_t)(sa.max_blocks + 1) * 4;
  if (const int e = smem_attr_once(union_devs, (const void*)qsa_union_kernel, 220 * 1024)) return e;
  if (const int pdl_rc = launch_pdl(qsa_union_kernel, dim3(S), dim3(qsa::THREADS), usmem, st, sa,
      status)) return pdl_rc;
  return (int)cudaGetLastError();
}

}  // namespace afb
