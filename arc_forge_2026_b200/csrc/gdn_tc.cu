// Gated DeltaNet speculative verify on the tensor cores: one persistent CTA per SM walks (sequence, value head)
// items; per item the accepted tokens of the previous cycle and this cycle's tokens are applied to the committed
// state S0 [Dk = 128, Dv = 128] (fp32; stored transposed, S0^T [Dv, Dk] row-major, so every tensor-core operand is
// K-major) as ONE chunk in the WY form, instead of token by token:
//
//   P   = S0^T [K ; Q]^T            [Dv, L + T]  tcgen05 kind::tf32, M = 128 (value rows of S0^T), N = 32, K = Dk;
//                                                S0 = hi + lo: hi is S0 itself (the MMA reads tf32, i.e. the top 19
//                                                bits), lo = S0 - hi goes to tensor memory as the A operand of a
//                                                second pass, so P carries fp32 accuracy
//   G   = [K ; Q] K^T               [L + T, L]   SIMT, fp32, from the bf16 rows (exact products)
//   u_s = beta_s (v_s - Gamma_s p_s - sum_{r<s} Gamma_s / Gamma_r (k_r . k_s) u_r)   (forward substitution, one
//                                                thread per value column, L <= 16)
//   o_t = Gamma_t S0^T q_t + sum_{s<=t} Gamma_t / Gamma_s (k_s . q_t) u_s           (this cycle's outputs)
//   S_c = Gamma_c S0 + sum_{s<np} Gamma_c / Gamma_s k_s u_s^T                         (committed state, np accepted)
//         as S_c^T = Gamma_c S0^T + U^T K: the rank-np update on tcgen05 (M = Dv, N = Dk, K = 8; U^T in tensor
//         memory as tf32 hi + lo, the keys as a K-major shared-memory tile), added to Gamma_c S0^T in fp32 and
//         stored by TMA
//
// with Gamma_s = exp(sum of the log decays of tokens 0..s of the chunk). This is the same recurrence as
// gdn_recurrent_kernel (S <- g S; S += k beta (v - k.S); o = S^T q), regrouped; the state is read and written once
// per item, and the per-token work left on the CUDA cores is O(L^2) per value column instead of O(L Dk).
// Staging per item (double-buffered, issued one item ahead by thread 0, no multicast): 4 TMA boxes {32, 128} of
// the state (128-byte swizzle: each 32-column block is a K-major A tile), 2-D boxes of the k / q / v rows of both
// cycles, and the gates.
#include <cudaTypedefs.h>


#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace afb {

namespace gdntc {
constexpr int DK = 128, DV = 128, MAXT = 8, MAXL = 2 * MAXT, NP = 32, THREADS = 512, MAXS = 1024;
constexpr uint32_t SUBS = 128 * 128;     // one 32-column block of the state: 128 rows x 128 B
constexpr uint32_t STATE = 4 * SUBS;     // 64 KB
constexpr uint32_t KQ_SUB = NP * 128;    // one 32-column block of the fp32 key / query rows: 32 rows x 128 B
// TMEM columns: lo(S0^T) [128 x Dk], the update D2 = U^T K [Dv x Dk], P [Dv x 32], U^T hi / lo [Dv x 8] each
constexpr uint32_t LO_COL = 0, D2_COL = 128, P_COL = 256, U_COL = 288, TMEM_COLS = 512;

struct Smem {
  alignas(1024) uint8_t kq[4 * KQ_SUB];          // fp32 rows: keys 0..L-1 (accepted, then new), queries from MAXL
  alignas(1024) uint8_t state[2][STATE];         // S0^T of the item (by parity), updated in place to S_c^T
  alignas(1024) uint8_t kt[128 * 128];           // accepted keys transposed, K-major: row k holds k_s[k], s < 8
  __nv_bfloat16 kst[2][2 * MAXT][DK];            // [buf][previous-cycle k rows 0..7 | this cycle's 0..7]
  __nv_bfloat16 qst[2][MAXT][DK];
  __nv_bfloat16 vst[2][2 * MAXT][DV];
  float gb[2][2][2 * MAXT];                      // [buf][previous / this cycle][token * 2 + (log decay, beta)]
  float gram[MAXL + MAXT][MAXL];                 // C[s][r] = Gamma_s / Gamma_r (k_r . k_s) (r < s), then from row
                                                 // MAXL the query rows CQ[t][s] = Gamma_t / Gamma_s (k_s . q_t)
                                                 // (s <= t, t = np + query index)
  alignas(16) float lgam[MAXL];                  // log Gamma_s (cumulative log decay of tokens 0..s)
  alignas(16) float gexp[MAXL];                  // Gamma_s
  alignas(16) float beta[MAXL];
  alignas(16) float usm[MAXL][DV];               // u_s of every value column (the forward substitution's result)
  float ssq[MAXT];
  int slot[MAXS], ncommit[MAXS];
  uint64_t full[2], mma1, mma2, fin;
  uint32_t tmem_slot;
};
}  // namespace gdntc

AFB_DEV void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(c0),
               "r"(c1), "r"(smem_u32(src))
               : "memory");
}
AFB_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
AFB_DEV void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
AFB_DEV void bulk_wait_all0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
AFB_DEV void bulk_g2s_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
AFB_DEV uint32_t kq_off(int row, int k) {  // K-major 128-byte swizzle, 32-column blocks of NP rows
  return (uint32_t)((k >> 5) * gdntc::KQ_SUB + row * 128 + ((((k & 31) >> 2) ^ (row & 7)) << 4) + (k & 3) * 4);
}
AFB_DEV float tf32_hi(float x) { return __int_as_float(__float_as_int(x) & 0xffffe000); }

__global__ void __launch_bounds__(gdntc::THREADS, 1)
    gdn_verify_tc_kernel(const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmQK,
                         const __grid_constant__ CUtensorMap tmV, GdnArgs a, int parity, uint32_t* status) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  using namespace gdntc;
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, wid = tid >> 5, lane = tid & 31;
  const int T = a.q_per_seq;
  const int nq = a.Hk * DK;
  const int cur = parity, prev = parity ^ 1;
  const int items = a.num_seqs * a.Hv;

  for (int i = tid; i < a.num_seqs; i += THREADS) {
    const int sl = a.seq_slot[i];
    sm.slot[i] = sl;
    sm.ncommit[i] = min(a.n_commit[sl], MAXT);
  }
  for (int i = tid; i < (int)(sizeof(sm.kq) / 4); i += THREADS) reinterpret_cast<float*>(sm.kq)[i] = 0.f;
  for (int i = tid; i < (int)(sizeof(sm.kt) / 4); i += THREADS) reinterpret_cast<float*>(sm.kt)[i] = 0.f;
  for (int i = tid; i < (int)(sizeof(sm.gram) / 4); i += THREADS) (&sm.gram[0][0])[i] = 0.f;
  if (tid == 0) {
    mbar_init(&sm.full[0], 1);
    mbar_init(&sm.full[1], 1);
    mbar_init(&sm.mma1, 1);
    mbar_init(&sm.mma2, 1);
    mbar_init(&sm.fin, 1);
    fence_mbar_init();
  }
  if (wid == 1) tmem_alloc(&sm.tmem_slot, TMEM_COLS);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_slot;

  // thread 0 stages an item into buffer b: the state (4 swizzled boxes), k / q / v rows of both cycles (2-D boxes of
  // max_q rows), and the two gate rows
  auto issue = [&](int item, int b) {
    const int seq = item / a.Hv, h = item % a.Hv;
    const int slot = sm.slot[seq];
    const int kh = h / (a.Hv / a.Hk);
    const uint32_t rows = a.max_q;
    mbar_arrive_expect_tx(&sm.full[b], STATE + rows * (3 * DK * 2 + 2 * DV * 2) + 2 * rows * 8);
    const int srow = (slot * a.Hv + h) * DV;
#pragma unroll
    for (int c = 0; c < 4; ++c) tma_load_2d(sm.state[b] + c * SUBS, &tmS, &sm.full[b], c * 32, srow);
    const int rp = (prev * a.pend_slots + slot) * a.max_q, rc = (cur * a.pend_slots + slot) * a.max_q;
    tma_load_2d(sm.kst[b][0], &tmQK, &sm.full[b], nq + kh * DK, rp);
    tma_load_2d(sm.kst[b][MAXT], &tmQK, &sm.full[b], nq + kh * DK, rc);
    tma_load_2d(sm.qst[b][0], &tmQK, &sm.full[b], kh * DK, rc);
    tma_load_2d(sm.vst[b][0], &tmV, &sm.full[b], h * DV, rp);
    tma_load_2d(sm.vst[b][MAXT], &tmV, &sm.full[b], h * DV, rc);
    bulk_g2s_1d(sm.gb[b][0], a.pend_gb + (((size_t)prev * a.pend_slots + slot) * a.Hv + h) * a.max_q * 2,
                rows * 8, &sm.full[b]);
    bulk_g2s_1d(sm.gb[b][1], a.pend_gb + (((size_t)cur * a.pend_slots + slot) * a.Hv + h) * a.max_q * 2, rows * 8,
                &sm.full[b]);
  };

  int issued = 0, done = 0, n_mma2 = 0;
  if (tid == 0 && blockIdx.x < items) {
    prefetch_tmap(&tmS);
    prefetch_tmap(&tmQK);
    prefetch_tmap(&tmV);
    issue(blockIdx.x, 0);
    issued = 1;
  }
  const float norm_w = __bfloat162float(a.norm_w[(wid & 3) * 32 + lane]);
  bool ok = true;
  int i = 0;
  // profiling (a.dbg): thread 0 (copies, solve) and thread 32 (MMA issue) sum their cycles per section
  long long sec[8] = {0, 0, 0, 0, 0, 0, 0, 0}, sub[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const bool prof = a.dbg != nullptr && (tid == 0 || tid == 32);
  long long tsub = 0;
  auto smark = [&](int k) {  // thread 0: sub-sections of the solve
    if (prof && tid == 0) {
      const long long now = clock64();
      if (k >= 0) sub[k] += now - tsub;
      tsub = now;
    }
  };
  long long tclk = prof ? clock64() : 0;
  auto mark = [&](int k) {
    if (prof) {
      const long long now = clock64();
      sec[k] += now - tclk;
      tclk = now;
    }
  };
  for (int item = blockIdx.x; item < items; item += gridDim.x, ++i) {
    const int b = i & 1;
    const int seq = item / a.Hv, h = item % a.Hv;
    const int slot = sm.slot[seq], np = sm.ncommit[seq];
    const int L = np + T;
    // ---------------------------------------------------------------- phase 0: staged data -> operands
    ok = __syncthreads_and(mbar_wait(&sm.full[b], (i >> 1) & 1, status));
    if (!ok) break;
    ++done;
    mark(0);
    // this cycle's output gate (warps 0-3, one value column per thread), in flight until the norm
    float z[2];  // tokens t = wid / 4 + 4 e of column (wid % 4) * 32 + lane
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int t = (wid >> 2) + 4 * e;
      z[e] = t < T ? __bfloat162float(
                         a.mixed[((size_t)seq * T + t) * a.mixed_ld + a.z_off + h * DV + (wid & 3) * 32 + lane])
                   : 0.f;
    }
    // fp32 key / query rows (K-major swizzled): rows 0..np-1 the accepted keys, np..L-1 this cycle's, queries at
    // rows MAXL..MAXL+T-1 (fixed positions, so every P column has a compile-time register index)
    for (int idx = tid; idx < (L + T) * (DK / 4); idx += THREADS) {
      const int e = idx / (DK / 4), k4 = (idx % (DK / 4)) * 4;
      const int row = e < L ? e : MAXL + e - L;
      const __nv_bfloat16* src = e < np ? sm.kst[b][e] : e < L ? sm.kst[b][MAXT + e - np] : sm.qst[b][e - L];
      const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + k4));
      const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + k4 + 2));
      *reinterpret_cast<float4*>(sm.kq + kq_off(row, k4)) = make_float4(f0.x, f0.y, f1.x, f1.y);
    }
    // lo(S0^T) into TMEM: warp w holds value rows 32 (w % 4) .. + 31 (its TMEM lane quadrant) and key columns
    // 32 (w / 4) .. + 31 (one 128-byte row of a swizzled state block per thread)
    {
      const int q = wid & 3, kb = wid >> 2, v = q * 32 + lane;
      const uint8_t* row = sm.state[b] + kb * SUBS + v * 128;
      uint32_t lo[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 x = *reinterpret_cast<const float4*>(row + ((c ^ (v & 7)) << 4));
        lo[4 * c] = __float_as_uint(x.x - tf32_hi(x.x));
        lo[4 * c + 1] = __float_as_uint(x.y - tf32_hi(x.y));
        lo[4 * c + 2] = __float_as_uint(x.z - tf32_hi(x.z));
        lo[4 * c + 3] = __float_as_uint(x.w - tf32_hi(x.w));
      }
      tmem_st32(tmem + ((uint32_t)(q * 32) << 16) + LO_COL + kb * 32, lo);
      tmem_st_wait();
    }
    // the accepted keys transposed (B of the rank-np update): row k, column s = k_s[k] (zero for s >= np); a warp
    // reads 32 consecutive elements of one key row
    for (int idx = tid; idx < DK * 8; idx += THREADS) {
      const int s2 = idx >> 7, k = idx & (DK - 1);
      const float x = s2 < np ? __bfloat162float(sm.kst[b][s2][k]) : 0.f;
      *reinterpret_cast<float*>(sm.kt + k * 128 + ((((s2 >> 2) ^ (k & 7))) << 4) + (s2 & 3) * 4) = x;
    }
    // gates: Gamma_s (cumulative log decay over the chunk) and beta_s
    if (tid < 32) {
      float g = 0.f, bt = 0.f;
      if (lane < L) {
        const float* gp = lane < np ? &sm.gb[b][0][2 * lane] : &sm.gb[b][1][2 * (lane - np)];
        g = gp[0];
        bt = gp[1];
      }
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float x = __shfl_up_sync(0xffffffffu, g, o);
        if (lane >= o) g += x;
      }
      if (lane < MAXL) {
        sm.lgam[lane] = g;
        sm.beta[lane] = bt;
      }
      if (lane < MAXT) sm.ssq[lane] = 0.f;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    mark(1);
    __syncthreads();
    tc_fence_after();
    mark(2);
    // ---------------------------------------------------------------- phase 1: P on the tensor cores, G on the cores
    if (tid == 0) {
      const int next = item + gridDim.x;
      if (next < items) {
        bulk_wait_read0();  // the previous item's state store has left buffer b ^ 1
        issue(next, b ^ 1);
        ++issued;
      }
    }
    if (wid == 1 && lane == 0) {
      constexpr uint32_t id_p = idesc_tf32(128, NP, 0, 0);  // A = S0^T, B = [K; Q], both K-major
      const uint32_t s_base = smem_u32(sm.state[b]), kq_base = smem_u32(sm.kq);
#pragma unroll
      for (int ks = 0; ks < DK / 8; ++ks) {
        const uint32_t koff = (ks & 3) * 32;
        const uint64_t db = sw128_desc(kq_base + (ks >> 2) * KQ_SUB + koff);
        umma_tf32(tmem + P_COL, sw128_desc(s_base + (ks >> 2) * SUBS + koff), db, id_p, ks > 0 ? 1u : 0u);
        umma_tf32_ta(tmem + P_COL, tmem + LO_COL + ks * 8, db, id_p, 1u);
      }
      umma_commit(&sm.mma1);
    }
    if (wid >= 4) {
      // Gram entries over the bf16 rows (12 warps, one (row, key) pair per thread; each thread starts its sweep at
      // its own 16-byte column so the pairs of one warp spread over the banks)
      const int e = tid - 128, r = e / MAXL, c = e % MAXL;  // rows 0..MAXL-1 keys, MAXL.. queries
      if ((r < L || (r >= MAXL && r < MAXL + T)) && c < L) {
        const __nv_bfloat16* x = r < np ? sm.kst[b][r] : r < L ? sm.kst[b][MAXT + r - np] : sm.qst[b][r - MAXL];
        const __nv_bfloat16* y = c < np ? sm.kst[b][c] : sm.kst[b][MAXT + c - np];
        float acc = 0.f;
#pragma unroll 4
        for (int jj = 0; jj < DK / 8; ++jj) {
          const int j = ((jj + c) & (DK / 8 - 1)) * 8;
          const uint4 xv = *reinterpret_cast<const uint4*>(x + j), yv = *reinterpret_cast<const uint4*>(y + j);
          const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&xv);
          const __nv_bfloat162* yp = reinterpret_cast<const __nv_bfloat162*>(&yv);
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const float2 xf = __bfloat1622float2(xp[m]), yf = __bfloat1622float2(yp[m]);
            acc = fmaf(xf.x, yf.x, acc);
            acc = fmaf(xf.y, yf.y, acc);
          }
        }
        // key row r < L: strictly lower part C[r][c] (c < r); query row: CQ over s = c <= np + (r - L)
        const int t = r < L ? r : np + (r - MAXL);
        const bool keep = r < L ? c < r : c <= t;
        sm.gram[r][c] = keep ? __expf(sm.lgam[t] - sm.lgam[c]) * acc : 0.f;
      }
      if (tid >= THREADS - MAXL) sm.gexp[tid - (THREADS - MAXL)] = __expf(sm.lgam[tid - (THREADS - MAXL)]);
    }
    // ---------------------------------------------------------------- phase 2: solve, outputs, norm (warps 0-3)
    mark(3);
    const bool mma_ok = __syncthreads_and(mbar_wait(&sm.mma1, i & 1, status));
    mark(4);
    tc_fence_after();
    if (!mma_ok) {
      ok = false;
      break;
    }
    {
      // every warp: value columns v of its TMEM lane quadrant; the forward substitution runs in all four warps of a
      // quadrant (it is short), and warp group j = wid / 4 finishes the tokens t = j, j + 4 of this cycle
      const int q = wid & 3, jg = wid >> 2, v = q * 32 + lane;
      smark(-1);
      float p[NP];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + P_COL, p);
      tmem_ld_wait();
      smark(0);
      // forward substitution without branches: rows s >= L have beta_s = 0 (so u_s = 0) and finite Gram entries, so
      // every load can be issued ahead of the chain; a chunk of at most 8 tokens runs the 8-row form
      // warp group 0 (one warp per value quadrant) runs the forward substitution and publishes u; the sixteen warps
      // then share the outputs
      float u[MAXL];
      if (jg == 0) {
        float bet[MAXL], gx[MAXL], base[MAXL];
#pragma unroll
        for (int s4 = 0; s4 < MAXL / 4; ++s4) {
          const float4 b4 = reinterpret_cast<const float4*>(sm.beta)[s4];
          const float4 g4v = reinterpret_cast<const float4*>(sm.gexp)[s4];
          bet[4 * s4] = b4.x, bet[4 * s4 + 1] = b4.y, bet[4 * s4 + 2] = b4.z, bet[4 * s4 + 3] = b4.w;
          gx[4 * s4] = g4v.x, gx[4 * s4 + 1] = g4v.y, gx[4 * s4 + 2] = g4v.z, gx[4 * s4 + 3] = g4v.w;
        }
#pragma unroll
        for (int s = 0; s < MAXL; ++s) {
          const int vr = s < np ? s : MAXT + s - np;
          const float vv = s < L ? __bfloat162float(sm.vst[b][min(vr, 2 * MAXT - 1)][v]) : 0.f;
          base[s] = bet[s] * (vv - gx[s] * p[s]);
        }
        // forward substitution (rows s >= L: beta = 0, so u_s = 0); Gram entries on and above the diagonal are zero
#pragma unroll
        for (int s = 0; s < MAXL; ++s) {
          float acc = 0.f;
          if (s < L) {
            const float4* g4 = reinterpret_cast<const float4*>(sm.gram[s]);
#pragma unroll
            for (int r4 = 0; r4 < (s + 3) / 4; ++r4) {
              const float4 gg = g4[r4];
              acc = fmaf(gg.x, u[4 * r4], acc);
              if (4 * r4 + 1 < s) acc = fmaf(gg.y, u[4 * r4 + 1], acc);
              if (4 * r4 + 2 < s) acc = fmaf(gg.z, u[4 * r4 + 2], acc);
              if (4 * r4 + 3 < s) acc = fmaf(gg.w, u[4 * r4 + 3], acc);
            }
          }
          u[s] = base[s] - bet[s] * acc;
          sm.usm[s][v] = u[s];
        }
      }
      named_bar_sync(3, THREADS);
      if (jg != 0) {
#pragma unroll
        for (int s = 0; s < MAXL; ++s) u[s] = sm.usm[s][v];
      }
      smark(1);
      // this warp group's query columns of P (selected without a runtime register index)
      float pq[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c0 = MAXL + 4 * e;
        pq[e] = jg == 0 ? p[c0] : jg == 1 ? p[c0 + 1] : jg == 2 ? p[c0 + 2] : p[c0 + 3];
      }
      float o[2], sq[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = jg + 4 * e;
        o[e] = 0.f;
        if (t < T) {
          const float4* g4 = reinterpret_cast<const float4*>(sm.gram[MAXL + t]);
          float a0 = sm.gexp[np + t] * pq[e], a1 = 0.f;  // two chains
#pragma unroll
          for (int r4 = 0; r4 < MAXL / 4; ++r4) {
            const float4 gg = g4[r4];  // zero past s = np + t
            a0 = fmaf(gg.x, u[4 * r4], a0);
            a1 = fmaf(gg.y, u[4 * r4 + 1], a1);
            a0 = fmaf(gg.z, u[4 * r4 + 2], a0);
            a1 = fmaf(gg.w, u[4 * r4 + 3], a1);
          }
          o[e] = a0 + a1;
        }
        sq[e] = o[e] * o[e];
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        sq[0] += __shfl_xor_sync(0xffffffffu, sq[0], off);
        sq[1] += __shfl_xor_sync(0xffffffffu, sq[1], off);
      }
      if (lane < 2 && jg + 4 * lane < T) atomicAdd(&sm.ssq[jg + 4 * lane], lane ? sq[1] : sq[0]);
      smark(2);
      // Gamma_c / Gamma_s u_s of the accepted tokens as tf32 hi + lo columns of U^T in TMEM (lane v, column s)
      if (np > 0 && jg == 0) {
        const float lc = sm.lgam[np - 1];
        uint32_t uh[MAXT], ul[MAXT];
#pragma unroll
        for (int s2 = 0; s2 < MAXT; ++s2) {
          const float us = s2 < np ? __expf(lc - sm.lgam[s2]) * u[s2] : 0.f;  // Gamma_c / Gamma_s, no overflow
          const float hi = tf32_hi(us);
          uh[s2] = __float_as_uint(hi);
          ul[s2] = __float_as_uint(us - hi);
        }
        tmem_st8(tmem + ((uint32_t)(q * 32) << 16) + U_COL, uh);
        tmem_st8(tmem + ((uint32_t)(q * 32) << 16) + U_COL + 8, ul);
        tmem_st_wait();
      }
      smark(3);
      __syncthreads();  // the sums of squares are complete
      smark(4);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = jg + 4 * e;
        if (t < T) {
          const size_t tok = (size_t)seq * T + t;
          const float rstd = rsqrtf(sm.ssq[t] / DV + a.eps);
          a.out[tok * (a.Hv * DV) + h * DV + v] = __float2bfloat16(o[e] * rstd * norm_w * silu(z[e]));
        }
      }
      smark(5);
    }
    tc_fence_before();
    mark(5);
    __syncthreads();
    mark(6);
    // ---------------------------------------------------------------- phase 3: committed state
    if (np > 0) {
      if (wid == 1 && lane == 0) {
        tc_fence_after();
        constexpr uint32_t id_c = idesc_tf32(128, DK, 0, 0);  // A = U^T (TMEM), B = K transposed (K-major)
        const uint64_t dk = sw128_desc(smem_u32(sm.kt));
        umma_tf32_ta(tmem + D2_COL, tmem + U_COL, dk, id_c, 0u);
        umma_tf32_ta(tmem + D2_COL, tmem + U_COL + 8, dk, id_c, 1u);
        umma_commit(&sm.mma2);
      }
      const bool ok2 = __all_sync(0xffffffffu, mbar_wait(&sm.mma2, n_mma2 & 1, status));
      ++n_mma2;
      tc_fence_after();
      if (!__syncthreads_and(ok2)) {
        ok = false;
        break;
      }
      // S_c^T = Gamma_c S0^T + D2: warp w reads value rows 32 (w % 4) .. (its lane quadrant), key columns 32 (w / 4)
      const int q = wid & 3, kb = wid >> 2, v = q * 32 + lane;
      const float gc = __expf(sm.lgam[np - 1]);
      float d[32];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + D2_COL + kb * 32, d);
      tmem_ld_wait();
      uint8_t* row = sm.state[b] + kb * SUBS + v * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float4* p4 = reinterpret_cast<float4*>(row + ((c ^ (v & 7)) << 4));
        const float4 s4 = *p4;
        *p4 = make_float4(fmaf(gc, s4.x, d[4 * c]), fmaf(gc, s4.y, d[4 * c + 1]), fmaf(gc, s4.z, d[4 * c + 2]),
                          fmaf(gc, s4.w, d[4 * c + 3]));
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        const int srow = (slot * a.Hv + h) * DV;
#pragma unroll
        for (int c = 0; c < 4; ++c) tma_store_2d(&tmS, sm.state[b] + c * SUBS, c * 32, srow);
        bulk_commit();
      }
    }
    mark(7);
  }
  if (prof) {
    long long* d = a.dbg + blockIdx.x * 24 + (tid == 0 ? 0 : 8);
    for (int k = 0; k < 8; ++k) d[k] = sec[k];
    if (tid == 0)
      for (int k = 0; k < 8; ++k) d[16 + k] = sub[k];
    if (tid == 0) d[7] += (long long)done << 40;  // item count in the high bits of thread 0's last slot
  }
  // drain: copies still in flight (only after a failed wait), bounded; the state stores
  if (tid == 0) {
    for (int j = done; j < issued; ++j) mbar_wait(&sm.full[j & 1], (j >> 1) & 1, status);
    bulk_wait_all0();
  }
  tc_fence_before();
  __syncthreads();
  if (wid == 1) {
    // every MMA this warp issued has completed before TMEM is released (also after a timeout)
    tc_fence_after();
    if (lane == 0) umma_commit(&sm.fin);
    __syncwarp();
    mbar_wait(&sm.fin, 0, status);
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// The tensor-core verify path: DK = DV = 128, at most 8 tokens per cycle, deferred commit (verify cycles); returns -1
// when the call is outside that set (the caller runs the CUDA-core kernels).
int gdn_verify_tc(const GdnArgs& a, int parity, int num_sms, uint32_t* status, cudaStream_t st) {
  using namespace gdntc;
  if (a.commit_current || a.Dk != DK || a.Dv != DV || a.max_q > MAXT || a.max_q % 2 || a.q_per_seq > a.max_q ||
      a.num_seqs > MAXS || num_sms <= 0)
    return -1;
  CUtensorMap ts{}, tq{}, tv{};
  // S^T [slots * Hv * Dv rows, Dk]: boxes of 32 key columns x 128 value rows
  int rc = make_tmap_2d(&ts, a.ssm_state, 4, DK, (uint64_t)a.num_slots * a.Hv * DV, (uint64_t)DK * 4, 32, DV, 1);
  if (rc) return 1000 + rc;
  const int nq = a.Hk * DK;
  rc = make_tmap_2d(&tq, a.pend_qk, 2, 2 * nq, (uint64_t)2 * a.pend_slots * a.max_q, (uint64_t)2 * nq * 2, DK,
                    a.max_q, 0);
  if (rc) return 1000 + rc;
  rc = make_tmap_2d(&tv, a.pend_v, 2, (uint64_t)a.Hv * DV, (uint64_t)2 * a.pend_slots * a.max_q,
                    (uint64_t)a.Hv * DV * 2, DV, a.max_q, 0);
  if (rc) return 1000 + rc;
  const size_t smem = sizeof(Smem) + 1024;
  static std::atomic<uint64_t> attr_devs{0};
  if (const int e = smem_attr_once(attr_devs, (const void*)gdn_verify_tc_kernel, (int)smem)) return e;
  const int items = a.num_seqs * a.Hv;
  return launch_pdl(gdn_verify_tc_kernel, dim3(items < num_sms ? items : num_sms), dim3(THREADS), smem, st, ts, tq,
      tv, a,
                    parity, status);
}

}  // namespace afb
