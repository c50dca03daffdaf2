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
    for (int j = 0; j < RPT; ++j) a.final_state[((size_t)bh * DK + rg * RPT + j) * Dv + c0 + c] = S[j];
}

template <bool REV, int DK>
static int launch_scan(const GdnScanArgs& a, cudaStream_t st) {
  const size_t smem = sizeof(gck::Smem<DK>) + 16;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gdn_chunk_scan_kernel<REV, DK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  gdn_chunk_scan_kernel<REV, DK><<<dim3(a.BH, a.Dv / gck::SL), gck::THREADS, smem, st>>>(a);
  return (int)cudaGetLastError();
}

int gdn_chunk_scan(const GdnScanArgs& a, bool reverse, cudaStream_t st) {
  if (a.C != gck::C || (a.Dk != 64 && a.Dk != 128) || a.Dv % gck::SL || a.n_chunks < 1 || a.BH < 1) return 3;
  if (a.Dk == 128) return reverse ? launch_scan<true, 128>(a, st) : launch_scan<false, 128>(a, st);
  return reverse ? launch_scan<true, 64>(a, st) : launch_scan<false, 64>(a, st);
}

}  // namespace afb
