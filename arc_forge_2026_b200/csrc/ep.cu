// Expert-parallel MoE exchange over NVLink peer memory (one process per GPU, experts split in contiguous blocks).
//
// Per MoE layer (all on one stream; every rank runs the same sequence):
//   1. ep_dispatch  -- each CTA takes one local token row: per-128-column amax, e4m3 quantisation, and stores of
//                      the e4m3 row, its group scales, its top-k expert ids and routing weights straight into
//                      EVERY rank's receive region (slot rank*T_cap + t). Fused all-gather + FP8 quantisation, in
//                      the role of the reference's ag_fp8q (hostcomm.cu:404-497) over NVSwitch instead of PCIe.
//                      Slots t in [T, T_cap) get expert id -1. The last CTA to finish raises the "dispatch"
//                      flag of this rank on every peer.
//   2. ep_wait      -- one warp: lane p waits (bounded) until rank p's flag reaches this exchange's number.
//   3. expert_sort  -- over all ranks' (token, slot) entries, keeping the local experts (expert_map).
//   4. ep_gather    -- sorted e4m3 rows + group scales for the grouped GEMM, from the local receive region.
//   5. w13 / w2 grouped GEMMs (moe_int3.cu); the w2 epilogue multiplies by the routing weight and stores each
//      routed row straight into its token owner's combine region [T_cap, k, H] (fused combine scatter; the owner
//      is encoded in the entry index), then raises the "combine" flag on every peer (last CTA).
//   6. ep_wait, then the owner's moe_combine sums its k rows in slot order (deterministic, no atomics).
//
// Flags are 64-bit exchange counters, never reset: the producer's last CTA publishes ++sent[type] with a
// release store at system scope; a waiter expects ++expected[type]. Each exchange is a full barrier (every rank
// waits for every rank), so a region is never rewritten before all its readers are done with it.
// Waits give up after AFB_WAIT_NS, flag AFB_ERR_PEER_TIMEOUT in the status word and return.
#include "common.cuh"
#include "kernels.h"

namespace afb {

AFB_DEV uint64_t* ep_flag(const EpArgs& a, int peer, int type, int src) {
  return reinterpret_cast<uint64_t*>(a.peer[peer] + a.off_flags) + type * EP_MAX_RANKS + src;
}

// Called by every thread of a CTA after its stores: the last CTA of the grid publishes the exchange.
AFB_DEV void ep_signal_last_cta(const EpArgs& a, int type) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&a.done[type], 1u);
    if (prev == gridDim.x - 1) {
      a.done[type] = 0;
      __threadfence_system();
      const uint64_t v = ++a.sent[type];
      for (int p = 0; p < a.world; ++p) st_release_sys_u64(ep_flag(a, p, type, a.rank), v);
    }
  }
}

// ------------------------------------------------------------------------------------------------ dispatch
__global__ void __launch_bounds__(128) ep_dispatch_kernel(EpArgs a, const __nv_bfloat16* __restrict__ x, int ldx,
                                                          const int* __restrict__ ids,
                                                          const float* __restrict__ weights) {
  const int t = blockIdx.x;  // local token slot, 0 .. T_cap-1
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t gt = (size_t)a.rank * a.T_cap + t;  // gathered token index
  const int groups = a.H / 128;
  if (t < a.T) {
    for (int g = warp; g < groups; g += 4) {
      const uint2 raw = *reinterpret_cast<const uint2*>(x + (size_t)t * ldx + g * 128 + lane * 4);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
      float f[4], m = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        f[i] = __bfloat162float(h[i]);
        m = fmaxf(m, fabsf(f[i]));
      }
      m = warp_max(m);
      const float s = m > 0.f ? m / 448.f : 1.f;  // same rule as quant_rows_e4m3
      const float inv = 1.f / s;
      __nv_fp8x4_e4m3 q(make_float4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv));
      const uint32_t qv = *reinterpret_cast<const uint32_t*>(&q);
      for (int p = 0; p < a.world; ++p) {
        *reinterpret_cast<uint32_t*>(a.peer[p] + a.off_x + gt * a.H + g * 128 + lane * 4) = qv;
        if (lane == 0) reinterpret_cast<float*>(a.peer[p] + a.off_s)[(size_t)g * a.ld_s + gt] = s;
      }
    }
  }
  if (threadIdx.x < a.k) {
    const int j = threadIdx.x;
    const int id = t < a.T ? ids[t * a.k + j] : -1;
    const float w = t < a.T ? weights[t * a.k + j] : 0.f;
    for (int p = 0; p < a.world; ++p) {
      reinterpret_cast<int*>(a.peer[p] + a.off_ids)[gt * a.k + j] = id;
      reinterpret_cast<float*>(a.peer[p] + a.off_w)[gt * a.k + j] = w;
    }
  }
  ep_signal_last_cta(a, EP_DISPATCH);
}

int ep_dispatch(const EpArgs& a, const void* x, int ldx, const int* ids, const float* weights, cudaStream_t st) {
  if (a.world < 1 || a.world > EP_MAX_RANKS || a.H % 128 || a.k > 128 || a.T > a.T_cap || a.T_cap < 1) return 3;
  ep_dispatch_kernel<<<a.T_cap, 128, 0, st>>>(a, (const __nv_bfloat16*)x, ldx, ids, weights);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ wait
__global__ void ep_wait_kernel(EpArgs a, int type, uint32_t* status) {
  const int lane = threadIdx.x;
  const uint64_t want = a.expected[type] + 1;
  if (lane < a.world) {
    const uint64_t* f = ep_flag(a, a.rank, type, lane);
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
  __syncwarp();
  if (lane == 0) a.expected[type] = want;
}

int ep_wait(const EpArgs& a, int type, uint32_t* status, cudaStream_t st) {
  if (a.world < 1 || a.world > EP_MAX_RANKS) return 3;
  ep_wait_kernel<<<1, 32, 0, st>>>(a, type, status);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ gather
// xq[r] = recv_x[row_token[r]], xs[g][r] = recv_s[g][row_token[r]] for r < rows (device count); one warp per
// (row, 128-column group), 4 bytes per lane.
__global__ void ep_gather_kernel(EpArgs a, const int* __restrict__ row_token, const int* __restrict__ nrows_dev,
                                 uint8_t* __restrict__ xq, float* __restrict__ xs, int ld_xs) {
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int groups = a.H / 128;
  const int r = gw / groups, g = gw % groups;
  if (r >= *nrows_dev) return;
  const size_t src = (size_t)row_token[r];
  const uint8_t* base = a.peer[a.rank];
  const uint32_t v = *reinterpret_cast<const uint32_t*>(base + a.off_x + src * a.H + g * 128 + lane * 4);
  *reinterpret_cast<uint32_t*>(xq + (size_t)r * a.H + g * 128 + lane * 4) = v;
  if (lane == 0) xs[(size_t)g * ld_xs + r] = reinterpret_cast<const float*>(base + a.off_s)[(size_t)g * a.ld_s + src];
}

int ep_gather(const EpArgs& a, const int* row_token, const int* nrows_dev, int rows_cap, void* xq, float* xs,
              int ld_xs, cudaStream_t st) {
  if (a.H % 128) return 3;
  if (rows_cap <= 0) return 0;
  const int warps = 8;
  const long long work = (long long)rows_cap * (a.H / 128);
  ep_gather_kernel<<<(unsigned)((work + warps - 1) / warps), warps * 32, 0, st>>>(a, row_token, nrows_dev,
                                                                                  (uint8_t*)xq, xs, ld_xs);
  return (int)cudaGetLastError();
}

}  // namespace afb
