// Expert-parallel MoE exchange over NVLink peer memory (one process per GPU, experts split in contiguous blocks).
//
// Per MoE layer (all on one stream; every rank runs the same sequence):
//   1. router top-k (local) also lists each expert's (token, slot) entries of this rank's tokens.
//   2. ep_dispatch  -- one CTA per local token row: row amax, e4m3 quantisation with one scale per row (the experts'
//                      W3A8 activation rule), and stores of the e4m3 row, its scale, its top-k expert ids and routing
//                      weights straight into EVERY rank's receive region (slot rank*T_cap + t): fused all-gather + FP8
//                      quantisation, in the role of the reference's ag_fp8q (hostcomm.cu:404-497) over NVSwitch
//                      instead of PCIe. Further CTAs copy the router's per-expert lists to each expert's owner (as
//                      global entry indices, into the owner's [source][local expert] lists). The last CTA raises this
//                      rank's "dispatch" flag on every peer.
//   3. w13 GEMM (moe_int3.cu): its CTAs wait (bounded) for every source's dispatch flag, then read the lists and
//      gather the activation rows from the local receive region themselves -- no sort, no gather, no wait launch.
//   4. per-row requantisation of h for the listed entries (quant_routed_rows).
//   5. w2 GEMM: the epilogue multiplies by the routing weight and stores each routed row straight into its token
//      owner's combine region [T_cap, k, H] (fused combine scatter; the owner is encoded in the entry index), then
//      raises the "combine" flag on every peer (last CTA).
//   6. moe_combine waits (bounded, in its prologue) for every rank's combine flag and sums the k rows of each token in
//      slot order (deterministic, no atomics) + shared expert + residual.
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
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  constexpr int MAXV = 3;  // 16-byte vectors per thread: H <= 128 * 8 * 3
  __shared__ float red[4];
  if (blockIdx.x >= a.T_cap) {  // list CTAs: warp w copies expert e's entries of this rank to e's owner
    const int e = (blockIdx.x - a.T_cap) * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (e < a.E_local * a.world) {
      const int owner = e / a.E_local, el = e - owner * a.E_local;
      const int n = a.lcnt[e];
      int* dst = reinterpret_cast<int*>(a.peer[owner] + a.off_rlist) + ((size_t)a.rank * a.E_local + el) * a.T_cap;
      const int base = a.rank * a.T_cap * a.k;  // local entry -> global entry
      for (int i = lane; i < n; i += 32) dst[i] = base + a.llist[(size_t)e * a.T_cap + i];
      if (lane == 0) reinterpret_cast<int*>(a.peer[owner] + a.off_rcnt)[a.rank * a.E_local + el] = n;
    }
    ep_signal_last_cta(a, EP_DISPATCH);
    return;
  }
  const int t = blockIdx.x;  // local token slot, 0 .. T_cap-1
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t gt = (size_t)a.rank * a.T_cap + t;  // gathered token index
  const int nv = a.H / 8;
  if (t < a.T) {
    uint4 raw[MAXV];
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int v = threadIdx.x + i * 128;
      raw[i] = v < nv ? reinterpret_cast<const uint4*>(x + (size_t)t * ldx)[v] : make_uint4(0, 0, 0, 0);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float s = fmaxf(m, 1e-30f) / 448.f;  // same rule as quant_rows_e4m3_row
    const float inv = 1.f / s;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int v = threadIdx.x + i * 128;
      if (v >= nv) break;
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
      float f[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 u = __bfloat1622float2(h[k]);
        f[2 * k] = u.x * inv;
        f[2 * k + 1] = u.y * inv;
      }
      const __nv_fp8x4_e4m3 lo(make_float4(f[0], f[1], f[2], f[3])), hi(make_float4(f[4], f[5], f[6], f[7]));
      const uint2 q = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
      for (int p = 0; p < a.world; ++p)
        reinterpret_cast<uint2*>(a.peer[p] + a.off_x + gt * a.H)[v] = q;
    }
    if (threadIdx.x == 0)
      for (int p = 0; p < a.world; ++p) reinterpret_cast<float*>(a.peer[p] + a.off_s)[gt] = s;
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
  if (a.world < 1 || a.world > EP_MAX_RANKS || a.H % 128 || a.H > 128 * 8 * 3 || a.k > 128 || a.T > a.T_cap ||
      a.T_cap < 1 || !a.lcnt || !a.llist || a.E_local < 1)
    return 3;
  const int E = a.E_local * a.world;
  {
    const int pdl_rc = launch_pdl(ep_dispatch_kernel, dim3(a.T_cap + (E + 3) / 4), dim3(128), 0, st, a,
        (const __nv_bfloat16*)x, ldx, ids, weights);
    if (pdl_rc) return pdl_rc;
  }
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

// ------------------------------------------------------------------------------------------------ routed quant
// q[e] = e4m3(x[e] * (1/s)), s = max(amax, 1e-30) / 448, for every entry e the lists name (one warp per list slot)
__global__ void quant_routed_rows_kernel(const __nv_bfloat16* __restrict__ x, int K, const int* __restrict__ cnt,
                                         const int* __restrict__ list, int E, int cap, uint8_t* __restrict__ q,
                                         float* __restrict__ scales, int slots) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (w >= slots) return;
  const int pe = w / cap, i = w - pe * cap;  // (source * E + expert), position
  if (i >= cnt[pe]) return;
  const int r = list[(size_t)pe * cap + i];
  const uint4* p = reinterpret_cast<const uint4*>(x + (size_t)r * K);
  const int nv = K / 8;
  float a = 0.f;
  for (int v = lane; v < nv; v += 32) {
    const uint4 raw = p[v];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
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
    for (int j = 0; j < 4; ++j) {
      const float2 u = __bfloat1622float2(h[j]);
      f[2 * j] = u.x * inv;
      f[2 * j + 1] = u.y * inv;
    }
    const __nv_fp8x4_e4m3 lo(make_float4(f[0], f[1], f[2], f[3])), hi(make_float4(f[4], f[5], f[6], f[7]));
    out[v] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
  }
  if (lane == 0) scales[r] = s;
}

int quant_routed_rows(const void* x, int K, const int* cnt, const int* list, int srcs, int E, int cap, void* q,
                      float* scales, cudaStream_t st) {
  if (K % 8 || srcs < 1 || E < 1 || cap < 1) return 3;
  const int slots = srcs * E * cap;
  const int warps = 8;
  {
    const int pdl_rc = launch_pdl(quant_routed_rows_kernel, dim3((slots + warps - 1) / warps), dim3(warps * 32), 0, st,
      (const __nv_bfloat16*)x, K, cnt, list, E, cap, (uint8_t*)q, scales, slots);
    if (pdl_rc) return pdl_rc;
  }
  return (int)cudaGetLastError();
}

}  // namespace afb
