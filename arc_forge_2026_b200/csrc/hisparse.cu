// HiSparse: the attention KV of long sessions lives in pinned host memory; the GPU keeps, per session and layer, a
// ring of the R most recent pages (where this cycle's tokens are written) and a cache of C page slots filled with
// the pages QSA selects. The reference offloads session history the same way (host pool + GPU hot blocks +
// swap-in; paper section 8.2 and its HiSparse bridge, agi2/work/qwen38fn_l4/kaggle/frozen_arc2/hisparse_bridge.py);
// here the swap-in is a device kernel that reads the host pool through its mapped device pointer, so a decode cycle
// needs no host round trip and stays inside one CUDA graph.
//
// GPU page pool of one layer: [S*C cache pages | S*R ring pages | staging pages | scratch page].
// Host pool of one layer: K and V pages by (session row, page index), bf16 [Hkv, 64, D] (exact) or e4m3 with one
// fp32 scale per (page, head) (half the host memory; dequantised on fetch, quantised on write-back).
//
// Per cycle:  hs_cycle_start  -- cycle counter, ring pages mapped into the block table for this cycle's window
//             hs_writeback    -- pages whose 64 tokens became committed go from their ring page to the host pool
//             (qsa_finalize, forward ... per QSA layer: qsa_select, then)
//             hs_fetch        -- every finalised page of the session's union is made resident: hits keep their
//                                slot, misses take the least recently used slot not needed this cycle and are
//                                copied from the host pool; the union's physical pages are rewritten.
#include "common.cuh"
#include "kernels.h"

namespace afb {

namespace hs {
constexpr int THREADS = 256;
constexpr int MAX_MISS = 256;
}  // namespace hs

AFB_DEV int ring_page(const HsArgs& a, int s, int p) { return a.S * a.C + s * a.R + (p % a.R); }

// ------------------------------------------------------------------------------------------------ cycle start
__global__ void hs_cycle_start_kernel(HsArgs a, int* block_table, const int* ctx, int W) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (blockIdx.x == 0 && threadIdx.x == 0) ++*a.cycle;
  if (s >= a.S) return;
  const int c = ctx[s];
  for (int p = c / 64; p <= (c + W - 1) / 64 && p < a.max_pages; ++p)
    block_table[(size_t)s * a.max_pages + p] = ring_page(a, s, p);
}

int hs_cycle_start(const HsArgs& a, int* block_table, const int* ctx, int W, cudaStream_t st) {
  if (a.S <= 0 || a.R < 2) return 3;
  hs_cycle_start_kernel<<<(a.S + 127) / 128, 128, 0, st>>>(a, block_table, ctx, W);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ page copies
// GPU page (bf16 [Hkv, 64, D]) -> host pool entry (bf16 copy, or e4m3 with per-head amax/448 scales)
AFB_DEV void page_to_host(const HsArgs& a, const HsLayer& L, int phys, int s, int p) {
  const size_t elems = (size_t)a.Hkv * 64 * a.D, per_head = (size_t)64 * a.D;
  for (int kv = 0; kv < 2; ++kv) {
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(kv ? L.gpu_v : L.gpu_k) + (size_t)phys * elems;
    const size_t entry = (size_t)s * a.max_pages + p;
    if (!a.fp8) {
      uint4* dst = reinterpret_cast<uint4*>(kv ? L.host_v : L.host_k) + entry * elems / 8;
      const uint4* s4 = reinterpret_cast<const uint4*>(src);
      for (size_t i = threadIdx.x; i < elems / 8; i += blockDim.x) dst[i] = s4[i];
      continue;
    }
    __shared__ float amax[8];
    float* scales = (kv ? L.host_sv : L.host_sk) + entry * a.Hkv;
    uint8_t* dst = (kv ? L.host_v : L.host_k) + entry * elems;
    for (int h = 0; h < a.Hkv; ++h) {
      float m = 0.f;
      for (size_t i = threadIdx.x; i < per_head; i += blockDim.x) m = fmaxf(m, fabsf(__bfloat162float(src[h * per_head + i])));
      m = warp_max(m);
      if ((threadIdx.x & 31) == 0) amax[threadIdx.x >> 5] = m;
      __syncthreads();
      float mm = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) mm = fmaxf(mm, amax[w]);
      const float sc = mm > 0.f ? mm / 448.f : 1.f, inv = 1.f / sc;
      for (size_t i = threadIdx.x * 4; i < per_head; i += blockDim.x * 4) {
        const __nv_bfloat16* x = src + h * per_head + i;
        __nv_fp8x4_e4m3 q(make_float4(__bfloat162float(x[0]) * inv, __bfloat162float(x[1]) * inv,
                                      __bfloat162float(x[2]) * inv, __bfloat162float(x[3]) * inv));
        *reinterpret_cast<__nv_fp8x4_e4m3*>(dst + h * per_head + i) = q;
      }
      if (threadIdx.x == 0) scales[h] = sc;
      __syncthreads();  // amax reused by the next head
    }
  }
}

// host pool entry -> GPU page
AFB_DEV void page_from_host(const HsArgs& a, const HsLayer& L, int phys, int s, int p) {
  const size_t elems = (size_t)a.Hkv * 64 * a.D, per_head = (size_t)64 * a.D;
  const size_t entry = (size_t)s * a.max_pages + p;
  for (int kv = 0; kv < 2; ++kv) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(kv ? L.gpu_v : L.gpu_k) + (size_t)phys * elems;
    if (!a.fp8) {
      const uint4* src = reinterpret_cast<const uint4*>(kv ? L.host_v : L.host_k) + entry * elems / 8;
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll 4
      for (size_t i = threadIdx.x; i < elems / 8; i += blockDim.x) d4[i] = src[i];
      continue;
    }
    const uint8_t* src = (kv ? L.host_v : L.host_k) + entry * elems;
    const float* scales = (kv ? L.host_sv : L.host_sk) + entry * a.Hkv;
#pragma unroll 2
    for (size_t i = threadIdx.x * 8; i < elems; i += blockDim.x * 8) {
      const float sc = scales[i / per_head];
      const uint2 raw = *reinterpret_cast<const uint2*>(src + i);
      const __nv_fp8x4_e4m3* q = reinterpret_cast<const __nv_fp8x4_e4m3*>(&raw);
      const float4 f0 = float4(q[0]), f1 = float4(q[1]);
      *reinterpret_cast<uint4*>(dst + i) = make_uint4(pack_bf16x2(f0.x * sc, f0.y * sc), pack_bf16x2(f0.z * sc, f0.w * sc),
                                                      pack_bf16x2(f1.x * sc, f1.y * sc), pack_bf16x2(f1.z * sc, f1.w * sc));
    }
  }
}

// ------------------------------------------------------------------------------------------------ write-back
// grid (sessions, layers): pages [fin[s], ctx[s]/64) -- complete and committed -- from their ring page to the host
__global__ void __launch_bounds__(hs::THREADS) hs_writeback_kernel(HsArgs a, HsLayers Ls, const int* block_table,
                                                                   const int* fin, const int* ctx) {
  const int s = blockIdx.x, l = blockIdx.y;
  const int hi = min(ctx[s] / 64, a.max_pages);
  for (int p = fin[s]; p < hi; ++p) page_to_host(a, Ls.l[l], block_table[(size_t)s * a.max_pages + p], s, p);
}

int hs_writeback(const HsArgs& a, const HsLayers& Ls, int layers, const int* block_table, const int* fin,
                 const int* ctx, cudaStream_t st) {
  if (layers < 1 || layers > QSA_MAX_LAYERS || a.Hkv > 8 || a.D % 8) return 3;
  if (a.S <= 0) return 0;
  hs_writeback_kernel<<<dim3(a.S, layers), hs::THREADS, 0, st>>>(a, Ls, block_table, fin, ctx);
  return (int)cudaGetLastError();
}

// staging -> host for pages [p0, p1) of one session, and staging -> ring for pages [p1, p2) (after a prefill)
__global__ void __launch_bounds__(hs::THREADS) hs_after_prefill_kernel(HsArgs a, HsLayers Ls, const int* block_table,
                                                                       int s, int p0, int p1, int p2) {
  const int l = blockIdx.y, p = p0 + blockIdx.x;
  if (p >= p2) return;
  const int src = block_table[(size_t)s * a.max_pages + p];
  if (p < p1) {
    page_to_host(a, Ls.l[l], src, s, p);
    return;
  }
  const int dst = ring_page(a, s, p);
  const size_t elems = (size_t)a.Hkv * 64 * a.D;
  for (int kv = 0; kv < 2; ++kv) {
    const uint4* s4 = reinterpret_cast<const uint4*>(kv ? Ls.l[l].gpu_v : Ls.l[l].gpu_k) + (size_t)src * elems / 8;
    uint4* d4 = reinterpret_cast<uint4*>(kv ? Ls.l[l].gpu_v : Ls.l[l].gpu_k) + (size_t)dst * elems / 8;
    for (size_t i = threadIdx.x; i < elems / 8; i += blockDim.x) d4[i] = s4[i];
  }
  if (Ls.l[l].raw) {  // raw index keys of the page's tokens (64 x 128 bf16)
    const uint4* s4 = reinterpret_cast<const uint4*>(Ls.l[l].raw + (size_t)src * 64 * 128);
    uint4* d4 = reinterpret_cast<uint4*>(Ls.l[l].raw + (size_t)dst * 64 * 128);
    for (int i = threadIdx.x; i < 64 * 128 / 8; i += blockDim.x) d4[i] = s4[i];
  }
}

int hs_after_prefill(const HsArgs& a, const HsLayers& Ls, int layers, const int* block_table, int s, int p0, int p1,
                     int p2, cudaStream_t st) {
  if (layers < 1 || layers > QSA_MAX_LAYERS) return 3;
  if (p2 <= p0) return 0;
  hs_after_prefill_kernel<<<dim3(p2 - p0, layers), hs::THREADS, 0, st>>>(a, Ls, block_table, s, p0, p1, p2);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ fetch
__global__ void __launch_bounds__(hs::THREADS) hs_fetch_kernel(HsArgs a, HsLayer L, int* u_page, const int* u_lpage,
                                                               const int* u_count, int ucap, const int* fin,
                                                               uint32_t* status) {
  __shared__ int miss_i[hs::MAX_MISS];
  __shared__ int miss_slot[hs::MAX_MISS];
  __shared__ int nmiss;
  const int s = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  const int cyc = *a.cycle, n = u_count[s], F = fin[s];
  int* res = L.res + (size_t)s * a.max_pages;
  int* slot_page = L.slot_page + (size_t)s * a.C;
  int* stamp = L.stamp + (size_t)s * a.C;
  if (tid == 0) nmiss = 0;
  __syncthreads();
  // hits keep their slot (and are stamped so no miss of this cycle evicts them)
  for (int i = tid; i < n; i += blockDim.x) {
    const int b = u_lpage[(size_t)s * ucap + i];
    if (b >= F) continue;  // local page: ring, already in the union
    const int slot = res[b];
    if (slot >= 0) {
      stamp[slot] = cyc;
      u_page[(size_t)s * ucap + i] = s * a.C + slot;
    } else {
      const int m = atomicAdd(&nmiss, 1);
      if (m < hs::MAX_MISS) miss_i[m] = i;
    }
  }
  __syncthreads();
  const int nm = min(nmiss, hs::MAX_MISS);
  if (tid == 0 && nmiss > hs::MAX_MISS) flag_error(status, AFB_ERR_BOUNDS);
  // victims: warp 0 picks, per miss, the least recently used slot not stamped this cycle (lowest slot on ties)
  if (tid < 32) {
    for (int m = 0; m < nm; ++m) {
      int best = -1;
      long long key = 0x7fffffffffffffffll;
      for (int c = lane; c < a.C; c += 32) {
        const int st = stamp[c];
        const long long k = ((long long)st << 20) | c;
        if (st != cyc && k < key) {
          key = k;
          best = c;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const long long ok = __shfl_xor_sync(0xffffffffu, key, o);
        const int ob = __shfl_xor_sync(0xffffffffu, best, o);
        if (ok < key) {
          key = ok;
          best = ob;
        }
      }
      if (lane == 0) {
        const int i = miss_i[m];
        const int b = u_lpage[(size_t)s * ucap + i];
        if (best < 0) {  // more pages wanted this cycle than slots: leave it on the scratch page
          flag_error(status, AFB_ERR_BOUNDS);
          miss_slot[m] = -1;
        } else {
          const int old = slot_page[best];
          if (old >= 0) res[old] = -1;
          res[b] = best;
          slot_page[best] = b;
          stamp[best] = cyc;
          miss_slot[m] = best;
          u_page[(size_t)s * ucap + i] = s * a.C + best;
        }
      }
      __syncwarp();
    }
  }
  __syncthreads();
  for (int m = 0; m < nm; ++m) {  // copies, all threads
    if (miss_slot[m] < 0) continue;
    page_from_host(a, L, s * a.C + miss_slot[m], s, u_lpage[(size_t)s * ucap + miss_i[m]]);
  }
}

int hs_fetch(const HsArgs& a, const HsLayer& L, int* u_page, const int* u_lpage, const int* u_count, int ucap,
             const int* fin, uint32_t* status, cudaStream_t st) {
  if (a.C < 1 || a.C >= (1 << 20) || a.D % 8) return 3;
  if (a.S <= 0) return 0;
  hs_fetch_kernel<<<a.S, hs::THREADS, 0, st>>>(a, L, u_page, u_lpage, u_count, ucap, fin, status);
  return (int)cudaGetLastError();
}

}  // namespace afb
