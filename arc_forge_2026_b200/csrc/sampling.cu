// Decode-step control kernels: token selection from logits, speculative accept, and the on-device builders of
// the next verify window / drafter block (positions, KV slots from the page table), so one speculative cycle runs
// without host inputs and can be replayed as a CUDA graph.
//
// Token selection: argmax, or exact categorical sampling at temperature T by the Gumbel-max trick,
// argmax_j (z_j / T + G_j) with G_j = -log(-log(u_j)) and u_j from a counter-based hash of (seed, step, row, j)
// (the 64-bit finaliser of splitmix64, Steele et al. 2014), so a replayed step draws the same tokens.
//
// Accept (one thread per sequence): the verify window of a sequence is [x0, d1..dK] at positions ctx..ctx+K
// and target[i] is the target's choice after window row i. The accepted prefix length m is
//   greedy:    the longest prefix with target[i] == d_{i+1}
//   bernoulli: the number of leading successes of Bernoulli(p) draws (BASELINE config 3 decouples acceptance
//              from random weights this way)
// The sequence emits d1..dm and the bonus target[m]; rows 0..m (m+1 tokens) become committed state
// (n_commit for the GDN deferred commit, ctx += m+1) and the bonus is the next anchor.
#include "common.cuh"
#include "kernels.h"

namespace afb {

AFB_DEV uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
AFB_DEV float uniform01(uint64_t seed, uint64_t a, uint64_t b, uint64_t c) {
  const uint64_t h = mix64(seed ^ mix64(a ^ mix64(b ^ mix64(c))));
  return ((h >> 40) + 0.5f) * (1.0f / 16777216.0f);  // 24 random bits, in (0, 1)
}

// one CTA per row; 8 bf16 per thread per step; ties -> lower index
__global__ void __launch_bounds__(256) select_tokens_kernel(const __nv_bfloat16* __restrict__ logits, int ld, int V,
                                                            int* __restrict__ out, float inv_temp, uint64_t seed,
                                                            const int* __restrict__ step, uint32_t* status) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int row = blockIdx.x;
  const __nv_bfloat16* z = logits + (size_t)row * ld;
  const uint64_t st = step ? (uint64_t)*step : 0;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x * 8; c < V; c += 256 * 8) {
    float f[8];
    if (c + 8 <= V) {
      uint4 q = *reinterpret_cast<const uint4*>(z + c);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&q);
#pragma unroll
      for (int t = 0; t < 8; ++t) f[t] = __bfloat162float(h[t]);
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) f[t] = (c + t < V) ? __bfloat162float(z[c + t]) : -INFINITY;
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      float v = f[t];
      if (inv_temp > 0.f && c + t < V) {
        const float u = uniform01(seed, st, row, c + t);
        v = v * inv_temp - __logf(-__logf(u));
      }
      if (v > best) {  // scanning in increasing index: strict > keeps the lowest index
        best = v;
        bi = c + t;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  __shared__ float sv[8];
  __shared__ int si[8];
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    if (bi >= V) {  // every logit NaN: report it and hand out a valid id
      flag_error(status, AFB_ERR_BOUNDS);
      bi = 0;
    }
    out[row] = bi;
  }
}

int select_tokens(const void* logits, int ld, int rows, int V, int* out, float temperature, uint64_t seed,
                  const int* step, uint32_t* status, cudaStream_t st) {
  if (!rows) return 0;
  if (ld % 8) return 3;
  if (const int pdl_rc = launch_pdl(select_tokens_kernel, dim3(rows), dim3(256), 0, st, (const __nv_bfloat16*)logits,
      ld, V, out,
                                             temperature > 0.f ? 1.f / temperature : 0.f, seed, step, status)) return pdl_rc;
  return (int)cudaGetLastError();
}

__global__ void spec_accept_kernel(SpecArgs a) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= a.num_seqs) return;
  const int K = a.k;
  const int W = K + 1;
  const int* win = a.window + (size_t)s * W;
  const int* tgt = a.target + (size_t)s * W;
  const int slot = a.seq_slot[s];
  int m = 0;
  if (a.active && !a.active[s]) {
    a.out_count[s] = 0;
    a.n_commit[slot] = 0;
    return;
  }
  if (a.mode == 1) {
    const uint64_t st = (uint64_t)*a.step;
    while (m < K && uniform01(a.seed, st, s, m + 0x5bd1e995u) < a.accept_prob) ++m;
  } else {
    while (m < K && tgt[m] == win[m + 1]) ++m;
  }
  int* out = a.out_tokens + (size_t)s * W;
  for (int i = 0; i < m; ++i) out[i] = win[i + 1];
  out[m] = tgt[m];
  for (int i = m + 1; i < W; ++i) out[i] = -1;
  a.out_count[s] = m + 1;
  a.n_commit[slot] = m + 1;
  a.ctx_len[s] += m + 1;
  a.anchor[s] = tgt[m];
  a.last_row[s] = s * W + m;
  if (a.total_emitted) atomicAdd(a.total_emitted, (unsigned long long)(m + 1));
}

// The next verify window: ids = [anchor, drafts], positions ctx..ctx+K, KV slots from the page table,
// attention length ctx + K + 1. One thread per window row. Also bumps the step counter (thread 0).
__global__ void build_window_kernel(WindowArgs a) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int W = a.width;
  if (i == 0 && a.step) *a.step += 1;
  if (i >= a.num_seqs * W) return;
  const int s = i / W, r = i % W;
  const int ctx = a.ctx_len[s];
  const int pos = ctx + r + a.pos_offset;
  a.ids[i] = r == 0 ? a.anchor[s] : (a.drafts ? a.drafts[(size_t)s * a.drafts_ld + r - 1] : a.fill_token);
  a.positions[i] = pos;
  const int page = a.block_table[(size_t)s * a.max_pages + pos / 64];
  a.slots[i] = page * 64 + (pos & 63);
  if (r == 0) a.attn_len[s] = pos + W;
}

int spec_accept(const SpecArgs& a, cudaStream_t st) {
  if (!a.num_seqs) return 0;
  if (const int pdl_rc = launch_pdl(spec_accept_kernel, dim3((a.num_seqs + 127) / 128), dim3(128), 0, st,
      a)) return pdl_rc;
  return (int)cudaGetLastError();
}

int build_window(const WindowArgs& a, cudaStream_t st) {
  const int n = a.num_seqs * a.width;
  if (!n) return 0;
  if (const int pdl_rc = launch_pdl(build_window_kernel, dim3((n + 255) / 256), dim3(256), 0, st, a)) return pdl_rc;
  return (int)cudaGetLastError();
}

// gather rows: out[i] = src[idx[i]] (bf16 rows of width H)
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ src, const int* __restrict__ idx,
                                   __nv_bfloat16* __restrict__ out, int H) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int i = blockIdx.x;
  const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)idx[i] * H);
  uint4* d = reinterpret_cast<uint4*>(out + (size_t)i * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) d[c] = s[c];
}

int gather_rows(const void* src, const int* idx, void* out, int rows, int H, cudaStream_t st) {
  if (!rows) return 0;
  if (H % 8) return 3;
  if (const int pdl_rc = launch_pdl(gather_rows_kernel, dim3(rows), dim3(128), 0, st, (const __nv_bfloat16*)src, idx,
      (__nv_bfloat16*)out, H)) return pdl_rc;
  return (int)cudaGetLastError();
}

}  // namespace afb
