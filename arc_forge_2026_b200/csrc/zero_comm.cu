// ZeRO-style optimizer step over NVLink peer memory (QAD / RL training, one process per GPU).
//
// The flat fp32 gradients and masters of every parameter group live in a symmetric heap (same offsets on every
// rank). Rank r owns elements [r*chunk, (r+1)*chunk) of each group. One step:
//   signal(GRADS) / wait(GRADS)   -- every rank's backward has finished writing its gradients
//   zero_rs        (per group)    -- reduce-scatter fused with the scale: shard[i] = scale * sum_p grad_p[r*chunk+i],
//                                    summed in rank order (bitwise the same sum on every run), plus per-block sums
//                                    of squares for the norm
//   zero_norm_publish             -- this rank's sum of squares (fixed-order reduction of the block partials) stored
//                                    into every rank's norm slot, then signal(NORM); wait(NORM)
//   zero_adamw     (per group)    -- global norm from the slots (rank order), clip factor, AdamW with bf16 moments on
//                                    the owned shard, new masters written in place
//   signal(PARAMS) / wait(PARAMS)
//   zero_ag        (per group)    -- all-gather by pull: each rank copies the other ranks' updated shards from their
//                                    heaps into its own masters (peer loads, 16-byte vectors)
// The reference reduce-scatters with NCCL inside FSDP2 (training/work/qwen38fn_qad/train_qad.py:140-165); here the
// scale, the clip and the update ride in the kernels that move the data. Waits are bounded (AFB_WAIT_NS) and report
// AFB_ERR_PEER_TIMEOUT. A rank's gradients are rewritten by its next backward only after the PARAMS exchange, which
// every rank enters after its own reduce-scatter reads: no buffer is overwritten while a peer still reads it.
#include "common.cuh"
#include "kernels.h"

namespace afb {

AFB_DEV uint64_t* zero_flag(const ZeroArgs& a, int peer, int type, int src) {
  return reinterpret_cast<uint64_t*>(a.peer[peer] + a.off_flags) + type * EP_MAX_RANKS + src;
}

__global__ void zero_signal_kernel(ZeroArgs a, int type) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  const uint64_t v = ++a.sent[type];
  for (int p = 0; p < a.world; ++p) st_release_sys_u64(zero_flag(a, p, type, a.rank), v);
}

__global__ void zero_wait_kernel(ZeroArgs a, int type, uint32_t* status) {
  const int lane = threadIdx.x;
  const uint64_t want = a.expected[type] + 1;
  if (lane < a.world) {
    const uint64_t* f = zero_flag(a, a.rank, type, lane);
    const uint64_t t0 = globaltimer_ns();
    uint32_t polls = 0;
    while (ld_acquire_sys_u64(f) < want) {
      if ((++polls & 63) == 0 && globaltimer_ns() - t0 > AFB_WAIT_NS) {
        flag_error(status, AFB_ERR_PEER_TIMEOUT);
        break;
      }
      __nanosleep(128);
    }
  }
  __syncwarp();
  if (lane == 0) a.expected[type] = want;
}

constexpr int ZT = 256;  // threads per block

AFB_DEV float block_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0)
    for (int w = 0; w < ZT / 32; ++w) t += red[w];  // fixed order
  return t;
}

__global__ void __launch_bounds__(ZT) zero_rs_kernel(ZeroArgs a, size_t grad_off, size_t chunk, float scale,
                                                     float* __restrict__ shard, float* __restrict__ partials) {
  __shared__ float red[ZT / 32];
  float sq = 0.f;
  const size_t c4 = chunk / 4;  // chunk % 4 == 0 and the heap offsets are 256-byte aligned: 16-byte peer loads
  const size_t base4 = (size_t)a.rank * c4;
  for (size_t i = (size_t)blockIdx.x * ZT + threadIdx.x; i < c4; i += (size_t)gridDim.x * ZT) {
    float4 v[EP_MAX_RANKS];
#pragma unroll
    for (int p = 0; p < EP_MAX_RANKS; ++p)  // every peer's load in flight before the first add
      if (p < a.world) v[p] = reinterpret_cast<const float4*>(a.peer[p] + grad_off)[base4 + i];
    float4 s = v[0];
#pragma unroll
    for (int p = 1; p < EP_MAX_RANKS; ++p)
      if (p < a.world) {  // rank order: the same sum on every run
        s.x += v[p].x;
        s.y += v[p].y;
        s.z += v[p].z;
        s.w += v[p].w;
      }
    s.x *= scale;
    s.y *= scale;
    s.z *= scale;
    s.w *= scale;
    reinterpret_cast<float4*>(shard)[i] = s;
    sq = fmaf(s.x, s.x, fmaf(s.y, s.y, fmaf(s.z, s.z, fmaf(s.w, s.w, sq))));
  }
  const float t = block_sum(sq, red);
  if (threadIdx.x == 0) partials[blockIdx.x] = t;
}

__global__ void zero_norm_publish_kernel(ZeroArgs a, const float* __restrict__ partials, int n) {
  if (threadIdx.x != 0) return;
  float t = 0.f;
  for (int i = 0; i < n; ++i) t += partials[i];  // fixed order
  for (int p = 0; p < a.world; ++p) reinterpret_cast<float*>(a.peer[p] + a.off_norm)[a.rank] = t;
  __threadfence_system();
  const uint64_t v = ++a.sent[ZERO_NORM];
  for (int p = 0; p < a.world; ++p) st_release_sys_u64(zero_flag(a, p, ZERO_NORM, a.rank), v);
}

__global__ void __launch_bounds__(ZT) zero_adamw_kernel(ZeroArgs a, size_t param_off, size_t chunk,
                                                        const float* __restrict__ g, __nv_bfloat16* __restrict__ m,
                                                        __nv_bfloat16* __restrict__ v, size_t n_valid, float lr,
                                                        float b1, float b2, float eps, float wd, float bc1, float bc2,
                                                        float max_norm) {
  float tot = 0.f;
  for (int p = 0; p < a.world; ++p) tot += reinterpret_cast<const float*>(a.peer[a.rank] + a.off_norm)[p];
  const float norm = sqrtf(tot);
  const float clip = (max_norm > 0.f && norm > max_norm) ? max_norm / (norm + 1e-6f) : 1.f;
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.norm_out) *a.norm_out = norm;
  if (!isfinite(norm)) return;  // every rank sees the same norm: all skip the update, the host raises
  float* p = reinterpret_cast<float*>(a.peer[a.rank] + param_off) + (size_t)a.rank * chunk;
  for (size_t i = (size_t)blockIdx.x * ZT + threadIdx.x; i < chunk; i += (size_t)gridDim.x * ZT) {
    if ((size_t)a.rank * chunk + i >= n_valid) break;  // padding of the last shard
    const float gi = g[i] * clip;
    const float mi = b1 * __bfloat162float(m[i]) + (1.f - b1) * gi;
    const float vi = b2 * __bfloat162float(v[i]) + (1.f - b2) * gi * gi;
    m[i] = __float2bfloat16(mi);
    v[i] = __float2bfloat16(vi);
    float pi = p[i];
    pi -= lr * (wd * pi + (mi / bc1) / (sqrtf(vi / bc2) + eps));
    p[i] = pi;
  }
}

__global__ void __launch_bounds__(ZT) zero_ag_kernel(ZeroArgs a, size_t param_off, size_t chunk) {
  float4* own = reinterpret_cast<float4*>(a.peer[a.rank] + param_off);
  const size_t c4 = chunk / 4;
  for (int q = 1; q < a.world; ++q) {
    const int p = (a.rank + q) % a.world;  // staggered: the ranks do not all read the same peer at once
    const float4* src = reinterpret_cast<const float4*>(a.peer[p] + param_off) + (size_t)p * c4;
    float4* dst = own + (size_t)p * c4;
    for (size_t i = (size_t)blockIdx.x * ZT + threadIdx.x; i < c4; i += (size_t)gridDim.x * ZT) dst[i] = src[i];
  }
}

int zero_signal(const ZeroArgs& a, int type, cudaStream_t st) {
  zero_signal_kernel<<<1, 32, 0, st>>>(a, type);
  return (int)cudaGetLastError();
}
int zero_wait(const ZeroArgs& a, int type, uint32_t* status, cudaStream_t st) {
  if (a.world > EP_MAX_RANKS) return 3;
  zero_wait_kernel<<<1, 32, 0, st>>>(a, type, status);
  return (int)cudaGetLastError();
}
int zero_rs(const ZeroArgs& a, size_t grad_off, size_t chunk, float scale, float* shard, float* partials, int blocks,
            cudaStream_t st) {
  if (chunk % 4 || (reinterpret_cast<uintptr_t>(shard) & 15) || a.world < 1 || a.world > EP_MAX_RANKS) return 3;
  zero_rs_kernel<<<blocks, ZT, 0, st>>>(a, grad_off, chunk, scale, shard, partials);
  return (int)cudaGetLastError();
}
int zero_norm_publish(const ZeroArgs& a, const float* partials, int n, cudaStream_t st) {
  zero_norm_publish_kernel<<<1, 32, 0, st>>>(a, partials, n);
  return (int)cudaGetLastError();
}
int zero_adamw(const ZeroArgs& a, size_t param_off, size_t chunk, const float* g, void* m, void* v, size_t n_valid,
               float lr, float b1, float b2, float eps, float wd, int step, float max_norm, int blocks,
               cudaStream_t st) {
  const float bc1 = 1.f - powf(b1, (float)step), bc2 = 1.f - powf(b2, (float)step);
  zero_adamw_kernel<<<blocks, ZT, 0, st>>>(a, param_off, chunk, g, (__nv_bfloat16*)m, (__nv_bfloat16*)v, n_valid, lr,
                                          b1, b2, eps, wd, bc1, bc2, max_norm);
  return (int)cudaGetLastError();
}
int zero_ag(const ZeroArgs& a, size_t param_off, size_t chunk, int blocks, cudaStream_t st) {
  if (chunk % 4) return 3;
  zero_ag_kernel<<<blocks, ZT, 0, st>>>(a, param_off, chunk);
  return (int)cudaGetLastError();
}

}  // namespace afb
