// ZeRO-style optimizer step over NVLink peer memory (QAD / RL training, one process per GPU).
//
// The flat fp32 gradients and masters of every parameter group live in a symmetric heap (same offsets on every
// rank). Rank r owns elements [r*chunk, (r+1)*chunk) of each group. One step:
//   signal(GRADS) / wait(GRADS)   -- every rank's backward has finished writing its gradients
//   zero_rs        (per group)    -- reduce-scatter fused with the scale: shard[i] = scale * sum_p grad_p[r*chunk+i],
//                                    pulled with 16-byte peer loads (every peer's load in flight before the adds),
//                                    summed in rank order (bitwise the same on every run), plus per-block sums of
//                                    squares for the norm
//   zero_norm_publish             -- this rank's sum of squares (fixed-order reduction of the block partials) stored
//                                    into every rank's norm slot, then signal(NORM); wait(NORM)
//   zero_adamw     (per group)    -- global norm from the slots (rank order), clip factor, AdamW with bf16 moments on
//                                    the owned shard; the new masters are stored into EVERY rank's heap (the
//                                    all-gather as fire-and-forget peer stores issued by the update itself)
//   signal(PARAMS) / wait(PARAMS) -- every rank's shard has landed everywhere
// The reference reduce-scatters with NCCL inside FSDP2 (training/work/qwen38fn_qad/train_qad.py:140-165); here the
// scale, the clip, the update and the gather ride in the kernels that move the data. Waits are bounded
// (AFB_WAIT_NS) and report AFB_ERR_PEER_TIMEOUT.
// Buffer reuse: a rank rewrites its gradients (next backward) only after wait(PARAMS), which follows every rank's
// wait(NORM), which follows every rank's reduce-scatter reads. A peer stores into this rank's copy of its shard only
// after wait(NORM), when this rank has finished reading gradients and is itself inside the update (it reads only its
// own shard there). The norm slots of step s+1 are written only after every rank passed wait(GRADS) of step s+1,
// which is past its update of step s.
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

// W ranks; U float4 per peer per thread in flight (W * U = 8 loads of 16 bytes per thread)
template <int W>
__global__ void __launch_bounds__(ZT) zero_rs_kernel(ZeroArgs a, size_t grad_off, size_t chunk, float scale,
                                                     float* __restrict__ shard, float* __restrict__ partials) {
  constexpr int U = W >= 8 ? 1 : 8 / W;
  __shared__ float red[ZT / 32];
  float sq = 0.f;
  const size_t c4 = chunk / 4;  // chunk % 4 == 0 and the heap offsets are 256-byte aligned: 16-byte peer loads
  const size_t base4 = (size_t)a.rank * c4;
  const float4* src[W];
#pragma unroll
  for (int p = 0; p < W; ++p) src[p] = reinterpret_cast<const float4*>(a.peer[p] + grad_off) + base4;
  const size_t stride = (size_t)gridDim.x * ZT;
  for (size_t i0 = (size_t)blockIdx.x * ZT + threadIdx.x; i0 < c4; i0 += stride * U) {
    float4 v[U][W];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int p = 0; p < W; ++p)
        if (i0 + u * stride < c4) v[u][p] = src[p][i0 + u * stride];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (i0 + u * stride < c4) {
        float4 s = v[u][0];
#pragma unroll
        for (int p = 1; p < W; ++p) {  // rank order
          s.x += v[u][p].x;
          s.y += v[u][p].y;
          s.z += v[u][p].z;
          s.w += v[u][p].w;
        }
        s.x *= scale;
        s.y *= scale;
        s.z *= scale;
        s.w *= scale;
        reinterpret_cast<float4*>(shard)[i0 + u * stride] = s;
        sq = fmaf(s.x, s.x, fmaf(s.y, s.y, fmaf(s.z, s.z, fmaf(s.w, s.w, sq))));
      }
    }
  }
  const float t = block_sum(sq, red);
  if (threadIdx.x == 0) partials[blockIdx.x] = t;
}

// The block partials of every group summed in a fixed assignment and order (thread t takes t, t + ZT, ...), the
// total stored into every rank's slot for this rank, then the NORM flag.
__global__ void __launch_bounds__(ZT) zero_norm_publish_kernel(ZeroArgs a, const float* __restrict__ partials, int n) {
  __shared__ float red[ZT / 32];
  float t = 0.f;
  for (int i = threadIdx.x; i < n; i += ZT) t += partials[i];
  t = block_sum(t, red);
  if (threadIdx.x != 0) return;
  for (int p = 0; p < a.world; ++p) reinterpret_cast<float*>(a.peer[p] + a.off_norm)[a.rank] = t;
  __threadfence_system();
  const uint64_t v = ++a.sent[ZERO_NORM];
  for (int p = 0; p < a.world; ++p) st_release_sys_u64(zero_flag(a, p, ZERO_NORM, a.rank), v);
}

AFB_DEV float adam_one(float p, float g, __nv_bfloat16& m, __nv_bfloat16& v, float lr, float b1, float b2, float eps,
                       float wd, float bc1, float bc2) {
  const float mi = b1 * __bfloat162float(m) + (1.f - b1) * g;
  const float vi = b2 * __bfloat162float(v) + (1.f - b2) * g * g;
  m = __float2bfloat16(mi);
  v = __float2bfloat16(vi);
  return p - lr * (wd * p + (mi / bc1) / (sqrtf(vi / bc2) + eps));
}

template <int W>
__global__ void __launch_bounds__(ZT) zero_adamw_kernel(ZeroArgs a, size_t param_off, size_t chunk,
                                                        const float* __restrict__ g, __nv_bfloat16* __restrict__ m,
                                                        __nv_bfloat16* __restrict__ v, size_t n_valid, float lr,
                                                        float b1, float b2, float eps, float wd, float bc1, float bc2,
                                                        float max_norm) {
  const float* slots = reinterpret_cast<const float*>(a.peer[a.rank] + a.off_norm);
  float tot = 0.f;
#pragma unroll
  for (int p = 0; p < W; ++p) tot += slots[p];  // rank order: the same norm on every rank
  const float norm = sqrtf(tot);
  const float clip = (max_norm > 0.f && norm > max_norm) ? max_norm / (norm + 1e-6f) : 1.f;
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.norm_out) *a.norm_out = norm;
  if (!isfinite(norm)) return;  // every rank sees the same norm: all skip the update, the host raises
  const size_t c4 = chunk / 4;
  const size_t e0 = (size_t)a.rank * chunk;  // first element of the owned shard
  float4* dst[W];
#pragma unroll
  for (int p = 0; p < W; ++p) dst[p] = reinterpret_cast<float4*>(a.peer[p] + param_off) + (size_t)a.rank * c4;
  const float4* own = reinterpret_cast<const float4*>(a.peer[a.rank] + param_off) + (size_t)a.rank * c4;
  for (size_t i = (size_t)blockIdx.x * ZT + threadIdx.x; i < c4; i += (size_t)gridDim.x * ZT) {
    float4 p4 = own[i];
    const float4 g4 = reinterpret_cast<const float4*>(g)[i];
    uint2 mr = reinterpret_cast<const uint2*>(m)[i], vr = reinterpret_cast<const uint2*>(v)[i];
    __nv_bfloat16* mb = reinterpret_cast<__nv_bfloat16*>(&mr);
    __nv_bfloat16* vb = reinterpret_cast<__nv_bfloat16*>(&vr);
    const size_t e = e0 + 4 * i;
    if (e + 0 < n_valid) p4.x = adam_one(p4.x, g4.x * clip, mb[0], vb[0], lr, b1, b2, eps, wd, bc1, bc2);
    if (e + 1 < n_valid) p4.y = adam_one(p4.y, g4.y * clip, mb[1], vb[1], lr, b1, b2, eps, wd, bc1, bc2);
    if (e + 2 < n_valid) p4.z = adam_one(p4.z, g4.z * clip, mb[2], vb[2], lr, b1, b2, eps, wd, bc1, bc2);
    if (e + 3 < n_valid) p4.w = adam_one(p4.w, g4.w * clip, mb[3], vb[3], lr, b1, b2, eps, wd, bc1, bc2);
    reinterpret_cast<uint2*>(m)[i] = mr;
    reinterpret_cast<uint2*>(v)[i] = vr;
#pragma unroll
    for (int p = 0; p < W; ++p) dst[p][i] = p4;  // the local master and the all-gather as peer stores
  }
  __threadfence_system();  // the peer stores are performed before the PARAMS signal that follows this kernel
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

#define AFB_ZERO_WORLDS(X) X(1) X(2) X(3) X(4) X(5) X(6) X(7) X(8)

// one full wave: the grid-stride loops then give every resident block the same share
template <typename K>
int full_wave(K kernel, int cap) {
  int dev = 0, sms = 0, occ = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, ZT, 0);
  const int b = sms * (occ > 0 ? occ : 1);
  return b < cap ? b : cap;
}

// `blocks` caps the grid (the partials buffer holds that many entries; the ones past the grid stay zero)
int zero_rs(const ZeroArgs& a, size_t grad_off, size_t chunk, float scale, float* shard, float* partials, int blocks,
            cudaStream_t st) {
  if (chunk % 4 || (reinterpret_cast<uintptr_t>(shard) & 15)) return 3;
  switch (a.world) {
#define X(w)                                                                              \
  case w:                                                                                 \
    zero_rs_kernel<w><<<full_wave(zero_rs_kernel<w>, blocks), ZT, 0, st>>>(a, grad_off, chunk, scale, shard, \
                                                                           partials);                      \
    break;
    AFB_ZERO_WORLDS(X)
#undef X
    default:
      return 3;
  }
  return (int)cudaGetLastError();
}
int zero_norm_publish(const ZeroArgs& a, const float* partials, int n, cudaStream_t st) {
  zero_norm_publish_kernel<<<1, ZT, 0, st>>>(a, partials, n);
  return (int)cudaGetLastError();
}
int zero_adamw(const ZeroArgs& a, size_t param_off, size_t chunk, const float* g, void* m, void* v, size_t n_valid,
               float lr, float b1, float b2, float eps, float wd, int step, float max_norm, int blocks,
               cudaStream_t st) {
  if (chunk % 4 || (reinterpret_cast<uintptr_t>(g) & 15) || (reinterpret_cast<uintptr_t>(m) & 7) ||
      (reinterpret_cast<uintptr_t>(v) & 7))
    return 3;
  const float bc1 = 1.f - powf(b1, (float)step), bc2 = 1.f - powf(b2, (float)step);
  switch (a.world) {
#define X(w)                                                                                                   \
  case w:                                                                                                      \
    zero_adamw_kernel<w><<<full_wave(zero_adamw_kernel<w>, blocks), ZT, 0, st>>>(                            \
        a, param_off, chunk, g, (__nv_bfloat16*)m, (__nv_bfloat16*)v, n_valid, lr, b1, b2, eps, wd, bc1, bc2, \
        max_norm);                                                                                             \
    break;
    AFB_ZERO_WORLDS(X)
#undef X
    default:
      return 3;
  }
  return (int)cudaGetLastError();
}

}  // namespace afb
