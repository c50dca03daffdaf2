// Cross-rank agreement check of a small int64 packet (the reference's pair_check_i64 device assert,
// agi2/work/qwen38fn_l4/probes/hostcomm/hostcomm.cu:1429-1441, used to guard that every rank runs the same speculative step): every rank
// stores its packet into every peer's slot, publishes a flag, waits (bounded) for every peer's flag and compares all
// packets with its own. A difference is counted and raises the status bit AFB_ERR_MISMATCH, read by the host: no
// device trap, the context stays usable. Slots are double-buffered by call parity, so a rank one check ahead never
// overwrites the packet a slower peer is still comparing (a rank cannot run two checks ahead: each check waits for
// every peer's flag).
#include "common.cuh"
#include "kernels.h"

namespace afb {

__global__ void __launch_bounds__(256) guard_check_kernel(GuardArgs a, const int64_t* __restrict__ packet, int n,
                                                          uint32_t* status) {
  __shared__ unsigned long long call;
  __shared__ int bad;
  const int tid = threadIdx.x;
  if (tid == 0) {
    call = a.calls[0] + 1;  // this check's sequence number (1-based)
    bad = 0;
  }
  __syncthreads();
  const int par = (int)(call & 1);
  auto slot = [&](int owner, int src) {
    return reinterpret_cast<int64_t*>(a.peer[owner] + a.off_slots) + ((size_t)par * EP_MAX_RANKS + src) * a.n_max;
  };
  for (int i = tid; i < n; i += blockDim.x) {
    const int64_t v = packet[i];
    for (int p = 0; p < a.world; ++p) slot(p, a.rank)[i] = v;
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    for (int p = 0; p < a.world; ++p)
      st_release_sys_u64(reinterpret_cast<uint64_t*>(a.peer[p] + a.off_flags) + a.rank, call);
  }
  if (tid < a.world) {  // bounded wait for every source's packet of this call
    const uint64_t* f = reinterpret_cast<const uint64_t*>(a.peer[a.rank] + a.off_flags) + tid;
    const uint64_t t0 = globaltimer_ns();
    uint32_t polls = 0;
    while (ld_acquire_sys_u64(f) < call) {
      if ((++polls & 63) == 0 && globaltimer_ns() - t0 > AFB_WAIT_NS) {
        flag_error(status, AFB_ERR_PEER_TIMEOUT);
        break;
      }
      __nanosleep(128);
    }
  }
  __syncthreads();
  int cnt = 0;
  for (int i = tid; i < n; i += blockDim.x) {
    const int64_t own = slot(a.rank, a.rank)[i];
    for (int p = 0; p < a.world; ++p) cnt += slot(a.rank, p)[i] != own;
  }
  if (cnt) atomicAdd(&bad, cnt);
  __syncthreads();
  if (tid == 0) {
    a.calls[0] = call;
    if (bad) {
      atomicAdd(a.mismatches, bad);
      flag_error(status, AFB_ERR_MISMATCH);
    }
  }
}

int guard_check(const GuardArgs& a, const int64_t* packet, int n, uint32_t* status, cudaStream_t st) {
  if (n < 1 || n > a.n_max || a.world < 1 || a.world > EP_MAX_RANKS) return 3;
  guard_check_kernel<<<1, 256, 0, st>>>(a, packet, n, status);
  return (int)cudaGetLastError();
}

}  // namespace afb
