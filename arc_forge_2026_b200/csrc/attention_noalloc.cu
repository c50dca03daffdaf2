// Allocation-free variant of the paged decode / verify attention (see attention_noalloc.h for who needs it, the
// size limit and the sharing rules). The split-KV partials live in one file-scope device array; the attention and
// merge kernels are the regular ones of attention.cu, launched through afb::paged_attention.
#include <cstdio>
#include <mutex>

#include "attention_noalloc.h"
#include "kernels.h"

namespace {

// the scratch: [splits, tokens, Hq] log-sum-exp partials, then (256-byte aligned) [splits, tokens, Hq, D] outputs
static __device__ __align__(256) unsigned char g_attn_scratch[AFB_ATTN_NOALLOC_SCRATCH_BYTES];
// the kernels' status word (AFB_ERR_* bits, accumulated by atomicOr until a reset)
static __device__ __align__(16) uint32_t g_attn_status;

constexpr int kMaxDevices = 64;
std::mutex g_mu;
struct DevAddrs {
  unsigned char* scratch = nullptr;
  uint32_t* status = nullptr;
};
DevAddrs g_addr[kMaxDevices];  // device addresses of the two symbols, per device, resolved on first use

// Resolve the symbols' device addresses for the current device (once per device). Host code must not use the
// symbols themselves as pointers: on the host they name stand-ins, not device memory.
const DevAddrs* addrs_for_current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  DevAddrs& d = g_addr[dev];
  if (!d.scratch || !d.status) {
    void* ps = nullptr;
    void* pw = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ps, g_attn_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&pw, g_attn_status);
    if (e != cudaSuccess || !ps || !pw) {
      std::fprintf(stderr, "afb_paged_attention_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", dev,
                   cudaGetErrorString(e));
      return nullptr;
    }
    d.scratch = static_cast<unsigned char*>(ps);
    d.status = static_cast<uint32_t*>(pw);
  }
  return &d;
}

}  // namespace

extern "C" int afb_paged_attention_noalloc(const afb_attn_noalloc_params* p, cudaStream_t stream) {
  if (!p || !p->q || !p->kcache || !p->vcache || !p->block_table || !p->seq_lens || !p->out || p->splits < 1 ||
      p->num_seqs < 0 || p->q_per_seq < 1 || p->Hq < 1 || p->Hkv < 1 || p->Hq % p->Hkv || p->max_pages < 1 ||
      (p->D != 128 && p->D != 256) || p->q_per_seq * (p->Hq / p->Hkv) > 64)
    return AFB_ATTN_NOALLOC_BAD_ARGS;
  const size_t tokens = (size_t)p->num_seqs * p->q_per_seq;
  const size_t lse_bytes = ((size_t)p->splits * tokens * p->Hq * sizeof(float) + 255) & ~size_t(255);
  const size_t o_bytes = (size_t)p->splits * tokens * p->Hq * p->D * sizeof(float);
  if (p->splits > 1 && lse_bytes + o_bytes > AFB_ATTN_NOALLOC_SCRATCH_BYTES) {
    std::fprintf(stderr,
                 "afb_paged_attention_noalloc: %d splits x %zu tokens x %d heads x (D=%d + 1) needs %zu bytes of "
                 "split scratch, more than the fixed %u; use fewer splits\n",
                 p->splits, tokens, p->Hq, p->D, lse_bytes + o_bytes, AFB_ATTN_NOALLOC_SCRATCH_BYTES);
    return AFB_ATTN_NOALLOC_TOO_LARGE;
  }
  const DevAddrs* dev = addrs_for_current_device();
  if (!dev) return AFB_ATTN_NOALLOC_SETUP_FAILED;
  unsigned char* base = dev->scratch;

  afb::AttnArgs a;
  a.q = static_cast<const __nv_bfloat16*>(p->q);
  a.kcache = p->kcache;
  a.vcache = p->vcache;
  a.num_pages = p->num_pages;
  a.block_table = p->block_table;
  a.max_pages = p->max_pages;
  a.seq_lens = p->seq_lens;
  a.num_seqs = p->num_seqs;
  a.q_per_seq = p->q_per_seq;
  a.num_tokens = (int)tokens;
  a.Hq = p->Hq;
  a.Hkv = p->Hkv;
  a.D = p->D;
  a.scale_log2 = p->scale * 1.4426950408889634f;
  a.pages_per_split = (p->max_pages + p->splits - 1) / p->splits;
  a.window = p->window;
  a.gate = static_cast<const __nv_bfloat16*>(p->gate);
  a.gate_ld = p->gate_ld;
  a.gate_head_stride = p->gate_head_stride;
  a.out = static_cast<__nv_bfloat16*>(p->out);
  if (p->splits > 1) {  // every partial the merge reads is written by this call's attention kernel first
    a.part_lse = reinterpret_cast<float*>(base);
    a.part_o = reinterpret_cast<float*>(base + lse_bytes);
  }
  const int rc = afb::paged_attention(a, p->splits, dev->status, stream);
  if (rc >= 1000) return AFB_ATTN_NOALLOC_TMAP_FAILED;  // tensor-map encoding (1000 + driver code)
  if (rc == 3 || rc == 4 || rc == 5) return AFB_ATTN_NOALLOC_UNSUPPORTED;  // the launcher's own refusals
  return rc;                                             // 0 or a cudaError_t of the launch
}

extern "C" int afb_paged_attention_noalloc_status(unsigned int* status, int reset) {
  if (!status) return AFB_ATTN_NOALLOC_BAD_ARGS;
  const DevAddrs* dev = addrs_for_current_device();
  if (!dev) return AFB_ATTN_NOALLOC_SETUP_FAILED;
  uint32_t v = 0;
  cudaError_t e = cudaMemcpy(&v, dev->status, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return (int)e;
  *status = v;
  if (reset) {
    e = cudaMemset(dev->status, 0, sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}
