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

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_addr[kMaxDevices] = {};  // device address of g_attn_scratch, per device, resolved on first use

// Resolve the array's device address for the current device (once per device). Host code must not use the
// symbol itself as a pointer: on the host it names a stand-in, not device memory.
unsigned char* scratch_for_current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || !p) {
      std::fprintf(stderr, "afb_paged_attention_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", dev,
                   cudaGetErrorString(e));
      return nullptr;
    }
    g_addr[dev] = static_cast<unsigned char*>(p);
  }
  return g_addr[dev];
}

}  // namespace

extern "C" int afb_paged_attention_noalloc(const afb_attn_noalloc_params* p, cudaStream_t stream) {
  if (!p || !p->q || !p->kcache || !p->vcache || !p->block_table || !p->seq_lens || !p->out || p->splits < 1 ||
      p->num_seqs < 0 || p->q_per_seq < 1 || p->Hq < 1 || p->Hkv < 1 || p->Hq % p->Hkv || p->max_pages < 1)
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
  unsigned char* base = scratch_for_current_device();
  if (!base) return AFB_ATTN_NOALLOC_SETUP_FAILED;

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
  return afb::paged_attention(a, p->splits, nullptr, stream);
}
