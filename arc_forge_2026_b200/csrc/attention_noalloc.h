// Allocation-free entry point of the paged decode / verify attention.
//
// This entry point has no counterpart in the reference; it exists for callers of this library that cannot
// allocate device memory themselves -- for example a host application that hands every byte of the GPU to its
// own memory pool, a plugin sandbox that forbids cudaMalloc/cudaFree, or a latency-critical loop that must not
// call them because they synchronise the whole device. It computes the same attention as the regular launcher
// (afb::paged_attention in attention.cu) and keeps the split-KV partial results in a fixed static device array
// instead of caller- or framework-allocated scratch.
//
// Limits and behaviour:
//  * the scratch array holds AFB_ATTN_NOALLOC_SCRATCH_BYTES (4 MiB) on every GPU that loads the library, until
//    the process exits; a call needs splits * num_tokens * Hq * (D + 1) * 4 bytes (plus alignment), and a call that
//    needs more is rejected with AFB_ATTN_NOALLOC_TOO_LARGE and a message on stderr (use fewer splits);
//  * the first call on a device looks up the array's device address (once per device, with that device
//    current); make that first call before any stream capture;
//  * all calls share the one array and it keeps the previous call's contents: every partial a call reads is
//    written by the same call first, and calls that overlap on the GPU (other streams, other threads) race;
//  * a bounded wait inside the attention kernel that gives up (a TMA page copy that never lands) sets a bit in a
//    second fixed device word instead of faulting; the call itself has already returned 0 by then, so after
//    synchronising the stream read the word with afb_paged_attention_noalloc_status (0 = every call since the last
//    reset finished its waits; any other value means some output of those calls is not valid);
//  * it allocates nothing: no cudaMalloc, no cudaFree, no allocating library routine.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AFB_ATTN_NOALLOC_SCRATCH_BYTES (4u << 20)
#define AFB_ATTN_NOALLOC_OK 0
#define AFB_ATTN_NOALLOC_BAD_ARGS (-1)
#define AFB_ATTN_NOALLOC_TOO_LARGE (-2)
#define AFB_ATTN_NOALLOC_SETUP_FAILED (-3)
#define AFB_ATTN_NOALLOC_TMAP_FAILED (-4)    // the K/V cache could not be described to the TMA unit (alignment)
#define AFB_ATTN_NOALLOC_UNSUPPORTED (-5)    // the launcher refused a shape the argument check let through

typedef struct afb_attn_noalloc_params {
  const void* q;            // bf16 [num_seqs * q_per_seq, Hq, D]
  const void* kcache;       // bf16 [num_pages, Hkv, 64, D]
  const void* vcache;       // bf16 [num_pages, Hkv, 64, D]
  int num_pages;
  const int* block_table;   // int32 [num_seqs, max_pages]
  int max_pages;
  const int* seq_lens;      // int32 [num_seqs], tokens in the cache including the q_per_seq new ones
  int num_seqs, q_per_seq, Hq, Hkv, D;
  float scale;              // softmax scale (1/sqrt(D) for standard attention)
  int splits;               // KV splits (>= 1); each split covers ceil(max_pages / splits) pages
  int window;               // > 0: sliding window over the last `window` keys of each query; 0: full causal
  const void* gate;         // optional bf16 output gate, element (tok, head, d) at gate + tok*gate_ld + head*stride + d
  int gate_ld, gate_head_stride;
  void* out;                // bf16 [num_seqs * q_per_seq, Hq, D]
} afb_attn_noalloc_params;

// Returns AFB_ATTN_NOALLOC_OK, a negative AFB_ATTN_NOALLOC_* code, or a positive cudaError_t from the launch.
// Argument errors (D not 128 or 256, Hq not a multiple of Hkv, more than 64 query rows per KV head and sequence,
// i.e. q_per_seq * Hq / Hkv > 64, null pointers) return AFB_ATTN_NOALLOC_BAD_ARGS before anything is launched.
int afb_paged_attention_noalloc(const afb_attn_noalloc_params* p, cudaStream_t stream);

// Reads the current device's kernel status word into *status (0 = clean) and clears it when `reset` is non-zero.
// Synchronous (it copies one word from the device): call it after the attention calls' stream has finished.
// Returns 0, AFB_ATTN_NOALLOC_SETUP_FAILED or a positive cudaError_t.
int afb_paged_attention_noalloc_status(unsigned int* status, int reset);

#ifdef __cplusplus
}
#endif
