// Arguments of the INT3 grouped expert GEMM (see moe_int3.cu for the contract and layouts).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace afb {

struct MoeGemmArgs {
  // weights (tile layout)
  const int32_t* codes = nullptr;  // [E, rows/128, K/128, 128, 12]
  const void* scales = nullptr;    // bf16 [E, rows/128, K/128, 128]
  int num_experts = 0;
  int rows = 0;  // weight rows per expert (2I for w13, H for w2)
  int K = 0;     // reduction dim (H for w13, I for w2)
  // activations, sorted by expert
  const int* expert_offsets = nullptr;  // [E+1] device
  const void* x_q = nullptr;            // e4m3 [num_rows_total, K]
  const float* x_scales = nullptr;      // fp32 [K/128, ld_xs] (group-major)
  int ld_xs = 0;
  int num_rows_total = 0;               // capacity of x_q (rows beyond the live count are ignored)
  // outputs
  uint8_t* out_q = nullptr;      // PAIR: e4m3 [rows_total, out_ld] (out_ld = I)
  float* out_scales = nullptr;   // PAIR: fp32 [I/128, ld_os] (group-major, feeds the next GEMM)
  int ld_os = 0;
  void* out_bf16 = nullptr;      // !PAIR: bf16 [rows_total, out_ld] (out_ld = H)
  int out_ld = 0;
  const float* route_w = nullptr;  // !PAIR: routing weight per (token, slot) entry, or null
  const int* row_entry = nullptr;  // !PAIR: sorted row -> entry index
  // block-FP8 experts instead of INT3 (the teacher): e4m3 weights [E, rows, K] and fp32 scales per 128 x 128 block
  // [E, rows/128, K/128]; codes / scales above are then unused
  const uint8_t* fp8_w = nullptr;
  const float* fp8_scales = nullptr;
  long long* dbg = nullptr;        // optional profiling counters [grid, 4 roles, 3]: wait cycles, total, k-steps
  // !PAIR under expert parallelism: row_entry indexes all ranks' (token, slot) entries; entry e belongs to rank
  // e / ep_entries_per_rank and its routed row goes to that rank's combine region at (e % ep_entries_per_rank);
  // the last CTA then publishes the combine exchange on every rank (flag protocol of ep.cu)
  int ep_world = 0, ep_rank = 0, ep_entries_per_rank = 0;
  uint8_t* ep_peer[8] = {};
  size_t ep_off_comb = 0, ep_off_flags = 0;
  unsigned* ep_done = nullptr;             // local CTA-completion counter of the combine exchange
  unsigned long long* ep_sent = nullptr;   // local published-combine counter
};

int moe_int3_gemm(const MoeGemmArgs& a, int pair, int num_sms, uint32_t* status, cudaStream_t st);

}  // namespace afb
