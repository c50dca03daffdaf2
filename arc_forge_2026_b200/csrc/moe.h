// Arguments of the INT3 / block-FP8 routed-expert GEMM (see moe_int3.cu for the contract and layouts).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace afb {

struct MoeGemmArgs {
  // weights (INT3 tile layout)
  const int32_t* codes = nullptr;  // [E, rows/128, K/128, 128, 12]
  const void* scales = nullptr;    // bf16 [E, rows/128, K/128, 128]
  int num_experts = 0;
  int rows = 0;  // weight rows per expert (2I for w13, H for w2)
  int K = 0;     // reduction dim (H for w13, I for w2)
  // routed rows: for source p < route_srcs and expert e, route_cnt[p * E + e] entries listed at
  // route_list[(p * E + e) * route_cap + i] (entry = token * top_k + slot, numbered over all sources); the
  // activation row of an entry is entry / x_div (x_div = top_k when x holds one row per token, 1 when it holds one
  // row per entry), its output row is the entry itself
  const int* route_cnt = nullptr;
  const int* route_list = nullptr;
  int route_cap = 0, route_srcs = 1, x_div = 1;
  const void* x_q = nullptr;        // e4m3 [x_rows, K]
  const float* x_scales = nullptr;  // INT3: fp32 [x_rows] (one per row); block FP8: group-major [K/128, ld_xs]
  int ld_xs = 0;
  int x_rows = 0;
  // outputs, one row per entry
  uint8_t* out_q = nullptr;      // block-FP8 PAIR: e4m3 [entries, I]
  float* out_scales = nullptr;   // block-FP8 PAIR: fp32 [I/128, ld_os] (group-major)
  int ld_os = 0;
  void* out_bf16 = nullptr;      // INT3 PAIR: h bf16 [entries, I]; !PAIR: y bf16 [entries, H]
  int out_ld = 0;
  const float* route_w = nullptr;  // !PAIR: routing weight per entry, or null
  // block-FP8 experts instead of INT3 (the teacher): e4m3 weights [E, rows, K] and fp32 scales per 128 x 128 block
  // [E, rows/128, K/128]; codes / scales above are then unused
  const uint8_t* fp8_w = nullptr;
  const float* fp8_scales = nullptr;
  long long* dbg = nullptr;        // optional profiling counters [grid, 4 roles, 5]: wait cycles, total, k-steps,
                                   // cycles of the role's main section and of a second one
  // !PAIR under expert parallelism: entry e belongs to rank e / ep_entries_per_rank and its routed row goes to that
  // rank's combine region at (e % ep_entries_per_rank); the last CTA then publishes the combine exchange on every
  // rank (flag protocol of ep.cu)
  int ep_world = 0, ep_rank = 0, ep_entries_per_rank = 0;
  uint8_t* ep_peer[8] = {};
  size_t ep_off_comb = 0, ep_off_flags = 0;
  unsigned* ep_done = nullptr;             // local CTA-completion counter of the combine exchange
  unsigned long long* ep_sent = nullptr;   // local published-combine counter
  // PAIR under expert parallelism: wait (bounded) in the prologue until every source rank has published this
  // exchange's dispatch (flags [sources] in the local heap), then count it consumed (last CTA)
  const uint64_t* ep_wait_flags = nullptr;
  unsigned long long* ep_wait_ns = nullptr;  // optional: block 0 adds its dispatch wait (ns) here
  unsigned long long* ep_expected = nullptr;
  unsigned* ep_wait_done = nullptr;
};

int moe_int3_gemm(const MoeGemmArgs& a, int pair, int num_sms, uint32_t* status, cudaStream_t st);

}  // namespace afb
