// Host-callable launchers of the non-GEMM kernels (raw device pointers + stream; no torch headers).
// Every launcher returns 0 on success, 3 for an unsupported shape, or a cudaError_t code.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace afb {

// elementwise.cu
int rmsnorm(const void* x, void* residual, const void* w, void* y, int rows, int H, float eps, int zero_centered,
            cudaStream_t st);
int qk_norm_rope_store(const void* qkv, int ld, int T, int Hq, int Hkv, int D, int rot, const void* qw, const void* kw,
                       const int* positions, const int* slots, const float* cos_t, const float* sin_t, float eps,
                       void* q_out, void* kcache, void* vcache, int page_size, cudaStream_t st,
                       uint8_t* kscale = nullptr, uint8_t* vscale = nullptr);  // scales given: NVFP4 cache
int router_topk(const float* logits, int ld, int T, int E, int k, int renorm, int* ids, float* weights,
                cudaStream_t st, int* cnt = nullptr, int* list = nullptr, int cap = 0);
int expert_sort(const int* ids, int n, int E, const int* expert_map, int* offsets, int* row_token, int* row_entry,
                int* entry_row, int k, int pad, cudaStream_t st);
int quant_rows_e4m3(const void* x, int ldx, const int* row_token, const int* nrows_dev, int nrows, int K, void* q,
                    float* scales, int ld_s, cudaStream_t st);
// one scale per row, s = max(amax, 1e-30) / 448 (the INT3 experts' W3A8 activation rule); K % 8 == 0
int quant_rows_e4m3_row(const void* x, int ldx, const int* row_token, const int* nrows_dev, int nrows, int K, void* q,
                        float* scales, cudaStream_t st);
int moe_combine(const void* y, const int* entry_row, int k, const void* shared, const float* router_logits,
                int ld_logits, int sg_col, const void* resid, void* out, int T, int H, cudaStream_t st,
                const struct EpArgs* wait_combine = nullptr, uint32_t* status = nullptr);
int swiglu(const void* x, void* y, int T, int I, cudaStream_t st);
int embedding(const int* ids, const void* table, void* out, int T, int H, int V, uint32_t* status, cudaStream_t st);

// attention.cu
struct AttnArgs {
  const __nv_bfloat16* q = nullptr;  // [num_tokens, Hq, D], num_tokens = num_seqs * q_per_seq
  const void* kcache = nullptr;      // [num_pages, Hkv, 64, D] bf16, or NVFP4: [num_pages, Hkv, 64, D/2] e2m1 pairs
  const void* vcache = nullptr;
  const uint8_t* kscale = nullptr;   // NVFP4 only: [num_pages, Hkv, 64, D/16] e4m3, one scale per 16 elements
  const uint8_t* vscale = nullptr;
  int num_pages = 0;
  const int* block_table = nullptr;  // [num_seqs, max_pages]
  int max_pages = 0;
  const int* seq_lens = nullptr;     // [num_seqs], including the q_per_seq new tokens
  int num_seqs = 0, q_per_seq = 1, num_tokens = 0;
  int Hq = 0, Hkv = 0, D = 0;
  float scale_log2 = 0.f;            // softmax scale * log2(e)
  int pages_per_split = 1 << 30;
  int window = 0;                    // > 0: sliding-window attention over the last `window` keys per query
  const int* bt_row = nullptr;       // optional [num_seqs]: block-table row of each (virtual) sequence
  const __nv_bfloat16* gate = nullptr;  // optional output gate: out *= sigmoid(gate[tok*gate_ld + head*stride + d])
  int gate_ld = 0, gate_head_stride = 0;
  __nv_bfloat16* out = nullptr;         // [num_tokens, Hq, D]
  float* part_o = nullptr;              // [splits, num_tokens, Hq, D]
  float* part_lse = nullptr;            // [splits, num_tokens, Hq]
  // QSA sparse mode (all null: dense). An entry is a block of sp_block tokens: sp_count[seq] entries are live,
  // sp_lpage gives each entry's block index in the sequence (key positions) and sp_mask the bitmask of verify rows
  // that attend to it (rows [seq, sp_ld]). sp_block 64: a block is a page and block_table rows hold the physical
  // page of each entry (the union; sp_ld = max_pages). sp_block < 64 (a divisor of 64; tcgen05 kernel only): the
  // block table is the sequences' own and the kernel gathers 64 / sp_block entries into each 64-key tile.
  const int* sp_count = nullptr;
  const int* sp_lpage = nullptr;
  const uint8_t* sp_mask = nullptr;
  int sp_block = 64, sp_ld = 0;
  const int* sp_slot = nullptr;      // sub-page mode: [seq, sp_ld] KV slot (page * 64 + offset) of each entry's first
                                     // token (the union builder resolves the block table once per entry)
  // 0: the tcgen05 kernel (attention_tc.cu) wherever it applies (bf16 cache, dense, no window, no virtual rows),
  // else the mma.sync kernel; 1: always the mma.sync kernel
  int impl = 0;
};
int paged_attention(const AttnArgs& a, int splits, uint32_t* status, cudaStream_t st);

// attention_train.cu: variable-length causal attention of packed training rows, forward and backward (tcgen05)
struct AttnTrainArgs {
  const __nv_bfloat16* q = nullptr;     // [T, Hq, D] (normed, rotated)
  const __nv_bfloat16* k = nullptr;     // [T, Hkv, D]
  const __nv_bfloat16* v = nullptr;     // [T, Hkv, D]
  const int* cu = nullptr;              // [segments + 1] row offsets
  const int2* tiles = nullptr;          // [ntiles] (segment, first position of a 64-position tile)
  int ntiles = 0;
  int T = 0, Hq = 0, Hkv = 0, D = 0;
  float scale = 0.f, scale_log2 = 0.f;  // softmax scale, and times log2(e)
  __nv_bfloat16* out = nullptr;         // forward: written; backward: read
  float* lse = nullptr;                 // [Hq, T] row log-sum-exp of the scaled scores, log2 domain
  const __nv_bfloat16* dout = nullptr;  // backward
  const float* delta = nullptr;         // [Hq, T] backward scratch: rowsum(dO * O)
  __nv_bfloat16* dq = nullptr;          // [T, Hq, D]
  __nv_bfloat16* dk = nullptr;          // [T, Hkv, D]
  __nv_bfloat16* dv = nullptr;
  float* dk_part = nullptr;             // [T, Hq, D] backward scratch: each query head's fp32 contribution
  float* dv_part = nullptr;
  // QSA (optional): per row, bit b of blkmap[row * blk_words + b / 32] = the row attends to block b of its segment
  // (blocks of qsa_block tokens); keys of unmarked blocks are masked like future keys
  const uint32_t* blkmap = nullptr;
  int blk_words = 0, qsa_block = 64;
  // 0: bidirectional within each segment (forward only; the vision tower's attention), 1: causal
  int causal = 1;
};
int attn_train_fwd(const AttnTrainArgs& a, uint32_t* status, cudaStream_t st);

// vision tower (csrc/vision.cu): acc = the fp32 patch-embedding GEMM output, bf16 elsewhere
int vit_patch_pos(const float* acc, const void* bias, const void* table, const int* idx, const void* wts, void* h,
                  int P, int C, cudaStream_t st);
int vit_qkv_rope(const void* qkv, const float* cosv, const float* sinv, int P, int H, int Dh, int Dp, void* q,
                 void* k, void* v, cudaStream_t st);
int vit_layernorm(const void* x, const void* w, const void* b, float eps, void* y, int rows, int C, cudaStream_t st);
// kv_tiles [nkv]: the 128-key tiles of the dK / dV kernels (most work first); a.tiles: 64-row query tiles of dQ
int attn_train_bwd(const AttnTrainArgs& a, const int2* kv_tiles, int nkv, uint32_t* status, cudaStream_t st);
// QSA training selection -> per-row block bitmap: row set s (W rows starting at packed row set_row0[s], the first
// set_rows[s] of them real) marks block u_lpage[s][e] for each row whose bit is set in u_mask[s][e]
int qsa_rowmap(const int* u_lpage, const uint8_t* u_mask, const int* u_count, const int* set_row0,
               const int* set_rows, int S, int W, int ucap, uint32_t* blkmap, int words, cudaStream_t st);

// qsa.cu: QSA indexer, block selection and union for block-sparse verify attention (block = `block` tokens, a
// divisor of the 64-token page: 64 makes a block one page)
constexpr int QSA_MAX_LAYERS = 64;
struct QsaArgs {
  int Hi = 4, Di = 128, rot = 64;           // index heads, head dim, RoPE dims
  float eps = 1e-6f;
  const __nv_bfloat16* q_norm = nullptr;    // [Di] (zero-centred weight: x * (1 + w))
  const float* cos_t = nullptr;             // [positions, rot/2]
  const float* sin_t = nullptr;
  __nv_bfloat16* idx_q = nullptr;           // [tokens, Hi, Di]
  __nv_bfloat16* idx_raw = nullptr;         // [num_pages * 64, Di] per-token raw index keys (by KV slot)
  const __nv_bfloat16* idx_key = nullptr;   // [S * max_blocks, Di] pooled keys of finalised blocks (session, block)
};
struct QsaSelectArgs {
  const int* block_table = nullptr;  // [S, max_pages]
  int max_pages = 0, max_blocks = 0;
  int block = 64;                    // tokens per block (divides 64)
  const int* fin = nullptr;          // [sessions] finalised blocks per session
  const int* seq_lens = nullptr;     // [S] tokens including this cycle's W verify rows
  const int* bt_row = nullptr;       // optional [S]: session of each row set (prefill); null: set s is session s
  int W = 1, K = 32;
  // blocks completed inside the verify window have no pooled key yet: they are pooled on the fly from the raw keys
  const __nv_bfloat16* k_norm = nullptr;
  uint32_t* sel = nullptr;           // [S, max_blocks + 1] row bitmasks, all zero between calls (the union clears them)
  int* u_page = nullptr;             // [S, ucap] physical page of each union entry (block 64), or the KV slot of
                                     // its first token (smaller blocks)
  int* u_lpage = nullptr;            // [S, ucap] block index in the sequence
  uint8_t* u_mask = nullptr;         // [S, ucap] rows that attend to the block
  int* u_count = nullptr;            // [S]
  int ucap = 0;
  // optional [S, W, scores_ld] fp32 scratch: the committed blocks' scores come from the tensor-core score kernel
  // (W * Hi <= 32); null: the per-row kernel scores them on the CUDA cores
  float* scores = nullptr;
  int scores_ld = 0;
  int key_rows = 0;                  // rows of idx_key (sessions * max_blocks), for its tensor map
  int q_rows = 0;                    // rows of idx_q
};
struct QsaFinalizeArgs {
  const __nv_bfloat16* idx_raw[QSA_MAX_LAYERS] = {};
  __nv_bfloat16* idx_key[QSA_MAX_LAYERS] = {};
  const __nv_bfloat16* k_norm[QSA_MAX_LAYERS] = {};
  const int* block_table = nullptr;  // [S, max_pages]
  int max_pages = 0, max_blocks = 0, block = 64;
  int* fin = nullptr;                // [S] in: finalised blocks so far; out: ctx / block
  const int* ctx = nullptr;          // [S] committed tokens
  const float* cos_t = nullptr;
  const float* sin_t = nullptr;
  int rot = 64;
  float eps = 1e-6f;
};
int qsa_prep(const QsaArgs& a, const void* proj, int ld, int T, const int* positions, const int* slots,
             cudaStream_t st);
int qsa_finalize(const QsaFinalizeArgs& f, int S, int layers, cudaStream_t st);
int qsa_select(const QsaArgs& a, const QsaSelectArgs& sa, int S, uint32_t* status, cudaStream_t st);

// hisparse.cu: host-memory KV pool with per-session GPU page caches (QSA layers)
struct HsArgs {
  int S = 0, max_pages = 0, C = 0, R = 4, Hkv = 0, D = 0;
  int fp8 = 0;            // host pool in e4m3 with per-(page, head) scales
  int* cycle = nullptr;   // device cycle counter (stamps of the cache slots)
};
struct HsLayer {
  uint8_t* gpu_k = nullptr;   // GPU page pool of the layer, bf16 [pages, Hkv, 64, D]
  uint8_t* gpu_v = nullptr;
  uint8_t* host_k = nullptr;  // device pointer of the mapped host pool [S * max_pages] pages (bf16 or e4m3)
  uint8_t* host_v = nullptr;
  float* host_sk = nullptr;   // e4m3 scales [S * max_pages, Hkv]
  float* host_sv = nullptr;
  int* res = nullptr;         // [S, max_pages] cache slot of each page, -1 if not resident
  int* slot_page = nullptr;   // [S, C] page held by each slot, -1 if empty
  int* stamp = nullptr;       // [S, C] cycle of last use, -1 if never
  __nv_bfloat16* raw = nullptr;  // optional raw index-key cache [pages * 64, 128] (moved with ring pages)
};
struct HsLayers {
  HsLayer l[QSA_MAX_LAYERS];
};
int hs_cycle_start(const HsArgs& a, int* block_table, const int* ctx, int W, cudaStream_t st);
int hs_writeback(const HsArgs& a, const HsLayers& Ls, int layers, const int* block_table, const int* fin,
                 const int* ctx, cudaStream_t st);
int hs_after_prefill(const HsArgs& a, const HsLayers& Ls, int layers, const int* block_table, int s, int p0, int p1,
                     int p2, cudaStream_t st);
int hs_fetch(const HsArgs& a, const HsLayer& L, int* u_page, const int* u_lpage, const int* u_count, int ucap,
             const int* fin, uint32_t* status, cudaStream_t st);

// gdn.cu
struct GdnArgs {
  const __nv_bfloat16* mixed = nullptr;  // in_proj output [tokens, mixed_ld]: [q|k|v] conv channels, z, b, a
  int mixed_ld = 0, z_off = 0, ba_off = 0;
  const float* conv_w = nullptr;         // [C, 4]
  __nv_bfloat16* conv_state = nullptr;   // [slots, 3, C]
  float* ssm_state = nullptr;            // [slots, Hv, Dv, Dk]: S transposed
  __nv_bfloat16* pend_in = nullptr;      // [2, pend_slots, max_q, C]
  __nv_bfloat16* pend_qk = nullptr;      // [2, pend_slots, max_q, 2*Hk*Dk]
  __nv_bfloat16* pend_v = nullptr;       // [2, pend_slots, max_q, Hv*Dv]
  float* pend_gb = nullptr;              // [2, pend_slots, Hv, max_q, 2] (g, beta), head-major
  const int* n_commit = nullptr;         // [slots] accepted tokens of the previous cycle
  const int* seq_slot = nullptr;         // [num_seqs]
  const float* A_log = nullptr;
  const float* dt_bias = nullptr;
  const __nv_bfloat16* norm_w = nullptr; // [Dv]
  __nv_bfloat16* out = nullptr;          // [tokens, Hv*Dv]
  int num_seqs = 0, q_per_seq = 1, max_q = 1, num_slots = 0, pend_slots = 0;
  int conv_dim = 0, Hk = 0, Hv = 0, Dk = 0, Dv = 0;
  int commit_current = 0;
  float eps = 1e-6f;
  long long* dbg = nullptr;  // optional profiling of the tensor-core verify kernel: per CTA 24 clock64 section sums
};
int gdn_decode(const GdnArgs& a, int parity, int num_sms, uint32_t* status, cudaStream_t st);

// gdn_chunk.cu: inter-chunk state scan of the chunked gated delta rule (training), fp32, contiguous
struct GdnScanArgs {
  const float* m1 = nullptr;      // [BH, n, C, Dk]
  const float* m2 = nullptr;      // [BH, n, C, Dk]
  const float* y = nullptr;       // [BH, n, C, Dv]
  const float* qm = nullptr;      // [BH, n, Dk, Dv] (reverse only, optional)
  const float* last = nullptr;    // [BH, n] log decay over the whole chunk
  const float* init = nullptr;    // [BH, Dk, Dv] optional initial state
  float* states = nullptr;        // [BH, n, Dk, Dv] state before each step
  float* x = nullptr;             // [BH, n, C, Dv]
  float* final_state = nullptr;   // [BH, Dk, Dv] optional
  uint32_t* status = nullptr;     // bounded-wait error bits
  int BH = 0, n_chunks = 0, C = 64, Dk = 128, Dv = 128;
  // tensor-core path (Dk = 128): m1 / m2 as bf16 [BH, n, 64, 128] tiles in the XOR-swizzled layout of
  // gdn_pack_tiles (16-byte chunk cc of row r stored at chunk cc ^ (r & 7)); null selects the fp32 SIMT path
  const __nv_bfloat16* m1h = nullptr;
  const __nv_bfloat16* m2h = nullptr;
  // optional [n] flags (packed sequences): chunk i starts a new sequence, so the state before it is zero; forward
  // zeroes S before chunk i, reverse stops the gradient from flowing from chunk i into chunk i - 1
  const int* reset = nullptr;
};
int gdn_chunk_scan(const GdnScanArgs& a, bool reverse, cudaStream_t st);
// fp32 [tiles, 64, 128] -> bf16 swizzled tiles for the tensor-core scan
int gdn_pack_tiles(const float* src, __nv_bfloat16* dst, int64_t tiles, cudaStream_t st);

// gdn_chunk_train.cu: the per-chunk work of the chunked gated delta rule for training (Dk = Dv = 128, chunk 64),
// forward and backward, around the inter-chunk scan above. Grouped values: value head h reads key head h / (Hv/Hk).
struct GdnTrainArgs {
  const __nv_bfloat16* q = nullptr;  // [B, T, Hk, 128] (normalised, scaled)
  const __nv_bfloat16* k = nullptr;  // [B, T, Hk, 128] (normalised)
  const __nv_bfloat16* v = nullptr;  // [B, T, Hv, 128]
  const float* g = nullptr;          // [B, T, Hv] log decay
  const float* beta = nullptr;       // [B, T, Hv]
  int B = 0, T = 0, Hk = 0, Hv = 0, n = 0;  // n = ceil(T / 64) chunks
  // forward products (per sequence-head bh = b * Hv + h and chunk)
  __nv_bfloat16* w_tiles = nullptr;   // [BH, n, 64, 128] swizzled (scan operand)
  __nv_bfloat16* kd_tiles = nullptr;  // [BH, n, 64, 128] swizzled
  float* u = nullptr;                 // [BH, n, 64, 128]
  float* gc = nullptr;                // [BH, n, 64] within-chunk cumulative log decay
  float* last = nullptr;              // [BH, n]
  float* A = nullptr;                 // [BH, n, 64, 64] (I + beta k k^T decay, strictly lower)^-1
  const float* states = nullptr;      // [BH, n, 128, 128] state before each chunk (from the scan)
  const float* vnew = nullptr;        // [BH, n, 64, 128] u - w S (from the scan)
  __nv_bfloat16* o = nullptr;         // [B, T, Hv, 128]
  // backward
  const __nv_bfloat16* dout = nullptr;  // [B, T, Hv, 128]
  float* P = nullptr;                   // [BH, n, 64, 128] attn^T dO
  float* Qm = nullptr;                  // [BH, n, 128, 128] (q e^{gc})^T dO
  const float* dnext = nullptr;         // [BH, n, 128, 128] dL/dS after each chunk (reverse scan states)
  const float* du = nullptr;            // [BH, n, 64, 128] dL/du (reverse scan X)
  float* dw = nullptr;                  // [BH, n, 64, 128]
  float* dgc = nullptr;                 // [BH, n, 64] dL/dgc of the inter-chunk part
  float* dq = nullptr;                  // [B, T, Hv, 128] per value head
  float* dk = nullptr;                  // [B, T, Hv, 128] per value head (inter-chunk part, then final)
  float* dv = nullptr;                  // [B, T, Hv, 128]
  float* dg = nullptr;                  // [B, T, Hv]
  float* dbeta = nullptr;               // [B, T, Hv]
};
int gdn_train_fwd_prep(const GdnTrainArgs& a, cudaStream_t st);
int gdn_train_fwd_out(const GdnTrainArgs& a, cudaStream_t st);
int gdn_train_bwd_prep(const GdnTrainArgs& a, cudaStream_t st);
int gdn_train_bwd_inter(const GdnTrainArgs& a, cudaStream_t st);
int gdn_train_bwd_wy(const GdnTrainArgs& a, cudaStream_t st);

// train_fused.cu: fused forward / backward of the student's element-wise and row-wise ops (bf16 I/O, fp32 math)
// pos (optional, [B * T] int32): position of each token inside its packed sequence (taps before its start read 0)
int conv_silu_fwd(const void* x, int64_t ldx, const float* w, void* y, int B, int T, int Cc, const int* pos,
                  cudaStream_t st);
int conv_silu_bwd(const void* x, int64_t ldx, const float* w, const void* dy, void* dx, int B, int T, int Cc,
                  const int* pos, cudaStream_t st);
// row r of a strided view: (r / inner) * ld_outer + (r % inner) * ld_inner elements
struct RowMap {
  int64_t inner = 1, ld_outer = 0, ld_inner = 0;
};
// z null: y = x rstd (1 + w); z given: y = x rstd w silu(z) (then dz is written in the backward); H = 128 .. 2048
// (powers of two); x / z rows may be strided views, y / dy / dx / dz are contiguous
int rmsnorm_train_fwd(const void* x, RowMap mx, const void* z, RowMap mz, const float* w, float eps, void* y,
                      float* rstd, int64_t rows, int H, cudaStream_t st);
int rmsnorm_train_bwd(const void* x, RowMap mx, const void* z, RowMap mz, const float* w, const float* rstd,
                      const void* dy, void* dx, void* dz, int64_t rows, int H, cudaStream_t st);
int swiglu_train_fwd(const void* gu, void* h, int64_t rows, int I, cudaStream_t st);
int swiglu_train_bwd(const void* gu, const void* dh, void* dgu, int64_t rows, int I, cudaStream_t st);
int moe_combine_train_fwd(const void* y, const int64_t* inv, const float* w, int K, void* out, int64_t T, int H,
                          cudaStream_t st);
int moe_combine_train_bwd(const void* y, const int64_t* inv, const float* w, int K, const void* dout, void* dy,
                          float* dw, int64_t T, int H, cudaStream_t st);
int moe_dispatch_train_bwd(const void* g, const int64_t* inv, int K, void* dx, int64_t T, int H, cudaStream_t st);

// ep.cu: expert-parallel MoE exchange over peer memory (symmetric heap regions at equal offsets on every rank)
constexpr int EP_MAX_RANKS = 8;
constexpr int EP_DISPATCH = 0, EP_COMBINE = 1;
struct EpArgs {
  int world = 1, rank = 0;
  int T = 0, T_cap = 0, H = 0, k = 0;      // local tokens this step, slots per rank, hidden, experts per token
  uint8_t* peer[EP_MAX_RANKS] = {};        // heap base of every rank (own included)
  // region offsets (bytes) inside every heap
  size_t off_x = 0;      // e4m3 [world*T_cap, H]
  size_t off_s = 0;      // fp32 [world*T_cap] one scale per row
  size_t off_ids = 0;    // int32 [world*T_cap, k]
  size_t off_w = 0;      // fp32 [world*T_cap, k]
  size_t off_comb = 0;   // bf16 [T_cap*k, H] routed rows of this rank's tokens
  size_t off_flags = 0;  // uint64 [2 types][EP_MAX_RANKS sources]
  size_t off_rcnt = 0;   // int [world sources][E_local]: how many of each source's entries go to each local expert
  size_t off_rlist = 0;  // int [world sources][E_local][T_cap]: those entries (global entry = src*T_cap*k + t*k + j)
  int ld_s = 0;
  int E_local = 0;       // experts per rank (expert e lives on rank e / E_local)
  unsigned* done = nullptr;             // local [2] CTA-completion counters
  unsigned long long* sent = nullptr;   // local [2] exchanges published
  unsigned long long* expected = nullptr;  // local [2] exchanges consumed
  unsigned* wait_done = nullptr;        // local [2] CTA-completion counters of the kernels that consume an exchange
  // dispatch: this rank's per-expert entry lists from the router (cnt [E], list [E, T_cap], local entry indices)
  const int* lcnt = nullptr;
  const int* llist = nullptr;
  // optional wait accounting: block 0 of the w13 GEMM adds its dispatch wait (ns) to wait_ns[0], block 0 of the
  // combine its combine wait to wait_ns[1] (a per-layer slot of the caller's log)
  unsigned long long* wait_ns = nullptr;
};
int ep_dispatch(const EpArgs& a, const void* x, int ldx, const int* ids, const float* weights, cudaStream_t st);
int ep_wait(const EpArgs& a, int type, uint32_t* status, cudaStream_t st);
// e4m3 per-row quantisation of the entry rows x [rows, K] that this rank's routing lists name (h between the expert
// GEMMs under expert parallelism): one warp per list slot, empty slots exit at once
int quant_routed_rows(const void* x, int K, const int* cnt, const int* list, int srcs, int E, int cap, void* q,
                      float* scales, cudaStream_t st);

// hc.cu: hyper-connection residual stream [rows, G, H] (bf16): grouped norm, branch mix, gated write-back, and
// their dX-only backward; H in {256, 512, 1024, 2048, 2560}, G <= 8
// ---- batched bf16 transpose with an optional row -> column remap (train_kernels.cu)
int transpose_bf16(const void* src, int64_t R, int64_t C, int64_t lds, int64_t batch, int64_t src_batch,
                   const int64_t* dst, void* out, int64_t ldo, int64_t out_batch, cudaStream_t st);

// ---- LoRA adapter products (lora.cu): R in {8, 16, 32, 64}; the small operand is fp32 (split into bf16 hi + lo)
int lora_rows_times(const void* P, int64_t ldp, const float* W, int T, int K, int R, float* out, cudaStream_t st);
int lora_tgrad(const void* P, int64_t ldp, const float* Q, int T, int M, int R, int splits, float* part, float* out,
               cudaStream_t st);

// ---- per-layer n-gram embedding lookup (ple.cu)
constexpr int PLE_MAX_SHARDS = 8;
struct PleLookupArgs {
  const int32_t* ext;      // tokens with their history inline
  int64_t ext_len;
  const int64_t* pos;      // [rows] index of each row's token in ext
  const int64_t* seg;      // [rows] index in ext of each row's segment start
  int rows;
  int n, hpn, head_dim;    // n-gram size, heads per order, dims per head
  int32_t eos;
  const int64_t* mult;     // [n]
  const int64_t* mod;      // [(n-1) * hpn]
  const int64_t* off;      // [(n-1) * hpn]
  const int64_t* hot_idx;  // compact table: sorted kept buckets of every head (nullptr: full table)
  const int64_t* hot_base; // [(n-1) * hpn]
  const int32_t* hot_len;  // [(n-1) * hpn]
  const void* shards[PLE_MAX_SHARDS];        // table rows [rows_per_shard, head_dim] per shard
  const float* scale_shards[PLE_MAX_SHARDS]; // e4m3 tables: 128 x 128 block scales per shard
  int64_t rows_per_shard, table_rows;
  int scale_ld;            // scale columns (ceil(head_dim / 128))
  void* out;               // bf16 [rows, heads * head_dim]
  int64_t* ids_out;        // optional [rows, heads] table rows (-1: hot-table miss)
  uint32_t* status;
};
int ple_lookup(const PleLookupArgs& a, bool fp8, cudaStream_t st);

int hc_norm_fwd(const void* h, const float* w, void* zb, float* rstd, int64_t rows, int G, int H, float eps,
                cudaStream_t st);
int hc_norm_bwd(const void* h, const float* w, const float* rstd, const float* dzb, void* dh, int64_t rows, int G,
                int H, cudaStream_t st);
int hc_mix_fwd(const void* pre, const void* zb, void* x, int64_t rows, int G, int H, cudaStream_t st);
int hc_act_fwd(const void* du, int ld, int64_t rows, int R, int G, void* s, void* gate, cudaStream_t st);
int hc_mix_bwd(const void* pre, const void* zb, const void* dx, void* dpre, float* dzb, int64_t rows, int G, int H,
               cudaStream_t st);
int hc_inject_fwd(const void* h, const void* y, const void* gate, void* out, int64_t rows, int G, int H,
                  cudaStream_t st);
int hc_inject_bwd(const void* y, const void* gate, const void* dout, void* dy, float* dgate, int64_t rows, int G,
                  int H, cudaStream_t st);

// guard.cu: cross-rank agreement of small int64 packets over peer memory (device-side replica check)
struct GuardArgs {
  int world = 1, rank = 0, n_max = 0;
  uint8_t* peer[EP_MAX_RANKS] = {};
  size_t off_slots = 0;  // int64 [2 parities][EP_MAX_RANKS sources][n_max]
  size_t off_flags = 0;  // uint64 [EP_MAX_RANKS sources]
  unsigned long long* calls = nullptr;  // local: checks issued
  int* mismatches = nullptr;            // local: running count of differing elements
};
int guard_check(const GuardArgs& a, const int64_t* packet, int n, uint32_t* status, cudaStream_t st);

// zero_comm.cu: ZeRO-style optimizer step over peer memory (symmetric heap)
constexpr int ZERO_GRADS = 0, ZERO_NORM = 1, ZERO_PARAMS = 2;
struct ZeroArgs {
  int world = 1, rank = 0;
  uint8_t* peer[EP_MAX_RANKS] = {};
  size_t off_flags = 0;  // uint64 [3 types][EP_MAX_RANKS sources]
  size_t off_norm = 0;   // float [EP_MAX_RANKS] sums of squares by rank
  unsigned long long* sent = nullptr;      // local [3]
  unsigned long long* expected = nullptr;  // local [3]
  float* norm_out = nullptr;               // local scalar: the global gradient norm of the last step
};
int zero_signal(const ZeroArgs& a, int type, cudaStream_t st);
int zero_wait(const ZeroArgs& a, int type, uint32_t* status, cudaStream_t st);
int zero_rs(const ZeroArgs& a, size_t grad_off, size_t chunk, float scale, float* shard, float* partials, int blocks,
            cudaStream_t st);
int zero_norm_publish(const ZeroArgs& a, const float* partials, int n, cudaStream_t st);
int zero_adamw(const ZeroArgs& a, size_t param_off, size_t chunk, const float* g, void* m, void* v, size_t n_valid,
               float lr, float b1, float b2, float eps, float wd, int step, float max_norm, int blocks,
               cudaStream_t st);


// sampling.cu
int select_tokens(const void* logits, int ld, int rows, int V, int* out, float temperature, uint64_t seed,
                  const int* step, uint32_t* status, cudaStream_t st);
struct SpecArgs {
  const int* window = nullptr;   // [S, K+1] verify window tokens (anchor, drafts)
  const int* target = nullptr;   // [S, K+1] target choice after each window row
  const int* seq_slot = nullptr; // [S]
  const int* active = nullptr;   // [S] or null
  int* ctx_len = nullptr;        // [S] committed tokens (in/out)
  int* n_commit = nullptr;       // [slots] out
  int* out_tokens = nullptr;     // [S, K+1] emitted tokens (-1 padded)
  int* out_count = nullptr;      // [S]
  int* anchor = nullptr;         // [S] next window's first token
  int* last_row = nullptr;       // [S] row index (into the window rows) of the last committed token
  const int* step = nullptr;     // device step counter (bernoulli draws)
  unsigned long long* total_emitted = nullptr;
  int num_seqs = 0, k = 4, mode = 0;
  float accept_prob = 0.7f;
  uint64_t seed = 0;
};
int spec_accept(const SpecArgs& a, cudaStream_t st);
struct WindowArgs {
  const int* anchor = nullptr;      // [S]
  const int* drafts = nullptr;      // [S, drafts_ld] or null (rows after the anchor get fill_token)
  int drafts_ld = 0, fill_token = 0;
  const int* ctx_len = nullptr;     // [S]
  const int* block_table = nullptr; // [S, max_pages]
  int max_pages = 0;
  int* ids = nullptr;               // [S*W]
  int* positions = nullptr;         // [S*W]
  int* slots = nullptr;             // [S*W]
  int* attn_len = nullptr;          // [S]
  int* step = nullptr;              // optional counter bumped once per call
  int num_seqs = 0, width = 5, pos_offset = 0;
};
int build_window(const WindowArgs& a, cudaStream_t st);
int gather_rows(const void* src, const int* idx, void* out, int rows, int H, cudaStream_t st);

// train_kernels.cu
int int3_dequant(const void* codes, const float* scales, int E, int R, int K, void* out, cudaStream_t st);
int int3_scale_grad(const void* codes, const void* dW, int E, int R, int K, float* dS, cudaStream_t st);
int fp8_block_fakequant(const float* w, int N, int K, void* out, float* scale_inv, cudaStream_t st);
int topk_tail_kl(const float* z, int ldz, int rows, int V, const long long* ids, int k, const float* t_lp,
                 const float* t_tail, int reverse, float grad_scale, float* loss, void* dz, int ldd, cudaStream_t st);
int adamw(float* p, const float* g, void* m, void* v, void* w, size_t n, float lr, float b1, float b2, float eps,
          float wd, int step, cudaStream_t st);

}  // namespace afb
