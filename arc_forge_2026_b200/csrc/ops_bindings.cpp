// Bindings of the elementwise / routing / attention / GDN / sampling kernels.
#include "binding_utils.h"
#include "kernels.h"
#include "moe.h"

using namespace afb_bind;

namespace {

void rmsnorm_op(const at::Tensor& x, c10::optional<at::Tensor> residual, const at::Tensor& w, at::Tensor& y,
                double eps, bool zero_centered) {
  AFB_CHECK_CUDA(x);
  AFB_CHECK_DT(x, at::kBFloat16);
  AFB_CHECK_CONTIG(x);
  AFB_CHECK_CONTIG(y);
  const int H = x.size(-1), rows = x.numel() / H;
  check_rc(afb::rmsnorm(x.data_ptr(), optr<void>(residual), w.data_ptr(), y.data_ptr(), rows, H, (float)eps,
                        zero_centered, stream()),
           "rmsnorm");
}

// NVFP4 KV cache: the e2m1 pairs [pages, Hkv, 64, D/2] (uint8) and their e4m3 scales [pages, Hkv, 64, D/16] (uint8)
uint8_t* kv_scale_ptr(const c10::optional<at::Tensor>& scale, const at::Tensor& cache, int64_t D) {
  if (!scale.has_value()) return nullptr;
  AFB_CHECK_CONTIG(scale.value());
  AFB_CHECK_CONTIG(cache);
  TORCH_CHECK(cache.scalar_type() == at::kByte && scale->scalar_type() == at::kByte, "NVFP4 cache and scales: uint8");
  TORCH_CHECK(cache.dim() == 4 && cache.size(2) == 64 && cache.size(3) * 2 == D && scale->dim() == 4 &&
                  scale->size(0) == cache.size(0) && scale->size(1) == cache.size(1) && scale->size(2) == 64 &&
                  scale->size(3) * 16 == D,
              "NVFP4 cache must be [pages, Hkv, 64, D/2] with scales [pages, Hkv, 64, D/16]");
  return scale->data_ptr<uint8_t>();
}

void qk_norm_rope_store_op(const at::Tensor& qkv, int64_t Hq, int64_t Hkv, int64_t D, int64_t rot,
                           const at::Tensor& qw, const at::Tensor& kw, const at::Tensor& positions,
                           const at::Tensor& slots, const at::Tensor& cos_t, const at::Tensor& sin_t, double eps,
                           at::Tensor& q_out, at::Tensor& kcache, at::Tensor& vcache,
                           c10::optional<at::Tensor> kscale, c10::optional<at::Tensor> vscale) {
  AFB_CHECK_DT(positions, at::kInt);
  AFB_CHECK_DT(slots, at::kInt);
  AFB_CHECK_DT(cos_t, at::kFloat);
  const int T = qkv.size(0);
  TORCH_CHECK(qkv.size(1) >= Hq * 2 * D + 2 * Hkv * D, "qkv width (extra columns, e.g. the QSA indexer, follow)");
  TORCH_CHECK(qkv.stride(1) == 1, "qkv inner stride");
  const int page_size = kcache.size(2);
  check_rc(afb::qk_norm_rope_store(qkv.data_ptr(), qkv.stride(0), T, Hq, Hkv, D, rot, qw.data_ptr(), kw.data_ptr(),
                                   ptr<int>(positions), ptr<int>(slots), ptr<float>(cos_t), ptr<float>(sin_t),
                                   (float)eps, q_out.data_ptr(), kcache.data_ptr(), vcache.data_ptr(), page_size,
                                   stream(), kv_scale_ptr(kscale, kcache, D), kv_scale_ptr(vscale, vcache, D)),
           "qk_norm_rope_store");
}

// Optional per-expert entry lists: cnt int [E] (cleared by the launcher), list int [E, cap], cap >= tokens.
void router_topk_op(const at::Tensor& logits, int64_t E, int64_t k, bool renorm, at::Tensor& ids,
                    at::Tensor& weights, c10::optional<at::Tensor> cnt, c10::optional<at::Tensor> list) {
  AFB_CHECK_DT(logits, at::kFloat);
  AFB_CHECK_DT(ids, at::kInt);
  AFB_CHECK_DT(weights, at::kFloat);
  TORCH_CHECK(logits.stride(1) == 1, "router logits need unit inner stride");
  int cap = 0;
  if (cnt.has_value()) {
    TORCH_CHECK(list.has_value() && cnt->numel() >= E && list->dim() == 2 && list->size(0) >= E &&
                    list->is_contiguous(),
                "router lists: cnt [E], list [E, cap]");
    cap = list->size(1);
  }
  check_rc(afb::router_topk(ptr<float>(logits), logits.stride(0), logits.size(0), E, k, renorm, ptr<int>(ids),
                            ptr<float>(weights), stream(), optr<int>(cnt), optr<int>(list), cap),
           "router_topk");
}

void expert_sort_op(const at::Tensor& ids, int64_t E, c10::optional<at::Tensor> expert_map, at::Tensor& offsets,
                    at::Tensor& row_token, at::Tensor& row_entry, at::Tensor& entry_row, int64_t pad) {
  AFB_CHECK_DT(ids, at::kInt);
  AFB_CHECK_CONTIG(ids);
  const int k = ids.size(-1);
  TORCH_CHECK(row_token.numel() >= ids.numel() + (pad - 1) * E, "row_token capacity must cover the padding");
  check_rc(afb::expert_sort(ptr<int>(ids), ids.numel(), E, optr<int>(expert_map), ptr<int>(offsets),
                            ptr<int>(row_token), ptr<int>(row_entry), ptr<int>(entry_row), k, (int)pad, stream()),
           "expert_sort");
}

// per-row e4m3 (the INT3 experts' activation format): q [>= rows, K], scales fp32 [>= rows]
void quant_rows_e4m3_row_op(const at::Tensor& x, c10::optional<at::Tensor> row_token,
                            c10::optional<at::Tensor> nrows_dev, int64_t nrows, at::Tensor& q, at::Tensor& scales) {
  AFB_CHECK_DT(x, at::kBFloat16);
  AFB_CHECK_DT(scales, at::kFloat);
  TORCH_CHECK(x.stride(-1) == 1 && x.stride(0) % 8 == 0, "x rows must be contiguous and 16-byte aligned");
  const int K = x.size(1);
  TORCH_CHECK(q.size(1) == K && q.stride(0) == K && q.size(0) >= nrows && scales.size(0) >= nrows,
              "quant_rows_e4m3_row shapes");
  check_rc(afb::quant_rows_e4m3_row(x.data_ptr(), x.stride(0), optr<int>(row_token), optr<int>(nrows_dev), nrows, K,
                                    q.data_ptr(), ptr<float>(scales), stream()),
           "quant_rows_e4m3_row");
}

void quant_rows_e4m3_op(const at::Tensor& x, c10::optional<at::Tensor> row_token, c10::optional<at::Tensor> nrows_dev,
                        int64_t nrows, at::Tensor& q, at::Tensor& scales, bool group_major) {
  AFB_CHECK_DT(x, at::kBFloat16);
  TORCH_CHECK(x.stride(-1) == 1, "x inner stride");
  const int K = x.size(1);
  if (group_major) TORCH_CHECK(scales.size(0) == K / 128 && scales.size(1) >= nrows, "group-major scales shape");
  check_rc(afb::quant_rows_e4m3(x.data_ptr(), x.stride(0), optr<int>(row_token), optr<int>(nrows_dev), nrows, K,
                                q.data_ptr(), ptr<float>(scales), group_major ? (int)scales.stride(0) : 0, stream()),
           "quant_rows_e4m3");
}

// INT3 grouped expert GEMM. pair=True: w13 with SwiGLU + e4m3 requant (out_q, out_scales group-major);
// pair=False: w2 with the routing weight (out_bf16).
// Expert-parallel exchange context: the region layout of the symmetric heap and the local counters.
struct EpCtx {
  afb::EpArgs a;
  EpCtx(int64_t world, int64_t rank, int64_t T_cap, int64_t H, int64_t k, int64_t E_local, std::vector<int64_t> peers,
        std::vector<int64_t> offsets, int64_t ld_s, const at::Tensor& done, const at::Tensor& sent,
        const at::Tensor& expected, const at::Tensor& wait_done) {
    TORCH_CHECK(world >= 1 && world <= afb::EP_MAX_RANKS && (int64_t)peers.size() == world, "EpCtx: world/peers");
    TORCH_CHECK(offsets.size() == 8, "EpCtx: offsets = (x, s, ids, w, comb, flags, rcnt, rlist)");
    AFB_CHECK_DT(done, at::kInt);
    AFB_CHECK_DT(sent, at::kLong);
    AFB_CHECK_DT(expected, at::kLong);
    AFB_CHECK_DT(wait_done, at::kInt);
    TORCH_CHECK(done.numel() >= 2 && sent.numel() >= 2 && expected.numel() >= 2 && wait_done.numel() >= 2,
                "EpCtx: counters");
    a.world = (int)world;
    a.rank = (int)rank;
    a.T_cap = (int)T_cap;
    a.H = (int)H;
    a.k = (int)k;
    a.E_local = (int)E_local;
    for (int p = 0; p < world; ++p) a.peer[p] = reinterpret_cast<uint8_t*>((uintptr_t)peers[p]);
    a.off_x = offsets[0];
    a.off_s = offsets[1];
    a.off_ids = offsets[2];
    a.off_w = offsets[3];
    a.off_comb = offsets[4];
    a.off_flags = offsets[5];
    a.off_rcnt = offsets[6];
    a.off_rlist = offsets[7];
    a.ld_s = (int)ld_s;
    a.done = reinterpret_cast<unsigned*>(done.data_ptr());
    a.sent = reinterpret_cast<unsigned long long*>(sent.data_ptr());
    a.expected = reinterpret_cast<unsigned long long*>(expected.data_ptr());
    a.wait_done = reinterpret_cast<unsigned*>(wait_done.data_ptr());
  }
  // lcnt / llist: this rank's router lists (int [E], [E, T_cap]) of local entry indices
  void dispatch(const at::Tensor& x, int64_t T, const at::Tensor& ids, const at::Tensor& w, const at::Tensor& lcnt,
                const at::Tensor& llist) {
    AFB_CHECK_DT(x, at::kBFloat16);
    AFB_CHECK_DT(ids, at::kInt);
    AFB_CHECK_DT(w, at::kFloat);
    AFB_CHECK_DT(lcnt, at::kInt);
    AFB_CHECK_DT(llist, at::kInt);
    TORCH_CHECK(x.stride(1) == 1 && x.size(1) == a.H && ids.size(1) == a.k, "ep dispatch shapes");
    TORCH_CHECK(lcnt.numel() >= (int64_t)a.E_local * a.world && llist.dim() == 2 && llist.size(1) == a.T_cap &&
                    llist.is_contiguous(),
                "ep dispatch lists: cnt [E], list [E, T_cap]");
    if (slots > 0) {  // this layer's wait slot, used by the w13 GEMM and the combine that follow
      slot = (slot + 1) % slots;
      a.wait_ns = reinterpret_cast<unsigned long long*>(wait_log.data_ptr()) + 2 * slot;
    }
    afb::EpArgs b = a;
    b.T = (int)T;
    b.lcnt = ptr<int>(lcnt);
    b.llist = ptr<int>(llist);
    check_rc(afb::ep_dispatch(b, x.data_ptr(), x.stride(0), ptr<int>(ids), ptr<float>(w), stream()), "ep_dispatch");
  }
  void wait(int64_t type) { check_rc(afb::ep_wait(a, (int)type, status_ptr(current_device()), stream()), "ep_wait"); }
  // per-layer wait accounting: log int64 [slots, 2] (dispatch, combine ns, accumulated); begin_step() restarts the
  // slot counter, each dispatch() moves to the next slot (under CUDA-graph capture every layer keeps its own slot)
  at::Tensor wait_log;
  int64_t slots = 0, slot = -1;
  void set_wait_log(const at::Tensor& log) {
    AFB_CHECK_DT(log, at::kLong);
    AFB_CHECK_CONTIG(log);
    TORCH_CHECK(log.dim() == 2 && log.size(1) == 2, "wait log is int64 [slots, 2]");
    wait_log = log;
    slots = log.size(0);
    slot = -1;
    a.wait_ns = nullptr;
  }
  void begin_step() { slot = -1; }
  // per-row e4m3 of the entry rows h [world * T_cap * k, I] that this rank's lists name
  void quant_routed(const at::Tensor& h, at::Tensor& q, at::Tensor& scales) {
    AFB_CHECK_DT(h, at::kBFloat16);
    AFB_CHECK_DT(scales, at::kFloat);
    AFB_CHECK_CONTIG(h);
    TORCH_CHECK(q.sizes() == h.sizes() && q.is_contiguous() && scales.numel() >= h.size(0), "quant_routed shapes");
    const int* cnt = reinterpret_cast<const int*>(a.peer[a.rank] + a.off_rcnt);
    const int* list = reinterpret_cast<const int*>(a.peer[a.rank] + a.off_rlist);
    check_rc(afb::quant_routed_rows(h.data_ptr(), h.size(1), cnt, list, a.world, a.E_local, a.T_cap, q.data_ptr(),
                                    ptr<float>(scales), stream()),
             "quant_routed_rows");
  }
  // out[t] = resid[t] + sigmoid(gate) * shared[t] + the k routed rows of token t from the combine region; waits for
  // every rank's combine rows first (in the kernel) and counts the exchange consumed
  void combine(const at::Tensor& comb, c10::optional<at::Tensor> shared, c10::optional<at::Tensor> router_logits,
               int64_t sg_col, c10::optional<at::Tensor> resid, at::Tensor& out, int64_t T) {
    const int ld = router_logits.has_value() ? router_logits->stride(0) : 0;
    check_rc(afb::moe_combine(comb.data_ptr(), nullptr, a.k, optr<void>(shared), optr<float>(router_logits), ld,
                              sg_col, optr<void>(resid), out.data_ptr(), (int)T, a.H, stream(), &a,
                              status_ptr(current_device())),
             "moe_combine(ep)");
  }
  static int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
  }
};

// Routed-expert GEMM (INT3 tile layout, or block FP8 when codes is e4m3). route_cnt int [srcs, E] (or [E]),
// route_list int [srcs, E, cap] (or [E, cap]): the entries of each expert; an entry's activation row is
// entry / x_div. pair=True: w13 (INT3: bf16 h per entry in out_bf16; FP8: e4m3 h + group scales per entry);
// pair=False: w2 with the routing weight per entry (out_bf16 per entry, or the expert-parallel combine scatter).
// ep: the exchange context (w2: scatter + publish; w13 with ep_wait: wait for the dispatch in the prologue).
void moe_int3_gemm_op(const at::Tensor& codes, const at::Tensor& scales, const at::Tensor& route_cnt,
                      const at::Tensor& route_list, int64_t x_div, const at::Tensor& x_q, const at::Tensor& x_scales,
                      bool pair, c10::optional<at::Tensor> out_q, c10::optional<at::Tensor> out_scales,
                      c10::optional<at::Tensor> out_bf16, c10::optional<at::Tensor> route_w,
                      c10::optional<at::Tensor> dbg, const EpCtx* ep, bool ep_wait) {
  AFB_CHECK_DT(route_cnt, at::kInt);
  AFB_CHECK_DT(route_list, at::kInt);
  AFB_CHECK_CONTIG(codes);
  AFB_CHECK_CONTIG(scales);
  AFB_CHECK_CONTIG(x_q);
  AFB_CHECK_CONTIG(route_cnt);
  AFB_CHECK_CONTIG(route_list);
  afb::MoeGemmArgs a;
  if (codes.scalar_type() == at::kFloat8_e4m3fn) {  // block-FP8 experts: weights [E, rows, K], scales [E, rows/128, K/128]
    AFB_CHECK_DT(scales, at::kFloat);
    TORCH_CHECK(codes.dim() == 3 && codes.size(1) % 128 == 0 && codes.size(2) % 128 == 0, "fp8 experts [E, R, K]");
    TORCH_CHECK(scales.dim() == 3 && scales.size(0) == codes.size(0) && scales.size(1) == codes.size(1) / 128 &&
                    scales.size(2) == codes.size(2) / 128,
                "fp8 block scales [E, R/128, K/128]");
    a.fp8_w = reinterpret_cast<const uint8_t*>(codes.data_ptr());
    a.fp8_scales = ptr<float>(scales);
    a.num_experts = codes.size(0);
    a.rows = codes.size(1);
    a.K = codes.size(2);
  } else {
    AFB_CHECK_DT(codes, at::kInt);
    AFB_CHECK_DT(scales, at::kBFloat16);
    TORCH_CHECK(codes.dim() == 5 && codes.size(3) == 128 && codes.size(4) == 12, "codes must be tile layout");
    a.codes = ptr<int32_t>(codes);
    a.scales = scales.data_ptr();
    a.num_experts = codes.size(0);
    a.rows = codes.size(1) * 128;
    a.K = codes.size(2) * 128;
  }
  const int E = a.num_experts;
  const int srcs = route_cnt.dim() == 2 ? route_cnt.size(0) : 1;
  TORCH_CHECK(route_cnt.numel() == (int64_t)srcs * E && route_list.dim() == route_cnt.dim() + 1 &&
                  route_list.numel() % ((int64_t)srcs * E) == 0,
              "route_cnt [srcs, E] and route_list [srcs, E, cap]");
  a.route_cnt = ptr<int>(route_cnt);
  a.route_list = ptr<int>(route_list);
  a.route_srcs = srcs;
  a.route_cap = route_list.size(-1);
  a.x_div = (int)x_div;
  TORCH_CHECK(x_q.size(1) == a.K && x_q.stride(0) == a.K, "x_q [rows, K]");
  a.x_q = x_q.data_ptr();
  a.x_scales = ptr<float>(x_scales);
  a.x_rows = x_q.size(0);
  if (a.fp8_w) {  // 1 x 128 activation scales, group-major
    a.ld_xs = x_scales.stride(0);
    TORCH_CHECK(x_scales.dim() == 2 && x_scales.size(0) == a.K / 128 && x_scales.size(1) >= a.x_rows,
                "fp8 experts: x_scales must be group-major [K/128, >= rows]");
  } else {  // one activation scale per row
    TORCH_CHECK(x_scales.dim() == 1 && x_scales.size(0) >= a.x_rows, "int3 experts: x_scales [rows]");
  }
  if (pair) {
    if (a.fp8_w) {  // e4m3 h with a scale per (entry, 128 columns), the next FP8 GEMM's input
      TORCH_CHECK(out_q.has_value() && out_scales.has_value(), "fp8 pair needs out_q and out_scales");
      a.out_q = optr<uint8_t>(out_q);
      a.out_scales = optr<float>(out_scales);
      a.ld_os = out_scales->stride(0);
      a.out_ld = out_q->stride(0);
      TORCH_CHECK(out_q->size(1) == a.rows / 2, "out_q width must be I");
    } else {  // bf16 h (quantised per row again before w2)
      TORCH_CHECK(out_bf16.has_value(), "int3 pair needs out_bf16 (h)");
      AFB_CHECK_DT((*out_bf16), at::kBFloat16);
      TORCH_CHECK(out_bf16->size(1) == a.rows / 2 && out_bf16->stride(1) == 1, "h must be bf16 [entries, I]");
      a.out_bf16 = out_bf16->data_ptr();
      a.out_ld = out_bf16->stride(0);
    }
    if (ep_wait) {
      TORCH_CHECK(ep, "ep_wait needs the exchange context");
      a.ep_wait_flags = reinterpret_cast<const uint64_t*>(ep->a.peer[ep->a.rank] + ep->a.off_flags);  // dispatch
      a.ep_wait_ns = ep->a.wait_ns;
      a.ep_expected = ep->a.expected;
      a.ep_wait_done = ep->a.wait_done;
      TORCH_CHECK(srcs == ep->a.world, "expert-parallel lists have one row per rank");
    }
  } else {
    TORCH_CHECK(out_bf16.has_value(), "w2 needs out_bf16");
    a.out_bf16 = out_bf16->data_ptr();
    a.out_ld = out_bf16->stride(0);
    a.route_w = optr<float>(route_w);
    if (ep) {
      TORCH_CHECK(a.route_w && a.out_ld == ep->a.H, "expert-parallel w2 needs route_w");
      a.ep_world = ep->a.world;
      a.ep_rank = ep->a.rank;
      a.ep_entries_per_rank = ep->a.T_cap * ep->a.k;
      for (int p = 0; p < ep->a.world; ++p) a.ep_peer[p] = ep->a.peer[p];
      a.ep_off_comb = ep->a.off_comb;
      a.ep_off_flags = ep->a.off_flags;
      a.ep_done = ep->a.done + afb::EP_COMBINE;
      a.ep_sent = ep->a.sent + afb::EP_COMBINE;
    }
  }
  a.dbg = optr<long long>(dbg);
  check_rc(afb::moe_int3_gemm(a, pair, num_sms(), status_ptr(codes.get_device()), stream()),
           a.fp8_w ? "moe_fp8_gemm" : "moe_int3_gemm");
}

void moe_combine_op(const at::Tensor& y, c10::optional<at::Tensor> entry_row, int64_t k, c10::optional<at::Tensor> shared,
                    c10::optional<at::Tensor> router_logits, int64_t sg_col, c10::optional<at::Tensor> resid,
                    at::Tensor& out) {
  const int T = out.size(0), H = out.size(1);
  const int ld = router_logits.has_value() ? router_logits->stride(0) : 0;
  check_rc(afb::moe_combine(y.data_ptr(), optr<int>(entry_row), k, optr<void>(shared), optr<float>(router_logits), ld,
                            sg_col, optr<void>(resid), out.data_ptr(), T, H, stream()),
           "moe_combine");
}

// Paged decode/verify attention. gate (optional): a strided view whose element (tok, head, d) sits at
// gate.data_ptr() + tok * gate_ld + head * gate_head_stride + d.
void paged_attention_op(const at::Tensor& q, const at::Tensor& kcache, const at::Tensor& vcache,
                        const at::Tensor& block_table, const at::Tensor& seq_lens, int64_t q_per_seq, double scale,
                        at::Tensor& out, c10::optional<at::Tensor> gate, int64_t gate_ld, int64_t gate_head_stride,
                        int64_t splits, int64_t pages_per_split, int64_t window, c10::optional<at::Tensor> bt_row,
                        c10::optional<at::Tensor> sp_count, c10::optional<at::Tensor> sp_lpage,
                        c10::optional<at::Tensor> sp_mask, c10::optional<at::Tensor> kscale,
                        c10::optional<at::Tensor> vscale, int64_t impl, int64_t sp_block,
                        c10::optional<at::Tensor> sp_slot) {
  AFB_CHECK_DT(q, at::kBFloat16);
  AFB_CHECK_CONTIG(q);
  AFB_CHECK_CONTIG(kcache);
  AFB_CHECK_CONTIG(out);
  AFB_CHECK_DT(block_table, at::kInt);
  AFB_CHECK_DT(seq_lens, at::kInt);
  TORCH_CHECK(kcache.dim() == 4 && kcache.size(2) == 64, "kv cache must be [pages, Hkv, 64, D]");
  afb::AttnArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.kcache = kcache.data_ptr();
  a.vcache = vcache.data_ptr();
  a.num_pages = kcache.size(0);
  a.Hkv = kcache.size(1);
  a.D = kcache.size(3) * (kscale.has_value() ? 2 : 1);
  a.Hq = q.size(1);
  TORCH_CHECK(q.size(2) == a.D, "q head dim must match the cache");
  if (kscale.has_value()) {  // NVFP4 cache
    TORCH_CHECK(vscale.has_value(), "NVFP4 attention needs both scale tensors");
    a.kscale = kv_scale_ptr(kscale, kcache, a.D);
    a.vscale = kv_scale_ptr(vscale, vcache, a.D);
  }
  a.block_table = ptr<int>(block_table);
  a.max_pages = block_table.size(1);
  a.seq_lens = ptr<int>(seq_lens);
  a.num_seqs = seq_lens.size(0);
  a.q_per_seq = q_per_seq;
  a.num_tokens = q.size(0);
  TORCH_CHECK(a.num_tokens == a.num_seqs * q_per_seq, "q rows must be num_seqs * q_per_seq");
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.pages_per_split = (int)pages_per_split;
  a.window = (int)window;
  a.bt_row = optr<int>(bt_row);
  a.impl = (int)impl;
  if (sp_count.has_value()) {  // QSA sparse mode: block_table rows are page unions
    TORCH_CHECK(sp_lpage.has_value() && sp_mask.has_value(), "sparse attention needs sp_count, sp_lpage and sp_mask");
    AFB_CHECK_DT(sp_count.value(), at::kInt);
    AFB_CHECK_DT(sp_lpage.value(), at::kInt);
    AFB_CHECK_DT(sp_mask.value(), at::kByte);
    TORCH_CHECK(sp_block >= 1 && 64 % sp_block == 0, "sp_block must divide the 64-token page");
    TORCH_CHECK(sp_lpage->dim() == 2 && sp_lpage->size(0) == a.num_seqs && sp_mask->sizes() == sp_lpage->sizes(),
                "sp_lpage / sp_mask must be [num_seqs, union capacity]");
    TORCH_CHECK(sp_block < 64 || sp_lpage->sizes() == block_table.sizes(),
                "page-block sparse mode: the block table rows are the page unions (same shape as sp_lpage)");
    TORCH_CHECK(sp_block == 64 || (impl == 0 && !kscale.has_value()),
                "sub-page QSA blocks run on the tcgen05 kernel only (bf16 cache)");
    TORCH_CHECK(sp_block < 64 || !bt_row.has_value(), "page-block sparse mode: the union rows are per sequence");
    TORCH_CHECK(q_per_seq <= 8 && window == 0, "sparse mode: at most 8 verify rows, no window");
    AFB_CHECK_CONTIG(sp_lpage.value());
    AFB_CHECK_CONTIG(sp_mask.value());
    a.sp_block = (int)sp_block;
    a.sp_ld = sp_lpage->size(1);
    if (sp_block < 64) {
      TORCH_CHECK(sp_slot.has_value() && sp_slot->sizes() == sp_lpage->sizes(),
                  "sub-page mode needs sp_slot (the union's first-token KV slots), shaped as sp_lpage");
      AFB_CHECK_DT(sp_slot.value(), at::kInt);
      AFB_CHECK_CONTIG(sp_slot.value());
      a.sp_slot = ptr<int>(sp_slot.value());
    }
    a.sp_count = ptr<int>(sp_count.value());
    a.sp_lpage = ptr<int>(sp_lpage.value());
    a.sp_mask = ptr<uint8_t>(sp_mask.value());
  }
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (gate.has_value()) {
    a.gate = reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr());
    a.gate_ld = gate_ld;
    a.gate_head_stride = gate_head_stride;
  }
  at::Tensor po, pl;
  if (splits > 1) {
    po = torch::empty({splits, a.num_tokens, a.Hq, a.D}, q.options().dtype(at::kFloat));
    pl = torch::empty({splits, a.num_tokens, a.Hq}, q.options().dtype(at::kFloat));
    a.part_o = ptr<float>(po);
    a.part_lse = ptr<float>(pl);
  }
  check_rc(afb::paged_attention(a, (int)splits, status_ptr(q.get_device()), stream()), "paged_attention");
}

// Training attention (attention_train.cu). tiles: int32 [n, 2] (segment, first position) on the device.
static afb::AttnTrainArgs train_attn_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                          const at::Tensor& cu, const at::Tensor& tiles, double scale) {
  for (const at::Tensor* t : {&q, &k, &v}) {
    AFB_CHECK_DT((*t), at::kBFloat16);
    AFB_CHECK_CONTIG((*t));
    TORCH_CHECK(t->dim() == 3, "q / k / v are [T, heads, D]");
  }
  AFB_CHECK_DT(cu, at::kInt);
  AFB_CHECK_DT(tiles, at::kInt);
  AFB_CHECK_CONTIG(tiles);
  TORCH_CHECK(tiles.dim() == 2 && tiles.size(1) == 2, "tiles is [n, 2]");
  TORCH_CHECK(k.sizes() == v.sizes() && k.size(0) == q.size(0) && k.size(2) == q.size(2), "k / v shapes");
  afb::AttnTrainArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.cu = ptr<int>(cu);
  a.tiles = reinterpret_cast<const int2*>(tiles.data_ptr());
  a.ntiles = tiles.size(0);
  a.T = q.size(0);
  a.Hq = q.size(1);
  a.Hkv = k.size(1);
  a.D = q.size(2);
  a.scale = (float)scale;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  return a;
}

static void train_attn_qsa(afb::AttnTrainArgs& a, const c10::optional<at::Tensor>& blkmap, int64_t qsa_block) {
  if (!blkmap.has_value()) return;
  AFB_CHECK_DT(blkmap.value(), at::kInt);
  AFB_CHECK_CONTIG(blkmap.value());
  TORCH_CHECK(blkmap->dim() == 2 && blkmap->size(0) == a.T, "blkmap is int32 [T, words]");
  TORCH_CHECK(qsa_block >= 2 && 64 % qsa_block == 0, "qsa_block must divide 64");
  a.blkmap = reinterpret_cast<const uint32_t*>(blkmap->data_ptr());
  a.blk_words = blkmap->size(1);
  a.qsa_block = (int)qsa_block;
}

void attn_train_fwd_op(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& cu,
                       const at::Tensor& tiles, double scale, at::Tensor& out, at::Tensor& lse,
                       c10::optional<at::Tensor> blkmap, int64_t qsa_block, bool causal) {
  afb::AttnTrainArgs a = train_attn_args(q, k, v, cu, tiles, scale);
  train_attn_qsa(a, blkmap, qsa_block);
  a.causal = causal ? 1 : 0;
  AFB_CHECK_CONTIG(out);
  TORCH_CHECK(out.sizes() == q.sizes() && out.scalar_type() == at::kBFloat16, "out is bf16 like q");
  AFB_CHECK_DT(lse, at::kFloat);
  TORCH_CHECK(lse.numel() == (int64_t)a.Hq * a.T, "lse is [Hq, T]");
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse = ptr<float>(lse);
  check_rc(afb::attn_train_fwd(a, status_ptr(q.get_device()), stream()), "attn_train_fwd");
}

// ------------------------------------------------------------------------------------------ vision tower
void vit_patch_pos_op(const at::Tensor& acc, const at::Tensor& bias, const at::Tensor& table, const at::Tensor& idx,
                      const at::Tensor& wts, at::Tensor& h) {
  AFB_CHECK_DT(acc, at::kFloat);
  AFB_CHECK_CONTIG(acc);
  AFB_CHECK_DT(idx, at::kInt);
  AFB_CHECK_CONTIG(idx);
  AFB_CHECK_DT(wts, at::kBFloat16);
  AFB_CHECK_DT(table, at::kBFloat16);
  AFB_CHECK_DT(h, at::kBFloat16);
  AFB_CHECK_CONTIG(h);
  const int P = acc.size(0), C = acc.size(1);
  TORCH_CHECK(h.size(0) == P && h.size(1) == C && idx.numel() == 4 * P && wts.numel() == 4 * P &&
                  table.size(1) == C && bias.numel() == C,
              "vit_patch_pos shapes");
  check_rc(afb::vit_patch_pos(ptr<float>(acc), bias.data_ptr(), table.data_ptr(), ptr<int>(idx), wts.data_ptr(),
                              h.data_ptr(), P, C, stream()),
           "vit_patch_pos");
}

void vit_qkv_rope_op(const at::Tensor& qkv, const at::Tensor& cosv, const at::Tensor& sinv, int64_t H, int64_t Dh,
                     at::Tensor& q, at::Tensor& k, at::Tensor& v) {
  AFB_CHECK_DT(qkv, at::kBFloat16);
  AFB_CHECK_CONTIG(qkv);
  AFB_CHECK_DT(cosv, at::kFloat);
  AFB_CHECK_DT(sinv, at::kFloat);
  AFB_CHECK_CONTIG(cosv);
  AFB_CHECK_CONTIG(sinv);
  for (const at::Tensor* t : {&q, &k, &v}) {
    AFB_CHECK_DT((*t), at::kBFloat16);
    AFB_CHECK_CONTIG((*t));
  }
  const int P = qkv.size(0), Dp = q.size(2);
  TORCH_CHECK(qkv.size(1) == 3 * H * Dh && q.size(0) == P && q.size(1) == H && k.sizes() == q.sizes() &&
                  v.sizes() == q.sizes() && cosv.numel() == (int64_t)P * (Dh / 2) && sinv.numel() == cosv.numel(),
              "vit_qkv_rope shapes");
  check_rc(afb::vit_qkv_rope(qkv.data_ptr(), ptr<float>(cosv), ptr<float>(sinv), P, (int)H, (int)Dh, Dp,
                             q.data_ptr(), k.data_ptr(), v.data_ptr(), stream()),
           "vit_qkv_rope");
}

void vit_layernorm_op(const at::Tensor& x, const at::Tensor& w, const at::Tensor& b, double eps, at::Tensor& y) {
  AFB_CHECK_DT(x, at::kBFloat16);
  AFB_CHECK_CONTIG(x);
  AFB_CHECK_DT(y, at::kBFloat16);
  AFB_CHECK_CONTIG(y);
  AFB_CHECK_DT(w, at::kBFloat16);
  AFB_CHECK_DT(b, at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && y.sizes() == x.sizes() && w.numel() == x.size(1) && b.numel() == x.size(1),
              "vit_layernorm shapes");
  check_rc(afb::vit_layernorm(x.data_ptr(), w.data_ptr(), b.data_ptr(), (float)eps, y.data_ptr(), x.size(0), x.size(1),
                              stream()),
           "vit_layernorm");
}

void attn_train_bwd_op(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& cu,
                       const at::Tensor& tiles, const at::Tensor& kv_tiles, double scale, const at::Tensor& out,
                       const at::Tensor& lse, const at::Tensor& dout, at::Tensor& delta, at::Tensor& dq,
                       at::Tensor& dk, at::Tensor& dv, at::Tensor& dk_part, at::Tensor& dv_part,
                       c10::optional<at::Tensor> blkmap, int64_t qsa_block) {
  afb::AttnTrainArgs a = train_attn_args(q, k, v, cu, tiles, scale);
  train_attn_qsa(a, blkmap, qsa_block);
  AFB_CHECK_CONTIG(dout);
  AFB_CHECK_CONTIG(out);
  TORCH_CHECK(dout.sizes() == q.sizes() && out.sizes() == q.sizes(), "out / dout shapes");
  TORCH_CHECK(dq.sizes() == q.sizes() && dk.sizes() == k.sizes() && dv.sizes() == v.sizes(), "gradient shapes");
  AFB_CHECK_CONTIG(dq);
  AFB_CHECK_CONTIG(dk);
  AFB_CHECK_CONTIG(dv);
  AFB_CHECK_DT(kv_tiles, at::kInt);
  AFB_CHECK_CONTIG(kv_tiles);
  TORCH_CHECK(kv_tiles.dim() == 2 && kv_tiles.size(1) == 2, "kv_tiles is [n, 2]");
  TORCH_CHECK(delta.numel() == (int64_t)a.Hq * a.T && lse.numel() == delta.numel(), "lse / delta are [Hq, T]");
  a.out = reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(out.data_ptr()));
  a.lse = const_cast<float*>(ptr<float>(lse));
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.delta = ptr<float>(delta);
  a.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  a.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  a.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  AFB_CHECK_DT(dk_part, at::kFloat);
  AFB_CHECK_DT(dv_part, at::kFloat);
  TORCH_CHECK(dk_part.numel() == q.numel() && dv_part.numel() == q.numel(), "dk_part / dv_part are fp32 [T, Hq, D]");
  a.dk_part = ptr<float>(dk_part);
  a.dv_part = ptr<float>(dv_part);
  check_rc(afb::attn_train_bwd(a, reinterpret_cast<const int2*>(kv_tiles.data_ptr()), (int)kv_tiles.size(0),
                               status_ptr(q.get_device()), stream()),
           "attn_train_bwd");
}

// QSA (see qsa.cu). proj: projection rows whose columns [idx_off, idx_off + (Hi + 1) * 128) hold the index
// query heads then the raw index key.
void qsa_prep_op(const at::Tensor& proj, int64_t idx_off, const at::Tensor& positions, const at::Tensor& slots,
                 const at::Tensor& q_norm, const at::Tensor& cos_t, const at::Tensor& sin_t, double eps, int64_t Hi,
                 int64_t rot, at::Tensor& idx_q, at::Tensor& idx_raw) {
  AFB_CHECK_DT(proj, at::kBFloat16);
  AFB_CHECK_DT(idx_q, at::kBFloat16);
  AFB_CHECK_DT(idx_raw, at::kBFloat16);
  TORCH_CHECK(proj.stride(1) == 1 && idx_off % 4 == 0 && proj.size(1) >= idx_off + (Hi + 1) * 128, "qsa proj");
  TORCH_CHECK(idx_q.numel() >= proj.size(0) * Hi * 128 && idx_raw.size(-1) == 128, "qsa outputs");
  afb::QsaArgs a;
  a.Hi = (int)Hi;
  a.rot = (int)rot;
  a.eps = (float)eps;
  a.q_norm = reinterpret_cast<const __nv_bfloat16*>(q_norm.data_ptr());
  a.cos_t = ptr<float>(cos_t);
  a.sin_t = ptr<float>(sin_t);
  a.idx_q = reinterpret_cast<__nv_bfloat16*>(idx_q.data_ptr());
  a.idx_raw = reinterpret_cast<__nv_bfloat16*>(idx_raw.data_ptr());
  const auto* base = reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()) + idx_off;
  check_rc(afb::qsa_prep(a, base, proj.stride(0), proj.size(0), ptr<int>(positions), ptr<int>(slots), stream()),
           "qsa_prep");
}

void qsa_select_op(const at::Tensor& idx_q, const at::Tensor& idx_key, const at::Tensor& idx_raw,
                   const at::Tensor& k_norm, const at::Tensor& block_table, const at::Tensor& fin,
                   const at::Tensor& seq_lens, int64_t W, int64_t K, int64_t Hi, int64_t block, at::Tensor& sel,
                   const at::Tensor& cos_t, const at::Tensor& sin_t, int64_t rot, double eps, at::Tensor& u_page,
                   at::Tensor& u_lpage, at::Tensor& u_mask, at::Tensor& u_count, c10::optional<at::Tensor> bt_row,
                   c10::optional<at::Tensor> scores) {
  AFB_CHECK_DT(idx_q, at::kBFloat16);
  AFB_CHECK_DT(idx_key, at::kBFloat16);
  AFB_CHECK_DT(idx_raw, at::kBFloat16);
  AFB_CHECK_DT(block_table, at::kInt);
  AFB_CHECK_DT(u_mask, at::kByte);
  AFB_CHECK_DT(sel, at::kInt);
  AFB_CHECK_DT(cos_t, at::kFloat);
  const int S = seq_lens.size(0);
  TORCH_CHECK(idx_q.numel() >= (int64_t)S * W * Hi * 128, "idx_q rows");
  TORCH_CHECK(u_page.size(0) >= S && u_page.sizes() == u_lpage.sizes() && u_page.sizes() == u_mask.sizes(),
              "union buffers");
  const int max_blocks = block_table.size(1) * (64 / (int)block);
  TORCH_CHECK(sel.numel() >= (int64_t)S * (max_blocks + 1), "sel scratch [S, max_blocks + 1]");
  TORCH_CHECK(idx_key.size(0) >= (int64_t)(bt_row.has_value() ? block_table.size(0) : S) * max_blocks,
              "pooled key rows [sessions * max_blocks]");
  if (bt_row.has_value()) {
    AFB_CHECK_DT(bt_row.value(), at::kInt);
    TORCH_CHECK(bt_row->numel() == S, "bt_row: one session per row set");
  }
  afb::QsaArgs a;
  a.Hi = (int)Hi;
  a.idx_q = reinterpret_cast<__nv_bfloat16*>(idx_q.data_ptr());
  a.idx_key = reinterpret_cast<const __nv_bfloat16*>(idx_key.data_ptr());
  a.idx_raw = reinterpret_cast<__nv_bfloat16*>(idx_raw.data_ptr());
  a.cos_t = ptr<float>(cos_t);
  a.sin_t = ptr<float>(sin_t);
  a.rot = (int)rot;
  a.eps = (float)eps;
  afb::QsaSelectArgs sa;
  sa.block_table = ptr<int>(block_table);
  sa.max_pages = block_table.size(1);
  sa.block = (int)block;
  sa.max_blocks = max_blocks;
  sa.fin = ptr<int>(fin);
  sa.seq_lens = ptr<int>(seq_lens);
  sa.W = (int)W;
  sa.K = (int)K;
  sa.k_norm = reinterpret_cast<const __nv_bfloat16*>(k_norm.data_ptr());
  sa.sel = reinterpret_cast<uint32_t*>(sel.data_ptr());
  sa.u_page = ptr<int>(u_page);
  sa.u_lpage = ptr<int>(u_lpage);
  sa.u_mask = ptr<uint8_t>(u_mask);
  sa.u_count = ptr<int>(u_count);
  sa.ucap = u_page.size(1);
  sa.bt_row = optr<int>(bt_row);
  if (scores.has_value()) {  // tensor-core scores of the committed blocks
    AFB_CHECK_DT(scores.value(), at::kFloat);
    TORCH_CHECK(scores->numel() >= (int64_t)S * W * max_blocks, "scores scratch [S * W * max_blocks]");
    AFB_CHECK_CONTIG(idx_q);
    AFB_CHECK_CONTIG(idx_key);
    sa.scores = ptr<float>(scores.value());
    sa.scores_ld = max_blocks;
    sa.key_rows = idx_key.size(0);
    sa.q_rows = idx_q.size(0) * Hi;
  }
  check_rc(afb::qsa_select(a, sa, S, status_ptr(idx_q.get_device()), stream()), "qsa_select");
}

void qsa_finalize_op(const std::vector<at::Tensor>& idx_raw, const std::vector<at::Tensor>& idx_key,
                     const std::vector<at::Tensor>& k_norm, const at::Tensor& block_table, at::Tensor& fin,
                     const at::Tensor& ctx, const at::Tensor& cos_t, const at::Tensor& sin_t, int64_t rot, double eps,
                     int64_t block) {
  const int L = idx_raw.size();
  TORCH_CHECK(L >= 1 && L <= afb::QSA_MAX_LAYERS && (int)idx_key.size() == L && (int)k_norm.size() == L,
              "qsa_finalize: one raw cache, key cache and norm per layer");
  afb::QsaFinalizeArgs f;
  for (int l = 0; l < L; ++l) {
    f.idx_raw[l] = reinterpret_cast<const __nv_bfloat16*>(idx_raw[l].data_ptr());
    f.idx_key[l] = reinterpret_cast<__nv_bfloat16*>(idx_key[l].data_ptr());
    f.k_norm[l] = reinterpret_cast<const __nv_bfloat16*>(k_norm[l].data_ptr());
  }
  f.block_table = ptr<int>(block_table);
  f.max_pages = block_table.size(1);
  f.block = (int)block;
  f.max_blocks = f.max_pages * (64 / (int)block);
  for (int l = 0; l < L; ++l)
    TORCH_CHECK(idx_key[l].size(0) >= (int64_t)fin.size(0) * f.max_blocks, "pooled key rows [S * max_blocks]");
  f.fin = ptr<int>(fin);
  f.ctx = ptr<int>(ctx);
  f.cos_t = ptr<float>(cos_t);
  f.sin_t = ptr<float>(sin_t);
  f.rot = (int)rot;
  f.eps = (float)eps;
  check_rc(afb::qsa_finalize(f, fin.size(0), L, stream()), "qsa_finalize");
}

// ZeRO step over peer memory (see zero_comm.cu)
// cross-rank agreement check (guard.cu)
struct GuardCtx {
  afb::GuardArgs a;
  GuardCtx(int64_t world, int64_t rank, std::vector<int64_t> peers, int64_t off_slots, int64_t off_flags, int64_t n_max,
           const at::Tensor& calls, const at::Tensor& mismatches) {
    TORCH_CHECK(world >= 1 && world <= afb::EP_MAX_RANKS && (int64_t)peers.size() == world, "GuardCtx: world");
    AFB_CHECK_DT(calls, at::kLong);
    AFB_CHECK_DT(mismatches, at::kInt);
    a.world = (int)world;
    a.rank = (int)rank;
    a.n_max = (int)n_max;
    for (int p = 0; p < world; ++p) a.peer[p] = reinterpret_cast<uint8_t*>((uintptr_t)peers[p]);
    a.off_slots = off_slots;
    a.off_flags = off_flags;
    a.calls = reinterpret_cast<unsigned long long*>(calls.data_ptr());
    a.mismatches = ptr<int>(mismatches);
  }
  void check(const at::Tensor& packet) {
    AFB_CHECK_DT(packet, at::kLong);
    AFB_CHECK_CONTIG(packet);
    int d = 0;
    cudaGetDevice(&d);
    check_rc(afb::guard_check(a, ptr<int64_t>(packet), packet.numel(), status_ptr(d), stream()), "guard_check");
  }
};

struct ZeroCtx {
  afb::ZeroArgs a;
  ZeroCtx(int64_t world, int64_t rank, std::vector<int64_t> peers, int64_t off_flags, int64_t off_norm,
          const at::Tensor& sent, const at::Tensor& expected, const at::Tensor& norm_out) {
    TORCH_CHECK(world >= 1 && world <= afb::EP_MAX_RANKS && (int64_t)peers.size() == world, "ZeroCtx: world");
    AFB_CHECK_DT(sent, at::kLong);
    AFB_CHECK_DT(expected, at::kLong);
    AFB_CHECK_DT(norm_out, at::kFloat);
    a.world = (int)world;
    a.rank = (int)rank;
    for (int p = 0; p < world; ++p) a.peer[p] = reinterpret_cast<uint8_t*>((uintptr_t)peers[p]);
    a.off_flags = off_flags;
    a.off_norm = off_norm;
    a.sent = reinterpret_cast<unsigned long long*>(sent.data_ptr());
    a.expected = reinterpret_cast<unsigned long long*>(expected.data_ptr());
    a.norm_out = ptr<float>(norm_out);
  }
  void signal(int64_t type) { check_rc(afb::zero_signal(a, (int)type, stream()), "zero_signal"); }
  void wait(int64_t type) {
    int d = 0;
    cudaGetDevice(&d);
    check_rc(afb::zero_wait(a, (int)type, status_ptr(d), stream()), "zero_wait");
  }
  void rs(int64_t grad_off, int64_t chunk, double scale, at::Tensor& shard, at::Tensor& partials) {
    AFB_CHECK_DT(shard, at::kFloat);
    AFB_CHECK_DT(partials, at::kFloat);
    TORCH_CHECK(shard.numel() >= chunk, "rs shard");
    check_rc(afb::zero_rs(a, grad_off, chunk, (float)scale, ptr<float>(shard), ptr<float>(partials), partials.numel(),
                          stream()),
             "zero_rs");
  }
  void norm_publish(const at::Tensor& partials) {
    check_rc(afb::zero_norm_publish(a, ptr<float>(partials), partials.numel(), stream()), "zero_norm_publish");
  }
  void adamw(int64_t param_off, int64_t chunk, const at::Tensor& g, at::Tensor& m, at::Tensor& v, int64_t n_valid,
             double lr, double b1, double b2, double eps, double wd, int64_t step, double max_norm, int64_t blocks) {
    AFB_CHECK_DT(m, at::kBFloat16);
    AFB_CHECK_DT(v, at::kBFloat16);
    check_rc(afb::zero_adamw(a, param_off, chunk, ptr<float>(g), m.data_ptr(), v.data_ptr(), n_valid, (float)lr,
                             (float)b1, (float)b2, (float)eps, (float)wd, (int)step, (float)max_norm, (int)blocks,
                             stream()),
             "zero_adamw");
  }
};

// HiSparse (see hisparse.cu): the host pools, GPU pools and residency tables of every QSA layer.
struct HsCtx {
  afb::HsArgs a;
  afb::HsLayers L;
  int layers = 0;
  // per layer: (gpu_k, gpu_v, host_k, host_v, host_sk, host_sv, res, slot_page, stamp, raw) as raw addresses (0 = none)
  HsCtx(int64_t S, int64_t max_pages, int64_t C, int64_t R, int64_t Hkv, int64_t D, bool fp8, const at::Tensor& cycle,
        const std::vector<std::vector<int64_t>>& ptrs) {
    TORCH_CHECK(ptrs.size() >= 1 && ptrs.size() <= afb::QSA_MAX_LAYERS, "HsCtx: 1..64 layers");
    AFB_CHECK_DT(cycle, at::kInt);
    a.S = (int)S;
    a.max_pages = (int)max_pages;
    a.C = (int)C;
    a.R = (int)R;
    a.Hkv = (int)Hkv;
    a.D = (int)D;
    a.fp8 = fp8 ? 1 : 0;
    a.cycle = ptr<int>(cycle);
    layers = (int)ptrs.size();
    for (int l = 0; l < layers; ++l) {
      TORCH_CHECK(ptrs[l].size() == 10, "HsCtx: 10 addresses per layer");
      auto u8 = [&](int i) { return reinterpret_cast<uint8_t*>((uintptr_t)ptrs[l][i]); };
      L.l[l].gpu_k = u8(0);
      L.l[l].gpu_v = u8(1);
      L.l[l].host_k = u8(2);
      L.l[l].host_v = u8(3);
      L.l[l].host_sk = reinterpret_cast<float*>(u8(4));
      L.l[l].host_sv = reinterpret_cast<float*>(u8(5));
      L.l[l].res = reinterpret_cast<int*>(u8(6));
      L.l[l].slot_page = reinterpret_cast<int*>(u8(7));
      L.l[l].stamp = reinterpret_cast<int*>(u8(8));
      L.l[l].raw = reinterpret_cast<__nv_bfloat16*>(u8(9));
    }
  }
  void cycle_start(at::Tensor& block_table, const at::Tensor& ctx, int64_t W) {
    check_rc(afb::hs_cycle_start(a, ptr<int>(block_table), ptr<int>(ctx), (int)W, stream()), "hs_cycle_start");
  }
  void writeback(const at::Tensor& block_table, const at::Tensor& fin, const at::Tensor& ctx) {
    check_rc(afb::hs_writeback(a, L, layers, ptr<int>(block_table), ptr<int>(fin), ptr<int>(ctx), stream()),
             "hs_writeback");
  }
  void after_prefill(const at::Tensor& block_table, int64_t s, int64_t p0, int64_t p1, int64_t p2) {
    check_rc(afb::hs_after_prefill(a, L, layers, ptr<int>(block_table), (int)s, (int)p0, (int)p1, (int)p2, stream()),
             "hs_after_prefill");
  }
  void fetch(int64_t layer, at::Tensor& u_page, const at::Tensor& u_lpage, const at::Tensor& u_count,
             const at::Tensor& fin) {
    TORCH_CHECK(layer >= 0 && layer < layers, "hs fetch: layer");
    check_rc(afb::hs_fetch(a, L.l[layer], ptr<int>(u_page), ptr<int>(u_lpage), ptr<int>(u_count), u_page.size(1),
                           ptr<int>(fin), status_ptr(u_page.get_device()), stream()),
             "hs_fetch");
  }
};

// GDN decode/verify (see gdn.cu). pend: (pend_in, pend_qk, pend_v, pend_gb) with a leading parity dim of 2.
void gdn_decode_op(const at::Tensor& mixed, int64_t z_off, int64_t ba_off, const at::Tensor& conv_w,
                   at::Tensor& conv_state, at::Tensor& ssm_state, at::Tensor& pend_in, at::Tensor& pend_qk,
                   at::Tensor& pend_v, at::Tensor& pend_gb, const at::Tensor& n_commit, const at::Tensor& seq_slot,
                   const at::Tensor& A_log, const at::Tensor& dt_bias, const at::Tensor& norm_w, at::Tensor& out,
                   int64_t q_per_seq, int64_t Hk, int64_t Dk, int64_t Hv, int64_t Dv, bool commit_current,
                   int64_t parity, double eps, c10::optional<at::Tensor> dbg) {
  AFB_CHECK_DT(mixed, at::kBFloat16);
  AFB_CHECK_DT(ssm_state, at::kFloat);
  AFB_CHECK_DT(conv_w, at::kFloat);
  AFB_CHECK_DT(seq_slot, at::kInt);
  AFB_CHECK_DT(n_commit, at::kInt);
  TORCH_CHECK(mixed.stride(1) == 1, "mixed inner stride");
  afb::GdnArgs a;
  a.mixed = reinterpret_cast<const __nv_bfloat16*>(mixed.data_ptr());
  a.mixed_ld = mixed.stride(0);
  a.z_off = z_off;
  a.ba_off = ba_off;
  a.conv_w = ptr<float>(conv_w);
  a.conv_state = reinterpret_cast<__nv_bfloat16*>(conv_state.data_ptr());
  a.ssm_state = ptr<float>(ssm_state);
  a.pend_in = reinterpret_cast<__nv_bfloat16*>(pend_in.data_ptr());
  a.pend_qk = reinterpret_cast<__nv_bfloat16*>(pend_qk.data_ptr());
  a.pend_v = reinterpret_cast<__nv_bfloat16*>(pend_v.data_ptr());
  a.pend_gb = ptr<float>(pend_gb);
  a.n_commit = ptr<int>(n_commit);
  a.seq_slot = ptr<int>(seq_slot);
  a.A_log = ptr<float>(A_log);
  a.dt_bias = ptr<float>(dt_bias);
  a.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w.data_ptr());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.num_seqs = seq_slot.size(0);
  a.q_per_seq = q_per_seq;
  a.pend_slots = pend_in.size(1);
  a.max_q = pend_in.size(2);
  a.num_slots = ssm_state.size(0);
  a.conv_dim = conv_w.size(0);
  a.Hk = Hk;
  a.Hv = Hv;
  a.Dk = Dk;
  a.Dv = Dv;
  a.commit_current = commit_current;
  a.eps = (float)eps;
  a.dbg = optr<long long>(dbg);
  TORCH_CHECK(mixed.size(0) == a.num_seqs * q_per_seq, "mixed rows must be num_seqs * q_per_seq");
  TORCH_CHECK(a.conv_dim == 2 * Hk * Dk + Hv * Dv, "conv_dim");
  TORCH_CHECK(pend_in.size(0) == 2 && pend_in.size(3) == a.conv_dim, "pend_in shape");
  TORCH_CHECK(!commit_current || a.pend_slots >= a.num_seqs, "prefill scratch needs one pending slot per sequence");
  check_rc(afb::gdn_decode(a, (int)parity, num_sms(), status_ptr(mixed.get_device()), stream()), "gdn_decode");
}

void gdn_chunk_scan_op(const at::Tensor& m1, const at::Tensor& m2, const at::Tensor& y,
                       const c10::optional<at::Tensor>& qm, const at::Tensor& last, const c10::optional<at::Tensor>& init,
                       at::Tensor& states, at::Tensor& x, c10::optional<at::Tensor> final_state, bool reverse,
                       bool precise, const c10::optional<at::Tensor>& reset) {
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&m1, &m2, &y, &last, &states, &x}) {
    AFB_CHECK_CUDA(*t);
    AFB_CHECK_DT(*t, at::kFloat);
    AFB_CHECK_CONTIG(*t);
  }
  TORCH_CHECK(m1.dim() == 4 && m2.sizes() == m1.sizes() && y.dim() == 4, "m1/m2 [BH, n, C, Dk], y [BH, n, C, Dv]");
  afb::GdnScanArgs a;
  a.BH = m1.size(0);
  a.n_chunks = m1.size(1);
  a.C = m1.size(2);
  a.Dk = m1.size(3);
  a.Dv = y.size(3);
  TORCH_CHECK(y.size(0) == a.BH && y.size(1) == a.n_chunks && y.size(2) == a.C, "y shape");
  TORCH_CHECK(last.numel() == (int64_t)a.BH * a.n_chunks, "last shape");
  TORCH_CHECK(states.numel() == (int64_t)a.BH * a.n_chunks * a.Dk * a.Dv && x.sizes() == y.sizes(), "outputs");
  for (const auto* o : std::initializer_list<const c10::optional<at::Tensor>*>{&qm, &init})
    if (o->has_value()) {
      AFB_CHECK_DT(o->value(), at::kFloat);
      AFB_CHECK_CONTIG(o->value());
    }
  if (qm) TORCH_CHECK(qm->numel() == states.numel(), "qm shape");
  if (init) TORCH_CHECK(init->numel() == (int64_t)a.BH * a.Dk * a.Dv, "init shape");
  if (final_state) {
    AFB_CHECK_CONTIG(final_state.value());
    TORCH_CHECK(final_state->numel() == (int64_t)a.BH * a.Dk * a.Dv, "final shape");
  }
  a.m1 = ptr<float>(m1);
  a.m2 = ptr<float>(m2);
  a.y = ptr<float>(y);
  a.qm = optr<float>(qm);
  a.last = ptr<float>(last);
  a.init = optr<float>(init);
  a.states = ptr<float>(states);
  a.x = ptr<float>(x);
  a.final_state = optr<float>(final_state);
  a.status = status_ptr(m1.get_device());
  if (reset) {
    AFB_CHECK_DT(reset.value(), at::kInt);
    TORCH_CHECK(reset->numel() == a.n_chunks, "reset: one flag per chunk");
    a.reset = ptr<int>(reset.value());
  }
  at::Tensor m1h, m2h;
  if (!precise && a.Dk == 128 && a.C == 64 && a.Dv % 32 == 0) {  // tensor-core path: bf16 swizzled M1 / M2 tiles
    const int64_t tiles = (int64_t)a.BH * a.n_chunks;
    m1h = at::empty({tiles, 64, 128}, m1.options().dtype(at::kBFloat16));
    m2h = at::empty_like(m1h);
    check_rc(afb::gdn_pack_tiles(a.m1, ptr<__nv_bfloat16>(m1h), tiles, stream()), "gdn_pack_tiles");
    check_rc(afb::gdn_pack_tiles(a.m2, ptr<__nv_bfloat16>(m2h), tiles, stream()), "gdn_pack_tiles");
    a.m1h = ptr<__nv_bfloat16>(m1h);
    a.m2h = ptr<__nv_bfloat16>(m2h);
  }
  check_rc(afb::gdn_chunk_scan(a, reverse, stream()), "gdn_chunk_scan");
}

// chunked-GDN training stages (gdn_chunk_train.cu). `t` holds, in order (None where a stage does not use it):
// q, k, v, g, beta, w_tiles, kd_tiles, u, gc, last, A, states, vnew, o, dout, P, Qm, dnext, du, dw, dgc, dq, dk, dv,
// dg, dbeta
void gdn_train_op(int64_t stage, const std::vector<c10::optional<at::Tensor>>& t, int64_t B, int64_t T, int64_t Hk,
                  int64_t Hv) {
  TORCH_CHECK(t.size() == 26, "gdn_train: 26 tensor slots");
  for (const auto& x : t)
    if (x.has_value()) {
      AFB_CHECK_CUDA(x.value());
      AFB_CHECK_CONTIG(x.value());
    }
  auto bf = [&](int i) -> __nv_bfloat16* {
    if (!t[i].has_value()) return nullptr;
    TORCH_CHECK(t[i]->scalar_type() == at::kBFloat16, "gdn_train: slot ", i, " must be bf16");
    return ptr<__nv_bfloat16>(t[i].value());
  };
  auto f32 = [&](int i) -> float* {
    if (!t[i].has_value()) return nullptr;
    TORCH_CHECK(t[i]->scalar_type() == at::kFloat, "gdn_train: slot ", i, " must be fp32");
    return ptr<float>(t[i].value());
  };
  afb::GdnTrainArgs a;
  a.q = bf(0);
  a.k = bf(1);
  a.v = bf(2);
  a.g = f32(3);
  a.beta = f32(4);
  a.w_tiles = bf(5);
  a.kd_tiles = bf(6);
  a.u = f32(7);
  a.gc = f32(8);
  a.last = f32(9);
  a.A = f32(10);
  a.states = f32(11);
  a.vnew = f32(12);
  a.o = bf(13);
  a.dout = bf(14);
  a.P = f32(15);
  a.Qm = f32(16);
  a.dnext = f32(17);
  a.du = f32(18);
  a.dw = f32(19);
  a.dgc = f32(20);
  a.dq = f32(21);
  a.dk = f32(22);
  a.dv = f32(23);
  a.dg = f32(24);
  a.dbeta = f32(25);
  a.B = (int)B;
  a.T = (int)T;
  a.Hk = (int)Hk;
  a.Hv = (int)Hv;
  a.n = (int)((T + 63) / 64);
  TORCH_CHECK(Hk >= 1 && Hv % Hk == 0, "gdn_train: Hv must be a multiple of Hk");
  // every slot a stage reads or writes must be present
  static const std::vector<std::vector<int>> need = {
      {1, 2, 3, 4, 5, 6, 7, 8, 9, 10},          // fwd_prep
      {0, 1, 8, 11, 12, 13},                    // fwd_out
      {0, 1, 8, 14, 15, 16},                    // bwd_prep
      {0, 1, 8, 11, 12, 14, 17, 18, 19, 20, 21, 22},  // bwd_inter
      {1, 2, 4, 8, 10, 18, 19, 20, 22, 23, 24, 25}};  // bwd_wy
  TORCH_CHECK(stage >= 0 && stage < 5, "gdn_train: stage 0..4");
  for (int i : need[stage]) TORCH_CHECK(t[i].has_value(), "gdn_train stage ", stage, ": slot ", i, " missing");
  int rc = 0;
  switch (stage) {
    case 0: rc = afb::gdn_train_fwd_prep(a, stream()); break;
    case 1: rc = afb::gdn_train_fwd_out(a, stream()); break;
    case 2: rc = afb::gdn_train_bwd_prep(a, stream()); break;
    case 3: rc = afb::gdn_train_bwd_inter(a, stream()); break;
    default: rc = afb::gdn_train_bwd_wy(a, stream()); break;
  }
  check_rc(rc, "gdn_train");
}

// the tensor-core scan on pre-swizzled bf16 tiles (written by the gdn_train forward prep)
void gdn_chunk_scan_tiles_op(const at::Tensor& m1h, const at::Tensor& m2h, const at::Tensor& y,
                             const c10::optional<at::Tensor>& qm, const at::Tensor& last,
                             const c10::optional<at::Tensor>& init, at::Tensor& states, at::Tensor& x,
                             c10::optional<at::Tensor> final_state, bool reverse,
                             const c10::optional<at::Tensor>& reset) {
  AFB_CHECK_DT(m1h, at::kBFloat16);
  AFB_CHECK_DT(m2h, at::kBFloat16);
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&y, &last, &states, &x}) {
    AFB_CHECK_CUDA(*t);
    AFB_CHECK_DT(*t, at::kFloat);
    AFB_CHECK_CONTIG(*t);
  }
  TORCH_CHECK(y.dim() == 4 && y.size(2) == 64 && y.size(3) % 32 == 0, "y [BH, n, 64, Dv]");
  afb::GdnScanArgs a;
  a.BH = y.size(0);
  a.n_chunks = y.size(1);
  a.C = 64;
  a.Dk = 128;
  a.Dv = y.size(3);
  TORCH_CHECK(m1h.numel() == (int64_t)a.BH * a.n_chunks * 64 * 128 && m2h.numel() == m1h.numel(), "tile shapes");
  TORCH_CHECK(last.numel() == (int64_t)a.BH * a.n_chunks, "last shape");
  TORCH_CHECK(states.numel() == (int64_t)a.BH * a.n_chunks * 128 * a.Dv && x.sizes() == y.sizes(), "outputs");
  if (qm) TORCH_CHECK(qm->numel() == states.numel() && qm->scalar_type() == at::kFloat, "qm");
  if (init) TORCH_CHECK(init->numel() == (int64_t)a.BH * 128 * a.Dv && init->scalar_type() == at::kFloat, "init");
  if (final_state) TORCH_CHECK(final_state->numel() == (int64_t)a.BH * 128 * a.Dv, "final shape");
  a.m1h = ptr<__nv_bfloat16>(m1h);
  a.m2h = ptr<__nv_bfloat16>(m2h);
  a.y = ptr<float>(y);
  a.qm = optr<float>(qm);
  a.last = ptr<float>(last);
  a.init = optr<float>(init);
  a.states = ptr<float>(states);
  a.x = ptr<float>(x);
  a.final_state = optr<float>(final_state);
  a.status = status_ptr(y.get_device());
  if (reset) {
    AFB_CHECK_DT(reset.value(), at::kInt);
    TORCH_CHECK(reset->numel() == a.n_chunks, "reset: one flag per chunk");
    a.reset = ptr<int>(reset.value());
  }
  check_rc(afb::gdn_chunk_scan(a, reverse, stream()), "gdn_chunk_scan_tiles");
}

// ---- fused training ops (train_fused.cu); row strides of the (possibly strided) inputs are taken from the tensors
static void check_rows(const at::Tensor& t, const char* what) {
  AFB_CHECK_CUDA(t);
  AFB_CHECK_DT(t, at::kBFloat16);
  TORCH_CHECK(t.stride(-1) == 1 && t.size(-1) % 4 == 0, what, ": inner stride must be 1");
}
// rows of a view [outer dims..., inner, H]: the outer dims must collapse to one stride
static afb::RowMap row_map(const at::Tensor& t, const char* what) {
  check_rows(t, what);
  afb::RowMap m;
  const int d = t.dim();
  TORCH_CHECK(d >= 2, what, ": at least 2 dims");
  m.inner = t.size(d - 2);
  m.ld_inner = t.stride(d - 2);
  m.ld_outer = d >= 3 ? t.stride(d - 3) : m.inner * m.ld_inner;
  for (int i = 0; i + 3 < d; ++i)
    TORCH_CHECK(t.stride(i) == t.stride(i + 1) * t.size(i + 1), what, ": outer dims must collapse");
  TORCH_CHECK(m.ld_inner % 4 == 0 && m.ld_outer % 4 == 0, what, ": row strides must keep 8-byte alignment");
  return m;
}

void conv_silu_op(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, c10::optional<at::Tensor> dy,
                  c10::optional<at::Tensor> dx, c10::optional<at::Tensor> pos) {
  check_rows(x, "conv_silu x");
  TORCH_CHECK(x.dim() == 3 && x.stride(0) == x.size(1) * x.stride(1), "x [B, T, C] with evenly strided rows");
  AFB_CHECK_DT(w, at::kFloat);
  AFB_CHECK_CONTIG(w);
  TORCH_CHECK(w.size(0) == x.size(2) && w.size(1) == 4, "w [C, 4]");
  const int B = x.size(0), T = x.size(1), Cc = x.size(2);
  const int* pp = nullptr;
  if (pos) {
    AFB_CHECK_DT(pos.value(), at::kInt);
    AFB_CHECK_CONTIG(pos.value());
    TORCH_CHECK(pos->numel() == (int64_t)B * T, "pos: one position per token");
    pp = ptr<int>(pos.value());
  }
  if (dy) {
    AFB_CHECK_CONTIG(dy.value());
    AFB_CHECK_CONTIG(dx.value());
    check_rc(afb::conv_silu_bwd(x.data_ptr(), x.stride(1), ptr<float>(w), dy->data_ptr(), dx->data_ptr(), B, T, Cc,
                                pp, stream()),
             "conv_silu_bwd");
  } else {
    AFB_CHECK_CONTIG(y);
    check_rc(afb::conv_silu_fwd(x.data_ptr(), x.stride(1), ptr<float>(w), y.data_ptr(), B, T, Cc, pp, stream()),
             "conv_silu_fwd");
  }
}

void rmsnorm_train_op(const at::Tensor& x, c10::optional<at::Tensor> z, const at::Tensor& w, double eps,
                      at::Tensor& y, at::Tensor& rstd, c10::optional<at::Tensor> dy, c10::optional<at::Tensor> dx,
                      c10::optional<at::Tensor> dz) {
  const afb::RowMap mx = row_map(x, "rmsnorm x");
  afb::RowMap mz;
  if (z) {
    mz = row_map(z.value(), "rmsnorm z");
    TORCH_CHECK(z->sizes() == x.sizes(), "rmsnorm: z shape");
  }
  AFB_CHECK_DT(w, at::kFloat);
  AFB_CHECK_CONTIG(w);
  AFB_CHECK_DT(rstd, at::kFloat);
  const int H = x.size(-1);
  const int64_t rows = x.numel() / H;
  TORCH_CHECK(w.numel() == H && rstd.numel() == rows, "rmsnorm shapes");
  const void* zp = z ? z->data_ptr() : nullptr;
  if (dy) {
    AFB_CHECK_CONTIG(dy.value());
    AFB_CHECK_CONTIG(dx.value());
    if (z) AFB_CHECK_CONTIG(dz.value());
    check_rc(afb::rmsnorm_train_bwd(x.data_ptr(), mx, zp, mz, ptr<float>(w), ptr<float>(rstd), dy->data_ptr(),
                                    dx->data_ptr(), dz ? dz->data_ptr() : nullptr, rows, H, stream()),
             "rmsnorm_train_bwd");
  } else {
    AFB_CHECK_CONTIG(y);
    check_rc(afb::rmsnorm_train_fwd(x.data_ptr(), mx, zp, mz, ptr<float>(w), (float)eps, y.data_ptr(),
                                    ptr<float>(rstd), rows, H, stream()),
             "rmsnorm_train_fwd");
  }
}

void swiglu_train_op(const at::Tensor& gu, at::Tensor& out, c10::optional<at::Tensor> dh) {
  AFB_CHECK_DT(gu, at::kBFloat16);
  AFB_CHECK_CONTIG(gu);
  AFB_CHECK_CONTIG(out);
  const int I = gu.size(-1) / 2;
  const int64_t rows = gu.numel() / (2 * I);
  if (dh) {
    AFB_CHECK_CONTIG(dh.value());
    check_rc(afb::swiglu_train_bwd(gu.data_ptr(), dh->data_ptr(), out.data_ptr(), rows, I, stream()), "swiglu_bwd");
  } else {
    check_rc(afb::swiglu_train_fwd(gu.data_ptr(), out.data_ptr(), rows, I, stream()), "swiglu_fwd");
  }
}

void moe_combine_train_op(const at::Tensor& y, const at::Tensor& inv, const at::Tensor& w, at::Tensor& out,
                          c10::optional<at::Tensor> dout, c10::optional<at::Tensor> dy, c10::optional<at::Tensor> dw) {
  AFB_CHECK_DT(y, at::kBFloat16);
  AFB_CHECK_CONTIG(y);
  AFB_CHECK_DT(inv, at::kLong);
  AFB_CHECK_CONTIG(inv);
  AFB_CHECK_DT(w, at::kFloat);
  AFB_CHECK_CONTIG(w);
  const int64_t T = w.size(0);
  const int K = w.size(1), H = y.size(-1);
  TORCH_CHECK(inv.numel() == T * K && y.size(0) == T * K, "combine shapes");
  if (dout) {
    check_rc(afb::moe_combine_train_bwd(y.data_ptr(), ptr<int64_t>(inv), ptr<float>(w), K, dout->data_ptr(),
                                        dy->data_ptr(), ptr<float>(dw.value()), T, H, stream()),
             "moe_combine_bwd");
  } else {
    check_rc(afb::moe_combine_train_fwd(y.data_ptr(), ptr<int64_t>(inv), ptr<float>(w), K, out.data_ptr(), T, H,
                                        stream()),
             "moe_combine_fwd");
  }
}

void moe_dispatch_bwd_op(const at::Tensor& g, const at::Tensor& inv, int64_t K, at::Tensor& dx) {
  AFB_CHECK_DT(g, at::kBFloat16);
  AFB_CHECK_CONTIG(g);
  AFB_CHECK_CONTIG(dx);
  AFB_CHECK_DT(inv, at::kLong);
  const int64_t T = dx.size(0);
  TORCH_CHECK(inv.numel() == T * K && g.size(0) == T * K, "dispatch shapes");
  check_rc(afb::moe_dispatch_train_bwd(g.data_ptr(), ptr<int64_t>(inv), (int)K, dx.data_ptr(), T, dx.size(-1),
                                       stream()),
           "moe_dispatch_bwd");
}

// ---- hyper-connections (hc.cu); the branch stream is [rows, G, H] contiguous bf16
static void hc_shape(const at::Tensor& h, int64_t& rows, int& G, int& H) {
  AFB_CHECK_DT(h, at::kBFloat16);
  AFB_CHECK_CONTIG(h);
  TORCH_CHECK(h.dim() >= 2, "hc: [..., G, H]");
  H = h.size(-1);
  G = h.size(-2);
  rows = h.numel() / ((int64_t)G * H);
}
// out[b, c, dst[r]] = src[b, r, c]: src [B, R, C] (or [R, C]) bf16 rows of unit inner stride, out [B, C, ldo]
void transpose_bf16_op(const at::Tensor& src, c10::optional<at::Tensor> dst, at::Tensor& out) {
  AFB_CHECK_DT(src, at::kBFloat16);
  AFB_CHECK_DT(out, at::kBFloat16);
  AFB_CHECK_CONTIG(out);
  TORCH_CHECK(src.stride(-1) == 1 && (src.dim() == 2 || src.dim() == 3) && out.dim() == src.dim(), "transpose shapes");
  const int64_t B = src.dim() == 3 ? src.size(0) : 1;
  const int64_t R = src.size(-2), C = src.size(-1);
  TORCH_CHECK(out.size(-2) == C && (src.dim() == 2 || out.size(0) == B), "transpose: out rows must be src columns");
  const int64_t ldo = out.size(-1);
  if (dst) {
    AFB_CHECK_DT(dst.value(), at::kLong);
    TORCH_CHECK(dst->numel() == R, "transpose: dst has one column per source row");
  } else {
    TORCH_CHECK(ldo >= R, "transpose: out too narrow");
  }
  check_rc(afb::transpose_bf16(src.data_ptr(), R, C, src.stride(-2), B, src.dim() == 3 ? src.stride(0) : 0,
                               dst ? dst->data_ptr<int64_t>() : nullptr, out.data_ptr(), ldo, C * ldo, stream()),
           "transpose_bf16");
}

// LoRA: rows_times(P [T, K] bf16, W [R, K] fp32) -> [T, R] fp32; tgrad(P [T, M] bf16, Q [T, R] fp32) -> [M, R] fp32
at::Tensor lora_rows_times_op(const at::Tensor& P, const at::Tensor& W) {
  AFB_CHECK_DT(P, at::kBFloat16);
  AFB_CHECK_DT(W, at::kFloat);
  AFB_CHECK_CONTIG(W);
  TORCH_CHECK(P.dim() == 2 && P.stride(1) == 1 && W.dim() == 2 && W.size(1) == P.size(1), "lora_rows_times shapes");
  const int T = P.size(0), K = P.size(1), R = W.size(0);
  at::Tensor out = torch::empty({T, R}, W.options());
  check_rc(afb::lora_rows_times(P.data_ptr(), P.stride(0), ptr<float>(W), T, K, R, ptr<float>(out), stream()),
           "lora_rows_times");
  return out;
}
at::Tensor lora_tgrad_op(const at::Tensor& P, const at::Tensor& Q, int64_t splits) {
  AFB_CHECK_DT(P, at::kBFloat16);
  AFB_CHECK_DT(Q, at::kFloat);
  AFB_CHECK_CONTIG(Q);
  TORCH_CHECK(P.dim() == 2 && P.stride(1) == 1 && Q.dim() == 2 && Q.size(0) == P.size(0), "lora_tgrad shapes");
  const int T = P.size(0), M = P.size(1), R = Q.size(1);
  at::Tensor part = torch::empty({splits, M, R}, Q.options());
  at::Tensor out = torch::empty({M, R}, Q.options());
  check_rc(afb::lora_tgrad(P.data_ptr(), P.stride(0), ptr<float>(Q), T, M, R, (int)splits, ptr<float>(part),
                           ptr<float>(out), stream()),
           "lora_tgrad");
  return out;
}

// ``shard_ptrs`` / ``scale_ptrs``: device addresses of the table shards (this process's tensors or peers' buffers
// mapped from a symmetric heap); the Python wrapper checks their shapes.
void ple_lookup_op(const at::Tensor& ext, const at::Tensor& pos, const at::Tensor& seg, int64_t n, int64_t hpn,
                   int64_t eos, const at::Tensor& mult, const at::Tensor& mod, const at::Tensor& off,
                   std::vector<int64_t> shard_ptrs, std::vector<int64_t> scale_ptrs, bool fp8, int64_t head_dim,
                   int64_t rows_per_shard, int64_t table_rows, at::Tensor& out, c10::optional<at::Tensor> ids_out,
                   c10::optional<at::Tensor> hot_idx, c10::optional<at::Tensor> hot_base,
                   c10::optional<at::Tensor> hot_len) {
  AFB_CHECK_DT(ext, at::kInt);
  for (const at::Tensor* t : {&pos, &seg, &mult, &mod, &off}) AFB_CHECK_DT((*t), at::kLong);
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&ext, &pos, &seg, &mult, &mod, &off, &out})
    AFB_CHECK_CONTIG((*t));
  AFB_CHECK_DT(out, at::kBFloat16);
  TORCH_CHECK(!shard_ptrs.empty() && (int)shard_ptrs.size() <= afb::PLE_MAX_SHARDS, "ple_lookup: 1..8 shards");
  TORCH_CHECK(!fp8 || scale_ptrs.size() == shard_ptrs.size(), "ple_lookup: one scale pointer per e4m3 shard");
  const int heads = (int)((n - 1) * hpn);
  TORCH_CHECK(mult.numel() == n && mod.numel() == heads && off.numel() == heads, "ple_lookup: hash shapes");
  TORCH_CHECK(pos.numel() == seg.numel() && out.numel() == pos.numel() * heads * head_dim, "ple_lookup: out shape");
  TORCH_CHECK((int64_t)shard_ptrs.size() * rows_per_shard >= table_rows, "ple_lookup: shards cover the table");
  afb::PleLookupArgs a{};
  a.ext = ext.data_ptr<int32_t>();
  a.ext_len = ext.numel();
  a.pos = pos.data_ptr<int64_t>();
  a.seg = seg.data_ptr<int64_t>();
  a.rows = (int)pos.numel();
  a.n = (int)n;
  a.hpn = (int)hpn;
  a.head_dim = (int)head_dim;
  a.eos = (int32_t)eos;
  a.mult = mult.data_ptr<int64_t>();
  a.mod = mod.data_ptr<int64_t>();
  a.off = off.data_ptr<int64_t>();
  for (size_t i = 0; i < shard_ptrs.size(); ++i) {
    a.shards[i] = reinterpret_cast<const void*>((uintptr_t)shard_ptrs[i]);
    if (fp8) a.scale_shards[i] = reinterpret_cast<const float*>((uintptr_t)scale_ptrs[i]);
  }
  a.rows_per_shard = rows_per_shard;
  a.table_rows = table_rows;
  a.scale_ld = (int)((head_dim + 127) / 128);
  a.out = out.data_ptr();
  if (ids_out) {
    AFB_CHECK_DT(ids_out.value(), at::kLong);
    TORCH_CHECK(ids_out->numel() == pos.numel() * heads, "ple_lookup: ids_out shape");
    a.ids_out = ids_out->data_ptr<int64_t>();
  }
  if (hot_idx) {
    AFB_CHECK_DT(hot_idx.value(), at::kLong);
    AFB_CHECK_DT(hot_base.value(), at::kLong);
    AFB_CHECK_DT(hot_len.value(), at::kInt);
    TORCH_CHECK(hot_base->numel() == heads && hot_len->numel() == heads, "ple_lookup: hot index shapes");
    a.hot_idx = hot_idx->data_ptr<int64_t>();
    a.hot_base = hot_base->data_ptr<int64_t>();
    a.hot_len = hot_len->data_ptr<int32_t>();
  }
  a.status = status_ptr(out.get_device());
  check_rc(afb::ple_lookup(a, fp8, stream()), "ple_lookup");
}
void hc_norm_op(const at::Tensor& h, const at::Tensor& w, double eps, at::Tensor& zb, at::Tensor& rstd,
                c10::optional<at::Tensor> dzb, c10::optional<at::Tensor> dh) {
  int64_t rows;
  int G, H;
  hc_shape(h, rows, G, H);
  AFB_CHECK_DT(w, at::kFloat);
  AFB_CHECK_DT(rstd, at::kFloat);
  TORCH_CHECK(w.numel() == (int64_t)G * H && rstd.numel() == rows * G, "hc_norm shapes");
  if (dzb) {
    AFB_CHECK_DT(dzb.value(), at::kFloat);
    AFB_CHECK_CONTIG(dzb.value());
    AFB_CHECK_CONTIG(dh.value());
    check_rc(afb::hc_norm_bwd(h.data_ptr(), ptr<float>(w), ptr<float>(rstd), ptr<float>(dzb.value()), dh->data_ptr(),
                              rows, G, H, stream()),
             "hc_norm_bwd");
  } else {
    AFB_CHECK_CONTIG(zb);
    check_rc(afb::hc_norm_fwd(h.data_ptr(), ptr<float>(w), zb.data_ptr(), ptr<float>(rstd), rows, G, H, (float)eps,
                              stream()),
             "hc_norm_fwd");
  }
}
void hc_mix_op(const at::Tensor& pre, const at::Tensor& zb, at::Tensor& x, c10::optional<at::Tensor> dx,
               c10::optional<at::Tensor> dpre, c10::optional<at::Tensor> dzb) {
  int64_t rows;
  int G, H;
  hc_shape(zb, rows, G, H);
  AFB_CHECK_CONTIG(pre);
  TORCH_CHECK(pre.numel() == zb.numel(), "hc_mix: pre and zb shapes");
  if (dx) {
    AFB_CHECK_CONTIG(dx.value());
    check_rc(afb::hc_mix_bwd(pre.data_ptr(), zb.data_ptr(), dx->data_ptr(), dpre->data_ptr(), ptr<float>(dzb.value()),
                             rows, G, H, stream()),
             "hc_mix_bwd");
  } else {
    AFB_CHECK_CONTIG(x);
    check_rc(afb::hc_mix_fwd(pre.data_ptr(), zb.data_ptr(), x.data_ptr(), rows, G, H, stream()), "hc_mix_fwd");
  }
}
void hc_act_op(const at::Tensor& du, int64_t R, int64_t G, at::Tensor& s, c10::optional<at::Tensor> gate) {
  AFB_CHECK_DT(du, at::kBFloat16);
  TORCH_CHECK(du.dim() == 2 && du.stride(1) == 1, "hc_act: du rows with unit column stride");
  AFB_CHECK_CONTIG(s);
  TORCH_CHECK(s.numel() == du.size(0) * R, "hc_act: s is [rows, R]");
  if (gate.has_value()) {
    AFB_CHECK_CONTIG(gate.value());
    TORCH_CHECK(gate->numel() == du.size(0) * G, "hc_act: gate is [rows, G]");
  }
  check_rc(afb::hc_act_fwd(du.data_ptr(), du.stride(0), du.size(0), R, G, s.data_ptr(),
                           gate.has_value() ? gate->data_ptr() : nullptr, stream()),
           "hc_act");
}
void hc_inject_op(const at::Tensor& h, const at::Tensor& y, const at::Tensor& gate, at::Tensor& out,
                  c10::optional<at::Tensor> dout, c10::optional<at::Tensor> dy, c10::optional<at::Tensor> dgate) {
  int64_t rows;
  int G, H;
  hc_shape(h, rows, G, H);
  AFB_CHECK_CONTIG(y);
  AFB_CHECK_CONTIG(gate);
  AFB_CHECK_DT(gate, at::kBFloat16);
  TORCH_CHECK(y.numel() == rows * H && gate.numel() == rows * G, "hc_inject shapes");
  if (dout) {
    AFB_CHECK_CONTIG(dout.value());
    check_rc(afb::hc_inject_bwd(y.data_ptr(), gate.data_ptr(), dout->data_ptr(), dy->data_ptr(),
                                ptr<float>(dgate.value()), rows, G, H, stream()),
             "hc_inject_bwd");
  } else {
    AFB_CHECK_CONTIG(out);
    check_rc(afb::hc_inject_fwd(h.data_ptr(), y.data_ptr(), gate.data_ptr(), out.data_ptr(), rows, G, H, stream()),
             "hc_inject_fwd");
  }
}

void select_tokens_op(const at::Tensor& logits, int64_t V, at::Tensor& out, double temperature, int64_t seed,
                      c10::optional<at::Tensor> step) {
  AFB_CHECK_DT(logits, at::kBFloat16);
  AFB_CHECK_DT(out, at::kInt);
  TORCH_CHECK(logits.stride(1) == 1, "logits inner stride");
  check_rc(afb::select_tokens(logits.data_ptr(), logits.stride(0), logits.size(0), V, ptr<int>(out),
                              (float)temperature, (uint64_t)seed, optr<int>(step), status_ptr(logits.get_device()),
                              stream()),
           "select_tokens");
}

void spec_accept_op(const at::Tensor& window, const at::Tensor& target, const at::Tensor& seq_slot,
                    c10::optional<at::Tensor> active, at::Tensor& ctx_len, at::Tensor& n_commit, at::Tensor& out_tokens,
                    at::Tensor& out_count, at::Tensor& anchor, at::Tensor& last_row, const at::Tensor& step,
                    c10::optional<at::Tensor> total_emitted, int64_t mode, double accept_prob, int64_t seed) {
  afb::SpecArgs a;
  a.window = ptr<int>(window);
  a.target = ptr<int>(target);
  a.seq_slot = ptr<int>(seq_slot);
  a.active = optr<int>(active);
  a.ctx_len = ptr<int>(ctx_len);
  a.n_commit = ptr<int>(n_commit);
  a.out_tokens = ptr<int>(out_tokens);
  a.out_count = ptr<int>(out_count);
  a.anchor = ptr<int>(anchor);
  a.last_row = ptr<int>(last_row);
  a.step = ptr<int>(step);
  a.total_emitted = optr<unsigned long long>(total_emitted);
  a.num_seqs = ctx_len.size(0);
  a.k = window.size(1) - 1;
  a.mode = mode;
  a.accept_prob = (float)accept_prob;
  a.seed = (uint64_t)seed;
  check_rc(afb::spec_accept(a, stream()), "spec_accept");
}

void build_window_op(const at::Tensor& anchor, c10::optional<at::Tensor> drafts, int64_t fill_token,
                     const at::Tensor& ctx_len, const at::Tensor& block_table, at::Tensor& ids, at::Tensor& positions,
                     at::Tensor& slots, at::Tensor& attn_len, c10::optional<at::Tensor> step, int64_t width,
                     int64_t pos_offset) {
  afb::WindowArgs a;
  a.anchor = ptr<int>(anchor);
  a.drafts = optr<int>(drafts);
  a.drafts_ld = drafts.has_value() ? drafts->stride(0) : 0;
  a.fill_token = fill_token;
  a.ctx_len = ptr<int>(ctx_len);
  a.block_table = ptr<int>(block_table);
  a.max_pages = block_table.size(1);
  a.ids = ptr<int>(ids);
  a.positions = ptr<int>(positions);
  a.slots = ptr<int>(slots);
  a.attn_len = ptr<int>(attn_len);
  a.step = optr<int>(step);
  a.num_seqs = ctx_len.size(0);
  a.width = width;
  a.pos_offset = pos_offset;
  check_rc(afb::build_window(a, stream()), "build_window");
}

void gather_rows_op(const at::Tensor& src, const at::Tensor& idx, at::Tensor& out) {
  check_rc(afb::gather_rows(src.data_ptr(), ptr<int>(idx), out.data_ptr(), idx.numel(), src.size(1), stream()),
           "gather_rows");
}

// ---- training kernels
void int3_dequant_op(const at::Tensor& codes, const at::Tensor& scales, at::Tensor& out) {
  AFB_CHECK_DT(scales, at::kFloat);
  AFB_CHECK_CONTIG(codes);
  AFB_CHECK_CONTIG(scales);
  const int E = codes.size(0), R = codes.size(1) * 128, K = codes.size(2) * 128;
  TORCH_CHECK(out.numel() == (int64_t)E * R * K && out.is_contiguous(), "int3_dequant: out must be [E, R, K]");
  check_rc(afb::int3_dequant(codes.data_ptr(), ptr<float>(scales), E, R, K, out.data_ptr(), stream()), "int3_dequant");
}

void int3_scale_grad_op(const at::Tensor& codes, const at::Tensor& dW, at::Tensor& dS) {
  AFB_CHECK_DT(dW, at::kBFloat16);
  AFB_CHECK_CONTIG(dW);
  const int E = codes.size(0), R = codes.size(1) * 128, K = codes.size(2) * 128;
  check_rc(afb::int3_scale_grad(codes.data_ptr(), dW.data_ptr(), E, R, K, ptr<float>(dS), stream()), "int3_scale_grad");
}

void fp8_block_fakequant_op(const at::Tensor& w, at::Tensor& out, c10::optional<at::Tensor> scale_inv) {
  AFB_CHECK_DT(w, at::kFloat);
  AFB_CHECK_CONTIG(w);
  check_rc(afb::fp8_block_fakequant(ptr<float>(w), w.size(0), w.size(1), out.data_ptr(), optr<float>(scale_inv),
                                    stream()),
           "fp8_block_fakequant");
}

void topk_tail_kl_op(const at::Tensor& z, const at::Tensor& ids, const at::Tensor& t_lp, const at::Tensor& t_tail,
                     bool reverse, double grad_scale, at::Tensor& loss, at::Tensor& dz) {
  AFB_CHECK_DT(z, at::kFloat);
  AFB_CHECK_DT(ids, at::kLong);
  AFB_CHECK_DT(dz, at::kBFloat16);
  check_rc(afb::topk_tail_kl(ptr<float>(z), z.stride(0), z.size(0), z.size(1), ptr<long long>(ids), ids.size(1),
                             ptr<float>(t_lp), ptr<float>(t_tail), reverse, (float)grad_scale, ptr<float>(loss),
                             dz.data_ptr(), dz.stride(0), stream()),
           "topk_tail_kl");
}

void adamw_op(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v, c10::optional<at::Tensor> w, double lr,
              double b1, double b2, double eps, double wd, int64_t step) {
  AFB_CHECK_DT(p, at::kFloat);
  AFB_CHECK_DT(g, at::kFloat);
  AFB_CHECK_DT(m, at::kBFloat16);
  check_rc(afb::adamw(ptr<float>(p), ptr<float>(g), m.data_ptr(), v.data_ptr(), optr<void>(w), p.numel(), (float)lr,
                      (float)b1, (float)b2, (float)eps, (float)wd, (int)step, stream()),
           "adamw");
}

void swiglu_op(const at::Tensor& x, at::Tensor& y) {
  const int T = x.size(0), I = x.size(1) / 2;
  check_rc(afb::swiglu(x.data_ptr(), y.data_ptr(), T, I, stream()), "swiglu");
}

void embedding_op(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out) {
  AFB_CHECK_DT(ids, at::kInt);
  check_rc(afb::embedding(ptr<int>(ids), table.data_ptr(), out.data_ptr(), ids.numel(), table.size(1), table.size(0),
                          status_ptr(ids.get_device()), stream()),
           "embedding");
}

}  // namespace

void register_kernel_ops(pybind11::module& m) {
  m.def("rmsnorm", &rmsnorm_op);
  m.def("qk_norm_rope_store", &qk_norm_rope_store_op, py::arg("qkv"), py::arg("Hq"), py::arg("Hkv"), py::arg("D"),
        py::arg("rot"), py::arg("qw"), py::arg("kw"), py::arg("positions"), py::arg("slots"), py::arg("cos_t"),
        py::arg("sin_t"), py::arg("eps"), py::arg("q_out"), py::arg("kcache"), py::arg("vcache"),
        py::arg("kscale") = py::none(), py::arg("vscale") = py::none());
  m.def("router_topk", &router_topk_op, py::arg("logits"), py::arg("E"), py::arg("k"), py::arg("renorm"),
        py::arg("ids"), py::arg("weights"), py::arg("cnt") = py::none(), py::arg("list") = py::none());
  m.def("expert_sort", &expert_sort_op);
  m.def("quant_rows_e4m3", &quant_rows_e4m3_op);
  m.def("quant_rows_e4m3_row", &quant_rows_e4m3_row_op);
  m.def("moe_combine", &moe_combine_op);
  m.def("moe_int3_gemm", &moe_int3_gemm_op, py::arg("codes"), py::arg("scales"), py::arg("route_cnt"),
        py::arg("route_list"), py::arg("x_div"), py::arg("x_q"), py::arg("x_scales"), py::arg("pair"), py::arg("out_q"),
        py::arg("out_scales"), py::arg("out_bf16"), py::arg("route_w"), py::arg("dbg") = py::none(),
        py::arg("ep") = nullptr, py::arg("ep_wait") = false);
  py::class_<EpCtx>(m, "EpCtx")
      .def(py::init<int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, std::vector<int64_t>, std::vector<int64_t>,
                    int64_t, const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&>())
      .def("dispatch", &EpCtx::dispatch)
      .def("wait", &EpCtx::wait)
      .def("quant_routed", &EpCtx::quant_routed)
      .def("combine", &EpCtx::combine)
      .def("set_wait_log", &EpCtx::set_wait_log)
      .def("begin_step", &EpCtx::begin_step);
  m.def("swiglu", &swiglu_op);
  m.def("int3_dequant", &int3_dequant_op);
  m.def("int3_scale_grad", &int3_scale_grad_op);
  m.def("fp8_block_fakequant", &fp8_block_fakequant_op);
  m.def("topk_tail_kl", &topk_tail_kl_op);
  m.def("adamw", &adamw_op);
  m.def("select_tokens", &select_tokens_op);
  m.def("spec_accept", &spec_accept_op);
  m.def("build_window", &build_window_op);
  m.def("gather_rows", &gather_rows_op);
  m.def("gdn_decode", &gdn_decode_op, py::arg("mixed"), py::arg("z_off"), py::arg("ba_off"), py::arg("conv_w"),
        py::arg("conv_state"), py::arg("ssm_state"), py::arg("pend_in"), py::arg("pend_qk"), py::arg("pend_v"),
        py::arg("pend_gb"), py::arg("n_commit"), py::arg("seq_slot"), py::arg("A_log"), py::arg("dt_bias"),
        py::arg("norm_w"), py::arg("out"), py::arg("q_per_seq"), py::arg("Hk"), py::arg("Dk"), py::arg("Hv"),
        py::arg("Dv"), py::arg("commit_current"), py::arg("parity"), py::arg("eps"), py::arg("dbg") = py::none());
  m.def("gdn_train", &gdn_train_op);
  m.def("ple_lookup", &ple_lookup_op);
  m.def("lora_rows_times", &lora_rows_times_op);
  m.def("transpose_bf16", &transpose_bf16_op, py::arg("src"), py::arg("dst"), py::arg("out"));
  m.def("lora_tgrad", &lora_tgrad_op);
  m.def("hc_norm", &hc_norm_op);
  m.def("hc_mix", &hc_mix_op);
  m.def("hc_act", &hc_act_op);
  m.def("hc_inject", &hc_inject_op);
  m.def("conv_silu", &conv_silu_op, py::arg("x"), py::arg("w"), py::arg("y"), py::arg("dy"), py::arg("dx"),
        py::arg("pos") = py::none());
  m.def("rmsnorm_train", &rmsnorm_train_op);
  m.def("swiglu_train", &swiglu_train_op);
  m.def("moe_combine_train", &moe_combine_train_op);
  m.def("moe_dispatch_bwd", &moe_dispatch_bwd_op);
  m.def("gdn_chunk_scan_tiles", &gdn_chunk_scan_tiles_op, py::arg("m1h"), py::arg("m2h"), py::arg("y"), py::arg("qm"),
        py::arg("last"), py::arg("init"), py::arg("states"), py::arg("x"), py::arg("final_state"), py::arg("reverse"),
        py::arg("reset") = py::none());
  m.def("gdn_chunk_scan", &gdn_chunk_scan_op, py::arg("m1"), py::arg("m2"), py::arg("y"), py::arg("qm"),
        py::arg("last"), py::arg("init"), py::arg("states"), py::arg("x"), py::arg("final_state"), py::arg("reverse"),
        py::arg("precise") = false, py::arg("reset") = py::none());
  m.def("paged_attention", &paged_attention_op, py::arg("q"), py::arg("kcache"), py::arg("vcache"),
        py::arg("block_table"), py::arg("seq_lens"), py::arg("q_per_seq"), py::arg("scale"), py::arg("out"),
        py::arg("gate"), py::arg("gate_ld"), py::arg("gate_head_stride"), py::arg("splits"),
        py::arg("pages_per_split"), py::arg("window"), py::arg("bt_row"), py::arg("sp_count") = py::none(),
        py::arg("sp_lpage") = py::none(), py::arg("sp_mask") = py::none(), py::arg("kscale") = py::none(),
        py::arg("vscale") = py::none(), py::arg("impl") = 0, py::arg("sp_block") = 64, py::arg("sp_slot") = py::none());
  m.def("qsa_prep", &qsa_prep_op);
  m.def("attn_train_fwd", &attn_train_fwd_op, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("cu"),
        py::arg("tiles"), py::arg("scale"), py::arg("out"), py::arg("lse"), py::arg("blkmap") = py::none(),
        py::arg("qsa_block") = 64, py::arg("causal") = true);
  m.def("vit_patch_pos", &vit_patch_pos_op);
  m.def("vit_qkv_rope", &vit_qkv_rope_op);
  m.def("vit_layernorm", &vit_layernorm_op);
  m.def("attn_train_bwd", &attn_train_bwd_op, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("cu"),
        py::arg("tiles"), py::arg("kv_tiles"), py::arg("scale"), py::arg("out"), py::arg("lse"), py::arg("dout"),
        py::arg("delta"), py::arg("dq"), py::arg("dk"), py::arg("dv"), py::arg("dk_part"), py::arg("dv_part"),
        py::arg("blkmap") = py::none(), py::arg("qsa_block") = 64);
  m.def("qsa_rowmap", [](const at::Tensor& u_lpage, const at::Tensor& u_mask, const at::Tensor& u_count,
                         const at::Tensor& set_row0, const at::Tensor& set_rows, int64_t W, at::Tensor& blkmap) {
    AFB_CHECK_DT(u_lpage, at::kInt);
    AFB_CHECK_DT(u_mask, at::kByte);
    AFB_CHECK_DT(blkmap, at::kInt);
    AFB_CHECK_CONTIG(blkmap);
    const int S = u_count.size(0);
    TORCH_CHECK(u_lpage.size(0) >= S && u_lpage.sizes() == u_mask.sizes() && set_row0.numel() >= S &&
                    set_rows.numel() >= S, "qsa_rowmap shapes");
    afb_bind::check_rc(afb::qsa_rowmap(afb_bind::ptr<int>(u_lpage), afb_bind::ptr<uint8_t>(u_mask),
                                       afb_bind::ptr<int>(u_count), afb_bind::ptr<int>(set_row0),
                                       afb_bind::ptr<int>(set_rows), S, (int)W, u_lpage.size(1),
                                       reinterpret_cast<uint32_t*>(blkmap.data_ptr()), blkmap.size(1),
                                       afb_bind::stream()),
                       "qsa_rowmap");
  });
  py::class_<GuardCtx>(m, "GuardCtx")
      .def(py::init<int64_t, int64_t, std::vector<int64_t>, int64_t, int64_t, int64_t, const at::Tensor&,
                    const at::Tensor&>())
      .def("check", &GuardCtx::check);
  py::class_<ZeroCtx>(m, "ZeroCtx")
      .def(py::init<int64_t, int64_t, std::vector<int64_t>, int64_t, int64_t, const at::Tensor&, const at::Tensor&,
                    const at::Tensor&>())
      .def("signal", &ZeroCtx::signal)
      .def("wait", &ZeroCtx::wait)
      .def("rs", &ZeroCtx::rs)
      .def("norm_publish", &ZeroCtx::norm_publish)
      .def("adamw", &ZeroCtx::adamw);
  py::class_<HsCtx>(m, "HsCtx")
      .def(py::init<int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, bool, const at::Tensor&,
                    const std::vector<std::vector<int64_t>>&>())
      .def("cycle_start", &HsCtx::cycle_start)
      .def("writeback", &HsCtx::writeback)
      .def("after_prefill", &HsCtx::after_prefill)
      .def("fetch", &HsCtx::fetch);
  m.def("qsa_select", &qsa_select_op, py::arg("idx_q"), py::arg("idx_key"), py::arg("idx_raw"), py::arg("k_norm"),
        py::arg("block_table"), py::arg("fin"), py::arg("seq_lens"), py::arg("W"), py::arg("K"), py::arg("Hi"),
        py::arg("block"), py::arg("sel"), py::arg("cos_t"), py::arg("sin_t"), py::arg("rot"), py::arg("eps"),
        py::arg("u_page"), py::arg("u_lpage"), py::arg("u_mask"), py::arg("u_count"), py::arg("bt_row") = py::none(), py::arg("scores") = py::none());

  m.def("qsa_finalize", &qsa_finalize_op);
  m.def("embedding", &embedding_op);
}
