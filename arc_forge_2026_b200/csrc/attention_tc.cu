// Paged decode / speculative-verify attention on the 5th-generation tensor cores (tcgen05, TMEM accumulators), bf16
// KV cache, dense causal mode: the path the serving verify step runs for every full-attention layer.
//
// One CTA per (sequence, KV head, KV split), as in attention.cu: its query rows are the q_per_seq verify positions x
// the Hq/Hkv query heads of the KV head (row r = t * group + h, at most 64 rows; a wider set, e.g. 8 positions x 12
// heads, is cut into runs of 64 / group positions over gridDim.z), so one KV page read serves every head and
// position. Per 64-key page:
//   S = Q K^T   tcgen05.mma kind::f16, M=128 (rows past the CTA's rows are never read), N=64, K=16 per op;
//               Q and the K page are K-major 128-byte-swizzled shared-memory operands, S lands in TMEM
//   softmax     two warps (TMEM lane quadrants 0 and 1 = rows 0..63) load S rows, mask (causality inside the verify
//               window, the split's pages), keep a running max m and sum l in the log2 domain and write P = 2^(S - m)
//               as bf16 into TMEM, where the next MMA reads it as its A operand
//   O += P V    tcgen05.mma with A = P from TMEM and B = the V page as an MN-major operand (keys x D, D contiguous),
//               N = D, accumulated in TMEM across pages
// The running max is raised lazily: a row's O is rescaled (read from TMEM, scaled, written back) only when its max
// grows by more than 8 (a factor of 256), which after the first pages almost never happens; P, l and O stay
// consistent with whatever max the row currently uses.
// Warp roles: 0 loader (TMA of Q and of the K and V pages, no multicast, 3-stage ring), 1 MMA issuer (+ TMEM),
// 4-5 softmax / output (the rows), the others idle. S and P are double-buffered so the QK^T of page i+1 overlaps the
// softmax of page i and the PV of page i-1. Splits write (O / l, m + log2 l) partials for attn_merge_kernel.
//
// QSA sparse modes (sp_count set): the CTA walks its sequence's block union instead of its pages. With 64-token
// blocks an entry is a page (the TMA loader reads the union's physical pages); with smaller blocks (4 for the
// reference's QSA) warps 2, 3 and 6..11 gather 64 / B entries into each 64-key tile with 16-byte cp.async copies
// written at the 128-byte-swizzled offsets the TMA would use, a proxy fence per thread before its arrive. The
// softmax warps turn each tile's (block, row mask) entries into a per-row 64-bit visibility mask (mask bit of the
// row's verify position and causality), so the MMA side is the same in every mode.
//
// NVFP4 KV (kscale set; dense or 64-token QSA blocks): warps 2, 3 and 6..11 read each page-head's e2m1 codes and e4m3
// scales (0.5625 bytes per element) with plain 16-byte loads one tile ahead, dequantise them exactly to f16 (the
// hardware e2m1x2 / e4m3x2 -> f16x2 conversions and one f16x2 multiply by the scale: e2m1 x e4m3 needs at most 5
// significant bits) and store the swizzled f16 tiles the MMAs read; Q is converted to f16 in place and P is written
// as f16, so the MMAs of this mode are f16 x f16 and NVFP4 moves 3.6x fewer bytes through the same pipeline.
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>

#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace afb {

namespace attn_tc {
constexpr int PAGE = 64;
constexpr int THREADS = 384;                   // warps 0..11 (8..11 work only in the NVFP4 mode)
constexpr int W_LD = 0, W_MMA = 1, W_SM0 = 4;  // softmax warps 4 and 5
constexpr float RESCALE = 8.f;                 // log2 growth of a row max that forces an O rescale
constexpr int GATHER_THREADS = 256;            // warps 2, 3, 6..11 in the sub-page gather mode
constexpr int CONV_THREADS = 256;              // warps 2, 3, 6, 7, 8..11 in the NVFP4 mode (every SM sub-partition)
AFB_DEV int conv_index(int warp) {             // gather / NVFP4 converter warp -> 0..7, or -1
  return warp == 2 || warp == 3 ? warp - 2 : warp == 6 || warp == 7 ? warp - 4 : warp >= 8 && warp < 12 ? warp - 4 : -1;
}

template <int D>
struct Smem {
  static constexpr uint32_t SUB = PAGE * 128;                 // one 64-row x 128-byte swizzled sub-tile
  static constexpr uint32_t Q_BYTES = (D / 64) * SUB;         // 64 query rows; the MMA's rows 64..127 alias what
                                                              // follows (their results are never read)
  static constexpr uint32_t KV_BYTES = (D / 64) * SUB;        // one K (or V) page of one head
  static constexpr int NS = D == 256 ? 3 : 6;                 // KV stages
  static constexpr uint32_t STAGE = 2 * KV_BYTES;
  static constexpr uint32_t KV_OFF = Q_BYTES;
  static constexpr uint32_t VIS_OFF = KV_OFF + NS * STAGE;    // sparse modes: per stage, per key, the verify
                                                              // positions (bits) that may see the key
  static constexpr uint32_t BAR_OFF = VIS_OFF + NS * PAGE * 4;
  // kv_full[NS], kv_empty[NS], s_full[2], s_empty[2], p_full[2], o_done[2], q_ready, mma_fin, q_conv, tmem slot
  static constexpr uint32_t TOTAL = BAR_OFF + (2 * NS + 11) * 8 + 16 + 1024;
  // TMEM columns: O [D], S [2][64], P [2][32] (bf16 pairs)
  static constexpr uint32_t O_COL = 0, S_COL = D, P_COL = D + 2 * PAGE;
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(P_COL + 2 * PAGE / 2 <= TMEM_COLS, "TMEM columns");
};
}  // namespace attn_tc

template <int D>
__global__ void __launch_bounds__(attn_tc::THREADS, 1)
    paged_attn_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                         const __grid_constant__ CUtensorMap tmQ, AttnArgs a, uint32_t* status) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  using namespace attn_tc;
  using L = Smem<D>;
  constexpr int NS = L::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* kv_empty = kv_full + NS;
  uint64_t* s_full = kv_empty + NS;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* q_ready = o_done + 2;
  uint64_t* mma_fin = q_ready + 1;
  uint64_t* q_conv = mma_fin + 1;  // NVFP4 mode: Q converted to f16 in place
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_conv + 1);
  uint32_t* vis_all = reinterpret_cast<uint32_t*>(smem + L::VIS_OFF);  // [NS][PAGE]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // blockIdx.x = (sequence, KV head, row run): the row runs of one (sequence, head) are neighbours in launch order,
  // so they stream the same KV close together in time (the second read mostly hits L2)
  const int group = a.Hq / a.Hkv;
  const int tpc = min(a.q_per_seq, 64 / group);
  const int nruns = (a.q_per_seq + tpc - 1) / tpc;
  const int run = blockIdx.x % nruns;
  const int seq = blockIdx.x / nruns / a.Hkv, kvh = blockIdx.x / nruns % a.Hkv;
  const int split = blockIdx.y;
  // query positions per CTA: all of them when q_per_seq x group <= 64, else a run of tpc positions
  const int tbase = run * tpc;
  const int QR = min(tpc, a.q_per_seq - tbase) * group;  // live query rows of this CTA (<= 64)
  const int seq_len = a.seq_lens[seq];
  const int past = seq_len - a.q_per_seq;
  const bool sparse = a.sp_count != nullptr;
  const bool gather = sparse && a.sp_block < PAGE;  // sub-page blocks gathered into 64-key tiles
  const bool fp4 = a.kscale != nullptr;             // NVFP4 pages dequantised into the tiles
  const int spb = sparse ? a.sp_block : PAGE;       // tokens per union entry
  const int ept = PAGE / spb;                       // entries per tile
  const int cnt = sparse ? a.sp_count[seq] : 0;
  const int npages = sparse ? (cnt + ept - 1) / ept : (seq_len + PAGE - 1) / PAGE;  // 64-key tiles
  // sliding window (dense mode): the first page any row of the CTA can see
  const int pbeg = (!sparse && a.window > 0) ? max(0, past + 1 - a.window) / PAGE : 0;
  const int p0 = pbeg + split * a.pages_per_split;
  const int p1 = min(npages, p0 + a.pages_per_split);
  const int n = max(0, p1 - p0);
  const int* bt = a.block_table + (size_t)(a.bt_row ? a.bt_row[seq] : seq) * a.max_pages;
  const int sp_ld = a.sp_ld ? a.sp_ld : a.max_pages;
  const int* spl = sparse ? a.sp_lpage + (size_t)seq * sp_ld : nullptr;
  const uint8_t* spm = sparse ? a.sp_mask + (size_t)seq * sp_ld : nullptr;

  if (n == 0) {  // an empty split (or a sequence without keys): nothing to stream, no TMEM
    const int r = threadIdx.x;
    if (r < QR) {
      const size_t tok = (size_t)seq * a.q_per_seq + tbase + r / group;
      const int head = kvh * group + r % group;
      if (gridDim.y > 1) {
        a.part_lse[((size_t)split * a.num_tokens + tok) * a.Hq + head] = -INFINITY;
      } else {
        __nv_bfloat16* op = a.out + (tok * a.Hq + head) * D;
        for (int c = 0; c < D; c += 8) *reinterpret_cast<uint4*>(op + c) = make_uint4(0, 0, 0, 0);
      }
    }
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&kv_full[s], fp4 ? CONV_THREADS : gather ? GATHER_THREADS : 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 2);  // the two softmax warps
      mbar_init(&p_full[b], 2);
      mbar_init(&o_done[b], 1);
    }
    mbar_init(q_ready, 1);
    mbar_init(q_conv, CONV_THREADS);
    mbar_init(mma_fin, 1);
    fence_mbar_init();
  }
  if (warp == W_MMA) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == W_LD) {
    // ------------------------------------------------------------------ loader
    // Q: one 3-D box {64 columns, group heads, tpc tokens} per 64-column sub-tile lands rows t * group + h (rows
    // past the live ones hold other positions or the out-of-range fill: never read)
    if (lane == 0) {
      if (!fp4) {
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
      }
      mbar_arrive_expect_tx(q_ready, (uint32_t)(tpc * group) * D * 2);
#pragma unroll
      for (int c = 0; c < D / 64; ++c)
        tma_load_3d(smem + c * L::SUB, &tmQ, q_ready, c * 64, kvh * group, seq * a.q_per_seq + tbase);
    }
    // block-table entries 32 at a time (one per lane), then one K + V fill per page (the gather warps fill the
    // tiles in the sub-page mode)
    int issued = 0;
    for (int base = 0; base < n && ok && !gather && !fp4; base += 32) {
      const int mine = base + lane < n ? bt[p0 + base + lane] : 0;
      const int cnt = min(32, n - base);
      for (int j = 0; j < cnt; ++j) {
        const int i = base + j, s = i % NS;
        const int page = __shfl_sync(0xffffffffu, mine, j);
        if (i >= NS && !__all_sync(0xffffffffu, mbar_wait(&kv_empty[s], ((i / NS) & 1) ^ 1, status))) {
          ok = false;
          break;
        }
        if (sparse) {  // page union: every key of entry p0 + i, its logical position and row mask
          const int e = p0 + i;
          const int lp = spl[e];
          const uint32_t mk = spm[e];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int pos = lp * PAGE + lane + 32 * h;
            uint32_t vb = 0;
#pragma unroll
            for (int tt = 0; tt < 8; ++tt)
              if (((mk >> tt) & 1u) && pos <= past + tt) vb |= 1u << tt;
            vis_all[s * PAGE + lane + 32 * h] = vb;
          }
          __syncwarp();
        }
        if (lane == 0) {
          const int row = (page * a.Hkv + kvh) * PAGE;
          uint8_t* st = smem + L::KV_OFF + s * L::STAGE;
          mbar_arrive_expect_tx(&kv_full[s], L::STAGE);
#pragma unroll
          for (int c = 0; c < D / 64; ++c) {
            tma_load_2d(st + c * L::SUB, &tmK, &kv_full[s], c * 64, row);
            tma_load_2d(st + L::KV_BYTES + c * L::SUB, &tmV, &kv_full[s], c * 64, row);
          }
        }
        ++issued;
      }
    }
    // no copy may still be landing when the CTA exits (after a timeout elsewhere the MMA warp may not have
    // consumed the last stages): wait, bounded, for Q and the last NS fills
    if (lane == 0) {
      mbar_wait(q_ready, 0, status);
      for (int i = max(0, issued - NS); i < issued; ++i) mbar_wait(&kv_full[i % NS], (i / NS) & 1, status);
    }
  } else if (fp4 && conv_index(warp) >= 0) {
    // ------------------------------------------------------------------ NVFP4 dequantisation into the tiles
    // thread gt converts units of 32 elements (16 bytes of codes + 2 scales) of the K and V page-head: unit u of a
    // tile is row u / (D / 32), column group u % (D / 32). The next tile's codes and scales are loaded (plain
    // loads) before this tile's stage wait; a tile is published (this thread's proxy fence, then its arrive) as
    // soon as its stores are done.
    constexpr int UPR = D / 32;                 // 32-element units per row
    constexpr int UPT = PAGE * UPR / CONV_THREADS;  // units per thread per K (or V) tile
    const int gt = conv_index(warp) * 32 + lane;
    // Q to f16 in place (the MMAs of this mode take f16 operands: K / V dequantise exactly to f16 with the
    // hardware e2m1 / e4m3 conversions; Q's bf16 values are exact in f16 at normalised magnitudes)
    if (!mbar_wait(q_ready, 0, status)) ok = false;
    for (int i = gt; i < (int)(L::Q_BYTES / 16); i += CONV_THREADS) {
      uint4* p = reinterpret_cast<uint4*>(smem) + i;
      uint4 v = *p;
      uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
        w[j] = pack_f16x2(f.x, f.y);
      }
      *p = v;
    }
    fence_proxy_async_smem();
    mbar_arrive(q_conv);
    const uint8_t* kc = reinterpret_cast<const uint8_t*>(a.kcache);
    const uint8_t* vc = reinterpret_cast<const uint8_t*>(a.vcache);
    uint4 ck[UPT], cv[UPT];
    uint32_t sk[UPT], sv2[UPT];
    // the page of tile i + 1 is read one iteration ahead, so a tile's code loads wait on no block-table load
    int page_next = n > 0 ? bt[p0] : 0;
    auto fetch = [&](int i) {
      if (i >= n) return;
      const size_t ph = (size_t)page_next * a.Hkv + kvh;  // page-head: 64 rows (union pages in QSA mode)
      page_next = i + 1 < n ? bt[p0 + i + 1] : 0;
#pragma unroll
      for (int u = 0; u < UPT; ++u) {
        const int unit = u * CONV_THREADS + gt, r = unit / UPR, cg = unit % UPR;
        const size_t crow = (ph * PAGE + r) * (D / 2) + cg * 16, srow = (ph * PAGE + r) * (D / 16) + cg * 2;
        ck[u] = __ldg(reinterpret_cast<const uint4*>(kc + crow));
        cv[u] = __ldg(reinterpret_cast<const uint4*>(vc + crow));
        sk[u] = *reinterpret_cast<const uint16_t*>(a.kscale + srow);
        sv2[u] = *reinterpret_cast<const uint16_t*>(a.vscale + srow);
      }
    };
    auto scale_h2 = [](uint32_t e4m3) -> uint32_t {  // e4m3 byte -> (s, s) in f16 (exact)
      uint32_t d;
      const uint16_t two = (uint16_t)(e4m3 | (e4m3 << 8));
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(two));
      return d;
    };
    auto e2m1x2_h2 = [](uint32_t byte) -> uint32_t {  // two e2m1 codes (first in the low nibble) -> f16 pair
      uint32_t d;
      const uint16_t b = (uint16_t)byte;
      asm("{\n\t.reg .b8 t;\n\tcvt.u8.u16 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(d) : "h"(b));
      return d;
    };
    auto store_unit = [&](uint8_t* tile, int unit, const uint4& codes, uint32_t scales) {
      const int r = unit / UPR, cg = unit % UPR;
      const uint32_t w[4] = {codes.x, codes.y, codes.z, codes.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        // step q stores word qq = (q + cg / 2) % 4 (8 elements, chunk cg * 4 + qq): the 8 lanes of a row then hit
        // 8 different 16-byte positions of their 128-byte row, whichever sub-tile each lands in (no bank conflict
        // beyond the four wavefronts a 16-byte store of 32 lanes needs)
        const int qq = (q + (cg >> 1)) & 3;
        const uint32_t wq = qq == 0 ? w[0] : qq == 1 ? w[1] : qq == 2 ? w[2] : w[3];
        const uint32_t s2 = scale_h2((scales >> (8 * (qq >> 1))) & 0xffu);
        uint32_t o[4];
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
          const uint32_t pr = e2m1x2_h2((wq >> (8 * bb)) & 0xffu);
          const __half2 x = __hmul2(*reinterpret_cast<const __half2*>(&pr), *reinterpret_cast<const __half2*>(&s2));
          o[bb] = *reinterpret_cast<const uint32_t*>(&x);
        }
        const int c = cg * 4 + qq;
        const uint32_t so = (c >> 3) * L::SUB + r * 128 + (((c & 7) ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(tile + so) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    };
    fetch(0);
    for (int i = 0; i < n; ++i) {
      const int s = i % NS;
      uint4 ck0[UPT], cv0[UPT];
      uint32_t sk0[UPT], sv0[UPT];
#pragma unroll
      for (int u = 0; u < UPT; ++u) {
        ck0[u] = ck[u];
        cv0[u] = cv[u];
        sk0[u] = sk[u];
        sv0[u] = sv2[u];
      }
      fetch(i + 1);  // in flight under this tile's wait and conversion
      if (i >= NS && !mbar_wait(&kv_empty[s], ((i / NS) & 1) ^ 1, status)) {
        ok = false;
        break;
      }
      if (sparse && gt < 32) {  // page union: the entry's positions and row mask (published by the arrive)
        const int e = p0 + i, lp = spl[e];
        const uint32_t mk = spm[e];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int pos = lp * PAGE + lane + 32 * h;
          uint32_t vb = 0;
#pragma unroll
          for (int tt = 0; tt < 8; ++tt)
            if (((mk >> tt) & 1u) && pos <= past + tt) vb |= 1u << tt;
          vis_all[s * PAGE + lane + 32 * h] = vb;
        }
      }
      uint8_t* st = smem + L::KV_OFF + s * L::STAGE;
#pragma unroll
      for (int u = 0; u < UPT; ++u) {
        store_unit(st, u * CONV_THREADS + gt, ck0[u], sk0[u]);
        store_unit(st + L::KV_BYTES, u * CONV_THREADS + gt, cv0[u], sv0[u]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&kv_full[s]);
    }
  } else if (gather && conv_index(warp) >= 0) {
    // ------------------------------------------------------------------ sub-page gather (QSA blocks < 64 tokens)
    // One 16-byte chunk per thread and copy: the 128 threads walk the tile's 64 rows x D/8 chunks chunk-fastest,
    // so a warp's copy covers whole contiguous rows (512 or 256 bytes). Lane l resolves keys l and l + 32 (KV slot,
    // position bits) for the NEXT tile while this tile's copies are issued; the slots go round by shuffles. Up to
    // NS - 1 tiles of copies are in flight; tile i - (NS - 1) is published (this thread's wait for its group, a
    // proxy fence, the arrive) BEFORE the wait for tile i's stage, since freeing that stage needs the QK^T of the
    // tile after the one that used it.
    constexpr int CH = D / 8;  // 16-byte chunks per row
    constexpr int ITERS = PAGE * CH / GATHER_THREADS;
    constexpr int LAG = NS - 1;
    const int gw = conv_index(warp);  // warps 2, 3, 6..11 -> 0..7
    const int gt = gw * 32 + lane;
    auto resolve = [&](int i, int (&slot)[2], uint32_t (&vb)[2]) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int k = lane + 32 * h, e = (p0 + i) * ept + k / spb;
        slot[h] = -1;
        vb[h] = 0;
        if (i < n && e < cnt) {
          const int sl = a.sp_slot[(size_t)seq * sp_ld + e] + k % spb;  // a block never crosses a page
          const int pos = spl[e] * spb + k % spb;
          const uint32_t mk = spm[e];
#pragma unroll
          for (int tt = 0; tt < 8; ++tt)
            if (((mk >> tt) & 1u) && pos <= past + tt) vb[h] |= 1u << tt;
          if (sl >= 0 && (sl >> 6) < a.num_pages) slot[h] = sl;
          else flag_error(status, AFB_ERR_BOUNDS);
        }
      }
    };
    int cur[2], nxt[2];
    uint32_t vcur[2], vnxt[2];
    resolve(0, cur, vcur);
    int issued = 0, published = 0;
    for (int i = 0; i < n; ++i) {
      const int s = i % NS;
      if (i >= LAG) {
        cp_async_wait<LAG - 1>();
        fence_proxy_async_smem();
        mbar_arrive(&kv_full[published % NS]);
        ++published;
      }
      resolve(i + 1, nxt, vnxt);  // loads in flight under this tile's copies
      if (i >= NS && !mbar_wait(&kv_empty[s], ((i / NS) & 1) ^ 1, status)) {
        ok = false;
        break;
      }
      if (gw == 0) {  // published by these threads' arrives for the tile
        vis_all[s * PAGE + lane] = vcur[0];
        vis_all[s * PAGE + 32 + lane] = vcur[1];
      }
      uint8_t* st = smem + L::KV_OFF + s * L::STAGE;
      const char* kb = reinterpret_cast<const char*>(a.kcache);
      const char* vbase = reinterpret_cast<const char*>(a.vcache);
#pragma unroll
      for (int it = 0; it < ITERS; ++it) {
        const int idx = it * GATHER_THREADS + gt, key = idx / CH, c = idx % CH;
        const int sl = __shfl_sync(0xffffffffu, key < 32 ? cur[0] : cur[1], key & 31);
        const uint32_t bytes = sl >= 0 ? 16u : 0u;
        const size_t off = sl >= 0 ? ((((size_t)(sl >> 6) * a.Hkv + kvh) * PAGE + (sl & 63)) * D * 2 + c * 16) : 0;
        const uint32_t so = (c >> 3) * L::SUB + key * 128 + (((c & 7) ^ (key & 7)) << 4);
        cp_async16(st + so, kb + off, bytes);
        cp_async16(st + L::KV_BYTES + so, vbase + off, bytes);
      }
      cp_async_commit();
      ++issued;
      cur[0] = nxt[0];
      cur[1] = nxt[1];
      vcur[0] = vnxt[0];
      vcur[1] = vnxt[1];
    }
    cp_async_wait<0>();
    fence_proxy_async_smem();
    for (; published < issued; ++published) mbar_arrive(&kv_full[published % NS]);
  } else if (warp == W_MMA) {
    // ------------------------------------------------------------------ MMA issuer
    // bf16 operands; f16 in the NVFP4 mode (Q converted in place, K / V dequantised to f16, P written as f16)
    const uint32_t idesc_s = idesc_f16(128, PAGE, fp4 ? 0 : 1);             // S = Q K^T
    const uint32_t idesc_o = idesc_f16(128, D, fp4 ? 0 : 1) | (1u << 16);   // O += P V, B (V) MN-major
    ok = __all_sync(0xffffffffu, mbar_wait(fp4 ? q_conv : q_ready, 0, status));
    tc_fence_after();
    const uint32_t q_base = smem_u32(smem);
    auto issue_pv = [&](int j) {  // page j: wait for its P, then O += P V
      const int sb = j & 1, s = j % NS;
      if (!__all_sync(0xffffffffu, mbar_wait(&p_full[sb], (j >> 1) & 1, status))) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t v_base = smem_u32(smem + L::KV_OFF + s * L::STAGE + L::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < PAGE / 16; ++kk)  // 16 keys per op: 2 KB into the page (two 8-row swizzle atoms)
          umma_f16_ta(tmem + L::O_COL, tmem + L::P_COL + sb * (PAGE / 2) + kk * 8,
                      sw128_desc_mn(v_base + kk * 16 * 128, L::SUB, 1024), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&o_done[sb]);
        umma_commit(&kv_empty[s]);
      }
      __syncwarp();
      return true;
    };
    for (int i = 0; i < n && ok; ++i) {
      const int s = i % NS, sb = i & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&kv_full[s], (i / NS) & 1, status)) ||
          (i >= 2 && !__all_sync(0xffffffffu, mbar_wait(&s_empty[sb], ((i >> 1) & 1) ^ 1, status)))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t k_base = smem_u32(smem + L::KV_OFF + s * L::STAGE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::SUB + (kk & 3) * 32;
          umma_f16(tmem + L::S_COL + sb * PAGE, sw128_desc(q_base + off), sw128_desc(k_base + off), idesc_s,
                   kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
      }
      __syncwarp();
      if (i >= 1 && !issue_pv(i - 1)) {
        ok = false;
        break;
      }
    }
    if (ok && n > 0) issue_pv(n - 1);
    // every MMA this thread issued has completed before TMEM is released (also after a timeout)
    if (lane == 0) umma_commit(mma_fin);
    __syncwarp();
    mbar_wait(mma_fin, 0, status);
  } else if (warp == W_SM0 || warp == W_SM0 + 1) {
    // ------------------------------------------------------------------ softmax + output (rows 0..63)
    const int quad = warp - W_SM0;
    const int r = quad * 32 + lane;  // query row = TMEM lane
    const int t = tbase + r / group, hq = r % group;  // verify position (0 .. q_per_seq - 1) and head
    const bool live = r < QR;
    const int vis = past + t + 1;  // keys this row may see: positions < vis
    const int win_lo = a.window > 0 ? vis - a.window : INT_MIN / 2;  // and >= win_lo (sliding window)
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    float m = -INFINITY, l = 0.f;
    for (int i = 0; i < n; ++i) {
      const int sb = i & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[sb], (i >> 1) & 1, status))) {
        ok = false;
        break;
      }
      // sparse: this row's visible keys of tile i, from the per-key position bits the loader wrote with the tile
      // (its stage is not refilled before this tile's PV): two ballots per verify position
      uint32_t vlo = 0, vhi = 0;
      if (sparse) {
        const int st = i % NS;
        if (!__all_sync(0xffffffffu, mbar_wait(&kv_full[st], (i / NS) & 1, status))) {
          ok = false;
          break;
        }
        const uint32_t vb0 = vis_all[st * PAGE + lane], vb1 = vis_all[st * PAGE + 32 + lane];
#pragma unroll
        for (int tt = 0; tt < 8; ++tt) {
          if (tt >= a.q_per_seq) break;
          const uint32_t b0 = __ballot_sync(0xffffffffu, (vb0 >> tt) & 1u);
          const uint32_t b1 = __ballot_sync(0xffffffffu, (vb1 >> tt) & 1u);
          if (tt == t) {
            vlo = b0;
            vhi = b1;
          }
        }
      }
      tc_fence_after();
      float sv[PAGE];
      tmem_ld32(lane_base + L::S_COL + sb * PAGE, sv);
      tmem_ld32(lane_base + L::S_COL + sb * PAGE + 32, sv + 32);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);
      // the page's visible key range, relative to its first key (hoisted: one compare pair per key)
      const int kbase = (p0 + i) * PAGE;
      const int j_hi = vis - kbase, j_lo = win_lo - kbase;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < PAGE; ++j) {
        const bool see = sparse ? (((j < 32 ? vlo >> j : vhi >> (j - 32)) & 1u) != 0) : (j < j_hi && j >= j_lo);
        const float x = (live && see) ? sv[j] * a.scale_log2 : -INFINITY;
        sv[j] = x;
        mx = fmaxf(mx, x);
      }
      // lazy max: keep the current one unless this page raises it by more than RESCALE
      float mnew = m;
      if (mx > m + RESCALE || m == -INFINITY) mnew = mx;
      const bool rescale = m != -INFINITY && mnew != m;
      if (__any_sync(0xffffffffu, rescale)) {
        // O must hold every earlier page before it is scaled: wait for the PV of page i - 1
        if (i >= 1 && !__all_sync(0xffffffffu, mbar_wait(&o_done[(i - 1) & 1], ((i - 1) >> 1) & 1, status))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float f = rescale ? exp2f(m - mnew) : 1.f;
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          float ov[32];
          tmem_ld32(lane_base + L::O_COL + c, ov);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) ov[j] *= f;
          tmem_st32(lane_base + L::O_COL + c, reinterpret_cast<const uint32_t*>(ov));
        }
        tmem_st_wait();
        l *= f;
      }
      m = mnew;
      const float base = m == -INFINITY ? 0.f : m;
      uint32_t pk[PAGE / 2];
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < PAGE / 2; ++j) {
        const float e0 = exp2f(sv[2 * j] - base), e1 = exp2f(sv[2 * j + 1] - base);
        rs += e0 + e1;
        pk[j] = fp4 ? pack_f16x2(e0, e1) : pack_bf16x2(e0, e1);
      }
      l += rs;
      // P of page i goes into P buffer sb; the PV of page i - 2 (which read that buffer) must be done
      if (i >= 2 && !__all_sync(0xffffffffu, mbar_wait(&o_done[sb], ((i - 2) >> 1) & 1, status))) {
        ok = false;
        break;
      }
      tmem_st32(lane_base + L::P_COL + sb * (PAGE / 2), pk);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
    }
    // ---- output: O / l of the last PV (splits: partials with the log2-sum-exp)
    if (ok && __all_sync(0xffffffffu, mbar_wait(&o_done[(n - 1) & 1], ((n - 1) >> 1) & 1, status))) {
      tc_fence_after();
      const size_t tok = (size_t)seq * a.q_per_seq + t;
      const int head = kvh * group + hq;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool direct = gridDim.y == 1;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        float ov[32];
        tmem_ld32(lane_base + L::O_COL + c, ov);
        tmem_ld_wait();
        if (!live) continue;
        if (direct) {
          __nv_bfloat16* op = a.out + (tok * a.Hq + head) * D + c;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            float g[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              g[e] = 1.f;
              if (a.gate) {
                const float z = __bfloat162float(a.gate[tok * a.gate_ld + head * a.gate_head_stride + c + j + e]);
                g[e] = 1.f / (1.f + __expf(-z));
              }
            }
            *reinterpret_cast<uint4*>(op + j) =
                make_uint4(pack_bf16x2(ov[j] * inv * g[0], ov[j + 1] * inv * g[1]),
                           pack_bf16x2(ov[j + 2] * inv * g[2], ov[j + 3] * inv * g[3]),
                           pack_bf16x2(ov[j + 4] * inv * g[4], ov[j + 5] * inv * g[5]),
                           pack_bf16x2(ov[j + 6] * inv * g[6], ov[j + 7] * inv * g[7]));
          }
        } else {
          float* pp = a.part_o + (((size_t)split * a.num_tokens + tok) * a.Hq + head) * D + c;
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(pp + j) =
                make_float4(ov[j] * inv, ov[j + 1] * inv, ov[j + 2] * inv, ov[j + 3] * inv);
        }
      }
      if (live && !direct)
        a.part_lse[((size_t)split * a.num_tokens + tok) * a.Hq + head] = l > 0.f ? m + log2f(l) : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == W_MMA) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

template <int D>
static int launch_attn_tc(const AttnArgs& a, int splits, uint32_t* status, cudaStream_t st) {
  using L = attn_tc::Smem<D>;
  CUtensorMap tk{}, tv{};
  const uint64_t rows = (uint64_t)a.num_pages * a.Hkv * attn_tc::PAGE;
  int rc = 0;
  if (!a.kscale) {  // NVFP4 pages are read by the converter warps, not by TMA
    rc = make_tmap_2d(&tk, a.kcache, 2, D, rows, (uint64_t)D * 2, 64, attn_tc::PAGE, 1);
    if (rc) return 1000 + rc;
    rc = make_tmap_2d(&tv, a.vcache, 2, D, rows, (uint64_t)D * 2, 64, attn_tc::PAGE, 1);
    if (rc) return 1000 + rc;
  }
  CUtensorMap tq{};
  const int group = a.Hq / a.Hkv;
  const uint64_t qdims[3] = {(uint64_t)D, (uint64_t)a.Hq, (uint64_t)a.num_tokens};
  const uint64_t qstr[2] = {(uint64_t)D * 2, (uint64_t)a.Hq * D * 2};
  const int tpc = std::min(a.q_per_seq, 64 / group);
  const uint32_t qbox[3] = {64, (uint32_t)group, (uint32_t)tpc};
  rc = make_tmap_3d_bf16(&tq, a.q, qdims, qstr, qbox);
  if (rc) return 1000 + rc;
  static std::atomic<uint64_t> attr_devs{0};
  if (const int e = smem_attr_once(attr_devs, (const void*)paged_attn_tc_kernel<D>, L::TOTAL)) return e;
  dim3 grid(a.num_seqs * a.Hkv * ((a.q_per_seq + tpc - 1) / tpc), splits);
  {
    const int pdl_rc = launch_pdl(paged_attn_tc_kernel<D>, dim3(grid), dim3(attn_tc::THREADS), L::TOTAL, st, tk, tv,
        tq, a, status);
    if (pdl_rc) return pdl_rc;
  }
  return (int)cudaGetLastError();
}

// The tcgen05 path serves bf16 decode / verify and prefill rows, dense (optionally a sliding window) or over a QSA
// block union, and NVFP4 KV dense or over a page union;
// returns -1 when the call is outside that set (the caller runs the mma.sync kernel), else the launch result.
int paged_attention_tc(const AttnArgs& a, int splits, uint32_t* status, cudaStream_t st) {
  if (a.impl == 1 || a.Hq / a.Hkv > 64) return -1;
  if (a.window > 0 && (a.sp_count || a.kscale)) return -1;  // windows: dense bf16 only
  if (a.kscale && (!a.vscale || (a.sp_count && a.sp_block != attn_tc::PAGE))) return -1;
  if (a.bt_row && a.sp_count && a.sp_block == attn_tc::PAGE) return -1;  // page unions are per sequence
  if (a.sp_count && (a.q_per_seq > 8 || a.sp_block < 1 || attn_tc::PAGE % a.sp_block)) return -1;
  if (a.D == 256) return launch_attn_tc<256>(a, splits, status, st);
  if (a.D == 128) return launch_attn_tc<128>(a, splits, status, st);
  return -1;
}

}  // namespace afb
