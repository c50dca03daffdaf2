// Variable-length causal attention for training (packed rows of segments), forward and backward, on the
// 5th-generation tensor cores: the student's attention in place of a library flash-attention.
//
// Layout: q [T, Hq, D], k / v [T, Hkv, D] bf16 (packed: segment s owns rows cu[s] .. cu[s+1]); a 64-position tile
// of one head is one 3-D TMA box {64 columns, 1 head, 64 positions}, i.e. 64 rows of 128 bytes per 64-column
// sub-tile, 128-byte swizzled, the K-major operand layout of tcgen05.mma.
//
//   forward  CTA (query head, 128-query tile): S = Q K^T (M 128, N 64) per 64-key tile into TMEM, four softmax
//            warps (TMEM lanes 0..127 = the query rows) with causal masking, lazy rescale of the running max, P as
//            bf16 back into TMEM, O += P V with P as the A operand from TMEM; writes O and the row log-sum-exp (log2).
//   dQ       CTA (query head, 64-query tile): per key tile S = Q K^T and dP = dO V^T into TMEM, the softmax warps
//            form dS = P (dP - delta) as bf16 in TMEM, dQ += dS K with K as an MN-major operand; dQ stays in TMEM.
//   dK / dV  CTA (query head, 128-key tile): walks every query row group at or after it; per unit S^T = K Q^T and
//            dP^T = V dO^T into TMEM, the epilogue warps (TMEM lanes = keys) form P^T and dS^T, dV += P^T dO and
//            dK += dS^T Q with dO / Q as MN-major operands, both resident in TMEM; each CTA writes its query head's
//            fp32 contribution, and a reduce kernel sums the heads of each KV group in a fixed order. With D = 256
//            the two accumulators do not fit TMEM together: dV and dK run as two launches.
// Every output element is produced by exactly one thread in a fixed order: no atomics, bitwise deterministic.
// Warp roles: 0 TMA loader (no multicast), 1 MMA issuer (+ TMEM); forward: 4-7 softmax (32 full rows each: the
// running max); dQ: 4, 5, 8, 9 epilogue (warps 4 and 8 share TMEM lanes 0..31, 5 and 9 lanes 32..63, each warp of a
// pair takes half of the 64 columns: no row-wide reduction is needed there); dK / dV: 4..11 epilogue (warp w the
// lanes of quadrant w & 3 = 32 keys, warps 4-7 and 8-11 the two halves of a unit's query columns).
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace afb {

namespace attn_tr {
constexpr int TILE = 64;
constexpr int THREADS = 256;
constexpr int THREADS_BWD = 320;  // dQ: warps 0..9, epilogue warps 4, 5, 8, 9
constexpr int THREADS_KV = 384;   // dK / dV: warps 0..11, epilogue warps 4..11
constexpr int W_LD = 0, W_MMA = 1, W_SM0 = 4;
AFB_DEV bool bwd_epi_warp(int w) { return w == 4 || w == 5 || w == 8 || w == 9; }
constexpr float RESCALE = 8.f;
constexpr uint32_t SUB = TILE * 128;  // 64 rows x 128 bytes: one swizzled 64-column sub-tile

template <int D>
struct Fwd {
  static constexpr int QT = 128;                              // query rows per CTA: the MMA's full M
  static constexpr uint32_t SUBQ = QT * 128;
  static constexpr uint32_t Q_BYTES = (D / 64) * SUBQ;
  static constexpr uint32_t KV_BYTES = (D / 64) * SUB;
  static constexpr int NS = D == 256 ? 2 : 6;
  static constexpr uint32_t STAGE = 2 * KV_BYTES;
  static constexpr uint32_t KV_OFF = Q_BYTES;
  static constexpr uint32_t BAR_OFF = KV_OFF + NS * STAGE;
  static constexpr uint32_t TOTAL = BAR_OFF + (2 * NS + 10) * 8 + 16 + 1024;
  static constexpr uint32_t O_COL = 0, S_COL = D, P_COL = D + 2 * TILE;
};

template <int D>
struct Dq {
  static constexpr uint32_t Q_BYTES = (D / 64) * SUB;
  static constexpr uint32_t KV_BYTES = (D / 64) * SUB;
  static constexpr int NS = D == 256 ? 2 : 4;
  static constexpr uint32_t STAGE = 2 * KV_BYTES;
  static constexpr uint32_t DO_OFF = Q_BYTES;
  static constexpr uint32_t KV_OFF = 2 * Q_BYTES;
  static constexpr uint32_t BAR_OFF = KV_OFF + NS * STAGE;
  static constexpr uint32_t TOTAL = BAR_OFF + (2 * NS + 10) * 8 + 16 + 1024;
  static constexpr uint32_t DQ_COL = 0, S_COL = D, DP_COL = D + TILE, DS_COL = D + 2 * TILE;  // dS: [2][32]
  static_assert(DS_COL + TILE <= 512, "TMEM columns");
};

template <int D, int MODE>  // MODE bit 0: dV, bit 1: dK
struct Dkv {
  static constexpr bool DV = MODE & 1, DK = MODE & 2;
  static constexpr int KT = 128;                              // keys per CTA: the MMA's full M
  static constexpr int QU = (D == 256 && DK) ? 32 : 64;       // query rows per unit (the N of S^T)
  static constexpr bool HAS_V = DK;                           // V is read only for dP^T
  static constexpr uint32_t KSUB = KT * 128;                  // one 128-key x 64-column sub-tile
  static constexpr uint32_t QSUB = QU * 128;
  static constexpr uint32_t T_BYTES = (D / 64) * KSUB;
  static constexpr uint32_t K_OFF = 0, V_OFF = T_BYTES;
  static constexpr int NS = 2;
  static constexpr uint32_t U_BYTES = (D / 64) * QSUB;        // Q (or dO) rows of one unit
  static constexpr uint32_t STAGE = 2 * U_BYTES;              // Q + dO
  static constexpr uint32_t ST_OFF = (HAS_V ? 2 : 1) * T_BYTES;
  static constexpr uint32_t ROWS_OFF = ST_OFF + NS * STAGE;   // lse[NS][QU], delta[NS][QU], qsa field[NS][QU]
  static constexpr uint32_t BAR_OFF = ROWS_OFF + NS * 3 * QU * 4;
  static constexpr uint32_t TOTAL = BAR_OFF + (2 * NS + 10) * 8 + 16 + 1024;
  static constexpr uint32_t DV_COL = 0;
  static constexpr uint32_t DK_COL = DV ? D : 0;
  static constexpr uint32_t S_COL = (DV ? D : 0) + (DK ? D : 0);
  static constexpr uint32_t DP_COL = S_COL + QU;                   // dK only
  static constexpr uint32_t PT_COL = S_COL + (DK ? 2 : 1) * QU;    // P^T bf16 pairs [2][QU / 2] (dV)
  static constexpr uint32_t DS_COL = PT_COL + (DV ? QU : 0);       // dS^T [2][QU / 2] (dK)
  static constexpr uint32_t END = DS_COL + (DK ? QU : 0);
  static_assert(END <= 512, "TMEM columns");
  static_assert(TOTAL <= 232448, "shared memory");
};
}  // namespace attn_tr

// QSA: the 64 keys of key tile kt that row `row` may see by its block selection (bit j = key kt * 64 + j); all
// ones without a map. Blocks of B tokens: the tile's 64 / B blocks are one aligned bit field of one map word.
AFB_DEV uint64_t qsa_key_mask(const AttnTrainArgs& a, size_t row, int kt) {
  if (!a.blkmap) return ~0ull;
  const int B = a.qsa_block, bpt = attn_tr::TILE / B, b0 = kt * bpt;
  const uint32_t w = a.blkmap[row * a.blk_words + (b0 >> 5)];
  const uint32_t f = (w >> (b0 & 31)) & (bpt == 32 ? 0xffffffffu : ((1u << bpt) - 1u));
  uint64_t m = 0;
  for (int b = 0; b < bpt; ++b)
    if ((f >> b) & 1u) m |= (B == 64 ? ~0ull : ((1ull << B) - 1ull)) << (b * B);
  return m;
}

// ---------------------------------------------------------------------------------------------------- forward
template <int D>
__global__ void __launch_bounds__(attn_tr::THREADS, 1)
    attn_train_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, AttnTrainArgs a, uint32_t* status) {
  using namespace attn_tr;
  using L = Fwd<D>;
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
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_fin + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qh = blockIdx.x, kvh = qh / (a.Hq / a.Hkv);
  const int2 tl = a.tiles[blockIdx.y];
  const int s0 = a.cu[tl.x], Lseg = a.cu[tl.x + 1] - s0, q0 = tl.y;
  const int QR = min(L::QT, Lseg - q0);
  // key tiles 0 .. n-1: up to the last query row (causal) or the whole segment (bidirectional)
  const int n = ((a.causal ? q0 + QR : Lseg) + TILE - 1) / TILE;
  const int klim_off = a.causal ? 0 : Lseg;  // bidirectional: keys below the segment end, whatever the row
  if (QR <= 0) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 4);
      mbar_init(&p_full[b], 4);
      mbar_init(&o_done[b], 1);
    }
    mbar_init(q_ready, 1);
    mbar_init(mma_fin, 1);
    fence_mbar_init();
  }
  if (warp == W_MMA) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == W_LD) {
    if (lane == 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_ready, L::Q_BYTES);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) tma_load_3d(smem + c * L::SUBQ, &tmQ, q_ready, c * 64, qh, s0 + q0);
      int issued = 0;
      for (int i = 0; i < n; ++i) {
        const int s = i % NS;
        if (i >= NS && !mbar_wait(&kv_empty[s], ((i / NS) & 1) ^ 1, status)) break;
        uint8_t* st = smem + L::KV_OFF + s * L::STAGE;
        mbar_arrive_expect_tx(&kv_full[s], L::STAGE);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_3d(st + c * SUB, &tmK, &kv_full[s], c * 64, kvh, s0 + i * TILE);
          tma_load_3d(st + L::KV_BYTES + c * SUB, &tmV, &kv_full[s], c * 64, kvh, s0 + i * TILE);
        }
        ++issued;
      }
      mbar_wait(q_ready, 0, status);
      for (int i = max(0, issued - NS); i < issued; ++i) mbar_wait(&kv_full[i % NS], (i / NS) & 1, status);
    }
  } else if (warp == W_MMA) {
    constexpr uint32_t idesc_s = idesc_f16(128, TILE, 1);
    constexpr uint32_t idesc_o = idesc_f16(128, D, 1) | (1u << 16);  // B (V) MN-major
    ok = __all_sync(0xffffffffu, mbar_wait(q_ready, 0, status));
    tc_fence_after();
    const uint32_t q_base = smem_u32(smem);
    auto issue_pv = [&](int j) {
      const int sb = j & 1, s = j % NS;
      if (!__all_sync(0xffffffffu, mbar_wait(&p_full[sb], (j >> 1) & 1, status))) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t v_base = smem_u32(smem + L::KV_OFF + s * L::STAGE + L::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < TILE / 16; ++kk)
          umma_f16_ta(tmem + L::O_COL, tmem + L::P_COL + sb * (TILE / 2) + kk * 8,
                      sw128_desc_mn(v_base + kk * 16 * 128, SUB, 1024), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
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
          const uint32_t off = (kk >> 2) * SUB + (kk & 3) * 32;
          umma_f16(tmem + L::S_COL + sb * TILE, sw128_desc(q_base + (kk >> 2) * L::SUBQ + (kk & 3) * 32),
                   sw128_desc(k_base + off), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
      }
      __syncwarp();
      if (i >= 1 && !issue_pv(i - 1)) {
        ok = false;
        break;
      }
    }
    if (ok) issue_pv(n - 1);
    if (lane == 0) umma_commit(mma_fin);
    __syncwarp();
    mbar_wait(mma_fin, 0, status);
  } else if (warp >= W_SM0 && warp < W_SM0 + 4) {
    const int quad = warp - W_SM0;
    const int r = quad * 32 + lane;
    const bool live = r < QR;
    const int qpos = q0 + r;
    const int kmax = klim_off ? klim_off - 1 : qpos;  // last visible key position
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    float m = -INFINITY, l = 0.f;
    for (int i = 0; i < n; ++i) {
      const int sb = i & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[sb], (i >> 1) & 1, status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[TILE];
      tmem_ld32(lane_base + L::S_COL + sb * TILE, sv);
      tmem_ld32(lane_base + L::S_COL + sb * TILE + 32, sv + 32);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);
      const int kbase = i * TILE;
      const uint64_t km = live ? qsa_key_mask(a, (size_t)(s0 + qpos), i) : 0ull;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < TILE; ++j) {
        const float x = (live && kbase + j <= kmax && ((km >> j) & 1ull)) ? sv[j] * a.scale_log2 : -INFINITY;
        sv[j] = x;
        mx = fmaxf(mx, x);
      }
      float mnew = m;
      if (mx > m + RESCALE || m == -INFINITY) mnew = mx;
      const bool rescale = m != -INFINITY && mnew != m;
      if (__any_sync(0xffffffffu, rescale)) {
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
      uint32_t pk[TILE / 2];
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < TILE / 2; ++j) {
        const float e0 = exp2f(sv[2 * j] - base), e1 = exp2f(sv[2 * j + 1] - base);
        rs += e0 + e1;
        pk[j] = pack_bf16x2(e0, e1);
      }
      l += rs;
      if (i >= 2 && !__all_sync(0xffffffffu, mbar_wait(&o_done[sb], ((i - 2) >> 1) & 1, status))) {
        ok = false;
        break;
      }
      tmem_st32(lane_base + L::P_COL + sb * (TILE / 2), pk);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(&o_done[(n - 1) & 1], ((n - 1) >> 1) & 1, status))) {
      tc_fence_after();
      const size_t row = (size_t)(s0 + qpos);
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        float ov[32];
        tmem_ld32(lane_base + L::O_COL + c, ov);
        tmem_ld_wait();
        if (!live) continue;
        __nv_bfloat16* op = a.out + (row * a.Hq + qh) * D + c;
#pragma unroll
        for (int j = 0; j < 32; j += 8)
          *reinterpret_cast<uint4*>(op + j) =
              make_uint4(pack_bf16x2(ov[j] * inv, ov[j + 1] * inv), pack_bf16x2(ov[j + 2] * inv, ov[j + 3] * inv),
                         pack_bf16x2(ov[j + 4] * inv, ov[j + 5] * inv), pack_bf16x2(ov[j + 6] * inv, ov[j + 7] * inv));
      }
      if (live) a.lse[(size_t)qh * a.T + row] = l > 0.f ? m + log2f(l) : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == W_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------------------------------- dQ
template <int D>
__global__ void __launch_bounds__(attn_tr::THREADS_BWD, 1)
    attn_train_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                         const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                         AttnTrainArgs a, uint32_t* status) {
  using namespace attn_tr;
  using L = Dq<D>;
  constexpr int NS = L::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* kv_empty = kv_full + NS;
  uint64_t* sd_full = kv_empty + NS;  // S and dP of a key tile are in TMEM
  uint64_t* sd_empty = sd_full + 1;   // the softmax warps have read them
  uint64_t* ds_full = sd_empty + 1;   // [2] dS written
  uint64_t* ds_done = ds_full + 2;    // [2] the dQ MMA that read it completed
  uint64_t* q_ready = ds_done + 2;
  uint64_t* mma_fin = q_ready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_fin + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qh = blockIdx.x, kvh = qh / (a.Hq / a.Hkv);
  const int2 tl = a.tiles[blockIdx.y];
  const int s0 = a.cu[tl.x], Lseg = a.cu[tl.x + 1] - s0, q0 = tl.y;
  const int QR = min(TILE, Lseg - q0);
  const int n = (q0 + QR + TILE - 1) / TILE;
  if (QR <= 0) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(sd_full, 1);
    mbar_init(sd_empty, 4);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ds_full[b], 4);
      mbar_init(&ds_done[b], 1);
    }
    mbar_init(q_ready, 1);
    mbar_init(mma_fin, 1);
    fence_mbar_init();
  }
  if (warp == W_MMA) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == W_LD) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_ready, 2 * L::Q_BYTES);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_3d(smem + c * SUB, &tmQ, q_ready, c * 64, qh, s0 + q0);
        tma_load_3d(smem + L::DO_OFF + c * SUB, &tmDO, q_ready, c * 64, qh, s0 + q0);
      }
      int issued = 0;
      for (int i = 0; i < n; ++i) {
        const int s = i % NS;
        if (i >= NS && !mbar_wait(&kv_empty[s], ((i / NS) & 1) ^ 1, status)) break;
        uint8_t* st = smem + L::KV_OFF + s * L::STAGE;
        mbar_arrive_expect_tx(&kv_full[s], L::STAGE);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_3d(st + c * SUB, &tmK, &kv_full[s], c * 64, kvh, s0 + i * TILE);
          tma_load_3d(st + L::KV_BYTES + c * SUB, &tmV, &kv_full[s], c * 64, kvh, s0 + i * TILE);
        }
        ++issued;
      }
      mbar_wait(q_ready, 0, status);
      for (int i = max(0, issued - NS); i < issued; ++i) mbar_wait(&kv_full[i % NS], (i / NS) & 1, status);
    }
  } else if (warp == W_MMA) {
    constexpr uint32_t idesc_s = idesc_f16(128, TILE, 1);
    constexpr uint32_t idesc_q = idesc_f16(128, D, 1) | (1u << 16);  // B (K) MN-major
    ok = __all_sync(0xffffffffu, mbar_wait(q_ready, 0, status));
    tc_fence_after();
    const uint32_t q_base = smem_u32(smem), do_base = smem_u32(smem + L::DO_OFF);
    auto issue_dq = [&](int j) {  // dQ += dS_j K_j
      const int b = j & 1, s = j % NS;
      if (!__all_sync(0xffffffffu, mbar_wait(&ds_full[b], (j >> 1) & 1, status))) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t k_base = smem_u32(smem + L::KV_OFF + s * L::STAGE);
#pragma unroll
        for (int kk = 0; kk < TILE / 16; ++kk)
          umma_f16_ta(tmem + L::DQ_COL, tmem + L::DS_COL + b * (TILE / 2) + kk * 8,
                      sw128_desc_mn(k_base + kk * 16 * 128, SUB, 1024), idesc_q, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&ds_done[b]);
        umma_commit(&kv_empty[s]);
      }
      __syncwarp();
      return true;
    };
    for (int i = 0; i < n && ok; ++i) {
      const int s = i % NS;
      if (!__all_sync(0xffffffffu, mbar_wait(&kv_full[s], (i / NS) & 1, status)) ||
          (i >= 1 && !__all_sync(0xffffffffu, mbar_wait(sd_empty, (i - 1) & 1, status)))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t k_base = smem_u32(smem + L::KV_OFF + s * L::STAGE);
        const uint32_t v_base = k_base + L::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * SUB + (kk & 3) * 32;
          umma_f16(tmem + L::S_COL, sw128_desc(q_base + off), sw128_desc(k_base + off), idesc_s, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * SUB + (kk & 3) * 32;
          umma_f16(tmem + L::DP_COL, sw128_desc(do_base + off), sw128_desc(v_base + off), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(sd_full);
      }
      __syncwarp();
      if (i >= 1 && !issue_dq(i - 1)) {
        ok = false;
        break;
      }
    }
    if (ok) issue_dq(n - 1);
    if (lane == 0) umma_commit(mma_fin);
    __syncwarp();
    mbar_wait(mma_fin, 0, status);
  } else if (bwd_epi_warp(warp)) {
    const int quad = warp & 1, half = warp >= 8;  // TMEM lane quadrant, column half
    const int r = quad * 32 + lane;
    const bool live = r < QR;
    const int qpos = q0 + r;
    const size_t row = (size_t)(s0 + qpos);
    const float lse = live ? a.lse[(size_t)qh * a.T + row] : 0.f;
    const float dlt = live ? a.delta[(size_t)qh * a.T + row] : 0.f;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    for (int i = 0; i < n; ++i) {
      const int b = i & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(sd_full, i & 1, status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[32], dp[32];
      tmem_ld32(lane_base + L::S_COL + half * 32, sv);
      tmem_ld32(lane_base + L::DP_COL + half * 32, dp);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sd_empty);
      const int kbase = i * TILE + half * 32;
      const uint32_t km = live ? (uint32_t)(qsa_key_mask(a, row, i) >> (half * 32)) : 0u;
      uint32_t pk[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float d2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int jj = 2 * j + e;
          const float p = (live && kbase + jj <= qpos && ((km >> jj) & 1u)) ? exp2f(sv[jj] * a.scale_log2 - lse) : 0.f;
          d2[e] = p * (dp[jj] - dlt);
        }
        pk[j] = pack_bf16x2(d2[0], d2[1]);
      }
      if (i >= 2 && !__all_sync(0xffffffffu, mbar_wait(&ds_done[b], ((i - 2) >> 1) & 1, status))) {
        ok = false;
        break;
      }
      tmem_st16(lane_base + L::DS_COL + b * (TILE / 2) + half * 16, pk);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[b]);
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(&ds_done[(n - 1) & 1], ((n - 1) >> 1) & 1, status))) {
      tc_fence_after();
#pragma unroll 1
      for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 32) {
        float v[32];
        tmem_ld32(lane_base + L::DQ_COL + c, v);
        tmem_ld_wait();
        if (!live) continue;
        __nv_bfloat16* op = a.dq + (row * a.Hq + qh) * D + c;
#pragma unroll
        for (int j = 0; j < 32; j += 8)
          *reinterpret_cast<uint4*>(op + j) = make_uint4(
              pack_bf16x2(v[j] * a.scale, v[j + 1] * a.scale), pack_bf16x2(v[j + 2] * a.scale, v[j + 3] * a.scale),
              pack_bf16x2(v[j + 4] * a.scale, v[j + 5] * a.scale), pack_bf16x2(v[j + 6] * a.scale, v[j + 7] * a.scale));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == W_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------------------------------- dK / dV
template <int D, int MODE>
__global__ void __launch_bounds__(attn_tr::THREADS_KV, 1)
    attn_train_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                           const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                           AttnTrainArgs a, uint32_t* status) {
  using namespace attn_tr;
  using L = Dkv<D, MODE>;
  constexpr int NS = L::NS, KT = L::KT, QU = L::QU;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* st_full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);  // [NS] Q + dO (+ rows) of a unit landed
  uint64_t* st_empty = st_full + NS;                                     // [NS] its accumulate MMAs completed
  uint64_t* sx_full = st_empty + NS;   // S^T (and dP^T) in TMEM
  uint64_t* sx_empty = sx_full + 1;    // the epilogue warps have read them
  uint64_t* pt_full = sx_empty + 1;    // [2] P^T / dS^T written
  uint64_t* pt_done = pt_full + 2;     // [2] the accumulate MMAs that read them completed
  uint64_t* kv_ready = pt_done + 2;
  uint64_t* mma_fin = kv_ready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_fin + 1);
  float* rows_lse = reinterpret_cast<float*>(smem + L::ROWS_OFF);            // [NS][QU]
  float* rows_dlt = rows_lse + NS * QU;                                        // [NS][QU]
  uint32_t* rows_map = reinterpret_cast<uint32_t*>(rows_dlt + NS * QU);       // [NS][QU]: the key tile's block bits

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qh = blockIdx.x, kvh = qh / (a.Hq / a.Hkv);
  const int2 tl = a.tiles[blockIdx.y];
  const int s0 = a.cu[tl.x], Lseg = a.cu[tl.x + 1] - s0, k0 = tl.y;
  const int KR = min(KT, Lseg - k0);
  const int nq = (Lseg + QU - 1) / QU, qt0 = k0 / QU;
  const int U = nq - qt0;  // units: the query row groups at or after this key tile
  if (KR <= 0 || U <= 0) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&st_full[s], 1);
      mbar_init(&st_empty[s], 1);
    }
    mbar_init(sx_full, 1);
    mbar_init(sx_empty, 8);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pt_full[b], 8);
      mbar_init(&pt_done[b], 1);
    }
    mbar_init(kv_ready, 1);
    mbar_init(mma_fin, 1);
    fence_mbar_init();
  }
  if (warp == W_MMA) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == W_LD) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_ready, (L::HAS_V ? 2 : 1) * L::T_BYTES);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_3d(smem + L::K_OFF + c * L::KSUB, &tmK, kv_ready, c * 64, kvh, s0 + k0);
        if (L::HAS_V) tma_load_3d(smem + L::V_OFF + c * L::KSUB, &tmV, kv_ready, c * 64, kvh, s0 + k0);
      }
    }
    int issued = 0;
    const int bpt = a.blkmap ? KT / a.qsa_block : 0, b0 = a.blkmap ? (k0 / a.qsa_block) : 0;
    for (int u = 0; u < U && ok; ++u) {
      const int s = u % NS;
      const int q0 = (qt0 + u) * QU;
      if (u >= NS && !__all_sync(0xffffffffu, mbar_wait(&st_empty[s], ((u / NS) & 1) ^ 1, status))) {
        ok = false;
        break;
      }
      // the unit's row statistics and QSA fields (plain loads; published by lane 0's arrive below)
      for (int r = lane; r < QU; r += 32) {
        const bool in = q0 + r < Lseg;
        const size_t idx = (size_t)qh * a.T + s0 + q0 + r;
        rows_lse[s * QU + r] = in ? a.lse[idx] : 0.f;
        rows_dlt[s * QU + r] = in ? a.delta[idx] : 0.f;
        uint32_t f = 0xffffffffu;
        if (a.blkmap && in) {  // this key tile's KT / B block bits of the row (one aligned field of one word)
          const uint32_t w = a.blkmap[(size_t)(s0 + q0 + r) * a.blk_words + (b0 >> 5)];
          f = bpt >= 32 ? w : (w >> (b0 & 31));
        }
        rows_map[s * QU + r] = f;
      }
      __syncwarp();
      if (lane == 0) {
        uint8_t* st = smem + L::ST_OFF + s * L::STAGE;
        mbar_arrive_expect_tx(&st_full[s], L::STAGE);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_3d(st + c * L::QSUB, &tmQ, &st_full[s], c * 64, qh, s0 + q0);
          tma_load_3d(st + L::U_BYTES + c * L::QSUB, &tmDO, &st_full[s], c * 64, qh, s0 + q0);
        }
      }
      __syncwarp();
      ++issued;
    }
    if (lane == 0) {
      mbar_wait(kv_ready, 0, status);
      for (int u = max(0, issued - NS); u < issued; ++u) mbar_wait(&st_full[u % NS], (u / NS) & 1, status);
    }
  } else if (warp == W_MMA) {
    constexpr uint32_t idesc_s = idesc_f16(128, QU, 1);             // S^T = K Q^T, dP^T = V dO^T
    constexpr uint32_t idesc_acc = idesc_f16(128, D, 1) | (1u << 16); // dV += P^T dO, dK += dS^T Q (B MN-major)
    ok = __all_sync(0xffffffffu, mbar_wait(kv_ready, 0, status));
    tc_fence_after();
    const uint32_t k_base = smem_u32(smem + L::K_OFF), v_base = smem_u32(smem + L::V_OFF);
    auto issue_acc = [&](int j) {
      const int b = j & 1, s = j % NS;
      if (!__all_sync(0xffffffffu, mbar_wait(&pt_full[b], (j >> 1) & 1, status))) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t q_base = smem_u32(smem + L::ST_OFF + s * L::STAGE);
        const uint32_t do_base = q_base + L::U_BYTES;
#pragma unroll
        for (int kk = 0; kk < QU / 16; ++kk) {
          if (L::DV)
            umma_f16_ta(tmem + L::DV_COL, tmem + L::PT_COL + b * (QU / 2) + kk * 8,
                        sw128_desc_mn(do_base + kk * 16 * 128, L::QSUB, 1024), idesc_acc,
                        (j > 0 || kk > 0) ? 1u : 0u);
          if (L::DK)
            umma_f16_ta(tmem + L::DK_COL, tmem + L::DS_COL + b * (QU / 2) + kk * 8,
                        sw128_desc_mn(q_base + kk * 16 * 128, L::QSUB, 1024), idesc_acc,
                        (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&pt_done[b]);
        umma_commit(&st_empty[s]);
      }
      __syncwarp();
      return true;
    };
    for (int u = 0; u < U && ok; ++u) {
      const int s = u % NS;
      if (!__all_sync(0xffffffffu, mbar_wait(&st_full[s], (u / NS) & 1, status)) ||
          (u >= 1 && !__all_sync(0xffffffffu, mbar_wait(sx_empty, (u - 1) & 1, status)))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t q_base = smem_u32(smem + L::ST_OFF + s * L::STAGE);
        const uint32_t do_base = q_base + L::U_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(tmem + L::S_COL, sw128_desc(k_base + (kk >> 2) * L::KSUB + (kk & 3) * 32),
                   sw128_desc(q_base + (kk >> 2) * L::QSUB + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
        if (L::DK) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16(tmem + L::DP_COL, sw128_desc(v_base + (kk >> 2) * L::KSUB + (kk & 3) * 32),
                     sw128_desc(do_base + (kk >> 2) * L::QSUB + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(sx_full);
      }
      __syncwarp();
      if (u >= 1 && !issue_acc(u - 1)) {
        ok = false;
        break;
      }
    }
    if (ok) issue_acc(U - 1);
    if (lane == 0) umma_commit(mma_fin);
    __syncwarp();
    mbar_wait(mma_fin, 0, status);
  } else if (warp >= 4 && warp < 12) {
    // epilogue: warp w owns TMEM lanes (w & 3) * 32 .. + 31 (keys) and half of the unit's QU columns
    constexpr int HC = QU / 2;  // columns per warp
    const int quad = warp & 3, half = warp >= 8;
    const int kr = quad * 32 + lane;
    const bool klive = kr < KR;
    const int kpos = k0 + kr;
    const int kblk = a.blkmap ? kr / a.qsa_block : 0;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    for (int u = 0; u < U; ++u) {
      const int b = u & 1, s = u % NS;
      const int q0 = (qt0 + u) * QU + half * HC;  // this warp's HC query columns
      if (!__all_sync(0xffffffffu, mbar_wait(sx_full, u & 1, status)) ||
          !__all_sync(0xffffffffu, mbar_wait(&st_full[s], (u / NS) & 1, status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[HC], dp[L::DK ? HC : 1];
      if constexpr (HC == 32) {
        tmem_ld32(lane_base + L::S_COL + half * HC, sv);
        if (L::DK) tmem_ld32(lane_base + L::DP_COL + half * HC, dp);
      } else {
        tmem_ld16(lane_base + L::S_COL + half * HC, sv);
        if (L::DK) tmem_ld16(lane_base + L::DP_COL + half * HC, dp);
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sx_empty);
      const float* lse = rows_lse + s * QU + half * HC;
      const float* dlt = rows_dlt + s * QU + half * HC;
      const uint32_t* fmap = rows_map + s * QU + half * HC;
      uint32_t ppk[L::DV ? HC / 2 : 1], dpk[L::DK ? HC / 2 : 1];
#pragma unroll
      for (int j = 0; j < HC / 2; ++j) {
        float pv[2], dv2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int c = 2 * j + e, qpos = q0 + c;
          const bool sel = ((fmap[c] >> kblk) & 1u) != 0u;
          const float p =
              (klive && kpos <= qpos && qpos < Lseg && sel) ? exp2f(sv[c] * a.scale_log2 - lse[c]) : 0.f;
          pv[e] = p;
          if (L::DK) dv2[e] = p * (dp[c] - dlt[c]);
        }
        if (L::DV) ppk[j] = pack_bf16x2(pv[0], pv[1]);
        if (L::DK) dpk[j] = pack_bf16x2(dv2[0], dv2[1]);
      }
      if (u >= 2 && !__all_sync(0xffffffffu, mbar_wait(&pt_done[b], ((u - 2) >> 1) & 1, status))) {
        ok = false;
        break;
      }
      if constexpr (HC == 32) {
        if (L::DV) tmem_st16(lane_base + L::PT_COL + b * (QU / 2) + half * (HC / 2), ppk);
        if (L::DK) tmem_st16(lane_base + L::DS_COL + b * (QU / 2) + half * (HC / 2), dpk);
      } else {
        if (L::DV) tmem_st8(lane_base + L::PT_COL + b * (QU / 2) + half * (HC / 2), ppk);
        if (L::DK) tmem_st8(lane_base + L::DS_COL + b * (QU / 2) + half * (HC / 2), dpk);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pt_full[b]);
    }
    // this query head's contribution, fp32 (the reduce kernel sums the group's heads in order)
    if (ok && __all_sync(0xffffffffu, mbar_wait(&pt_done[(U - 1) & 1], ((U - 1) >> 1) & 1, status))) {
      tc_fence_after();
      const size_t row = (size_t)(s0 + kpos);
#pragma unroll 1
      for (int pass = 0; pass < 2; ++pass) {
        if ((pass == 0 && !L::DV) || (pass == 1 && !L::DK)) continue;
        const uint32_t col = pass == 0 ? L::DV_COL : L::DK_COL;
        float* dst = pass == 0 ? a.dv_part : a.dk_part;
#pragma unroll 1
        for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 32) {
          float v[32];
          tmem_ld32(lane_base + col + c, v);
          tmem_ld_wait();
          if (!klive) continue;
          float* op = dst + (row * a.Hq + qh) * D + c;
#pragma unroll
          for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(op + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == W_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dK / dV of every (t, KV head): the group's per-head fp32 contributions summed in head order (dK times the
// softmax scale), bf16. One thread per 4 elements.
__global__ void attn_train_dkdv_reduce_kernel(const float* __restrict__ dk_part, const float* __restrict__ dv_part,
                                              __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv,
                                              int T, int Hq, int Hkv, int D, float scale) {
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i >= (int64_t)T * Hkv * D) return;
  const int d = (int)(i % D);
  const int64_t th = i / D;
  const int kvh = (int)(th % Hkv);
  const int64_t t = th / Hkv;
  const int group = Hq / Hkv;
  float4 sk = make_float4(0.f, 0.f, 0.f, 0.f), sv = sk;
  for (int g = 0; g < group; ++g) {
    const size_t o = ((size_t)t * Hq + kvh * group + g) * D + d;
    const float4 x = *reinterpret_cast<const float4*>(dk_part + o), y = *reinterpret_cast<const float4*>(dv_part + o);
    sk.x += x.x;
    sk.y += x.y;
    sk.z += x.z;
    sk.w += x.w;
    sv.x += y.x;
    sv.y += y.y;
    sv.z += y.z;
    sv.w += y.w;
  }
  *reinterpret_cast<uint2*>(dk + i) = make_uint2(pack_bf16x2(sk.x * scale, sk.y * scale), pack_bf16x2(sk.z * scale, sk.w * scale));
  *reinterpret_cast<uint2*>(dv + i) = make_uint2(pack_bf16x2(sv.x, sv.y), pack_bf16x2(sv.z, sv.w));
}

// delta[h, t] = sum_d dO[t, h, d] * O[t, h, d] (fp32): one warp per (t, h)
__global__ void attn_train_delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                        float* __restrict__ delta, int T, int Hq, int D) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (int64_t)T * Hq) return;
  const int t = (int)(w / Hq), h = (int)(w % Hq);
  const __nv_bfloat16* op = o + w * D;
  const __nv_bfloat16* dp = dout + w * D;
  float acc = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    const uint4 x = *reinterpret_cast<const uint4*>(op + c), y = *reinterpret_cast<const uint4*>(dp + c);
    const __nv_bfloat162* xa = reinterpret_cast<const __nv_bfloat162*>(&x);
    const __nv_bfloat162* ya = reinterpret_cast<const __nv_bfloat162*>(&y);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 xf = __bfloat1622float2(xa[i]), yf = __bfloat1622float2(ya[i]);
      acc += xf.x * yf.x + xf.y * yf.y;
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) delta[(size_t)h * T + t] = acc;
}

// ---------------------------------------------------------------------------------------------------- launchers
static int qkv_maps(const AttnTrainArgs& a, CUtensorMap* tq, CUtensorMap* tk, CUtensorMap* tv, CUtensorMap* tdo,
                    int q_rows = attn_tr::TILE) {
  const uint64_t qd[3] = {(uint64_t)a.D, (uint64_t)a.Hq, (uint64_t)a.T};
  const uint64_t qs[2] = {(uint64_t)a.D * 2, (uint64_t)a.Hq * a.D * 2};
  const uint64_t kd[3] = {(uint64_t)a.D, (uint64_t)a.Hkv, (uint64_t)a.T};
  const uint64_t ks[2] = {(uint64_t)a.D * 2, (uint64_t)a.Hkv * a.D * 2};
  const uint32_t box[3] = {64, 1, (uint32_t)attn_tr::TILE};
  const uint32_t qbox[3] = {64, 1, (uint32_t)q_rows};
  int rc = make_tmap_3d_bf16(tq, a.q, qd, qs, qbox);
  if (!rc) rc = make_tmap_3d_bf16(tk, a.k, kd, ks, box);
  if (!rc) rc = make_tmap_3d_bf16(tv, a.v, kd, ks, box);
  if (!rc && tdo) rc = make_tmap_3d_bf16(tdo, a.dout, qd, qs, box);
  return rc ? 1000 + rc : 0;
}

static int check_args(const AttnTrainArgs& a) {
  if ((a.D != 128 && a.D != 256) || a.Hkv < 1 || a.Hq % a.Hkv || a.T < 1 || !a.cu || !a.tiles) return 3;
  if (a.blkmap && (a.qsa_block < 4 || attn_tr::TILE % a.qsa_block || a.blk_words < 1)) return 3;
  return 0;
}

// QSA row map from the per-set unions: one thread per (set, union entry), OR-ing the entry's block into the bitmap
// row of every real row its mask names (distinct bits: the result does not depend on the order)
__global__ void qsa_rowmap_kernel(const int* __restrict__ u_lpage, const uint8_t* __restrict__ u_mask,
                                  const int* __restrict__ u_count, const int* __restrict__ set_row0,
                                  const int* __restrict__ set_rows, int S, int W, int ucap, uint32_t* blkmap,
                                  int words) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)S * ucap) return;
  const int s = (int)(i / ucap), e = (int)(i % ucap);
  if (e >= u_count[s]) return;
  const int b = u_lpage[i];
  const uint32_t m = u_mask[i];
  if (b < 0 || (b >> 5) >= words) return;
  for (int r = 0; r < min(W, set_rows[s]); ++r)
    if ((m >> r) & 1u) atomicOr(&blkmap[(size_t)(set_row0[s] + r) * words + (b >> 5)], 1u << (b & 31));
}

int qsa_rowmap(const int* u_lpage, const uint8_t* u_mask, const int* u_count, const int* set_row0,
               const int* set_rows, int S, int W, int ucap, uint32_t* blkmap, int words, cudaStream_t st) {
  if (S <= 0) return 0;
  if (W < 1 || W > 8 || ucap < 1 || words < 1) return 3;
  const int64_t n = (int64_t)S * ucap;
  qsa_rowmap_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(u_lpage, u_mask, u_count, set_row0, set_rows, S, W,
                                                                 ucap, blkmap, words);
  return (int)cudaGetLastError();
}

template <int D>
static int launch_fwd(const AttnTrainArgs& a, uint32_t* status, cudaStream_t st) {
  using L = attn_tr::Fwd<D>;
  CUtensorMap tq{}, tk{}, tv{};
  if (const int rc = qkv_maps(a, &tq, &tk, &tv, nullptr, L::QT)) return rc;
  static std::atomic<uint64_t> devs{0};
  if (const int e = smem_attr_once(devs, (const void*)attn_train_fwd_kernel<D>, L::TOTAL)) return e;
  attn_train_fwd_kernel<D><<<dim3(a.Hq, a.ntiles), attn_tr::THREADS, L::TOTAL, st>>>(tq, tk, tv, a, status);
  return (int)cudaGetLastError();
}

// a.tiles: 128-position query tiles (the backward's are 64-position tiles)
int attn_train_fwd(const AttnTrainArgs& a, uint32_t* status, cudaStream_t st) {
  if (const int e = check_args(a)) return e;
  if (!a.causal && a.blkmap) return 3;  // QSA maps are causal selections
  if (a.ntiles == 0) return 0;
  return a.D == 256 ? launch_fwd<256>(a, status, st) : launch_fwd<128>(a, status, st);
}

// dK / dV: 128-key tiles (kv_tiles lists them) and QU-row query units
template <int D, int MODE>
static int launch_dkdv(const AttnTrainArgs& a, uint32_t* status, cudaStream_t st) {
  using L = attn_tr::Dkv<D, MODE>;
  CUtensorMap tq{}, tk{}, tv{}, tdo{};
  const uint64_t qd[3] = {(uint64_t)a.D, (uint64_t)a.Hq, (uint64_t)a.T};
  const uint64_t qs[2] = {(uint64_t)a.D * 2, (uint64_t)a.Hq * a.D * 2};
  const uint64_t kd[3] = {(uint64_t)a.D, (uint64_t)a.Hkv, (uint64_t)a.T};
  const uint64_t ks[2] = {(uint64_t)a.D * 2, (uint64_t)a.Hkv * a.D * 2};
  const uint32_t kbox[3] = {64, 1, (uint32_t)L::KT}, qbox[3] = {64, 1, (uint32_t)L::QU};
  int rc = make_tmap_3d_bf16(&tq, a.q, qd, qs, qbox);
  if (!rc) rc = make_tmap_3d_bf16(&tdo, a.dout, qd, qs, qbox);
  if (!rc) rc = make_tmap_3d_bf16(&tk, a.k, kd, ks, kbox);
  if (!rc) rc = make_tmap_3d_bf16(&tv, a.v, kd, ks, kbox);
  if (rc) return 1000 + rc;
  static std::atomic<uint64_t> devs{0};
  if (const int e = smem_attr_once(devs, (const void*)attn_train_dkdv_kernel<D, MODE>, L::TOTAL)) return e;
  attn_train_dkdv_kernel<D, MODE><<<dim3(a.Hq, a.ntiles), attn_tr::THREADS_KV, L::TOTAL, st>>>(tq, tdo, tk, tv, a,
                                                                                             status);
  return (int)cudaGetLastError();
}

template <int D>
static int launch_bwd(const AttnTrainArgs& a, const int2* kv_tiles, int nkv, uint32_t* status, cudaStream_t st) {
  using Lq = attn_tr::Dq<D>;
  CUtensorMap tq{}, tk{}, tv{}, tdo{};
  if (const int rc = qkv_maps(a, &tq, &tk, &tv, &tdo)) return rc;
  const int64_t rows = (int64_t)a.T * a.Hq;
  attn_train_delta_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>(a.out, a.dout, const_cast<float*>(a.delta),
                                                                               a.T, a.Hq, D);
  static std::atomic<uint64_t> devs{0};
  if (const int e = smem_attr_once(devs, (const void*)attn_train_dq_kernel<D>, Lq::TOTAL)) return e;
  attn_train_dq_kernel<D><<<dim3(a.Hq, a.ntiles), attn_tr::THREADS_BWD, Lq::TOTAL, st>>>(tq, tdo, tk, tv, a, status);
  AttnTrainArgs b = a;
  b.tiles = kv_tiles;
  b.ntiles = nkv;
  int rc;
  if constexpr (D == 128) {
    rc = launch_dkdv<D, 3>(b, status, st);
  } else {  // dV and dK accumulators (2 x 256 TMEM columns) do not fit together: two passes
    rc = launch_dkdv<D, 1>(b, status, st);
    if (!rc) rc = launch_dkdv<D, 2>(b, status, st);
  }
  if (rc) return rc;
  const int64_t n4 = (int64_t)a.T * a.Hkv * D / 4;
  attn_train_dkdv_reduce_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(a.dk_part, a.dv_part, a.dk, a.dv, a.T,
                                                                              a.Hq, a.Hkv, D, a.scale);
  return (int)cudaGetLastError();
}

int attn_train_bwd(const AttnTrainArgs& a, const int2* kv_tiles, int nkv, uint32_t* status, cudaStream_t st) {
  if (const int e = check_args(a)) return e;
  if (!a.dout || !a.out || !a.delta || !a.dq || !a.dk || !a.dv || !a.dk_part || !a.dv_part || !kv_tiles) return 3;
  if (a.ntiles == 0) return 0;
  return a.D == 256 ? launch_bwd<256>(a, kv_tiles, nkv, status, st) : launch_bwd<128>(a, kv_tiles, nkv, status, st);
}

}  // namespace afb
