// Paged decode / speculative-verify attention with GQA (gated-attention layers).
//
// One CTA per (sequence, KV head, KV split). Its query rows are the q_per_seq verify positions x the Hq/Hkv
// query heads of that KV head (row = t * group + h), so one KV page read from HBM serves every head of the
// group and every verify position. Pages ([num_pages, Hkv, page_size=64, D] bf16) arrive by TMA in the
// 128-byte swizzle into a 2-deep ring; 8 warps = 4 row tiles of 16 x 2 halves of each page's 64 keys.
// S = Q K^T and O += P V run on the tensor cores (m16n8k16 bf16, fp32 accumulate; the kernel streams KV at
// HBM speed, so the MMA generation is not the limit), softmax is online in fp32 with exp2.
// Causality inside the verify window: position t sees keys < past_len + t + 1.
// With one split the output is written directly as bf16 * sigmoid(gate); with several, each split writes
// (O, log-sum-exp) partials and attn_merge_kernel combines them in split order (deterministic).
//
// NVFP4 KV (FP4 = true): a page-head holds 64 x D/2 bytes of e2m1 pairs and 64 x D/16 e4m3 scales (one per 16
// elements), both contiguous, so each arrives by one 1-D bulk copy per tensor into a 2-deep ring (3.6x fewer bytes
// than bf16). All 256 threads dequantise a landed page into swizzled f16 tiles: one e2m1x2 -> f16x2 conversion and
// one f16x2 multiply by the block scale per element pair (e2m1 x e4m3 has at most 6 significant bits and stays
// within f16's range, so the tile holds the dequantised values exactly). This variant runs its MMAs in f16 (Q and
// the softmax probabilities converted to f16; fp32 accumulation). Block-wide barriers order the dequantisation
// against the previous page's MMAs, and the stage is refilled right after it.
#include <cudaTypedefs.h>
#include <cuda_fp4.h>

#include <type_traits>

#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace afb {

namespace attn {
constexpr int PAGE = 64;
constexpr int WARPS = 8;
}

// byte offset of (row, 16-byte chunk cc in 0..D/8) inside a [rows x D] bf16 tile stored as D/64 sub-tiles of
// [rows x 128 B] in the 128-byte swizzle (the layout TMA writes with a {64, rows} box)
template <int ROWS>
AFB_DEV uint32_t sw_off(int row, int cc) {
  return (uint32_t)((cc >> 3) * ROWS * 128 + row * 128 + (((cc & 7) ^ (row & 7)) << 4));
}

template <int D>
struct AttnSmem {
  static constexpr uint32_t KV_BYTES = attn::PAGE * D * 2;  // one K (or V) page of one head
  static constexpr uint32_t Q_BYTES = 64 * D * 2;
  static constexpr uint32_t STAGE = 2 * KV_BYTES;
  static constexpr uint32_t Q_OFF = 2 * STAGE;
  static constexpr uint32_t BAR_OFF = Q_OFF + Q_BYTES;
  static constexpr int SBT = 1024;                             // block-table entries staged in shared memory
  static constexpr uint32_t SBT_OFF = BAR_OFF + 64;
  static constexpr uint32_t TOTAL = SBT_OFF + SBT * 4 + 1024;
  static constexpr int NS = 2;  // TMA stages
};

// NVFP4 layout: NS stages of packed K, packed V, K scales, V scales, then two f16 K + V tile pairs (the MMA operands
// of page i and page i + 1)
template <int D>
struct AttnSmemFp4 {
  static constexpr int NS = 3;
  static constexpr uint32_t PK = attn::PAGE * D / 2;           // e2m1 bytes of one page-head
  static constexpr uint32_t PS = attn::PAGE * D / 16;          // e4m3 scale bytes of one page-head
  static constexpr uint32_t KV_BYTES = attn::PAGE * D * 2;     // one dequantised f16 tile
  static constexpr uint32_t BUF = 2 * KV_BYTES;                // one K + V pair
  static constexpr uint32_t STAGE = 2 * PK + 2 * PS;
  static constexpr uint32_t BF_OFF = NS * STAGE;
  static constexpr uint32_t Q_BYTES = 64 * D * 2;
  static constexpr uint32_t Q_OFF = BF_OFF + 2 * BUF;
  static constexpr uint32_t BAR_OFF = Q_OFF + Q_BYTES;
  static constexpr int SBT = 1024;
  static constexpr uint32_t SBT_OFF = BAR_OFF + 64;
  static constexpr uint32_t TOTAL = SBT_OFF + SBT * 4 + 1024;
  static_assert(BF_OFF % 1024 == 0 && Q_OFF % 1024 == 0, "swizzled tiles need 1 KB alignment");
  static_assert(BF_OFF >= 4 * 16 * D * 4 + 64 * 2 * 4 || Q_OFF >= 4 * 16 * D * 4 + 64 * 2 * 4,
                "the half-merge scratch must fit below Q");
};

AFB_DEV void mma_f16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <bool F16>
AFB_DEV void mma_kv(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (F16)
    mma_f16(c, a0, a1, a2, a3, b0, b1);
  else
    mma_bf16(c, a0, a1, a2, a3, b0, b1);
}
template <bool F16>
AFB_DEV uint32_t pack_kv(float a, float b) {
  if constexpr (F16) {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    return pack_bf16x2(a, b);
  }
}

// one landed NVFP4 page-head pair (packed + scales at `st`) -> swizzled f16 K and V tiles at `bf`
template <int D>
AFB_DEV void dequant_fp4_page(const uint8_t* st, uint8_t* bf) {
  using S = AttnSmemFp4<D>;
  constexpr int PC = D / 32;  // 16-byte packed chunks per row (32 elements, 2 scales)
  for (int q = threadIdx.x; q < 2 * attn::PAGE * PC; q += blockDim.x) {
    const int m = q / (attn::PAGE * PC), rq = q % (attn::PAGE * PC);
    const int row = rq / PC, pc = rq % PC;
    const uint8_t* pk = st + m * S::PK + row * (D / 2) + pc * 16;
    const uint8_t* sc = st + 2 * S::PK + m * S::PS + row * (D / 16) + pc * 2;
    const uint4 v = *reinterpret_cast<const uint4*>(pk);
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&v);
    uint8_t* dst = bf + m * S::KV_BYTES;
#pragma unroll
    for (int half = 0; half < 2; ++half) {  // 16 elements share one scale
      const __half2 s2 = __half2half2(__half(__nv_cvt_fp8_to_halfraw(sc[half], __NV_E4M3)));
#pragma unroll
      for (int c8 = 0; c8 < 2; ++c8) {  // two 8-element f16 chunks
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const __half2 h2 = __hmul2(__half2(__nv_cvt_fp4x2_to_halfraw2(b[half * 8 + c8 * 4 + j], __NV_E2M1)), s2);
          w[j] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        const int cc = pc * 4 + half * 2 + c8;
        *reinterpret_cast<uint4*>(dst + sw_off<attn::PAGE>(row, cc)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
}

template <int D, bool FP4>
__global__ void __launch_bounds__(256, 1)
    paged_attn_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      AttnArgs a, uint32_t* status) {
  using S = typename std::conditional<FP4, AttnSmemFp4<D>, AttnSmem<D>>::type;
  constexpr int NT_O = D / 8;  // output n-tiles per row tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + S::Q_OFF;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* empty = full + S::NS;  // bf16 path only

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq = blockIdx.x / a.Hkv, kvh = blockIdx.x % a.Hkv;
  const int split = blockIdx.y;
  const int group = a.Hq / a.Hkv;
  const int QR = a.q_per_seq * group;  // query rows of this CTA (<= 64)
  const int seq_len = a.seq_lens[seq];
  const int past = seq_len - a.q_per_seq;
  const bool sparse = a.sp_count != nullptr;  // QSA: the block-table row is this sequence's page union
  const int npages = sparse ? a.sp_count[seq] : (seq_len + attn::PAGE - 1) / attn::PAGE;
  // sliding window: query t sees keys [past + t + 1 - window, past + t]
  const int kv_lo = a.window > 0 && !sparse ? max(0, past + 1 - a.window) : 0;
  const int pbeg = kv_lo / attn::PAGE;
  const int p0 = pbeg + split * a.pages_per_split;
  const int p1 = min(npages, p0 + a.pages_per_split);
  const int n = max(0, p1 - p0);
  const int* bt = a.block_table + (size_t)(a.bt_row ? a.bt_row[seq] : seq) * a.max_pages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::NS; ++s) {
      mbar_init(&full[s], 1);
      if (!FP4) mbar_init(&empty[s], attn::WARPS);
    }
    fence_mbar_init();
  }
  // this split's page ids, staged once: the TMA issue of each page then needs no global load on its path
  int* sbt = reinterpret_cast<int*>(smem + S::SBT_OFF);
  for (int i = threadIdx.x; i < min(n, S::SBT); i += blockDim.x) sbt[i] = bt[p0 + i];
  // Q rows -> smem (swizzled); rows >= QR are zero
  for (int idx = threadIdx.x; idx < 64 * (D / 8); idx += blockDim.x) {
    const int r = idx / (D / 8), cc = idx % (D / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < QR) {
      const int t = r / group, h = r % group;
      const __nv_bfloat16* src =
          a.q + ((size_t)(seq * a.q_per_seq + t) * a.Hq + kvh * group + h) * D + cc * 8;
      v = *reinterpret_cast<const uint4*>(src);
      if constexpr (FP4) {  // the f16 MMA path: queries to f16
        const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&v);
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = pack_kv<true>(__low2float(hb[j]), __high2float(hb[j]));
        v = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    *reinterpret_cast<uint4*>(sQ + sw_off<64>(r, cc)) = v;
  }
  __syncthreads();

  auto issue = [&](int i) {
    const int s = i % S::NS;
    const int page = i < S::SBT ? sbt[i] : bt[p0 + i];
    const int row = (page * a.Hkv + kvh) * attn::PAGE;
    uint8_t* st = smem + s * S::STAGE;
    if constexpr (FP4) {  // contiguous page-heads: one plain bulk copy per tensor (no tensor map)
      const size_t ph = (size_t)page * a.Hkv + kvh;
      mbar_arrive_expect_tx(&full[s], S::STAGE);
      bulk_load_1d(st, reinterpret_cast<const uint8_t*>(a.kcache) + ph * S::PK, S::PK, &full[s]);
      bulk_load_1d(st + S::PK, reinterpret_cast<const uint8_t*>(a.vcache) + ph * S::PK, S::PK, &full[s]);
      bulk_load_1d(st + 2 * S::PK, a.kscale + ph * S::PS, S::PS, &full[s]);
      bulk_load_1d(st + 2 * S::PK + S::PS, a.vscale + ph * S::PS, S::PS, &full[s]);
    } else {
      mbar_arrive_expect_tx(&full[s], 2 * S::KV_BYTES);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_2d(st + c * attn::PAGE * 128, &tmK, &full[s], c * 64, row);
        tma_load_2d(st + S::KV_BYTES + c * attn::PAGE * 128, &tmV, &full[s], c * 64, row);
      }
    }
  };
  int issued = 0;  // meaningful in thread 0 only
  if (threadIdx.x == 0) {
    if constexpr (!FP4) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
    }
    for (int i = 0; i < min(S::NS, n); ++i) issue(i);
    issued = min(S::NS, n);
  }

  const int mt = warp >> 1, kh = warp & 1;
  const bool active = mt * 16 < QR;
  const int r0 = mt * 16 + (lane >> 2), r1 = r0 + 8;  // this thread's two rows
  const int t0 = r0 / group, t1 = r1 / group;
  float o[NT_O][4];
#pragma unroll
  for (int i = 0; i < NT_O; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const uint32_t q_base = smem_u32(sQ);
  bool ok = true;

  for (int i = 0; i < n && ok; ++i) {
    const int s = i & 1;
    uint32_t k_base;
    if constexpr (FP4) {
      if (i == 0) {  // page 0 -> f16 buffer 0. Every thread waits (bounded); one block-wide vote keeps exits uniform
        const bool landed = mbar_wait(&full[0], 0, status);
        if (!__syncthreads_and(landed)) {
          ok = false;
          break;
        }
        dequant_fp4_page<D>(smem, smem + S::BF_OFF);
        __syncthreads();
        if (threadIdx.x == 0 && S::NS < n) {  // stage 0 is consumed: refill it
          issue(S::NS);
          ++issued;
        }
      }
      k_base = smem_u32(smem + S::BF_OFF + (i & 1) * S::BUF);
    } else {
      if (!mbar_wait(&full[s], (i >> 1) & 1, status)) {
        ok = false;
        break;
      }
      k_base = smem_u32(smem + s * S::STAGE);
    }
    const uint32_t v_base = k_base + S::KV_BYTES;
    if (active) {
      // ---- S = Q K^T for 32 keys (4 n-tiles of 8)
      float sc[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t a0, a1, a2, a3;
        {
          const int row = mt * 16 + (lane & 15);
          const int cc = ks * 2 + (lane >> 4);
          ldsm_x4(q_base + sw_off<64>(row, cc), a0, a1, a2, a3);
        }
#pragma unroll
        for (int np = 0; np < 2; ++np) {  // pairs of n-tiles (16 keys)
          uint32_t b0, b1, b2, b3;
          const int key = kh * 32 + np * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int cc = ks * 2 + ((lane >> 3) & 1);
          ldsm_x4(k_base + sw_off<attn::PAGE>(key, cc), b0, b1, b2, b3);
          mma_kv<FP4>(sc[np * 2], a0, a1, a2, a3, b0, b1);
          mma_kv<FP4>(sc[np * 2 + 1], a0, a1, a2, a3, b2, b3);
        }
      }
      // ---- mask + online softmax (log2 domain)
      const size_t ui = (size_t)(a.bt_row ? a.bt_row[seq] : seq) * a.max_pages + p0 + i;  // union entry (sparse)
      const int kbase = (sparse ? a.sp_lpage[ui] : p0 + i) * attn::PAGE + kh * 32;
      const uint32_t rmask = sparse ? a.sp_mask[ui] : 0xffffffffu;
      const bool see0 = (rmask >> min(t0, 31)) & 1u, see1 = (rmask >> min(t1, 31)) & 1u;
      float mx0 = m0, mx1 = m1;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = kbase + j * 8 + (lane & 3) * 2 + e;
          float v0 = sc[j][e] * a.scale_log2, v1 = sc[j][2 + e] * a.scale_log2;
          if (key >= past + t0 + 1 || r0 >= QR || !see0 || (a.window > 0 && key < past + t0 + 1 - a.window))
            v0 = -INFINITY;
          if (key >= past + t1 + 1 || r1 >= QR || !see1 || (a.window > 0 && key < past + t1 + 1 - a.window))
            v1 = -INFINITY;
          sc[j][e] = v0;
          sc[j][2 + e] = v1;
          mx0 = fmaxf(mx0, v0);
          mx1 = fmaxf(mx1, v1);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float base0 = mx0 == -INFINITY ? 0.f : mx0, base1 = mx1 == -INFINITY ? 0.f : mx1;
      const float c0 = exp2f(m0 - base0), c1 = exp2f(m1 - base1);
      m0 = mx0;
      m1 = mx1;
      float rs0 = 0.f, rs1 = 0.f;
      uint32_t p[4][2];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float e0 = exp2f(sc[j][0] - base0), e1 = exp2f(sc[j][1] - base0);
        const float e2 = exp2f(sc[j][2] - base1), e3 = exp2f(sc[j][3] - base1);
        rs0 += e0 + e1;
        rs1 += e2 + e3;
        p[j][0] = pack_kv<FP4>(e0, e1);
        p[j][1] = pack_kv<FP4>(e2, e3);
      }
      l0 = l0 * c0 + rs0;
      l1 = l1 * c1 + rs1;
#pragma unroll
      for (int d = 0; d < NT_O; ++d) {
        o[d][0] *= c0;
        o[d][1] *= c0;
        o[d][2] *= c1;
        o[d][3] *= c1;
      }
      // ---- O += P V over the 32 keys (2 k-steps of 16)
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const uint32_t pa0 = p[2 * kk][0], pa1 = p[2 * kk][1], pa2 = p[2 * kk + 1][0], pa3 = p[2 * kk + 1][1];
#pragma unroll
        for (int dp = 0; dp < NT_O / 2; ++dp) {
          uint32_t b0, b1, b2, b3;
          const int key = kh * 32 + kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
          const int cc = dp * 2 + (lane >> 4);
          ldsm_x4_t(v_base + sw_off<attn::PAGE>(key, cc), b0, b1, b2, b3);
          mma_kv<FP4>(o[dp * 2], pa0, pa1, pa2, pa3, b0, b1);
          mma_kv<FP4>(o[dp * 2 + 1], pa0, pa1, pa2, pa3, b2, b3);
        }
      }
    }
    if constexpr (FP4) {
      // page i + 1 -> the other f16 buffer, right after this warp's MMAs on page i (warps with fewer rows start
      // early); that buffer's last reader, page i - 1, finished before the previous barrier
      bool landed = true;
      if (i + 1 < n) {
        const int s1 = (i + 1) % S::NS;
        landed = mbar_wait(&full[s1], ((i + 1) / S::NS) & 1, status);
        if (landed) dequant_fp4_page<D>(smem + s1 * S::STAGE, smem + S::BF_OFF + ((i + 1) & 1) * S::BUF);
      }
      if (!__syncthreads_and(landed)) {
        ok = false;
        break;
      }
      if (threadIdx.x == 0 && i + 1 + S::NS < n) {  // the stage of page i + 1 is consumed: refill it
        issue(i + 1 + S::NS);
        ++issued;
      }
    } else {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (threadIdx.x == 0 && i + 2 < n) {
        if (!mbar_wait(&empty[s], (i >> 1) & 1, status)) {
          ok = false;
        } else {
          issue(i + 2);
          ++issued;
        }
      }
    }
  }
  // drain copies still in flight before the smem is reused (bounded)
  if (threadIdx.x == 0) {
    for (int i = max(0, issued - S::NS); i < issued; ++i) mbar_wait(&full[i % S::NS], (i / S::NS) & 1, status);
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  __syncthreads();
  // ---- merge the two key halves: kh=1 publishes (m, l, O) through smem
  float* xo = reinterpret_cast<float*>(smem);                    // [4 mt][16 rows][D]
  float* xm = reinterpret_cast<float*>(smem + 4 * 16 * D * 4);   // [4 mt][16 rows][2] (m, l)
  if (active && kh == 1) {
#pragma unroll
    for (int d = 0; d < NT_O; ++d) {
      const int col = d * 8 + (lane & 3) * 2;
      float* q0 = xo + (mt * 16 + (lane >> 2)) * D + col;
      float* q1 = xo + (mt * 16 + (lane >> 2) + 8) * D + col;
      q0[0] = o[d][0];
      q0[1] = o[d][1];
      q1[0] = o[d][2];
      q1[1] = o[d][3];
    }
    if ((lane & 3) == 0) {
      xm[(mt * 16 + (lane >> 2)) * 2] = m0;
      xm[(mt * 16 + (lane >> 2)) * 2 + 1] = l0;
      xm[(mt * 16 + (lane >> 2) + 8) * 2] = m1;
      xm[(mt * 16 + (lane >> 2) + 8) * 2 + 1] = l1;
    }
  }
  __syncthreads();
  if (!active || kh == 1 || !ok) return;
  const float om0 = xm[(mt * 16 + (lane >> 2)) * 2], ol0 = xm[(mt * 16 + (lane >> 2)) * 2 + 1];
  const float om1 = xm[(mt * 16 + (lane >> 2) + 8) * 2], ol1 = xm[(mt * 16 + (lane >> 2) + 8) * 2 + 1];
  const float M0 = fmaxf(m0, om0), M1 = fmaxf(m1, om1);
  const float B0 = M0 == -INFINITY ? 0.f : M0, B1 = M1 == -INFINITY ? 0.f : M1;
  const float sa0 = exp2f(m0 - B0), sb0 = exp2f(om0 - B0), sa1 = exp2f(m1 - B1), sb1 = exp2f(om1 - B1);
  const float L0 = l0 * sa0 + ol0 * sb0, L1 = l1 * sa1 + ol1 * sb1;
  const bool direct = gridDim.y == 1;
  // every split stores its own normalised output; the merge weights splits by exp2(lse_s - lse_max)
  const float inv0 = L0 > 0.f ? 1.f / L0 : 1.f, inv1 = L1 > 0.f ? 1.f / L1 : 1.f;
#pragma unroll
  for (int d = 0; d < NT_O; ++d) {
    const int col = d * 8 + (lane & 3) * 2;
    const float* q0 = xo + (mt * 16 + (lane >> 2)) * D + col;
    const float* q1 = xo + (mt * 16 + (lane >> 2) + 8) * D + col;
    float v[2][2] = {{(o[d][0] * sa0 + q0[0] * sb0) * inv0, (o[d][1] * sa0 + q0[1] * sb0) * inv0},
                     {(o[d][2] * sa1 + q1[0] * sb1) * inv1, (o[d][3] * sa1 + q1[1] * sb1) * inv1}};
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int r = h2 ? r1 : r0;
      if (r >= QR) continue;
      const int t = r / group, hh = r % group;
      const size_t tok = (size_t)seq * a.q_per_seq + t;
      const int head = kvh * group + hh;
      if (direct) {
        float g0 = 1.f, g1 = 1.f;
        if (a.gate) {
          const __nv_bfloat16* gp = a.gate + tok * a.gate_ld + head * a.gate_head_stride + col;
          g0 = 1.f / (1.f + __expf(-__bfloat162float(gp[0])));
          g1 = 1.f / (1.f + __expf(-__bfloat162float(gp[1])));
        }
        __nv_bfloat16* op = a.out + (tok * a.Hq + head) * D + col;
        *reinterpret_cast<uint32_t*>(op) = pack_bf16x2(v[h2][0] * g0, v[h2][1] * g1);
      } else {
        float* pp = a.part_o + (((size_t)split * a.num_tokens + tok) * a.Hq + head) * D + col;
        pp[0] = v[h2][0];
        pp[1] = v[h2][1];
        if ((lane & 3) == 0 && d == 0) {
          const float M = h2 ? M1 : M0, L = h2 ? L1 : L0;
          // log2-sum-exp of this split (-inf when the split saw no visible key)
          a.part_lse[((size_t)split * a.num_tokens + tok) * a.Hq + head] = L > 0.f ? M + log2f(L) : -INFINITY;
        }
      }
    }
  }
}

// combine split partials in split order: out = sum_s exp2(lse_s - LSE) O_s * sigmoid(gate)
template <int D>
__global__ void attn_merge_kernel(AttnArgs a, int splits) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int th = blockIdx.x;  // (token, head)
  const int tok = th / a.Hq, head = th % a.Hq;
  float lse_max = -INFINITY;
  for (int s = 0; s < splits; ++s) lse_max = fmaxf(lse_max, a.part_lse[((size_t)s * a.num_tokens + tok) * a.Hq + head]);
  float wsum = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float l = a.part_lse[((size_t)s * a.num_tokens + tok) * a.Hq + head];
    wsum += l == -INFINITY ? 0.f : exp2f(l - lse_max);
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float l = a.part_lse[((size_t)s * a.num_tokens + tok) * a.Hq + head];
      if (l == -INFINITY) continue;
      acc += exp2f(l - lse_max) * a.part_o[(((size_t)s * a.num_tokens + tok) * a.Hq + head) * D + d];
    }
    acc = wsum > 0.f ? acc / wsum : 0.f;
    if (a.gate) {
      const float g = __bfloat162float(a.gate[(size_t)tok * a.gate_ld + head * a.gate_head_stride + d]);
      acc *= 1.f / (1.f + __expf(-g));
    }
    a.out[((size_t)tok * a.Hq + head) * D + d] = __float2bfloat16(acc);
  }
}

template <int D, bool FP4>
static int launch_attn(const AttnArgs& a, int splits, uint32_t* status, cudaStream_t st) {
  using S = typename std::conditional<FP4, AttnSmemFp4<D>, AttnSmem<D>>::type;
  CUtensorMap tk{}, tv{};
  int rc;
  if (!FP4) {
    const uint64_t rows = (uint64_t)a.num_pages * a.Hkv * attn::PAGE;
    rc = make_tmap_2d(&tk, a.kcache, 2, D, rows, (uint64_t)D * 2, 64, attn::PAGE, 1);
    if (rc) return 1000 + rc;
    rc = make_tmap_2d(&tv, a.vcache, 2, D, rows, (uint64_t)D * 2, 64, attn::PAGE, 1);
    if (rc) return 1000 + rc;
  } else if (!a.kscale || !a.vscale || (reinterpret_cast<uintptr_t>(a.kcache) | reinterpret_cast<uintptr_t>(a.vcache) |
                                         reinterpret_cast<uintptr_t>(a.kscale) |
                                         reinterpret_cast<uintptr_t>(a.vscale)) % 16) {
    return 5;  // bulk copies need 16-byte aligned sources
  }
  static std::atomic<uint64_t> attr_devs{0};
  if (const int e = smem_attr_once(attr_devs, (const void*)paged_attn_kernel<D, FP4>, S::TOTAL)) return e;
  dim3 grid(a.num_seqs * a.Hkv, splits);
  paged_attn_kernel<D, FP4><<<grid, 256, S::TOTAL, st>>>(tk, tv, a, status);
  rc = (int)cudaGetLastError();
  if (rc || splits == 1) return rc;
  {
    const int pdl_rc = launch_pdl(attn_merge_kernel<D>, dim3(a.num_tokens * a.Hq), dim3(128), 0, st, a, splits);
    if (pdl_rc) return pdl_rc;
  }
  return (int)cudaGetLastError();
}

int paged_attention_tc(const AttnArgs& a, int splits, uint32_t* status, cudaStream_t st);  // attention_tc.cu

int paged_attention(const AttnArgs& a, int splits, uint32_t* status, cudaStream_t st) {
  if (splits > 1 && (!a.part_o || !a.part_lse)) return 4;
  if (a.num_seqs == 0) return 0;
  const bool fp4 = a.kscale != nullptr;
  const bool gather = a.sp_count && a.sp_block != 64;  // sub-page QSA blocks: the tcgen05 kernel or nothing
  if (gather && (a.sp_block < 1 || 64 % a.sp_block || a.sp_ld < 1)) return 3;
  if (const int rc = paged_attention_tc(a, splits, status, st); rc != -1) {
    if (rc || splits == 1) return rc;
    const dim3 grid(a.num_tokens * a.Hq);
    return a.D == 256 ? launch_pdl(attn_merge_kernel<256>, grid, dim3(128), 0, st, a, splits)
                      : launch_pdl(attn_merge_kernel<128>, grid, dim3(128), 0, st, a, splits);
  }
  if (gather || a.q_per_seq * (a.Hq / a.Hkv) > 64) return 3;  // the mma.sync kernel holds <= 64 rows per CTA
  if (a.D == 256) return fp4 ? launch_attn<256, true>(a, splits, status, st) : launch_attn<256, false>(a, splits, status, st);
  if (a.D == 128) return fp4 ? launch_attn<128, true>(a, splits, status, st) : launch_attn<128, false>(a, splits, status, st);
  return 3;
}

}  // namespace afb
