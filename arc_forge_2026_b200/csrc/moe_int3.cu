// INT3 (uint3 g128) routed-expert grouped GEMM, W3A8, on tcgen05 (kind::f8f6f4) with TMEM accumulators.
//
// Contract (the reference's serving W3A8, training/work/qwen38fn_lora/int3_moe.py:1-14): weight code c in 0..7
// means (c - 4) * s_w with a signed scale per (row, 128-column group); activations are e4m3 with one fp32 scale
// per (row, 128-column group); e4m3 x e4m3 products accumulate in fp32 and each group's partial sum is scaled by
// s_w * s_x before it joins the running sum. (c - 4) in -4..3 is exact in e4m3, so the tensor-core operand is
// lossless and the only roundings are the activation quantisation and fp32 accumulation.
//
// Weight layout read here ("tile layout", produced once at load by quant/int3_tiles.py from the Humming pack):
//   codes  int32 [E, R/128, K/128, 128 rows, 12 words]   (exactly 3 bits per weight, like the Humming stream)
//   scales bf16  [E, R/128, K/128, 128 rows]
// For 32 codes c0..c31 of a row the 3 words are two low-bit planes and one high-bit plane:
//   L0 nibble n = (c_n & 3) | (c_{8+n} & 3) << 2        L1 nibble n = (c_{16+n} & 3) | (c_{24+n} & 3) << 2
//   H  nibble n = (c_{16+n} >> 2) | (c_{24+n} >> 2) << 1 | (c_n >> 2) << 2 | (c_{8+n} >> 2) << 3
// so each 8-code selector word is one AND/OR of a plane and a shifted H, and one byte-permute maps 4 selectors
// to 4 e4m3 bytes through an 8-entry table held in two registers.
//
// One persistent CTA per SM, warp-specialised:
//   warp 0      loader: bulk copies of the code/scale tiles, TMA of the activation rows (no multicast),
//               activation scales by the 32 lanes
//   warps 1-4   dequant: codes -> e4m3 (c-4) into the 128-byte-swizzled A tile, then arrive
//   warp 5      MMA: M=128 (weight rows) x N=32 (tokens) x K=32 per op, one 128-K group per accumulator buffer
//   warps 6-9   epilogue: per group D * s_w * s_x into registers; at the end of a chunk:
//               PAIR (w13): h = silu(gate) * up, quantised to e4m3 per (token, 128-column group) for w2
//               !PAIR (w2): y = acc * route_weight, bf16
// A work unit is (expert, 128 output rows [+ the matching 128 up rows when PAIR]) x chunks of 32 tokens.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemm.h"
#include "moe.h"

namespace afb {

namespace moe {
constexpr int NTOK = 32;                  // tokens per chunk = MMA N
constexpr uint32_t CODE_TILE = 128 * 48;  // bytes of one 128-row x 128-K code tile
constexpr uint32_t A_TILE = 128 * 128;    // e4m3 128x128
constexpr uint32_t X_TILE = NTOK * 128;   // e4m3 32x128
constexpr uint32_t E4M3_LO = 0xB8C0C4C8u; // table bytes 0..3: e4m3(-4), e4m3(-3), e4m3(-2), e4m3(-1)
constexpr uint32_t E4M3_HI = 0x44403800u; // table bytes 4..7: e4m3(0), e4m3(1), e4m3(2), e4m3(3)

template <bool PAIR>
struct Layout {
  static constexpr int T = PAIR ? 2 : 1;  // weight tiles per k-step
  static constexpr uint32_t A_OFF = 0;
  static constexpr uint32_t X_OFF = A_OFF + T * A_TILE;
  static constexpr uint32_t C_OFF = X_OFF + X_TILE;
  static constexpr uint32_t SW_OFF = C_OFF + T * CODE_TILE;
  static constexpr uint32_t SX_OFF = SW_OFF + T * 128 * 2;
  static constexpr uint32_t STAGE_RAW = SX_OFF + NTOK * 4;
  static constexpr uint32_t STAGE = (STAGE_RAW + 1023) & ~1023u;
  static constexpr int STAGES = PAIR ? 4 : 6;
  static constexpr uint32_t BAR_OFF = STAGES * STAGE;
  // full[S], aready[S], empty[S], dfull[2], dempty[2]
  static constexpr uint32_t TOTAL = BAR_OFF + (3 * STAGES + 4) * 8 + 16 + 4 * 32 * 4 + 1024;
  static constexpr uint32_t RED_OFF = BAR_OFF + (3 * STAGES + 4) * 8 + 16;
  static constexpr uint32_t TMEM_COLS = 128;
};
}  // namespace moe

AFB_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

AFB_DEV void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// 32 codes (3 words of the tile layout) -> 32 e4m3 bytes (8 words), in code order
AFB_DEV void decode32(uint32_t L0, uint32_t L1, uint32_t H, uint32_t* o) {
  const uint32_t s0 = (L0 & 0x33333333u) | (H & 0x44444444u);
  const uint32_t s1 = ((L0 >> 2) & 0x33333333u) | ((H >> 1) & 0x44444444u);
  const uint32_t s2 = (L1 & 0x33333333u) | ((H << 2) & 0x44444444u);
  const uint32_t s3 = ((L1 >> 2) & 0x33333333u) | ((H << 1) & 0x44444444u);
  o[0] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, s0);
  o[1] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, s0 >> 16);
  o[2] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, s1);
  o[3] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, s1 >> 16);
  o[4] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, s2);
  o[5] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, s2 >> 16);
  o[6] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, s3);
  o[7] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, s3 >> 16);
}

// dequantise one 128-code row (12 words at `src`) into row `r` of a 128x128 e4m3 SW128 tile
AFB_DEV void dequant_row(const uint32_t* src, uint8_t* tile, int r) {
  const uint4 a = reinterpret_cast<const uint4*>(src)[0];
  const uint4 b = reinterpret_cast<const uint4*>(src)[1];
  const uint4 c = reinterpret_cast<const uint4*>(src)[2];
  const uint32_t w[12] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t o[8];
    decode32(w[3 * q], w[3 * q + 1], w[3 * q + 2], o);
    *reinterpret_cast<uint4*>(tile + sw128_offset(r, 2 * q)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(tile + sw128_offset(r, 2 * q + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

template <bool PAIR>
__global__ void __launch_bounds__(320, 1)
    moe_int3_gemm_kernel(const __grid_constant__ CUtensorMap tmX, MoeGemmArgs args, uint32_t* status) {
  using L = moe::Layout<PAIR>;
  constexpr int S = L::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* aready = full + S;
  uint64_t* empty = aready + S;
  uint64_t* dfull = empty + S;
  uint64_t* dempty = dfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dempty + 2);
  float* red = reinterpret_cast<float*>(smem + L::RED_OFF);  // [4 warps][32 tokens] amax exchange

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = args.num_experts;
  const int NB = args.rows / 128 / (PAIR ? 2 : 1);  // units per expert
  const int KG = args.K / 128;                       // k-steps (groups) per chunk
  const int units = E * NB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&aready[s], 128);
      mbar_init(&empty[s], 1 + 4);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&dfull[b], 1);
      mbar_init(&dempty[b], 4);
    }
    fence_mbar_init();
  }
  if (warp == 5) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int* off = args.expert_offsets;

  // every role walks the same (unit, chunk, group) sequence
  uint32_t kstep = 0;
  bool bail = false;
  for (int u = blockIdx.x; u < units && !bail; u += gridDim.x) {
    const int e = u % E, j = u / E;  // neighbouring CTAs take different experts
    const int row0 = off[e], n = off[e + 1] - row0;
    const int nchunks = (n + moe::NTOK - 1) / moe::NTOK;
    for (int ch = 0; ch < nchunks && !bail; ++ch) {
      const int crow = row0 + ch * moe::NTOK;
      const int cn = min(moe::NTOK, n - ch * moe::NTOK);
      if (warp == 0) {
        // ---------------------------------------------------------------- loader
        for (int g = 0; g < KG; ++g, ++kstep) {
          const int s = kstep % S;
          const uint32_t ph = (kstep / S) & 1;
          if (kstep >= (uint32_t)S && !mbar_wait(&empty[s], ph ^ 1, status)) {
            bail = true;
            break;
          }
          uint8_t* st = smem + s * L::STAGE;
          if (lane == 0) {
            // activation scales of this group for the chunk's 32 rows (group-major, segment starts are 8-aligned)
            const uint32_t bytes = L::T * (moe::CODE_TILE + 256) + moe::X_TILE + moe::NTOK * 4;
            mbar_arrive_expect_tx(&full[s], bytes);
            bulk_g2s(st + L::SX_OFF, args.x_scales + (size_t)g * args.ld_xs + crow, moe::NTOK * 4, &full[s]);
#pragma unroll
            for (int t = 0; t < L::T; ++t) {
              const int rb = PAIR ? (t == 0 ? j : NB + j) : j;  // gate block j, up block NB + j
              const size_t tile = ((size_t)e * (args.rows / 128) + rb) * KG + g;
              bulk_g2s(st + L::C_OFF + t * moe::CODE_TILE, args.codes + tile * (moe::CODE_TILE / 4), moe::CODE_TILE,
                       &full[s]);
              bulk_g2s(st + L::SW_OFF + t * 256, reinterpret_cast<const uint16_t*>(args.scales) + tile * 128, 256, &full[s]);
            }
            tma_load_2d(st + L::X_OFF, &tmX, &full[s], g * 128, crow);
          }
          __syncwarp();
        }
      } else if (warp >= 1 && warp <= 4) {
        // ---------------------------------------------------------------- dequant
        const int r = threadIdx.x - 32;  // 0..127: row of the weight tile
        for (int g = 0; g < KG; ++g, ++kstep) {
          const int s = kstep % S;
          const uint32_t ph = (kstep / S) & 1;
          if (!mbar_wait(&full[s], ph, status)) {
            bail = true;
            break;
          }
          uint8_t* st = smem + s * L::STAGE;
#pragma unroll
          for (int t = 0; t < L::T; ++t)
            dequant_row(reinterpret_cast<const uint32_t*>(st + L::C_OFF + t * moe::CODE_TILE) + r * 12,
                        st + L::A_OFF + t * moe::A_TILE, r);
          fence_proxy_async_smem();  // generic-proxy smem writes -> visible to the tensor core
          mbar_arrive(&aready[s]);
        }
      } else if (warp == 5) {
        // ---------------------------------------------------------------- MMA
        constexpr uint32_t idesc = idesc_e4m3(128, moe::NTOK);
        for (int g = 0; g < KG; ++g, ++kstep) {
          const int s = kstep % S;
          const uint32_t ph = (kstep / S) & 1;
          const int b = kstep & 1;
          const uint32_t bph = (kstep >> 1) & 1;
          bool ok = mbar_wait(&aready[s], ph, status);
          if (ok && kstep >= 2) ok = mbar_wait(&dempty[b], bph ^ 1, status);
          if (!ok) {
            bail = true;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            uint8_t* st = smem + s * L::STAGE;
            const uint64_t dx = sw128_desc(smem_u32(st + L::X_OFF));
#pragma unroll
            for (int t = 0; t < L::T; ++t) {
              const uint64_t da = sw128_desc(smem_u32(st + L::A_OFF + t * moe::A_TILE));
              const uint32_t d = tmem + (uint32_t)((b * 2 + t) * moe::NTOK);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) umma_f8(d, da + 2 * kk, dx + 2 * kk, idesc, kk != 0);
            }
            umma_commit(&dfull[b]);
            umma_commit(&empty[s]);
          }
          __syncwarp();
        }
      } else {
        // ---------------------------------------------------------------- epilogue (warps 6..9)
        const int quad = warp & 3;
        const int r = quad * 32 + lane;  // TMEM lane = row of the weight tile
        float acc0[moe::NTOK], acc1[PAIR ? moe::NTOK : 1];
#pragma unroll
        for (int i = 0; i < moe::NTOK; ++i) acc0[i] = 0.f;
#pragma unroll
        for (int i = 0; i < (PAIR ? moe::NTOK : 1); ++i) acc1[i] = 0.f;
        for (int g = 0; g < KG; ++g, ++kstep) {
          const int s = kstep % S;
          const int b = kstep & 1;
          const uint32_t bph = (kstep >> 1) & 1;
          if (!mbar_wait(&dfull[b], bph, status)) {
            bail = true;
            break;
          }
          tc_fence_after();
          float d0[moe::NTOK], d1[moe::NTOK];
          const uint32_t ta = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * 2 * moe::NTOK);
          tmem_ld32(ta, d0);
          if (PAIR) tmem_ld32(ta + moe::NTOK, d1);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dempty[b]);
          const uint8_t* st = smem + s * L::STAGE;
          const float* sx = reinterpret_cast<const float*>(st + L::SX_OFF);
          const float sw0 = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(st + L::SW_OFF)[r]);
          const float sw1 = PAIR ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(st + L::SW_OFF + 256)[r]) : 0.f;
#pragma unroll
          for (int i = 0; i < moe::NTOK; ++i) {
            const float x = sx[i];
            acc0[i] = fmaf(sw0 * x, d0[i], acc0[i]);
            if (PAIR) acc1[i] = fmaf(sw1 * x, d1[i], acc1[i]);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (bail) break;
        if (PAIR) {
          // h = silu(gate) * up -> e4m3 with a scale per (token, this 128-column group)
          const int col = j * 128 + r;  // intermediate column
          float amax[moe::NTOK];
#pragma unroll
          for (int i = 0; i < moe::NTOK; ++i) {
            acc0[i] = silu(acc0[i]) * acc1[i];
            amax[i] = warp_max(fabsf(acc0[i]));
          }
          if (lane == 0) {
#pragma unroll
            for (int i = 0; i < moe::NTOK; ++i) red[quad * 32 + i] = amax[i];
          }
          named_bar(1, 128);
#pragma unroll
          for (int i = 0; i < moe::NTOK; ++i)
            amax[i] = fmaxf(fmaxf(red[i], red[32 + i]), fmaxf(red[64 + i], red[96 + i]));
          named_bar(1, 128);  // red is reused by the next chunk
#pragma unroll
          for (int i = 0; i < moe::NTOK; ++i) {
            if (i >= cn) break;
            const float sc = amax[i] > 0.f ? amax[i] / 448.f : 1.f;
            const __nv_fp8_e4m3 q(acc0[i] / sc);
            args.out_q[(size_t)(crow + i) * args.out_ld + col] = *reinterpret_cast<const uint8_t*>(&q);
            if (r == 0) args.out_scales[(size_t)j * args.ld_os + crow + i] = sc;
          }
        } else {
          const int col = j * 128 + r;  // hidden column
#pragma unroll
          for (int i = 0; i < moe::NTOK; ++i) {
            if (i >= cn) break;
            const float w = args.route_w ? args.route_w[args.row_entry[crow + i]] : 1.f;
            reinterpret_cast<__nv_bfloat16*>(args.out_bf16)[(size_t)(crow + i) * args.out_ld + col] = __float2bfloat16(acc0[i] * w);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

int moe_int3_gemm(const MoeGemmArgs& a, int pair, int num_sms, uint32_t* status, cudaStream_t st) {
  if (a.K % 128 || a.rows % (pair ? 256 : 128)) return 3;
  if (a.num_rows_total <= 0) return 0;
  CUtensorMap tx;
  int rc = make_tmap_2d(&tx, a.x_q, 1, a.K, a.num_rows_total, (uint64_t)a.K, 128, moe::NTOK, 1);
  if (rc) return 1000 + rc;
  const int units = a.num_experts * (a.rows / 128 / (pair ? 2 : 1));
  const int grid = units < num_sms ? units : num_sms;
  if (pair) {
    using L = moe::Layout<true>;
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(moe_int3_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
      attr = true;
    }
    moe_int3_gemm_kernel<true><<<grid, 320, L::TOTAL, st>>>(tx, a, status);
  } else {
    using L = moe::Layout<false>;
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(moe_int3_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
      attr = true;
    }
    moe_int3_gemm_kernel<false><<<grid, 320, L::TOTAL, st>>>(tx, a, status);
  }
  return (int)cudaGetLastError();
}

}  // namespace afb
