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
// One persistent CTA per SM, warp-specialised; the dequant and epilogue roles are latency-bound chains, so they get
// 6 and 8 warps. A ring of raw stages feeds a ring of dequantised tiles and the MMA runs up to 8 (w13) / 16 (w2)
// groups ahead of the epilogue in TMEM. The dequant warps also copy each group's scales into a per-accumulator-buffer
// slot, so a raw stage is released once dequant and MMA are done with it and never waits on the epilogue:
//   warp 0      loader: bulk copies of the code/scale tiles and of the activation scales, TMA of the activation
//               rows (no multicast)
//   warps 1-6   dequant: codes -> e4m3 (c-4) into the 128-byte-swizzled A tile, in tasks of 32 codes spread
//               evenly over the 192 threads, then arrive
//   warp 7      MMA: M=128 (weight rows) x N=32 (tokens) x K=32 per op, one 128-K group per accumulator buffer
//   warps 8-15  epilogue (two per TMEM lane quadrant, 16 token columns each): per group D * s_w * s_x into
//               registers; at the end of a chunk:
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
constexpr int MAX_E = 1024;               // experts whose segment offsets are staged in shared memory

// Rings: raw stages (codes, weight scales, activation tile and scales, all moved by bulk/TMA copies), dequantised
// e4m3 A tiles (dequant -> MMA), and per TMEM accumulator buffer a copy of the group's scales (dequant -> epilogue).
template <bool PAIR, bool F8 = false>
struct Layout {
  static constexpr int T = PAIR ? 2 : 1;  // weight tiles per k-step
  static constexpr uint32_t X_OFF = 0;    // 1024-aligned (TMA 128-byte swizzle)
  // INT3: code tiles (bulk copies), then per-row bf16 scales. F8: the e4m3 weight tiles themselves (TMA, swizzled:
  // they are the MMA's A operand as they land) -- their fp32 block scales are read by the scale warps.
  static constexpr uint32_t WA_OFF = X_OFF + X_TILE;
  static constexpr uint32_t C_OFF = X_OFF + X_TILE;
  static constexpr uint32_t SW_OFF = F8 ? WA_OFF + T * A_TILE : C_OFF + T * CODE_TILE;
  static constexpr uint32_t SX_OFF = SW_OFF + (F8 ? 0 : T * 128 * 2);
  static constexpr uint32_t RAW_BYTES = SX_OFF + NTOK * 4;
  static constexpr uint32_t RAW = (RAW_BYTES + 1023) & ~1023u;
  static constexpr int CTAS_PER_SM = 1;
  static constexpr int RS = F8 ? (PAIR ? 5 : 8) : (PAIR ? 6 : 8);  // raw stages
  static constexpr int AS = PAIR ? 3 : 4;     // dequantised stages (F8: no A ring, barriers only)
  static constexpr int NBUF = PAIR ? 8 : 16;  // TMEM accumulator buffers (T * 32 columns each)
  static constexpr uint32_t ESC = 640;        // per-buffer copy of the group's scales (INT3: T*128 bf16 s_w, then
                                              // 32 fp32 s_x; F8: T fp32 block scales, s_x at byte 16)
  static constexpr uint32_t A_STAGE = F8 ? 0 : T * A_TILE;
  static constexpr uint32_t A_OFF = RS * RAW;
  static constexpr uint32_t ESC_OFF = A_OFF + AS * A_STAGE;         // scale ring [NBUF][ESC]
  static constexpr uint32_t OFFS_OFF = ESC_OFF + NBUF * ESC;         // int offsets[MAX_E + 1]
  static constexpr uint32_t RED_OFF = OFFS_OFF + (MAX_E + 1) * 4;   // float [2 halves][4 quads][16]
  static constexpr uint32_t BAR_OFF = (RED_OFF + 2 * 4 * 16 * 4 + 7) & ~7u;
  // full[RS], empty[RS], afull[AS], aempty[AS], dfull[NBUF], dempty[NBUF], sready[NBUF], tmem slot
  static constexpr uint32_t TOTAL = BAR_OFF + (2 * RS + 2 * AS + 3 * NBUF) * 8 + 16 + 1024;
  static constexpr uint32_t TMEM_COLS = 512 / CTAS_PER_SM;
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

// warp roles (16 warps = 4 per SM sub-partition, so 128 registers per thread fit; with 18 warps some
// sub-partitions hold 5 and the per-thread budget drops below 100): 0 loader, 1-6 dequant, 7 MMA (+TMEM alloc),
// 8-15 epilogue
namespace moe {
constexpr int W_DQ0 = 1, N_DQ = 6, W_MMA = 7, W_EP0 = 8, N_EP = 8, THREADS = 16 * 32;
}

// one dequant task = 32 codes (3 words at word offset 3*q of the row) -> 32 e4m3 bytes (2 swizzled chunks)
AFB_DEV void dequant_task(const uint32_t* row_words, uint8_t* tile, int r, int q) {
  uint32_t o[8];
  decode32(row_words[3 * q], row_words[3 * q + 1], row_words[3 * q + 2], o);
  *reinterpret_cast<uint4*>(tile + sw128_offset(r, 2 * q)) = make_uint4(o[0], o[1], o[2], o[3]);
  *reinterpret_cast<uint4*>(tile + sw128_offset(r, 2 * q + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
}

template <bool PAIR, bool F8>
__global__ void __launch_bounds__(moe::THREADS, 1)
    moe_int3_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                         MoeGemmArgs args, uint32_t* status) {
  using L = moe::Layout<PAIR, F8>;
  constexpr int RS = L::RS, AS = L::AS, NBUF = L::NBUF;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + RS;
  uint64_t* afull = empty + RS;
  uint64_t* aempty = afull + AS;
  uint64_t* dfull = aempty + AS;
  uint64_t* dempty = dfull + NBUF;
  uint64_t* sready = dempty + NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sready + NBUF);
  int* off = reinterpret_cast<int*>(smem + L::OFFS_OFF);
  float* red = reinterpret_cast<float*>(smem + L::RED_OFF);  // [2 halves][4 quads][16 tokens] amax exchange

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = args.num_experts;
  const int NB = args.rows / 128 / (PAIR ? 2 : 1);  // units per expert
  const int KG = args.K / 128;                       // k-steps (groups) per chunk
  const int units = E * NB;

  for (int e = threadIdx.x; e <= E; e += blockDim.x) off[e] = args.expert_offsets[e];
  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], moe::N_DQ + 1);  // dequant warps (codes and scales read) + MMA commit (X read)
    }
    for (int s = 0; s < AS; ++s) {
      mbar_init(&afull[s], moe::N_DQ);
      mbar_init(&aempty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&dfull[b], 1);
      mbar_init(&dempty[b], moe::N_EP);
      mbar_init(&sready[b], moe::N_DQ);
    }
    fence_mbar_init();
  }
  if (warp == moe::W_MMA) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // every role walks the same (unit, chunk, group) sequence
  uint32_t kstep = 0;
  bool bail = false;
  long long t_wait = 0;  // profiling counters (args.dbg): cycles spent in waits by this role
  const long long t_start = clock64();
#define AFB_TIMED_WAIT(expr) ([&]() { const long long _t = clock64(); const bool _r = (expr); t_wait += clock64() - _t; return _r; }())
  for (int u = blockIdx.x; u < units && !bail; u += gridDim.x) {
    const int e = u % E, j = u / E;  // neighbouring CTAs take different experts
    const int row0 = off[e], n = off[e + 1] - row0;
    const int nchunks = (n + moe::NTOK - 1) / moe::NTOK;
    for (int ch = 0; ch < nchunks && !bail; ++ch) {
      const int crow = row0 + ch * moe::NTOK;
      const int cn = min(moe::NTOK, n - ch * moe::NTOK);
      if (warp == 0) {
        // ---------------------------------------------------------------- loader
        if (lane == 0) {
          for (int g = 0; g < KG; ++g, ++kstep) {
            const int s = kstep % RS;
            const uint32_t ph = (kstep / RS) & 1;
            if (kstep >= (uint32_t)RS && !AFB_TIMED_WAIT(mbar_wait(&empty[s], ph ^ 1, status))) {
              bail = true;
              break;
            }
            uint8_t* st = smem + s * L::RAW;
            mbar_arrive_expect_tx(&full[s], F8 ? L::T * moe::A_TILE + moe::X_TILE + moe::NTOK * 4
                                               : L::T * (moe::CODE_TILE + 256) + moe::X_TILE + moe::NTOK * 4);
            // activation scales of this group for the chunk's 32 rows (group-major, segment starts 8-aligned)
            bulk_g2s(st + L::SX_OFF, args.x_scales + (size_t)g * args.ld_xs + crow, moe::NTOK * 4, &full[s]);
#pragma unroll
            for (int t = 0; t < L::T; ++t) {
              const int rb = PAIR ? (t == 0 ? j : NB + j) : j;  // gate block j, up block NB + j
              if constexpr (F8) {
                tma_load_2d(st + L::WA_OFF + t * moe::A_TILE, &tmW, &full[s], g * 128, e * args.rows + rb * 128);
              } else {
                const size_t tile = ((size_t)e * (args.rows / 128) + rb) * KG + g;
                bulk_g2s(st + L::C_OFF + t * moe::CODE_TILE, args.codes + tile * (moe::CODE_TILE / 4),
                         moe::CODE_TILE, &full[s]);
                bulk_g2s(st + L::SW_OFF + t * 256, reinterpret_cast<const uint16_t*>(args.scales) + tile * 128, 256,
                         &full[s]);
              }
            }
            tma_load_2d(st + L::X_OFF, &tmX, &full[s], g * 128, crow);
          }
        }
        __syncwarp();
        bail = __shfl_sync(0xffffffffu, bail, 0);
      } else if (warp >= moe::W_DQ0 && warp < moe::W_DQ0 + moe::N_DQ) {
        // ---------------------------------------------------------------- dequant: 192 threads, 32-code tasks
        const int dq = threadIdx.x - 32 * moe::W_DQ0;  // 0..191
        constexpr int NT = moe::N_DQ * 32;
        constexpr int TASKS = L::T * 128 * 4;         // (tile, row, 32-code sub-group)
        for (int g = 0; g < KG; ++g, ++kstep) {
          const int s = kstep % RS;
          const int as = kstep % AS;
          const int b = kstep % NBUF;
          bool ok = AFB_TIMED_WAIT(mbar_wait(&full[s], (kstep / RS) & 1, status));
          if (ok && kstep >= (uint32_t)AS) ok = AFB_TIMED_WAIT(mbar_wait(&aempty[as], ((kstep / AS) & 1) ^ 1, status));
          if (ok && kstep >= (uint32_t)NBUF)
            ok = AFB_TIMED_WAIT(mbar_wait(&dempty[b], ((kstep / NBUF) & 1) ^ 1, status));
          if (!ok) {
            bail = true;
            break;
          }
          const uint8_t* st = smem + s * L::RAW;
          uint8_t* at = smem + L::A_OFF + as * L::A_STAGE;
          if constexpr (F8) {  // nothing to decode: only the scales move to the epilogue's slot b
            float* dst = reinterpret_cast<float*>(smem + L::ESC_OFF + b * L::ESC);
            if (dq < L::T) {
              const int rb = PAIR ? (dq == 0 ? j : NB + j) : j;
              dst[dq] = args.fp8_scales[((size_t)e * (args.rows / 128) + rb) * KG + g];
            } else if (dq >= 32 && dq < 32 + moe::NTOK) {
              dst[4 + dq - 32] = reinterpret_cast<const float*>(st + L::SX_OFF)[dq - 32];
            }
            __syncwarp();
            if (lane == 0) {
              mbar_arrive(&afull[as]);
              mbar_arrive(&sready[b]);
              mbar_arrive(&empty[s]);
            }
            continue;
          }
          {  // the group's scales move to the epilogue's ring slot b, so the raw stage can be refilled early
            constexpr int SW_WORDS = L::T * 64, WORDS = SW_WORDS + moe::NTOK;
            uint32_t* dst = reinterpret_cast<uint32_t*>(smem + L::ESC_OFF + b * L::ESC);
            if (dq < WORDS)
              dst[dq] = dq < SW_WORDS ? reinterpret_cast<const uint32_t*>(st + L::SW_OFF)[dq]
                                      : reinterpret_cast<const uint32_t*>(st + L::SX_OFF)[dq - SW_WORDS];
          }
          {  // all code words of this thread's tasks are loaded first (independent loads in flight), then decoded
            constexpr int PER = (TASKS + NT - 1) / NT;
            uint32_t w[PER][3];
#pragma unroll
            for (int i = 0; i < PER; ++i) {
              const int task = dq + i * NT;
              if (task < TASKS) {
                const int t = task >> 9, r = (task >> 2) & 127, sq = task & 3;
                const uint32_t* rw = reinterpret_cast<const uint32_t*>(st + L::C_OFF + t * moe::CODE_TILE) + r * 12;
                w[i][0] = rw[3 * sq];
                w[i][1] = rw[3 * sq + 1];
                w[i][2] = rw[3 * sq + 2];
              }
            }
#pragma unroll
            for (int i = 0; i < PER; ++i) {
              const int task = dq + i * NT;
              if (task < TASKS) {
                const int t = task >> 9, r = (task >> 2) & 127, sq = task & 3;
                uint32_t o[8];
                decode32(w[i][0], w[i][1], w[i][2], o);
                uint8_t* tile = at + t * moe::A_TILE;
                *reinterpret_cast<uint4*>(tile + sw128_offset(r, 2 * sq)) = make_uint4(o[0], o[1], o[2], o[3]);
                *reinterpret_cast<uint4*>(tile + sw128_offset(r, 2 * sq + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
              }
            }
          }
          fence_proxy_async_smem();  // generic-proxy smem writes -> visible to the tensor core
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&afull[as]);
            mbar_arrive(&sready[b]);
            mbar_arrive(&empty[s]);
          }
        }
      } else if (warp == moe::W_MMA) {
        // ---------------------------------------------------------------- MMA
        constexpr uint32_t idesc = idesc_e4m3(128, moe::NTOK);
        for (int g = 0; g < KG; ++g, ++kstep) {
          const int s = kstep % RS;
          const int as = kstep % AS;
          const int b = kstep % NBUF;
          bool ok = AFB_TIMED_WAIT(mbar_wait(&afull[as], (kstep / AS) & 1, status));
          if (ok && kstep >= (uint32_t)NBUF) ok = AFB_TIMED_WAIT(mbar_wait(&dempty[b], ((kstep / NBUF) & 1) ^ 1, status));
          if (!ok) {
            bail = true;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint8_t* st = smem + s * L::RAW;
            const uint8_t* at = F8 ? st + L::WA_OFF : smem + L::A_OFF + as * L::A_STAGE;
            const uint64_t dx = sw128_desc(smem_u32(st + L::X_OFF));
#pragma unroll
            for (int t = 0; t < L::T; ++t) {
              const uint64_t da = sw128_desc(smem_u32(at + t * moe::A_TILE));
              const uint32_t d = tmem + (uint32_t)((b * L::T + t) * moe::NTOK);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) umma_f8(d, da + 2 * kk, dx + 2 * kk, idesc, kk != 0);
            }
            umma_commit(&dfull[b]);
            umma_commit(&aempty[as]);
            umma_commit(&empty[s]);
          }
          __syncwarp();
        }
      } else {
        // ---------------------------------------------------------------- epilogue (warps 8..15)
        // each TMEM lane quadrant is read by two warps: half 0 takes token columns 0..15, half 1 columns 16..31
        const int quad = warp & 3;
        const int half = (warp - moe::W_EP0) >> 2;
        const int r = quad * 32 + lane;  // TMEM lane = row of the weight tile
        constexpr int NH = moe::NTOK / 2;
        float acc0[NH], acc1[PAIR ? NH : 1];
#pragma unroll
        for (int i = 0; i < NH; ++i) acc0[i] = 0.f;
#pragma unroll
        for (int i = 0; i < (PAIR ? NH : 1); ++i) acc1[i] = 0.f;
        // w2: the chunk's entry indices and routing weights are fetched now, as independent loads, so they are in
        // registers when the K loop ends (fetched inside the store loop they were a chain of dependent misses)
        int ent[PAIR ? 1 : NH];
        float rwt[PAIR ? 1 : NH];
        if constexpr (!PAIR) {
#pragma unroll
          for (int i = 0; i < NH; ++i) {
            const int row = crow + half * NH + i;
            ent[i] = (half * NH + i < cn && args.row_entry) ? args.row_entry[row] : -1;
          }
#pragma unroll
          for (int i = 0; i < NH; ++i) rwt[i] = args.route_w ? (ent[i] >= 0 ? args.route_w[ent[i]] : 0.f) : 1.f;
        }
        for (int g = 0; g < KG; ++g, ++kstep) {
          const int b = kstep % NBUF;
          const uint32_t ph = (kstep / NBUF) & 1;
          if (!AFB_TIMED_WAIT(mbar_wait(&dfull[b], ph, status) && mbar_wait(&sready[b], ph, status))) {
            bail = true;
            break;
          }
          tc_fence_after();
          const uint8_t* esc = smem + L::ESC_OFF + b * L::ESC;  // INT3: [T][128] bf16 s_w, [32] fp32 s_x
          const float* sx = reinterpret_cast<const float*>(esc + (F8 ? 16 : L::T * 256)) + half * NH;
          const float sw0 = F8 ? reinterpret_cast<const float*>(esc)[0]
                               : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(esc)[r]);
          const float sw1 = !PAIR ? 0.f
                            : F8 ? reinterpret_cast<const float*>(esc)[1]
                                 : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(esc + 256)[r]);
          const uint32_t ta = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * L::T * moe::NTOK + half * NH);
          float d[NH];  // one 16-column load at a time keeps the role inside 128 registers
          tmem_ld16(ta, d);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < NH; ++i) acc0[i] = fmaf(sw0 * sx[i], d[i], acc0[i]);
          if (PAIR) {
            tmem_ld16(ta + moe::NTOK, d);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < NH; ++i) acc1[i] = fmaf(sw1 * sx[i], d[i], acc1[i]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dempty[b]);  // TMEM buffer b and scale slot b are free again
        }
        if (bail) break;
        const int t0 = half * NH;  // first token column of this warp
        if (PAIR) {
          // h = silu(gate) * up -> e4m3 with a scale per (token, this 128-column group)
          const int col = j * 128 + r;  // intermediate column
          float* rd = red + half * 4 * NH;
#pragma unroll
          for (int i = 0; i < NH; ++i) {
            acc0[i] = silu(acc0[i]) * acc1[i];
            const float m = warp_max(fabsf(acc0[i]));
            if (lane == 0) rd[quad * NH + i] = m;
          }
          named_bar(1 + half, 128);
#pragma unroll
          for (int i = 0; i < NH; ++i) {
            if (t0 + i >= cn) break;
            const float amax = fmaxf(fmaxf(rd[i], rd[NH + i]), fmaxf(rd[2 * NH + i], rd[3 * NH + i]));
            const float sc = amax > 0.f ? amax / 448.f : 1.f;
            const __nv_fp8_e4m3 q(acc0[i] / sc);
            args.out_q[(size_t)(crow + t0 + i) * args.out_ld + col] = *reinterpret_cast<const uint8_t*>(&q);
            if (r == 0) args.out_scales[(size_t)j * args.ld_os + crow + t0 + i] = sc;
          }
          named_bar(1 + half, 128);  // rd is reused by the next chunk
        } else {
          const int col = j * 128 + r;  // hidden column
#pragma unroll
          for (int i = 0; i < NH; ++i) {
            if (t0 + i >= cn) break;
            const int entry = ent[PAIR ? 0 : i];  // -1: segment padding
            if (args.ep_world > 0) {
              if (entry < 0) continue;
              const int dst = entry / args.ep_entries_per_rank, le = entry - dst * args.ep_entries_per_rank;
              reinterpret_cast<__nv_bfloat16*>(args.ep_peer[dst] + args.ep_off_comb)[(size_t)le * args.out_ld + col] =
                  __float2bfloat16(acc0[i] * rwt[PAIR ? 0 : i]);
              continue;
            }
            reinterpret_cast<__nv_bfloat16*>(args.out_bf16)[(size_t)(crow + t0 + i) * args.out_ld + col] =
                __float2bfloat16(acc0[i] * rwt[PAIR ? 0 : i]);
          }
        }
      }
    }
  }
#undef AFB_TIMED_WAIT
  if (args.dbg && lane == 0 && (warp == 0 || warp == moe::W_DQ0 || warp == moe::W_MMA || warp == moe::W_EP0)) {
    const int role = warp == 0 ? 0 : warp == moe::W_DQ0 ? 1 : warp == moe::W_MMA ? 2 : 3;
    args.dbg[(blockIdx.x * 4 + role) * 3 + 0] = t_wait;
    args.dbg[(blockIdx.x * 4 + role) * 3 + 1] = clock64() - t_start;
    args.dbg[(blockIdx.x * 4 + role) * 3 + 2] = kstep;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == moe::W_MMA) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
  if (!PAIR && args.ep_world > 0) {  // publish the combine exchange once every CTA's peer stores are out
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(args.ep_done, 1u) == gridDim.x - 1) {
      *args.ep_done = 0;
      __threadfence_system();
      const uint64_t v = ++*args.ep_sent;
      for (int p = 0; p < args.ep_world; ++p)
        st_release_sys_u64(reinterpret_cast<uint64_t*>(args.ep_peer[p] + args.ep_off_flags) + 8 + args.ep_rank, v);
    }
  }
}

template <bool PAIR, bool F8>
static int launch_moe(const CUtensorMap& tx, const CUtensorMap& tw, const MoeGemmArgs& a, int grid, uint32_t* status,
                      cudaStream_t st) {
  using L = moe::Layout<PAIR, F8>;
  static std::atomic<uint64_t> attr_devs{0};
  if (const int e = smem_attr_once(attr_devs, (const void*)moe_int3_gemm_kernel<PAIR, F8>, L::TOTAL)) return e;
  moe_int3_gemm_kernel<PAIR, F8><<<grid, moe::THREADS, L::TOTAL, st>>>(tx, tw, a, status);
  return (int)cudaGetLastError();
}

int moe_int3_gemm(const MoeGemmArgs& a, int pair, int num_sms, uint32_t* status, cudaStream_t st) {
  if (a.K % 128 || a.rows % (pair ? 256 : 128) || a.num_experts > moe::MAX_E) return 3;
  if (a.num_rows_total <= 0) return 0;
  CUtensorMap tx, tw;
  int rc = make_tmap_2d(&tx, a.x_q, 1, a.K, a.num_rows_total, (uint64_t)a.K, 128, moe::NTOK, 1);
  if (rc) return 1000 + rc;
  if (a.fp8_w) {  // e4m3 weights [E * rows, K]: 128 x 128 tiles, 128-byte swizzle (the MMA's A layout)
    if (!a.fp8_scales) return 3;
    rc = make_tmap_2d(&tw, a.fp8_w, 1, a.K, (uint64_t)a.num_experts * a.rows, (uint64_t)a.K, 128, 128, 1);
    if (rc) return 2000 + rc;
  } else {
    tw = tx;  // unused by the INT3 kernels
  }
  const int units = a.num_experts * (a.rows / 128 / (pair ? 2 : 1));
  const int grid = units < num_sms ? units : num_sms;
  if (a.fp8_w) return pair ? launch_moe<true, true>(tx, tw, a, grid, status, st)
                           : launch_moe<false, true>(tx, tw, a, grid, status, st);
  return pair ? launch_moe<true, false>(tx, tw, a, grid, status, st)
              : launch_moe<false, false>(tx, tw, a, grid, status, st);
}

}  // namespace afb
