// INT3 (uint3 g128) routed-expert grouped GEMM, W3A8, on tcgen05 (kind::f8f6f4) with TMEM accumulators; the same
// kernel runs block-FP8 experts (the QAD teacher's format).
//
// Contract (the reference's serving W3A8, training/work/qwen38fn_lora/int3_moe.py:1-14, i.e. Humming's
// quant_input(group_size=row)): weight code c in 0..7 means (c - 4) * s_w with a signed scale per (row, 128-column
// group); activations are e4m3 with ONE fp32 scale per token row, s_x = max(amax, 1e-30) / 448; e4m3 x e4m3
// products accumulate in fp32, each group's partial sum is scaled by its s_w as it joins the running sum and the
// row scale s_x is applied at the end. (c - 4) in -4..3 is exact in e4m3, so the tensor-core operand is lossless.
// Between the two GEMMs the SwiGLU output is stored in bf16 and quantised per row again (quant_rows_e4m3), as the
// reference's server does. Block-FP8 experts use 1 x 128 activation scales and 128 x 128 weight scales instead
// (both applied per group) and keep the e4m3-per-128 SwiGLU output of w13.
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
// Routing: the router appends each (token, slot) entry to its expert's list (per source rank under expert
// parallelism); a work unit is (expert, 256 weight rows as two 128-row tiles) x chunks of 32 of the expert's entries,
// whose activation rows are gathered straight from the token rows (w13) or the entry rows (w2) -- no sort, no
// gathered copy. Outputs are written per entry. w13 pairs gate block j with up block j + I/128 (SwiGLU in the
// epilogue), w2 takes output blocks 2j and 2j+1. One persistent CTA per SM, warp-specialised so that every SM
// sub-partition (warp % 4) carries the same share of the decode and epilogue:
//   warp 0      loader: bulk copies of the code / scale tiles (lane 0); the 32 lanes gather the chunk's 32
//               activation rows with 16-byte async copies into the 128-byte-swizzled B tile (no multicast)
//   warp 1      MMA: M=128 (weight rows) x N=32 (tokens) x K=32 per op, one 128-K group per accumulator buffer
//   warp 2      chunk metadata: per chunk the 32 entries and their activation scales (x routing weights for w2)
//               into a shared-memory ring, so the epilogue holds none of them in registers
//   warps 4-11  dequant: one weight row (128 codes, three 16-byte shared loads) per thread and k-step ->
//               e4m3 (c - 4) written straight into tensor memory (tcgen05.st, warp w owns TMEM lane quadrant
//               w % 4), where the MMA reads its A operand -- no shared-memory tile, no proxy fence; warps 4-7 also
//               copy the group's weight scales to the epilogue's slot
//   warps 12-15 epilogue, one per TMEM lane quadrant, all 32 token columns: per group acc += s_w * D; at the end of
//               a chunk w13: h = silu(gate * s_x) * (up * s_x) -> bf16; w2: y = acc * s_x * route weight -> bf16
//               (or into the token owner's combine region on a peer under expert parallelism)
// A ring of raw stages (bulk copies in flight) feeds a ring of dequantised A tiles in TMEM; the MMA runs up to 4
// groups ahead of the epilogue, and a raw stage is released once dequant and MMA are done with it (never waits on
// the epilogue). Ring positions advance incrementally (no division in the loop), and a producer's first lap waits on
// the opposite parity of a fresh barrier, which completes at once.
#include <cudaTypedefs.h>

#include <cstring>

#include "common.cuh"
#include "gemm.h"
#include "moe.h"

namespace afb {

namespace moe {
constexpr int NTOK = 32;                  // tokens per chunk = MMA N
constexpr int T = 2;                      // weight tiles per unit
constexpr uint32_t CODE_TILE = 128 * 48;  // bytes of one 128-row x 128-K code tile
constexpr uint32_t A_TILE = 128 * 128;    // e4m3 128x128
constexpr uint32_t X_TILE = NTOK * 128;   // e4m3 32x128
constexpr uint32_t E4M3_LO = 0xB8C0C4C8u; // table bytes 0..3: e4m3(-4), e4m3(-3), e4m3(-2), e4m3(-1)
constexpr uint32_t E4M3_HI = 0x44403800u; // table bytes 4..7: e4m3(0), e4m3(1), e4m3(2), e4m3(3)
constexpr int MAX_SRC = 8;                // source ranks of the routing lists
constexpr int W_LD = 0, W_MMA = 1, W_META = 2, W_DQ0 = 4, N_DQ = 8, W_EP0 = 12, N_EP = 4, THREADS = 16 * 32;
constexpr int MS = 4;                     // chunk-metadata ring slots
constexpr uint32_t META = 256;            // per slot: float scale[32], int entry[32]

template <bool F8>
struct Layout {
  static constexpr uint32_t X_OFF = 0;  // 1024-aligned (TMA 128-byte swizzle)
  // INT3: code tiles (bulk copies) then per-row bf16 weight scales. F8: the e4m3 weight tiles themselves (TMA,
  // swizzled: they are the MMA's A operand as they land) then the chunk's 1 x 128 activation scales of the group.
  static constexpr uint32_t C_OFF = X_OFF + X_TILE;
  static constexpr uint32_t WA_OFF = X_OFF + X_TILE;
  static constexpr uint32_t SW_OFF = C_OFF + T * CODE_TILE;
  static constexpr uint32_t RAW_BYTES = F8 ? WA_OFF + T * A_TILE : SW_OFF + T * 128 * 2;
  static constexpr uint32_t RAW = (RAW_BYTES + 1023) & ~1023u;
  static constexpr int RS = F8 ? 5 : 12;   // raw stages
  static constexpr int AS = F8 ? 3 : 4;    // dequantised A stages (INT3: in TMEM; F8: barriers only)
  static constexpr int NBUF = F8 ? 8 : 4;  // TMEM accumulator buffers of T * 32 columns
  static constexpr uint32_t ACC_COLS = NBUF * T * NTOK;
  static constexpr uint32_t A_COL = ACC_COLS;  // INT3: A stages after the accumulators, T * 32 columns each
  static_assert(ACC_COLS + (F8 ? 0 : AS * T * 32) <= 512, "TMEM columns");
  static constexpr uint32_t ESC = 512;   // per-buffer copy of the group's scales (INT3: T*128 bf16 s_w; F8: T fp32
                                         // block scales, then 32 fp32 s_x at byte 16)
  static constexpr uint32_t ESC_OFF = RS * RAW;
  static constexpr uint32_t META_OFF = ESC_OFF + NBUF * ESC;
  static constexpr uint32_t RED_OFF = META_OFF + MS * META;         // float [4 quads][32 tokens] (F8 amax)
  static constexpr uint32_t BAR_OFF = (RED_OFF + 4 * NTOK * 4 + 7) & ~7u;
  // full[RS], empty[RS], afull[AS], aempty[AS], dfull[NBUF], dempty[NBUF], sready[NBUF], mfull[MS], mempty[MS],
  // tmem slot
  static constexpr uint32_t TOTAL = BAR_OFF + (2 * RS + 2 * AS + 3 * NBUF + 2 * MS) * 8 + 16 + 1024;
  static constexpr uint32_t TMEM_COLS = 512;
};

// position in a ring of N barriers: slot and the parity of the current lap
template <int N>
struct Ring {
  uint32_t i = 0, ph = 0;
  AFB_DEV void next() {
    if (++i == (uint32_t)N) {
      i = 0;
      ph ^= 1u;
    }
  }
};
}  // namespace moe

AFB_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

AFB_DEV void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// the arrive of this thread's async copies (cp_async16) on an mbarrier (counted in the barrier's expected arrivals)
AFB_DEV void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// The entries of one expert over the sources' lists, read by a whole warp: n (total), and entry number i of the
// concatenation (sources in rank order), or -1 past the end.
struct MoeRoute {
  int n, cnt, start;  // lane p < srcs: that source's count and start in the concatenation
  AFB_DEV void load(const MoeGemmArgs& a, int E, int e) {
    const int lane = threadIdx.x & 31;
    cnt = lane < a.route_srcs ? a.route_cnt[lane * E + e] : 0;
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < moe::MAX_SRC; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    start = incl - cnt;
    n = __shfl_sync(0xffffffffu, incl, moe::MAX_SRC - 1);
  }
  AFB_DEV int entry(const MoeGemmArgs& a, int E, int e, int i) const {  // every lane its own i; warp-wide call
    int res = -1;
#pragma unroll
    for (int p = 0; p < moe::MAX_SRC; ++p) {
      const int s0 = __shfl_sync(0xffffffffu, start, p), c0 = __shfl_sync(0xffffffffu, cnt, p);
      if (p < a.route_srcs && i >= s0 && i < s0 + c0)
        res = a.route_list[((size_t)p * E + e) * a.route_cap + (i - s0)];
    }
    return res;
  }
};

// Shifts done as integer multiplies (x * 2^k, high word of x * 2^(32-k)) run on the FMA pipe, which the decode
// leaves idle, instead of the integer ALU pipe that the masks and byte-permutes already fill.
AFB_DEV uint32_t shl_f(uint32_t x, uint32_t k) {
  uint32_t r;
  asm("mul.lo.u32 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(1u << k));
  return r;
}
AFB_DEV uint32_t shr_f(uint32_t x, uint32_t k) {
  uint32_t r;
  asm("mul.hi.u32 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(1u << (32 - k)));
  return r;
}

// 32 codes (3 words of the tile layout) -> 32 e4m3 bytes (8 words), in code order
AFB_DEV void decode32(uint32_t L0, uint32_t L1, uint32_t H, uint32_t* o) {
  const uint32_t s0 = (L0 & 0x33333333u) | (H & 0x44444444u);
  const uint32_t s1 = (shr_f(L0, 2) & 0x33333333u) | (shr_f(H, 1) & 0x44444444u);
  const uint32_t s2 = (L1 & 0x33333333u) | (shl_f(H, 2) & 0x44444444u);
  const uint32_t s3 = (shr_f(L1, 2) & 0x33333333u) | (shl_f(H, 1) & 0x44444444u);
  o[0] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, s0);
  o[1] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, shr_f(s0, 16));
  o[2] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, s1);
  o[3] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, shr_f(s1, 16));
  o[4] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, s2);
  o[5] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, shr_f(s2, 16));
  o[6] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, s3);
  o[7] = __byte_perm(moe::E4M3_LO, moe::E4M3_HI, shr_f(s3, 16));
}

template <bool PAIR, bool F8, bool PROF>
__global__ void __launch_bounds__(moe::THREADS, 1)
    moe_int3_gemm_kernel(const __grid_constant__ CUtensorMap tmW, MoeGemmArgs args, uint32_t* status) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  using L = moe::Layout<F8>;
  constexpr int RS = L::RS, AS = L::AS, NBUF = L::NBUF, T = moe::T, NT = moe::NTOK, MS = moe::MS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + RS;
  uint64_t* afull = empty + RS;
  uint64_t* aempty = afull + AS;
  uint64_t* dfull = aempty + AS;
  uint64_t* dempty = dfull + NBUF;
  uint64_t* sready = dempty + NBUF;
  uint64_t* mfull = sready + NBUF;
  uint64_t* mempty = mfull + MS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mempty + MS);
  float* red = reinterpret_cast<float*>(smem + L::RED_OFF);  // [4 quads][32 tokens] amax exchange (F8 w13)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = args.num_experts;
  const int NB = args.rows / 256;  // units per expert
  const int KG = args.K / 128;     // k-steps (groups) per chunk
  const int units = E * NB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; ++s) {
      mbar_init(&full[s], 1 + 32);          // loader lane 0 (+ bulk-copy bytes) and the 32 gathering lanes
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
    for (int m = 0; m < MS; ++m) {
      mbar_init(&mfull[m], 1);
      mbar_init(&mempty[m], moe::N_EP);
    }
    fence_mbar_init();
    if (args.ep_wait_flags) {  // the routed rows of every source rank have landed in this rank's heap
      const uint64_t want = *args.ep_expected + 1;
      const uint64_t tw0 = globaltimer_ns();
      for (int p = 0; p < args.route_srcs; ++p) {
        const uint64_t t0 = globaltimer_ns();
        uint32_t polls = 0;
        while (ld_acquire_sys_u64(args.ep_wait_flags + p) < want) {
          if ((++polls & 63) == 0 && globaltimer_ns() - t0 > AFB_WAIT_NS) {
            flag_error(status, AFB_ERR_PEER_TIMEOUT);
            break;
          }
          __nanosleep(64);
        }
      }
      if (args.ep_wait_ns && blockIdx.x == 0) atomicAdd(args.ep_wait_ns, (unsigned long long)(globaltimer_ns() - tw0));
    }
  }
  if (warp == moe::W_MMA) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // every role walks the same (unit, chunk, group) sequence, each with its own ring positions
  moe::Ring<RS> rs;
  moe::Ring<AS> ra;
  moe::Ring<NBUF> rb;
  moe::Ring<MS> rm;
  uint32_t ksteps = 0;
  bool bail = false;
  long long t_wait = 0;  // profiling counters (PROF only): cycles spent in waits by this role
  long long t_sec = 0, t_sec2 = 0;  // PROF: cycles in the role's main work (see the role) and a second section
  const long long t_start = PROF ? clock64() : 0;
  auto clk = [&]() -> long long { return PROF ? clock64() : 0; };
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if constexpr (PROF) {
      const long long t0 = clock64();
      const bool ok = mbar_wait(bar, parity, status);
      t_wait += clock64() - t0;
      return ok;
    } else {
      return mbar_wait(bar, parity, status);
    }
  };
  const bool active = warp == moe::W_LD || warp == moe::W_MMA || warp == moe::W_META || warp >= moe::W_DQ0;
  MoeRoute route;
  for (int u = blockIdx.x; u < units && !bail && active; u += gridDim.x) {
    const int e = u % E, j = u / E;  // neighbouring CTAs take different experts
    route.load(args, E, e);
    const int n = route.n;
    const int nchunks = (n + NT - 1) / NT;
    for (int ch = 0; ch < nchunks && !bail; ++ch) {
      const int cn = min(NT, n - ch * NT);
      if (warp == moe::W_LD) {
        // ---------------------------------------------------------------- loader
        const int ent = route.entry(args, E, e, ch * NT + lane);  // lane l: the chunk's entry l (or -1)
        const uint8_t* xrow = reinterpret_cast<const uint8_t*>(args.x_q) +
                              (size_t)(ent >= 0 ? ent / args.x_div : 0) * args.K;
        const uint32_t xbytes = ent >= 0 ? 16u : 0u;  // zero-filled rows past the chunk
        for (int g = 0; g < KG; ++g, rs.next()) {
          if (lane == 0) bail = !wait(&empty[rs.i], rs.ph ^ 1);
          bail = __shfl_sync(0xffffffffu, bail, 0);
          if (bail) break;
          uint8_t* st = smem + rs.i * L::RAW;
          uint64_t* bar = &full[rs.i];
          const long long c0 = clk();
          if (lane == 0) {
            mbar_arrive_expect_tx(bar, F8 ? T * moe::A_TILE : T * (moe::CODE_TILE + 256));
#pragma unroll
            for (int t = 0; t < T; ++t) {
              const int rblk = PAIR ? (t == 0 ? j : NB + j) : 2 * j + t;  // gate block j / up block NB + j
              if constexpr (F8) {
                tma_load_2d(st + L::WA_OFF + t * moe::A_TILE, &tmW, bar, g * 128, e * args.rows + rblk * 128);
              } else {
                const size_t tile = ((size_t)e * (args.rows / 128) + rblk) * KG + g;
                bulk_g2s(st + L::C_OFF + t * moe::CODE_TILE, args.codes + tile * (moe::CODE_TILE / 4),
                         moe::CODE_TILE, bar);
                bulk_g2s(st + L::SW_OFF + t * 256, reinterpret_cast<const uint16_t*>(args.scales) + tile * 128, 256,
                         bar);
              }
            }
          }
          // this lane's activation row: 8 chunks of 16 bytes into row `lane` of the swizzled B tile
          uint8_t* xt = st + L::X_OFF + lane * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) cp_async16(xt + ((c ^ (lane & 7)) << 4), xrow + g * 128 + c * 16, xbytes);
          cp_async_arrive(bar);
          t_sec += clk() - c0;
        }
      } else if (warp == moe::W_META) {
        // ---------------------------------------------------------------- chunk metadata
        const int ent = route.entry(args, E, e, ch * NT + lane);
        if (!wait(&mempty[rm.i], rm.ph ^ 1)) {
          bail = true;
          break;
        }
        float* ms = reinterpret_cast<float*>(smem + L::META_OFF + rm.i * moe::META);
        int* me = reinterpret_cast<int*>(ms + NT);
        float sc = 0.f;
        if (ent >= 0) {
          sc = F8 ? 1.f : args.x_scales[ent / args.x_div];  // INT3: per-row activation scale
          if (!PAIR && args.route_w) sc *= args.route_w[ent];
        }
        ms[lane] = sc;
        me[lane] = ent >= 0 ? ent : -2;  // -2: column beyond the chunk
        __syncwarp();
        if (lane == 0) mbar_arrive(&mfull[rm.i]);  // release: the warp's stores are ordered before it
        rm.next();
      } else if (warp >= moe::W_DQ0 && warp < moe::W_DQ0 + moe::N_DQ) {
        // ---------------------------------------------------------------- dequant: a weight row per thread
        const int dq = threadIdx.x - 32 * moe::W_DQ0;  // 0..255
        const int quad = warp & 3, t = (warp - moe::W_DQ0) >> 2;
        const int r = quad * 32 + lane;  // row of tile t = TMEM lane
        int xrow = 0;  // F8: the row of this lane's chunk column (warp W_DQ0 + 1 gathers the activation scales)
        if (F8 && warp == moe::W_DQ0 + 1) {
          const int ent = route.entry(args, E, e, ch * NT + lane);
          xrow = ent >= 0 ? ent / args.x_div : -1;
        }
        for (int g = 0; g < KG; ++g, rs.next(), ra.next(), rb.next()) {
          bool ok = wait(&full[rs.i], rs.ph);
          if (ok) ok = wait(&aempty[ra.i], ra.ph ^ 1);
          if (ok) ok = wait(&dempty[rb.i], rb.ph ^ 1);  // the epilogue is done with scale slot rb.i
          if (!ok) {
            bail = true;
            break;
          }
          const uint8_t* st = smem + rs.i * L::RAW;
          uint8_t* esc = smem + L::ESC_OFF + rb.i * L::ESC;
          if constexpr (F8) {  // nothing to decode: the block scales and the chunk's activation scales move to slot
            float* dst = reinterpret_cast<float*>(esc);
            if (dq < T) {
              const int rblk = PAIR ? (dq == 0 ? j : NB + j) : 2 * j + dq;
              dst[dq] = args.fp8_scales[((size_t)e * (args.rows / 128) + rblk) * KG + g];
            } else if (warp == moe::W_DQ0 + 1) {
              dst[4 + lane] = xrow >= 0 ? args.x_scales[(size_t)g * args.ld_xs + xrow] : 0.f;
            }
            __syncwarp();
          } else {
            // the group's weight scales move to the epilogue's slot, so the raw stage can be refilled early
            if (dq < T * 64) reinterpret_cast<uint32_t*>(esc)[dq] = reinterpret_cast<const uint32_t*>(st + L::SW_OFF)[dq];
            const long long c0 = clk();
            const uint4* rw = reinterpret_cast<const uint4*>(st + L::C_OFF + t * moe::CODE_TILE + r * 48);
            const uint4 w0 = rw[0], w1 = rw[1], w2 = rw[2];  // the row's 12 words (128 codes)
            uint32_t o[32];
            decode32(w0.x, w0.y, w0.z, o);
            decode32(w0.w, w1.x, w1.y, o + 8);
            decode32(w1.z, w1.w, w2.x, o + 16);
            decode32(w2.y, w2.z, w2.w, o + 24);
            // row r of the A tile: 32 columns of 4 e4m3 each, in K order
            const long long c1 = clk();
            tmem_st32(tmem + ((uint32_t)(quad * 32) << 16) + L::A_COL + (ra.i * T + t) * 32, o);
            tmem_st_wait();
            t_sec += c1 - c0;
            t_sec2 += clk() - c1;
            tc_fence_before();
            __syncwarp();
          }
          if (lane == 0) {
            mbar_arrive(&afull[ra.i]);
            mbar_arrive(&sready[rb.i]);
            mbar_arrive(&empty[rs.i]);
          }
        }
      } else if (warp == moe::W_MMA) {
        // ---------------------------------------------------------------- MMA
        constexpr uint32_t idesc = idesc_e4m3(128, NT);
        for (int g = 0; g < KG; ++g, rs.next(), ra.next(), rb.next()) {
          bool ok = wait(&afull[ra.i], ra.ph);
          if (ok) ok = wait(&dempty[rb.i], rb.ph ^ 1);
          if (!ok) {
            bail = true;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            // the B tile came in through the generic proxy (async copies observed via the barriers): order it
            // before the tensor core's reads
            const long long c0 = clk();
            fence_proxy_async_smem();
            const uint8_t* st = smem + rs.i * L::RAW;
            const uint64_t dx = sw128_desc(smem_u32(st + L::X_OFF));
            // the two tiles' accumulations alternate, so consecutive MMAs never chain on the same accumulator
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
              for (int t = 0; t < T; ++t) {
                const uint32_t d = tmem + (uint32_t)((rb.i * T + t) * NT);
                if constexpr (F8) {
                  const uint64_t da = sw128_desc(smem_u32(st + L::WA_OFF + t * moe::A_TILE));
                  umma_f8(d, da + 2 * kk, dx + 2 * kk, idesc, kk != 0);
                } else {
                  umma_f8_ta(d, tmem + L::A_COL + (ra.i * T + t) * 32 + 8 * kk, dx + 2 * kk, idesc, kk != 0);
                }
              }
            }
            const long long c1 = clk();
            umma_commit(&dfull[rb.i]);
            umma_commit(&aempty[ra.i]);
            umma_commit(&empty[rs.i]);
            t_sec += c1 - c0;
            t_sec2 += clk() - c1;
          }
          __syncwarp();
        }
      } else if (warp >= moe::W_EP0) {
        // ---------------------------------------------------------------- epilogue (warps 12..15)
        const int quad = warp & 3;
        const int r = quad * 32 + lane;  // TMEM lane = row of the weight tile
        float acc0[NT], acc1[NT];
#pragma unroll
        for (int i = 0; i < NT; ++i) acc0[i] = acc1[i] = 0.f;
        for (int g = 0; g < KG; ++g, rb.next()) {
          bool ok = wait(&dfull[rb.i], rb.ph);
          if (ok) ok = wait(&sready[rb.i], rb.ph);
          if (!ok) {
            bail = true;
            break;
          }
          tc_fence_after();
          const uint8_t* esc = smem + L::ESC_OFF + rb.i * L::ESC;
          const uint32_t ta = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(rb.i * T * NT);
          float sw0, sw1;
          const float* sx = reinterpret_cast<const float*>(esc + 16);  // F8: this group's activation scales
          if constexpr (F8) {  // block scale x 1 x 128 activation scale, both per group
            sw0 = reinterpret_cast<const float*>(esc)[0];
            sw1 = reinterpret_cast<const float*>(esc)[1];
          } else {  // weight scale per (row, group); the row scale of the activations waits for the chunk's end
            sw0 = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(esc)[r]);
            sw1 = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(esc + 256)[r]);
          }
          // 16 columns at a time keeps the role at 32 accumulators per tile plus one 16-wide load in registers
          const long long c0 = clk();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int t = q >> 1, c0 = (q & 1) * 16;
            float d[16];
            tmem_ld16(ta + t * NT + c0, d);
            tmem_ld_wait();
            float* acc = t == 0 ? acc0 : acc1;
            const float sw = t == 0 ? sw0 : sw1;
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[c0 + i] = fmaf(F8 ? sw * sx[c0 + i] : sw, d[i], acc[c0 + i]);
          }
          t_sec += clk() - c0;
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dempty[rb.i]);  // TMEM buffer and scale slot rb.i are free again
        }
        if (bail) break;
        if (!wait(&mfull[rm.i], rm.ph)) {
          bail = true;
          break;
        }
        const float* ms = reinterpret_cast<const float*>(smem + L::META_OFF + rm.i * moe::META);
        const int* me = reinterpret_cast<const int*>(ms + NT);
        if (PAIR && F8) {
          // h = silu(gate) * up -> e4m3 with a scale per (entry, this 128-column group), for the next FP8 GEMM
          const int col = j * 128 + r;  // intermediate column
#pragma unroll
          for (int i = 0; i < NT; ++i) {
            acc0[i] = silu(acc0[i]) * acc1[i];
            const float mx = warp_max(fabsf(acc0[i]));
            if (lane == 0) red[quad * NT + i] = mx;
          }
          named_bar(1, 32 * moe::N_EP);
#pragma unroll
          for (int i = 0; i < NT; ++i) {
            if (i >= cn) break;
            const int ent = me[i];
            const float amax = fmaxf(fmaxf(red[i], red[NT + i]), fmaxf(red[2 * NT + i], red[3 * NT + i]));
            const float sc = amax > 0.f ? amax / 448.f : 1.f;
            const __nv_fp8_e4m3 q(acc0[i] / sc);
            args.out_q[(size_t)ent * args.out_ld + col] = *reinterpret_cast<const uint8_t*>(&q);
            if (r == 0) args.out_scales[(size_t)j * args.ld_os + ent] = sc;
          }
          named_bar(1, 32 * moe::N_EP);  // red is reused by the next chunk
        } else if (PAIR) {
          // h = silu(gate * s_x) * (up * s_x) in fp32, stored bf16 per entry (quantised per row before w2)
          __nv_bfloat16* hp = reinterpret_cast<__nv_bfloat16*>(args.out_bf16) + j * 128 + r;
#pragma unroll
          for (int i = 0; i < NT; ++i) {
            if (i >= cn) break;
            const float sx = ms[i];
            hp[(size_t)me[i] * args.out_ld] = __float2bfloat16(silu(acc0[i] * sx) * (acc1[i] * sx));
          }
        } else {
          // y = acc * s_x * route weight (the metadata slot holds the product), bf16, one row per entry
#pragma unroll
          for (int t = 0; t < T; ++t) {
            const int col = (2 * j + t) * 128 + r;  // hidden column
#pragma unroll
            for (int i = 0; i < NT; ++i) {
              if (i >= cn) break;
              const float v = (t == 0 ? acc0[i] : acc1[i]) * ms[i];
              const int entry = me[i];
              if (args.ep_world > 0) {
                const int dst = entry / args.ep_entries_per_rank, le = entry - dst * args.ep_entries_per_rank;
                reinterpret_cast<__nv_bfloat16*>(args.ep_peer[dst] + args.ep_off_comb)[(size_t)le * args.out_ld + col] =
                    __float2bfloat16(v);
              } else {
                reinterpret_cast<__nv_bfloat16*>(args.out_bf16)[(size_t)entry * args.out_ld + col] = __float2bfloat16(v);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&mempty[rm.i]);
        rm.next();
      }
      ksteps += KG;
    }
  }
  if (PROF && args.dbg && lane == 0 &&
      (warp == moe::W_LD || warp == moe::W_DQ0 || warp == moe::W_MMA || warp == moe::W_EP0)) {
    const int role = warp == moe::W_LD ? 0 : warp == moe::W_DQ0 ? 1 : warp == moe::W_MMA ? 2 : 3;
    long long* d = args.dbg + (blockIdx.x * 4 + role) * 5;
    d[0] = t_wait;
    d[1] = clock64() - t_start;
    d[2] = ksteps;
    d[3] = t_sec;
    d[4] = t_sec2;
  }
  if (warp == moe::W_LD) {  // no async copy of this warp may still be writing shared memory at exit
    asm volatile("cp.async.wait_all;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  if (warp == moe::W_MMA) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
  if (PAIR && args.ep_wait_flags && threadIdx.x == 0) {  // the dispatch exchange is consumed (last CTA counts it)
    __threadfence();
    if (atomicAdd(args.ep_wait_done, 1u) == gridDim.x - 1) {
      *args.ep_wait_done = 0;
      *args.ep_expected += 1;
    }
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

template <bool PAIR, bool F8, bool PROF>
static int launch_moe_t(const CUtensorMap& tw, const MoeGemmArgs& a, int grid, uint32_t* status, cudaStream_t st) {
  using L = moe::Layout<F8>;
  static std::atomic<uint64_t> attr_devs{0};
  if (const int e = smem_attr_once(attr_devs, (const void*)moe_int3_gemm_kernel<PAIR, F8, PROF>, L::TOTAL)) return e;
  {
    const int pdl_rc = launch_pdl(moe_int3_gemm_kernel<PAIR, F8, PROF>, dim3(grid), dim3(moe::THREADS), L::TOTAL, st,
        tw, a, status);
    if (pdl_rc) return pdl_rc;
  }
  return (int)cudaGetLastError();
}

template <bool PAIR, bool F8>
static int launch_moe(const CUtensorMap& tw, const MoeGemmArgs& a, int grid, uint32_t* status, cudaStream_t st) {
  return a.dbg ? launch_moe_t<PAIR, F8, true>(tw, a, grid, status, st)
               : launch_moe_t<PAIR, F8, false>(tw, a, grid, status, st);
}

int moe_int3_gemm(const MoeGemmArgs& a, int pair, int num_sms, uint32_t* status, cudaStream_t st) {
  if (a.K % 128 || a.rows % 256 || a.route_srcs < 1 || a.route_srcs > moe::MAX_SRC || a.x_div < 1 ||
      !a.route_cnt || !a.route_list)
    return 3;
  if (reinterpret_cast<uintptr_t>(a.x_q) % 16) return 3;  // 16-byte async copies of the activation rows
  if (pair && a.ep_wait_flags && (!a.ep_expected || !a.ep_wait_done)) return 3;
  CUtensorMap tw;
  std::memset(&tw, 0, sizeof(tw));
  if (a.fp8_w) {  // e4m3 weights [E * rows, K]: 128 x 128 tiles, 128-byte swizzle (the MMA's A layout)
    if (!a.fp8_scales) return 3;
    const int rc = make_tmap_2d(&tw, a.fp8_w, 1, a.K, (uint64_t)a.num_experts * a.rows, (uint64_t)a.K, 128, 128, 1);
    if (rc) return 2000 + rc;
  }
  const int units = a.num_experts * (a.rows / 256);
  const int grid = units < num_sms ? units : num_sms;
  if (grid <= 0) return 0;
  if (a.fp8_w) return pair ? launch_moe<true, true>(tw, a, grid, status, st)
                           : launch_moe<false, true>(tw, a, grid, status, st);
  return pair ? launch_moe<true, false>(tw, a, grid, status, st) : launch_moe<false, false>(tw, a, grid, status, st);
}

}  // namespace afb
