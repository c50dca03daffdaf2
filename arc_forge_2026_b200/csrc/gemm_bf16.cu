// Dense bf16 GEMM on the 5th-gen tensor cores: C[M,N] = act(alpha * A[M,K] * B[N,K]^T + bias) (+ residual),
// act none / tanh-GELU / erf-GELU, bias bf16 [N] (both optional).
//
// Both operands are K-major (nn.Linear layout). One CTA computes a 128 x BN tile:
//   warp 0      one elected thread issues TMA loads (128-byte swizzle) into a STAGES-deep ring
//   warp 1      allocates TMEM and one elected thread issues tcgen05.mma (M=128, N=BN, K=16 per op)
//   warps 2..5  epilogue: tcgen05.ld of the fp32 accumulator, convert, optional residual add, store
// Split-K (gridDim.z > 1) writes fp32 partials that a reduce kernel sums in a fixed order.
// Both launch with programmatic stream serialization (programmatic dependent launch): a CTA sets up its barriers and
// TMEM (and, for one-M-tile decode GEMMs, starts its first weight tiles into L2) while the previous kernel in the
// stream finishes, and waits for it before touching anything that kernel may have written.
// Grouped forms (GemmGroups, gemm.h) run the experts of a MoE layer in one launch: each CTA maps its tile to a
// group (and to that group's A rows / B rows, or to its K range) before the usual pipeline.
// Used for every dense projection of the serving and training paths (QKV/in_proj, o_proj/out_proj,
// shared expert, router, LM head) in place of the reference's cuBLAS/CUTLASS dense GEMMs.
#include <cudaTypedefs.h>


#include "common.cuh"
#include "gemm.h"

namespace afb {

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int BM = 128, BK = 64;
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t BAR_OFF = STAGES * (A_BYTES + B_BYTES);
  static constexpr uint32_t TOTAL = BAR_OFF + (2 * STAGES + 1) * 8 + 16 + 1024;  // +1024 for manual alignment
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
};

// epilogue math on 4 consecutive columns: v = act(alpha * acc + bias) (+ the residual, by the caller)
AFB_DEV float gemm_act(float x, int act) {
  if (act == 1) return 0.5f * x * (1.f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
  if (act == 2) return 0.5f * x * (1.f + erff(x * 0.7071067811865476f));
  return x;
}
AFB_DEV void gemm_bias_act4(float* v, const GemmEpilogue& epi, int col) {
  if (epi.bias) {
    const uint2 q = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(epi.bias) + col);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&q);
#pragma unroll
    for (int t = 0; t < 4; ++t) v[t] += __bfloat162float(h[t]);
  }
  if (epi.act) {
#pragma unroll
    for (int t = 0; t < 4; ++t) v[t] = gemm_act(v[t], epi.act);
  }
}

template <int BN, int STAGES, int GMODE = 0>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                        int K, GemmEpilogue epi, uint32_t* status, GemmGroups grp = GemmGroups()) {
  using S = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // M tiles vary fastest: the CTAs that share a weight (B) tile run together, so B streams from HBM once while
  // the (small) activation tiles stay in L2
  const int tile_m = blockIdx.x, tile_n = blockIdx.y;
  // split-K range of this CTA
  const int num_kb_total = (K + S::BK - 1) / S::BK;
  const int splits = gridDim.z;
  const int kb_per = (num_kb_total + splits - 1) / splits;
  int kb0 = blockIdx.z * kb_per;
  int kb1 = min(num_kb_total, kb0 + kb_per);
  int a_row0 = tile_m * S::BM, b_row0 = tile_n * BN, m_end = M, col0_base = tile_n * BN;
  if constexpr (GMODE == 1) {  // rows of group e: find e with tiles[e] <= tile_m < tiles[e + 1]
    if (tile_m >= grp.tiles[grp.E]) return;  // surplus CTA of the upper-bound grid (before any barrier / TMEM)
    int lo = 0, hi = grp.E;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (grp.tiles[mid] <= tile_m) lo = mid; else hi = mid;
    }
    a_row0 = grp.seg[lo] + (tile_m - grp.tiles[lo]) * S::BM;
    m_end = grp.seg[lo + 1];
    b_row0 = lo * grp.group_rows + tile_n * BN;
  } else if constexpr (GMODE == 2) {  // group e = tile_m / m-tiles; its K range is its segment
    const int mt_per = (grp.group_rows + S::BM - 1) / S::BM;
    const int e = tile_m / mt_per;
    a_row0 = (tile_m % mt_per) * S::BM;
    m_end = grp.group_rows;
    kb0 = grp.seg[e] / S::BK;
    kb1 = grp.seg[e + 1] / S::BK;
    epi.out = reinterpret_cast<uint8_t*>(epi.out) + (size_t)e * grp.group_out_stride * (epi.out_fp32 ? 4 : 2);
  }
  const int num_kb = max(0, kb1 - kb0);
  if constexpr (GMODE == 0) {
    // decode-shaped GEMM (one M tile): the first weight tiles of this CTA's slice stream into L2 while the previous
    // kernel may still run; the weights are not what it writes, and L2 is the point of coherence, so a prefetch is
    // never stale
    if (threadIdx.x == 0 && gridDim.x == 1) {
      prefetch_tmap(&tmB);
      for (int i = 0; i < min(num_kb, 2 * STAGES); ++i) tma_prefetch_l2_2d(&tmB, (kb0 + i) * S::BK, b_row0);
    }
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, S::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // from here on the kernel reads the activations and writes its output: the previous kernel must be complete
  grid_dep_wait();
  if (threadIdx.x == 0) grid_dep_trigger();

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      int issued = 0;
      for (int i = 0; i < num_kb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (i >= STAGES && !mbar_wait(&empty[s], ph ^ 1, status)) break;
        mbar_arrive_expect_tx(&full[s], S::A_BYTES + S::B_BYTES);
        tma_load_2d(sA + s * S::A_BYTES, &tmA, &full[s], (kb0 + i) * S::BK, a_row0);
        tma_load_2d(sB + s * S::B_BYTES, &tmB, &full[s], (kb0 + i) * S::BK, b_row0);
        ++issued;
      }
      // drain: every issued copy has landed before the CTA may exit (bounded)
      for (int i = max(0, issued - STAGES); i < issued; ++i) mbar_wait(&full[i % STAGES], (i / STAGES) & 1, status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(128, BN, 1);
      for (int i = 0; i < num_kb; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&full[s], (i / STAGES) & 1, status)) break;
        tc_fence_after();
        const uint64_t da = sw128_desc(smem_u32(sA + s * S::A_BYTES));
        const uint64_t db = sw128_desc(smem_u32(sB + s * S::B_BYTES));
#pragma unroll
        for (int kk = 0; kk < S::BK / 16; ++kk) {
          // +32 bytes along K per MMA: the descriptor's start address is in 16-byte units
          umma_f16(tmem, da + 2 * kk, db + 2 * kk, idesc, (i | kk) != 0);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(done);  // also covers the error path: the epilogue waits for every issued MMA
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quadrant (warp % 4)
    const int quad = warp & 3;
    const bool ok = mbar_wait(done, 0, status);
    tc_fence_after();
    const int row = a_row0 + quad * 32 + lane;
    const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float v[32];
      tmem_ld32(taddr + c, v);
      tmem_ld_wait();
      const int col0 = col0_base + c;
      if (!ok || row >= m_end || col0 >= N) continue;
      if (num_kb == 0) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;  // an empty split-K slice contributes zeros
      }
      if (splits > 1) {
        float* out = reinterpret_cast<float*>(epi.partial) + ((size_t)blockIdx.z * M + row) * N + col0;
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          if (col0 + j < N) *reinterpret_cast<float4*>(out + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        continue;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= epi.alpha;
      if (epi.bias || epi.act) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          if (col0 + j < N) gemm_bias_act4(v + j, epi, col0 + j);
      }
      if (epi.residual) {
        const __nv_bfloat16* r = reinterpret_cast<const __nv_bfloat16*>(epi.residual) + (size_t)row * epi.ldr + col0;
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          if (col0 + j >= N) break;
          uint4 q = *reinterpret_cast<const uint4*>(r + j);
          const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&q);
#pragma unroll
          for (int t = 0; t < 8; ++t) v[j + t] += __bfloat162float(h[t]);
        }
      }
      if (epi.out_fp32) {
        float* out = reinterpret_cast<float*>(epi.out) + (size_t)row * epi.ldo + col0;
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          if (col0 + j < N) *reinterpret_cast<float4*>(out + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      } else {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(epi.out) + (size_t)row * epi.ldo + col0;
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          if (col0 + j >= N) break;
          uint4 q = make_uint4(pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                               pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7]));
          *reinterpret_cast<uint4*>(out + j) = q;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

// Fixed-order sum of split-K partials [splits, M, N] fp32 -> out (+ residual), alpha applied.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int M, int N, GemmEpilogue epi) {
  grid_dep_wait();  // the partials are the GEMM's output
  const size_t idx = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  const size_t total = (size_t)M * N;
  if (idx >= total) return;
  const int row = idx / N, col = idx % N;
  float4 acc = *reinterpret_cast<const float4*>(part + idx);
  for (int s = 1; s < splits; ++s) {
    float4 p = *reinterpret_cast<const float4*>(part + (size_t)s * total + idx);
    acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
  }
  float v[4] = {acc.x * epi.alpha, acc.y * epi.alpha, acc.z * epi.alpha, acc.w * epi.alpha};
  gemm_bias_act4(v, epi, col);
  if (epi.residual) {
    const __nv_bfloat16* r = reinterpret_cast<const __nv_bfloat16*>(epi.residual) + (size_t)row * epi.ldr + col;
    for (int t = 0; t < 4; ++t) v[t] += __bfloat162float(r[t]);
  }
  if (epi.out_fp32) {
    float* o = reinterpret_cast<float*>(epi.out) + (size_t)row * epi.ldo + col;
    *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(epi.out) + (size_t)row * epi.ldo + col;
    *reinterpret_cast<uint2*>(o) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
  }
}

// ------------------------------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// The encoder validates the address against the calling thread's current context. A thread that has made no CUDA
// runtime call yet (PyTorch's autograd device thread, when a backward starts with a native op) has none: a runtime
// call makes the device's primary context current.
static bool ensure_context() {
  int dev = 0;
  return cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess && cudaFree(nullptr) == cudaSuccess;
}

int make_tmap_2d(CUtensorMap* map, const void* base, int dtype_bytes, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, int swizzle128) {
  auto encode = get_encode();
  if (!encode) return -1;
  CUtensorMapDataType dt = dtype_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                           : dtype_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                              : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  auto run = [&] {
    return encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = run();
  if (r == CUDA_ERROR_INVALID_CONTEXT && ensure_context()) r = run();
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

int make_tmap_3d_bf16(CUtensorMap* map, const void* base, const uint64_t dims[3], const uint64_t strides_bytes[2],
                      const uint32_t box[3]) {
  auto encode = get_encode();
  if (!encode) return -1;
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t str[2] = {strides_bytes[0], strides_bytes[1]};
  cuuint32_t bx[3] = {box[0], box[1], box[2]};
  cuuint32_t estr[3] = {1, 1, 1};
  auto run = [&] {
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), d, str, bx, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = run();
  if (r == CUDA_ERROR_INVALID_CONTEXT && ensure_context()) r = run();
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

template <int BN, int STAGES>
static int launch_gemm(const void* A, int lda, const void* B, int ldb, int M, int N, int K, int splits,
                       const GemmEpilogue& epi, uint32_t* status, cudaStream_t stream) {
  using S = GemmSmem<BN, STAGES>;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, 2, K, M, (uint64_t)lda * 2, S::BK, S::BM, 1);
  if (rc) return 1000 + rc;
  rc = make_tmap_2d(&tb, B, 2, K, N, (uint64_t)ldb * 2, S::BK, BN, 1);
  if (rc) return 2000 + rc;
  auto kern = gemm_bf16_tn_kernel<BN, STAGES>;
  static std::atomic<uint64_t> attr_devs{0};
  if (const int e = smem_attr_once(attr_devs, (const void*)kern, S::TOTAL)) return e;
  const dim3 grid((M + S::BM - 1) / S::BM, (N + BN - 1) / BN, splits);
  return launch_pdl(kern, grid, dim3(192), S::TOTAL, stream, ta, tb, M, N, K, epi, status, GemmGroups());
}

// Grouped launch (one tile width: 256; no split-K). A ROWS grid covers max_tiles m-tiles (an upper bound of
// sum ceil(rows_e / 128)); a REDUCE grid covers E x ceil(group_rows / 128).
int gemm_bf16_grouped(const void* A, int lda, int rows_a, const void* B, int ldb, int rows_b, int N, int K,
                      const GemmEpilogue& epi, const GemmGroups& g, int max_tiles, uint32_t* status,
                      cudaStream_t stream) {
  constexpr int BN = 256, STAGES = 4;  // 128 x 256 tiles: half the CTAs of 128-wide ones (each CTA's setup and
                                       // pipeline fill is paid once per tile; REDUCE tiles have few K blocks)
  using S = GemmSmem<BN, STAGES>;
  if (g.mode != 1 && g.mode != 2) return 3;
  if ((K % 8) || (lda % 8) || (ldb % 8) || (N % 8) || epi.partial || epi.bias || epi.act) return 3;
  if (rows_a <= 0 || rows_b <= 0 || N <= 0 || g.E <= 0) return 0;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, 2, K, rows_a, (uint64_t)lda * 2, S::BK, S::BM, 1);
  if (rc) return 1000 + rc;
  rc = make_tmap_2d(&tb, B, 2, K, rows_b, (uint64_t)ldb * 2, S::BK, BN, 1);
  if (rc) return 2000 + rc;
  dim3 grid;
  if (g.mode == 1) {
    auto kern = gemm_bf16_tn_kernel<BN, STAGES, 1>;
    static std::atomic<uint64_t> attr_devs{0};
    if (const int e = smem_attr_once(attr_devs, (const void*)kern, S::TOTAL)) return e;
    grid = dim3(max_tiles, (N + BN - 1) / BN, 1);
    kern<<<grid, 192, S::TOTAL, stream>>>(ta, tb, rows_a, N, K, epi, status, g);
  } else {
    auto kern = gemm_bf16_tn_kernel<BN, STAGES, 2>;
    static std::atomic<uint64_t> attr_devs{0};
    if (const int e = smem_attr_once(attr_devs, (const void*)kern, S::TOTAL)) return e;
    grid = dim3(g.E * ((g.group_rows + S::BM - 1) / S::BM), (N + BN - 1) / BN, 1);
    kern<<<grid, 192, S::TOTAL, stream>>>(ta, tb, rows_a, N, K, epi, status, g);
  }
  return (int)cudaGetLastError();
}

// Tile/split choice: fill 148 SMs (two CTAs fit per SM at BN<=128 with 3-4 stages).
// Tile width and split-K count by a small cost model: the grid runs in ceil(CTAs / SMs) waves and each CTA streams
// its B slice (bn x K/splits weights from DRAM) plus the A slice (128 x K/splits, mostly L2 hits, weighted 1/4);
// split-K adds the fp32 partials written and read back (M x N x 4 x (splits + 1)). This keeps skinny decode GEMMs
// (M <= 128, weights streamed once) on whole waves instead of a mostly-empty second wave.
GemmPlan plan_gemm(int M, int N, int K, int num_sms) {
  GemmPlan best;
  double best_cost = 1e300;
  const int mt = (M + 127) / 128;
  const int kb = (K + 63) / 64;
  const int bns[3] = {64, 128, 256};
  const int sps[6] = {1, 2, 3, 4, 6, 8};
  for (int bn : bns) {
    const long long tiles = (long long)mt * ((N + bn - 1) / bn);
    for (int sp : sps) {
      if (sp > 1 && kb / sp < 4) continue;
      const long long ctas = tiles * sp;
      const long long waves = (ctas + num_sms - 1) / num_sms;
      const double kper = (double)((kb + sp - 1) / sp) * 64.0;
      const double per_cta = (bn + 0.25 * 128.0) * kper * 2.0;
      double cost = (double)waves * per_cta * num_sms;
      if (sp > 1) cost += (double)M * N * 4.0 * (sp + 1);
      if (cost < best_cost * 0.97) {  // prefer fewer splits / narrower tiles unless clearly cheaper
        best_cost = cost;
        best.bn = bn;
        best.splits = sp;
      }
    }
  }
  return best;
}

int gemm_bf16_tn(const void* A, int lda, const void* B, int ldb, int M, int N, int K, const GemmEpilogue& epi,
                 int bn, int splits, uint32_t* status, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if ((K % 8) || (N % 8) || (lda % 8) || (ldb % 8) || epi.act < 0 || epi.act > 2) return 3;
  if (splits > 1 && !epi.partial) return 4;
  int rc;
  if (bn == 128)
    rc = launch_gemm<128, 3>(A, lda, B, ldb, M, N, K, splits, epi, status, stream);
  else if (bn == 256)
    rc = launch_gemm<256, 4>(A, lda, B, ldb, M, N, K, splits, epi, status, stream);
  else
    rc = launch_gemm<64, 4>(A, lda, B, ldb, M, N, K, splits, epi, status, stream);
  if (rc || splits <= 1) return rc;
  const size_t total = (size_t)M * N;
  const int threads = 256;
  const int blocks = (int)((total / 4 + threads - 1) / threads);
  return launch_pdl(splitk_reduce_kernel, dim3(blocks), dim3(threads), 0, stream,
                          reinterpret_cast<const float*>(epi.partial), splits, M, N, epi);
}

}  // namespace afb
