// Per-layer n-gram embedding (PLE) lookup: hash + table gather + dequantisation in one pass.
//
// For every row r (a token) and head h:
//   prev_s  = ext[pos[r] - s] if pos[r] - s >= seg[r] and no EOS in ext[pos[r]-s .. pos[r]-1], else EOS
//   mix_2   = ext[pos[r]] * m_0 ^ prev_1 * m_1;  mix_n = mix_(n-1) ^ prev_(n-1) * m_(n-1)      (wrapping int64)
//   id      = (mix_n mod p_h) + off_h                    heads h of order n use mix_n
//   out[r, h*D:(h+1)*D] = dequant(table[id])             e4m3 with 128 x 128 block scales, or bf16
//
// ``ext`` holds the tokens with their history inline (a packed training row: the row itself; serving: each
// session's last n-1 committed tokens followed by the step's tokens), so the history test is local: no scan.
//
// The table may be split by rows over several shards (``rows_per_shard`` rows each, a multiple of 128): the row's
// shard pointer is then read from ``shards``; on a multi-GPU job these are peers' buffers mapped into this process
// and read with plain 16-byte loads over NVLink (no TMA, no multicast), so the lookup needs no all-gather of ids or
// reduce-scatter of rows. A hot (compact) table maps each head's kept buckets through a sorted index (binary
// search); a miss reads zeros.
//
// One warp per token: lane h hashes head h (the 64-bit modulo of each head runs once, in parallel across lanes),
// then the 32 lanes copy the token's heads x 16-byte chunks, each taking its head's row id by a shuffle.
#include "common.cuh"
#include "kernels.h"

namespace afb {
namespace pled {
using bf16 = __nv_bfloat16;

AFB_DEV int64_t wrap_mul(int64_t a, int64_t b) {
  return (int64_t)((uint64_t)a * (uint64_t)b);
}

template <bool FP8>
__global__ void __launch_bounds__(256) ple_lookup_kernel(PleLookupArgs a) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;  // one warp per token
  const int lane = threadIdx.x & 31;
  const int heads = (a.n - 1) * a.hpn;  // <= 32 (checked at launch): lane h hashes head h
  if (r >= a.rows) return;
  const int64_t p = a.pos[r];
  const int64_t seg = a.seg[r];
  const bool bad = p < 0 || p >= a.ext_len || seg < 0 || seg > p;
  if (bad && lane == 0) flag_error(a.status, AFB_ERR_BOUNDS);  // bad index: recorded, the row reads zeros
  long long row = -1;
  if (lane < heads && !bad) {
    const int h = lane;
    const int order = 2 + h / a.hpn;
    int64_t mix = wrap_mul((int64_t)a.ext[p], a.mult[0]);
    bool ok = true;
    for (int s = 1; s < order; ++s) {
      const int64_t q = p - s;
      ok = ok && q >= seg && a.ext[q] != a.eos;
      mix ^= wrap_mul(ok ? (int64_t)a.ext[q] : (int64_t)a.eos, a.mult[s]);
    }
    int64_t m = mix % a.mod[h];
    if (m < 0) m += a.mod[h];
    row = m + a.off[h];
    if (a.hot_idx) {  // compact table: binary search of the bucket among this head's kept ones
      const int64_t* b = a.hot_idx + a.hot_base[h];
      int lo = 0, hi = a.hot_len[h];
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (b[mid] < m) lo = mid + 1; else hi = mid;
      }
      row = (lo < a.hot_len[h] && b[lo] == m) ? a.hot_base[h] + lo : -1;
    }
  }
  if (a.ids_out && lane < heads) a.ids_out[(int64_t)r * heads + lane] = row;
  const int D = a.head_dim;
  const int C = FP8 ? D / 16 : D / 8;  // 16-byte chunks of one table row
  bf16* out = reinterpret_cast<bf16*>(a.out) + (int64_t)r * heads * D;
  for (int base = 0; base < heads * C; base += 32) {  // uniform trip count: every lane joins each shuffle
    const int t = base + lane;
    const int h = min(t / C, heads - 1), c = t % C;
    const long long rh = __shfl_sync(0xffffffffu, row, h);
    if (t >= heads * C) continue;
    uint4 o0, o1;
    if (rh < 0 || rh >= a.table_rows) {
      o0 = make_uint4(0, 0, 0, 0);
      o1 = o0;
    } else {
      const int shard = (int)(rh / a.rows_per_shard);
      const int64_t lr = rh - (int64_t)shard * a.rows_per_shard;
      if (FP8) {
        const uint8_t* tp = reinterpret_cast<const uint8_t*>(a.shards[shard]) + lr * D + c * 16;
        const uint4 v = *reinterpret_cast<const uint4*>(tp);
        const float sc = a.scale_shards[shard][(lr / 128) * a.scale_ld + (c * 16) / 128];
        const __nv_fp8x4_e4m3* e = reinterpret_cast<const __nv_fp8x4_e4m3*>(&v);
        float f[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 x = float4(e[i]);
          f[4 * i] = x.x * sc;
          f[4 * i + 1] = x.y * sc;
          f[4 * i + 2] = x.z * sc;
          f[4 * i + 3] = x.w * sc;
        }
        o0 = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                        pack_bf16x2(f[6], f[7]));
        o1 = make_uint4(pack_bf16x2(f[8], f[9]), pack_bf16x2(f[10], f[11]), pack_bf16x2(f[12], f[13]),
                        pack_bf16x2(f[14], f[15]));
      } else {
        const bf16* tp = reinterpret_cast<const bf16*>(a.shards[shard]) + lr * D + c * 8;
        o0 = *reinterpret_cast<const uint4*>(tp);
      }
    }
    bf16* dst = out + (int64_t)h * D;
    if (FP8) {
      reinterpret_cast<uint4*>(dst + c * 16)[0] = o0;
      reinterpret_cast<uint4*>(dst + c * 16)[1] = o1;
    } else {
      reinterpret_cast<uint4*>(dst + c * 8)[0] = o0;
    }
  }
}
}  // namespace pled

int ple_lookup(const PleLookupArgs& a, bool fp8, cudaStream_t st) {
  if (a.n < 2 || a.n > 8 || a.hpn < 1 || (a.n - 1) * a.hpn > 32 || a.head_dim % 16 || a.rows_per_shard <= 0 ||
      a.rows_per_shard % 128)
    return 3;
  const int64_t warps = a.rows;
  if (warps == 0) return 0;
  const int64_t blocks = (warps * 32 + 255) / 256;
  const int rc = fp8 ? launch_pdl(pled::ple_lookup_kernel<true>, dim3((unsigned)blocks), dim3(256), 0, st, a)
                    : launch_pdl(pled::ple_lookup_kernel<false>, dim3((unsigned)blocks), dim3(256), 0, st, a);
  return rc == 0 ? 0 : 1;
}
}  // namespace afb
