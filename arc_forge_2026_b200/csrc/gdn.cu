// Gated DeltaNet (GDN) for decode and speculative verify, with the accepted-prefix commit deferred into the
// next cycle (so a verify cycle reads and writes each recurrent state once, the same traffic as plain decode).
//
// Per sequence slot the engine keeps:
//   conv_state [slots, 3, C]            last 3 committed pre-conv inputs (C = 2*Hk*Dk + Hv*Dv channels)
//   ssm_state  [slots, Hv, Dk, Dv] fp32 committed recurrent state S (o_t = S^T q_t)
//   pending buffers, two parities:      the last cycle's pre-conv inputs, normalised q/k, v, g, beta per token
//   n_commit [slots]                    how many of the last cycle's tokens were accepted (written by accept)
// Cycle `parity` reads pending[parity ^ 1] for the commit and writes pending[parity] for the next one.
// commit_current = 1 (prefill / plain decode) applies and stores every new token instead.
//
// gdn_conv_prep: per (seq, 128-channel block): commit the conv state, causal depthwise conv (kernel 4) + SiLU
//   for the new tokens, per-head L2 norm of q/k (q scaled by Dk^-0.5), gates beta = sigmoid(b),
//   g = -exp(A_log) * softplus(a + dt_bias).
// gdn_recurrent: per (seq, value head), one thread per value column: commit the accepted tokens into S, write S,
//   then run the new tokens through the gated delta rule for their outputs, and apply the gated RMSNorm
//   (rms over Dv, * w * silu(z)) before the bf16 store.
// The math is the recurrence of training/work (FlashQLA's chunked kernels compute the same rule in chunks).
#include "common.cuh"
#include "kernels.h"

namespace afb {

template <int DK>
__global__ void __launch_bounds__(DK) gdn_conv_prep_kernel(GdnArgs a, int parity) {
  const int seq = blockIdx.x;
  const int slot = a.seq_slot[seq];
  const int c = blockIdx.y * DK + threadIdx.x;
  const int C = a.conv_dim;
  const int T = a.q_per_seq;
  const int tok0 = seq * T;
  const int nq = a.Hk * DK;  // q channels, then k channels, then v channels
  const int cur = parity, prev = parity ^ 1;
  const int ps = a.commit_current ? seq : slot;  // pending-buffer slot (prefill scratch is indexed by sequence)
  __shared__ float red[32];

  // ---- conv state: commit the accepted part of the previous cycle
  float s0 = __bfloat162float(a.conv_state[((size_t)slot * 3 + 0) * C + c]);
  float s1 = __bfloat162float(a.conv_state[((size_t)slot * 3 + 1) * C + c]);
  float s2 = __bfloat162float(a.conv_state[((size_t)slot * 3 + 2) * C + c]);
  if (!a.commit_current) {
    const int nprev = a.n_commit[slot];
    const __nv_bfloat16* pin = a.pend_in + (((size_t)prev * a.pend_slots + ps) * a.max_q) * C + c;
    for (int t = 0; t < nprev; ++t) {
      const float x = __bfloat162float(pin[(size_t)t * C]);
      s0 = s1;
      s1 = s2;
      s2 = x;
    }
  }
  const float w0 = a.conv_w[c * 4 + 0], w1 = a.conv_w[c * 4 + 1], w2 = a.conv_w[c * 4 + 2], w3 = a.conv_w[c * 4 + 3];
  float x3 = s0, x2 = s1, x1 = s2;  // x_{t-3}, x_{t-2}, x_{t-1}
  __nv_bfloat16* pin_cur = a.pend_in + (((size_t)cur * a.pend_slots + ps) * a.max_q) * C + c;
  for (int t = 0; t < T; ++t) {
    const float x = __bfloat162float(a.mixed[(size_t)(tok0 + t) * a.mixed_ld + c]);
    if (!a.commit_current) pin_cur[(size_t)t * C] = __float2bfloat16(x);
    float y = w0 * x3 + w1 * x2 + w2 * x1 + w3 * x;
    y = silu(y);
    x3 = x2;
    x2 = x1;
    x1 = x;
    if (c < 2 * nq) {
      // per-head L2 norm over the DK channels of this block
      float ss = warp_sum(y * y);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
      __syncthreads();
      float tot = 0.f;
      for (int w = 0; w < DK / 32; ++w) tot += red[w];
      __syncthreads();
      float v = y * rsqrtf(tot + 1e-6f);
      if (c < nq) v *= rsqrtf((float)DK);
      a.pend_qk[(((size_t)cur * a.pend_slots + ps) * a.max_q + t) * (2 * nq) + c] = __float2bfloat16(v);
    } else {
      a.pend_v[(((size_t)cur * a.pend_slots + ps) * a.max_q + t) * (C - 2 * nq) + (c - 2 * nq)] = __float2bfloat16(y);
    }
  }
  if (a.commit_current) {  // all new tokens are committed: the state is the last 3 inputs
    s0 = x3;
    s1 = x2;
    s2 = x1;
  }
  a.conv_state[((size_t)slot * 3 + 0) * C + c] = __float2bfloat16(s0);
  a.conv_state[((size_t)slot * 3 + 1) * C + c] = __float2bfloat16(s1);
  a.conv_state[((size_t)slot * 3 + 2) * C + c] = __float2bfloat16(s2);

  // ---- gates (one block column computes them for every value head)
  if (blockIdx.y == 0) {
    for (int h = threadIdx.x; h < a.Hv; h += blockDim.x) {
      const float A = -__expf(a.A_log[h]);
      const float dt = a.dt_bias[h];
      for (int t = 0; t < T; ++t) {
        const __nv_bfloat16* row = a.mixed + (size_t)(tok0 + t) * a.mixed_ld + a.ba_off;
        const float b = __bfloat162float(row[h]);
        const float av = __bfloat162float(row[a.Hv + h]) + dt;
        const float sp = av > 20.f ? av : log1pf(__expf(av));
        float* gb = a.pend_gb + ((((size_t)cur * a.pend_slots + ps) * a.Hv + h) * a.max_q + t) * 2;
        gb[0] = A * sp;                       // g (log decay)
        gb[1] = 1.f / (1.f + __expf(-b));     // beta
      }
    }
  }
}

// float offset of row kk (0..31) of thread t's slice in the swizzled state layout (DK = DV = 128, 4 threads per
// column; see the persistent verify kernel)
AFB_DEV int gdn_state_off(int t, int kk) { return t * 32 + ((((kk >> 2) ^ (t & 7))) << 2) + (kk & 3); }

// QT threads per value column (adjacent lanes), each holding DK/QT state rows in registers; dot products over DK
// are reduced with log2(QT) shuffles. QT=4 (512 threads) doubles the warps per SM over one thread pair per column,
// so the strided state loads of some warps overlap the recurrence of others.
template <int DK, int DV, int QT>
__global__ void __launch_bounds__(QT * DV, 1) gdn_recurrent_kernel(GdnArgs a, int parity) {
  constexpr int HK = DK / QT;
  const int seq = blockIdx.x, h = blockIdx.y;
  const int slot = a.seq_slot[seq];
  const int v = threadIdx.x / QT, part = threadIdx.x % QT;
  const int T = a.q_per_seq;
  const int kh = h / (a.Hv / a.Hk);
  const int nq = a.Hk * DK;
  const int cur = parity, prev = parity ^ 1;
  const int ps = a.commit_current ? seq : slot;
  __shared__ float kq[2][DK];
  __shared__ float red[32];

  float S[HK];
  // DK = DV = 128 with 4 threads per column: the swizzled thread-major layout the persistent verify kernel uses
  // (thread t = QT * v + part owns its 32 rows contiguously); other shapes: plain [Dk, Dv]
  constexpr bool SWZ = DK == 128 && DV == 128 && QT == 4;
  float* sp = SWZ ? a.ssm_state + ((size_t)slot * a.Hv + h) * DK * DV
                  : a.ssm_state + (((size_t)slot * a.Hv + h) * DK + part * HK) * DV + v;
  auto sidx = [&](int k) -> size_t { return SWZ ? (size_t)gdn_state_off(threadIdx.x, k) : (size_t)k * DV; };
#pragma unroll
  for (int k = 0; k < HK; ++k) S[k] = sp[sidx(k)];

  auto load_kq = [&](int par, int t) {
    const size_t base = ((size_t)par * a.pend_slots + ps) * a.max_q + t;
    const __nv_bfloat16* qk = a.pend_qk + base * (2 * nq);
    __syncthreads();
    for (int k = threadIdx.x; k < DK; k += blockDim.x) {
      kq[0][k] = __bfloat162float(qk[nq + kh * DK + k]);
      kq[1][k] = __bfloat162float(qk[kh * DK + k]);
    }
    __syncthreads();
    return base;
  };
  auto reduce = [&](float x) {
#pragma unroll
    for (int o = 1; o < QT; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
  };
  auto update = [&](size_t base) {
    const size_t pslot = base / a.max_q, tt = base % a.max_q;  // base = (par * pend_slots + ps) * max_q + t
    const float* gb = a.pend_gb + ((pslot * a.Hv + h) * a.max_q + tt) * 2;
    const float decay = __expf(gb[0]), beta = gb[1];
    const float vv = __bfloat162float(a.pend_v[base * (a.Hv * DV) + h * DV + v]);
    const float* kk = kq[0] + part * HK;
    float mem = 0.f;
#pragma unroll
    for (int k = 0; k < HK; ++k) {
      S[k] *= decay;
      mem = fmaf(kk[k], S[k], mem);
    }
    mem = reduce(mem);
    const float delta = beta * (vv - mem);
#pragma unroll
    for (int k = 0; k < HK; ++k) S[k] = fmaf(kk[k], delta, S[k]);
  };

  if (!a.commit_current) {
    const int nprev = a.n_commit[slot];
    for (int t = 0; t < nprev; ++t) update(load_kq(prev, t));
#pragma unroll
    for (int k = 0; k < HK; ++k) sp[sidx(k)] = S[k];
  }
  for (int t = 0; t < T; ++t) {
    update(load_kq(cur, t));
    const float* qq = kq[1] + part * HK;
    float o = 0.f;
#pragma unroll
    for (int k = 0; k < HK; ++k) o = fmaf(qq[k], S[k], o);
    o = reduce(o);
    // gated RMSNorm over the DV outputs of this head (each column counted once)
    const float ss = warp_sum(part ? 0.f : o * o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < (QT * DV) / 32; ++w) tot += red[w];
    if (!part) {
      const size_t tok = (size_t)seq * T + t;
      const float z = __bfloat162float(a.mixed[tok * a.mixed_ld + a.z_off + h * DV + v]);
      const float y = o * rsqrtf(tot / DV + a.eps) * __bfloat162float(a.norm_w[v]) * silu(z);
      a.out[tok * (a.Hv * DV) + h * DV + v] = __float2bfloat16(y);
    }
  }
  if (a.commit_current) {
#pragma unroll
    for (int k = 0; k < HK; ++k) sp[sidx(k)] = S[k];
  }
}

// ------------------------------------------------------------------------------------------ persistent verify path
// One CTA (512 threads, 4 per value column) per SM loops over (sequence, value head) items. While it runs the
// recurrence of item i, bulk copies (no multicast) stage item i+1 into the other half of a shared-memory double
// buffer: its 64 KB committed state, the k (and q) rows of the previous cycle's and this cycle's tokens, their v rows,
// and gates (the z rows of the output gate are read from global memory by the norm pass).
//
// Per item:
//   * keys and queries are converted once to fp32 into part-padded rows (conflict-free 16-byte loads);
//   * the recurrence keeps S / Gamma in registers, Gamma = the product of the decays since the item started, so a
//     step is two FMA passes (the dot k.S and the rank-1 update) instead of three -- the decay is applied to the
//     scalar, S_true = Gamma * S. When log Gamma falls below -60 the registers are rescaled and Gamma restarts at 1;
//   * after the accepted tokens of the previous cycle the committed state Gamma * S goes back into its shared-memory
//     slot and each warp stores its 4 KB with one bulk copy (the state is not rewritten when no token was accepted);
//   * this cycle's raw outputs go to shared memory with per-token sums of squares; the gated RMSNorm of an item is
//     finished after the next item's barrier, one column per thread (fp32 keys, queries and outputs are
//     double-buffered by item parity, the sums rotate over three slots), so each item costs one block-wide barrier;
//     the output gate's z values of an item are loaded into registers when its recurrence starts, so the norm pass
//     waits on no global load.
// State layout (DK = DV = 128, per (slot, head)): thread t = 4 * v + part owns rows part*32 .. part*32+31 of column v
// and stores them contiguously, 16-byte chunk c at chunk position c ^ (t & 7) -- so every thread moves its slice
// with 16-byte accesses and no two lanes of a quarter warp touch the same bank.
namespace gdnp {
constexpr int DK = 128, DV = 128, QT = 4, HK = DK / QT, THREADS = QT * DV, MAXT = 8, MAXS = 1024;
constexpr int KP = HK + 4;  // padded fp32 slice of a key / query row per part
struct Smem {
  float state[2][DK * DV];
  __nv_bfloat16 kq[2][2 * MAXT][2][DK];  // token slots 0..7: previous cycle (k only), 8..15: this cycle (k, q)
  __nv_bfloat16 v[2][2 * MAXT][DV];
  float gb[2][2][2 * MAXT];              // [buf][previous / this cycle][token * 2 + (g, beta)]
  float kf[2][2 * MAXT][QT * KP];        // per item parity: keys, fp32, compact token order (accepted, then new)
  float qf[2][MAXT][QT * KP];            // per item parity: queries, fp32
  float o[2][MAXT][DV];                  // per item parity: raw outputs of this cycle's tokens
  float ssq[3][MAXT];                    // per item (mod 3): sum of squares of each token's raw outputs
  int slot[MAXS], ncommit[MAXS];
  uint64_t full[2];
};
}  // namespace gdnp

AFB_DEV void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
AFB_DEV void bulk_store(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(ssrc)),
               "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
AFB_DEV void bulk_store_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
AFB_DEV void bulk_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(gdnp::THREADS, 1) gdn_verify_persistent_kernel(GdnArgs a, int parity,
                                                                                  uint32_t* status) {
  using namespace gdnp;
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int tid = threadIdx.x, v = tid / QT, part = tid % QT;
  const int wid = tid >> 5, lane = tid & 31;
  const int T = a.q_per_seq;
  const int nq = a.Hk * DK;
  const int cur = parity, prev = parity ^ 1;
  const int items = a.num_seqs * a.Hv;
  for (int i = tid; i < a.num_seqs; i += THREADS) {
    const int sl = a.seq_slot[i];
    sm.slot[i] = sl;
    sm.ncommit[i] = a.n_commit[sl];
  }
  if (tid == 0) {
    mbar_init(&sm.full[0], 1);
    mbar_init(&sm.full[1], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // every warp stages a share of an item: copy c is issued by lane c / 16 of warp c % 16 (so no warp's recurrence
  // is held back by a run of copy issues), and thread 0 arms the barrier with the item's bytes (the transaction
  // count may go below zero until it does)
  auto issue = [&](int item, int b) {
    const int seq = item / a.Hv, h = item % a.Hv;
    const int slot = sm.slot[seq], np = sm.ncommit[seq];
    const int kh = h / (a.Hv / a.Hk);
    if (tid == 0) {
      const uint32_t bytes = DK * DV * 4 + np * (DK + DV) * 2 + T * (2 * DK + DV) * 2 + 2 * a.max_q * 8;
      mbar_arrive_expect_tx(&sm.full[b], bytes);
    }
    // copy list: 0 state, 1 gb prev, 2 gb cur, then per accepted token (k, v), then per new token (k, q, v)
    const int ncopies = 3 + 2 * np + 3 * T;
    for (int c = wid + (THREADS / 32) * lane; c < ncopies; c += THREADS) {
      if (c == 0) {
        bulk_copy(sm.state[b], a.ssm_state + ((size_t)slot * a.Hv + h) * DK * DV, DK * DV * 4, &sm.full[b]);
      } else if (c <= 2) {
        const int par = c == 1 ? prev : cur;
        bulk_copy(sm.gb[b][c - 1], a.pend_gb + (((size_t)par * a.pend_slots + slot) * a.Hv + h) * a.max_q * 2,
                  a.max_q * 8, &sm.full[b]);
      } else if (c < 3 + 2 * np) {
        const int t = (c - 3) >> 1;
        const size_t base = ((size_t)prev * a.pend_slots + slot) * a.max_q + t;
        if (((c - 3) & 1) == 0)
          bulk_copy(sm.kq[b][t][0], a.pend_qk + base * (2 * nq) + nq + kh * DK, DK * 2, &sm.full[b]);
        else
          bulk_copy(sm.v[b][t], a.pend_v + base * (a.Hv * DV) + h * DV, DV * 2, &sm.full[b]);
      } else {
        const int t = (c - 3 - 2 * np) / 3, w = (c - 3 - 2 * np) % 3;
        const size_t base = ((size_t)cur * a.pend_slots + slot) * a.max_q + t;
        if (w == 0)
          bulk_copy(sm.kq[b][MAXT + t][0], a.pend_qk + base * (2 * nq) + nq + kh * DK, DK * 2, &sm.full[b]);
        else if (w == 1)
          bulk_copy(sm.kq[b][MAXT + t][1], a.pend_qk + base * (2 * nq) + kh * DK, DK * 2, &sm.full[b]);
        else
          bulk_copy(sm.v[b][MAXT + t], a.pend_v + base * (a.Hv * DV) + h * DV, DV * 2, &sm.full[b]);
      }
    }
  };
  // gated RMSNorm of one finished item's raw outputs: the thread of part 0 of column v finishes column v of every
  // token (the sums of squares were accumulated while the outputs were produced); z is read from global memory, so
  // the item's staging buffer is already free for the next copies
  const float norm_w = part == 0 ? __bfloat162float(a.norm_w[v]) : 0.f;
  float zr[MAXT];  // part 0: silu(z) of column v for the item being normalised next, loaded one item ahead
  auto load_z = [&](int item) {
    const int seq = item / a.Hv, h = item % a.Hv;
#pragma unroll
    for (int t = 0; t < MAXT; ++t)
      zr[t] = (part == 0 && t < T)
                  ? __bfloat162float(a.mixed[((size_t)seq * T + t) * a.mixed_ld + a.z_off + h * DV + v])
                  : 0.f;
  };
  auto norm_pass = [&](int item, int x, int q3) {
    const int seq = item / a.Hv, h = item % a.Hv;
    if (part == 0) {
#pragma unroll
      for (int t = 0; t < MAXT; ++t) {
        if (t >= T) break;
        const size_t tok = (size_t)seq * T + t;
        const float rstd = rsqrtf(sm.ssq[q3][t] / DV + a.eps);
        a.out[tok * (a.Hv * DV) + h * DV + v] = __float2bfloat16(sm.o[x][t][v] * rstd * norm_w * silu(zr[t]));
      }
    }
  };
  for (int q = tid; q < 3 * MAXT; q += THREADS) (&sm.ssq[0][0])[q] = 0.f;

  int issued = 0, done = 0;
  if (blockIdx.x < items) {
    issue(blockIdx.x, 0);
    issued = 1;
  }
  int i = 0, last = -1;
  long long sec[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // profiling (a.dbg): thread 0's cycles per section
  long long tclk = a.dbg ? clock64() : 0;
  auto mark = [&](int k) {
    if (a.dbg && tid == 0) {
      const long long now = clock64();
      sec[k] += now - tclk;
      tclk = now;
    }
  };
  for (int item = blockIdx.x; item < items; item += gridDim.x, ++i) {
    const int b = i & 1;  // staging buffer = item parity (kf / qf / o use the same parity)
    // every thread acquires the copies through the barrier; the vote makes a timeout (flagged in the status word)
    // end the loop on every thread together
    const bool ok = __syncthreads_and(mbar_wait(&sm.full[b], (i >> 1) & 1, status));
    if (!ok) break;
    mark(0);
    ++done;
    const int seq = item / a.Hv, h = item % a.Hv;
    const int slot = sm.slot[seq], np = sm.ncommit[seq];
    const int L = np + T;  // tokens of this item: the accepted ones of the previous cycle, then this cycle's

    // ---- keys / queries -> fp32, part-padded (token order: accepted 0..np-1, then new np..np+T-1)
    for (int idx = tid; idx < (L + T) * (DK / 2); idx += THREADS) {
      const int row = idx / (DK / 2), c2 = (idx % (DK / 2)) * 2;
      const __nv_bfloat16* src;
      float* dst;
      if (row < L) {
        src = sm.kq[b][row < np ? row : MAXT + row - np][0] + c2;
        dst = sm.kf[b][row];
      } else {
        src = sm.kq[b][MAXT + row - L][1] + c2;
        dst = sm.qf[b][row - L];
      }
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src));
      const int pc = (c2 / HK) * KP + (c2 % HK);
      dst[pc] = f.x;
      dst[pc + 1] = f.y;
    }
    // ---- this thread's 32 state values
    float S[HK];
#pragma unroll
    for (int c = 0; c < HK / 4; ++c) {
      const float4 x = *reinterpret_cast<const float4*>(&sm.state[b][tid * 32 + ((c ^ (tid & 7)) << 2)]);
      S[4 * c] = x.x;
      S[4 * c + 1] = x.y;
      S[4 * c + 2] = x.z;
      S[4 * c + 3] = x.w;
    }
    if (lane == 0) bulk_store_wait_read();  // this warp's state store of the last item has left buffer b ^ 1
    // the one barrier per item: fp32 keys / queries ready; every thread is done with the previous item, so its
    // staging buffer can be refilled and its outputs normalised
    __syncthreads();
    mark(1);
    const int next = item + gridDim.x;
    if (next < items) {
      issue(next, b ^ 1);
      ++issued;
    }
    mark(6);
    if (last >= 0) norm_pass(last, b ^ 1, (i + 2) % 3);
    mark(7);
    load_z(item);  // in flight while this item's recurrence runs; read by its norm pass after the next barrier
    if (tid < MAXT) sm.ssq[(i + 1) % 3][tid] = 0.f;  // item i - 2's sums (read by the last norm pass) -> item i + 1
    mark(2);

    float lg = 0.f;  // log Gamma
    // partial dot of this thread's slice with an fp32 row (four FMA chains), summed over the QT lanes of a column
    auto dot = [&](const float* row) {
      const float4* r4 = reinterpret_cast<const float4*>(row + part * KP);
      float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
      for (int c = 0; c < HK / 4; ++c) {
        const float4 x = r4[c];
        d0 = fmaf(x.x, S[4 * c], d0);
        d1 = fmaf(x.y, S[4 * c + 1], d1);
        d2 = fmaf(x.z, S[4 * c + 2], d2);
        d3 = fmaf(x.w, S[4 * c + 3], d3);
      }
      float d = (d0 + d1) + (d2 + d3);
#pragma unroll
      for (int o = 1; o < QT; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      return d;
    };
    // one token of the gated delta rule on S / Gamma: decay g (log), gate beta, value vv, key row kr
    auto step = [&](float g, float beta, float vv, const float* kr) {
      float lgn = lg + g;
      // the key slice stays in registers for both passes (the dot and the rank-1 update)
      float4 kx[HK / 4];
      const float4* r4 = reinterpret_cast<const float4*>(kr + part * KP);
#pragma unroll
      for (int q = 0; q < HK / 4; ++q) kx[q] = r4[q];
      float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
      for (int q = 0; q < HK / 4; ++q) {
        d0 = fmaf(kx[q].x, S[4 * q], d0);
        d1 = fmaf(kx[q].y, S[4 * q + 1], d1);
        d2 = fmaf(kx[q].z, S[4 * q + 2], d2);
        d3 = fmaf(kx[q].w, S[4 * q + 3], d3);
      }
      float d = (d0 + d1) + (d2 + d3);
#pragma unroll
      for (int o = 1; o < QT; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      const float mem = __expf(lgn) * d;
      if (lgn < -60.f) {  // uniform over the CTA: the gates are per (token, head)
        const float f = __expf(lgn);
#pragma unroll
        for (int k = 0; k < HK; ++k) S[k] *= f;
        lgn = 0.f;
      }
      lg = lgn;
      const float c = beta * (vv - mem) * __expf(-lg);  // delta / Gamma
#pragma unroll
      for (int q = 0; q < HK / 4; ++q) {
        const float4 x = kx[q];
        S[4 * q] = fmaf(x.x, c, S[4 * q]);
        S[4 * q + 1] = fmaf(x.y, c, S[4 * q + 1]);
        S[4 * q + 2] = fmaf(x.z, c, S[4 * q + 2]);
        S[4 * q + 3] = fmaf(x.w, c, S[4 * q + 3]);
      }
    };
    for (int t = 0; t < np; ++t)
      step(sm.gb[b][0][2 * t], sm.gb[b][0][2 * t + 1], __bfloat162float(sm.v[b][t][v]), sm.kf[b][t]);
    mark(3);
    if (np > 0) {
      // the committed state Gamma * S back into its slot; each warp stores its 32 threads' slices (4 KB,
      // contiguous in the swizzled layout) with one bulk copy, so no block-wide barrier is needed
      const float gam = __expf(lg);
#pragma unroll
      for (int c = 0; c < HK / 4; ++c)
        *reinterpret_cast<float4*>(&sm.state[b][tid * 32 + ((c ^ (tid & 7)) << 2)]) =
            make_float4(gam * S[4 * c], gam * S[4 * c + 1], gam * S[4 * c + 2], gam * S[4 * c + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0)
        bulk_store(a.ssm_state + ((size_t)slot * a.Hv + h) * DK * DV + wid * 32 * 32, &sm.state[b][wid * 32 * 32],
                   32 * 32 * 4);
    }
    mark(4);
    for (int t = 0; t < T; ++t) {
      step(sm.gb[b][1][2 * t], sm.gb[b][1][2 * t + 1], __bfloat162float(sm.v[b][MAXT + t][v]), sm.kf[b][np + t]);
      const float o = __expf(lg) * dot(sm.qf[b][t]);
      if (part == 0) sm.o[b][t][v] = o;
      const float sq = warp_sum(part == 0 ? o * o : 0.f);  // this warp's 8 columns
      if (lane == 0) atomicAdd(&sm.ssq[i % 3][t], sq);
    }
    mark(5);
    last = item;
  }
  if (a.dbg && tid == 0) {
    for (int k = 0; k < 8; ++k) a.dbg[blockIdx.x * 10 + k] = sec[k];
    a.dbg[blockIdx.x * 10 + 8] = done;
  }
  __syncthreads();
  if (last >= 0) norm_pass(last, (i - 1) & 1, (i - 1) % 3);
  // drain copies still in flight (only after a failed wait), bounded; then this warp's committed-state stores
  if (tid == 0)
    for (int j = done; j < issued; ++j) mbar_wait(&sm.full[j & 1], (j >> 1) & 1, status);
  if (lane == 0) bulk_store_wait_all();
}

int gdn_decode(const GdnArgs& a, int parity, int num_sms, uint32_t* status, cudaStream_t st) {
  if (a.num_seqs == 0) return 0;
  if (a.q_per_seq > a.max_q) return 3;
  const int C = a.conv_dim;
  if (a.Dk == 128 && a.Dv == 128) {
    if (C % 128) return 3;
    gdn_conv_prep_kernel<128><<<dim3(a.num_seqs, C / 128), 128, 0, st>>>(a, parity);
    if (!a.commit_current && a.max_q <= gdnp::MAXT && a.max_q % 2 == 0 && a.num_seqs <= gdnp::MAXS && num_sms > 0) {
      const size_t smem = sizeof(gdnp::Smem) + 128;
      static std::atomic<uint64_t> attr_devs{0};
      if (const int e = smem_attr_once(attr_devs, (const void*)gdn_verify_persistent_kernel, (int)smem)) return e;
      const int items = a.num_seqs * a.Hv;
      gdn_verify_persistent_kernel<<<items < num_sms ? items : num_sms, gdnp::THREADS, smem, st>>>(a, parity, status);
      return (int)cudaGetLastError();
    }
    gdn_recurrent_kernel<128, 128, 4><<<dim3(a.num_seqs, a.Hv), 512, 0, st>>>(a, parity);
  } else if (a.Dk == 64 && a.Dv == 64) {
    if (C % 64) return 3;
    gdn_conv_prep_kernel<64><<<dim3(a.num_seqs, C / 64), 64, 0, st>>>(a, parity);
    gdn_recurrent_kernel<64, 64, 2><<<dim3(a.num_seqs, a.Hv), 128, 0, st>>>(a, parity);
  } else {
    return 3;
  }
  return (int)cudaGetLastError();
}

}  // namespace afb
