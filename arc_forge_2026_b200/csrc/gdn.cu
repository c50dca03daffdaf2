// Gated DeltaNet (GDN) for decode and speculative verify, with the accepted-prefix commit deferred into the
// next cycle (so a verify cycle reads and writes each recurrent state once, the same traffic as plain decode).
//
// Per sequence slot the engine keeps:
//   conv_state [slots, 3, C]            last 3 committed pre-conv inputs (C = 2*Hk*Dk + Hv*Dv channels)
//   ssm_state  [slots, Hv, Dv, Dk] fp32 committed recurrent state, stored transposed (S^T; o_t = S^T q_t)
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
//   (rms over Dv, * w * silu(z)) before the bf16 store. Verify cycles with Dk = Dv = 128 run gdn_verify_tc_kernel
//   (gdn_tc.cu) instead: the same rule as one chunk on the tensor cores.
// The math is the recurrence of training/work (FlashQLA's chunked kernels compute the same rule in chunks).
#include "common.cuh"
#include "kernels.h"

namespace afb {

template <int DK>
__global__ void __launch_bounds__(DK) gdn_conv_prep_kernel(GdnArgs a, int parity) {
  grid_dep_wait();     // launched with programmatic serialization: the previous kernel must be complete
  grid_dep_trigger();
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
  // the state is stored transposed, S^T [Dv, Dk] row-major (the layout the tensor-core verify kernel moves with
  // TMA): this thread's 32 rows of column v are contiguous
  float* sp = a.ssm_state + (((size_t)slot * a.Hv + h) * DV + v) * DK + part * HK;
  auto sidx = [&](int k) -> size_t { return (size_t)k; };
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

int gdn_verify_tc(const GdnArgs& a, int parity, int num_sms, uint32_t* status, cudaStream_t st);  // gdn_tc.cu

int gdn_decode(const GdnArgs& a, int parity, int num_sms, uint32_t* status, cudaStream_t st) {
  if (a.num_seqs == 0) return 0;
  if (a.q_per_seq > a.max_q) return 3;
  const int C = a.conv_dim;
  if (a.Dk == 128 && a.Dv == 128) {
    if (C % 128) return 3;
    if (const int rc = launch_pdl(gdn_conv_prep_kernel<128>, dim3(a.num_seqs, C / 128), dim3(128), 0, st, a,
        parity)) return rc;
    if (const int rc = gdn_verify_tc(a, parity, num_sms, status, st); rc != -1) return rc;
    gdn_recurrent_kernel<128, 128, 4><<<dim3(a.num_seqs, a.Hv), 512, 0, st>>>(a, parity);
  } else if (a.Dk == 64 && a.Dv == 64) {
    if (C % 64) return 3;
    if (const int rc = launch_pdl(gdn_conv_prep_kernel<64>, dim3(a.num_seqs, C / 64), dim3(64), 0, st, a,
        parity)) return rc;
    gdn_recurrent_kernel<64, 64, 2><<<dim3(a.num_seqs, a.Hv), 128, 0, st>>>(a, parity);
  } else {
    return 3;
  }
  return (int)cudaGetLastError();
}

}  // namespace afb
