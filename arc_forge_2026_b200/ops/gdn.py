"""Gated DeltaNet decode / speculative verify on the native kernels, its state buffers, and the oracle.

State per sequence slot (see csrc/gdn.cu): conv state [slots, 3, C] bf16, recurrent state [slots, Hv, Dk, Dv]
fp32, two parities of pending buffers for the deferred commit, and ``n_commit`` [slots] (accepted tokens of the
previous cycle, written by the accept kernel).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ..models import reference as R
from ._ext import C


@dataclass
class GdnShape:
    Hk: int
    Dk: int
    Hv: int
    Dv: int

    @property
    def conv_dim(self):
        return 2 * self.Hk * self.Dk + self.Hv * self.Dv

    @property
    def z_off(self):
        return self.conv_dim

    @property
    def ba_off(self):
        return self.conv_dim + self.Hv * self.Dv

    @property
    def mixed_dim(self):
        return self.ba_off + 2 * self.Hv


class GdnState:
    """Recurrent + conv state of every slot for one GDN layer, and the pending buffers of the deferred commit."""

    def __init__(self, shape: GdnShape, slots: int, max_q: int, device, state_dtype=torch.float32):
        s = shape
        dev = torch.device(device)
        max_q += max_q % 2  # even: each head's (g, beta) block is then 16-byte aligned for bulk copies
        self.shape = s
        self.conv = torch.zeros(slots, 3, s.conv_dim, dtype=torch.bfloat16, device=dev)
        self.ssm = torch.zeros(slots, s.Hv, s.Dv, s.Dk, dtype=state_dtype, device=dev)  # S transposed
        self.pend_in = torch.zeros(2, slots, max_q, s.conv_dim, dtype=torch.bfloat16, device=dev)
        self.pend_qk = torch.zeros(2, slots, max_q, 2 * s.Hk * s.Dk, dtype=torch.bfloat16, device=dev)
        self.pend_v = torch.zeros(2, slots, max_q, s.Hv * s.Dv, dtype=torch.bfloat16, device=dev)
        self.pend_gb = torch.zeros(2, slots, s.Hv, max_q, 2, dtype=torch.float32, device=dev)

    def nbytes(self):
        return sum(t.numel() * t.element_size() for t in (self.conv, self.ssm, self.pend_in, self.pend_qk,
                                                          self.pend_v, self.pend_gb))


class GdnScratch:
    """Pending buffers for a prefill/commit-all call of up to ``seqs`` sequences x ``max_q`` tokens."""

    def __init__(self, shape: GdnShape, seqs: int, max_q: int, device):
        s = shape
        self.pend_in = torch.empty(2, 1, 1, s.conv_dim, dtype=torch.bfloat16, device=device)
        self.pend_in = torch.empty(2, seqs, max_q, s.conv_dim, dtype=torch.bfloat16, device=device)
        self.pend_qk = torch.empty(2, seqs, max_q, 2 * s.Hk * s.Dk, dtype=torch.bfloat16, device=device)
        self.pend_v = torch.empty(2, seqs, max_q, s.Hv * s.Dv, dtype=torch.bfloat16, device=device)
        self.pend_gb = torch.empty(2, seqs, s.Hv, max_q, 2, dtype=torch.float32, device=device)


def gdn_decode(mixed, shape: GdnShape, state: GdnState, conv_w, A_log, dt_bias, norm_w, n_commit, seq_slot, out,
               q_per_seq: int, parity: int = 0, commit_current: bool = False, scratch: GdnScratch | None = None,
               eps: float = 1e-6, dbg=None):
    """mixed [S*q, mixed_dim] bf16 -> out [S*q, Hv*Dv] bf16 (gated-RMSNorm'd GDN output). ``dbg``: optional int64
    [CTAs * 24] section clocks of the tensor-core verify kernel (profiling)."""
    pend = scratch if commit_current else state
    C().gdn_decode(mixed, shape.z_off, shape.ba_off, conv_w, state.conv, state.ssm, pend.pend_in, pend.pend_qk,
                   pend.pend_v, pend.pend_gb, n_commit, seq_slot, A_log, dt_bias, norm_w, out, q_per_seq,
                   shape.Hk, shape.Dk, shape.Hv, shape.Dv, commit_current, parity, eps, dbg)
    return out


def gdn_reference_from_mixed(mixed: torch.Tensor, shape: GdnShape, conv_w, A_log, dt_bias, norm_w, eps=1e-6):
    """Sequential fp32 oracle for one sequence: mixed [L, mixed_dim] -> out [L, Hv*Dv]."""
    s = shape
    x = mixed.float()[None]  # [1, L, W]
    conv_in = x[..., : s.conv_dim]
    y, _ = R.causal_conv1d(conv_in, conv_w.float(), None)
    q = y[..., : s.Hk * s.Dk].reshape(1, -1, s.Hk, s.Dk)
    k = y[..., s.Hk * s.Dk: 2 * s.Hk * s.Dk].reshape(1, -1, s.Hk, s.Dk)
    v = y[..., 2 * s.Hk * s.Dk:].reshape(1, -1, s.Hv, s.Dv)
    rep = s.Hv // s.Hk
    q = (R.l2norm(q) * s.Dk ** -0.5).repeat_interleave(rep, 2)
    k = R.l2norm(k).repeat_interleave(rep, 2)
    b = x[..., s.ba_off: s.ba_off + s.Hv]
    a = x[..., s.ba_off + s.Hv: s.ba_off + 2 * s.Hv]
    g, beta = R.gdn_gates(b, a, A_log, dt_bias)
    o, _ = R.gated_delta_rule(q, k, v, g, beta)
    z = x[..., s.z_off: s.z_off + s.Hv * s.Dv].reshape(1, -1, s.Hv, s.Dv)
    o = R.gated_rms_norm(o, z, norm_w.float(), eps)
    return o.reshape(-1, s.Hv * s.Dv)
