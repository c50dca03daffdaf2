"""Chunked gated delta rule for training (autograd-friendly, PyTorch ops).

The sequence is cut into chunks of C tokens; inside a chunk the delta-rule recurrence is solved in closed form
(lower-triangular system on ``beta * k k^T`` weighted by the within-chunk decay), and a [Dk, Dv] state carries
across chunks (the WY formulation of DeltaNet, Yang et al. 2024, with the gate of Gated DeltaNet). It computes
exactly the recurrence of ``models.reference.gated_delta_rule`` (tests compare them); the GPU decode path uses
the recurrent kernels in csrc/gdn.cu.
"""
from __future__ import annotations

import torch


def chunk_gated_delta_rule(q, k, v, g, beta, chunk: int = 64, state=None):
    """q, k [B, T, H, Dk] (normalised, q scaled), v [B, T, H, Dv], g/beta [B, T, H] -> (o [B,T,H,Dv], state)."""
    B, T, H, Dk = k.shape
    Dv = v.shape[-1]
    dt = torch.float32
    pad = (chunk - T % chunk) % chunk
    q, k, v = (x.transpose(1, 2).to(dt) for x in (q, k, v))  # [B, H, T, D]
    g, beta = g.transpose(1, 2).to(dt), beta.transpose(1, 2).to(dt)
    if pad:
        q = torch.nn.functional.pad(q, (0, 0, 0, pad))
        k = torch.nn.functional.pad(k, (0, 0, 0, pad))
        v = torch.nn.functional.pad(v, (0, 0, 0, pad))
        g = torch.nn.functional.pad(g, (0, pad))
        beta = torch.nn.functional.pad(beta, (0, pad))
    n = q.shape[2] // chunk
    q, k, v = (x.reshape(B, H, n, chunk, -1) for x in (q, k, v))
    g, beta = g.reshape(B, H, n, chunk), beta.reshape(B, H, n, chunk)
    v_beta = v * beta[..., None]
    k_beta = k * beta[..., None]
    gc = g.cumsum(-1)  # within-chunk cumulative log decay
    tri_incl = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool, device=q.device))
    tri_strict = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool, device=q.device), -1)
    decay = (gc[..., :, None] - gc[..., None, :]).masked_fill(~tri_incl, float("-inf")).exp()
    # A = (I + strict_lower(beta k k^T * decay))^-1
    a = -(k_beta @ k.transpose(-1, -2) * decay).masked_fill(~tri_strict, 0.0)
    eye = torch.eye(chunk, dtype=dt, device=q.device)
    A = torch.linalg.solve_triangular(eye - a, eye.expand_as(a), upper=False, unitriangular=True)
    u = A @ v_beta                                   # pseudo-values
    w = A @ (k_beta * gc.exp()[..., None])          # decayed keys
    S = torch.zeros(B, H, Dk, Dv, dtype=dt, device=q.device) if state is None else state.to(dt).transpose(0, 0)
    outs = []
    qk_mask = ~tri_incl
    for i in range(n):
        qi, ki = q[:, :, i], k[:, :, i]
        attn = (qi @ ki.transpose(-1, -2) * decay[:, :, i]).masked_fill(qk_mask, 0.0)
        v_new = u[:, :, i] - w[:, :, i] @ S
        o_inter = (qi * gc[:, :, i].exp()[..., None]) @ S
        outs.append(o_inter + attn @ v_new)
        last = gc[:, :, i, -1]
        S = S * last.exp()[..., None, None] + (ki * (last[..., None] - gc[:, :, i]).exp()[..., None]).transpose(-1, -2) @ v_new
    o = torch.stack(outs, 2).reshape(B, H, n * chunk, Dv)[:, :, :T]
    return o.transpose(1, 2), S
