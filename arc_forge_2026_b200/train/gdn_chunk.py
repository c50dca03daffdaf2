"""Chunked gated delta rule for training.

The sequence is cut into chunks of C tokens; inside a chunk the delta-rule recurrence is solved in closed form
(lower-triangular system on ``beta * k k^T`` weighted by the within-chunk decay), and a [Dk, Dv] state carries
across chunks (the WY formulation of DeltaNet, Yang et al. 2024, with the gate of Gated DeltaNet). It computes
exactly the recurrence of ``models.reference.gated_delta_rule`` (tests compare them).

Work split (the reference trains through FlashQLA's chunk scan, ``train/preflight.py:280-365``):

* everything inside a chunk (decay matrix, triangular solve, pseudo-values ``u``, decayed keys ``w``, the
  intra-chunk attention, the outputs) is a handful of batched products over all chunks at once;
* the only sequential part -- the state passed from chunk to chunk -- is one native kernel per direction
  (``csrc/gdn_chunk.cu``): forward ``X_i = U_i - W_i S_i``, ``S_{i+1} = e^{last} S_i + Kd_i^T X_i``, and the
  reverse pass of its gradient; :class:`_InterChunk` carries the hand-derived backward of that recurrence, so
  autograd never unrolls a per-chunk loop.

On CPU the same two recurrences run as a plain loop (the oracle the native kernel is tested against).
"""
from __future__ import annotations

import torch


def _scan(m1, m2, y, qm, last, init, reverse: bool, precise: bool = False, reset=None):
    """X = Y + s1 * M1 St ; St <- e^{last} St (+ Qm) + s2 * M2^T X over chunks (forward, or reverse order).

    m1, m2 [BH, n, C, Dk]; y [BH, n, C, Dv]; qm [BH, n, Dk, Dv] or None; last [BH, n]; init [BH, Dk, Dv] or None.
    Returns (states before each step [BH, n, Dk, Dv], X [BH, n, C, Dv], final state [BH, Dk, Dv]).
    On CUDA with Dk = 128 the scan runs on tensor cores with bf16 operands and fp32 accumulation (the precision
    class of the chunk kernels the reference trains with); ``precise`` selects the fp32 SIMT kernel. ``reset`` [n]
    int32 (packed sequences): chunk i starts a new sequence (zero state before it, no gradient across it)."""
    BH, n, C, Dk = m1.shape
    Dv = y.shape[-1]
    if m1.is_cuda:
        from ..ops import C as ext
        m1, m2, y, last = (t.float().contiguous() for t in (m1, m2, y, last))
        qm = qm.float().contiguous() if qm is not None else None
        init = init.float().contiguous() if init is not None else None
        states = torch.empty(BH, n, Dk, Dv, device=m1.device, dtype=torch.float32)
        x = torch.empty_like(y)
        final = torch.empty(BH, Dk, Dv, device=m1.device, dtype=torch.float32)
        ext().gdn_chunk_scan(m1, m2, y, qm, last, init, states, x, final, reverse, precise, reset)
        return states, x, final
    s1, s2 = (1.0, -1.0) if reverse else (-1.0, 1.0)
    St = torch.zeros(BH, Dk, Dv, dtype=y.dtype) if init is None else init.clone()
    states = torch.empty(BH, n, Dk, Dv, dtype=y.dtype)
    x = torch.empty_like(y)
    rs = None if reset is None else [bool(r) for r in reset.tolist()]
    for i in (range(n - 1, -1, -1) if reverse else range(n)):
        if rs is not None and (rs[i + 1] if reverse and i + 1 < n else (rs[i] if not reverse else False)):
            St = torch.zeros_like(St)
        states[:, i] = St
        xi = y[:, i] + s1 * (m1[:, i] @ St)
        x[:, i] = xi
        St = last[:, i].exp()[:, None, None] * St + s2 * (m2[:, i].transpose(-1, -2) @ xi)
        if qm is not None:
            St = St + qm[:, i]
    if reverse and rs is not None and rs[0]:
        St = torch.zeros_like(St)
    return states, x, St


class _InterChunk(torch.autograd.Function):
    """o = (q e^{gc}) S_i + attn_i (u_i - w_i S_i), with the state S carried across chunks.

    q, k, w [BH, n, C, Dk]; u [BH, n, C, Dv]; gc [BH, n, C] (within-chunk cumulative log decay)."""

    @staticmethod
    def _intra(q, k, gc):
        C = q.shape[-2]
        tri = torch.ones(C, C, dtype=torch.bool, device=q.device).tril()
        D = (gc[..., :, None] - gc[..., None, :]).masked_fill(~tri, float("-inf")).exp()
        attn = (q @ k.transpose(-1, -2)) * D
        qd = q * gc.exp()[..., None]
        last = gc[..., -1]
        kd = k * (last[..., None] - gc).exp()[..., None]
        return D, attn, qd, kd, last

    @staticmethod
    def forward(ctx, q, k, u, w, gc, init, precise=False, reset=None):
        D, attn, qd, kd, last = _InterChunk._intra(q, k, gc)
        states, vnew, final = _scan(w, kd, u, None, last, init, reverse=False, precise=precise, reset=reset)
        ctx.precise, ctx.reset = precise, reset
        o = qd @ states + attn @ vnew
        ctx.save_for_backward(q, k, w, gc, states, vnew)
        ctx.has_init = init is not None
        return o, final

    @staticmethod
    def backward(ctx, do, dfinal):
        q, k, w, gc, states, vnew = ctx.saved_tensors
        D, attn, qd, kd, last = _InterChunk._intra(q, k, gc)
        do = do.float().contiguous()
        P = attn.transpose(-1, -2) @ do                      # attn^T dO
        Qm = qd.transpose(-1, -2) @ do                       # qd^T dO
        dnext, dv, dS0 = _scan(kd, w, P, Qm, last, dfinal if dfinal is not None else None, reverse=True,
                               precise=ctx.precise, reset=ctx.reset)
        # dnext[:, i] = dS_{i+1}; dv = dL/du = dL/d(vnew)
        dw = -(dv @ states.transpose(-1, -2))
        dqd = do @ states.transpose(-1, -2)
        dq = dqd * gc.exp()[..., None]
        dgc = (dqd * qd).sum(-1)
        dattn = do @ vnew.transpose(-1, -2)                  # zero above the diagonal through D
        G = dattn * attn
        dq = dq + (dattn * D) @ k
        dk = (dattn * D).transpose(-1, -2) @ q
        dgc = dgc + G.sum(-1) - G.sum(-2)
        dkd = vnew @ dnext.transpose(-1, -2)
        dk = dk + dkd * (last[..., None] - gc).exp()[..., None]
        E = (dkd * kd).sum(-1)
        dgc = dgc - E
        dlast = E.sum(-1) + last.exp() * (dnext * states).sum((-1, -2))
        dgc = torch.cat([dgc[..., :-1], (dgc[..., -1] + dlast)[..., None]], -1)
        return dq, dk, dv, dw, dgc, (dS0 if ctx.has_init else None), None, None


class _GdnChunkNative(torch.autograd.Function):
    """The whole chunked rule in native kernels (``csrc/gdn_chunk_train.cu`` around the tensor-core scan of
    ``csrc/gdn_chunk.cu``): q, k [B, T, Hk, 128] bf16, v [B, T, Hv, 128] bf16 (value head h reads key head
    h // (Hv / Hk): no repeat of q / k), g, beta [B, T, Hv] fp32 -> o [B, T, Hv, 128] bf16, final state
    [B, Hv, 128, 128] fp32. Backward: attn^T dO / Qm, the reverse scan, then the inter-chunk and WY gradients."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, reset=None):
        from ..ops import C as ext
        B, T, Hk, D = q.shape
        Hv = v.shape[2]
        n, BH = (T + 63) // 64, B * Hv
        dev = q.device
        f32 = dict(device=dev, dtype=torch.float32)
        w_t = torch.empty(BH, n, 64, 128, device=dev, dtype=torch.bfloat16)
        kd_t = torch.empty_like(w_t)
        u = torch.empty(BH, n, 64, 128, **f32)
        gc = torch.empty(BH, n, 64, **f32)
        last = torch.empty(BH, n, **f32)
        A = torch.empty(BH, n, 64, 64, **f32)
        slots = [None] * 26
        slots[0:11] = [q, k, v, g, beta, w_t, kd_t, u, gc, last, A]
        c = ext()
        c.gdn_train(0, slots, B, T, Hk, Hv)
        states = torch.empty(BH, n, 128, 128, **f32)
        vnew = torch.empty_like(u)
        final = torch.empty(BH, 128, 128, **f32)
        c.gdn_chunk_scan_tiles(w_t, kd_t, u, None, last, None, states, vnew, final, False, reset)
        o = torch.empty(B, T, Hv, 128, device=dev, dtype=torch.bfloat16)
        slots[11:14] = [states, vnew, o]
        c.gdn_train(1, slots, B, T, Hk, Hv)
        ctx.save_for_backward(q, k, v, g, beta, w_t, kd_t, gc, last, A, states, vnew)
        ctx.dims, ctx.reset = (B, T, Hk, Hv), reset
        return o, final.view(B, Hv, 128, 128)

    @staticmethod
    def backward(ctx, do, dfinal):
        from ..ops import C as ext
        q, k, v, g, beta, w_t, kd_t, gc, last, A, states, vnew = ctx.saved_tensors
        B, T, Hk, Hv = ctx.dims
        BH = B * Hv
        c = ext()
        do = (torch.zeros(B, T, Hv, 128, device=q.device, dtype=torch.bfloat16) if do is None
              else do.to(torch.bfloat16).contiguous())
        P, Qm = torch.empty_like(vnew), torch.empty_like(states)
        slots = [None] * 26
        slots[0:5] = [q, k, v, g, beta]
        slots[8], slots[10], slots[11], slots[12] = gc, A, states, vnew
        slots[14], slots[15], slots[16] = do, P, Qm
        c.gdn_train(2, slots, B, T, Hk, Hv)
        dnext, du = torch.empty_like(states), torch.empty_like(vnew)
        ds0 = torch.empty(BH, 128, 128, device=q.device, dtype=torch.float32)
        init = None if dfinal is None else dfinal.float().reshape(BH, 128, 128).contiguous()
        c.gdn_chunk_scan_tiles(kd_t, w_t, P, Qm, last, init, dnext, du, ds0, True, ctx.reset)
        del P, Qm
        f32 = dict(device=q.device, dtype=torch.float32)
        dq = torch.empty(B, T, Hv, 128, **f32)
        dk, dv = torch.empty_like(dq), torch.empty_like(dq)
        dw, dgc = torch.empty_like(vnew), torch.empty_like(gc)
        dg, dbeta = torch.empty(B, T, Hv, **f32), torch.empty(B, T, Hv, **f32)
        slots[17:26] = [dnext, du, dw, dgc, dq, dk, dv, dg, dbeta]
        c.gdn_train(3, slots, B, T, Hk, Hv)
        c.gdn_train(4, slots, B, T, Hk, Hv)
        rep = Hv // Hk
        if rep > 1:
            dq = dq.view(B, T, Hk, rep, 128).sum(3)
            dk = dk.view(B, T, Hk, rep, 128).sum(3)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), dg, dbeta, None


def _native_ok(q, k, v, g, chunk, state, precise) -> bool:
    return (q.is_cuda and not precise and state is None and chunk == 64 and q.shape[-1] == 128
            and v.shape[-1] == 128 and v.shape[2] % k.shape[2] == 0)


def chunk_gated_delta_rule(q, k, v, g, beta, chunk: int = 64, state=None, precise: bool = False, chunk_reset=None):
    """q, k [B, T, Hk, Dk] (normalised, q scaled), v [B, T, Hv, Dv], g/beta [B, T, Hv] -> (o [B,T,Hv,Dv], state).

    Grouped values: value head h uses key head h // (Hv / Hk). On CUDA with Dk = Dv = 128 and no initial state the
    whole rule runs in the native kernels (bf16 operands, fp32 accumulation, o in bf16); ``precise`` keeps the
    fp32 torch path with the fp32 scan. ``chunk_reset`` [ceil(T / chunk)] int32 (packed sequences aligned to
    chunks, B = 1): chunk i starts a new sequence, so no state or gradient crosses into it."""
    from . import kernels
    if kernels.use("gdn_chunk") and _native_ok(q, k, v, g, chunk, state, precise):
        kernels.hit("gdn_chunk", True)
        bf = torch.bfloat16
        return _GdnChunkNative.apply(q.to(bf).contiguous(), k.to(bf).contiguous(), v.to(bf).contiguous(),
                                     g.float().contiguous(), beta.float().contiguous(),
                                     None if chunk_reset is None else chunk_reset.int().contiguous())
    if q.is_cuda and not precise:
        kernels.hit("gdn_chunk", False)
    if k.shape[2] != v.shape[2]:
        rep = v.shape[2] // k.shape[2]
        q, k = q.repeat_interleave(rep, 2), k.repeat_interleave(rep, 2)
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
    q, k, v = (x.reshape(B * H, n, chunk, -1) for x in (q, k, v))
    g, beta = g.reshape(B * H, n, chunk), beta.reshape(B * H, n, chunk)
    k_beta = k * beta[..., None]
    gc = g.cumsum(-1)  # within-chunk cumulative log decay
    tri_incl = torch.ones(chunk, chunk, dtype=torch.bool, device=q.device).tril()
    tri_strict = torch.ones(chunk, chunk, dtype=torch.bool, device=q.device).tril(-1)
    decay = (gc[..., :, None] - gc[..., None, :]).masked_fill(~tri_incl, float("-inf")).exp()
    # A = (I + strict_lower(beta k k^T * decay))^-1
    a = -(k_beta @ k.transpose(-1, -2) * decay).masked_fill(~tri_strict, 0.0)
    eye = torch.eye(chunk, dtype=dt, device=q.device)
    A = torch.linalg.solve_triangular(eye - a, eye.expand_as(a), upper=False, unitriangular=True)
    u = A @ (v * beta[..., None])                    # pseudo-values
    w = A @ (k_beta * gc.exp()[..., None])          # decayed keys
    init = None if state is None else state.to(dt).reshape(B * H, Dk, Dv)
    o, S = _InterChunk.apply(q, k, u, w, gc, init, precise,
                             None if chunk_reset is None else chunk_reset.int().to(q.device).contiguous())
    o = o.reshape(B, H, n * chunk, Dv)[:, :, :T]
    return o.transpose(1, 2), S.reshape(B, H, Dk, Dv)


def chunk_gated_delta_rule_loop(q, k, v, g, beta, chunk: int = 64, state=None):
    """The same computation with the inter-chunk state as an autograd-unrolled loop (test oracle)."""
    B, T, H, Dk = k.shape
    Dv = v.shape[-1]
    dt = torch.float32
    pad = (chunk - T % chunk) % chunk
    q, k, v = (x.transpose(1, 2).to(dt) for x in (q, k, v))
    g, beta = g.transpose(1, 2).to(dt), beta.transpose(1, 2).to(dt)
    if pad:
        q, k, v = (torch.nn.functional.pad(x, (0, 0, 0, pad)) for x in (q, k, v))
        g, beta = torch.nn.functional.pad(g, (0, pad)), torch.nn.functional.pad(beta, (0, pad))
    n = q.shape[2] // chunk
    q, k, v = (x.reshape(B, H, n, chunk, -1) for x in (q, k, v))
    g, beta = g.reshape(B, H, n, chunk), beta.reshape(B, H, n, chunk)
    k_beta = k * beta[..., None]
    gc = g.cumsum(-1)
    tri_incl = torch.ones(chunk, chunk, dtype=torch.bool, device=q.device).tril()
    tri_strict = torch.ones(chunk, chunk, dtype=torch.bool, device=q.device).tril(-1)
    decay = (gc[..., :, None] - gc[..., None, :]).masked_fill(~tri_incl, float("-inf")).exp()
    a = -(k_beta @ k.transpose(-1, -2) * decay).masked_fill(~tri_strict, 0.0)
    eye = torch.eye(chunk, dtype=dt, device=q.device)
    A = torch.linalg.solve_triangular(eye - a, eye.expand_as(a), upper=False, unitriangular=True)
    u = A @ (v * beta[..., None])
    w = A @ (k_beta * gc.exp()[..., None])
    S = torch.zeros(B, H, Dk, Dv, dtype=dt, device=q.device) if state is None else state.to(dt)
    outs = []
    for i in range(n):
        qi, ki = q[:, :, i], k[:, :, i]
        attn = (qi @ ki.transpose(-1, -2) * decay[:, :, i]).masked_fill(~tri_incl, 0.0)
        v_new = u[:, :, i] - w[:, :, i] @ S
        outs.append((qi * gc[:, :, i].exp()[..., None]) @ S + attn @ v_new)
        last = gc[:, :, i, -1]
        S = S * last.exp()[..., None, None] + (ki * (last[..., None] - gc[:, :, i]).exp()[..., None]).transpose(-1, -2) @ v_new
    o = torch.stack(outs, 2).reshape(B, H, n * chunk, Dv)[:, :, :T]
    return o.transpose(1, 2), S
