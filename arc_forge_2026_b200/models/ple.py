"""Per-layer n-gram embeddings (PLE): the hash contract, the fp32 reference layer and the hot-table tools.

Hash contract (the reference's ``training/work/qwen38fn_eval/ple_ngram.py:23-33,55-84``, read there from the serving
model; kept identical so a table trained elsewhere indexes the same rows):

    m_i   = 2 * (splitmix64(seed + GAMMA * (i + 1)) mod half) + 1,   half = max(1, ((2^63 - 1) // vocab) // 2)
    mix_2 = cur * m_0  XOR  prev_1 * m_1                      (int64, wrapping)
    mix_n = mix_(n-1)  XOR  prev_(n-1) * m_(n-1)
    id_h  = (mix_n mod p_h) + offset_h       heads h of order n share mix_n and differ only in the prime modulus

``p_h`` is the (h+1)-th prime after ``ngram_vocab_size_base - 1``; ``offset_h`` the sum of the earlier moduli. History
restarts after an EOS token and at a packed segment's start: a missing previous token reads as EOS
(``qwen38fn_lora/ple_packed.py:22-45``).

The layer (``ple_packed.py:48-76``), over a stream of G branches (G = 1 without hyper-connections):

    e     = concat_h table[id_h]                               [T, E]      E = ple_embed_dim
    k     = rmsnorm_g(e @ W_key^T)                             [T, G, H]   grouped per branch
    q     = rmsnorm_g(h)                                       [T, G, H]
    g     = (k . q) / sqrt(H);  g = sign(g) sqrt(max(|g|, 1e-6))
    v     = sigmoid(g) * (e @ W_value^T)                       [T, G, H]
    out   = v + causal_conv(rmsnorm_g(v))                      depthwise, kernel 4, per segment, zero left pad
    h    += out

Choices where the reference's model code is not in its tree: the three norms are grouped per branch (as the
hyper-connection norm is), the conv's dilation is a config field (default 1), the layer is applied before the
layer's attention / GDN sub-layer, and ``ple_layer_ids`` counts layers from 0.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

_MASK64 = (1 << 64) - 1
_GAMMA = 0x9E3779B97F4A7C15
_SM1 = 0xBF58476D1CE4E5B9
_SM2 = 0x94D049BB133111EB


def splitmix64(x: int) -> int:
    """One output of the SplitMix64 generator for state ``x`` (Steele, Lea, Flood 2014)."""
    x = (x + _GAMMA) & _MASK64
    x = ((x ^ (x >> 30)) * _SM1) & _MASK64
    x = ((x ^ (x >> 27)) * _SM2) & _MASK64
    return (x ^ (x >> 31)) & _MASK64


def ngram_multipliers(vocab: int, ngram_size: int, seed: int = 1234) -> list[int]:
    """Odd multipliers, one per n-gram position, small enough that ``m * (vocab - 1)`` fits in int64."""
    half = max(1, (((1 << 63) - 1) // vocab) // 2)
    out = [2 * (splitmix64((seed + _GAMMA * (i + 1)) & _MASK64) % half) + 1 for i in range(ngram_size)]
    assert all(m * (vocab - 1) < (1 << 63) for m in out)
    return out


def _is_prime(n: int) -> bool:
    """Deterministic Miller-Rabin for n < 3.3e24 (bases: the first 13 primes)."""
    if n < 2:
        return False
    small = (2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37, 41)
    for p in small:
        if n % p == 0:
            return n == p
    d, r = n - 1, 0
    while d % 2 == 0:
        d //= 2
        r += 1
    for a in small:
        x = pow(a, d, n)
        if x in (1, n - 1):
            continue
        for _ in range(r - 1):
            x = x * x % n
            if x == n - 1:
                break
        else:
            return False
    return True


def ngram_moduli(base: int, heads: int) -> list[int]:
    """The ``heads`` consecutive primes after ``base - 1``."""
    out, p = [], base - 1
    while len(out) < heads:
        p += 1
        if _is_prime(p):
            out.append(p)
    return out


class NgramHash:
    """The hash parameters of one model: multipliers, moduli, offsets (all int64)."""

    def __init__(self, cfg):
        self.n, self.hpn = cfg.ngram_size, cfg.heads_per_ngram
        self.eos = cfg.eos_token_id
        self.mult = ngram_multipliers(cfg.vocab_size, cfg.ngram_size, cfg.ngram_seed)
        self.moduli = ngram_moduli(cfg.ngram_vocab_size_base, cfg.ngram_heads)
        self.offsets = [0]
        for p in self.moduli[:-1]:
            self.offsets.append(self.offsets[-1] + p)
        self.rows = sum(self.moduli)

    def tensors(self, device):
        i64 = dict(dtype=torch.int64, device=device)
        return (torch.tensor(self.mult, **i64), torch.tensor(self.moduli, **i64), torch.tensor(self.offsets, **i64))

    def ids(self, tokens: torch.Tensor, seg_start: torch.Tensor | None = None,
            history: torch.Tensor | None = None) -> torch.Tensor:
        """tokens [T] (one sequence or a packed row) -> n-gram row ids [T, heads] (int64).
        ``seg_start`` [T]: index of each token's segment start (None: one segment from 0). ``history``: the up to
        n-1 tokens of the same sequence before ``tokens[0]`` (incremental decoding; fewer when the sequence is
        shorter)."""
        if history is not None and history.numel():
            full = self.ids(torch.cat([history.long().to(tokens.device), tokens.long()]))
            return full[history.numel():]
        T = tokens.shape[0]
        dev = tokens.device
        toks = tokens.long()
        pos = torch.arange(T, device=dev)
        eos_pos = torch.where(toks == self.eos, pos, torch.full_like(pos, -1))
        prev_eos = torch.cat([eos_pos.new_full((1,), -1), torch.cummax(eos_pos, 0).values[:-1]])
        start = prev_eos + 1 if seg_start is None else torch.maximum(seg_start.long(), prev_eos + 1)
        in_seg = pos - start
        eos = torch.full_like(toks, self.eos)
        mult, mod, off = self.tensors(dev)
        out = []
        mix = toks * mult[0]
        for order in range(2, self.n + 1):
            s = order - 1
            prev = torch.where(in_seg >= s, toks[(pos - s).clamp_min(0)], eos)
            mix = torch.bitwise_xor(mix, prev * mult[s])
            lo = (order - 2) * self.hpn
            out.append(torch.remainder(mix[:, None], mod[lo:lo + self.hpn][None]) + off[lo:lo + self.hpn][None])
        return torch.cat(out, 1)


def _group_rms(x: torch.Tensor, w: torch.Tensor, G: int, eps: float) -> torch.Tensor:
    """RMSNorm of every branch (the last dim is G*H) with the zero-centred weight [G*H]."""
    z = x.float().unflatten(-1, (G, -1))
    z = z * torch.rsqrt(z.square().mean(-1, keepdim=True) + eps)
    return z.flatten(-2) * (1.0 + w.float())


class PLELayer(nn.Module):
    """fp32 reference of one PLE layer. ``forward(h [.., T, G, H], tokens [.., T])`` returns the stream update."""

    def __init__(self, cfg):
        super().__init__()
        G, H, E = cfg.hc_count, cfg.hidden_size, cfg.ple_embed_dim
        self.G, self.H, self.E, self.eps = G, H, E, cfg.rms_norm_eps
        self.k, self.dil = cfg.ple_conv_kernel, cfg.ple_conv_dilation
        self.hash = NgramHash(cfg)
        self.head_dim = E // cfg.ngram_heads
        self.table = nn.Parameter(torch.zeros(self.hash.rows, self.head_dim))
        self.key_proj = nn.Parameter(torch.zeros(G * H, E))
        self.value_proj = nn.Parameter(torch.zeros(H, E))
        self.norm_key = nn.Parameter(torch.zeros(G * H))
        self.norm_query = nn.Parameter(torch.zeros(G * H))
        self.norm_conv = nn.Parameter(torch.zeros(G * H))
        self.conv = nn.Parameter(torch.zeros(G * H, self.k))

    def embed(self, rows: torch.Tensor) -> torch.Tensor:
        return self.table[rows].flatten(-2).float()                            # [T, E]

    def mix(self, h, e, seg_start=None, conv_state=None):
        """h [T, G, H], e [T, E] -> (update [T, G, H], conv inputs [T, G*H]). ``conv_state`` [(k-1)*dil, G*H]: the
        conv inputs before row 0 (incremental decoding)."""
        G, H = self.G, self.H
        T = h.shape[0]
        k = _group_rms(e @ self.key_proj.float().t(), self.norm_key, G, self.eps).view(T, G, H)
        q = _group_rms(h.reshape(T, G * H), self.norm_query, G, self.eps).view(T, G, H)
        g = (k * q).sum(-1, keepdim=True) / math.sqrt(H)
        g = g.abs().clamp_min(1e-6).sqrt() * g.sign()
        v = torch.sigmoid(g) * (e @ self.value_proj.float().t())[:, None, :]    # [T, G, H]
        c = _group_rms(v.reshape(T, G * H), self.norm_conv, G, self.eps)        # [T, G*H]
        return v + causal_conv(c, self.conv.float(), self.dil, seg_start, conv_state).view(T, G, H), c

    def forward(self, h, tokens, seg_start=None):
        """One sequence or packed row: h [T, G, H], tokens [T] -> update [T, G, H]."""
        return self.mix(h, self.embed(self.hash.ids(tokens, seg_start)), seg_start)[0]


def causal_conv(x: torch.Tensor, w: torch.Tensor, dil: int = 1, seg_start=None, state=None) -> torch.Tensor:
    """Depthwise causal conv over rows: out[t] = sum_j w[:, j] * x[t - (k-1-j) dil]. Rows before a row's segment
    start read zero; before row 0 they read ``state`` [(k-1) dil, C] when given (incremental decoding), else zero."""
    T, C = x.shape
    k = w.shape[1]
    pad = (k - 1) * dil
    prev = state.float() if state is not None else torch.zeros(pad, C, dtype=torch.float32, device=x.device)
    ext = torch.cat([prev, x.float()])
    pos = torch.arange(T, device=x.device)
    out = torch.zeros(T, C, dtype=torch.float32, device=x.device)
    for j in range(k):
        back = (k - 1 - j) * dil
        src = ext[pos + pad - back]
        if seg_start is not None:
            src = torch.where((pos - back >= seg_start.long())[:, None], src, torch.zeros_like(src))
        out += src * w[:, j].float()
    return out


# ---------------------------------------------------------------------------------------------- hot-table tools
def bucket_counts(hash_: NgramHash, sequences, head: int) -> np.ndarray:
    """Lookups per bucket of one head over token sequences (each sequence hashed on its own)."""
    counts = np.zeros(hash_.moduli[head], dtype=np.int64)
    for toks in sequences:
        ids = hash_.ids(torch.as_tensor(toks))[:, head] - hash_.offsets[head]
        counts += np.bincount(ids.numpy(), minlength=hash_.moduli[head])
    return counts


def build_hot(hash_: NgramHash, sequences, fracs: dict[int, float]) -> dict[int, np.ndarray]:
    """Per head, the sorted bucket indices of the most used ``frac`` of that head's table (``fracs``: n-gram order ->
    fraction). Raises when the corpus touches fewer buckets than asked for (padding with cold buckets wastes rows)."""
    hot = {}
    for h in range(len(hash_.moduli)):
        frac = fracs[2 + h // hash_.hpn]
        cnt = bucket_counts(hash_, sequences, h)
        keep = int(hash_.moduli[h] * frac)
        nz = int((cnt > 0).sum())
        if keep > nz:
            raise ValueError(f"head {h}: asked for {keep} buckets, the corpus touches {nz}")
        hot[h] = np.sort(np.argpartition(cnt, -keep)[-keep:]).astype(np.int64) if keep else np.zeros(0, np.int64)
    return hot


def hot_rows(hash_: NgramHash, hot: dict[int, np.ndarray], ids: torch.Tensor) -> torch.Tensor:
    """Full-table row ids [T, heads] -> rows of the compact hot table (heads concatenated in order), -1 for a miss
    (the lookup reads zeros there)."""
    out = torch.full_like(ids, -1)
    base = 0
    for h in range(ids.shape[1]):
        b = torch.as_tensor(hot[h])
        local = ids[:, h] - hash_.offsets[h]
        j = torch.searchsorted(b, local).clamp_max(max(len(b) - 1, 0))
        hit = (b[j] == local) if len(b) else torch.zeros_like(local, dtype=torch.bool)
        out[:, h] = torch.where(hit, j + base, torch.full_like(j, -1))
        base += len(b)
    return out
