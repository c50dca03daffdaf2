"""Drafter training objectives beyond next-token CE: D-PACE-weighted CE with a candidate selector, the
temperature-matched acceptance objective (coverage KL + WTV), and the on-policy (OPD) terms over recorded verify
cycles, with an importance-weighted estimate of the expected accepted length.

Semantics follow the reference's drafter trainer (``training/work/qwen38fn_dflash/objective.py:7-303``: dpace_weights,
objective, acceptance_objective, importance_terms, opd_objective; the knobs of ``train.py:35-70`` ``Objective``; the
selector of ``model.py:612-633``). Everything here is written over the draft vocabulary of this repository's drafter:
``logits`` [A, M, Vd] are the drafter's block logits (slot j of the block at anchor a proposes x[a + j + 1]),
``teacher_logits`` [A, M, Vd] the target's logits at the same positions restricted to the draft vocabulary, and token
ids are draft ids (-1: a token outside the draft vocabulary, which never counts as valid or covered).

Notation per slot (temperature T): the teacher p = softmax(teacher / T); the drafter's unary distribution
r = softmax(U / T); the candidates C = top-k of U; the proposal q = softmax(S / T) over C with S the selector's scores
given the slot's predecessor token. a = sum over v in C of min(p(v), q(v)) is the probability that rejection sampling
accepts the slot's draft; prod over j <= k of a_j is the probability that the first k + 1 drafts survive.

All term functions return additive sums (numerators, denominators, per-slot vectors) so chunks and ranks can be
summed before normalising; :func:`combine` turns them into the training loss of an :class:`Objective`.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn


class CandidateSelector(nn.Module):
    """Re-ranks the top-k draft candidates of a slot: score(c) = U(c) + < P[pred] * (W h), S[c] >, a rank-r bilinear
    term in the predecessor token (``pred``), the slot's hidden state ``h`` and the candidate. P is indexed by draft
    id with one extra row for a predecessor outside the draft vocabulary; S starts at zero, so an untrained selector
    ranks exactly like the unary logits."""

    def __init__(self, draft_vocab: int, hidden: int, top_k: int, rank: int, device="cpu", generator=None,
                 std: float = 0.02):
        super().__init__()
        if not 1 <= top_k <= draft_vocab or rank < 1:
            raise ValueError(f"selector top_k {top_k} / rank {rank} out of range for {draft_vocab} draft ids")
        self.top_k, self.rank, self.draft_vocab = top_k, rank, draft_vocab
        self.pred_codebook = nn.Parameter(torch.randn(draft_vocab + 1, rank, generator=generator, device=device) * std)
        self.succ_codebook = nn.Parameter(torch.zeros(draft_vocab, rank, device=device))
        self.proj = nn.Parameter(torch.randn(rank, hidden, generator=generator, device=device) * std)

    def pred_rows(self, pred: torch.Tensor) -> torch.Tensor:
        return torch.where(pred >= 0, pred, torch.full_like(pred, self.draft_vocab))

    def forward(self, candidates, unary, hidden, pred):
        """candidates / unary [..., k], hidden [..., H], pred [...] (draft ids, -1 outside) -> scores [..., k]."""
        ctx = self.pred_codebook[self.pred_rows(pred)] * (hidden.float() @ self.proj.t())       # [..., r]
        return unary + torch.einsum("...r,...kr->...k", ctx, self.succ_codebook[candidates])


def dpace_weights(prob: torch.Tensor, valid: torch.Tensor, alpha: float = 0.5) -> torch.Tensor:
    """D-PACE position weights [A, M], detached: with s_j = alpha + (1 - alpha) p_j on a valid slot (p_j the
    drafter's probability of the data token) and 1 elsewhere, slot i weighs sum over j >= i of valid_j prod over
    l <= j of s_l -- the expected number of later slots a draft at i lets the cycle reach."""
    if not 0.0 <= alpha <= 1.0 or prob.shape != valid.shape:
        raise ValueError("D-PACE needs alpha in [0, 1] and one probability per slot")
    s = torch.where(valid, alpha + (1.0 - alpha) * prob.detach(), torch.ones_like(prob))
    reach = torch.cumprod(s, dim=-1) * valid
    return torch.flip(torch.cumsum(torch.flip(reach, (-1,)), -1), (-1,)).detach()


def _slot_tensors(logits, selector, hidden, pred, joint: bool):
    """Candidates, unary logits and selector scores of every slot."""
    unary, cand = logits.topk(selector.top_k, dim=-1)
    h = hidden
    if not joint:
        unary, h = unary.detach(), hidden.detach()
    return cand, unary, selector(cand, unary, h, pred).float()


def dpace_terms(logits, labels, pred, hidden, selector, teacher_logits=None, alpha: float = 0.5):
    """Hard CE of the data token weighted by D-PACE, the selector's CE towards the data token on covered slots, and
    a forward KL to the teacher on the first two slots (all at T = 1). labels / pred [A, M] draft ids."""
    A, M, V = logits.shape
    valid = labels >= 0
    lab = labels.clamp_min(0)
    logits = logits.float()
    ce = F.cross_entropy(logits.reshape(-1, V), lab.reshape(-1), reduction="none").view(A, M)
    w = dpace_weights((-ce).exp(), valid, alpha) * valid
    cand, unary, scores = _slot_tensors(logits.detach(), selector, hidden.detach(), pred, joint=False)
    match = cand == lab[..., None]
    covered = match.any(-1) & valid
    sel_ce = F.cross_entropy(scores.reshape(-1, selector.top_k), match.long().argmax(-1).reshape(-1),
                             reduction="none").view(A, M)
    sel_w = w * covered
    terms = {"ce_num": (ce * w).sum(), "ce_den": w.sum(), "selector_num": (sel_ce * sel_w).sum(),
             "selector_den": sel_w.sum()}
    if teacher_logits is not None:
        early = min(2, M)
        t_logp = teacher_logits[:, :early].float().log_softmax(-1)
        kl = (t_logp.exp() * (t_logp - logits[:, :early].log_softmax(-1))).sum(-1)
        terms["kl_num"] = (kl * valid[:, :early]).sum()
        terms["kl_den"] = valid[:, :early].sum()
    with torch.no_grad():
        chosen = cand.gather(-1, scores.argmax(-1, keepdim=True)).squeeze(-1)
        accept = (chosen == labels) & valid
        run = accept.long().cumprod(-1)
        terms.update(covered=covered.sum(), positions=valid.sum(), selector_correct=(accept & covered).sum(),
                     accept_prefix=run.sum(0), accept_histogram=torch.bincount(run.sum(-1), minlength=M + 1),
                     blocks=torch.tensor(A, device=logits.device))
    return terms


def acceptance_terms(logits, labels, pred, hidden, selector, teacher_logits, temperature: float, joint: bool = False):
    """Coverage KL(p || r) on every valid slot and the WTV acceptance loss 1 - (1/M) sum_k prod_{j<=k} a_j per block
    (a slot past the supervised run counts as accepted and carries no gradient). With ``joint`` the acceptance term's
    gradient reaches the backbone through U on C and the selector's hidden projection."""
    if temperature <= 0:
        raise ValueError("the acceptance objective needs a positive temperature")
    A, M, V = logits.shape
    valid = labels >= 0
    inv = 1.0 / temperature
    logits = logits.float()
    with torch.no_grad():
        t_logp = (teacher_logits.float() * inv).log_softmax(-1)
    p = t_logp.exp()
    coverage = (p * (t_logp - (logits * inv).log_softmax(-1))).sum(-1)
    cand, unary, scores = _slot_tensors(logits, selector, hidden, pred, joint)
    q = (scores * inv).softmax(-1)
    mass = p.gather(-1, cand)
    overlap = torch.where(valid, torch.minimum(mass, q).sum(-1), torch.ones_like(mass[..., 0]))
    survival = overlap.cumprod(-1)
    with torch.no_grad():
        lab = labels.clamp_min(0)
        covered = (cand == lab[..., None]).any(-1) & valid
        chosen = cand.gather(-1, scores.argmax(-1, keepdim=True)).squeeze(-1)
        accept = (chosen == labels) & valid
        run = accept.long().cumprod(-1)
    return {"cov_num": (coverage * valid).sum(), "accept_num": ((1 - survival) * valid).sum() / M,
            "blocks": torch.tensor(A, device=logits.device), "positions": valid.sum(),
            "overlap_position": (overlap.detach() * valid).sum(0),
            "survival_position": (survival.detach() * valid).sum(0),
            "mass_position": (mass.detach().sum(-1) * valid).sum(0), "covered": covered.sum(),
            "selector_correct": (accept & covered).sum(), "accept_prefix": run.sum(0),
            "accept_histogram": torch.bincount(run.sum(-1), minlength=M + 1)}


WEIGHT_DRIFT = 1.2  # importance weights above this mark a drafter that has moved well away from the sampler


def importance_terms(overlap, q_drafted, p_drafted, sampler_q, cand, q, sampler_cand):
    """Expected accepted drafts of THIS drafter on cycles another drafter (the sampler, q^s) rolled out: slot k's
    closed-form acceptance a_k times the importance weights of the drafts before it, w_j = min(p_j, q_j)(y_j) /
    q^s_j(y_j). Unbiased for E[L] wherever q^s covers this drafter's proposal; its gradient flows through a_k and
    q_j(y_j)."""
    if sampler_q.shape != q_drafted.shape or sampler_cand.shape != cand.shape:
        raise ValueError("the sampler's q and candidates must align with the cycles")
    if (sampler_q <= 0).any():
        raise ValueError("a recorded draft with sampler probability <= 0 could not have been drawn")
    w = torch.minimum(p_drafted, q_drafted) / sampler_q
    before = torch.cat((torch.ones_like(w[:, :1]), torch.cumprod(w[:, :-1], -1)), 1)
    est = overlap * before
    with torch.no_grad():
        on_sampler = (q * (cand[..., :, None] == sampler_cand[..., None, :]).any(-1)).sum(-1)
        diag = {"is_survival_position": est.detach().sum(0), "sampler_covered_position": on_sampler.sum(0),
                "is_weight_drifted": (w[:, :-1] > WEIGHT_DRIFT).sum()}
    return {"is_num": est.sum()} | diag


def opd_terms(logits, drafted, anchor_pred, hidden, selector, teacher_logits, accepted, temperature: float,
              joint: bool = False, sampler_q=None, sampler_cand=None):
    """On-policy terms of recorded verify cycles: the drafter at a cycle's anchor judged on the path it proposed.
    drafted [A, M] draft ids it proposed, anchor_pred [A] the anchor token (draft id or -1), teacher_logits
    [A, M, Vd] the target's logits on the proposal prefix (the verify forward's rows), accepted [A] drafts the cycle
    accepted. Slot j's predecessor is the SAMPLED token (the anchor, then drafts 0..j-1).

    reach_num / reach_den: 1 - a_j over the reached slots (every accepted draft and the first rejection);
    wtv_num: the path WTV 1 - (1/M) sum_k prod_{j<=k} a_j over the whole recorded path; cov_num: coverage KL on the
    reached slots; rho_survival_position: the per-path acceptance with rho_j = min(1, p_j(y_j) / q_j(y_j)) (what a
    fresh replay expects). With sampler_q / sampler_cand (the recording drafter's q of each draft and candidates),
    adds :func:`importance_terms`."""
    if (sampler_q is None) != (sampler_cand is None):
        raise ValueError("sampler_q and sampler_cand go together")
    A, M, V = logits.shape
    if drafted.shape != (A, M) or anchor_pred.shape != (A,) or accepted.shape != (A,):
        raise ValueError("drafts [cycles, slots], one anchor token and one accepted count per cycle")
    if ((accepted < 0) | (accepted > M)).any():
        raise ValueError("accepted drafts out of range")
    inv = 1.0 / temperature
    pred = torch.cat((anchor_pred[:, None], drafted[:, :-1]), 1)
    logits = logits.float()
    with torch.no_grad():
        t_logp = (teacher_logits.float() * inv).log_softmax(-1)
    p = t_logp.exp()
    coverage = (p * (t_logp - (logits * inv).log_softmax(-1))).sum(-1)
    cand, unary, scores = _slot_tensors(logits, selector, hidden, pred, joint)
    q = (scores * inv).softmax(-1)
    mass = p.gather(-1, cand)
    overlap = torch.minimum(mass, q).sum(-1)
    survival = overlap.cumprod(-1)
    reached = torch.arange(M, device=logits.device)[None] <= accepted.clamp(max=M - 1)[:, None]
    picked = cand == drafted[..., None]
    q_drafted = (q * picked).sum(-1)
    with torch.no_grad():
        p_drafted = p.gather(-1, drafted.clamp_min(0)[..., None]).squeeze(-1)
        rho = torch.where(q_drafted > 0, (p_drafted / q_drafted.clamp_min(1e-30)).clamp(max=1.0),
                          torch.zeros_like(q_drafted))
    out = {} if sampler_q is None else importance_terms(overlap, q_drafted, p_drafted, sampler_q, cand, q, sampler_cand)
    return out | {"reach_num": ((1 - overlap) * reached).sum(), "reach_den": reached.sum(),
                  "wtv_num": (1 - survival.sum(-1) / M).sum(), "cov_num": (coverage * reached).sum(),
                  "blocks": torch.tensor(A, device=logits.device),
                  "overlap_position": overlap.detach().sum(0), "reached_position": reached.sum(0),
                  "drafted_candidate_position": picked.any(-1).sum(0),
                  "rho_survival_position": rho.cumprod(-1).sum(0), "accepted_observed": accepted.sum(),
                  "accepted_histogram": torch.bincount(accepted, minlength=M + 1)}


@dataclass(frozen=True)
class Objective:
    """The drafter trainer's objective and its knobs. ``ce``: mean next-token CE (+ kl_weight x KL to the teacher);
    ``dpace``: D-PACE-weighted CE + selector CE + 0.1 x early KL; ``acceptance``: accept_weight x WTV +
    cov_weight x coverage KL at ``temperature`` (``joint``: the WTV gradient reaches the backbone), plus
    opd_weight x an OPD term (``opd_loss`` reached | wtv | importance) over recorded cycles."""
    name: str = "ce"
    temperature: float = 1.0
    cov_weight: float = 0.0
    joint: bool = False
    kl_weight: float = 0.0
    dpace_alpha: float = 0.5
    accept_weight: float = 1.0
    opd_weight: float = 0.0
    opd_loss: str = "reached"

    def __post_init__(self):
        if self.name not in ("ce", "dpace", "acceptance"):
            raise ValueError(f"unknown drafter objective {self.name!r}")
        if self.name == "acceptance" and not (self.temperature > 0 and self.cov_weight >= 0):
            raise ValueError("the acceptance objective needs a positive temperature and a nonnegative coverage weight")
        if self.opd_loss not in ("reached", "wtv", "importance") or self.opd_weight < 0:
            raise ValueError(f"invalid OPD settings: weight {self.opd_weight}, loss {self.opd_loss!r}")
        if self.opd_weight and self.name != "acceptance":
            raise ValueError("OPD trains with the acceptance objective")
        if self.name == "acceptance" and not (self.accept_weight or self.cov_weight or self.opd_weight):
            raise ValueError("every term of the acceptance objective is weighted 0")


def combine(obj: Objective, terms: dict, opd: dict | None = None) -> torch.Tensor:
    """The scalar loss of summed terms (one chunk, or sums over chunks and ranks)."""
    if obj.name == "dpace":
        loss = terms["ce_num"] / terms["ce_den"].clamp_min(1e-9) + \
            terms["selector_num"] / terms["selector_den"].clamp_min(1e-9)
        if "kl_num" in terms:
            loss = loss + 0.1 * terms["kl_num"] / terms["kl_den"].clamp_min(1)
        return loss
    if obj.name != "acceptance":
        raise ValueError("combine() covers the dpace and acceptance objectives")
    loss = obj.accept_weight * terms["accept_num"] / terms["blocks"].clamp_min(1) + \
        obj.cov_weight * terms["cov_num"] / terms["positions"].clamp_min(1)
    if opd is not None and obj.opd_weight:
        if obj.opd_loss == "reached":
            o = opd["reach_num"] / opd["reach_den"].clamp_min(1)
        elif obj.opd_loss == "wtv":
            o = opd["wtv_num"] / opd["blocks"].clamp_min(1)
        else:
            if "is_num" not in opd:
                raise ValueError("the importance OPD loss needs the sampler's record")
            o = -opd["is_num"] / opd["reach_den"].clamp_min(1)
        loss = loss + obj.opd_weight * o
    return loss
