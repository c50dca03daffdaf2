"""DFlash drafter training on CPU: the block objective learns a deterministic continuation; KL to teacher logits
joins the loss."""
import torch

from arc_forge_2026_b200.config import drafter_preset
from arc_forge_2026_b200.train.drafter_train import DrafterTrain


def _data(V=256, T=200, Ht=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.empty(T, dtype=torch.long)
    x[0] = 5
    for t in range(1, T):  # x[t+1] = f(x[t]): learnable from the anchor token alone
        x[t] = (x[t - 1] * 7 + 3) % V
    proj = torch.randn(V, Ht, generator=g)
    return x, proj[x] * 0.5  # stand-in target hidden states


def test_drafter_block_objective_learns():
    cfg = drafter_preset("tiny", num_layers=1, hidden_size=128, num_attention_heads=2, num_kv_heads=1,
                         intermediate_size=256)
    V = 256
    tokens, hidden = _data(V)
    d = DrafterTrain(cfg, hidden.shape[1], V, torch.arange(V))
    opt = torch.optim.Adam(d.parameters(), lr=3e-3)
    g = torch.Generator().manual_seed(1)
    losses = []
    for _ in range(60):
        anchors = torch.randint(1, tokens.shape[0] - cfg.k - 1, (16,), generator=g)
        loss = d.loss(tokens, hidden, anchors)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(loss))
    assert losses[-1] < 0.5 * losses[0], (losses[0], losses[-1])
    teacher = torch.randn(tokens.shape[0], V)
    mixed = d.loss(tokens, hidden, torch.tensor([10, 40]), teacher_logits=teacher, kl_weight=0.5)
    assert torch.isfinite(mixed) and float(mixed) > float(d.loss(tokens, hidden, torch.tensor([10, 40])))


# ---------------------------------------------------------------------------------------------------- objectives
from arc_forge_2026_b200.train.drafter_objective import (CandidateSelector, Objective, acceptance_terms,  # noqa: E402
                                                         combine, dpace_weights, importance_terms, opd_terms)


def test_dpace_weights_by_hand():
    p = torch.tensor([[1.0, 0.5, 0.0]])
    w = dpace_weights(p, torch.ones_like(p, dtype=torch.bool), alpha=0.5)
    # s = [1, .75, .5] -> reach = [1, .75, .375] -> reverse sums
    assert torch.allclose(w, torch.tensor([[2.125, 1.125, 0.375]]))
    p2 = torch.tensor([[0.5, 0.9, 0.5]])
    w2 = dpace_weights(p2, torch.tensor([[True, False, True]]), alpha=0.5)
    # s = [.75, 1, .75] -> reach = [.75, 0, .5625]
    assert torch.allclose(w2, torch.tensor([[1.3125, 0.5625, 0.5625]]))


def _sel_setup(A=3, M=4, V=16, H=8, k=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    sel = CandidateSelector(V, H, k, 4, generator=g)
    logits = torch.randn(A, M, V, generator=g, requires_grad=True)
    hidden = torch.randn(A, M, H, generator=g, requires_grad=True)
    labels = torch.randint(0, V, (A, M), generator=g)
    pred = torch.randint(-1, V, (A, M), generator=g)
    return sel, logits, hidden, labels, pred


def test_acceptance_terms_vanish_when_the_drafter_is_the_teacher():
    """All candidates (k = V), an untrained selector (scores = unary): q = r = p, so every slot is accepted with
    probability 1 (WTV loss 0) and the coverage KL is 0."""
    sel, logits, hidden, labels, pred = _sel_setup()
    t = acceptance_terms(logits, labels, pred, hidden, sel, logits.detach().clone(), temperature=0.7, joint=True)
    assert float(t["accept_num"]) < 1e-5 and float(t["cov_num"]) < 1e-5
    assert torch.allclose(t["survival_position"], torch.full((4,), 3.0), atol=1e-5)


def test_acceptance_terms_bounds_and_gradients():
    sel, logits, hidden, labels, pred = _sel_setup(seed=3)
    labels[0, 2] = -1  # a slot outside the supervised run: accepted, no gradient
    teacher = torch.randn(3, 4, 16) * 3
    t = acceptance_terms(logits, labels, pred, hidden, sel, teacher, temperature=1.0, joint=True)
    assert 0.0 <= float(t["accept_num"]) <= 3.0 and float(t["cov_num"]) > 0
    assert int(t["positions"]) == 11
    loss = combine(Objective("acceptance", cov_weight=0.5, joint=True), t)
    loss.backward()
    assert logits.grad is not None and hidden.grad is not None and sel.proj.grad is not None
    # without joint the acceptance term does not reach the backbone's hidden states
    sel2, logits2, hidden2, labels2, pred2 = _sel_setup(seed=3)
    t2 = acceptance_terms(logits2, labels2, pred2, hidden2, sel2, teacher, temperature=1.0, joint=False)
    combine(Objective("acceptance", cov_weight=0.0, accept_weight=1.0), t2).backward()
    assert hidden2.grad is None or float(hidden2.grad.abs().sum()) == 0.0


def test_opd_reached_slots_and_importance_at_a_fresh_replay():
    sel, logits, hidden, _, _ = _sel_setup(A=3, M=4, seed=5)
    g = torch.Generator().manual_seed(9)
    teacher = torch.randn(3, 4, 16, generator=g)
    with torch.no_grad():
        cand = logits.topk(16, -1).indices
    drafted = cand[..., 0]
    accepted = torch.tensor([0, 2, 4])
    anchor = torch.tensor([1, -1, 7])
    t = opd_terms(logits, drafted, anchor, hidden, sel, teacher, accepted, temperature=1.0, joint=True)
    assert int(t["reach_den"]) == 1 + 3 + 4  # every accepted draft and the first rejection
    assert t["reached_position"].tolist() == [3, 2, 2, 1]
    # sampler = this drafter: the importance weights are min(1, p / q) of the drafted tokens
    pred = torch.cat((anchor[:, None], drafted[:, :-1]), 1)
    with torch.no_grad():
        scores = sel(cand, logits.topk(16, -1).values, hidden, pred)
        q = scores.softmax(-1)
        q_d = (q * (cand == drafted[..., None])).sum(-1)
    t2 = opd_terms(logits, drafted, anchor, hidden, sel, teacher, accepted, 1.0, True, sampler_q=q_d,
                   sampler_cand=cand)
    p = teacher.softmax(-1)
    p_d = p.gather(-1, drafted[..., None]).squeeze(-1)
    a = torch.minimum(p.gather(-1, cand), q).sum(-1)
    w = torch.minimum(p_d, q_d) / q_d
    before = torch.cat((torch.ones(3, 1), w[:, :-1].cumprod(-1)), 1)
    assert torch.allclose(t2["is_num"], (a * before).sum(), atol=1e-5)
    with __import__("pytest").raises(ValueError):
        importance_terms(a, q_d, p_d, torch.zeros_like(q_d), cand, q, cand)


def test_drafter_trains_with_the_acceptance_objective_and_proposes_through_the_selector():
    """A drafter with a candidate selector learns the deterministic continuation under the acceptance objective
    (teacher = one-hot-ish target logits): the WTV loss falls and the greedy proposal chain becomes the data."""
    cfg = drafter_preset("tiny", num_layers=1, hidden_size=96, num_attention_heads=2, num_kv_heads=1,
                         intermediate_size=192, selector_top_k=8, selector_rank=16)
    V = 128
    tokens, hidden = _data(V, T=160, Ht=48)
    teacher = torch.full((tokens.shape[0], V), -4.0)
    teacher[torch.arange(tokens.shape[0] - 1), tokens[1:]] = 6.0  # the target predicts the data token
    d = DrafterTrain(cfg, hidden.shape[1], V, torch.arange(V))
    obj = Objective("acceptance", temperature=1.0, cov_weight=1.0, joint=True)
    opt = torch.optim.Adam(d.parameters(), lr=3e-3)
    g = torch.Generator().manual_seed(2)
    first = last = None
    for it in range(80):
        anchors = torch.randint(1, tokens.shape[0] - cfg.k - 1, (16,), generator=g)
        terms = d.objective_terms(tokens, hidden, anchors, obj, teacher)
        loss = combine(obj, terms)
        opt.zero_grad()
        loss.backward()
        opt.step()
        wtv = float(terms["accept_num"] / terms["blocks"])
        first = wtv if first is None else first
        last = wtv
    assert last < 0.5 * first, (first, last)
    an = torch.tensor([20, 60, 100])
    prop = d.propose_greedy(tokens, hidden, an)
    want = tokens[an[:, None] + 1 + torch.arange(cfg.k)[None]]
    assert (prop == want).float().mean() > 0.9
    dp = d.objective_loss(tokens, hidden, an, Objective("dpace"), teacher)
    assert torch.isfinite(dp)
