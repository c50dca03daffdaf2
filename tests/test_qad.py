"""QAD student, fused loss and optimizer on CPU (oracle paths) against the reference model and plain autograd."""
import pytest
import torch

from arc_forge_2026_b200.config import preset
from arc_forge_2026_b200.models.reference import build_reference
from arc_forge_2026_b200.quant.gptq import rtn_quantize
from arc_forge_2026_b200.train.kl import teacher_topk
from arc_forge_2026_b200.train.losses import fused_topk_tail_kl
from arc_forge_2026_b200.train.optim import AdamWBF16
from arc_forge_2026_b200.train.student import QADStudent


def _student():
    cfg = preset("tiny_cpu")
    ref = build_reference(cfg, seed=0)
    cs = []
    with torch.no_grad():
        for moe in ref.moe_layers():  # the reference gets the dequantised INT3 experts: only FP8 QAT differs
            c13, s13 = rtn_quantize(moe.w13.float())
            c2, s2 = rtn_quantize(moe.w2.float())
            s13, s2 = s13.bfloat16().float(), s2.bfloat16().float()
            moe.w13.copy_((c13.float() - 4) * s13.repeat_interleave(128, -1))
            moe.w2.copy_((c2.float() - 4) * s2.repeat_interleave(128, -1))
            cs.append((c13, s13, c2, s2))
    return cfg, ref, QADStudent(cfg, ref, cs, compute_dtype=torch.float32)


def test_student_forward_close_to_reference_and_trains():
    cfg, ref, st = _student()
    ids = torch.randint(0, cfg.vocab_size, (2, 40), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        h_ref = ref.hidden(ids)
        h = st.hidden(ids)
    # same INT3 experts; the block-FP8 QAT of the dense projections is the main difference (e4m3 keeps 3 mantissa
    # bits: ~3% without it, ~13% with it through 4 random-init layers)
    rel = ((h.float() - h_ref.float()).norm() / h_ref.float().norm()).item()
    assert rel < 0.2, rel
    # distillation against the reference teacher's top-8 targets decreases the loss
    with torch.no_grad():  # a sharper teacher than the student, so there is something to learn
        zt = 3.0 * ref(ids).reshape(-1, cfg.vocab_size)
    t_ids, t_lp, t_tail = teacher_topk(zt, 8)
    groups = st.param_groups()
    opt = AdamWBF16([{"params": groups[k], "lr": 1e-4} for k in groups])
    losses = []
    for _ in range(6):
        opt.zero_grad()
        h = st.hidden(ids).reshape(-1, cfg.hidden_size)
        loss = fused_topk_tail_kl(h, st.lm_head, st.lm_head_t, t_ids, t_lp, t_tail, "reverse") / h.shape[0]
        loss.backward()
        assert st.layers[0].moe.w13_scales.grad is not None
        assert st.layers[3].q_proj.grad is not None
        opt.step()
        losses.append(float(loss.detach()))
    assert losses[-1] < losses[0]


def test_gradient_accumulation_matches_one_batch():
    """Two accumulated micro-batches give the gradients of one batch holding both (mean over all positions)."""
    from arc_forge_2026_b200.config import QADConfig
    from arc_forge_2026_b200.train.qad import build_optimizer, enforce_scale_invariants, train_step
    grads = []
    for split in (False, True):
        cfg, ref, st = _student()
        qc = QADConfig(seq_len=24, topk=8, direction="forward")
        ids = torch.randint(0, cfg.vocab_size, (2, 24), generator=torch.Generator().manual_seed(1))
        with torch.no_grad():
            zt = 3.0 * ref(ids).reshape(-1, cfg.vocab_size)
        t_ids, t_lp, t_tail = teacher_topk(zt, 8)
        opt = build_optimizer(st, qc)
        signs = enforce_scale_invariants(st, None)
        if split:
            n = ids.shape[1]
            for i in range(2):
                tg = {"ids": t_ids[i * n:(i + 1) * n], "lp": t_lp[i * n:(i + 1) * n], "tail": t_tail[i * n:(i + 1) * n]}
                train_step(st, opt, ids[i:i + 1], tg, qc, signs, accumulate=True, micro_batches=2, first=i == 0)
        else:
            opt.zero_grad()
            n = ids.numel()
            h = st.hidden(ids).reshape(n, -1)
            (fused_topk_tail_kl(h, st.lm_head, st.lm_head_t, t_ids, t_lp, t_tail, "forward") / n).backward()
        grads.append([p.grad.clone() for grp in opt.param_groups for p in grp["params"]])
    # the STE weight gradients of the INT3-scale and FP8-QAT paths are rounded to bf16 once per micro-batch
    # (0.2% apart); every other gradient agrees to fp32 summation order
    for a, b in zip(*grads):
        assert ((a - b).norm() / b.norm().clamp_min(1e-30)).item() < 5e-3


def test_kernel_registry_counts_and_rejects_fallbacks():
    from arc_forge_2026_b200.train import kernels
    old = {n for n in kernels.NAMES if kernels.enabled(n)}
    try:
        everything = kernels.enable("all")
        assert "grouped_gemm" in kernels.OPT_IN and not everything & kernels.OPT_IN and "gdn_chunk" in everything
        assert "grouped_gemm" in kernels.enable("gdn_chunk,grouped_gemm")  # opt-in kernels run when named
        assert kernels.enable("rms_norm,swiglu") == {"rms_norm", "swiglu"}
        assert kernels.use("rms_norm") and not kernels.use("gdn_chunk")
        kernels.reset()
        kernels.hit("rms_norm", True)
        kernels.hit("rms_norm", True)
        kernels.hit("gdn_chunk", False)  # disabled: a fallback there is allowed
        assert kernels.assert_step_calls({"rms_norm": 2})["native"]["rms_norm"] == 2
        kernels.hit("swiglu", False)
        with pytest.raises(RuntimeError, match="swiglu"):
            kernels.assert_step_calls()
        with pytest.raises(RuntimeError, match="expected 3"):
            kernels.assert_step_calls({"rms_norm": 3}, no_fallback=False)
        with pytest.raises(ValueError):
            kernels.enable("not_a_kernel")
        assert kernels.enable("none") == set()
    finally:
        kernels.enable(sorted(old))


def test_hyper_connection_student_matches_reference():
    """A student of an HC model (4 branches) follows the reference model and takes gradients through the
    frozen hyper-connection reads and write-backs."""
    cfg = preset("tiny_cpu", hc_count=4, hc_lowrank=32)
    ref = build_reference(cfg, seed=1)
    cs = []
    with torch.no_grad():
        for moe in ref.moe_layers():
            c13, s13 = rtn_quantize(moe.w13.float())
            c2, s2 = rtn_quantize(moe.w2.float())
            s13, s2 = s13.bfloat16().float(), s2.bfloat16().float()
            moe.w13.copy_((c13.float() - 4) * s13.repeat_interleave(128, -1))
            moe.w2.copy_((c2.float() - 4) * s2.repeat_interleave(128, -1))
            cs.append((c13, s13, c2, s2))
    st = QADStudent(cfg, ref, cs, compute_dtype=torch.float32, checkpoint_layers=False)
    ids = torch.randint(0, cfg.vocab_size, (1, 30), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        h_ref, h = ref.hidden(ids), st.hidden(ids)
    rel = ((h - h_ref).norm() / h_ref.norm()).item()
    assert rel < 0.2, rel
    h = st.hidden(ids)
    h.pow(2).mean().backward()
    assert st.layers[0].moe.w13_scales.grad is not None
    assert all(not p.requires_grad for p in st.layers[0].hc_attn.parameters())
