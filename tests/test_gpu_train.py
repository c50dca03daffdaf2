"""GPU numerics of the QAD training kernels against their fp32 PyTorch oracles, and a tiny GPU training run."""
import pytest
import torch

from arc_forge_2026_b200.ops import C, check_status
from arc_forge_2026_b200.quant import fp8 as fp8q
from arc_forge_2026_b200.quant.int3_tiles import codes_to_tiles
from arc_forge_2026_b200.train.fakequant import FP8BlockSTE, Int3ScaleSTE
from arc_forge_2026_b200.train.kl import teacher_topk, topk_tail_kl

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def test_int3_dequant_and_scale_grad():
    g = torch.Generator().manual_seed(0)
    codes = torch.randint(0, 8, (3, 256, 384), generator=g, dtype=torch.uint8)
    tiles = codes_to_tiles(codes)
    scales = torch.randn(3, 256, 3, generator=g) * 0.01
    w_cpu = Int3ScaleSTE.apply(scales, tiles)
    w_gpu = Int3ScaleSTE.apply(scales.to(dev), tiles.to(dev))
    assert torch.equal(w_gpu.cpu(), w_cpu)
    dW = torch.randn(3, 256, 384, generator=g).bfloat16()
    s_cpu = scales.clone().requires_grad_(True)
    Int3ScaleSTE.apply(s_cpu, tiles).backward(dW)
    s_gpu = scales.to(dev).requires_grad_(True)
    Int3ScaleSTE.apply(s_gpu, tiles.to(dev)).backward(dW.to(dev))
    torch.testing.assert_close(s_gpu.grad.cpu(), s_cpu.grad, rtol=1e-5, atol=1e-4)


def test_fp8_block_fakequant():
    g = torch.Generator().manual_seed(1)
    w = torch.randn(300, 520, generator=g) * 0.05
    ref = FP8BlockSTE.apply(w)
    got = FP8BlockSTE.apply(w.to(dev)).cpu()
    assert _rel(got, ref) < 2e-3  # the two sides may round a handful of values at ties differently
    _, s = fp8q.quantize_weight_block(w.bfloat16().float())
    sinv = torch.empty(3, 5, device=dev)
    out = torch.empty(300, 520, dtype=torch.bfloat16, device=dev)
    C().fp8_block_fakequant(w.to(dev), out, sinv)
    torch.testing.assert_close(sinv.cpu(), s, rtol=1e-6, atol=0)


@pytest.mark.parametrize("reverse", [False, True])
def test_topk_tail_kl_kernel(reverse):
    g = torch.Generator().manual_seed(2)
    N, V, k = 37, 5000, 64
    zt = torch.randn(N, V, generator=g) * 2
    ids, lp, tail = teacher_topk(zt, k)
    zs = torch.randn(N, V, generator=g) * 2
    loss_ref, dz_ref = topk_tail_kl(zs, ids, lp, tail, "reverse" if reverse else "forward")
    loss = torch.empty(N, device=dev)
    dz = torch.empty(N, V, dtype=torch.bfloat16, device=dev)
    C().topk_tail_kl(zs.to(dev), ids.to(dev), lp.to(dev), tail.to(dev), reverse, 1.0, loss, dz)
    torch.cuda.synchronize()
    torch.testing.assert_close(loss.cpu(), loss_ref, rtol=2e-3, atol=1e-4)
    assert _rel(dz.cpu(), dz_ref) < 1e-2


def test_adamw_kernel():
    g = torch.Generator().manual_seed(3)
    p = torch.randn(10000, generator=g)
    grad = torch.randn(10000, generator=g)
    m = torch.zeros(10000, dtype=torch.bfloat16)
    v = torch.zeros(10000, dtype=torch.bfloat16)
    pg, mg, vg = p.to(dev), m.to(dev), v.to(dev)
    for step in (1, 2, 3):
        C().adamw(pg, grad.to(dev), mg, vg, None, 1e-3, 0.9, 0.95, 1e-8, 0.01, step)
        mm = 0.9 * m.float() + 0.1 * grad
        vv = 0.95 * v.float() + 0.05 * grad * grad
        m.copy_(mm)
        v.copy_(vv)
        p -= 1e-3 * (0.01 * p + (mm / (1 - 0.9**step)) / ((vv / (1 - 0.95**step)).sqrt() + 1e-8))
    torch.testing.assert_close(pg.cpu(), p, rtol=1e-4, atol=1e-5)


def test_tiny_qad_training_on_gpu():
    from arc_forge_2026_b200.config import QADConfig, preset
    from arc_forge_2026_b200.formats.topk_targets import synthetic_targets
    from arc_forge_2026_b200.train.qad import build_optimizer, enforce_scale_invariants, train_step
    from arc_forge_2026_b200.train.student import random_student
    cfg = preset("tiny_gpu")
    st = random_student(cfg, dev, seed=0)
    qc = QADConfig(seq_len=256, topk=16, direction="reverse", lr_scale=1e-3, lr_router=1e-3, lr_dense=1e-3)
    opt = build_optimizer(st, qc, sharded=True)
    signs = enforce_scale_invariants(st, None)
    gen = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (2, 256), generator=gen).to(dev)
    t = synthetic_targets(ids.numel(), 16, cfg.vocab_size, gen, dev)
    losses = [train_step(st, opt, ids, t, qc, signs)[0] for _ in range(5)]
    torch.cuda.synchronize()
    check_status()
    assert losses[-1] < losses[0], losses


def test_gdn_chunk_scan_kernel_matches_cpu_scan():
    """fp32 SIMT kernel to 1e-5; the tensor-core kernel (bf16 operands, fp32 accumulation) to 2e-2."""
    from arc_forge_2026_b200.train.gdn_chunk import _scan
    g = torch.Generator().manual_seed(11)
    BH, n, Cc, Dk, Dv = 3, 5, 64, 128, 128
    m1 = torch.randn(BH, n, Cc, Dk, generator=g) * 0.05
    m2 = torch.randn(BH, n, Cc, Dk, generator=g) * 0.05
    y = torch.randn(BH, n, Cc, Dv, generator=g)
    qm = torch.randn(BH, n, Dk, Dv, generator=g)
    last = -torch.rand(BH, n, generator=g) * 3
    init = torch.randn(BH, Dk, Dv, generator=g)
    for reverse, q in ((False, None), (True, qm)):
        ref = _scan(m1, m2, y, q, last, init, reverse)
        for precise, tol in ((True, 1e-5), (False, 2e-2)):
            got = _scan(m1.to(dev), m2.to(dev), y.to(dev), None if q is None else q.to(dev), last.to(dev),
                        init.to(dev), reverse, precise=precise)
            for a, b in zip(got, ref):
                assert _rel(a.cpu(), b) < tol, (reverse, precise, _rel(a.cpu(), b))
    check_status()


def test_chunked_gdn_gradients_on_gpu_match_unrolled_loop():
    from arc_forge_2026_b200.train.gdn_chunk import chunk_gated_delta_rule, chunk_gated_delta_rule_loop
    g = torch.Generator().manual_seed(12)
    B, T, H, Dk, Dv = 1, 300, 4, 128, 128
    q = torch.nn.functional.normalize(torch.randn(B, T, H, Dk, generator=g), dim=-1) * Dk ** -0.5
    k = torch.nn.functional.normalize(torch.randn(B, T, H, Dk, generator=g), dim=-1)
    v = torch.randn(B, T, H, Dv, generator=g)
    gate = -torch.rand(B, T, H, generator=g) * 0.3
    beta = torch.rand(B, T, H, generator=g)
    dout = torch.randn(B, T, H, Dv, generator=g)

    def run(fn, **kw):
        ins = [t.to(dev).requires_grad_(True) for t in (q, k, v, gate, beta)]
        o, _ = fn(*ins, **kw)
        (o * dout.to(dev)).sum().backward()
        return [o.detach()] + [t.grad for t in ins]
    ref = run(chunk_gated_delta_rule_loop)
    for precise, tol in ((True, 1e-4), (False, 3e-2)):
        for a, b in zip(run(chunk_gated_delta_rule, precise=precise), ref):
            assert _rel(a, b) < tol, (precise, _rel(a, b))


def test_native_chunked_gdn_matches_fp32_oracle():
    """The native chunk kernels (grouped values, T not a multiple of 64, B > 1, a final-state gradient) against the
    fp32 recurrence on the same bf16-rounded inputs: outputs and every input gradient."""
    from arc_forge_2026_b200.train.gdn_chunk import chunk_gated_delta_rule, chunk_gated_delta_rule_loop
    g = torch.Generator().manual_seed(13)
    B, T, Hk, Hv, D = 2, 200, 2, 4, 128
    rep = Hv // Hk
    q = (torch.nn.functional.normalize(torch.randn(B, T, Hk, D, generator=g), dim=-1) * D ** -0.5).bfloat16().float()
    k = torch.nn.functional.normalize(torch.randn(B, T, Hk, D, generator=g), dim=-1).bfloat16().float()
    v = torch.randn(B, T, Hv, D, generator=g).bfloat16().float()
    gate = -torch.rand(B, T, Hv, generator=g) * 0.3
    beta = torch.rand(B, T, Hv, generator=g)
    dout = torch.randn(B, T, Hv, D, generator=g)
    dS = torch.randn(B, Hv, D, D, generator=g) * 0.1

    def run(native):
        ins = [t.to(dev).requires_grad_(True) for t in (q, k, v, gate, beta)]
        if native:
            o, S = chunk_gated_delta_rule(ins[0].bfloat16(), ins[1].bfloat16(), ins[2].bfloat16(), ins[3], ins[4])
        else:
            o, S = chunk_gated_delta_rule_loop(ins[0].repeat_interleave(rep, 2), ins[1].repeat_interleave(rep, 2),
                                               ins[2], ins[3], ins[4])
        ((o.float() * dout.to(dev)).sum() + (S.float() * dS.to(dev)).sum()).backward()
        return [o.detach().float(), S.detach().float()] + [t.grad.float() for t in ins]
    got, ref = run(True), run(False)
    torch.cuda.synchronize()
    check_status()
    names = ["o", "state", "dq", "dk", "dv", "dg", "dbeta"]
    errs = {n: round(_rel(a, b), 5) for n, a, b in zip(names, got, ref)}
    assert all(e < 3e-2 for e in errs.values()), errs


def test_fused_training_ops_match_torch():
    """conv+SiLU (strided input), RMSNorm (H 2048 and a strided H 256 view), gated RMSNorm (H 128, strided z),
    SwiGLU, MoE combine and dispatch: outputs and input gradients against the plain-torch math."""
    from arc_forge_2026_b200.models import reference as R
    from arc_forge_2026_b200.train import fused
    g = torch.Generator().manual_seed(21)

    def grads(fn, *ts):
        ins = [t.detach().clone().requires_grad_(t.is_floating_point() and t.dtype != torch.float32 or
                                                 getattr(t, "_want_grad", False)) for t in ts]
        out = fn(*ins)
        dout = torch.randn(out.shape, generator=torch.Generator().manual_seed(99)).to(dev).to(out.dtype)
        (out.float() * dout.float()).sum().backward()
        return [out.detach().float()] + [i.grad.float() for i in ins if i.grad is not None]

    def check(name, fast, ref, *ts, tol=2e-2):
        a, b = grads(fast, *ts), grads(ref, *ts)
        assert len(a) == len(b), name
        for i, (x, y) in enumerate(zip(a, b)):
            assert _rel(x, y) < tol, (name, i, _rel(x, y))

    B, T, C = 2, 150, 256
    base = torch.randn(B, T, C + 64, generator=g).bfloat16().to(dev)
    w4 = (torch.randn(C, 4, generator=g) * 0.3).to(dev)
    check("conv", lambda x: fused.conv_silu(x[..., :C], w4), lambda x: R.causal_conv1d(x[..., :C], w4)[0], base)
    x = torch.randn(B, T, 2048, generator=g).bfloat16().to(dev)
    wn = (torch.randn(2048, generator=g) * 0.1).to(dev)
    check("rms2048", lambda x: fused.rms_norm(x, wn, 1e-6), lambda x: R.rms_norm(x, wn, 1e-6), x)
    qg = torch.randn(B, T, 4, 512, generator=g).bfloat16().to(dev)
    w256 = (torch.randn(256, generator=g) * 0.1).to(dev)
    check("rms256view", lambda q: fused.rms_norm(q[..., :256], w256, 1e-6),
          lambda q: R.rms_norm(q[..., :256], w256, 1e-6), qg)
    o = torch.randn(B, T, 4, 128, generator=g).bfloat16().to(dev)
    zq = torch.randn(B, T, 64 + 4 * 128, generator=g).bfloat16().to(dev)
    w128 = (1 + torch.randn(128, generator=g) * 0.1).to(dev)
    check("gated128", lambda o, z: fused.gated_rms_norm(o, z[..., 64:].reshape(B, T, 4, 128), w128, 1e-6),
          lambda o, z: R.gated_rms_norm(o, z[..., 64:].reshape(B, T, 4, 128), w128, 1e-6), o, zq)
    gu = torch.randn(300, 1024, generator=g).bfloat16().to(dev)
    check("swiglu", fused.swiglu, lambda t: torch.nn.functional.silu(t[:, :512].float()).bfloat16() * t[:, 512:], gu)
    Tk, K, H = 97, 10, 2048
    y = torch.randn(Tk * K, H, generator=g).bfloat16().to(dev)
    inv = torch.randperm(Tk * K, generator=g).to(dev)
    wt = torch.rand(Tk, K, generator=g).to(dev)
    wt._want_grad = True

    def comb_ref(y, w):
        return (y.index_select(0, inv).view(Tk, K, H) * w.to(y.dtype)[..., None]).sum(1)
    check("combine", lambda y, w: fused.moe_combine(y, inv, w), comb_ref, y, wt)
    xt = torch.randn(Tk, H, generator=g).bfloat16().to(dev)
    order = torch.argsort(inv)
    check("dispatch", lambda x: fused.moe_dispatch(x, order, inv, K),
          lambda x: x.index_select(0, torch.div(order, K, rounding_mode="floor")), xt)
    check_status()


def test_packed_gdn_and_conv_on_gpu_match_fp32_paths():
    """Chunk resets (packed sequences) in the native GDN kernels and the positioned conv: outputs and gradients
    against the fp32 torch path / the plain-torch conv."""
    from arc_forge_2026_b200.train.fused import conv_silu, conv_silu_reference
    from arc_forge_2026_b200.train.gdn_chunk import chunk_gated_delta_rule
    g = torch.Generator().manual_seed(14)
    T, Hk, Hv, D = 320, 2, 4, 128
    reset = torch.tensor([1, 0, 1, 1, 0], dtype=torch.int32)
    q = (torch.nn.functional.normalize(torch.randn(1, T, Hk, D, generator=g), dim=-1) * D ** -0.5).bfloat16().float()
    k = torch.nn.functional.normalize(torch.randn(1, T, Hk, D, generator=g), dim=-1).bfloat16().float()
    v = torch.randn(1, T, Hv, D, generator=g).bfloat16().float()
    gate = -torch.rand(1, T, Hv, generator=g) * 0.3
    beta = torch.rand(1, T, Hv, generator=g)
    dout = torch.randn(1, T, Hv, D, generator=g)

    def run(native):
        ins = [t.to(dev).requires_grad_(True) for t in (q, k, v, gate, beta)]
        a = [ins[0].bfloat16(), ins[1].bfloat16(), ins[2].bfloat16()] if native else ins[:3]
        o, _ = chunk_gated_delta_rule(*a, ins[3], ins[4], precise=not native, chunk_reset=reset.to(dev))
        (o.float() * dout.to(dev)).sum().backward()
        return [o.detach().float()] + [t.grad.float() for t in ins]
    got, ref = run(True), run(False)
    errs = [round(_rel(a, b), 5) for a, b in zip(got, ref)]
    assert all(e < 3e-2 for e in errs), errs
    assert got[1][0, :64].abs().max() > 0  # sanity: the first sequence has gradient
    # positioned conv
    x = torch.randn(1, T, 256 + 64, generator=g).bfloat16().to(dev)
    w4 = (torch.randn(256, 4, generator=g) * 0.3).to(dev)
    pos = torch.cat([torch.arange(128), torch.arange(64), torch.arange(128)]).int()[None].to(dev)
    xa = x.clone().requires_grad_(True)
    xb = x.clone().requires_grad_(True)
    ya = conv_silu(xa[..., :256], w4, pos)
    yb = conv_silu_reference(xb[..., :256], w4, pos)
    dy = torch.randn(ya.shape, generator=g).to(dev).bfloat16()
    (ya.float() * dy.float()).sum().backward()
    (yb.float() * dy.float()).sum().backward()
    assert _rel(ya.float(), yb.float()) < 1e-2 and _rel(xa.grad.float(), xb.grad.float()) < 1e-2
    check_status()


def test_sft_packed_bins_with_checkpoint_offload_on_gpu(tmp_path, capsys):
    """SFT over packed bins on the GPU (native GDN with chunk resets, positioned conv, varlen attention): identical
    losses with the layer checkpoints offloaded to pinned host memory and kept on the device."""
    import json
    import random
    from arc_forge_2026_b200.train import sft
    rng = random.Random(1)
    d = tmp_path / "d.jsonl"
    d.write_text("".join(json.dumps({"ids": [rng.randrange(1, 500) for _ in range(rng.randrange(60, 300))]}) + "\n"
                         for _ in range(8)))
    losses = []
    for extra in ([], ["--offload-checkpoints"]):
        sft.main(["--data", str(d), "--preset", "tiny_gpu", "--max-len", "1024", "--bins-per-step", "2",
                  "--steps", "3", "--lr", "1e-3", "--out", str(tmp_path / ("o" + str(len(extra))))] + extra)
        out = capsys.readouterr().out.splitlines()
        losses.append([json.loads(x)["loss"] for x in out if x.startswith('{"step"')])
    check_status()
    assert losses[0] == losses[1] and len(losses[0]) == 3, losses


def test_hyper_connection_kernels_match_reference():
    """Native hyper-connection read (norm, projections, mix, gate) and write-back against the fp32 reference
    module: outputs and the gradient of the branch stream (weights frozen)."""
    from arc_forge_2026_b200.config import preset
    from arc_forge_2026_b200.models import reference as R
    from arc_forge_2026_b200.train.hc import hc_inject, hc_read
    cfg = preset("tiny_cpu", hc_count=4, hc_lowrank=32, hidden_size=256)
    g = torch.Generator().manual_seed(31)
    mod = R.HyperConnection(cfg).to(dev)
    with torch.no_grad():
        for p in (mod.w_down, mod.w_up, mod.w_inject):
            p.copy_(torch.randn(p.shape, generator=g) * 0.05)
        mod.hc_norm.weight.copy_(torch.randn(mod.hc_norm.weight.shape, generator=g) * 0.1)
    mod.requires_grad_(False)
    h0 = torch.randn(3, 37, 4, 256, generator=g).bfloat16().to(dev)
    dx = torch.randn(3, 37, 256, generator=g).to(dev)
    dg = torch.randn(3, 37, 4, generator=g).to(dev)
    y0 = torch.randn(3, 37, 256, generator=g).bfloat16().to(dev)
    dout = torch.randn(3, 37, 4, 256, generator=g).to(dev)

    def run(native):
        h = h0.clone().requires_grad_(True)
        y = y0.clone().requires_grad_(True)
        x, gate = hc_read(h, mod) if native else mod(h)
        out = hc_inject(h, y, gate) if native else R.hc_inject(h, y, gate)
        ((x.float() * dx).sum() + (gate.float() * dg).sum() + (out.float() * dout).sum()).backward()
        return [x.detach().float(), gate.detach().float(), out.detach().float(), h.grad.float(), y.grad.float()]
    got, ref = run(True), run(False)
    errs = [round(_rel(a, b), 5) for a, b in zip(got, ref)]
    assert all(e < 2e-2 for e in errs), errs
    check_status()


def test_hyper_connection_student_trains_on_native_kernels():
    """A QAD student with 4 hyper-connection branches steps on the GPU with every HC read on the native path."""
    from arc_forge_2026_b200.config import QADConfig, preset
    from arc_forge_2026_b200.formats.topk_targets import synthetic_targets
    from arc_forge_2026_b200.train import kernels
    from arc_forge_2026_b200.train.qad import build_optimizer, enforce_scale_invariants, train_step
    from arc_forge_2026_b200.train.student import random_student
    cfg = preset("tiny_gpu", hc_count=4, hc_lowrank=64)
    st = random_student(cfg, dev, seed=0)
    qc = QADConfig(seq_len=256, topk=16, direction="reverse", lr_scale=1e-3, lr_router=1e-3, lr_dense=1e-3)
    opt = build_optimizer(st, qc, sharded=True)
    signs = enforce_scale_invariants(st, None)
    gen = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (2, 256), generator=gen).to(dev)
    t = synthetic_targets(ids.numel(), 16, cfg.vocab_size, gen, dev)
    kernels.reset()
    losses = [train_step(st, opt, ids, t, qc, signs)[0] for _ in range(4)]
    torch.cuda.synchronize()
    check_status()
    c = kernels.counts()
    assert c["native"].get("hc", 0) >= 4 * (2 * cfg.num_layers + 1) and "hc" not in c["fallback"], c
    assert losses[-1] < losses[0], losses


def test_ple_student_trains_with_the_native_lookup():
    """A QAD student with a PLE layer (and 2 hyper-connection branches) steps on the GPU; the n-gram lookup runs
    on the native kernel."""
    from arc_forge_2026_b200.config import QADConfig, preset
    from arc_forge_2026_b200.formats.topk_targets import synthetic_targets
    from arc_forge_2026_b200.train import kernels
    from arc_forge_2026_b200.train.qad import build_optimizer, enforce_scale_invariants, train_step
    from arc_forge_2026_b200.train.student import random_student
    cfg = preset("tiny_gpu", ple_layer_ids=(1,), ngram_vocab_size_base=4001, ple_embed_dim=256, hc_count=2,
                 hc_lowrank=64)
    st = random_student(cfg, dev, seed=0)
    qc = QADConfig(seq_len=256, topk=16, direction="reverse", lr_scale=1e-3, lr_router=1e-3, lr_dense=1e-3)
    opt = build_optimizer(st, qc, sharded=True)
    signs = enforce_scale_invariants(st, None)
    gen = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (2, 256), generator=gen).to(dev)
    t = synthetic_targets(ids.numel(), 16, cfg.vocab_size, gen, dev)
    kernels.reset()
    losses = [train_step(st, opt, ids, t, qc, signs)[0] for _ in range(4)]
    torch.cuda.synchronize()
    check_status()
    c = kernels.counts()
    assert c["native"].get("ple", 0) >= 4 * 2 and "ple" not in c["fallback"], c
    assert losses[-1] < losses[0], losses


def test_native_fp8_teacher_targets_agree_with_its_prefill():
    from arc_forge_2026_b200.config import ServeConfig, preset
    from arc_forge_2026_b200.models.hybrid import HybridModel
    from arc_forge_2026_b200.serve.engine import SpecEngine
    from arc_forge_2026_b200.train.teacher import NativeTeacher
    cfg = preset("tiny_gpu", expert_format="fp8")
    model = HybridModel.random(cfg, dev, seed=1)
    with torch.no_grad():
        model.lm_head.mul_(20.0)
    ids = torch.randint(0, cfg.vocab_size, (300,), generator=torch.Generator().manual_seed(3))
    t_ids, t_lp, t_tail = NativeTeacher(model, 300).targets(ids, 8)
    torch.cuda.synchronize()
    check_status()
    assert t_ids.shape == (300, 8) and torch.all(t_lp[:, :-1] >= t_lp[:, 1:])
    total = torch.logsumexp(torch.cat([t_lp, t_tail[:, None]], 1), 1)
    assert torch.allclose(total, torch.zeros_like(total), atol=1e-4)  # top-k + tail is the whole distribution
    eng = SpecEngine(model, None, ServeConfig(spec_k=0, accept_mode="greedy"), 1, 400)
    eng.add_session(0, ids.tolist(), 2)
    assert eng.sessions[0].generated[0] == int(t_ids[-1, 0])


@pytest.mark.parametrize("r", [16, 64])
def test_lora_native_products_match_fp32(r):
    """The native LoRA products (bf16 big operand, fp32 small operand as bf16 hi + lo) against fp64 torch: forward
    output and the gradients of x, A and B; T and N not multiples of the tiles."""
    from arc_forge_2026_b200.train import kernels
    from arc_forge_2026_b200.train.lora import LoRAAdapter
    g = torch.Generator().manual_seed(r)
    T, K, N = 3001, 2048, 1000
    ad = LoRAAdapter(K, N, r, 32.0, dev)
    with torch.no_grad():
        ad.B.copy_(torch.randn(N, r, generator=g) * 0.05)
    x = torch.randn(T, K, generator=g).bfloat16().to(dev).requires_grad_(True)
    dy = torch.randn(T, N, generator=g).bfloat16().float().to(dev)
    kernels.reset()
    y = ad(x)
    y.backward(dy)
    assert kernels.counts()["native"].get("lora_grad", 0) == 1
    xd, A, B = x.detach().double(), ad.A.detach().double(), ad.B.detach().double()
    s = xd @ A.t()
    ref_y = (s @ B.t()) * ad.scale
    dyd = dy.double()
    ref_dB = (dyd.t() @ s) * ad.scale
    ds = (dyd @ B) * ad.scale
    ref_dA = ds.t() @ xd
    ref_dx = ds @ A
    for got, ref in ((y, ref_y), (ad.B.grad, ref_dB), (ad.A.grad, ref_dA), (x.grad, ref_dx)):
        assert _rel(got.double(), ref) < (5e-3 if got is x.grad else 1e-4), _rel(got.double(), ref)
    check_status()


def test_grouped_expert_gemm_matches_per_expert_gemms():
    """The grouped tcgen05 GEMM (ROWS for the forward and dX, REDUCE for dW) against one fp32 GEMM per expert, with
    empty experts and segment lengths that are not multiples of the tiles."""
    from arc_forge_2026_b200.train.grouped import GroupedLinear
    g = torch.Generator().manual_seed(21)
    E, K, N = 9, 512, 384
    counts = torch.tensor([0, 5, 200, 1, 0, 130, 64, 63, 300])
    R = int(counts.sum())
    x = torch.randn(R, K, generator=g).bfloat16().to(dev).requires_grad_(True)
    w = (torch.randn(E, N, K, generator=g) * 0.05).bfloat16().to(dev).requires_grad_(True)
    dy = torch.randn(R, N, generator=g).bfloat16().to(dev)
    for _ in range(2):  # twice: the second call reuses the kernel's cached state
        x.grad = w.grad = None
        y = GroupedLinear.apply(x, w, counts.to(dev))
        y.backward(dy)
    torch.cuda.synchronize()
    check_status()
    xs, ws, dys = x.detach().float(), w.detach().float(), dy.float()
    ys, dxs, dws, o = [], [], [], 0
    for e, c in enumerate(counts.tolist()):
        ys.append(xs[o:o + c] @ ws[e].t())
        dxs.append(dys[o:o + c] @ ws[e])
        dws.append(dys[o:o + c].t() @ xs[o:o + c])
        o += c
    assert _rel(y, torch.cat(ys)) < 1e-2
    assert _rel(x.grad, torch.cat(dxs)) < 1e-2
    assert _rel(w.grad, torch.stack(dws)) < 1e-2
    assert w.grad[0].abs().max() == 0 and w.grad[4].abs().max() == 0  # empty experts: zero gradient
