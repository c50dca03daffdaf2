"""Native training attention (csrc/attention_train.cu) against the fp32 varlen causal oracle: forward output and
the q / k / v gradients, GQA, D 128 and 256, ragged packed segments; bitwise reproducible across runs."""
import pytest
import torch

from arc_forge_2026_b200.ops import check_status
from arc_forge_2026_b200.train.attention import varlen_attention, varlen_attention_reference

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("Hq,Hkv,D,lens", [
    (4, 1, 128, [300, 129, 64, 1000]),
    (16, 2, 256, [77, 513, 200]),
    (24, 2, 256, [130, 640]),     # the reference model's heads (GQA 12)
    (8, 8, 128, [1, 63, 65, 128]),
])
def test_forward_and_gradients_match_oracle(Hq, Hkv, D, lens):
    g = torch.Generator().manual_seed(Hq + D)
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    q = torch.randn(T, Hq, D, generator=g).bfloat16().to(dev).requires_grad_()
    k = torch.randn(T, Hkv, D, generator=g).bfloat16().to(dev).requires_grad_()
    v = torch.randn(T, Hkv, D, generator=g).bfloat16().to(dev).requires_grad_()
    do = torch.randn(T, Hq, D, generator=g).bfloat16().to(dev)
    out = varlen_attention(q, k, v, cu)
    out.backward(do)
    torch.cuda.synchronize()
    check_status()
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    ref = varlen_attention_reference(qf, kf, vf, cu)
    ref.backward(do.float())
    assert _rel(out, ref) < 1e-2
    assert _rel(q.grad, qf.grad) < 2e-2
    assert _rel(k.grad, kf.grad) < 2e-2
    assert _rel(v.grad, vf.grad) < 2e-2
    # bitwise reproducible: one owner per output element, fixed order
    grads = [t.grad.clone() for t in (q, k, v)]
    for t in (q, k, v):
        t.grad = None
    out2 = varlen_attention(q, k, v, cu)
    out2.backward(do)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    for a, t in zip(grads, (q, k, v)):
        assert torch.equal(a, t.grad)


@pytest.mark.parametrize("D,lens", [(128, [300, 129, 64, 1000]), (256, [77, 513])])
def test_bidirectional_forward_matches_oracle(D, lens):
    """The forward's bidirectional mode (every key of the segment, e.g. a vision tower's attention within a frame)
    against fp32 softmax attention per segment."""
    from arc_forge_2026_b200.ops import C
    from arc_forge_2026_b200.train.attention import tile_lists
    g = torch.Generator().manual_seed(D)
    T, Hq, Hkv = sum(lens), 8, 2
    cu_host = [0] + torch.tensor(lens).cumsum(0).tolist()
    q = torch.randn(T, Hq, D, generator=g).bfloat16().to(dev)
    k = torch.randn(T, Hkv, D, generator=g).bfloat16().to(dev)
    v = torch.randn(T, Hkv, D, generator=g).bfloat16().to(dev)
    out = torch.empty_like(q)
    lse = torch.empty(Hq, T, dtype=torch.float32, device=dev)
    cu = torch.tensor(cu_host, dtype=torch.int32, device=dev)
    C().attn_train_fwd(q, k, v, cu, tile_lists(cu_host, dev)[0], D ** -0.5, out, lse, None, 64, False)
    torch.cuda.synchronize()
    check_status()
    ref = torch.empty(T, Hq, D, device=dev)
    rep = Hq // Hkv
    for s0, s1 in zip(cu_host[:-1], cu_host[1:]):
        qq = q[s0:s1].float().transpose(0, 1)
        kk = k[s0:s1].float().repeat_interleave(rep, 1).transpose(0, 1)
        vv = v[s0:s1].float().repeat_interleave(rep, 1).transpose(0, 1)
        ref[s0:s1] = ((qq @ kk.transpose(1, 2)) * D ** -0.5).softmax(-1).matmul(vv).transpose(0, 1)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("block,topk,D", [(4, 32, 128), (4, 24, 256), (64, 3, 128)])
def test_qsa_training_selection_and_attention_match_oracle(block, topk, D):
    """QSA in training: the packed-row selection (serving select kernels over row sets) equals the per-query
    oracle, and the masked forward / backward equal fp32 attention restricted to each row's selected blocks."""
    from arc_forge_2026_b200.models.reference import rope_cos_sin
    from arc_forge_2026_b200.ops.qsa import pooled_key_reference
    from arc_forge_2026_b200.train.attention import qsa_select_packed
    g = torch.Generator().manual_seed(block * 100 + topk)
    lens = [300, 700, 45]
    Hq, Hkv, Hi, rot = 8, 2, 4, 64
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    cos, sin = (t.contiguous() for t in rope_cos_sin(torch.arange(2048), rot, 1.0e7))
    idx_q = torch.randn(T, Hi, 128, generator=g).bfloat16()
    raw = torch.randn(T, 128, generator=g).bfloat16()
    kn = (torch.randn(128, generator=g) * 0.1).bfloat16()
    blkmap = qsa_select_packed(idx_q.to(dev), raw.to(dev), kn.to(dev), cos.to(dev), sin.to(dev), rot, 1e-6, cu,
                               block, topk)
    torch.cuda.synchronize()
    check_status()
    bm = blkmap.cpu()
    allowed = torch.zeros(T, T, dtype=torch.bool)
    for s, (s0, s1) in enumerate(zip(cu[:-1].tolist(), cu[1:].tolist())):
        L = s1 - s0
        keys = torch.stack([pooled_key_reference(raw[s0 + b * block:s0 + (b + 1) * block], b, kn, cos, sin, rot,
                                                 block=block).bfloat16().float() for b in range(L // block)]) \
            if L >= block else torch.zeros(0, 128)
        for p in range(L):
            n = (p + 1) // block
            if n <= topk:
                chosen = list(range(n))
            else:
                sc = torch.relu(idx_q[s0 + p].float() @ keys[:n].t()).sum(0) / 128 ** 0.5
                chosen = sorted(sorted(range(n), key=lambda b: (-float(sc[b]), b))[:topk])
            if (p + 1) % block:
                chosen.append(n)
            got = [b for b in range(bm.shape[1] * 32) if (int(bm[s0 + p, b // 32]) >> (b % 32)) & 1]
            assert got == chosen, (s, p, got[:8], chosen[:8])
            for b in chosen:
                allowed[s0 + p, s0 + b * block:min(s1, s0 + (b + 1) * block)] = True
    q = torch.randn(T, Hq, D, generator=g).bfloat16().to(dev).requires_grad_()
    k = torch.randn(T, Hkv, D, generator=g).bfloat16().to(dev).requires_grad_()
    v = torch.randn(T, Hkv, D, generator=g).bfloat16().to(dev).requires_grad_()
    do = torch.randn(T, Hq, D, generator=g).bfloat16().to(dev)
    out = varlen_attention(q, k, v, cu, blkmap, block)
    out.backward(do)
    torch.cuda.synchronize()
    check_status()
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    ref = varlen_attention_reference(qf, kf, vf, cu, allowed)
    ref.backward(do.float())
    assert _rel(out, ref) < 1e-2
    for a, b in ((q.grad, qf.grad), (k.grad, kf.grad), (v.grad, vf.grad)):
        assert _rel(a, b) < 2e-2
    dense = varlen_attention_reference(qf.detach(), kf.detach(), vf.detach(), cu)
    assert _rel(out, dense) > 5e-2  # the selection matters at these lengths


def test_packed_student_with_qsa_follows_the_reference_and_trains():
    """A packed QAD student with QSA (4-token blocks, top-8: sparse past 32 tokens) against the fp32 reference
    model with its QSA, sequence by sequence; its backward runs through the masked native attention."""
    import dataclasses

    from arc_forge_2026_b200.config import FULL, preset
    from arc_forge_2026_b200.models.reference import build_reference
    from arc_forge_2026_b200.quant.gptq import rtn_quantize
    from arc_forge_2026_b200.train import kernels
    from arc_forge_2026_b200.train.packing import pack
    from arc_forge_2026_b200.train.student import QADStudent
    cfg = preset("tiny_gpu", qsa_block=4, qsa_topk=8)
    ref = build_reference(cfg, seed=6)
    cs = []
    with torch.no_grad():
        for moe in ref.moe_layers():
            c13, s13 = rtn_quantize(moe.w13.float())
            c2, s2 = rtn_quantize(moe.w2.float())
            s13, s2 = s13.bfloat16().float(), s2.bfloat16().float()
            moe.w13.copy_((c13.float() - 4) * s13.repeat_interleave(128, -1))
            moe.w2.copy_((c2.float() - 4) * s2.repeat_interleave(128, -1))
            cs.append((c13, s13, c2, s2))
        # dense projections the student trains in block FP8 start on the FP8 grid, so its QAT forward is exact and
        # the comparison isolates attention (bf16 activations remain)
        from arc_forge_2026_b200.quant import fp8 as fp8q
        for lay in ref.layers:
            for name in (("q_proj", "k_proj", "v_proj") if lay.kind == FULL else ("in_proj_qkvz", "out_proj")):
                w = getattr(lay.mixer, name).weight
                qv, sv = fp8q.quantize_weight_block(w.bfloat16().float())
                w.copy_(fp8q.dequant_weight_block(qv, sv).bfloat16().float())
    st = QADStudent(cfg, ref, cs, checkpoint_layers=False).to(dev)
    g = torch.Generator().manual_seed(6)
    seqs = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (150, 90)]
    (b,) = pack(seqs, 512)
    b = b.to(dev)
    kernels.reset()
    h = st.hidden(b.ids[None], pack=b.forward_args())[0].float()
    h.pow(2).mean().backward()
    torch.cuda.synchronize()
    check_status()
    assert kernels.counts()["native"].get("attention", 0) == 0  # QSA rows take the masked native path directly
    dense_cfg = dataclasses.replace(cfg, qsa_topk=1 << 20)
    errs, errs_dense = [], []
    with torch.no_grad():
        for s0, i in zip(b.cu_seqlens.tolist(), b.seq_index):
            n = len(seqs[i])
            r = ref.hidden(torch.tensor([seqs[i]]))[0].float()
            for lay in ref.layers:
                if lay.kind == FULL:
                    lay.mixer.cfg = dense_cfg
            rd = ref.hidden(torch.tensor([seqs[i]]))[0].float()
            for lay in ref.layers:
                if lay.kind == FULL:
                    lay.mixer.cfg = cfg
            got = h[s0:s0 + n].detach().cpu()
            e = (got - r).norm(dim=-1) / r.norm(dim=-1)
            ed = (got - rd).norm(dim=-1) / rd.norm(dim=-1)
            errs.append(e[40:])
            errs_dense.append(ed[40:])
    e, ed = torch.cat(errs), torch.cat(errs_dense)
    assert e.median() < 0.06, (e.median(), ed.median())
    assert e.median() < 0.5 * ed.median(), (e.median(), ed.median())
