"""Compression pipeline (the reference's A1 -> A5: saliency capture, gEAN pruning, GPTQ INT3, packing, deploy
package; ``training/work/qwen38fn_eval/{saliency_hook,reap_mm_select,prune_experts,gptq_hess_hook,
quantize_int3_gptq,build_int3_deploy}.py``), on the fp32 oracle model.

    python -m arc_forge_2026_b200.quant.pipeline --preset tiny_cpu --keep 20 --calib-tokens 512 --out pkg

Steps:

1. REAP saliency of every (layer, expert) over the calibration tokens, keep the top ``keep`` experts per layer
   (gEAN mask), prune them out of the model (router rows included);
2. per-expert Hessians of the routed calibration rows: ``H13_e = X_e^T X_e`` of the expert's inputs (for w13) and
   ``H2_e = h_e^T h_e`` of its SwiGLU activations (for w2), shrunk toward the layer's pooled Hessian with a prior
   of ``prior_tokens`` pseudo-rows (experts with few rows borrow the layer's statistics; none -> pure prior);
3. GPTQ INT3 g128 (symmetric uint3, zero 4, signed bf16 scales, MSE clip search) per expert with damping; RTN if
   the layer saw no rows at all;
4. pack (Humming uint3) and write the INT3 deploy package (``formats/int3_package.py``) with a pipeline record.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch
import torch.nn.functional as F

from ..config import preset
from ..models import reference as R
from . import gptq, saliency


@torch.no_grad()
def collect_hessians(model: R.HybridMoE, batches, prior_tokens: int = 256):
    """Per layer: (H13 [E, H, H], H2 [E, I, I], rows [E]) with the pooled-prior shrinkage applied."""
    c = model.cfg
    E, Hd, I = c.num_experts, c.hidden_size, c.moe_intermediate_size
    acc = [dict(h13=torch.zeros(E, Hd, Hd), h2=torch.zeros(E, I, I), n=torch.zeros(E)) for _ in model.layers]
    hooks = []

    def make(li):
        def pre(mod, args):
            x = args[0].reshape(-1, Hd).float()
            _, ids = R.route(mod.gate(x), c.num_experts_per_tok, c.norm_topk_prob)
            for e in torch.unique(ids).tolist():
                tok = (ids == e).any(-1).nonzero(as_tuple=True)[0]
                xe = x[tok]
                h = xe @ mod.w13[e].float().t()
                he = F.silu(h[:, :I]) * h[:, I:]
                acc[li]["h13"][e] += xe.t() @ xe
                acc[li]["h2"][e] += he.t() @ he
                acc[li]["n"][e] += xe.shape[0]
        return pre
    for li, layer in enumerate(model.layers):
        hooks.append(layer.mlp.register_forward_pre_hook(make(li)))
    try:
        for ids in batches:
            model(ids)
    finally:
        for h in hooks:
            h.remove()
    out = []
    for a in acc:
        n = a["n"]
        tot = float(n.sum())
        pool13 = a["h13"].sum(0) / max(tot, 1.0)
        pool2 = a["h2"].sum(0) / max(tot, 1.0)
        w = (n + prior_tokens)[:, None, None]
        h13 = (a["h13"] + prior_tokens * pool13) / w
        h2 = (a["h2"] + prior_tokens * pool2) / w
        out.append((h13, h2, n, tot))
    return out


def quantize_model(model: R.HybridMoE, hessians, damp: float = 0.01):
    """GPTQ every expert; returns per layer (w13_codes, w13_scales, w2_codes, w2_scales) and error stats."""
    packs, stats = [], []
    for moe, (h13, h2, n, tot) in zip(model.moe_layers(), hessians):
        if tot == 0:
            c13, s13 = gptq.rtn_quantize(moe.w13.detach().float())
            c2, s2 = gptq.rtn_quantize(moe.w2.detach().float())
        else:
            c13, s13 = gptq.gptq_quantize(moe.w13.detach().float(), h13, damp=damp)
            c2, s2 = gptq.gptq_quantize(moe.w2.detach().float(), h2, damp=damp)
        packs.append((c13, s13.to(torch.bfloat16), c2, s2.to(torch.bfloat16)))
        # output reconstruction error weighted by the Hessian: tr(dW H dW^T) / tr(W H W^T)
        dw = gptq.dequant(c13, s13.to(torch.bfloat16)) - moe.w13.detach().float()
        num = torch.einsum("eok,ekl,eol->", dw, h13, dw)
        den = torch.einsum("eok,ekl,eol->", moe.w13.detach().float(), h13, moe.w13.detach().float())
        stats.append({"rows": int(n.sum()), "w13_rel_err": float(num / den.clamp_min(1e-30))})
    return packs, stats


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="tiny_cpu")
    ap.add_argument("--keep", type=int, default=20, help="experts kept per layer (gEAN)")
    ap.add_argument("--calib-tokens", dest="calib_tokens", type=int, default=512)
    ap.add_argument("--prior-tokens", dest="prior_tokens", type=int, default=256)
    ap.add_argument("--damp", type=float, default=0.01)
    ap.add_argument("--seq", type=int, default=256)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--dense-fp8", dest="dense_fp8", action="store_true", help="block-FP8 dense projections")
    ap.add_argument("--out", type=Path, required=True)
    args = ap.parse_args(argv)
    from ..formats.int3_package import package_tensors, write_package
    cfg = preset(args.preset)
    model = R.build_reference(cfg, seed=args.seed)
    g = torch.Generator().manual_seed(args.seed + 1)
    nseq = max(1, args.calib_tokens // args.seq)
    batches = [torch.randint(0, cfg.vocab_size, (1, args.seq), generator=g) for _ in range(nseq)]
    acc = saliency.collect_saliency(model, batches)
    scores = saliency.reap_scores(acc.acc)
    drop = saliency.keep_mask(scores, args.keep)
    mass = saliency.retained_mass(scores, drop)
    model = saliency.prune_experts(model, drop)
    hess = collect_hessians(model, batches, args.prior_tokens)
    packs, stats = quantize_model(model, hess, args.damp)
    record = {"preset": args.preset, "keep": args.keep, "calib_tokens": nseq * args.seq,
              "retained_mass": mass, "layers": stats, "prior_tokens": args.prior_tokens, "damp": args.damp}
    path = write_package(package_tensors(model, packs, args.dense_fp8), model.cfg, args.out,
                         dense_fp8=args.dense_fp8, meta={"pipeline": record})
    print(json.dumps({"package": str(path), "retained_mass_mean": mass["mean"],
                      "w13_rel_err_mean": sum(s["w13_rel_err"] for s in stats) / len(stats)}))
    return path


if __name__ == "__main__":
    main()
