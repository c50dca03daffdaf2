"""Drafter conversions: the on-disk drafter layout, HC -> plain conversion, layer expansion, trained export and the
block-FP8 deployment copy (the reference's ``training/work/qwen38fn_dflash/{init_mtp3,convert_plain,expand_layers,
export_trained,make_dense_deploy}.py``).

Layout of a drafter directory (one per published drafter; written into ``<out>.tmp-<pid>`` and renamed into place,
so a reader never sees a half-written one):

    config.json                      DrafterConfig fields + target_hidden, vocab_size
    interface.safetensors            embed, fc, lm_head, draft_vocab, final_norm | hc_final.*
    layer-<i>.safetensors            one decoder layer's tensors (names as in ``DrafterTrain``)
    initialization_manifest.json     kind (export | plain-conversion | layer-expansion | deploy), provenance
    calibration.json                 plain conversions only: every fit's relative residual and the fold statistics
    SHA256SUMS                       of every other file

Deployment copies hold the chosen linears as e4m3 ``<name>`` plus fp32 ``<name>_scale_inv`` per 128 x 128 block
(``quant/fp8.py``); every other tensor is copied bit for bit.

HC -> plain (``convert_plain``): the plain drafter's weights are derived from the HC / dense_shared source —

* bit for bit: embed, fc, lm_head, draft_vocab, every layer's ``w_qkv``, q/k/ctx norms;
* ``w13 = [gate_r; gate_s; up_r; up_s]``, ``w2 = [w2_r, s * w2_s] * gm``, s = E[sigmoid(shared gate)], gm = the
  layer's mean MLP write-back gate; ``w_o * ga`` with ga the mean attention write-back gate (the mean branch's
  update);
* every RMSNorm gain (in / post / final) is fitted one site at a time on calibration blocks, per channel by least
  squares of the plain stream's unit-RMS state onto the HC mix output it replaces, with the plain model's own
  upstream (earlier gains already fitted).

The injected context (``ctx_norm`` and the k/v rows of ``w_qkv``) does not read the stream, so it carries over as is.
The conversion is exact when the HC source is a single stream in disguise (constant mixes, unit gates, a constant
shared gate); ``tests/test_drafter_tools.py`` checks that.
"""
from __future__ import annotations

import argparse
import dataclasses
import hashlib
import json
import os
import re
import shutil
from pathlib import Path

import torch
from safetensors.torch import load_file, save_file

from ..config import DrafterConfig
from ..quant.fp8 import dequant_weight_block, quantize_weight_block
from .drafter_train import DrafterTrain

RIDGE = 1e-6
_LINEARS = {"attn": ("w_qkv", "w_o"), "mlp": ("w13", "w2", "sw13", "sw2")}


# ---------------------------------------------------------------------------------------------------- layout I/O
def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def _state(model: DrafterTrain) -> tuple[dict, list[dict]]:
    """(interface tensors, per-layer tensors) of a training twin, fp32 on the CPU."""
    iface, layers = {}, [{} for _ in model.layers]
    for name, t in list(model.named_parameters()) + list(model.named_buffers()):
        if name == "to_draft":
            continue
        m = re.match(r"^layers\.(\d+)\.(.*)$", name)
        t = t.detach().cpu().contiguous()
        if m:
            layers[int(m.group(1))][m.group(2)] = t
        else:
            iface[name] = t
    return iface, layers


def save_dir(model: DrafterTrain, out, kind: str, manifest: dict | None = None, calibration: dict | None = None,
             fp8: tuple[str, ...] = ()) -> Path:
    """Publish ``model`` as a drafter directory; ``fp8``: linear groups ("attn", "mlp") stored in block FP8."""
    out = Path(out)
    tmp = out.with_name(out.name + f".tmp-{os.getpid()}")
    if tmp.exists():
        shutil.rmtree(tmp)
    tmp.mkdir(parents=True)
    iface, layers = _state(model)
    quantized = {n for g in fp8 for n in _LINEARS[g]}
    save_file(iface, str(tmp / "interface.safetensors"))
    for i, t in enumerate(layers):
        out_t = {}
        for n, v in t.items():
            if n in quantized:
                q, s = quantize_weight_block(v.float())
                out_t[n], out_t[n + "_scale_inv"] = q, s
            else:
                out_t[n] = v
        save_file(out_t, str(tmp / f"layer-{i}.safetensors"))
    cfg = dict(dataclasses.asdict(model.cfg), target_hidden=model.fc.shape[1], vocab_size=model.vocab_size)
    (tmp / "config.json").write_text(json.dumps(cfg, indent=1, sort_keys=True))
    (tmp / "initialization_manifest.json").write_text(
        json.dumps(dict(manifest or {}, kind=kind, fp8_groups=list(fp8)), indent=1, sort_keys=True))
    if calibration is not None:
        (tmp / "calibration.json").write_text(json.dumps(calibration, indent=1, sort_keys=True))
    sums = [f"{_sha256(p)}  {p.name}" for p in sorted(tmp.iterdir())]
    (tmp / "SHA256SUMS").write_text("\n".join(sums) + "\n")
    if out.exists():
        shutil.rmtree(out)
    os.replace(tmp, out)
    return out


def verify_dir(path) -> None:
    path = Path(path)
    for line in (path / "SHA256SUMS").read_text().splitlines():
        digest, name = line.split("  ", 1)
        if _sha256(path / name) != digest:
            raise ValueError(f"{path / name}: sha256 mismatch")


def load_dir(path, device="cpu", verify: bool = True) -> DrafterTrain:
    """A drafter directory as a training twin (fp32; block-FP8 linears dequantised)."""
    path = Path(path)
    if verify:
        verify_dir(path)
    raw = json.loads((path / "config.json").read_text())
    target_hidden, vocab = raw.pop("target_hidden"), raw.pop("vocab_size")
    cfg = DrafterConfig(**raw)
    iface = load_file(str(path / "interface.safetensors"))
    model = DrafterTrain(cfg, target_hidden, vocab, iface["draft_vocab"], device=device)
    state = {k: v for k, v in iface.items()}
    for i in range(cfg.num_layers):
        t = load_file(str(path / f"layer-{i}.safetensors"))
        for n, v in t.items():
            if n.endswith("_scale_inv"):
                continue
            if v.dtype == torch.float8_e4m3fn:
                v = dequant_weight_block(v, t[n + "_scale_inv"])
            state[f"layers.{i}.{n}"] = v
    state["to_draft"] = model.to_draft
    model.load_state_dict({k: v.to(device) for k, v in state.items()})
    return model


def manifest_of(path) -> dict:
    return json.loads((Path(path) / "initialization_manifest.json").read_text())


# ---------------------------------------------------------------------------------------------------- HC -> plain
def plain_config(c: DrafterConfig) -> DrafterConfig:
    if c.residual != "hc" or c.ffn != "dense_shared":
        raise ValueError("the conversion takes an HC dense_shared drafter")
    return dataclasses.replace(c, residual="plain", hc_count=1, ffn="dense",
                               intermediate_size=c.intermediate_size + c.shared_intermediate_size,
                               shared_intermediate_size=0)


class _Stop(Exception):
    pass


def _record_source(src: DrafterTrain, calib) -> dict:
    """Per site, the HC source's sub-layer inputs (and gates, shared-gate logits) over the calibration blocks."""
    rows: dict[str, list] = {}

    def probe(site, stream, y, gate):
        rows.setdefault(site, []).append((y.detach().reshape(-1, y.shape[-1]).float(),
                                          None if gate is None else gate.detach().reshape(-1, gate.shape[-1]).float()))
    with torch.no_grad():
        for tokens, hidden, anchors in calib:
            src.block_logits(tokens, hidden, anchors, probe=probe)
    return {k: (torch.cat([a for a, _ in v]), None if v[0][1] is None else torch.cat([b for _, b in v]))
            for k, v in rows.items()}


def _unit(x, eps):
    z = x.float()
    return z * torch.rsqrt(z.square().mean(-1, keepdim=True) + eps)


def _channel_gain(n, target):
    """Per channel argmin_g ||g n - target||^2 (small ridge) and the fit's relative residual (and that of g = 1)."""
    n, target = n.double(), target.double()
    nn2 = n.square().sum(0)
    gain = (n * target).sum(0) / (nn2 + RIDGE * nn2.mean())
    norm = target.norm()
    return gain.float(), {"relative_residual": ((gain * n - target).norm() / norm).item(),
                          "relative_residual_unit_gain": ((n - target).norm() / norm).item()}


@torch.no_grad()
def convert_plain(src: DrafterTrain, calib) -> tuple[DrafterTrain, dict]:
    """The plain / dense drafter of an HC dense_shared source. ``calib``: list of (tokens [T], hidden [T, Ht],
    anchors [A]) calibration sequences. Returns (model, calibration report)."""
    c = plain_config(src.cfg)
    I, Is = src.cfg.intermediate_size, src.cfg.shared_intermediate_size
    rec = _record_source(src, calib)
    model = DrafterTrain(c, src.fc.shape[1], src.vocab_size, src.draft_vocab.cpu(), device=src.fc.device)
    stats = []
    for i, (ms, md) in enumerate(zip(src.layers, model.layers)):
        s = torch.sigmoid(rec[f"shared{i}"][0]).mean().item()
        ga = rec[f"attn{i}"][1].mean().item()
        gm = rec[f"mlp{i}"][1].mean().item()
        stats.append({"layer": i, "shared_sigmoid_mean": s, "attention_gate_mean": ga, "mlp_gate_mean": gm,
                      "attention_gate_std_over_branches": rec[f"attn{i}"][1].std(-1).mean().item(),
                      "mlp_gate_std_over_branches": rec[f"mlp{i}"][1].std(-1).mean().item()})
        for n in ("ctx_norm", "w_qkv", "q_norm", "k_norm"):
            getattr(md, n).copy_(getattr(ms, n))
        md.w_o.copy_(ms.w_o * ga)
        md.w13.copy_(torch.cat([ms.w13[:I], ms.sw13[:Is], ms.w13[I:], ms.sw13[Is:]]))
        md.w2.copy_(torch.cat([ms.w2, ms.sw2 * s], 1) * gm)
        md.in_norm.zero_()
        md.post_norm.zero_()
    for n in ("embed", "fc", "lm_head"):
        getattr(model, n).copy_(getattr(src, n))
    if src.selector is not None:  # the selector reads the final hidden state, which the fitted final norm keeps
        model.selector.load_state_dict(src.selector.state_dict())
    model.final_norm.zero_()
    # the gains, one site at a time, each on the converted model's own upstream
    fits = {}
    sites = [s for i in range(c.num_layers) for s in (f"attn{i}", f"mlp{i}")] + ["final"]
    for site in sites:
        got = []

        def probe(name, stream, y, gate, site=site):
            if name == site:
                got.append(_unit(stream, c.rms_norm_eps).reshape(-1, stream.shape[-1]))
                raise _Stop
        for tokens, hidden, anchors in calib:
            try:
                model.block_logits(tokens, hidden, anchors, probe=probe)
            except _Stop:
                pass
        gain, rep = _channel_gain(torch.cat(got), rec[site][0])
        if site == "final":
            w = model.final_norm
        else:
            L = model.layers[int(site[4:] if site.startswith("attn") else site[3:])]
            w = L.in_norm if site.startswith("attn") else L.post_norm
        w.copy_(gain - 1.0)  # zero-centred weights: the norm multiplies by (1 + w)
        fits[site] = rep
    return model, {"fits": fits, "layers": stats, "calibration_blocks": sum(int(a.numel()) for _, _, a in calib)}


# ---------------------------------------------------------------------------------------------------- expansion
@torch.no_grad()
def expand_layers(src: DrafterTrain, order: list[int], zero_repeats: bool = True) -> DrafterTrain:
    """Layer j of the result is a copy of source layer ``order[j]``. ``zero_repeats`` (block expansion): a repeat —
    a source layer already used earlier in the order — gets ``w_o`` and ``w2`` zeroed, so it adds exactly zero to
    the stream and the expanded drafter computes the source's function. Plain residual only (a hyper-connection
    layer also mixes the branches, so a zeroed output is not an identity there)."""
    if src.hc:
        raise ValueError("layer expansion takes a plain-residual drafter")
    if not order or min(order) < 0 or max(order) >= len(src.layers):
        raise ValueError(f"order {order} out of range for {len(src.layers)} layers")
    c = dataclasses.replace(src.cfg, num_layers=len(order))
    model = DrafterTrain(c, src.fc.shape[1], src.vocab_size, src.draft_vocab.cpu(), device=src.fc.device)
    sd = {k: v for k, v in src.state_dict().items() if not k.startswith("layers.")}
    seen = set()
    for j, i in enumerate(order):
        for k, v in src.layers[i].state_dict().items():
            v = v.clone()
            if zero_repeats and i in seen and k in ("w_o", "w2", "sw2"):
                v.zero_()
            sd[f"layers.{j}.{k}"] = v
        seen.add(i)
    model.load_state_dict(sd)
    return model


# ---------------------------------------------------------------------------------------------------- CLI
def _calibration(path, device) -> list:
    """Calibration sequences: a ``.pt`` list of dicts with tokens [T], hidden [T, Ht] and anchors [A]."""
    items = torch.load(path, map_location=device)
    return [(d["tokens"].long(), d["hidden"].float(), d["anchors"].long()) for d in items]


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    a = sub.add_parser("plain", help="HC dense_shared drafter -> plain dense drafter")
    a.add_argument("--source", required=True)
    a.add_argument("--calibration", required=True)
    a.add_argument("--out", required=True)
    b = sub.add_parser("expand", help="repeat decoder layers")
    b.add_argument("--source", required=True)
    b.add_argument("--order", required=True, help="comma list of source layers, e.g. 0,1,2,3,1,2,3,4")
    b.add_argument("--no-zero-repeats", action="store_true")
    b.add_argument("--out", required=True)
    d = sub.add_parser("deploy", help="deployment copy with block-FP8 linears")
    d.add_argument("--source", required=True)
    d.add_argument("--fp8", default="attn,mlp", help="linear groups in block FP8 (empty: an all-BF16 copy)")
    d.add_argument("--out", required=True)
    e = sub.add_parser("export", help="a trainer checkpoint (torch state dict of DrafterTrain) as a drafter dir")
    e.add_argument("--checkpoint", required=True)
    e.add_argument("--config", required=True, help="a drafter directory whose config.json the checkpoint matches")
    e.add_argument("--out", required=True)
    args = ap.parse_args(argv)
    if args.cmd == "plain":
        src = load_dir(args.source)
        model, report = convert_plain(src, _calibration(args.calibration, "cpu"))
        out = save_dir(model, args.out, "plain-conversion", {"source": str(args.source)}, report)
    elif args.cmd == "expand":
        order = [int(x) for x in args.order.split(",")]
        model = expand_layers(load_dir(args.source), order, not args.no_zero_repeats)
        out = save_dir(model, args.out, "layer-expansion",
                       {"source": str(args.source), "order": order, "zero_repeats": not args.no_zero_repeats})
    elif args.cmd == "deploy":
        groups = tuple(g for g in args.fp8.split(",") if g)
        bad = set(groups) - set(_LINEARS)
        if bad:
            raise SystemExit(f"unknown fp8 groups {sorted(bad)}; known: {sorted(_LINEARS)}")
        out = save_dir(load_dir(args.source), args.out, "deploy", {"source": str(args.source)}, fp8=groups)
    else:
        model = load_dir(args.config)
        model.load_state_dict(torch.load(args.checkpoint, map_location="cpu"))
        out = save_dir(model, args.out, "export", {"checkpoint": str(args.checkpoint)})
    print(json.dumps({"out": str(out), "kind": manifest_of(out)["kind"]}))
    return out


if __name__ == "__main__":
    main()
