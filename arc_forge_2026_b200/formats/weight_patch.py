"""RL overlay and delta-only weight patch of a deploy package, in the reference's two formats so either tool chain
can consume the other's output (``training/work/qwen38fn_rl/rl_overlay_package.py:1-20``,
``training/work/qwen38fn_rl/rl_weight_patch.py:1-26,94-190``).

Overlay (``arcforge.kaggle.model_overlay.v1``) -- a merged RL version (``fn-lora-merged-v2`` directory) against the
package it was trained on: only the shards holding a merged tensor, rewritten with those tensors (same names, dtypes
and shapes; nothing added or requantised), the package's ``deploy_manifest.json`` with those shards' new entries and
an ``rl_merged`` block, and ``overlay.json``::

    <overlay>/<shard>.safetensors ...   rewritten shards
    <overlay>/deploy_manifest.json      the package's manifest, rewritten entries, + rl_merged
    <overlay>/overlay.json              schema, base_manifest_sha256, deploy_manifest_sha256, files, rl_merged, report
    <overlay>/DONE

Weight patch (``arcforge.kaggle.weight_patch.v1``) -- overlay + package -> only the tensors whose bytes changed,
one ``patch-<shard>`` safetensors per rewritten shard (metadata ``patch_of``), the overlay's manifest, and::

    <patch>/patch.json   schema, base / deploy manifest sha256, overlay_files, rl_merged,
                         files {patch-<shard>: sha256, bytes, shard, tensors},
                         tensors {name: file, shard, dtype, shape, sha256}, report

Both are published as ``<out>.partial`` renamed to ``<out>``, then ``DONE``. The checks mirror the contract: the
base manifest the overlay names is rebuilt from the overlay's manifest with the package's own entries for the
rewritten shards and must hash to ``base_manifest_sha256`` (manifests are written as ``json.dumps(m, indent=2)`` +
newline, as the package writer does); rewritten shards keep the package's header byte for byte; the patch is read
back and base + patch must reproduce every overlay shard's sha256. :class:`WeightPatch` is the serving side: it hands
a loader the patch's tensor wherever the package's would go (each exactly once, dtype / shape / sha256 checked).

    python -m arc_forge_2026_b200.formats.weight_patch overlay --source PKG --source-manifest-sha256 SHA \\
        --merged MERGED_DIR --out OVERLAY
    python -m arc_forge_2026_b200.formats.weight_patch patch --base PKG --overlay OVERLAY --out PATCH
"""
from __future__ import annotations

import argparse
import hashlib
import json
import struct
from pathlib import Path

import torch

OVERLAY_SCHEMA = "arcforge.kaggle.model_overlay.v1"
PATCH_SCHEMA = "arcforge.kaggle.weight_patch.v1"
MERGED_FORMAT = "fn-lora-merged-v2"
RL_META_KEYS = ("weight_version", "step", "optimizer_step", "run", "base_model", "lora_rank", "lora_alpha",
                "dense_qat")


def file_sha(path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


def tensor_sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().cpu().contiguous().reshape(-1).view(torch.uint8).numpy().tobytes()).hexdigest()


def manifest_bytes(m: dict) -> bytes:
    """The byte form every manifest here is written in (and the base-manifest rebuild hashes)."""
    return (json.dumps(m, indent=2) + "\n").encode()


def _header(path: Path) -> tuple[bytes, dict]:
    """(8-byte length + JSON header bytes, parsed header) of a safetensors file."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise EOFError(path)
        n = struct.unpack("<Q", raw)[0]
        if n > (64 << 20):
            raise ValueError(f"{path}: safetensors header of {n} bytes")
        body = f.read(n)
    return raw + body, json.loads(body)


def _payload_order(header: dict) -> tuple[list, int]:
    """Tensors by data offset; checks that they cover the payload with no gap or overlap."""
    items = sorted(((k, v) for k, v in header.items() if k != "__metadata__"), key=lambda kv: kv[1]["data_offsets"])
    end = 0
    for name, ent in items:
        a, b = ent["data_offsets"]
        if a != end or b < a:
            raise ValueError(f"{name}: payload gap or overlap at byte {end}")
        end = b
    return items, end


def _publish(partial: Path, out: Path):
    partial.rename(out)
    (out / "DONE").write_text("ok\n")


def _fresh(out: Path) -> Path:
    partial = out.with_name(out.name + ".partial")
    if out.exists() or partial.exists():
        raise FileExistsError(out)
    return partial


# ----------------------------------------------------------------------------------------------------- overlay
def build_overlay(source, source_manifest_sha256: str, merged, out, step_is_optimizer_step: bool = False) -> dict:
    """Rewrite the package shards that hold a merged tensor; returns overlay.json's content."""
    from safetensors import safe_open
    from safetensors.torch import save_file
    src, merged, out = Path(source), Path(merged), Path(out)
    partial = _fresh(out)
    if not (merged / "DONE").exists():
        raise RuntimeError(f"{merged} is not published (no DONE)")
    if file_sha(src / "deploy_manifest.json") != source_manifest_sha256:
        raise RuntimeError(f"{src}/deploy_manifest.json does not hash to {source_manifest_sha256}")
    deploy = json.loads((src / "deploy_manifest.json").read_text())
    mman_path = merged / "merged_manifest.json"
    mman = json.loads(mman_path.read_text())
    if mman.get("format") != MERGED_FORMAT:
        raise RuntimeError(f"{merged}: format {mman.get('format')!r}, expected {MERGED_FORMAT}")
    shards = sorted(p.name for p in merged.glob("*.safetensors"))
    if shards != ["model.safetensors"]:
        raise RuntimeError(f"{merged}: expected exactly model.safetensors, found {shards}")
    with safe_open(str(merged / "model.safetensors"), "pt") as h:
        new = {k: h.get_tensor(k) for k in h.keys()}
    if set(new) != set(mman["keys"]):
        raise RuntimeError(f"{merged}: tensors and merged_manifest.json keys differ")
    for k, t in new.items():
        if tensor_sha(t) != mman["keys"][k]["merged_sha256"]:
            raise RuntimeError(f"{k}: bytes differ from merged_manifest.json")
    wmap = json.loads((src / "model.safetensors.index.json").read_text())["weight_map"]
    unknown = sorted(set(new) - set(wmap))
    if unknown:
        raise KeyError(f"{len(unknown)} merged tensors are not in the package, e.g. {unknown[:3]}")
    by_shard: dict[str, list[str]] = {}
    for k in sorted(new):
        by_shard.setdefault(wmap[k], []).append(k)
    for shard in by_shard:
        ent = deploy["files"][shard]
        if (src / shard).stat().st_size != ent["bytes"] or file_sha(src / shard) != ent["sha256"]:
            raise RuntimeError(f"{src}/{shard} does not match its manifest entry")
    partial.mkdir(parents=True)
    report = {"replaced": 0, "changed_bytes": 0, "rewritten_shards": sorted(by_shard)}
    for shard, keys in sorted(by_shard.items()):
        with safe_open(str(src / shard), "pt") as h:
            meta = h.metadata()
            tensors = {}
            for k in h.keys():
                t = h.get_tensor(k)
                if k in new:
                    m = new[k]
                    if m.dtype != t.dtype or m.shape != t.shape:
                        raise TypeError(f"{k}: merged {m.dtype}{tuple(m.shape)}, package {t.dtype}{tuple(t.shape)}")
                    report["changed_bytes"] += int((m.contiguous().view(torch.uint8) !=
                                                    t.contiguous().view(torch.uint8)).sum())
                    report["replaced"] += 1
                    t = m
                tensors[k] = t.contiguous()
        save_file(tensors, str(partial / shard), metadata=meta)
        if _header(partial / shard)[0] != _header(src / shard)[0]:
            raise RuntimeError(f"{shard}: the rewritten header differs from the package's (layout changed)")
        with safe_open(str(partial / shard), "pt") as h, safe_open(str(src / shard), "pt") as s:
            for k in h.keys():
                want = mman["keys"][k]["merged_sha256"] if k in new else tensor_sha(s.get_tensor(k))
                if tensor_sha(h.get_tensor(k)) != want:
                    raise RuntimeError(f"{shard}/{k}: read-back mismatch")
    if report["replaced"] != len(new):
        raise RuntimeError(f"replaced {report['replaced']} of {len(new)} merged tensors")
    files = {}
    for shard in sorted(by_shard):
        ent = {"sha256": file_sha(partial / shard), "bytes": (partial / shard).stat().st_size}
        deploy["files"][shard] = ent
        files[shard] = ent
    if "optimizer_step" not in mman:
        if not step_is_optimizer_step:
            raise KeyError(f"{merged}: merged manifest has no optimizer_step (pass step_is_optimizer_step)")
        mman = {**mman, "optimizer_step": mman["step"]}
    rl = {k: mman.get(k) for k in RL_META_KEYS}
    rl["merged_dir"] = str(merged)
    rl["merged_manifest_sha256"] = file_sha(mman_path)
    deploy["rl_merged"] = {**rl, "source_package": str(src), "source_manifest_sha256": source_manifest_sha256,
                           "rewritten_shards": report["rewritten_shards"]}
    (partial / "deploy_manifest.json").write_bytes(manifest_bytes(deploy))
    overlay = {"schema": OVERLAY_SCHEMA, "base_manifest_sha256": source_manifest_sha256,
               "deploy_manifest_sha256": file_sha(partial / "deploy_manifest.json"), "files": files,
               "rl_merged": rl, "report": report}
    (partial / "overlay.json").write_text(json.dumps(overlay, indent=1) + "\n")
    _publish(partial, out)
    return overlay


# ------------------------------------------------------------------------------------------------------- patch
def build_patch(base, overlay, out) -> dict:
    """The changed tensors of an overlay's rewritten shards against ``base``; returns patch.json's content."""
    from safetensors import safe_open
    from safetensors.torch import save_file
    base, ov, out = Path(base), Path(overlay), Path(out)
    partial = _fresh(out)
    if not (ov / "DONE").exists():
        raise RuntimeError(f"{ov} is not published (no DONE)")
    ovj = json.loads((ov / "overlay.json").read_text())
    if ovj.get("schema") != OVERLAY_SCHEMA:
        raise RuntimeError(f"{ov}: schema {ovj.get('schema')!r}")
    if file_sha(ov / "deploy_manifest.json") != ovj["deploy_manifest_sha256"]:
        raise RuntimeError(f"{ov}/deploy_manifest.json is not the one overlay.json names")
    target = json.loads((ov / "deploy_manifest.json").read_text())
    pkg_files = json.loads((base / "deploy_manifest.json").read_text())["files"]
    rewritten = sorted(ovj["files"])
    rebuilt = json.loads(json.dumps(target))
    rebuilt.pop("rl_merged")
    for shard in rewritten:
        rebuilt["files"][shard] = pkg_files[shard]
    got = hashlib.sha256(manifest_bytes(rebuilt)).hexdigest()
    if got != ovj["base_manifest_sha256"]:
        raise RuntimeError(f"the overlay's manifest with {base}'s entries for {rewritten} hashes to {got}, not the "
                           f"base it names ({ovj['base_manifest_sha256']})")
    partial.mkdir(parents=True)
    tensors, files = {}, {}
    for shard in rewritten:
        head, header = _header(base / shard)
        if _header(ov / shard)[0] != head:
            raise RuntimeError(f"{shard}: package and overlay headers differ; a patch replaces bytes, not layout")
        items, _ = _payload_order(header)
        hb, ho = hashlib.sha256(head), hashlib.sha256(head)
        changed = []
        with open(base / shard, "rb") as fb, open(ov / shard, "rb") as fo:
            fb.seek(len(head))
            fo.seek(len(head))
            for name, ent in items:
                n = ent["data_offsets"][1] - ent["data_offsets"][0]
                a, b = fb.read(n), fo.read(n)
                if len(a) != n or len(b) != n:
                    raise EOFError(f"{shard}:{name}")
                hb.update(a)
                ho.update(b)
                if a != b:
                    changed.append(name)
            if fb.read(1) or fo.read(1):
                raise RuntimeError(f"{shard}: bytes after the last tensor")
        if hb.hexdigest() != pkg_files[shard]["sha256"]:
            raise RuntimeError(f"{base}/{shard} does not match its manifest entry")
        if ho.hexdigest() != ovj["files"][shard]["sha256"]:
            raise RuntimeError(f"{ov}/{shard} does not match overlay.json")
        if not changed:
            raise RuntimeError(f"{shard}: rewritten, yet no tensor changed")
        pname = "patch-" + shard
        with safe_open(str(ov / shard), "pt") as h:
            sel = {k: h.get_tensor(k).contiguous() for k in changed}
        save_file(sel, str(partial / pname), metadata={"format": "pt", "patch_of": shard})
        for k, t in sel.items():
            tensors[k] = {"file": pname, "shard": shard, "dtype": header[k]["dtype"], "shape": header[k]["shape"],
                          "sha256": tensor_sha(t)}
        files[pname] = {"sha256": file_sha(partial / pname), "bytes": (partial / pname).stat().st_size,
                        "shard": shard, "tensors": len(sel)}
    # read back: the patch alone, then every overlay shard rebuilt from package + patch
    for pname, ent in files.items():
        p_head, p_header = _header(partial / pname)
        mine = {k for k, t in tensors.items() if t["file"] == pname}
        if set(p_header) - {"__metadata__"} != mine:
            raise RuntimeError(f"{pname}: tensor set read back differs")
        head, header = _header(base / ent["shard"])
        h = hashlib.sha256(head)
        with open(base / ent["shard"], "rb") as fb, open(partial / pname, "rb") as fp:
            fb.seek(len(head))
            for k, e in _payload_order(header)[0]:
                n = e["data_offsets"][1] - e["data_offsets"][0]
                data = fb.read(n)
                if k in p_header:
                    fp.seek(len(p_head) + p_header[k]["data_offsets"][0])
                    data = fp.read(n)
                    if hashlib.sha256(data).hexdigest() != tensors[k]["sha256"]:
                        raise RuntimeError(f"{pname}/{k}: read-back mismatch")
                h.update(data)
        if h.hexdigest() != ovj["files"][ent["shard"]]["sha256"]:
            raise RuntimeError(f"package {ent['shard']} + {pname} does not reproduce the overlay's shard")
    (partial / "deploy_manifest.json").write_bytes((ov / "deploy_manifest.json").read_bytes())
    patch = {"schema": PATCH_SCHEMA, "base_manifest_sha256": ovj["base_manifest_sha256"],
             "deploy_manifest_sha256": ovj["deploy_manifest_sha256"], "overlay_files": ovj["files"],
             "rl_merged": ovj["rl_merged"], "files": files, "tensors": tensors,
             "report": {"tensors": len(tensors), "bytes": sum(f["bytes"] for f in files.values())}}
    (partial / "patch.json").write_text(json.dumps(patch, indent=1) + "\n")
    _publish(partial, out)
    return patch


class WeightPatch:
    """Serving side of a weight patch: the patch's tensors replace the package's under the same names. Every patch
    tensor must be asked for exactly once, with the package's dtype and shape; its bytes must hash to patch.json."""

    def __init__(self, root, base_manifest_sha256: str | None = None):
        self.root = Path(root)
        if not (self.root / "DONE").exists():
            raise RuntimeError(f"{self.root} is not published (no DONE)")
        self.manifest = json.loads((self.root / "patch.json").read_text())
        if self.manifest.get("schema") != PATCH_SCHEMA:
            raise ValueError(f"{self.root}/patch.json schema {self.manifest.get('schema')!r}, expected {PATCH_SCHEMA}")
        if base_manifest_sha256 is not None and base_manifest_sha256 != self.manifest["base_manifest_sha256"]:
            raise ValueError(f"{self.root} patches the package {self.manifest['base_manifest_sha256']}, not "
                             f"{base_manifest_sha256}")
        self.pending = dict(self.manifest["tensors"])
        self.done: set[str] = set()
        self._handles = {}

    def replace(self, name: str, tensor: torch.Tensor) -> torch.Tensor:
        from safetensors import safe_open
        if name in self.done:
            raise ValueError(f"weight patch: {name} requested twice")
        ent = self.pending.pop(name)
        if ent["file"] not in self._handles:
            self._handles[ent["file"]] = safe_open(str(self.root / ent["file"]), "pt")
        new = self._handles[ent["file"]].get_tensor(name)
        if new.dtype != tensor.dtype or tuple(new.shape) != tuple(tensor.shape):
            raise ValueError(f"weight patch {name}: {new.dtype}{tuple(new.shape)}, the package has "
                             f"{tensor.dtype}{tuple(tensor.shape)}")
        if tensor_sha(new) != ent["sha256"]:
            raise ValueError(f"weight patch {name}: bytes do not hash to patch.json's sha256")
        self.done.add(name)
        return new.to(tensor.device)

    def apply(self, tensors: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
        """A copy of ``tensors`` with every patch tensor substituted; raises if one is missing from ``tensors``."""
        out = {k: (self.replace(k, t) if k in self.pending else t) for k, t in tensors.items()}
        if self.pending:
            raise KeyError(f"weight patch: {len(self.pending)} tensors never loaded, e.g. {sorted(self.pending)[:3]}")
        return out


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m arc_forge_2026_b200.formats.weight_patch")
    sub = ap.add_subparsers(dest="cmd", required=True)
    o = sub.add_parser("overlay", help="merged RL version + package -> overlay")
    o.add_argument("--source", required=True, type=Path)
    o.add_argument("--source-manifest-sha256", required=True)
    o.add_argument("--merged", required=True, type=Path)
    o.add_argument("--out", required=True, type=Path)
    o.add_argument("--step-is-optimizer-step", action="store_true")
    p = sub.add_parser("patch", help="overlay + package -> weight patch")
    p.add_argument("--base", required=True, type=Path)
    p.add_argument("--overlay", required=True, type=Path)
    p.add_argument("--out", required=True, type=Path)
    a = ap.parse_args(argv)
    if a.cmd == "overlay":
        r = build_overlay(a.source, a.source_manifest_sha256, a.merged, a.out, a.step_is_optimizer_step)
        print(json.dumps({"out": str(a.out), "deploy_manifest_sha256": r["deploy_manifest_sha256"], **r["report"]}))
    else:
        r = build_patch(a.base, a.overlay, a.out)
        print(json.dumps({"out": str(a.out), "patch_sha256": file_sha(a.out / "patch.json"), **r["report"]}))


if __name__ == "__main__":
    main()
