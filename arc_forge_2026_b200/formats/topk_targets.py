"""``qad-topk-v1``: teacher top-k targets aligned to a dataset's supervised positions.

Layout (the reference's contract, ``training/work/qwen38fn_qad/topk_targets.py:1-30``)::

    <root>/topk.json              format, k, source, teacher, per-split row counts and hashes
    <root>/<split>/ids.i32        [N, k] token ids, best first
    <root>/<split>/lp.f16         [N, k] log-probs normalised over the full vocabulary (T = 1)
    <root>/<split>/tail.f32       [N]    log(1 - sum exp(lp)); -inf when no mass is left
    <root>/<split>/flags.u8       [N]    bits of logit processing (0 = natural); flagged rows leave the loss
    <root>/<split>/labels.i32     [N]    the supervised token, for the alignment check
    <root>/<split>/DONE           summary JSON, written last; readers refuse a split without it

Reading renormalises the (k + 1)-class teacher in fp32 (f16 log-probs plus the tail miss 1 by ~1e-3).
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import torch

FORMAT = "qad-topk-v1"
FILES = {"ids": ("ids.i32", "<i4", True), "lp": ("lp.f16", "<f2", True), "tail": ("tail.f32", "<f4", False),
         "flags": ("flags.u8", "u1", False), "labels": ("labels.i32", "<i4", False)}


def _sha(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


class TopKWriter:
    """Append rows of one split, then ``close()`` writes DONE (atomic publication of the split)."""

    def __init__(self, root: Path, split: str, k: int):
        self.root, self.split, self.k = Path(root), split, k
        self.dir = self.root / split
        if (self.dir / "DONE").exists():
            raise FileExistsError(self.dir / "DONE")
        self.dir.mkdir(parents=True, exist_ok=True)
        self.handles = {name: open(self.dir / fn, "wb") for name, (fn, _, _) in FILES.items()}
        self.rows = 0

    def append(self, ids, lp, tail, labels, flags=None):
        n = ids.shape[0]
        if ids.shape[1] != self.k or lp.shape != ids.shape:
            raise ValueError("rows must be [n, k]")
        arrs = {"ids": ids.to(torch.int32).cpu().numpy().astype("<i4"),
                "lp": lp.to(torch.float16).cpu().numpy().astype("<f2"),
                "tail": tail.to(torch.float32).cpu().numpy().astype("<f4"),
                "flags": (flags if flags is not None else torch.zeros(n, dtype=torch.uint8)).cpu().numpy().astype("u1"),
                "labels": labels.to(torch.int32).cpu().numpy().astype("<i4")}
        for name, a in arrs.items():
            self.handles[name].write(np.ascontiguousarray(a).tobytes())
        self.rows += n

    def close(self, meta: dict | None = None):
        for h in self.handles.values():
            h.close()
        summary = {"rows": self.rows, "k": self.k,
                   "sha256": {fn: _sha(self.dir / fn) for fn, _, _ in FILES.values()}}
        tmp = self.dir / "DONE.tmp"
        tmp.write_text(json.dumps(summary) + "\n")
        tmp.rename(self.dir / "DONE")
        top = self.root / "topk.json"
        doc = json.loads(top.read_text()) if top.exists() else {"format": FORMAT, "k": self.k, "splits": {}}
        doc.update(meta or {})
        doc["splits"][self.split] = summary
        t2 = self.root / "topk.json.tmp"
        t2.write_text(json.dumps(doc, indent=1) + "\n")
        t2.rename(top)
        return summary


class TopKReader:
    def __init__(self, root: Path, split: str):
        self.root, self.dir = Path(root), Path(root) / split
        done = self.dir / "DONE"
        if not done.exists():
            raise FileNotFoundError(f"{self.dir}: split not published (no DONE)")
        doc = json.loads((self.root / "topk.json").read_text())
        if doc.get("format") != FORMAT:
            raise ValueError(f"{self.root}: format {doc.get('format')!r}, expected {FORMAT}")
        self.k = int(doc["k"])
        self.rows = int(json.loads(done.read_text())["rows"])
        self.arr = {}
        for name, (fn, dt, two_d) in FILES.items():
            a = np.memmap(self.dir / fn, dtype=dt, mode="r")
            self.arr[name] = a.reshape(self.rows, self.k) if two_d else a

    def rows_slice(self, start: int, end: int, device="cpu"):
        """Rows [start, end): ids int64, lp fp32 and tail fp32 renormalised to a (k+1)-class distribution,
        labels, and the keep mask (flags == 0)."""
        ids = torch.from_numpy(np.array(self.arr["ids"][start:end])).long()
        lp = torch.from_numpy(np.array(self.arr["lp"][start:end]).astype(np.float32))
        tail = torch.from_numpy(np.array(self.arr["tail"][start:end]).astype(np.float32))
        logz = torch.logsumexp(torch.cat([lp, tail[:, None]], 1), 1)
        out = {"ids": ids, "lp": lp - logz[:, None], "tail": tail - logz,
               "labels": torch.from_numpy(np.array(self.arr["labels"][start:end])).long(),
               "keep": torch.from_numpy(np.array(self.arr["flags"][start:end]) == 0)}
        return {k: v.to(device) for k, v in out.items()}


def synthetic_targets(n: int, k: int, vocab: int, generator: torch.Generator, device="cpu"):
    """Random but valid teacher targets: distinct ids per row, normalised (k+1)-class log-probs."""
    z = torch.randn(n, k + 1, generator=generator) * 2.0
    lp_all = torch.log_softmax(z, -1)
    ids = torch.stack([torch.randperm(vocab, generator=generator)[:k] for _ in range(min(n, 64))])
    ids = ids.repeat((n + ids.shape[0] - 1) // ids.shape[0], 1)[:n]
    return {"ids": ids.to(device), "lp": lp_all[:, :k].contiguous().to(device),
            "tail": lp_all[:, k].contiguous().to(device)}
