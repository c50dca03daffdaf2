"""TITO session ledger v1: the exact token-in / token-out record of every served session, written by the server and
read back as training data (the format of the reference's ``training/src/arcforge/tito/ledger.py:1-120``; kept
alike so ledgers interchange; writer and reader here are this repository's own).

One instance directory ``DIR/<instance>/``:

* ``server.json``                {"instance", "ledger": {"logprob_dist": "raw_t1"}, ...}
* ``events.<n>.jsonl``           one event per line, files numbered from 0 with no holes
* ``routing.<n>.bin``            concatenated routing arrays (dtype / shape in the events)
* ``topk.<n>.bin``               per append ``<i4 ids [n,k] | <f2 lp [n,k] | <f4 tail [n] | u1 flags [n]``

Events: ``seg_open {sid, seg, t, cause}``, ``append {sid, seg, k, rid, t0, t1, prefix_len, tail, gen, finish,
stop_substituted, rewind, sampling, usage, replay, media, logprobs, routing, [top_logprobs]}``, ``seg_close {sid, seg,
t, reason, n_tokens, sha256}``, plus ``start`` / ``end`` / ``status`` / ``lossy``. Ids are base64 of little-endian
int32, logprobs base64 of float32.

Reconstruction of a segment's sequence S: ``S = S[:prefix_len] + tail + gen`` per append (``prefix_len + rewind ==
len(S)``, ``rewind <= len(previous gen)``). Checked invariants (codes as in the reference): ids_in_vocab,
append_order, prefix_len, rewind, finish, logprobs_len, topk_len, topk_file, routing_len, routing_file, close_len,
close_sha256, sid_mismatch, unknown_segment, duplicate_segment, closed_segment. Strict reading raises
``LedgerInvariantError``; non-strict marks the segment ``broken`` and keeps reading. Format errors (bad JSON, missing
keys, unknown events, holes in file numbers) always raise, except an unterminated last line of the last events file
(a live or crashed writer), which is skipped and recorded.
"""
from __future__ import annotations

import base64
import hashlib
import json
import os
import threading
import time
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

TOPK_LAYOUT = "ids_i4,lp_f2,tail_f4,flags_u1"
EVENT_KEYS = {
    "start": ("v", "instance", "t"),
    "seg_open": ("sid", "seg", "t", "cause"),
    "append": ("sid", "seg", "k", "rid", "t0", "t1", "prefix_len", "tail", "gen", "finish", "stop_substituted",
               "rewind", "sampling", "usage", "replay", "media", "logprobs", "routing"),
    "attempt": ("sid", "rid", "t", "kind", "input_len", "gen_len"),
    "seg_close": ("sid", "seg", "t", "reason", "n_tokens", "sha256"),
    "lossy": ("t", "dropped"),
    "status": ("t", "status"),
    "end": ("t", "status"),
}
ROUTING_KEYS = ("file", "offset", "nbytes", "start", "n_tokens", "shape", "dtype")
TOPK_KEYS = ("k", "n", "bytes", "file", "offset", "layout")


class LedgerFormatError(ValueError):
    pass


class LedgerInvariantError(ValueError):
    def __init__(self, code: str, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def b64_ids(ids) -> str:
    return base64.b64encode(np.asarray(ids, dtype="<i4").tobytes()).decode()


def b64_f32(x) -> str:
    return base64.b64encode(np.asarray(x, dtype="<f4").tobytes()).decode()


def _b64(value, dtype, where) -> np.ndarray:
    if not isinstance(value, str):
        raise LedgerFormatError(f"{where}: expected a base64 string")
    try:
        raw = base64.b64decode(value, validate=True)
    except ValueError as e:
        raise LedgerFormatError(f"{where}: bad base64") from e
    if len(raw) % np.dtype(dtype).itemsize:
        raise LedgerFormatError(f"{where}: {len(raw)} bytes is not a whole number of {dtype}")
    return np.frombuffer(raw, dtype=dtype).astype(dtype.lstrip("<"), copy=True)


def seq_sha256(ids) -> str:
    return hashlib.sha256(np.asarray(ids, dtype="<i4").tobytes()).hexdigest()


# ------------------------------------------------------------------------------------------------------- writer
class LedgerWriter:
    """Thread-safe writer of one instance directory. ``routing`` arrays ([n_tokens, layers, top_k] integers) and
    top-k blocks are appended to their sidecars before the event line that references them."""

    def __init__(self, root, instance: str | None = None, max_events_bytes: int = 64 << 20, meta: dict | None = None):
        self.instance = instance or f"afb-{os.getpid()}-{int(time.time())}"
        self.dir = Path(root) / self.instance
        self.dir.mkdir(parents=True, exist_ok=False)
        (self.dir / "server.json").write_text(json.dumps({"instance": self.instance,
                                                          "ledger": {"logprob_dist": "raw_t1"}, **(meta or {})}) + "\n")
        self.lock = threading.Lock()
        self.max_bytes = max_events_bytes
        self.n = 0
        self.f = open(self.dir / "events.0.jsonl", "a")
        self.next_seg = 0
        self.segments: dict[int, dict] = {}  # seg -> {sid, S, k, last_gen}
        self._emit({"ev": "start", "v": 1, "instance": self.instance, "t": time.time()})

    def _emit(self, ev: dict):
        line = json.dumps(ev, separators=(",", ":")) + "\n"
        if self.f.tell() + len(line) > self.max_bytes and self.f.tell() > 0:
            self.f.close()
            self.n += 1
            self.f = open(self.dir / f"events.{self.n}.jsonl", "a")
        self.f.write(line)
        self.f.flush()

    def _sidecar(self, kind: str, raw: bytes) -> tuple[str, int]:
        name = f"{kind}.{self.n}.bin"
        p = self.dir / name
        offset = p.stat().st_size if p.exists() else 0
        with open(p, "ab") as f:
            f.write(raw)
        return name, offset

    def open_segment(self, sid: str | None, cause: str = "new") -> int:
        with self.lock:
            seg = self.next_seg
            self.next_seg += 1
            self.segments[seg] = {"sid": sid, "S": [], "k": 0, "last_gen": 0}
            self._emit({"ev": "seg_open", "sid": sid, "seg": seg, "t": time.time(),
                        "cause": "single" if sid is None else cause})
            return seg

    def append(self, seg: int, rid: str, tail, gen, finish: dict, logprobs=None, routing=None, topk=None,
               rewind: int = 0, usage: dict | None = None, t0: float | None = None):
        """One request of the segment: ``tail`` new input tokens after the kept prefix, ``gen`` sampled tokens
        (with the stop token), ``logprobs`` [len(gen)] of the sampled tokens, ``routing`` [n, layers, top_k] ints of
        the forwarded positions [max(prefix_len - 1, 0), prefix_len + len(tail) + len(gen) - 1) (the turn's last
        sampled token is forwarded in the next turn), ``topk`` (ids [n,k], lp [n,k], tail [n], flags [n]) over the
        gen tokens."""
        with self.lock:
            st = self.segments[seg]
            S = st["S"]
            prefix = len(S) - rewind
            if rewind > st["last_gen"] or prefix < 0:
                raise ValueError("rewind reaches past the previous generation")
            tail, gen = [int(x) for x in tail], [int(x) for x in gen]
            ev = {"ev": "append", "sid": st["sid"], "seg": seg, "k": st["k"], "rid": rid,
                  "t0": t0 if t0 is not None else time.time(), "t1": time.time(), "prefix_len": prefix,
                  "tail": b64_ids(tail), "gen": b64_ids(gen), "finish": finish, "stop_substituted": False,
                  "rewind": rewind, "sampling": None, "usage": usage, "replay": None, "media": [],
                  "logprobs": None if logprobs is None else b64_f32(logprobs), "routing": None}
            if routing is not None:
                r = np.ascontiguousarray(routing)
                name, off = self._sidecar("routing", r.tobytes())
                ev["routing"] = {"file": name, "offset": off, "nbytes": r.nbytes, "start": max(prefix - 1, 0),
                                 "n_tokens": int(r.shape[0]), "shape": list(r.shape), "dtype": r.dtype.str}
            if topk is not None:
                ids, lp, tl, flags = topk
                ids = np.asarray(ids, dtype="<i4")
                n, k = ids.shape
                raw = (ids.tobytes() + np.asarray(lp, dtype="<f2").tobytes() + np.asarray(tl, dtype="<f4").tobytes()
                       + np.asarray(flags, dtype="u1").tobytes())
                name, off = self._sidecar("topk", raw)
                ev["top_logprobs"] = {"k": k, "n": n, "bytes": len(raw), "file": name, "offset": off,
                                      "layout": TOPK_LAYOUT}
            self._emit(ev)
            st["S"] = S[:prefix] + tail + gen
            st["k"] += 1
            st["last_gen"] = len(gen)

    def close_segment(self, seg: int, reason: str = "closed"):
        with self.lock:
            st = self.segments.pop(seg)
            self._emit({"ev": "seg_close", "sid": st["sid"], "seg": seg, "t": time.time(),
                        "reason": "single" if st["sid"] is None else reason, "n_tokens": len(st["S"]),
                        "sha256": seq_sha256(st["S"])})

    def close(self):
        with self.lock:
            for seg in list(self.segments):
                st = self.segments.pop(seg)
                self._emit({"ev": "seg_close", "sid": st["sid"], "seg": seg, "t": time.time(), "reason": "shutdown",
                            "n_tokens": len(st["S"]), "sha256": seq_sha256(st["S"])})
            self._emit({"ev": "end", "t": time.time(), "status": {}})
            self.f.close()


# ------------------------------------------------------------------------------------------------------- reader
@dataclass
class Append:
    k: int
    rid: str
    prefix_len: int
    rewind: int
    tail: np.ndarray
    gen: np.ndarray
    finish: dict
    logprobs: np.ndarray | None
    routing: dict | None
    topk: dict | None

    @property
    def gen_start(self) -> int:
        return self.prefix_len + len(self.tail)


@dataclass
class Segment:
    seg: int
    sid: str | None
    cause: str
    appends: list[Append] = field(default_factory=list)
    S: list[int] = field(default_factory=list)
    status: str = "open"            # open (no seg_close: server crash), closed, broken
    error: str | None = None
    close: dict | None = None


@dataclass
class Instance:
    path: Path
    server: dict
    segments: dict[int, Segment]
    truncated_tail: bool = False
    skipped_events: int = 0


class _Reader:
    def __init__(self, path: Path, id_bound: int, strict: bool):
        self.path, self.id_bound, self.strict = path, id_bound, strict
        self.segments: dict[int, Segment] = {}
        self.closed: set[int] = set()
        self.skipped = 0

    def fail(self, seg: Segment | None, code: str, where: str, msg: str):
        if self.strict or seg is None:
            raise LedgerInvariantError(code, f"{where}: {msg}")
        seg.status, seg.error = "broken", f"[{code}] {where}: {msg}"

    def event(self, ev: dict, where: str):
        kind = ev["ev"]
        if kind == "seg_open":
            s = int(ev["seg"])
            if s in self.segments:
                return self.fail(None, "duplicate_segment", where, f"segment {s} opened twice")
            self.segments[s] = Segment(s, ev["sid"], ev["cause"])
            return
        if kind not in ("append", "seg_close"):
            return
        s = int(ev["seg"])
        seg = self.segments.get(s)
        if seg is None:
            return self.fail(None, "unknown_segment", where, f"segment {s} was never opened")
        if seg.status == "broken":
            self.skipped += 1
            return
        if s in self.closed:
            return self.fail(seg, "closed_segment", where, f"event after segment {s} closed")
        if ev["sid"] != seg.sid:
            return self.fail(seg, "sid_mismatch", where, f"sid {ev['sid']!r} != {seg.sid!r}")
        if kind == "seg_close":
            if int(ev["n_tokens"]) != len(seg.S):
                return self.fail(seg, "close_len", where, f"n_tokens {ev['n_tokens']} != {len(seg.S)}")
            if ev["sha256"] != seq_sha256(seg.S):
                return self.fail(seg, "close_sha256", where, "sha256 of S differs")
            seg.close = {"reason": ev["reason"], "n_tokens": len(seg.S)}
            seg.status = "closed"
            self.closed.add(s)
            return
        k, prefix, rewind = int(ev["k"]), int(ev["prefix_len"]), int(ev["rewind"])
        tail, gen = _b64(ev["tail"], "<i4", f"{where} tail"), _b64(ev["gen"], "<i4", f"{where} gen")
        for name, arr in (("tail", tail), ("gen", gen)):
            if arr.size and (int(arr.min()) < 0 or int(arr.max()) >= self.id_bound):
                return self.fail(seg, "ids_in_vocab", where, f"{name} has ids outside [0, {self.id_bound})")
        if k != len(seg.appends):
            return self.fail(seg, "append_order", where, f"k={k} after {len(seg.appends)} records")
        if k == 0 and (prefix != 0 or rewind != 0):
            return self.fail(seg, "prefix_len", where, "the first record needs prefix_len = rewind = 0")
        if k > 0 and prefix + rewind != len(seg.S):
            return self.fail(seg, "prefix_len", where, f"prefix_len {prefix} + rewind {rewind} != len(S) {len(seg.S)}")
        if k > 0 and rewind > len(seg.appends[-1].gen):
            return self.fail(seg, "rewind", where, "rewind reaches past the previous generation")
        fin = ev["finish"]
        if not isinstance(fin, dict) or fin.get("type") not in ("stop", "length", "abort"):
            return self.fail(seg, "finish", where, f"finish {fin!r}")
        if fin.get("type") == "stop" and isinstance(fin.get("matched"), int) and (not gen.size or
                                                                                 int(gen[-1]) != fin["matched"]):
            return self.fail(seg, "finish", where, "the last gen token is not the matched stop token")
        lp = None
        if ev["logprobs"] is not None:
            lp = _b64(ev["logprobs"], "<f4", f"{where} logprobs")
            if lp.size != gen.size or np.isnan(lp).any():
                return self.fail(seg, "logprobs_len", where, f"{lp.size} logprobs for {gen.size} gen tokens")
        routing = ev["routing"]
        if routing is not None:
            if any(x not in routing for x in ROUTING_KEYS):
                raise LedgerFormatError(f"{where}: routing misses keys")
            shp = routing["shape"]
            end = prefix + len(tail) + len(gen) - 1  # the turn's last sampled token is forwarded next turn
            if len(shp) != 3 or shp[0] != routing["n_tokens"] or routing["start"] + routing["n_tokens"] != end:
                return self.fail(seg, "routing_len", where, f"routing rows [{routing['start']}, +{shp[0]}) vs end {end}")
            item = np.dtype(routing["dtype"]).itemsize
            fp = self.path / routing["file"]
            if (np.dtype(routing["dtype"]).kind not in "iu" or routing["nbytes"] != int(np.prod(shp)) * item
                    or not fp.is_file() or routing["offset"] + routing["nbytes"] > fp.stat().st_size):
                return self.fail(seg, "routing_file", where, "routing sidecar cannot hold the record")
        topk = ev.get("top_logprobs")
        if topk is not None:
            if topk["n"] != gen.size or topk["k"] < 1:
                return self.fail(seg, "topk_len", where, f"top_logprobs n={topk['n']} for {gen.size} gen tokens")
            fp = self.path / topk["file"]
            if (topk["layout"] != TOPK_LAYOUT or topk["bytes"] != topk["n"] * topk["k"] * 6 + topk["n"] * 5
                    or not fp.is_file() or topk["offset"] + topk["bytes"] > fp.stat().st_size):
                return self.fail(seg, "topk_file", where, "top-k sidecar does not hold the record")
        seg.S = seg.S[:prefix] + tail.tolist() + gen.tolist()
        seg.appends.append(Append(k, ev["rid"], prefix, rewind, tail, gen, fin, lp, routing, topk))


def read_instance(path, id_bound: int, strict: bool = True) -> Instance:
    path = Path(path)
    if not (path / "server.json").is_file():
        raise LedgerFormatError(f"{path}: no server.json")
    server = json.loads((path / "server.json").read_text())
    files = sorted(path.glob("events.*.jsonl"), key=lambda p: int(p.name.split(".")[1]))
    if [int(p.name.split(".")[1]) for p in files] != list(range(len(files))):
        raise LedgerFormatError(f"{path}: events files are not numbered 0..n-1")
    rd = _Reader(path, id_bound, strict)
    truncated = False
    for fi, fp in enumerate(files):
        data = fp.read_text()
        lines = data.split("\n")
        unterminated = lines[-1] != ""
        if unterminated and fi != len(files) - 1:
            raise LedgerFormatError(f"{fp}: unterminated line in a file that is not the last")
        for li, line in enumerate(lines[:-1] if not unterminated else lines):
            if unterminated and li == len(lines) - 1:
                truncated = True  # a writer that is live or died mid-line
                break
            if not line:
                continue
            where = f"{fp.name}:{li + 1}"
            try:
                ev = json.loads(line)
            except json.JSONDecodeError as e:
                raise LedgerFormatError(f"{where}: bad JSON") from e
            if ev.get("ev") not in EVENT_KEYS:
                raise LedgerFormatError(f"{where}: unknown event {ev.get('ev')!r}")
            miss = [k for k in EVENT_KEYS[ev["ev"]] if k not in ev]
            if miss:
                raise LedgerFormatError(f"{where}: missing keys {miss}")
            rd.event(ev, where)
    return Instance(path, server, rd.segments, truncated, rd.skipped)


# ------------------------------------------------------------------------------------------------------- exports
def routing_rows(inst: Instance, a: Append) -> np.ndarray | None:
    if a.routing is None:
        return None
    r = a.routing
    with open(inst.path / r["file"], "rb") as f:
        f.seek(r["offset"])
        raw = f.read(r["nbytes"])
    return np.frombuffer(raw, dtype=np.dtype(r["dtype"])).reshape(r["shape"])


def rl_examples(seg: Segment) -> list[dict]:
    """One example per append: ids = S up to the end of that append's gen, trained positions = its gen tokens, with
    their sampling log-probabilities (``behavior_logp``) when the ledger has them."""
    out, S = [], []
    for a in seg.appends:
        S = S[:a.prefix_len] + a.tail.tolist() + a.gen.tolist()
        n = len(S)
        g0 = a.gen_start
        mask = [0] * n
        beh = [0.0] * n
        for j in range(g0, n):
            mask[j] = 1
            if a.logprobs is not None:
                beh[j] = float(a.logprobs[j - g0])
        out.append({"ids": list(S), "gen_mask": mask,
                    "behavior_logp": beh if a.logprobs is not None else None, "rid": a.rid})
    return out


def sft_examples(inst: Instance, closed_only: bool = True) -> list[dict]:
    """Final sequence of every (closed) segment with its generated tokens as the loss mask (``train/sft.py`` input)."""
    out = []
    for seg in inst.segments.values():
        if seg.status == "broken" or (closed_only and seg.status != "closed") or not seg.appends:
            continue
        mask = [0] * len(seg.S)
        for i, a in enumerate(seg.appends):
            # a later append that rewound keeps only the part of this generation before its prefix_len
            end = a.gen_start + len(a.gen)
            if i + 1 < len(seg.appends):
                end = min(end, seg.appends[i + 1].prefix_len)
            for j in range(a.gen_start, min(end, len(seg.S))):
                mask[j] = 1
        out.append({"ids": list(seg.S), "loss_mask": mask})
    return out
