"""OpenAI-compatible HTTP server over a serving engine (the GPU ``SpecEngine`` or the CPU reference engine).

Routes (the surface the reference's agents use through its sglang fork: chat/completions, the Responses API with
server-side sessions and ``/close_session``, usage accounting):

    GET  /health                 liveness
    GET  /v1/models              the served model
    POST /v1/completions         {"prompt": str | [int], "max_tokens", "stream", "images"?}; "images" (an extension):
                                 [{"pixels": processor patches [P][patch_dim], "grid_thw": [t, h, w]}] for the
                                 prompt's image-token runs, served by an engine with a vision tower
    POST /v1/chat/completions    {"messages": [...], "max_tokens", "stream"}
    POST /v1/responses           {"input": str | [messages], "session_id"?, "max_output_tokens", "stream"}
                                 a session keeps its transcript (and, on engines that can extend a session, its
                                 KV / recurrent state) until /close_session
    POST /close_session          {"session_id"}
    POST /abort_request          {"rid"}: stop a queued or running request (its response ends with finish_reason
                                 "abort"); generation routes accept an optional "rid" to name the request
    POST /update_weights_from_disk {"model_path"}: load new weights between engine steps, in place (a deploy
                                 package for the native engine, a state-dict file for the CPU engine)
    GET  /metrics                Prometheus text (requests, tokens, active sessions, step latency)

With ``--session-ledger DIR`` every request is recorded in a TITO session ledger (``formats/tito.py``): a
Responses-API session is one segment (each turn appends its new input tokens and its generated tokens; /close_session
closes it), any other request a single-append segment.

One engine thread owns the engine: it admits queued requests when a session slot is free, runs ``engine.step()``
while any request is live and hands emitted tokens to the waiting HTTP handlers through their event loops.

    python -m arc_forge_2026_b200.serve.server --preset tiny_cpu --port 8000          # CPU reference engine
    python -m arc_forge_2026_b200.serve.server --preset tiny_gpu --gpu --port 8000    # native engine
"""
from __future__ import annotations

import argparse
import asyncio
import collections
import itertools
import json
import threading
import time
import uuid
from dataclasses import dataclass, field

from .tokenizer import ByteTokenizer


@dataclass
class Request:
    prompt: list[int]
    max_new: int
    loop: asyncio.AbstractEventLoop
    queue: asyncio.Queue
    session_key: str | None = None
    extend: list[int] | None = None   # continuation tokens for an existing session
    sid: int = -1
    n_out: int = 0
    t0: float = field(default_factory=time.perf_counter)
    rid: str = ""
    aborted: bool = False
    out: list = field(default_factory=list)
    images: list | None = None         # [(pixels [P, patch_dim], (t, h, w))] for the prompt's image tokens


class EngineLoop:
    """Runs the engine on one thread; requests come in through ``submit`` and tokens go out per request."""

    def __init__(self, engine, eos_id: int | None = None, metrics=None, ledger=None):
        self.engine = engine
        self.ledger = ledger                      # formats.tito.LedgerWriter or None
        self.ledger_segs: dict[str, int] = {}     # session_id -> open ledger segment
        self.eos_id = eos_id
        self.metrics = metrics
        self.cv = threading.Condition()
        self.pending: collections.deque[Request] = collections.deque()
        self.live: dict[int, Request] = {}
        self.keyed: dict[str, int] = {}          # session_id -> engine sid (kept until /close_session)
        self.transcripts: dict[str, list[int]] = {}
        self.by_rid: dict[str, Request] = {}
        self.commands: collections.deque = collections.deque()  # (fn, concurrent Future) run between steps
        self._sids = itertools.count(1)
        self._stop = False
        self.thread = threading.Thread(target=self._run, name="afb-engine", daemon=True)
        self.thread.start()

    def submit(self, req: Request):
        with self.cv:
            self.pending.append(req)
            if req.rid:
                self.by_rid[req.rid] = req
            self.cv.notify()

    def abort(self, rid: str) -> bool:
        """Queued: dropped now; running: finished by the engine thread before its next step."""
        with self.cv:
            req = self.by_rid.get(rid)
            if req is None:
                return False
            req.aborted = True
            if req in self.pending:
                self.pending.remove(req)
                self.by_rid.pop(rid, None)
                self._emit(req, ("done", "abort"))
            self.cv.notify()
            return True

    def call(self, fn):
        """Run ``fn(engine)`` on the engine thread between steps; returns a concurrent future."""
        import concurrent.futures
        fut = concurrent.futures.Future()
        with self.cv:
            self.commands.append((fn, fut))
            self.cv.notify()
        return fut

    def close_session(self, key: str) -> bool:
        with self.cv:
            sid = self.keyed.pop(key, None)
            self.transcripts.pop(key, None)
            seg = self.ledger_segs.pop(key, None)
            if seg is not None:
                self.ledger.close_segment(seg)
            has = (self.engine.has_session(sid) if hasattr(self.engine, "has_session")
                   else sid in self.engine.sessions)
            if sid is not None and sid not in self.live and has:
                self.engine.release(sid)
            return sid is not None

    def shutdown(self):
        with self.cv:
            self._stop = True
            self.cv.notify()
        self.thread.join(timeout=10)

    # ---------------------------------------------------------------- engine thread
    def _emit(self, req: Request, item):
        req.loop.call_soon_threadsafe(req.queue.put_nowait, item)

    def _admit(self, req: Request):
        eng = self.engine
        key = req.session_key
        try:
            if key is not None and key in self.keyed:
                sid = self.keyed[key]
                if hasattr(eng, "continue_session") and eng.has_session(sid):
                    # only the tokens after the committed state are prefilled (a parked session is restored first)
                    sess = eng.continue_session(sid, self.transcripts[key] + (req.extend or []), req.max_new)
                elif hasattr(eng, "extend_session") and sid in eng.sessions:
                    sess = eng.extend_session(sid, req.extend or [], req.max_new)
                else:  # engine without continuation: re-prefill the whole transcript
                    if sid in eng.sessions:
                        eng.release(sid)
                    sess = eng.add_session(sid, self.transcripts[key] + (req.extend or []), req.max_new)
            else:
                sid = next(self._sids)
                if req.images:
                    if getattr(eng, "vision", None) is None:
                        raise ValueError("this engine has no vision tower: image prompts are not served")
                    sess = eng.add_session(sid, req.prompt, req.max_new, images=req.images)
                else:
                    sess = eng.add_session(sid, req.prompt, req.max_new)
                if key is not None:
                    self.keyed[key] = sid
        except Exception as e:  # noqa: BLE001 - reported to the client
            self._emit(req, ("error", str(e)))
            return
        req.sid = sid
        self.live[sid] = req
        self._deliver(req, list(sess.generated))

    def _deliver(self, req: Request, toks: list[int]):
        for t in toks:
            if req.n_out >= req.max_new:
                break
            req.n_out += 1
            req.out.append(int(t))
            self._emit(req, ("token", t))
            if self.metrics:
                self.metrics["tokens"].inc()
            if self.eos_id is not None and t == self.eos_id:
                req.n_out = req.max_new
                break
        if req.n_out >= req.max_new:
            self._finish(req)

    def _record(self, req: Request, reason: str | None):
        """The request's tokens into the session ledger (the tail: this turn's new input tokens)."""
        lg = self.ledger
        if lg is None:
            return
        stop = self.eos_id is not None and req.out and req.out[-1] == self.eos_id
        fin = {"type": "abort" if reason == "abort" else ("stop" if stop else "length")}
        if stop:
            fin["matched"] = int(self.eos_id)
        if req.session_key is None:
            seg = lg.open_segment(None)
            lg.append(seg, req.rid, req.prompt, req.out, fin, t0=None)
            lg.close_segment(seg)
            return
        seg = self.ledger_segs.get(req.session_key)
        first = seg is None
        if first:
            seg = self.ledger_segs[req.session_key] = lg.open_segment(req.session_key)
        lg.append(seg, req.rid, req.prompt if first else (req.extend or []), req.out, fin)

    def _finish(self, req: Request, reason: str | None = None):
        self.live.pop(req.sid, None)
        self.by_rid.pop(req.rid, None)
        self._record(req, reason)
        eng = self.engine
        if req.session_key is None:
            if req.sid in eng.sessions:
                eng.release(req.sid)
        else:
            s = eng.sessions.get(req.sid)
            if s is not None:
                self.transcripts[req.session_key] = list(s.prompt) + list(s.generated)
                s.done = True
                s.last_used = time.monotonic()
                if hasattr(s, "row") and hasattr(eng, "active"):
                    eng.active[s.row] = 0  # keep the session's pages, stop decoding it
        self._emit(req, ("done", reason))
        if self.metrics:
            self.metrics["latency"].observe(time.perf_counter() - req.t0)

    def _run(self):
        while True:
            with self.cv:
                while not self._stop and not self.pending and not self.live and not self.commands:
                    self.cv.wait()
                if self._stop:
                    return
                commands = list(self.commands)
                self.commands.clear()
                aborted = [r for r in self.live.values() if r.aborted]
            for fn, fut in commands:
                try:
                    fut.set_result(fn(self.engine))
                except Exception as e:  # noqa: BLE001 - reported to the caller
                    fut.set_exception(e)
            for req in aborted:
                self._finish(req, "abort")
            with self.cv:
                admit = []
                free = self._free_slots()
                while self.pending:
                    req = self.pending[0]
                    reuse = req.session_key is not None and req.session_key in self.keyed
                    # a keyed session keeps its row between turns unless it was parked
                    held = reuse and self.keyed[req.session_key] in getattr(self.engine, "sessions", {})
                    if not held and free <= 0:
                        break
                    admit.append(self.pending.popleft())
                    free -= 1  # a new / parked session takes a row; a held idle one stops counting as parkable
            for req in admit:
                self._admit(req)
            if self.live:
                t0 = time.perf_counter()
                out = self.engine.step()
                if self.metrics:
                    self.metrics["step"].observe(time.perf_counter() - t0)
                for sid, toks in out.items():
                    req = self.live.get(sid)
                    if req is not None:
                        self._deliver(req, toks)
                for sid, req in list(self.live.items()):  # engine-side completion (its own max_new)
                    s = self.engine.sessions.get(sid)
                    if s is not None and s.done and req.n_out < req.max_new:
                        self._finish(req)
            if self.metrics:
                self.metrics["active"].set(len(self.live))
            if not self.live and self.pending and not admit:
                time.sleep(0.001)  # full: wait for a slot

    def _free_slots(self) -> int:
        eng = self.engine
        if hasattr(eng, "free_slots"):
            return eng.free_slots
        if hasattr(eng, "free_rows"):
            return len(eng.free_rows)
        return 1


def _metrics():
    from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram
    reg = CollectorRegistry()
    return reg, {
        "requests": Counter("afb_requests_total", "HTTP generation requests", ["route"], registry=reg),
        "tokens": Counter("afb_generated_tokens_total", "tokens sent to clients", registry=reg),
        "active": Gauge("afb_active_requests", "requests being decoded", registry=reg),
        "step": Histogram("afb_engine_step_seconds", "engine.step() wall time", registry=reg),
        "latency": Histogram("afb_request_seconds", "request wall time", registry=reg),
    }


def create_app(engine, tokenizer=None, model_name: str = "arc-forge-b200", ledger=None):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    tok = tokenizer or ByteTokenizer()
    registry, metrics = _metrics()
    loop_ = EngineLoop(engine, getattr(tok, "eos_id", None), metrics, ledger)
    from contextlib import asynccontextmanager

    @asynccontextmanager
    async def lifespan(_app):
        yield
        loop_.shutdown()
        if ledger is not None:
            ledger.close()

    app = FastAPI(title="arc_forge_2026_b200", lifespan=lifespan)
    app.state.engine_loop = loop_

    async def _generate(prompt, max_new, key=None, extend=None, rid=None, state=None, images=None):
        loop = asyncio.get_running_loop()
        req = Request(prompt, max_new, loop, asyncio.Queue(), key, extend, rid=rid or "", images=images)
        loop_.submit(req)
        while True:
            kind, val = await req.queue.get()
            if kind == "error":
                raise HTTPException(400, val)
            if kind == "done":
                if state is not None and val:
                    state["reason"] = val
                return
            yield val

    def _reason(state, n, max_new):
        return state.get("reason") or ("length" if n >= max_new else "stop")

    async def _collect(gen):
        return [t async for t in gen]

    def _usage(p, c):
        return {"prompt_tokens": p, "completion_tokens": c, "total_tokens": p + c}

    def _sse(chunks):
        async def body():
            async for c in chunks:
                yield f"data: {json.dumps(c)}\n\n"
            yield "data: [DONE]\n\n"
        return StreamingResponse(body(), media_type="text/event-stream")

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "arc_forge_2026_b200"}]}

    @app.get("/metrics")
    async def prom():
        from prometheus_client import generate_latest
        return PlainTextResponse(generate_latest(registry).decode())

    @app.post("/v1/completions")
    async def completions(body: dict):
        metrics["requests"].labels("completions").inc()
        prompt = body.get("prompt", "")
        ids = list(prompt) if isinstance(prompt, list) else tok.encode(prompt)
        max_new = int(body.get("max_tokens", 16))
        rid = body.get("rid") or "cmpl-" + uuid.uuid4().hex[:24]
        st = {}
        # images (an extension of this server): the processor's flattened patches and grid of each image, in the
        # order of the prompt's image-token runs
        images = [(im["pixels"], tuple(int(x) for x in im["grid_thw"])) for im in body.get("images") or []] or None
        if body.get("stream"):
            async def chunks():
                async for t in _generate(ids, max_new, rid=rid, state=st, images=images):
                    yield {"id": rid, "object": "text_completion", "model": model_name,
                           "choices": [{"index": 0, "text": tok.decode([t]), "token_ids": [t], "finish_reason": None}]}
            return _sse(chunks())
        out = await _collect(_generate(ids, max_new, rid=rid, state=st, images=images))
        return {"id": rid, "object": "text_completion", "created": int(time.time()), "model": model_name,
                "choices": [{"index": 0, "text": tok.decode(out), "token_ids": out,
                             "finish_reason": _reason(st, len(out), max_new)}],
                "usage": _usage(len(ids), len(out))}

    @app.post("/v1/chat/completions")
    async def chat(body: dict):
        metrics["requests"].labels("chat").inc()
        ids = tok.chat(body.get("messages", []))
        max_new = int(body.get("max_tokens", body.get("max_completion_tokens", 16)))
        rid = body.get("rid") or "chatcmpl-" + uuid.uuid4().hex[:24]
        st = {}
        if body.get("stream"):
            async def chunks():
                async for t in _generate(ids, max_new, rid=rid, state=st):
                    yield {"id": rid, "object": "chat.completion.chunk", "model": model_name,
                           "choices": [{"index": 0, "delta": {"content": tok.decode([t])}, "finish_reason": None}]}
            return _sse(chunks())
        out = await _collect(_generate(ids, max_new, rid=rid, state=st))
        return {"id": rid, "object": "chat.completion", "created": int(time.time()), "model": model_name,
                "choices": [{"index": 0, "message": {"role": "assistant", "content": tok.decode(out)},
                             "finish_reason": _reason(st, len(out), max_new)}],
                "usage": _usage(len(ids), len(out))}

    @app.post("/v1/responses")
    async def responses(body: dict):
        metrics["requests"].labels("responses").inc()
        inp = body.get("input", "")
        msgs = [{"role": "user", "content": inp}] if isinstance(inp, str) else list(inp)
        key = body.get("session_id")
        max_new = int(body.get("max_output_tokens", 16))
        rid = body.get("rid") or "resp_" + uuid.uuid4().hex[:24]
        st = {}
        if key is not None and key in loop_.keyed:
            ext = tok.encode("".join(f"<|{m.get('role', 'user')}|>{m.get('content', '')}\n" for m in msgs)
                             + "<|assistant|>") if isinstance(tok, ByteTokenizer) else tok.chat(msgs)
            prompt_len = len(loop_.transcripts.get(key, [])) + len(ext)
            gen = _generate([], max_new, key, ext, rid=rid, state=st)
        else:
            ids = tok.chat(msgs)
            prompt_len = len(ids)
            gen = _generate(ids, max_new, key, rid=rid, state=st)
        out = await _collect(gen)
        text = tok.decode(out)
        return {"id": rid, "object": "response", "created_at": int(time.time()),
                "model": model_name, "status": "incomplete" if st.get("reason") == "abort" else "completed",
                "session_id": key,
                "output": [{"type": "message", "role": "assistant",
                            "content": [{"type": "output_text", "text": text}]}],
                "output_text": text,
                "usage": {"input_tokens": prompt_len, "output_tokens": len(out),
                          "total_tokens": prompt_len + len(out)}}

    @app.post("/close_session")
    async def close_session(body: dict):
        key = body.get("session_id")
        if key is None:
            raise HTTPException(400, "session_id is required")
        return JSONResponse({"session_id": key, "closed": loop_.close_session(key)})

    @app.post("/abort_request")
    async def abort_request(body: dict):
        rid = body.get("rid")
        if not rid:
            raise HTTPException(400, "rid is required")
        return {"rid": rid, "aborted": loop_.abort(rid)}

    @app.post("/update_weights_from_disk")
    async def update_weights(body: dict):
        path = body.get("model_path")
        if not path:
            raise HTTPException(400, "model_path is required")
        fut = loop_.call(lambda eng: eng.update_weights(path))
        try:
            info = await asyncio.wrap_future(fut)
        except Exception as e:  # noqa: BLE001 - reported to the client
            return JSONResponse({"success": False, "message": str(e)}, status_code=400)
        return {"success": True, "message": "weights updated", **(info or {})}

    return app


def _build_engine(args):
    """The serving engine of the command line (the reference's B200 launch script,
    ``training/work/qwen38fn_eval/serve_qwen38fn_0520.sh:1-80``): a deploy package (``--package``) or random-init
    weights of ``--preset``; a drafter directory (``--drafter-dir``) or a random drafter of ``--drafter``; the
    speculative width, acceptance rule, KV / QSA / HiSparse options."""
    import torch
    from ..config import ServeConfig, drafter_preset, preset
    if args.package and not args.gpu:
        raise SystemExit("--package needs --gpu (the CPU engine serves the fp32 oracle of a preset)")
    cfg = preset(args.preset)
    if not args.gpu:
        from ..models.reference import build_reference
        from .cpu_engine import CPUEngine
        return CPUEngine(build_reference(cfg, seed=args.seed), args.sessions, args.max_context), cfg
    from ..models.drafter import Drafter
    from ..models.hybrid import HybridModel
    from .engine import SpecEngine
    dev = torch.device("cuda", 0)
    if args.package:
        model = HybridModel.from_package(args.package, dev)
        cfg = model.cfg
    else:
        model = HybridModel.random(cfg, dev, seed=args.seed)
    drafter = None
    if args.spec_k > 0:
        drafter = (Drafter.from_dir(args.drafter_dir, dev) if args.drafter_dir else
                   Drafter(drafter_preset(args.drafter), cfg.hidden_size, cfg.vocab_size, dev, seed=args.seed + 1))
    scfg = ServeConfig(spec_k=args.spec_k, accept_mode=args.accept_mode, temperature=args.temperature,
                       kv_dtype=args.kv_dtype, hisparse=args.hisparse, seed=args.seed)
    eng = SpecEngine(model, drafter, scfg, args.sessions, args.max_context)
    return eng, cfg


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="tiny_cpu")
    ap.add_argument("--gpu", action="store_true", help="native engine on cuda:0 (random-init weights unless --package)")
    ap.add_argument("--package", default=None, help="INT3 deploy package directory (formats/int3_package.py)")
    ap.add_argument("--drafter", default="tiny")
    ap.add_argument("--drafter-dir", dest="drafter_dir", default=None,
                    help="drafter directory (train/drafter_tools.py layout) instead of a random drafter")
    ap.add_argument("--spec-k", dest="spec_k", type=int, default=4)
    ap.add_argument("--accept-mode", dest="accept_mode", default="rejection",
                    choices=["rejection", "greedy", "bernoulli"])
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--hisparse", action="store_true", help="host KV pool for idle pages (QSA models)")
    ap.add_argument("--kv-dtype", dest="kv_dtype", default="bf16", choices=["bf16", "nvfp4"],
                    help="target KV cache format (nvfp4: e2m1 with e4m3 scales per 16 elements)")
    ap.add_argument("--sessions", type=int, default=8)
    ap.add_argument("--max-context", dest="max_context", type=int, default=4096)
    ap.add_argument("--tokenizer", default=None, help="local Hugging Face tokenizer directory (default: bytes)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--session-ledger", dest="session_ledger", default=None,
                    help="directory of the TITO session ledger (one instance subdirectory per server run)")
    args = ap.parse_args(argv)
    import uvicorn
    from .tokenizer import HFTokenizer
    engine, cfg = _build_engine(args)
    tok = HFTokenizer(args.tokenizer) if args.tokenizer else ByteTokenizer()
    if not args.tokenizer and cfg.vocab_size < ByteTokenizer.vocab_size:
        raise SystemExit(f"vocab {cfg.vocab_size} is smaller than the byte tokenizer's {ByteTokenizer.vocab_size}")
    ledger = None
    if args.session_ledger:
        from ..formats.tito import LedgerWriter
        ledger = LedgerWriter(args.session_ledger, meta={"model": cfg.name, "vocab_size": cfg.vocab_size})
    uvicorn.run(create_app(engine, tok, cfg.name, ledger), host=args.host, port=args.port, log_level="info")


if __name__ == "__main__":
    main()
