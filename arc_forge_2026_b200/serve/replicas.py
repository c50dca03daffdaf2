"""Several serving replicas controlled as one policy (the reference's ``training/work/qwen38fn_rl/replica_control.py``):
health and identity are read from every replica, weight updates go to every replica, and a weight update that
reaches only some of them closes the controller for good (until ``/reset`` after the replicas were reconciled), so
rollouts never mix policies silently. Generation traffic goes to the replicas directly, never through here.

    python -m arc_forge_2026_b200.serve.replicas --backends http://127.0.0.1:30571,http://127.0.0.1:30572 --port 30570

Routes: ``GET /health`` (every replica's health; ``ok`` only if all answer and the controller is open),
``POST /update_weights_from_disk {"model_path", "weight_version"?}`` (fan-out; versions must increase),
``POST /reset`` (reopen after a partial update), ``GET /state``.
"""
from __future__ import annotations

import argparse
import json
import threading
import urllib.error
import urllib.request
from concurrent.futures import ThreadPoolExecutor


class ReplicaError(RuntimeError):
    pass


def http_json(root: str, method: str, path: str, body: dict | None = None, timeout: float = 1800.0):
    data = None if body is None else json.dumps(body).encode()
    req = urllib.request.Request(root.rstrip("/") + path, data=data, method=method,
                                 headers={"Content-Type": "application/json"})
    try:
        with urllib.request.urlopen(req, timeout=timeout) as r:
            raw = r.read()
    except urllib.error.HTTPError as e:  # the replica answered with an error body
        raw = e.read()
        try:
            return e.code, json.loads(raw)
        except (json.JSONDecodeError, ValueError):
            return e.code, {"message": raw.decode(errors="replace")}
    return 200, (json.loads(raw) if raw else None)


class Replicas:
    """``transport(root, method, path, body) -> (status, json)``; defaults to HTTP (tests pass an in-process one)."""

    def __init__(self, backends: list[str], transport=None):
        if not backends:
            raise ValueError("no backends")
        self.backends = list(backends)
        self.transport = transport or http_json
        self.lock = threading.Lock()
        self.closed: str | None = None      # reason, after a partial weight update
        self.weight_version = 0
        self.model_path: str | None = None

    def _all(self, method, path, body=None):
        with ThreadPoolExecutor(len(self.backends)) as ex:
            futs = [ex.submit(self._one, b, method, path, body) for b in self.backends]
            return [f.result() for f in futs]

    def _one(self, b, method, path, body):
        try:
            return self.transport(b, method, path, body)
        except Exception as e:  # noqa: BLE001 - a dead replica is a result, not a crash
            return 599, {"message": f"{type(e).__name__}: {e}"}

    def health(self) -> dict:
        res = self._all("GET", "/health")
        reps = [{"backend": b, "status": s, "body": j} for b, (s, j) in zip(self.backends, res)]
        ok = all(s == 200 for s, _ in res) and self.closed is None
        return {"ok": ok, "closed": self.closed, "weight_version": self.weight_version, "model_path": self.model_path,
                "replicas": reps}

    def update_weights(self, model_path: str, weight_version: int | None = None) -> dict:
        with self.lock:
            if self.closed is not None:
                raise ReplicaError(f"controller closed: {self.closed}")
            v = self.weight_version + 1 if weight_version is None else int(weight_version)
            if v <= self.weight_version:
                raise ReplicaError(f"weight_version {v} must exceed {self.weight_version}")
            res = self._all("POST", "/update_weights_from_disk", {"model_path": model_path})
            good = [s == 200 and (j or {}).get("success", False) for s, j in res]
            if all(good):
                self.weight_version, self.model_path = v, model_path
                return {"success": True, "weight_version": v, "replicas": len(good)}
            if any(good):  # some replicas serve the new policy, some the old one: fail closed
                self.closed = (f"partial weight update to {model_path} (v{v}): "
                               f"{sum(good)}/{len(good)} replicas updated")
                raise ReplicaError(self.closed)
            raise ReplicaError(f"no replica accepted {model_path}: {[j for _, j in res]}")

    def reset(self) -> dict:
        with self.lock:
            was, self.closed = self.closed, None
            return {"reopened": was is not None, "was": was}


def create_app(replicas: Replicas):
    from fastapi import FastAPI, HTTPException

    app = FastAPI(title="arc_forge_2026_b200 replica control")

    @app.get("/health")
    def health():
        return replicas.health()

    @app.get("/state")
    def state():
        return {"backends": replicas.backends, "closed": replicas.closed, "weight_version": replicas.weight_version,
                "model_path": replicas.model_path}

    @app.post("/update_weights_from_disk")
    def update(body: dict):
        if not body.get("model_path"):
            raise HTTPException(400, "model_path is required")
        try:
            return replicas.update_weights(body["model_path"], body.get("weight_version"))
        except ReplicaError as e:
            raise HTTPException(409, str(e)) from e

    @app.post("/reset")
    def reset():
        return replicas.reset()

    return app


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--backends", required=True, help="comma-separated replica base URLs")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=30570)
    a = ap.parse_args(argv)
    import uvicorn
    uvicorn.run(create_app(Replicas([b for b in a.backends.split(",") if b])), host=a.host, port=a.port)


if __name__ == "__main__":
    main()
