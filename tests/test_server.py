"""OpenAI-compatible server over the CPU reference engine: completions, chat, streaming, Responses-API sessions,
/close_session, metrics, and agreement of the served tokens with the reference model's own greedy decode."""
import json

import pytest
import torch

from arc_forge_2026_b200.config import preset
from arc_forge_2026_b200.models.reference import build_reference
from arc_forge_2026_b200.serve.cpu_engine import CPUEngine
from arc_forge_2026_b200.serve.server import create_app
from arc_forge_2026_b200.serve.tokenizer import ByteTokenizer

fastapi = pytest.importorskip("fastapi")
from fastapi.testclient import TestClient  # noqa: E402


class _NoEos(ByteTokenizer):
    eos_id = None  # random weights: do not stop early on the eos byte


@pytest.fixture(scope="module")
def setup():
    cfg = preset("tiny_cpu")
    ref = build_reference(cfg, seed=0)
    app = create_app(CPUEngine(ref, max_sessions=4), _NoEos(), "tiny")
    with TestClient(app) as client:
        yield client, ref


def test_completion_matches_reference_greedy(setup):
    client, ref = setup
    prompt = [5, 17, 99, 3, 250, 41]
    r = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 6})
    assert r.status_code == 200, r.text
    body = r.json()
    toks, _ = ref.greedy_decode(torch.tensor([prompt]), 6)
    assert body["choices"][0]["token_ids"] == toks[0].tolist()
    assert body["usage"] == {"prompt_tokens": 6, "completion_tokens": 6, "total_tokens": 12}


def test_chat_and_stream(setup):
    client, _ = setup
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4})
    assert r.status_code == 200 and r.json()["choices"][0]["message"]["role"] == "assistant"
    with client.stream("POST", "/v1/completions", json={"prompt": "abc", "max_tokens": 5, "stream": True}) as s:
        lines = [ln for ln in s.iter_lines() if ln.startswith("data: ")]
    assert lines[-1] == "data: [DONE]"
    assert len([json.loads(ln[6:]) for ln in lines[:-1]]) == 5


def test_responses_session_continues_and_closes(setup):
    client, ref = setup
    r1 = client.post("/v1/responses", json={"input": "first", "session_id": "s1", "max_output_tokens": 3})
    assert r1.status_code == 200, r1.text
    u1 = r1.json()["usage"]
    r2 = client.post("/v1/responses", json={"input": "second", "session_id": "s1", "max_output_tokens": 3})
    assert r2.status_code == 200, r2.text
    # the second turn's input includes the whole transcript so far (server-side session)
    assert r2.json()["usage"]["input_tokens"] > u1["input_tokens"] + u1["output_tokens"]
    assert client.post("/close_session", json={"session_id": "s1"}).json()["closed"] is True
    assert client.post("/close_session", json={"session_id": "s1"}).json()["closed"] is False


def test_concurrent_requests_beyond_slots_and_metrics(setup):
    client, _ = setup
    import concurrent.futures as cf
    with cf.ThreadPoolExecutor(8) as ex:
        futs = [ex.submit(client.post, "/v1/completions", json={"prompt": [7 + i, 8], "max_tokens": 3})
                for i in range(10)]
        res = [f.result() for f in futs]
    assert all(r.status_code == 200 and len(r.json()["choices"][0]["token_ids"]) == 3 for r in res)
    m = client.get("/metrics").text
    assert "afb_generated_tokens_total" in m and "afb_engine_step_seconds" in m
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"


def test_abort_request_ends_a_running_generation(setup):
    client, _ = setup
    import concurrent.futures as cf
    import time
    with cf.ThreadPoolExecutor(2) as ex:
        fut = ex.submit(client.post, "/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 3000, "rid": "r-abort"})
        aborted = False
        for _ in range(200):  # the request may still be queued on the first tries
            time.sleep(0.05)
            if client.post("/abort_request", json={"rid": "r-abort"}).json()["aborted"]:
                aborted = True
                break
        r = fut.result(timeout=120)
    assert aborted and r.status_code == 200, r.text
    ch = r.json()["choices"][0]
    assert ch["finish_reason"] == "abort" and len(ch["token_ids"]) < 3000
    assert client.post("/abort_request", json={"rid": "r-abort"}).json()["aborted"] is False
    ok = client.post("/v1/completions", json={"prompt": [1, 2], "max_tokens": 2})  # the engine keeps serving
    assert ok.status_code == 200 and len(ok.json()["choices"][0]["token_ids"]) == 2


def test_update_weights_from_disk_swaps_the_served_model(tmp_path):
    cfg = preset("tiny_cpu")
    a, b = build_reference(cfg, seed=0), build_reference(cfg, seed=7)
    path = tmp_path / "b.pt"
    torch.save(b.state_dict(), path)
    app = create_app(CPUEngine(a, max_sessions=2), _NoEos(), "tiny")
    prompt = [3, 1, 4, 1, 5]
    with TestClient(app) as client:
        r = client.post("/update_weights_from_disk", json={"model_path": str(path)})
        assert r.status_code == 200 and r.json()["success"], r.text
        out = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 4}).json()["choices"][0]
        bad = client.post("/update_weights_from_disk", json={"model_path": str(tmp_path / "missing.pt")})
        assert bad.status_code == 400 and bad.json()["success"] is False
    ref = build_reference(cfg, seed=7).eval()
    ids = list(prompt)
    with torch.no_grad():
        for _ in range(4):
            ids.append(int(ref(torch.tensor([ids]))[0, -1].argmax()))
    assert out["token_ids"] == ids[len(prompt):]


def test_completion_with_an_image_matches_the_engine(setup):
    """Image prompts through the server (the ``images`` extension of /v1/completions) give the CPU engine's tokens;
    an engine without a vision tower refuses them with a 400."""
    from arc_forge_2026_b200.models.vision import VisionConfig, VisionTower
    client, _ = setup
    img = 7
    prompt = [11, 12] + [img] * 6 + [13]
    pixels = torch.randn(24, 96, generator=torch.Generator().manual_seed(9))
    body = {"prompt": prompt, "max_tokens": 4, "images": [{"pixels": pixels.tolist(), "grid_thw": [1, 4, 6]}]}
    assert client.post("/v1/completions", json=body).status_code == 400
    cfg = preset("tiny_cpu", mrope_section=(4, 2, 2))
    ref = build_reference(cfg, seed=1)
    tower = VisionTower.random(VisionConfig(depth=1, hidden_size=64, num_heads=4, intermediate_size=96, patch_size=4,
                                            out_hidden_size=cfg.hidden_size, num_position_embeddings=64,
                                            deepstack_visual_indexes=()), seed=2)
    app = create_app(CPUEngine(ref, max_sessions=2, vision=tower, image_token_id=img), _NoEos(), "tiny")
    with TestClient(app) as c2:
        r = c2.post("/v1/completions", json=body)
        assert r.status_code == 200, r.text
        got = r.json()["choices"][0]["token_ids"]
    eng = CPUEngine(ref, vision=tower, image_token_id=img)
    s = eng.add_session(0, prompt, 4, images=[(pixels, (1, 4, 6))])
    while not s.done:
        eng.step()
    assert got == s.generated
