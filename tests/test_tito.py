"""TITO session ledger v1 (formats/tito.py): writer -> reader round trip with routing and top-k sidecars and a
rewind, the invariants on broken files (strict raises with the code, non-strict marks the segment), a live writer's
unterminated last line, RL / SFT exports, and the server recording its sessions."""
import json

import numpy as np
import pytest

from arc_forge_2026_b200.formats import tito


def _write(tmp_path):
    w = tito.LedgerWriter(tmp_path, "inst")
    s = w.open_segment("sess-1")
    rt = np.arange(5 * 2 * 3, dtype=np.int16).reshape(5, 2, 3)
    tk = (np.array([[1, 2], [3, 4]]), np.array([[-0.1, -2.0], [-0.2, -3.0]]), np.array([-5.0, -6.0]), np.array([0, 0]))
    w.append(s, "r0", [1, 2, 3, 4], [7, 8], {"type": "length"}, logprobs=[-0.5, -0.25], routing=rt, topk=tk)
    w.append(s, "r1", [9], [10, 11, 12], {"type": "stop", "matched": 12}, logprobs=[-1, -1, -1], rewind=1)
    w.close_segment(s)
    s2 = w.open_segment(None)
    w.append(s2, "r2", [5, 6], [6], {"type": "length"})
    w.close_segment(s2)
    w.close()
    return tmp_path / "inst"


def test_round_trip_and_exports(tmp_path):
    d = _write(tmp_path)
    inst = tito.read_instance(d, id_bound=100)
    seg = inst.segments[0]
    assert seg.status == "closed" and seg.sid == "sess-1"
    assert seg.S == [1, 2, 3, 4, 7, 9, 10, 11, 12]  # the second append rewound the last generated token
    assert tito.routing_rows(inst, seg.appends[0]).shape == (5, 2, 3)
    assert inst.segments[1].sid is None and inst.segments[1].S == [5, 6, 6]
    rl = tito.rl_examples(seg)
    assert rl[1]["ids"] == seg.S and rl[1]["gen_mask"] == [0] * 6 + [1, 1, 1]
    assert rl[0]["behavior_logp"][4:6] == [-0.5, -0.25]
    sft = tito.sft_examples(inst)
    assert sft[0]["loss_mask"] == [0, 0, 0, 0, 1, 0, 1, 1, 1]


def _mutate(d, fn):
    p = d / "events.0.jsonl"
    lines = [json.loads(x) for x in p.read_text().splitlines()]
    fn(lines)
    p.write_text("".join(json.dumps(x) + "\n" for x in lines))


@pytest.mark.parametrize("code,fn", [
    ("ids_in_vocab", lambda ls: ls[2].update(gen=tito.b64_ids([7, 800]))),
    ("append_order", lambda ls: ls[3].update(k=5)),
    ("prefix_len", lambda ls: ls[3].update(prefix_len=3)),
    ("logprobs_len", lambda ls: ls[3].update(logprobs=tito.b64_f32([-1.0]))),
    ("finish", lambda ls: ls[3].update(finish={"type": "stop", "matched": 99})),
    ("close_sha256", lambda ls: ls[4].update(sha256="0" * 64)),
    ("sid_mismatch", lambda ls: ls[3].update(sid="other")),
])
def test_invariants_strict_and_lenient(tmp_path, code, fn):
    d = _write(tmp_path)
    _mutate(d, fn)
    with pytest.raises(tito.LedgerInvariantError) as e:
        tito.read_instance(d, id_bound=100)
    assert e.value.code == code
    inst = tito.read_instance(d, id_bound=100, strict=False)
    assert inst.segments[0].status == "broken" and inst.segments[1].status == "closed"


def test_format_errors_and_live_tail(tmp_path):
    d = _write(tmp_path)
    p = d / "events.0.jsonl"
    p.write_text(p.read_text() + '{"ev": "append", "sid"')  # a writer mid-line
    inst = tito.read_instance(d, id_bound=100)
    assert inst.truncated_tail and inst.segments[0].status == "closed"
    p.write_text(p.read_text().rsplit("\n", 1)[0] + "\n" + '{"ev": "nope", "t": 0}\n')
    with pytest.raises(tito.LedgerFormatError):
        tito.read_instance(d, id_bound=100)


def test_server_writes_a_ledger(tmp_path):
    fastapi = pytest.importorskip("fastapi")
    from fastapi.testclient import TestClient
    from arc_forge_2026_b200.config import preset
    from arc_forge_2026_b200.models.reference import build_reference
    from arc_forge_2026_b200.serve.cpu_engine import CPUEngine
    from arc_forge_2026_b200.serve.server import create_app
    from arc_forge_2026_b200.serve.tokenizer import ByteTokenizer

    class NoEos(ByteTokenizer):
        eos_id = None
    cfg = preset("tiny_cpu")
    w = tito.LedgerWriter(tmp_path, "srv")
    app = create_app(CPUEngine(build_reference(cfg, seed=0), max_sessions=2), NoEos(), "tiny", ledger=w)
    with TestClient(app) as c:
        r1 = c.post("/v1/responses", json={"input": "hi", "session_id": "s", "max_output_tokens": 3}).json()
        c.post("/v1/responses", json={"input": "more", "session_id": "s", "max_output_tokens": 2})
        c.post("/close_session", json={"session_id": "s"})
        c.post("/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 2})
    inst = tito.read_instance(tmp_path / "srv", id_bound=cfg.vocab_size)
    segs = sorted(inst.segments.values(), key=lambda s: s.seg)
    assert segs[0].sid == "s" and segs[0].status == "closed" and len(segs[0].appends) == 2
    assert len(segs[0].appends[0].gen) == 3 and len(segs[0].appends[1].gen) == 2
    assert r1["usage"]["input_tokens"] == len(segs[0].appends[0].tail)
    assert segs[1].sid is None and segs[1].S[:3] == [1, 2, 3] and len(segs[1].S) == 5
