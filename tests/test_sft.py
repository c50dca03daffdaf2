"""SFT / LoRA trainer over packed bins on CPU: examples (ids + mask, prompt / completion) pack into bins, the loss
falls on a small memorised set, training resumes from its state, and the merged export is written."""
import json

from arc_forge_2026_b200.train import sft


def _data(tmp_path, n=6):
    import random
    rng = random.Random(0)
    p = tmp_path / "d.jsonl"
    with open(p, "w") as f:
        for i in range(n):
            ids = [rng.randrange(1, 200) for _ in range(rng.randrange(20, 90))]
            if i % 2:
                f.write(json.dumps({"prompt_ids": ids[:10], "completion_ids": ids[10:]}) + "\n")
            else:
                f.write(json.dumps({"ids": ids}) + "\n")
    return p


def test_sft_trains_resumes_and_exports(tmp_path, capsys):
    d = _data(tmp_path)
    seqs, masks = sft.load_examples(d)
    assert len(seqs) == 6 and masks[1][:10] == [0] * 10 and masks[1][10] == 1
    out = tmp_path / "run"
    common = ["--data", str(d), "--preset", "tiny_cpu", "--max-len", "256", "--bins-per-step", "1", "--lr", "3e-3",
              "--lora-r", "8", "--out", str(out)]
    sft.main(common + ["--steps", "8"])
    logs = [json.loads(x) for x in capsys.readouterr().out.splitlines() if x.startswith("{")]
    steps = [r for r in logs if "step" in r]
    assert logs[0]["bins"] >= 2 and len(steps) == 8
    first, last = steps[0]["loss"], steps[-1]["loss"]
    assert last < first, (first, last)
    sft.main(common + ["--steps", "10", "--resume", "--export"])
    steps2 = [json.loads(x) for x in capsys.readouterr().out.splitlines() if x.startswith('{"step"')]
    assert [r["step"] for r in steps2] == [8, 9]
    assert (out / "merged" / "DONE").exists() and (out / "trainer_state.pt").exists()
