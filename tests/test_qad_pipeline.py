"""QAD pipeline on CPU: qad-topk-v1 round trip, trainer CLI (teacher -> train -> resume -> export), delta
materialisation, and the sharded optimizer over two gloo ranks against a single-process AdamW."""
import json
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from safetensors.torch import save_file

from arc_forge_2026_b200.formats import qad_delta
from arc_forge_2026_b200.formats.topk_targets import TopKReader, TopKWriter
from arc_forge_2026_b200.train import qad
from arc_forge_2026_b200.train.kl import teacher_topk


def test_topk_targets_roundtrip(tmp_path):
    g = torch.Generator().manual_seed(0)
    z = torch.randn(50, 300, generator=g)
    ids, lp, tail = teacher_topk(z, 8)
    labels = torch.randint(0, 300, (50,), generator=g)
    w = TopKWriter(tmp_path, "train", 8)
    w.append(ids[:20], lp[:20], tail[:20], labels[:20])
    w.append(ids[20:], lp[20:], tail[20:], labels[20:])
    w.close({"teacher": "test"})
    r = TopKReader(tmp_path, "train")
    assert r.rows == 50 and r.k == 8
    out = r.rows_slice(10, 30)
    assert torch.equal(out["ids"], ids[10:30])
    total = torch.logsumexp(torch.cat([out["lp"], out["tail"][:, None]], 1), 1)
    torch.testing.assert_close(total, torch.zeros(20), atol=1e-5, rtol=0)
    torch.testing.assert_close(out["lp"], lp[10:30], atol=2e-3, rtol=0)
    with pytest.raises(FileExistsError):
        TopKWriter(tmp_path, "train", 8)


def test_trainer_cli_teacher_train_resume_export(tmp_path, capsys):
    common = ["--preset", "tiny_cpu", "--seq-len", "32", "--batch", "1", "--topk", "8"]
    qad.main(["--mode", "teacher", "--steps", "2", "--out", str(tmp_path / "targets")] + common)
    assert TopKReader(tmp_path / "targets", "train").rows == 64
    ck = tmp_path / "ckpt"
    qad.main(["--mode", "train", "--steps", "2", "--targets", str(tmp_path / "targets"), "--out", str(ck)] + common)
    assert json.loads((ck / "trainer.json").read_text())["step"] == 2
    # resume continues from step 2 with the same plan (steps is part of the plan, so a longer run is a new plan)
    with pytest.raises(RuntimeError, match="refusing to resume"):
        qad.main(["--mode", "train", "--steps", "3", "--targets", str(tmp_path / "targets"), "--out", str(ck),
                  "--resume"] + common)
    capsys.readouterr()
    qad.main(["--mode", "train", "--steps", "2", "--targets", str(tmp_path / "targets"), "--out", str(ck), "--resume",
              "--export", str(tmp_path / "delta")] + common)
    assert capsys.readouterr().out.strip() == ""  # nothing left to train
    d = qad_delta.load_delta(tmp_path / "delta")
    assert any(k.endswith("mlp.experts.w13_scales") for k in d)
    assert any(k.endswith("q_proj.weight_scale_inv") for k in d)
    assert all(v.dtype in (torch.bfloat16, torch.float8_e4m3fn, torch.float32) for v in d.values())


def test_materialize_package(tmp_path):
    src = tmp_path / "pkg"
    src.mkdir()
    save_file({"a": torch.zeros(3, dtype=torch.bfloat16), "b": torch.ones(2)}, str(src / "model-00001.safetensors"))
    qad_delta.export_delta({"a": torch.full((3,), 2.0, dtype=torch.bfloat16)}, tmp_path / "delta")
    out = qad_delta.materialize(src, tmp_path / "delta", tmp_path / "out")
    from safetensors.torch import load_file
    t = load_file(str(out / "model-00001.safetensors"))
    assert torch.equal(t["a"], torch.full((3,), 2.0, dtype=torch.bfloat16)) and torch.equal(t["b"], torch.ones(2))
    assert (out / "DONE").exists()


def _sharded_worker(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from arc_forge_2026_b200.parallel.shard_optim import ShardedAdamW
    torch.manual_seed(0)
    p1, p2 = torch.nn.Parameter(torch.randn(7, 5)), torch.nn.Parameter(torch.randn(11))
    opt = ShardedAdamW([{"params": [p1, p2], "lr": 1e-2}], group=dist.group.WORLD)
    for step in range(3):
        opt.zero_grad()
        g = torch.Generator().manual_seed(100 * step + rank)
        loss = (p1 * torch.randn(7, 5, generator=g)).sum() + (p2 * torch.randn(11, generator=g)).sum()
        loss.backward()
        opt.step(max_norm=0.0)
    if rank == 0:
        torch.save({"p1": p1.detach().clone(), "p2": p2.detach().clone()}, result_path)
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_adamw_matches_single_process(tmp_path):
    port = 29500 + (os.getpid() % 1000)
    res = tmp_path / "r.pt"
    mp.spawn(_sharded_worker, args=(2, port, str(res)), nprocs=2, join=True)
    got = torch.load(res)
    torch.manual_seed(0)
    p1, p2 = torch.nn.Parameter(torch.randn(7, 5)), torch.nn.Parameter(torch.randn(11))
    from arc_forge_2026_b200.train.optim import AdamWBF16
    opt = AdamWBF16([p1, p2], lr=1e-2)
    for step in range(3):
        opt.zero_grad()
        # the reference gradient: mean over ranks of each rank's gradient (same draws as the workers)
        gg1, gg2 = [], []
        for r in range(2):
            gr = torch.Generator().manual_seed(100 * step + r)
            gg1.append(torch.randn(7, 5, generator=gr))
            gg2.append(torch.randn(11, generator=gr))
        p1.grad = (gg1[0] + gg1[1]) / 2
        p2.grad = (gg2[0] + gg2[1]) / 2
        opt.step()
    torch.testing.assert_close(got["p1"], p1.detach(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(got["p2"], p2.detach(), rtol=1e-5, atol=1e-6)


def test_trainer_cli_save_interval_and_profile_step(tmp_path, monkeypatch):
    """--save-every writes a checkpoint only every N steps (and after the last); --profile-step writes the op tables
    and a Chrome trace of that one step."""
    from arc_forge_2026_b200.train import qad as qad_mod
    saved = []
    real = qad_mod.save_checkpoint
    monkeypatch.setattr(qad_mod, "save_checkpoint", lambda path, st, opt, step, ph, rank: (saved.append(step),
                                                                                          real(path, st, opt, step, ph,
                                                                                               rank)))
    common = ["--preset", "tiny_cpu", "--seq-len", "32", "--batch", "1", "--topk", "8", "--synthetic"]
    ck = tmp_path / "ckpt"
    qad_mod.main(["--mode", "train", "--steps", "5", "--save-every", "2", "--profile-step", "1", "--out", str(ck)]
                 + common)
    assert saved == [2, 4, 5]
    assert json.loads((ck / "trainer.json").read_text())["step"] == 5
    table = (ck / "profile_step1_rank0.txt").read_text()
    assert "aten::" in table
    assert json.loads((ck / "profile_step1_rank0.trace.json").read_text())
