"""DCP checkpoints (train/checkpoint.py): a ZeRO optimizer state saved by 2 gloo ranks loads into one process, and
a one-process save loads back into 2 ranks, each rank receiving exactly its slice of the moments."""
import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class _Model(torch.nn.Module):
    def __init__(self):
        super().__init__()
        g = torch.Generator().manual_seed(0)
        self.a = torch.nn.Parameter(torch.randn(7, 5, generator=g))
        self.b = torch.nn.Parameter(torch.randn(11, generator=g))
        self.c = torch.nn.Parameter(torch.randn(3, 3, generator=g))


def _groups(m):
    return [{"params": [m.a, m.b], "lr": 1e-2}, {"params": [m.c], "lr": 1e-3}]


def _train(model, opt, rank, steps=3):
    for step in range(steps):
        opt.zero_grad()
        g = torch.Generator().manual_seed(100 * step + rank)
        loss = sum((p * torch.randn(p.shape, generator=g)).sum() for p in (model.a, model.b, model.c))
        loss.backward()
        opt.step(max_norm=0.0) if getattr(opt, "sharded", False) else opt.step()


def _save_worker(rank, world, port, ckpt, ref):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from arc_forge_2026_b200.parallel.shard_optim import ShardedAdamW
    from arc_forge_2026_b200.train.checkpoint import save_dcp
    m = _Model()
    opt = ShardedAdamW(_groups(m), group=dist.group.WORLD)
    _train(m, opt, rank)
    save_dcp(ckpt, m, opt, step=3, plan="p")
    torch.save({"params": {n: p.detach().clone() for n, p in m.named_parameters()},
                "m": [g["m"].clone() for g in opt.groups], "v": [g["v"].clone() for g in opt.groups],
                "chunk": [g["chunk"] for g in opt.groups]}, f"{ref}.{rank}")
    dist.barrier()
    dist.destroy_process_group()


def _load_worker(rank, world, port, ckpt, ref):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from arc_forge_2026_b200.parallel.shard_optim import ShardedAdamW
    from arc_forge_2026_b200.train.checkpoint import load_dcp
    m = _Model()
    with torch.no_grad():
        for p in m.parameters():
            p.zero_()
    opt = ShardedAdamW(_groups(m), group=dist.group.WORLD)
    assert load_dcp(ckpt, m, opt, plan="p") == 3
    want = torch.load(ref)
    ok = all(torch.equal(p, want["params"][n]) for n, p in m.named_parameters())
    for gi, g in enumerate(opt.groups):
        n = sum(p.numel() for p in g["params"])
        lo, hi = min(n, rank * g["chunk"]), min(n, (rank + 1) * g["chunk"])
        ok &= torch.equal(g["m"][: hi - lo], want["m"][gi][lo:hi]) and torch.equal(g["v"][: hi - lo], want["v"][gi][lo:hi])
        ok &= g["step"] == 3
    torch.save(bool(ok), f"{ref}.ok{rank}")
    dist.barrier()
    dist.destroy_process_group()


def test_dcp_checkpoint_reshards_between_world_sizes(tmp_path):
    from arc_forge_2026_b200.train.checkpoint import load_dcp, save_dcp
    from arc_forge_2026_b200.train.optim import AdamWBF16
    port = 29600 + (os.getpid() % 500)
    ckpt, ref = tmp_path / "ck2", tmp_path / "ref"
    mp.spawn(_save_worker, args=(2, port, str(ckpt), str(ref)), nprocs=2, join=True)
    r0, r1 = torch.load(f"{ref}.0"), torch.load(f"{ref}.1")
    # 2 ranks -> 1 process (AdamWBF16, per-parameter state)
    m = _Model()
    opt = AdamWBF16(_groups(m))
    assert load_dcp(ckpt, m, opt, plan="p") == 3
    for n, p in m.named_parameters():
        assert torch.equal(p.detach(), r0["params"][n])
    for gi, params in enumerate(([m.a, m.b], [m.c])):
        n = sum(p.numel() for p in params)
        c = r0["chunk"][gi]
        flat_m = torch.cat([r0["m"][gi][: min(c, n)], r1["m"][gi][: max(0, n - c)]])
        got_m = torch.cat([opt.state[p]["m"].reshape(-1) for p in params])
        assert torch.equal(got_m, flat_m)
        assert all(opt.state[p]["step"] == 3 for p in params)
    # 1 process -> 2 ranks: each rank gets its slice
    ck1 = tmp_path / "ck1"
    save_dcp(ck1, m, opt, step=3, plan="p")
    flat = {"params": {n: p.detach().clone() for n, p in m.named_parameters()},
            "m": [torch.cat([opt.state[p]["m"].reshape(-1) for p in ps]) for ps in ([m.a, m.b], [m.c])],
            "v": [torch.cat([opt.state[p]["v"].reshape(-1) for p in ps]) for ps in ([m.a, m.b], [m.c])]}
    torch.save(flat, tmp_path / "flat")
    mp.spawn(_load_worker, args=(2, port + 1, str(ck1), str(tmp_path / "flat")), nprocs=2, join=True)
    assert torch.load(f"{tmp_path / 'flat'}.ok0") and torch.load(f"{tmp_path / 'flat'}.ok1")
