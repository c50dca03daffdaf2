"""Worker of the multi-GPU fused ZeRO optimizer test (run under torchrun by tests/test_gpu_multi.py).

Every rank holds the same parameters and its own gradients. The fused peer-memory step
(``parallel.zero.FusedShardedAdamW``) must match the NCCL ``ShardedAdamW`` (same masters within bf16-moment
rounding, same global norm) over steps with and without clipping. A step with a non-finite gradient on one rank
must leave every rank's masters unchanged and raise. The last part times both optimizers on one 64M-element
group (CUDA events, max over ranks). Prints one JSON line per rank."""
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist


def _time(fn, iters=10, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from arc_forge_2026_b200.parallel.shard_optim import ShardedAdamW
    from arc_forge_2026_b200.parallel.zero import FusedShardedAdamW

    shapes = [(300, 257), (1001,), (64, 63)]

    def make():
        g = torch.Generator().manual_seed(0)
        return [torch.randn(s, generator=g).to(dev).requires_grad_() for s in shapes]

    def groups(ps):
        return [{"params": ps[:2], "lr": 1e-2}, {"params": ps[2:], "lr": 3e-3}]

    pa, pb = make(), make()
    oa = ShardedAdamW(groups(pa), weight_decay=0.01)
    ob = FusedShardedAdamW(groups(pb), weight_decay=0.01)
    ok = True
    errs, norm_errs = [], []
    for it in range(5):
        gg = torch.Generator().manual_seed(1000 + 10 * rank + it)
        grads = [torch.randn(s, generator=gg).to(dev) * (5.0 if it == 1 else 1.0) for s in shapes]
        oa.zero_grad()
        ob.zero_grad()
        for p, g in zip(pa, grads):
            p.grad.copy_(g)
        for p, g in zip(pb, grads):
            p.grad.copy_(g)
        clip = 1.0 if it in (1, 3) else 0.0
        na, nb = oa.step(clip), ob.step(clip)
        norm_errs.append(abs(na - nb) / na)
        errs.append(max(float((a - b).abs().max()) for a, b in zip(pa, pb)))
    ok &= max(errs) < 3e-4 and max(norm_errs) < 1e-5
    # a non-finite gradient on the last rank: every rank skips the update and raises
    before = [p.detach().clone() for p in pb]
    ob.zero_grad()
    if rank == world - 1:
        pb[1].grad[7] = float("inf")
    try:
        ob.step(1.0)
        raised = False
    except FloatingPointError:
        raised = True
    unchanged = all(torch.equal(a, b) for a, b in zip(before, pb))
    ok &= raised and unchanged
    # the exchange counters stay in step after the skipped update
    gg = torch.Generator().manual_seed(77 + rank)
    grads = [torch.randn(s, generator=gg).to(dev) for s in shapes]
    oa.zero_grad()
    ob.zero_grad()
    for p, g in zip(pa, grads):
        p.grad.copy_(g)
    for p, g in zip(pb, grads):
        p.grad.copy_(g)
    oa.step(0.0)
    ob.step(0.0)
    after = max(float((a - b).abs().max()) for a, b in zip(pa, pb))
    ok &= after < 3e-4
    dist.barrier()
    ob.close()

    # throughput on one large group (the reduce-scatter and all-gather move 2 (world-1)/world x 4 bytes per element
    # into every rank over NVLink)
    n = 64 << 20
    big_a = [torch.zeros(n, device=dev, requires_grad=True)]
    big_b = [torch.zeros(n, device=dev, requires_grad=True)]
    fa = ShardedAdamW([{"params": big_a, "lr": 1e-3}])
    fb = FusedShardedAdamW([{"params": big_b, "lr": 1e-3}])
    big_a[0].grad.normal_()
    big_b[0].grad.normal_()
    ms_nccl = _time(lambda: fa.step(1.0))
    ms_fused = _time(lambda: fb.step(1.0))
    ms_fused_async = _time(lambda: fb.step(1.0, sync=False))
    nvlink_bytes = 2 * (world - 1) / world * 4 * n
    dist.barrier()
    fb.close()
    print(json.dumps({"rank": rank, "max_abs_err": errs, "norm_rel_err": norm_errs, "skip_ok": raised and unchanged,
                      "after_skip_err": after, "elements": n, "ms_nccl_sharded": round(ms_nccl, 4),
                      "ms_fused": round(ms_fused, 4), "ms_fused_no_host_sync": round(ms_fused_async, 4),
                      "fused_nvlink_gbs_per_rank": round(nvlink_bytes / (ms_fused_async * 1e-3) / 1e9, 1)}), flush=True)
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
