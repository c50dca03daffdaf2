"""Worker of the multi-GPU expert-parallel test (run under torchrun by tests/test_gpu_multi.py).

Every rank builds the same full expert bank, keeps its block of experts, and runs the expert-parallel MoE over its
own tokens; the result must equal the single-GPU MoE with the full bank on the same tokens. A second exchange with
a different token count checks that the exchange counters stay in step. Prints one JSON line per rank."""
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from arc_forge_2026_b200.ops import check_status
    from arc_forge_2026_b200.ops.moe import Int3ExpertBank, MoEWorkspace, moe_forward, router_weight_with_shared_gate
    from arc_forge_2026_b200.parallel.ep import EPMoEWorkspace, ExpertParallel, local_bank, moe_forward_ep

    E, k, H, I, Is, T_cap = 32, 4, 512, 256, 256, 24
    g = torch.Generator().manual_seed(0)
    bank = Int3ExpertBank.random(E, H, I, dev, seed=1)
    router = router_weight_with_shared_gate((torch.randn(E, H, generator=g) * 0.05).bfloat16(),
                                            (torch.randn(1, H, generator=g) * 0.05).bfloat16()).to(dev)
    sh13 = (torch.randn(2 * Is, H, generator=g) * 0.05).bfloat16().to(dev)
    sh2 = (torch.randn(H, Is, generator=g) * 0.05).bfloat16().to(dev)
    ep = ExpertParallel(world, rank, T_cap, H, k, E, dev)
    mine = local_bank(bank, world, rank)
    ws_ep = EPMoEWorkspace(ep, I, Is, dev)
    ws_1 = MoEWorkspace(T_cap, E, k, H, I, Is, dev)
    errs = []
    for it, T in enumerate((T_cap - 3 * rank, 5 + rank)):
        gx = torch.Generator().manual_seed(100 + 10 * rank + it)
        x = torch.randn(T, H, generator=gx).bfloat16().to(dev)
        resid = torch.randn(T, H, generator=gx).bfloat16().to(dev)
        out_ep = torch.empty_like(x)
        moe_forward_ep(x, resid, router, mine, sh13, sh2, ep, ws_ep, out_ep)
        out_1 = moe_forward(x, resid, router, bank, sh13, sh2, k, ws_1)
        torch.cuda.synchronize()
        check_status()
        errs.append(((out_ep.float() - out_1.float()).norm() / out_1.float().norm()).item())
    dist.barrier()
    ep.close()
    print(json.dumps({"rank": rank, "rel_err": errs}), flush=True)
    dist.destroy_process_group()
    return 0 if max(errs) < 1e-3 else 1


if __name__ == "__main__":
    sys.exit(main())
