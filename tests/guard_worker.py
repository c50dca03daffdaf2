"""Worker of the multi-GPU replica-guard test (run under torchrun by tests/test_gpu_multi.py): agreeing packets pass,
one differing element raises the cross-rank mismatch on every rank, and the guard keeps working after it."""
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
    from arc_forge_2026_b200.parallel.guard import ReplicaGuard
    g = ReplicaGuard(world, rank, dev)
    res = {"rank": rank}
    for i in range(5):  # several calls: both slot parities
        g.check([7, i, 123456789012])
    torch.cuda.synchronize()
    check_status()
    res["agree_ok"] = True
    g.check([7, 99 if rank == world - 1 else 98, 1])
    torch.cuda.synchronize()
    try:
        check_status()
        res["mismatch_raised"] = False
    except RuntimeError as e:
        res["mismatch_raised"] = "cross-rank mismatch" in str(e)
    g.check([1, 2, 3])
    torch.cuda.synchronize()
    check_status()
    res["after_ok"] = True
    dist.barrier()
    g.close()
    print(json.dumps(res), flush=True)
    dist.destroy_process_group()
    return 0 if res["mismatch_raised"] else 1


if __name__ == "__main__":
    sys.exit(main())
