"""Worker of the multi-GPU row-sharded PLE test (run under torchrun by tests/test_gpu_multi.py): the table split by
rows over the ranks; the native lookup reads every row from its owner's HBM over peer memory and matches the
collective path (all-gather of ids, local rows, reduce-scatter) and the unsharded contract."""
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
    from arc_forge_2026_b200.config import preset
    from arc_forge_2026_b200.models.ple import NgramHash
    from arc_forge_2026_b200.ops import check_status
    from arc_forge_2026_b200.parallel.ple_shard import ShardedPleTable, shard_rows
    from arc_forge_2026_b200.quant.fp8 import dequant_weight_block, quantize_weight_block
    cfg = preset("tiny_cpu", vocab_size=248320, ple_layer_ids=(1,), ngram_vocab_size_base=8009, ple_embed_dim=2560)
    h = NgramHash(cfg)
    w = torch.randn(h.rows, 160, generator=torch.Generator().manual_seed(3))
    per = shard_rows(h.rows, world)
    shard = w[rank * per:(rank + 1) * per]
    peer = ShardedPleTable(h, shard, rank, world, dev, fp8=True)
    coll = ShardedPleTable(h, shard, rank, world, dev, fp8=True, peer=False)
    toks = torch.randint(0, cfg.vocab_size, (300 + 50 * rank,), generator=torch.Generator().manual_seed(10 + rank))
    got = peer.lookup_tokens(toks)
    via = coll.lookup_tokens(toks)
    torch.cuda.synchronize()
    check_status()
    full = torch.cat([w, w.new_zeros(per * world - h.rows, 160)])
    q, s = quantize_weight_block(full)
    want = dequant_weight_block(q, s)[h.ids(toks)].flatten(-2)
    res = {"rank": rank, "peer_vs_contract": (got.float().cpu() - want.bfloat16().float()).abs().max().item(),
           "collective_vs_contract": (via.float().cpu() - want).abs().max().item()}
    dist.barrier()
    peer.close()
    print(json.dumps(res), flush=True)
    dist.destroy_process_group()
    return 0 if res["peer_vs_contract"] == 0 and res["collective_vs_contract"] < 1e-6 else 1


if __name__ == "__main__":
    sys.exit(main())
