"""Headline benchmark: speculative decode throughput at 128 concurrent sessions (BASELINE configs 2+3).

Model: Qwen3-Next-80B-A3B-shaped hybrid MoE (48 layers, hidden 2048, GDN:attention 3:1, 320 routed experts top-10
in uint3 g128 INT3 + shared expert, attention 16Q/2KV x 256, GDN 16/32 heads x 128, vocab 151,936), random init,
plus an 8-layer DFlash-style drafter (hidden 2048) proposing K=4 tokens per cycle. Acceptance per position is a
seeded Bernoulli(0.7) draw. 128 sessions with synthetic contexts of U[4k, 24k] tokens
(KV pages, GDN states and drafter window filled with random data: the bench measures decode, not prefill).

Timed region: K speculative cycles (CUDA-graph replays), bracketed by a barrier and torch.cuda.synchronize on both
sides, timed with CUDA events on the launching stream; the max over ranks is reported. ``value`` = emitted tokens
(accepted drafts + the bonus token) of all sessions on all ranks / wall time of the timed region.
``e2e`` = the same metric through the engine's public ``step()`` API, which each cycle uploads the page table from
pinned host memory and reads back the emitted tokens.

With N GPUs (torchrun), attention / GDN / drafter run data-parallel: the 128 sessions (contexts drawn once) are dealt
to the ranks in snake order of decreasing length, so every rank holds 128/N sessions and nearly the same KV; the
routed experts are split over the ranks (expert parallelism, fused peer-memory dispatch / combine).
``--mode qsa`` runs BASELINE config 5 (110 sessions, 64k contexts, QSA top-32 of 64-token blocks; ``--hisparse``
keeps the KV history in pinned host memory); ``--mode qad`` the QAD training step (config 4).
``--impl reference`` runs the unmodified reference when it is installed under baseline/_ref, else prints its
``unavailable`` line.
"""
from __future__ import annotations

import argparse
import collections
import json
import os
import statistics
import subprocess
import sys
import threading
import time

METRIC = "decode tok/s @128 sessions (8xB200, spec K=4); p50 TPOT; QAD train tok/s"
QSA_METRIC = "decode tok/s @110 sessions, 64k contexts, QSA top-32 x 64-token blocks (spec K=4)"
# The reference publishes no decode number for this model on B200: its 128-session figures (2,141 / 2,343 tok/s,
# paper section 8.3 and Table 10) are for 4 x L4 over PCIe, so no published number is comparable and vs_baseline
# stays null for the serving modes.
SERVE_BASELINE_NOTE = ("no comparable published number: the reference's 128-session decode figures are 4xL4/PCIe "
                       "(2,141 tok/s, paper section 8.3); its B200 figure is a 41 ms cycle for its own 2560-hidden "
                       "HC4/PLE model at 64 sessions (paper App. E.11)")


def _reference_arm(args):
    ref = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")
    why = ("pip reports the reference 'is not installable' (no setup.py or pyproject.toml anywhere in the tree); its "
           "serving engine is a private sglang fork (only its patch set ships) and its INT3 MoE kernels come from a "
           "closed binary wheel (humming-kernels), neither of which is in the offline wheelhouse")
    if os.path.isdir(ref) and any(n.endswith(".dist-info") for n in os.listdir(ref)):
        why = "baseline/_ref holds a package, but " + why
    line = {"impl": "reference", "unavailable": why, "n_gpus": args.gpus}
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(line))


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._proc = None

    def __enter__(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self._proc = None
        return self

    def _read(self):
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for s in self.samples:
            for name, v in zip(names, s[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.samples)}


def ep_wait_summary(wait_log, steps: int, world: int, rank: int):
    """Per-rank expert-parallel wait accounting of the timed cycles (every rank takes part in the gather; rank 0
    gets the summary): how long each rank's w13 GEMM waited for the dispatch exchange and its combine for the combine
    exchange, per cycle, and the distribution of the per-(rank, layer) waits."""
    import torch
    import torch.distributed as dist
    allw = [torch.zeros_like(wait_log) for _ in range(world)]
    dist.all_gather(allw, wait_log)
    if rank != 0:
        return None
    w = torch.stack(allw).double().cpu() / max(steps, 1) / 1e3  # [world, layers, 2] microseconds per cycle
    edges = [0, 10, 25, 50, 100, 200, 500, float("inf")]

    def hist(x):
        x = x.flatten()
        return {f"{lo:g}-{hi:g}us" if hi != float("inf") else f">{lo:g}us": int(((x >= lo) & (x < hi)).sum())
                for lo, hi in zip(edges[:-1], edges[1:])}

    def q(x, p):
        return round(float(torch.quantile(x.flatten(), p)), 1)
    return {"per_rank_ms_per_cycle": {"dispatch": [round(float(v), 3) for v in w[:, :, 0].sum(1) / 1e3],
                                      "combine": [round(float(v), 3) for v in w[:, :, 1].sum(1) / 1e3]},
            "per_layer_us": {"dispatch": {"p50": q(w[:, :, 0], 0.5), "p90": q(w[:, :, 0], 0.9),
                                          "max": q(w[:, :, 0], 1.0), "hist": hist(w[:, :, 0])},
                             "combine": {"p50": q(w[:, :, 1], 0.5), "p90": q(w[:, :, 1], 0.9),
                                         "max": q(w[:, :, 1], 1.0), "hist": hist(w[:, :, 1])}},
            "note": "block 0 of each w13 GEMM / combine kernel, wall time from entering its wait to the last flag"}


def count_launches(fn, census_out=None, time_out=None):
    """Kernels of this repository launched by one call of ``fn`` (kernel list from the profiler's trace; used
    only for counting, never for timing)."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    ours = ("gemm_bf16", "splitk_reduce", "moe_int3", "rmsnorm", "qk_norm_rope", "router_topk", "expert_sort",
            "quant_rows", "moe_combine", "swiglu", "embedding", "paged_attn", "attn_merge", "gdn_", "select_tokens",
            "spec_accept", "build_window", "gather_rows", "expert_sort", "int3_dequant", "int3_scale_grad",
            "fp8_block_fakequant", "topk_tail_kl", "adamw_kernel", "train_kernel", "ep_dispatch", "ep_wait",
            "ep_gather", "gdn_chunk_scan", "quant_routed")
    n_ours = n_all = 0
    census = collections.Counter()
    for e in prof.events():
        if e.device_type.name == "CUDA" and not e.name.startswith("Memcpy") and not e.name.startswith("Memset"):
            n_all += 1
            census[e.name[:90]] += 1
            if time_out is not None:
                time_out[e.name[:90]] += e.device_time_total
            if "afb::" in e.name or any(k in e.name for k in ours):  # every kernel of csrc/ lives in namespace afb
                n_ours += 1
    if census_out is not None:
        census_out.update(census)
    return n_ours, n_all


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--sessions", type=int, default=None, help="default 128 (serve), 110 (qsa)")
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--min-ctx", type=int, default=None, help="default 4096 (serve), 65536 (qsa)")
    ap.add_argument("--max-ctx", type=int, default=None, help="default 24576 (serve), 65536 (qsa)")
    ap.add_argument("--out-tokens", type=int, default=None, help="default 2048 (serve), 4096 (qsa)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--mode", default="serve", choices=["serve", "qad", "qsa"],
                    help="serve: spec-decode serving (default, configs 2+3); qsa: long-context serving with QSA "
                         "block-sparse attention (config 5); qad: QAD training step (config 4)")
    ap.add_argument("--seq-len", dest="seq_len", type=int, default=16384, help="qad: tokens per sequence")
    ap.add_argument("--global-batch", dest="global_batch", type=int, default=32, help="qad: sequences per step")
    ap.add_argument("--topk", type=int, default=64, help="qad: teacher top-k")
    ap.add_argument("--census", action="store_true", help="print the kernel-time shares of one step (stderr)")
    ap.add_argument("--model", default="qwen3next_80b", choices=["qwen3next_80b", "qwen38fn"],
                    help="serve / qsa: the served model. qwen38fn: the reference's own shape (HC4, PLE at layer 2, "
                         "hidden 2560, 24Q/2KV x 256, QSA top-512 of 4-token blocks), the like-for-like anchor "
                         "against its published ~41 ms per cycle")
    ap.add_argument("--experts", type=int, default=None,
                    help="routed experts (default: 320 for both models, the gEAN-pruned count)")
    ap.add_argument("--qsa-block", dest="qsa_block", type=int, default=64,
                    help="qsa: tokens per block (64: BASELINE config 5; 4: the reference model's own QSA)")
    ap.add_argument("--qsa-topk", dest="qsa_topk", type=int, default=None,
                    help="qsa: blocks kept per query (default 2048 tokens / block: 32 at block 64, 512 at block 4)")
    ap.add_argument("--hisparse", action="store_true", help="qsa: KV history in pinned host memory (HiSparse)")
    ap.add_argument("--hisparse-fp8", dest="hisparse_fp8", action="store_true",
                    help="qsa: host pool in e4m3 with per-(page, head) scales")
    args = ap.parse_args()
    if args.impl == "reference":
        _reference_arm(args)
        return
    if args.mode == "qad":
        return qad_main(args)
    qsa = args.mode == "qsa"
    anchor = args.model == "qwen38fn"
    for k, serve_v, qsa_v in (("sessions", 64 if anchor else 128, 110), ("min_ctx", 4096, 65536),
                              ("max_ctx", 24576, 65536), ("out_tokens", 2048, 4096)):
        if getattr(args, k) is None:
            setattr(args, k, qsa_v if qsa else serve_v)
    if args.warmup < 3:
        args.warmup = 3
    if args.qsa_topk is None:
        args.qsa_topk = 2048 // args.qsa_block

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    from arc_forge_2026_b200.config import ServeConfig, drafter_preset, preset
    from arc_forge_2026_b200.models.drafter import Drafter
    from arc_forge_2026_b200.models.hybrid import HybridModel
    from arc_forge_2026_b200.ops import check_status
    from arc_forge_2026_b200.ops.attention import PAGE
    from arc_forge_2026_b200.serve.engine import SpecEngine

    dev = torch.device("cuda", local)
    if anchor:  # the model's own QSA (top-512 of 4-token blocks) in every mode
        cfg = preset("qwen38fn", num_layers=args.layers, num_experts=args.experts or 320)
    else:
        cfg = preset("qwen3next_80b", num_layers=args.layers, num_experts=args.experts or 320,
                     **(dict(qsa_block=args.qsa_block, qsa_topk=args.qsa_topk) if qsa else {}))
    S_total = args.sessions
    # contexts of all sessions drawn once, dealt to ranks in snake order of decreasing length (equal counts,
    # near-equal KV per rank: the placement a serving scheduler makes so no rank gates the per-layer exchanges)
    ctx_all = torch.randint(args.min_ctx, args.max_ctx + 1, (S_total,), generator=torch.Generator().manual_seed(
        args.seed * 1000 + 17))
    order = torch.argsort(ctx_all, descending=True, stable=True).tolist()
    mine = [order[i] for i in range(S_total) if (i // world) % 2 == 0 and i % world == rank or
            (i // world) % 2 == 1 and world - 1 - i % world == rank]
    S = len(mine)
    K = 4
    model = HybridModel.random(cfg, dev, seed=args.seed, ep_world=world)
    if world > 1:  # attention/GDN data-parallel over sessions, routed experts split over the ranks
        # one capacity on every rank (sessions need not split evenly): the exchange layout depends on it
        model.enable_expert_parallel(world, rank, T_cap=-(-S_total // world) * (K + 1))
    drafter = Drafter(drafter_preset("dflash_8l"), cfg.hidden_size, cfg.vocab_size, dev, seed=args.seed + 1)
    scfg = ServeConfig(spec_k=K, accept_mode="bernoulli", accept_prob=0.7, seed=args.seed + 7 * rank,
                       hisparse=bool(qsa and args.hisparse), hisparse_fp8=bool(args.hisparse_fp8))
    g = torch.Generator().manual_seed(args.seed * 1000 + rank)
    ctx = ctx_all[mine]
    need_pages = int(sum((int(c) + args.out_tokens + 2 * (K + 1) + 8 + PAGE - 1) // PAGE for c in ctx))
    max_context = args.max_ctx + args.out_tokens + 64
    eng = SpecEngine(model, drafter, scfg, S, max_context, num_pages=need_pages)

    # synthetic sessions: contexts already "prefilled" with random KV / recurrent state
    with torch.no_grad():
        for kc, vc in eng.kv:
            kc.normal_(0, 1.0, generator=None)
            vc.normal_(0, 1.0)
        for st in eng.gdn:
            st.ssm.normal_(0, 0.02)
            st.conv.normal_(0, 0.5)
        for kc, vc in eng.dkv:
            kc.normal_(0, 1.0)
            vc.normal_(0, 1.0)
        from arc_forge_2026_b200.serve.engine import Session
        for i in range(S):
            sess = Session(i, i, [0] * int(ctx[i]), 10**9)
            eng.sessions[i] = sess
            eng.free_rows.remove(i)
            if eng.hs is None:
                eng.alloc.ensure(i, int(ctx[i]) + args.out_tokens + 2 * (K + 1) + 8)
        if eng.hs is None:
            eng._sync_pages()
        else:  # host pools: random valid values (e4m3 or bf16 of N(0, 1)), written in chunks from the device
            for hk, hv in eng.hs.host_tensors():
                for host in (hk, hv):
                    step = 1 << 28
                    for o in range(0, host.numel(), step):
                        n = min(step, host.numel() - o)
                        if args.hisparse_fp8:
                            src = torch.randn(n, device=dev).to(torch.float8_e4m3fn).view(torch.uint8)
                        else:
                            src = torch.randn(n // 2, device=dev).bfloat16().view(torch.uint8)
                        host[o:o + n].copy_(src)
        eng.ctx_len.copy_(ctx.int().to(dev))
        eng.anchor.copy_(torch.randint(0, cfg.vocab_size, (S,), generator=g).int().to(dev))
        eng.drafts.copy_(torch.randint(0, cfg.vocab_size, (S, K), generator=g).int().to(dev))
        eng.active.fill_(1)
        if eng.qsa is not None:  # indexer state of the synthetic contexts: random raw and pooled keys
            for raw, key in eng.qsa.cache:
                raw.normal_(0, 1.0)
                key.normal_(0, 1.0)
            eng.qsa.fin.copy_((ctx // cfg.qsa_block).int().to(dev))
    torch.cuda.synchronize()
    eng.capture()
    check_status()

    def barrier():
        if world > 1:
            dist.barrier()

    # The timed cycles sample the whole decode span: they run in G groups, group g starting with every session's
    # context advanced by (g + 1/2) * out_tokens / G tokens (midpoints of G equal slices of the output), so the KV
    # read per cycle averages over the span instead of its first tokens. The pages of the full span were
    # allocated above; the jump is one device copy of the context lengths (and the QSA finalisation mark).
    ctx_dev = ctx.int().to(dev)
    G = 1 if scfg.hisparse else max(1, min(4, args.steps))
    offsets = [int((g + 0.5) * args.out_tokens / G) for g in range(G)]

    def at_offset(i, n):
        g = i * G // n
        if i == 0 or g != (i - 1) * G // n:
            eng.ctx_len.copy_(ctx_dev + offsets[g])
            if eng.qsa is not None:
                eng.qsa.fin.copy_((ctx_dev + offsets[g]) // cfg.qsa_block)

    # ---------------- device-timed: K graph replays
    for _ in range(args.warmup):
        eng.run_cycle()
    counts = torch.zeros(args.steps, S, dtype=torch.int32, device=dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    total0 = int(eng.total.item())
    wait_log = model.ep.wait_log if (world > 1 and model.ep is not None) else None
    if wait_log is not None:
        wait_log.zero_()
        torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        ev[0].record()
        for i in range(args.steps):
            at_offset(i, args.steps)
            eng.run_cycle()
            counts[i].copy_(eng.out_count)
            ev[i + 1].record()
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[-1])
    ep_waits = ep_wait_summary(wait_log, args.steps, world, rank) if wait_log is not None else None
    cyc_ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
    emitted = int(eng.total.item()) - total0
    check_status()
    cnt = counts.cpu()
    tpot = []
    for i in range(args.steps):
        for s in range(S):
            c = int(cnt[i, s])
            if c > 0:
                tpot.append(cyc_ms[i] / c)

    # ---------------- end-to-end through the public step() API (H2D page table, D2H emitted tokens)
    for _ in range(2):
        eng.step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_tokens = 0
    e0.record()
    for i in range(args.steps):
        at_offset(i, args.steps)
        e_tokens += sum(len(v) for v in eng.step().values())
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e_ms = e0.elapsed_time(e1)
    h2d = eng.bt_host.numel() * 4
    d2h = (eng.out_host.numel() + eng.cnt_host.numel()) * 4

    census, ktime = collections.Counter(), collections.Counter()
    n_ours, n_all = count_launches(eng.run_cycle, census, ktime)
    if args.census and rank == 0:  # kernel-time shares of one cycle for the log (profiler time: not a result)
        tot = sum(ktime.values())
        for name, us in ktime.most_common(30):
            print(f"kernel {us / 1000:8.3f} ms {100 * us / tot:5.1f}%  x{census[name]:5d}  {name}", file=sys.stderr)

    # ---------------- reduce over ranks (max time, summed tokens)
    if world > 1:
        t = torch.tensor([ms, e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e_ms = float(t[0]), float(t[1])
        n = torch.tensor([emitted, e_tokens], device=dev, dtype=torch.float64)
        dist.all_reduce(n)
        emitted, e_tokens = int(n[0]), int(n[1])
        tp = torch.tensor([statistics.median(tpot) if tpot else 0.0], device=dev, dtype=torch.float64)
        dist.all_reduce(tp, op=dist.ReduceOp.MAX)
        p50 = float(tp[0])
    else:
        p50 = statistics.median(tpot) if tpot else None
    value = emitted / (ms / 1000.0)
    e2e = e_tokens / (e_ms / 1000.0)
    out = {
        "metric": QSA_METRIC if qsa else METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
        "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "baseline_note": SERVE_BASELINE_NOTE, "dtype": "bf16",
        "data": f"synthetic (random-init weights; random tokens; contexts U[{args.min_ctx},{args.max_ctx}] as random "
                f"KV/GDN/indexer state)",
        "config": {"model": (f"qwen38fn (reference shape: HC4, PLE layer 2, hidden 2560, 24Q/2KV x 256, GDN 16/48 "
                             f"heads), {args.layers}L, {cfg.num_experts} experts x 640 top-10 INT3 g128 + shared, "
                             f"QSA top-{cfg.qsa_topk} of {cfg.qsa_block}-token blocks; 8-layer DFlash drafter")
                            if anchor else
                            (f"qwen3next_80b-shaped hybrid MoE, {args.layers}L, {cfg.num_experts} experts top-10 INT3 "
                             f"g128 + shared; 8-layer DFlash drafter"),
                   "global_batch": S_total, "seq_len": f"U[{args.min_ctx},"
                            f"{args.max_ctx}] context + decode",
                   "parallelism": f"dp{world}-attn+ep{world}" if world > 1 else "dp1",
                   "placement": "sessions dealt to ranks in snake order of context length" if world > 1 else None,
                   "spec_k": K, "acceptance": "seeded Bernoulli(0.7) per position", "layers": args.layers,
                   "attention": (f"QSA top-{cfg.qsa_topk} of {cfg.qsa_block}-token blocks (+ each row's own incomplete "
                                  f"block)") if cfg.qsa_topk else "dense",
                   "kv_offload": ("HiSparse host pool " + ("e4m3" if args.hisparse_fp8 else "bf16"))
                   if scfg.hisparse else "none (all KV on the GPU)",
                   "l2": "inputs larger than L2 (weights 24 GB, KV > 40 GB streamed every cycle)",
                   "decode_span": f"timed cycles in {G} groups at context + {offsets} of {args.out_tokens} output "
                                  f"tokens"},
        "p50_tpot_ms": round(p50, 3) if p50 else None,
        "ep_waits": ep_waits,
        "cycle_ms": round(ms / args.steps, 3),
        "reference_cycle_ms": 41.0 if anchor else None,  # paper App. E.11 (p. 85): ~41 ms per cycle on one B200
        "accepted_per_cycle": round(emitted / (args.steps * S_total), 3),
        "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": n_ours * args.steps,
        "gpu_launches_per_step": {"ours": n_ours, "all": n_all},
        "clocks": clocks.summary(),
    }
    if rank == 0:
        print(json.dumps(out))
    eng.graphs.clear()
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()  # no rank still reads a peer's heap
        model.ep.close()
        dist.destroy_process_group()


QAD_METRIC = "QAD train tok/s"
QAD_BASELINE_TOKS = 19900.0  # reference, 4 x B200, fused gradient kernels


def qad_main(args):
    """QAD training throughput on the config-4 shape: the 48-layer student (320 INT3 experts with STE, FP8 QAT
    dense), forward KL on top-``topk`` teacher targets, ``global_batch`` sequences of ``seq_len`` tokens per
    optimizer step (one sequence per micro-batch, gradients accumulated), sharded bf16 AdamW over the ranks."""
    if args.warmup < 3:
        args.warmup = 3
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    from arc_forge_2026_b200.config import QADConfig, preset
    from arc_forge_2026_b200.formats.topk_targets import synthetic_targets
    from arc_forge_2026_b200.train.qad import build_optimizer, enforce_scale_invariants, train_step
    from arc_forge_2026_b200.train.student import random_student

    if args.global_batch % world:
        raise SystemExit(f"--global-batch {args.global_batch} is not a multiple of {world} ranks")
    micro = args.global_batch // world
    cfg = preset("qwen3next_80b", num_layers=args.layers)
    qc = QADConfig(seq_len=args.seq_len, topk=args.topk, direction="forward")
    student = random_student(cfg, dev, seed=args.seed)
    opt = build_optimizer(student, qc, sharded=True, group=dist.group.WORLD if world > 1 else None)
    signs = enforce_scale_invariants(student, None)
    g = torch.Generator().manual_seed(args.seed * 7919 + rank)
    T = args.seq_len
    # host-side inputs for every micro-batch (pinned), copied to the device inside the e2e timed region
    host = []
    for _ in range(micro):
        ids = torch.randint(0, cfg.vocab_size, (1, T), generator=g, dtype=torch.int64)
        t = synthetic_targets(T, args.topk, cfg.vocab_size, g)
        host.append({"ids": ids.pin_memory(), "t_ids": t["ids"].int().pin_memory(),
                     "lp": t["lp"].float().pin_memory(), "tail": t["tail"].float().pin_memory()})
    dev_in = [{k: v.to(dev) for k, v in h.items()} for h in host]
    h2d = sum(v.numel() * v.element_size() for h in host for v in h.values())

    def one_step(inputs):
        losses = []
        for i, x in enumerate(inputs):
            tg = {"ids": x["t_ids"].long(), "lp": x["lp"], "tail": x["tail"]}  # int32 on the wire, as stored
            losses.append(train_step(student, opt, x["ids"], tg, qc, signs, accumulate=i < len(inputs) - 1,
                                     sync=False, micro_batches=len(inputs), first=i == 0))
        return torch.stack(losses).mean()

    def barrier():
        if world > 1:
            dist.barrier()

    from arc_forge_2026_b200.train import kernels
    for i in range(args.warmup):
        if i == args.warmup - 1:
            kernels.reset()
        one_step(dev_in)
    kernels.assert_step_calls(no_fallback=True)  # every native training kernel ran; none fell back to PyTorch
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        ev0.record()
        for _ in range(args.steps):
            loss = one_step(dev_in)
        ev1.record()
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)

    # end to end: pinned host -> device copies of every micro-batch and the loss read back, each step
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        inputs = [{k: v.to(dev, non_blocking=True) for k, v in h.items()} for h in host]
        last_loss = float(one_step(inputs))
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms, e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e_ms = float(t[0]), float(t[1])
    census, ktime = collections.Counter(), collections.Counter()
    n_ours, n_all = count_launches(lambda: one_step(dev_in), census, ktime)
    if args.census and rank == 0:  # device time by framework op (which PyTorch ops the elementwise kernels are)
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], record_shapes=True) as prof:
            one_step(dev_in)
            torch.cuda.synchronize()
        rows = sorted(prof.key_averages(), key=lambda e: -e.self_device_time_total)[:30]
        for e in rows:
            print(f"op ms/step {e.self_device_time_total / 1000:9.1f}  x{e.count:6d}  {e.key[:80]}", file=sys.stderr)
        rows = sorted(prof.key_averages(group_by_input_shape=True), key=lambda e: -e.self_device_time_total)[:60]
        for e in rows:
            if e.key.startswith("aten::"):
                print(f"op+shape ms/step {e.self_device_time_total / 1000:9.1f}  x{e.count:6d}  {e.key[:40]}  "
                      f"{str(e.input_shapes)[:140]}", file=sys.stderr)
    if rank == 0:  # where one step's launches and kernel time go, for the log (profiler time: not a result)
        for name, cnt in census.most_common(12):
            print(f"launches/step {cnt:8d}  {name}", file=sys.stderr)
        for name, us in ktime.most_common(25):
            print(f"kernel ms/step {us / 1000:9.1f}  x{census[name]:6d}  {name}", file=sys.stderr)
    tokens = args.global_batch * T * args.steps
    value = tokens / (ms / 1000.0)
    out = {
        "metric": QAD_METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
        "scaling": "strong", "dtype": "bf16",
        # the published 19.9k tok/s is a 4 x B200 figure: compared only at the same GPU count
        "vs_baseline": round(value / QAD_BASELINE_TOKS, 3) if world == 4 else None,
        "data": "synthetic (random-init student; uniform random tokens; random valid top-k teacher targets)",
        "config": {"model": "qwen3next_80b-shaped student, 48L, 320 INT3 experts (STE scales), FP8 QAT dense",
                   "global_batch": args.global_batch, "seq_len": T, "parallelism": f"dp{world}+" + ("fused-zero-adamw" if type(opt).__name__ == "FusedShardedAdamW" else "sharded-adamw"),
                   "loss": f"forward KL, teacher top-{args.topk} + tail", "layers": args.layers,
                   "optimizer": "bf16-state AdamW", "l2": "inputs larger than L2 (weights and activations)"},
        "loss": round(last_loss, 5),
        "e2e": {"value": round(tokens / (e_ms / 1000.0), 1), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": 4},
        "gpu_launches": n_ours * args.steps,
        "gpu_launches_per_step": {"ours": n_ours, "all": n_all},
        "peak_gib": round(torch.cuda.max_memory_allocated() / 2**30, 2),
        "clocks": clocks.summary(),
    }
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
