"""Kernel micro-benchmarks (CUDA events, warm-up, L2 flushed between timed launches).

    python -m arc_forge_2026_b200.utils.kbench moe      # INT3 w13/w2 expert GEMMs at the verify-step shape
    python -m arc_forge_2026_b200.utils.kbench gemm     # dense bf16 GEMMs of the decode step
    python -m arc_forge_2026_b200.utils.kbench gdn_scan # chunked-GDN inter-chunk scan at the QAD shape
    python -m arc_forge_2026_b200.utils.kbench gdn_train # chunked-GDN layer forward + backward at the QAD shape
    python -m arc_forge_2026_b200.utils.kbench qsa      # QSA selection + sparse verify attention (block 4 and 64)
    python -m arc_forge_2026_b200.utils.kbench vision   # the 27-block vision tower beside the HF bf16 model

Prints one JSON line per kernel: time, bytes, FLOPs and the fraction of MEASURED_PEAKS.json.
"""
from __future__ import annotations

import argparse
import json
import os

import torch

PEAKS = {"hbm_gbs": 6554.9, "bf16_tflops": 1668.7}


def load_peaks(path: str | None = None):
    path = path or os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"]}
    except (OSError, KeyError, ValueError):
        return dict(PEAKS)


def time_cuda(fn, iters: int = 20, warmup: int = 3, flush_bytes: int = 256 << 20) -> float:
    """Median milliseconds of ``fn`` with an L2 flush (write of ``flush_bytes``) before every timed launch."""
    flush = torch.empty(flush_bytes, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def bench_moe(T=640, E=320, H=2048, I=512, k=10):
    """The routed-expert path of one MoE layer at the verify-step shape: per-row quantisation of the token rows, the
    w13 GEMM over each expert's listed entries (SwiGLU epilogue, bf16 h), the per-row requantisation of h and the w2
    GEMM. Bytes are the algorithmic ones: the INT3 weights and scales once, the activations read and written once."""
    from ..ops import C
    from ..ops.moe import Int3ExpertBank, MoEWorkspace
    peaks = load_peaks()
    dev = "cuda"
    bank = Int3ExpertBank.random(E, H, I, dev)
    ws = MoEWorkspace(T, E, k, H, I, I, dev)
    x = torch.randn(T, H, device=dev).bfloat16()
    logits = torch.randn(T, E + 8, device=dev)
    c = C()
    n = T * k
    c.router_topk(logits, E, k, True, ws.ids[:T], ws.weights[:T], ws.cnt, ws.list)
    c.quant_rows_e4m3_row(x, None, None, T, ws.xq[:T], ws.xs)
    rw = ws.weights[:T].reshape(-1)
    w13 = lambda dbg=None: c.moe_int3_gemm(bank.w13_codes, bank.w13_scales, ws.cnt, ws.list, k, ws.xq[:T],  # noqa
                                           ws.xs, True, None, None, ws.h[:n], None, dbg)
    hq = lambda: c.quant_rows_e4m3_row(ws.h[:n], None, None, n, ws.hq[:n], ws.hs)  # noqa
    w2 = lambda dbg=None: c.moe_int3_gemm(bank.w2_codes, bank.w2_scales, ws.cnt, ws.list, 1, ws.hq[:n], ws.hs,  # noqa
                                          False, None, None, ws.y[:n], rw, dbg)
    w13()
    hq()
    torch.cuda.synchronize()
    out = []
    for name, fn in (("moe_w13_int3", w13), ("moe_w2_int3", w2)):
        dbg = torch.zeros(148 * 4 * 5, dtype=torch.int64, device=dev)
        fn(dbg)
        torch.cuda.synchronize()
        d = dbg.view(148, 4, 5).float()
        live = d[:, 0, 2] > 0
        ks = d[live, :, 2].clamp_min(1)
        # per role and k-step: cycles waiting, in the main section (loader: copy issue; dequant: load + decode; MMA:
        # MMA issue; epilogue: TMEM loads + FMAs) and in a second section (dequant: TMEM store; MMA: commits)
        out.append({"kernel": name + "_roles", "roles": ["loader", "dequant", "mma", "epilogue"],
                    "wait_frac": [round(float(v), 3) for v in (d[live, :, 0] / d[live, :, 1]).mean(0)],
                    "cycles_per_kstep": round(float((d[live, 0, 1] / d[live, 0, 2].clamp_min(1)).mean()), 1),
                    "section_cycles_per_kstep": [round(float(v), 1) for v in (d[live, :, 3] / ks).mean(0)],
                    "section2_cycles_per_kstep": [round(float(v), 1) for v in (d[live, :, 4] / ks).mean(0)]})
    wb13 = bank.w13_codes.nbytes + bank.w13_scales.nbytes
    wb2 = bank.w2_codes.nbytes + bank.w2_scales.nbytes
    for name, fn, byts, fl in (
            ("moe_w13_int3", w13, wb13 + T * H + n * I * 2, 2 * n * H * 2 * I),
            ("quant_rows_e4m3_row(h)", hq, n * I * 2 + n * I, 0),
            ("moe_w2_int3", w2, wb2 + n * I + n * H * 2, 2 * n * I * H)):
        ms = time_cuda(fn)
        out.append({"kernel": name, "T": T, "E": E, "ms": round(ms, 4), "bytes": byts,
                    "gbs": round(byts / ms / 1e6, 1), "frac_hbm_of_measured": round(byts / ms / 1e6 / peaks["hbm_gbs"], 3),
                    "tflops": round(fl / ms / 1e9, 1)})
    return out


def bench_gemm(M=640):
    from ..ops import C
    peaks = load_peaks()
    out = []
    for name, N, K in (("in_proj_gdn", 12352, 2048), ("qkv_attn", 9216, 2048), ("out_proj_gdn", 2048, 4096),
                       ("o_proj_attn", 2048, 4096), ("lm_head", 151936, 2048), ("router+shared", 1352, 2048)):
        a = torch.randn(M, K, device="cuda").bfloat16()
        b = torch.randn(N, K, device="cuda").bfloat16()
        o = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ms = time_cuda(lambda: C().gemm(a, b, out=o))
        byts = (M * K + N * K + M * N) * 2
        fl = 2 * M * N * K
        ms_ref = time_cuda(lambda: torch.matmul(a, b.t(), out=o))
        out.append({"kernel": "gemm_bf16_tn", "shape": name, "M": M, "N": N, "K": K, "ms": round(ms, 4),
                    "tflops": round(fl / ms / 1e9, 1), "gbs": round(byts / ms / 1e6, 1),
                    "frac_bf16_of_measured": round(fl / ms / 1e9 / peaks["bf16_tflops"], 3),
                    "frac_hbm_of_measured": round(byts / ms / 1e6 / peaks["hbm_gbs"], 3),
                    "cublas_ms": round(ms_ref, 4), "plan": list(C().gemm_plan(M, N, K))})
    # the decode step's dense chain: 24 layers' worth of the six shapes back to back in one CUDA graph (distinct
    # weights, so each one streams from HBM as in a step), where launch gaps and prologues count
    shapes = [(N, K) for _, N, K in (("in_proj_gdn", 12352, 2048), ("out_proj_gdn", 2048, 4096),
                                     ("qkv_attn", 9216, 2048), ("o_proj_attn", 2048, 4096),
                                     ("router+shared", 1352, 2048))] * 24
    ws = [torch.randn(N, K, device="cuda").bfloat16() for N, K in shapes]
    xs = {K: torch.randn(M, K, device="cuda").bfloat16() for K in {K for _, K in shapes}}
    os_ = [torch.empty(M, N, device="cuda", dtype=torch.bfloat16) for N, _ in shapes]

    def chain():
        for w, o in zip(ws, os_):
            C().gemm(xs[w.shape[1]], w, out=o)
    chain()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        chain()
    ms = time_cuda(g.replay, iters=10)
    byts = sum(N * K * 2 for N, K in shapes)
    out.append({"kernel": "gemm_bf16_tn chain (graph)", "M": M, "launches": len(shapes), "ms": round(ms, 4),
                "weight_bytes": byts, "frac_hbm_of_measured": round(byts / ms / 1e6 / peaks["hbm_gbs"], 3),
                "pdl": os.environ.get("AFB_NO_PDL") is None})
    del g
    return out


def bench_vision(grids=((1, 64, 64), (1, 32, 48)), depth=27, seed=0):
    """The vision tower (full width, 27 blocks, random weights) on one batch of images: the native path (tcgen05 GEMMs,
    bidirectional tcgen05 attention, csrc/vision.cu) beside Hugging Face's bf16 Qwen3-VL vision model (SDPA) with the
    same weights on the same inputs."""
    from ..models.vision import VisionConfig, VisionTower
    cfg = VisionConfig(depth=depth)
    P = sum(t * h * w for t, h, w in grids)
    pixels = torch.randn(P, cfg.patch_dim, generator=torch.Generator().manual_seed(seed)).cuda()
    grid = torch.tensor(grids)
    tower = VisionTower.random(cfg, seed=seed)
    out = []
    try:
        from transformers.models.qwen3_vl_moe import configuration_qwen3_vl_moe as hfc
        from transformers.models.qwen3_vl_moe import modeling_qwen3_vl_moe as hfm
        c = hfc.Qwen3VLMoeVisionConfig(depth=depth, out_hidden_size=cfg.out_hidden_size)
        c._attn_implementation = "sdpa"
        model = hfm.Qwen3VLMoeVisionModel(c)
        model.load_state_dict(tower.state_dict(), strict=True)
        model = model.cuda().bfloat16().eval()
        with torch.no_grad():
            ms_hf = time_cuda(lambda: model(pixels.bfloat16(), grid_thw=grid.cuda()), iters=5)
        del model
    except ImportError:
        ms_hf = None
    tower = tower.cuda()
    ms = time_cuda(lambda: tower(pixels, grid), iters=5)
    # where one block's time goes (each piece timed alone, times the depth)
    from ..ops import C
    from ..train.attention import tile_lists
    H, Dp = cfg.num_heads, 128
    cu_host = [0]
    for t, h, w in grids:
        for _ in range(t):
            cu_host.append(cu_host[-1] + h * w)
    cu = torch.tensor(cu_host, dtype=torch.int32, device="cuda")
    tiles = tile_lists(cu_host, "cuda")[0]
    q, k, v, o = (torch.randn(P, H, Dp, device="cuda").bfloat16() for _ in range(4))
    lse = torch.empty(H, P, device="cuda")
    ms_attn = time_cuda(lambda: C().attn_train_fwd(q, k, v, cu, tiles, cfg.head_dim ** -0.5, o, lse, None, 64, False),
                        iters=5)
    b = tower._native["blocks"][0]
    y = torch.randn(P, cfg.hidden_size, device="cuda").bfloat16()
    m = torch.randn(P, cfg.intermediate_size, device="cuda").bfloat16()

    def gemms():
        C().gemm(y, b["wqkv"], bias=b["bqkv"])
        C().gemm(o.view(P, H * Dp), b["wproj"], bias=b["bproj"])
        C().gemm(y, b["w1"], bias=b["b1"], act=1)
        C().gemm(m, b["w2"], bias=b["b2"])
    ms_gemm = time_cuda(gemms, iters=5)
    att_flops = sum(4 * (h * w) ** 2 * 128 * H * t for t, h, w in grids)
    flops = 2 * P * cfg.depth * (4 * cfg.hidden_size ** 2 + 2 * cfg.hidden_size * cfg.intermediate_size)
    out.append({"kernel": "vision tower (27 blocks, native)", "patches": P, "ms": round(ms, 3),
                "patches_per_s": round(P / ms * 1e3), "linear_tflops": round(flops / ms / 1e9, 1),
                "hf_bf16_sdpa_ms": None if ms_hf is None else round(ms_hf, 3),
                "attention_ms_x_depth": round(ms_attn * cfg.depth, 3),
                "attention_tflops_padded": round(att_flops / ms_attn / 1e9, 1),
                "block_gemms_ms_x_depth": round(ms_gemm * cfg.depth, 3)})
    return out


def bench_gdn(S=128, T=5):
    from ..ops.gdn import GdnShape, GdnState, gdn_decode
    peaks = load_peaks()
    dev = "cuda"
    sh = GdnShape(16, 128, 32, 128)
    st = GdnState(sh, S, T, dev)
    st.ssm.normal_(0, 0.02)
    mixed = torch.randn(S * T, sh.mixed_dim, device=dev).bfloat16()
    conv_w = torch.randn(sh.conv_dim, 4, device=dev) * 0.3
    A_log = torch.zeros(sh.Hv, device=dev)
    dt = torch.zeros(sh.Hv, device=dev)
    nw = torch.ones(sh.Dv, device=dev).bfloat16()
    n_commit = torch.full((S,), 3, dtype=torch.int32, device=dev)
    slots = torch.arange(S, dtype=torch.int32, device=dev)
    out = torch.empty(S * T, sh.Hv * sh.Dv, device=dev).bfloat16()
    par = [0]

    def fn():
        gdn_decode(mixed, sh, st, conv_w, A_log, dt, nw, n_commit, slots, out, T, par[0] & 1)
        par[0] += 1
    ms = time_cuda(fn)
    byts = 2 * st.ssm.nbytes + mixed.nbytes + out.nbytes
    dbg = torch.zeros(148 * 24, dtype=torch.int64, device=dev)
    gdn_decode(mixed, sh, st, conv_w, A_log, dt, nw, n_commit, slots, out, T, par[0] & 1, dbg=dbg)
    torch.cuda.synchronize()
    d = dbg.view(148, 24).cpu()
    items = int((d[:, 7] >> 40).sum())
    d[:, 7] &= (1 << 40) - 1
    names = ["wait", "stage", "barrier A", "phase 1", "mma1 wait", "solve", "barrier C", "commit"]
    sections = {}
    if items:
        for who, off in (("thread0", 0), ("mma_thread", 8)):
            sections[who] = {n: round(float(d[:, off + k].sum()) / items) for k, n in enumerate(names)}
        sections["solve_parts"] = {n: round(float(d[:, 16 + k].sum()) / items) for k, n in
                                   enumerate(["P load", "u chain", "outputs+sums", "U^T", "sums barrier", "norm"])}
    return [{"kernel": "gdn_decode(conv_prep+recurrent)", "S": S, "T": T, "ms": round(ms, 4), "bytes": byts,
             "gbs": round(byts / ms / 1e6, 1), "frac_hbm_of_measured": round(byts / ms / 1e6 / peaks["hbm_gbs"], 3),
             "cycles_per_item": sections}]


def bench_attn(S=128, T=5, seed=0):
    from ..ops.attention import paged_attention
    peaks = load_peaks()
    dev = "cuda"
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(4096, 24577, (S,), generator=g) + T
    pages = (lens + 63) // 64
    P = int(pages.sum())
    maxp = int(pages.max())
    kc = torch.randn(P, 2, 64, 256, device=dev).bfloat16()
    vc = torch.randn(P, 2, 64, 256, device=dev).bfloat16()
    bt = torch.zeros(S, maxp, dtype=torch.int32)
    o = 0
    for i in range(S):
        bt[i, : int(pages[i])] = torch.arange(o, o + int(pages[i]))
        o += int(pages[i])
    bt = bt.to(dev)
    seq_lens = lens.int().to(dev)
    q = torch.randn(S * T, 16, 256, device=dev).bfloat16()
    out = torch.empty_like(q)
    ms = time_cuda(lambda: paged_attention(q, kc, vc, bt, seq_lens, T, out, max_pages=maxp), flush_bytes=1 << 20)
    byts = int(lens.sum()) * 2 * 2 * 256 * 2
    ms1 = time_cuda(lambda: paged_attention(q, kc, vc, bt, seq_lens, T, out, max_pages=maxp, impl=1),
                    flush_bytes=1 << 20)
    res = [{"kernel": "paged_attn_verify (tcgen05)", "S": S, "T": T, "ms": round(ms, 4), "kv_bytes": byts,
            "gbs": round(byts / ms / 1e6, 1), "frac_hbm_of_measured": round(byts / ms / 1e6 / peaks["hbm_gbs"], 3)},
           {"kernel": "paged_attn_verify (mma.sync)", "S": S, "T": T, "ms": round(ms1, 4),
            "frac_hbm_of_measured": round(byts / ms1 / 1e6 / peaks["hbm_gbs"], 3)}]
    # the same contexts in an NVFP4 cache (random codes, unit scales): 0.5625 bytes per element
    del kc, vc
    k4 = torch.randint(0, 256, (P, 2, 64, 128), dtype=torch.uint8, device=dev)
    v4 = torch.randint(0, 256, (P, 2, 64, 128), dtype=torch.uint8, device=dev)
    ks = torch.full((P, 2, 64, 16), 0x38, dtype=torch.uint8, device=dev)  # e4m3 1.0
    vs = ks.clone()
    ms4 = time_cuda(lambda: paged_attention(q, k4, v4, bt, seq_lens, T, out, max_pages=maxp, kv_scales=(ks, vs)),
                    flush_bytes=1 << 20)
    b4 = int(lens.sum()) * 2 * 2 * (128 + 16)
    res.append({"kernel": "paged_attn_verify_nvfp4", "S": S, "T": T, "ms": round(ms4, 4), "kv_bytes": b4,
                "gbs": round(b4 / ms4 / 1e6, 1), "frac_hbm_of_measured": round(b4 / ms4 / 1e6 / peaks["hbm_gbs"], 3),
                "speedup_vs_bf16": round(ms / ms4, 2)})
    return res


def bench_qsa(S=110, ctx=32100, W=8, block=4, K=512, Hq=24, Hkv=2, D=256, seed=0):
    """QSA verify step of one full-attention layer: selection (scores over every complete block of each verify row,
    top-K, the per-session union) and the block-sparse attention over the union. Defaults: the reference model's
    QSA (4-token blocks, top-512, 24Q/2KV x 256) at BASELINE config 5's 110 sessions x 64k context; ``block=64,
    K=32, Hq=16`` is config 5's own shape. Bytes: pooled keys read by the selection; K + V of the union's tokens.
    The reference publishes 149.4 us for its grouped indexer logits alone at B=110, ctx 32,100, 8 rows
    (``runtime/patches/sglang-0.5.20/README.md:177-184``); ``qsa_select`` here is scores + top-K + union."""
    from ..models.reference import rope_cos_sin
    from ..ops.qsa import PAGE, QsaWorkspace, qsa_attention
    peaks = load_peaks()
    dev = "cuda"
    g = torch.Generator().manual_seed(seed)
    lens = torch.full((S,), ctx + W, dtype=torch.int64)
    maxp = (ctx + W + PAGE - 1) // PAGE
    P = S * maxp
    bt = torch.randperm(P, generator=g).view(S, maxp).int().to(dev)
    kc = torch.randn(P, Hkv, PAGE, D, device=dev).bfloat16()
    vc = torch.randn(P, Hkv, PAGE, D, device=dev).bfloat16()
    raw = torch.randn(P * PAGE, 128, device=dev).bfloat16()
    ws = QsaWorkspace(S, W, K, maxp, 4, dev, block=block)
    keys = torch.randn(S * ws.max_blocks, 128, device=dev).bfloat16()
    kn = torch.zeros(128, dtype=torch.bfloat16, device=dev)
    cos, sin = (t.contiguous().to(dev) for t in rope_cos_sin(torch.arange(ctx + 2 * W + 64), 64, 1.0e7))
    ws.idx_q.copy_(torch.randn(S * W, 4, 128, device=dev).bfloat16())
    q = torch.randn(S * W, Hq, D, device=dev).bfloat16()
    out = torch.empty_like(q)
    seq_lens = lens.int().to(dev)
    fin = (seq_lens - W) // block
    c = __import__("arc_forge_2026_b200.ops._ext", fromlist=["C"]).C()

    def select():
        c.qsa_select(ws.idx_q, keys, raw, kn, bt, fin, seq_lens, W, K, 4, block, ws.sel, cos, sin, 64, 1e-6,
                     ws.u_page, ws.u_lpage, ws.u_mask, ws.u_count, None, ws.scores)

    def full():
        qsa_attention(q, kc, vc, bt, seq_lens, fin, keys, ws, out, splits=4, raw=raw, k_norm=kn, rope=(cos, sin))

    ms_sel = time_cuda(select, flush_bytes=256 << 20)
    ms_all = time_cuda(full, flush_bytes=256 << 20)
    torch.cuda.synchronize()
    union_tokens = int(ws.u_count.sum()) * block
    sel_bytes = S * (ctx // block) * 128 * 2
    att_bytes = union_tokens * Hkv * D * 2 * 2
    ms_att = max(ms_all - ms_sel, 1e-6)
    tag = f"block {block} top-{K}"
    return [{"kernel": f"qsa_select ({tag})", "S": S, "ctx": ctx, "W": W, "ms": round(ms_sel, 4),
             "key_bytes": sel_bytes, "frac_hbm_of_measured": round(sel_bytes / ms_sel / 1e6 / peaks["hbm_gbs"], 3)},
            {"kernel": f"qsa_sparse_attention ({tag}, {Hq}Q/{Hkv}KV x {D})", "S": S, "ctx": ctx, "W": W,
             "ms": round(ms_att, 4), "union_tokens_per_session": round(union_tokens / S, 1), "kv_bytes": att_bytes,
             "frac_hbm_of_measured": round(att_bytes / ms_att / 1e6 / peaks["hbm_gbs"], 3)},
            {"kernel": f"qsa_layer_total ({tag})", "ms": round(ms_all, 4)}]


def bench_train_attn(T=16384, segs=(16384,), Hq=16, Hkv=2, D=256, seed=0):
    """Training attention of one packed row (QAD shape: 16Q/2KV x 256, 16k tokens): the native tcgen05 forward and
    backward (``train/attention.py``) beside the library flash-attention varlen kernels on the same inputs.
    FLOPs: causal 2 x 2 x sum(L^2 / 2) x Hq x D forward, 2.5x that backward."""
    from ..train.attention import varlen_attention
    peaks = load_peaks()
    g = torch.Generator(device="cuda").manual_seed(seed)
    cu = torch.tensor([0] + list(torch.tensor(segs).cumsum(0)), dtype=torch.int32)
    q = torch.randn(T, Hq, D, device="cuda", generator=g).bfloat16().requires_grad_()
    k = torch.randn(T, Hkv, D, device="cuda", generator=g).bfloat16().requires_grad_()
    v = torch.randn(T, Hkv, D, device="cuda", generator=g).bfloat16().requires_grad_()
    do = torch.randn(T, Hq, D, device="cuda", generator=g).bfloat16()
    flops_f = sum(2 * 2 * L * L / 2 * Hq * D for L in segs)
    res = []
    arms = [("native tcgen05", lambda: varlen_attention(q, k, v, cu))]
    try:
        from flash_attn import flash_attn_varlen_func
        cud = cu.cuda()
        arms.append(("flash_attn varlen (library)", lambda: flash_attn_varlen_func(
            q, k, v, cud, cud, max(segs), max(segs), causal=True, deterministic=True)))
    except ImportError:
        pass
    for name, fn in arms:
        ms_f = time_cuda(lambda: fn(), flush_bytes=1 << 20)
        out = fn()
        ms_fb = time_cuda(lambda: torch.autograd.grad(fn(), (q, k, v), do), flush_bytes=1 << 20)
        ms_b = ms_fb - ms_f
        res.append({"kernel": f"train attention fwd ({name})", "T": T, "segments": len(segs), "ms": round(ms_f, 3),
                    "tflops": round(flops_f / ms_f / 1e9, 1),
                    "frac_bf16_of_measured": round(flops_f / ms_f / 1e9 / peaks["bf16_tflops"], 3)})
        res.append({"kernel": f"train attention bwd ({name})", "T": T, "ms": round(ms_b, 3),
                    "tflops": round(2.5 * flops_f / ms_b / 1e9, 1),
                    "frac_bf16_of_measured": round(2.5 * flops_f / ms_b / 1e9 / peaks["bf16_tflops"], 3)})
        del out
    return res


def _ref_kernels():
    """The reference's own Triton / torch trainer modules, unmodified, from the reference tree beside the repository
    (``baseline/_ref/kernels``: ``scale_grad_triton.py``, ``topk_tail_kl.py``, ``hc_mix.py``, ``int3_moe.py`` and its
    ``fp8_moe.py`` import); None when absent."""
    import importlib
    import sys
    d = os.path.join(os.path.dirname(__file__), "..", "..", "baseline", "_ref", "kernels")
    if not os.path.isdir(d):
        return None
    if d not in sys.path:
        sys.path.insert(0, d)
    return {n: importlib.import_module(n) for n in ("scale_grad_triton", "topk_tail_kl", "hc_mix", "int3_moe")}


def bench_ref_triton(E=320, I=640, H=2560, rows=1_200_000, T_kl=4096, V=248_320, T_hc=16384, seed=0):
    """The reference's trainer kernels run unmodified beside this repository's equivalents on the same inputs (the
    reference model's shapes: hidden 2560, 320 experts x 640, vocab 248,320, 4 HC branches x rank 320):
      dequant   ``int3_moe._dequant_bank_kernel`` (E4M3 codes + bf16 group scales -> bf16 bank) vs ``int3_dequant``
                (packed 3-bit tiles -> bf16 bank);
      scale-grad ``scale_grad_triton._scale_grad_kernel`` (fused G^T A per expert x codes, 1.2M routed rows, K 2560;
                 published 28.7 ms) vs this repository's path: the per-expert dW GEMM (``torch._grouped_mm``) plus
                 ``int3_scale_grad``;
      KL32_tail ``topk_tail_kl.fused_topk_tail_kl`` (torch, chunked) vs ``train/losses.py`` (fused kernel), forward
                 + backward;
      HC mix    ``hc_mix.mix_fwd`` (Triton norm + mix) vs ``train/hc.py`` ``hc_read`` (native), forward."""
    from ..ops import C
    from ..quant.int3_tiles import codes_to_tiles
    ref = _ref_kernels()
    if ref is None:
        return [{"kernel": "reference Triton arms", "unavailable": "baseline/_ref/kernels is absent"}]
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(seed)
    res = []
    N = 2 * I
    # ---- dequant bank (w13)
    codes = torch.randint(0, 8, (E, N, H), device=dev, dtype=torch.uint8, generator=g)
    sc = (torch.rand(E, N, H // 128, device=dev, generator=g) * 0.02 + 0.001)
    w8 = (codes.float() - 4).to(torch.float8_e4m3fn)
    s16 = sc.bfloat16()
    tiles = codes_to_tiles(codes)
    out = torch.empty(E, N, H, dtype=torch.bfloat16, device=dev)
    ms_r = time_cuda(lambda: ref["int3_moe"].dequant_bank(w8, s16), flush_bytes=256 << 20)
    ms_o = time_cuda(lambda: C().int3_dequant(tiles, s16.float(), out), flush_bytes=256 << 20)
    same = bool(torch.equal(ref["int3_moe"].dequant_bank(w8, s16), (C().int3_dequant(tiles, s16.float(), out), out)[1]))
    res.append({"kernel": "dequant bank w13 [320, 1280, 2560]", "reference_ms": round(ms_r, 3), "ours_ms": round(ms_o, 3),
                "speedup": round(ms_r / ms_o, 2), "bitwise_equal": same})
    del w8, out
    # ---- scale gradients (w13: N 1280, K 2560)
    counts = torch.full((E,), rows // E, dtype=torch.int64)
    counts[: rows - int(counts.sum())] += 1
    ends = torch.cat([torch.zeros(1, dtype=torch.int64), counts.cumsum(0)]).int().to(dev)
    G = (torch.randn(rows, N, device=dev, generator=g) * 0.01).bfloat16()
    A = torch.randn(rows, H, device=dev, generator=g).to(torch.float8_e4m3fn)
    a_scale = torch.ones(rows, device=dev)
    cw = (codes.float() - 4).to(torch.float8_e4m3fn)
    dS_ref = torch.empty(E, N, H // 128, device=dev)
    ms_r = time_cuda(lambda: ref["scale_grad_triton"].scale_gradients_fused(G, A, a_scale, cw, ends, dS_ref),
                     flush_bytes=256 << 20)
    A16 = A.bfloat16()
    offs = ends[1:].contiguous()
    dS = torch.empty(E, N, H // 128, device=dev)

    def ours_sg():
        dW = torch._grouped_mm(G.t(), A16, offs=offs)  # [E, N, K] per-expert G^T A
        C().int3_scale_grad(tiles, dW.to(torch.bfloat16), dS)
    ms_o = time_cuda(ours_sg, flush_bytes=256 << 20)
    ref["scale_grad_triton"].scale_gradients_fused(G, A, a_scale, cw, ends, dS_ref)
    ours_sg()
    rel = float((dS - dS_ref).norm() / dS_ref.norm())
    res.append({"kernel": f"INT3 scale grad w13 ({rows} routed rows, K 2560)", "reference_ms": round(ms_r, 3),
                "ours_ms": round(ms_o, 3), "speedup": round(ms_r / ms_o, 2), "rel_diff": round(rel, 4),
                "ours_form": "grouped dW GEMM (library) + native int3_scale_grad", "reference_published_ms": 28.7})
    del G, A, A16, cw, codes, tiles
    # ---- KL32_tail forward + backward
    from ..train.losses import fused_topk_tail_kl
    W = (torch.randn(V, H, device=dev, generator=g) * 0.02).bfloat16()
    Wt = W.t().contiguous()
    hid = torch.randn(T_kl, H, device=dev, generator=g).bfloat16().requires_grad_()
    ids = torch.randint(0, V, (T_kl, 32), device=dev, generator=g)
    lp = torch.log_softmax(torch.randn(T_kl, 33, device=dev, generator=g), -1)
    t_lp, t_tail = lp[:, :32].contiguous(), lp[:, 32].contiguous()

    def ref_kl():
        ref["topk_tail_kl"].fused_topk_tail_kl(hid, W, ids, t_lp, t_tail).backward()

    def ours_kl():
        fused_topk_tail_kl(hid, W, Wt, ids, t_lp, t_tail).backward()
    ms_r = time_cuda(ref_kl, flush_bytes=256 << 20)
    ms_o = time_cuda(ours_kl, flush_bytes=256 << 20)
    res.append({"kernel": f"KL32_tail fwd+bwd ({T_kl} rows, vocab {V})", "reference_ms": round(ms_r, 3),
                "ours_ms": round(ms_o, 3), "speedup": round(ms_r / ms_o, 2)})
    del W, Wt, hid
    # ---- HC mix forward
    from ..models.reference import HyperConnection
    from ..config import preset
    from ..train.hc import hc_read
    cfg = preset("qwen38fn")
    mod = HyperConnection(cfg).to(dev)
    with torch.no_grad():
        for p_ in mod.parameters():
            p_.normal_(0, 0.02)
    h = torch.randn(T_hc, 4, H, device=dev, generator=g).bfloat16()
    nw = mod.hc_norm.weight.detach().float().contiguous()
    wd, wu, wi = (t.detach().bfloat16() for t in (mod.w_down, mod.w_up, mod.w_inject))
    ms_r = time_cuda(lambda: ref["hc_mix"].mix_fwd(h, nw, wd, wu, wi, True, mod.eps), flush_bytes=256 << 20)
    ms_o = time_cuda(lambda: hc_read(h, mod), flush_bytes=256 << 20)
    xr = ref["hc_mix"].mix_fwd(h, nw, wd, wu, wi, True, mod.eps)[0]
    xo = hc_read(h, mod)[0]
    res.append({"kernel": f"HC mix forward ({T_hc} x 4 x 2560)", "reference_ms": round(ms_r, 3),
                "ours_ms": round(ms_o, 3), "speedup": round(ms_r / ms_o, 2),
                "rel_diff": round(float((xo.float() - xr.float()).norm() / xr.float().norm()), 4)})
    return res


def bench_grouped(E=320, T=16384, k=10, H=2048, I=512, seed=0):
    """Grouped expert GEMMs of one QAD layer (w13: K=H, N=2I; w2: K=I, N=H; routed rows T*k): the native grouped
    tcgen05 GEMM (forward, dX, dW) against torch._grouped_mm."""
    from ..train.grouped import grouped_reduce, grouped_rows, transposed_bank
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(seed)
    ids = torch.randint(0, E, (T * k,), generator=g, device=dev)
    counts = torch.bincount(ids, minlength=E)
    offs = counts.cumsum(0).int()
    res = []
    for name, K, N in (("w13", H, 2 * I), ("w2", I, H)):
        x = torch.randn(T * k, K, generator=g, device=dev).bfloat16()
        w = (torch.randn(E, N, K, generator=g, device=dev) * 0.02).bfloat16()
        dy = torch.randn(T * k, N, generator=g, device=dev).bfloat16()
        cases = {
            "fwd_native": lambda: grouped_rows(x, w, counts),
            "fwd_library": lambda: torch._grouped_mm(x, w.transpose(-2, -1), offs=offs),
            "dx_native": lambda: grouped_rows(dy, transposed_bank(w), counts),
            "dx_library": lambda: torch._grouped_mm(dy, w, offs=offs),
            "dw_native": lambda: grouped_reduce(dy, x, counts),
            "dw_library": lambda: torch._grouped_mm(dy.t(), x, offs=offs),
        }
        for cname, fn in cases.items():
            ms = time_cuda(fn, flush_bytes=1 << 20)
            res.append({"kernel": f"grouped_{name}_{cname}", "ms": round(ms, 4),
                        "tflops": round(2 * T * k * K * N / ms / 1e9, 1)})
    return res


def bench_ple(T=16384, base=250_000, seed=0):
    """PLE lookup of one packed 16k-token row: 16 heads (2- and 3-grams x 8) of 160 e4m3 dims from a table of
    ~4M rows (a quarter-size stand-in of the 20M-bucket heads; the gather is random either way)."""
    from ..config import preset
    from ..models.ple import NgramHash
    from ..ops.ple import PleTable
    peaks = load_peaks()
    dev = "cuda"
    cfg = preset("tiny_cpu", vocab_size=248320, ple_layer_ids=(1,), ngram_vocab_size_base=base, ple_embed_dim=2560)
    h = NgramHash(cfg)
    g = torch.Generator(device=dev).manual_seed(seed)
    rows = torch.randint(-120, 120, (h.rows, 160), generator=g, device=dev, dtype=torch.int8).view(torch.float8_e4m3fn)
    scale = torch.full(((h.rows + 127) // 128, 2), 0.01, device=dev)
    table = PleTable(h, rows, scale)
    toks = torch.randint(0, cfg.vocab_size, (T,), generator=g, device=dev)
    seg = torch.zeros(T, dtype=torch.long, device=dev)
    ms = time_cuda(lambda: table.lookup_tokens(toks, seg), flush_bytes=1 << 20)
    byts = T * 16 * (160 + 320) + T * 16 * 4  # e4m3 rows read, bf16 rows written, scales
    return [{"kernel": "ple_lookup", "T": T, "table_rows": h.rows, "ms": round(ms, 4), "bytes": byts,
             "gbs": round(byts / ms / 1e6, 1), "frac_hbm_of_measured": round(byts / ms / 1e6 / peaks["hbm_gbs"], 3)}]


def bench_gdn_scan(BH=32, n=256, steps=(False, True)):
    """Inter-chunk scan of one GDN layer at seq 16,384 (256 chunks of 64), 32 value heads, Dk = Dv = 128: the
    tensor-core kernel and the fp32 SIMT kernel, forward and reverse (the reverse adds the Qm term)."""
    from ..ops import C
    peaks = load_peaks()
    dev = "cuda"
    Dk = Dv = 128
    m1 = torch.randn(BH, n, 64, Dk, device=dev) * 0.05
    m2 = torch.randn(BH, n, 64, Dk, device=dev) * 0.05
    y = torch.randn(BH, n, 64, Dv, device=dev)
    qm = torch.randn(BH, n, Dk, Dv, device=dev)
    last = -torch.rand(BH, n, device=dev)
    states = torch.empty(BH, n, Dk, Dv, device=dev)
    x = torch.empty_like(y)
    fin = torch.empty(BH, Dk, Dv, device=dev)
    c = C()
    res = []
    flops = 2 * 2 * BH * n * 64 * Dk * Dv
    for reverse in steps:
        for precise in (False, True):
            q = qm if reverse else None
            ms = time_cuda(lambda: c.gdn_chunk_scan(m1, m2, y, q, last, None, states, x, fin, reverse, precise),
                           iters=5)
            byts = m1.nbytes + m2.nbytes + y.nbytes + x.nbytes + states.nbytes + (qm.nbytes if reverse else 0)
            res.append({"kernel": "gdn_chunk_scan" + ("_fp32" if precise else "_tc") + ("_rev" if reverse else ""),
                        "BH": BH, "chunks": n, "ms": round(ms, 4), "us_per_step": round(ms * 1000 / n, 2),
                        "tflops": round(flops / ms / 1e9, 1), "gbs": round(byts / ms / 1e6, 1),
                        "frac_hbm_of_measured": round(byts / ms / 1e6 / peaks["hbm_gbs"], 3)})
    return res


def bench_gdn_train(B=1, T=16384, Hk=16, Hv=32):
    """One GDN layer's chunked rule, forward and forward + backward, at seq 16,384 (the QAD shape): the native
    kernels against the torch path with the fp32 scan."""
    from ..train.gdn_chunk import chunk_gated_delta_rule
    dev = "cuda"
    D = 128
    q = (torch.nn.functional.normalize(torch.randn(B, T, Hk, D, device=dev), dim=-1) * D ** -0.5).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(B, T, Hk, D, device=dev), dim=-1).bfloat16()
    v = torch.randn(B, T, Hv, D, device=dev).bfloat16()
    gate = -torch.rand(B, T, Hv, device=dev) * 0.3
    beta = torch.rand(B, T, Hv, device=dev)
    dout = torch.randn(B, T, Hv, D, device=dev).bfloat16()
    res = []
    for precise in (False, True):
        ins = [t.clone().requires_grad_(True) for t in (q, k, v, gate, beta)]

        def fwd():
            with torch.no_grad():
                chunk_gated_delta_rule(*ins, precise=precise)

        def fwd_bwd():
            o, _ = chunk_gated_delta_rule(*ins, precise=precise)
            o.backward(dout.to(o.dtype))
        ms_f = time_cuda(fwd, iters=5, flush_bytes=1 << 20)
        ms_fb = time_cuda(fwd_bwd, iters=5, flush_bytes=1 << 20)
        res.append({"kernel": "gdn_chunk_layer" + ("_torch_fp32scan" if precise else "_native"), "T": T, "Hv": Hv,
                    "ms_fwd": round(ms_f, 3), "ms_fwd_bwd": round(ms_fb, 3)})
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["moe", "gemm", "gdn", "attn", "qsa", "train_attn", "ref_triton", "gdn_scan", "gdn_train", "grouped", "ple", "vision", "all"])
    ap.add_argument("--T", type=int, default=640)
    ap.add_argument("--S", type=int, default=128, help="sessions of the attn case")
    ap.add_argument("--seq", type=int, default=16384, help="sequence length of the gdn_scan / gdn_train cases")
    a = ap.parse_args()
    res = []
    if a.what in ("moe", "all"):
        res += bench_moe(T=a.T)
    if a.what in ("gemm", "all"):
        res += bench_gemm(M=a.T)
    if a.what in ("gdn", "all"):
        res += bench_gdn()
    if a.what in ("attn", "all"):
        res += bench_attn(S=a.S)
    if a.what in ("qsa", "all"):
        res += bench_qsa(ctx=32100, W=8)                      # the reference's published shape (B=110, S=8)
        res += bench_qsa(ctx=65536, W=5)                      # config 5 sessions and context, the model's blocks
        res += bench_qsa(ctx=65536, W=5, block=64, K=32, Hq=16)  # config 5 as specified
    if a.what in ("train_attn", "all"):
        res += bench_train_attn()
        res += bench_train_attn(T=16384, segs=(4096,) * 4, Hq=24, Hkv=2)
    if a.what in ("ref_triton", "all"):
        res += bench_ref_triton()
    if a.what in ("gdn_scan", "all"):
        res += bench_gdn_scan(n=(a.seq + 63) // 64)
    if a.what in ("ple", "all"):
        res += bench_ple()
    if a.what in ("grouped", "all"):
        res += bench_grouped()
    if a.what in ("gdn_train", "all"):
        res += bench_gdn_train(T=a.seq)
    if a.what in ("vision", "all"):
        res += bench_vision()
    for r in res:
        print(json.dumps(r))


if __name__ == "__main__":
    main()
