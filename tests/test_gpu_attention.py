"""GPU numerics of the paged decode/verify attention against the fp32 oracle."""
import pytest
import torch

from arc_forge_2026_b200.ops import check_status
from arc_forge_2026_b200.ops.attention import paged_attention, paged_attention_reference

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("impl", [0, 1])  # tcgen05 kernel, mma.sync kernel
@pytest.mark.parametrize("D,Hq,Hkv,qp,lens,splits", [
    (256, 16, 2, 5, [5, 64, 70, 1000], None),
    (256, 16, 2, 1, [1, 300, 4097], 4),
    (128, 16, 2, 5, [7, 129, 2000], 3),
    (256, 16, 2, 5, [24000, 4100], None),
    (256, 16, 2, 8, [8, 520, 3000], 1),
    (128, 8, 1, 8, [100, 1100], 2),
])
def test_paged_attention(D, Hq, Hkv, qp, lens, splits, impl):
    g = torch.Generator(device="cpu").manual_seed(D + qp + len(lens))
    S = len(lens)
    maxp = max((L + 63) // 64 for L in lens)
    P = S * maxp + 3
    kc = torch.randn(P, Hkv, 64, D, generator=g).bfloat16().to(dev)
    vc = torch.randn(P, Hkv, 64, D, generator=g).bfloat16().to(dev)
    perm = torch.randperm(P, generator=g)[: S * maxp].view(S, maxp).int().to(dev)  # scattered pages
    seq_lens = torch.tensor(lens, dtype=torch.int32, device=dev)
    q = torch.randn(S * qp, Hq, D, generator=g).bfloat16().to(dev)
    qkv_like = torch.randn(S * qp, Hq, 2 * D, generator=g).bfloat16().to(dev)  # gate at [..., D:]
    gate_view = qkv_like[..., D:]
    out = torch.empty_like(q)
    paged_attention(q, kc, vc, perm, seq_lens, qp, out, gate=qkv_like[..., D:], gate_ld=Hq * 2 * D,
                    gate_head_stride=2 * D, splits=splits, impl=impl)
    torch.cuda.synchronize()
    check_status()
    ref = paged_attention_reference(q, kc, vc, perm, seq_lens, qp, gate=gate_view)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("splits", [1, 3])
def test_paged_attention_growing_scores(splits):
    """Scores that grow page after page, so a row's running max jumps by more than 2^8 several times: the tcgen05
    kernel's lazy rescale of O in tensor memory must keep O, l and m consistent."""
    g = torch.Generator(device="cpu").manual_seed(7)
    D, Hq, Hkv, qp, L = 256, 16, 2, 4, 1500
    maxp = (L + 63) // 64
    q = (torch.randn(qp, Hq, D, generator=g) * 3).bfloat16().to(dev)
    grow = (1 + torch.arange(maxp).float() / 2).repeat_interleave(64)[:, None]        # per key position
    kc = (torch.randn(maxp, Hkv, 64, D, generator=g) * grow.view(maxp, 1, 64, 1)).bfloat16().to(dev)
    vc = torch.randn(maxp, Hkv, 64, D, generator=g).bfloat16().to(dev)
    bt = torch.arange(maxp, dtype=torch.int32, device=dev)[None]
    seq_lens = torch.tensor([L], dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    paged_attention(q, kc, vc, bt, seq_lens, qp, out, splits=splits)
    torch.cuda.synchronize()
    check_status()
    ref = paged_attention_reference(q, kc, vc, bt, seq_lens, qp)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("window", [64, 1024])
def test_paged_attention_window_and_virtual_rows(window):
    """Sliding window (drafter) and prefill-style virtual sequences sharing one block-table row."""
    g = torch.Generator(device="cpu").manual_seed(window)
    D, Hq, Hkv, qp = 128, 16, 2, 4
    L = 3000
    maxp = (L + 63) // 64
    kc = torch.randn(maxp + 2, Hkv, 64, D, generator=g).bfloat16().to(dev)
    vc = torch.randn(maxp + 2, Hkv, 64, D, generator=g).bfloat16().to(dev)
    bt = torch.randperm(maxp + 2, generator=g)[:maxp].view(1, maxp).int().to(dev)
    # three virtual sequences = query chunks ending at 1000, 2000, 3000 of the same sequence
    ends = [1000, 2000, 3000]
    seq_lens = torch.tensor(ends, dtype=torch.int32, device=dev)
    bt_row = torch.zeros(3, dtype=torch.int32, device=dev)
    q = torch.randn(3 * qp, Hq, D, generator=g).bfloat16().to(dev)
    out = torch.empty_like(q)
    paged_attention(q, kc, vc, bt, seq_lens, qp, out, window=window, bt_row=bt_row, max_pages=maxp)
    torch.cuda.synchronize()
    check_status()
    ref = paged_attention_reference(q, kc, vc, bt.expand(3, maxp), seq_lens, qp, window=window)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("D,splits", [(256, None), (128, 3)])
def test_nvfp4_kv_store_and_attention(D, splits):
    """The KV store writes e2m1 codes with e4m3 scales per 16 elements (close to the bf16 rows); attention over the
    NVFP4 cache (bulk-copied packed pages dequantised in shared memory, f16 MMAs) agrees with attention over the same
    values in bf16 pages and with the fp32 oracle."""
    from arc_forge_2026_b200.ops import C
    from arc_forge_2026_b200.ops.attention import new_nvfp4_kv, nvfp4_dequant
    from arc_forge_2026_b200.models.reference import rope_cos_sin
    g = torch.Generator(device="cpu").manual_seed(D)
    Hq, Hkv, qp, rot = 16, 2, 5, 64
    lens = [70, 333, 1200]
    S = len(lens)
    maxp = max((L + 63) // 64 for L in lens)
    P = S * maxp + 2
    bt = torch.randperm(P, generator=g)[: S * maxp].view(S, maxp).int().to(dev)
    kc = torch.zeros(P, Hkv, 64, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    k4, v4, ks, vs = new_nvfp4_kv(P, Hkv, D, dev)
    cos, sin = rope_cos_sin(torch.arange(4096, device=dev), rot, 1e7)
    qw = (torch.randn(D, generator=g) * 0.1).bfloat16().to(dev)
    kw = (torch.randn(D, generator=g) * 0.1).bfloat16().to(dev)
    width = Hq * 2 * D + 2 * Hkv * D
    for s, L in enumerate(lens):  # the whole context through the store kernel, both formats
        qkv = (torch.randn(L, width, generator=g) * 2).bfloat16().to(dev)
        pos = torch.arange(L, dtype=torch.int32, device=dev)
        slots = (bt[s, pos.long() // 64] * 64 + pos % 64).int()
        qo = torch.empty(L, Hq, D, dtype=torch.bfloat16, device=dev)
        C().qk_norm_rope_store(qkv, Hq, Hkv, D, rot, qw, kw, pos, slots, cos.contiguous(), sin.contiguous(), 1e-6,
                               qo, kc, vc)
        C().qk_norm_rope_store(qkv, Hq, Hkv, D, rot, qw, kw, pos, slots, cos.contiguous(), sin.contiguous(), 1e-6,
                               qo, k4, v4, kscale=ks, vscale=vs)
    torch.cuda.synchronize()
    check_status()
    kd, vd = nvfp4_dequant(k4, ks), nvfp4_dequant(v4, vs)
    used = bt.reshape(-1).long()
    for deq, ref in ((kd, kc), (vd, vc)):
        err = _rel(deq[used], ref[used])
        assert 0 < err < 0.15, err  # e2m1: one mantissa bit
    seq_lens = torch.tensor(lens, dtype=torch.int32, device=dev)
    q = torch.randn(S * qp, Hq, D, generator=g).bfloat16().to(dev)
    gate = torch.randn(S * qp, Hq, 2 * D, generator=g).bfloat16().to(dev)
    out4, outb = torch.empty_like(q), torch.empty_like(q)
    paged_attention(q, k4, v4, bt, seq_lens, qp, out4, gate=gate[..., D:], gate_ld=Hq * 2 * D, gate_head_stride=2 * D,
                    splits=splits, kv_scales=(ks, vs))
    paged_attention(q, kd.bfloat16(), vd.bfloat16(), bt, seq_lens, qp, outb, gate=gate[..., D:], gate_ld=Hq * 2 * D,
                    gate_head_stride=2 * D, splits=splits)
    torch.cuda.synchronize()
    check_status()
    assert _rel(out4, outb) < 1e-2, _rel(out4, outb)
    ref = paged_attention_reference(q, kd.bfloat16(), vd.bfloat16(), bt, seq_lens, qp, gate=gate[..., D:])
    assert _rel(out4, ref) < 1e-2
