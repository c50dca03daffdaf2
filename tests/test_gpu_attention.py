"""GPU numerics of the paged decode/verify attention against the fp32 oracle."""
import pytest
import torch

from arc_forge_2026_b200.ops import check_status
from arc_forge_2026_b200.ops.attention import paged_attention, paged_attention_reference

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("D,Hq,Hkv,qp,lens,splits", [
    (256, 16, 2, 5, [5, 64, 70, 1000], None),
    (256, 16, 2, 1, [1, 300, 4097], 4),
    (128, 16, 2, 5, [7, 129, 2000], 3),
    (256, 16, 2, 5, [24000, 4100], None),
])
def test_paged_attention(D, Hq, Hkv, qp, lens, splits):
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
                    gate_head_stride=2 * D, splits=splits)
    torch.cuda.synchronize()
    check_status()
    ref = paged_attention_reference(q, kc, vc, perm, seq_lens, qp, gate=gate_view)
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
